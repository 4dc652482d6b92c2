// Integer metadata kernels for the full-sequence hierarchical layout:
// dense mask rows, 128x128 block classification (Flex BlockMask lists), and
// the attention work plan (query tiles, key tiles, per-row key bitmasks).
//
// The mask predicate follows build_stage2_hier_self_attn_mask
// (multics/models/hier_masks.py:364-507) and its membership variant
// (hier_masks.py:510-641).  Inside a "unit" (one player frame of L tokens,
// one local-hub slot of K_L tokens, one global frame of K_G tokens) the mask
// is uniform, except for the token-level self edge of inactive local-hub
// rows (hier_masks.py:484-486), so blocks are classified on the unit-level
// matrix and only partial blocks are expanded to token bitmasks.

#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace hier {

struct Dims {
  int P, T, L, N, KL, KG, nblk, win, direct, no_local, mem;
  int64_t A, LS, S;
  int U;
  const int64_t* labels;
  const uint8_t* membership;
  const uint8_t* go;
  const uint8_t* active;
};

static Dims make_dims(const hier_grouping* g) {
  Dims d;
  d.P = g->P;
  d.T = g->T;
  d.L = g->L;
  d.N = g->N;
  d.KL = g->KL;
  d.KG = g->KG;
  d.nblk = g->n_block;
  d.win = g->local_attn;
  d.direct = g->direct;
  d.no_local = g->no_local;
  d.mem = g->membership_mode;
  d.A = (int64_t)g->P * g->T * g->L;
  d.LS = (int64_t)g->T * g->N * g->KL;
  d.S = d.A + d.LS + (int64_t)g->T * g->KG;
  d.U = g->P * g->T + g->T * g->N + g->T;
  d.labels = g->labels;
  d.membership = g->membership;
  d.go = g->global_only;
  d.active = g->active;
  return d;
}

struct Unit {
  int kind;  // 0 player, 1 local hub, 2 global hub, 3 padding
  int t, p, g, u;
  int64_t start, end;  // token range of the unit
};

__device__ __forceinline__ Unit unit_of_token(const Dims& d, int64_t i) {
  Unit r;
  r.p = 0;
  r.g = 0;
  r.t = 0;
  if (i < d.A) {
    const int64_t tl = (int64_t)d.T * d.L;
    r.kind = 0;
    r.p = (int)(i / tl);
    r.t = (int)((i % tl) / d.L);
    r.u = r.p * d.T + r.t;
    r.start = (int64_t)r.u * d.L;
    r.end = r.start + d.L;
  } else if (i < d.A + d.LS) {
    const int64_t loc = i - d.A;
    r.kind = 1;
    r.t = (int)(loc / ((int64_t)d.N * d.KL));
    r.g = (int)((loc % ((int64_t)d.N * d.KL)) / d.KL);
    r.u = d.P * d.T + r.t * d.N + r.g;
    r.start = d.A + ((int64_t)r.t * d.N + r.g) * d.KL;
    r.end = r.start + d.KL;
  } else if (i < d.S) {
    const int64_t glob = i - d.A - d.LS;
    r.kind = 2;
    r.t = (int)(glob / d.KG);
    r.u = d.P * d.T + d.T * d.N + r.t;
    r.start = d.A + d.LS + (int64_t)r.t * d.KG;
    r.end = r.start + d.KG;
  } else {
    r.kind = 3;
    r.u = -1;
    r.start = i;
    r.end = i + 1;
  }
  return r;
}

__device__ __forceinline__ Unit unit_of_index(const Dims& d, int u) {
  Unit r;
  r.u = u;
  r.p = 0;
  r.g = 0;
  if (u < d.P * d.T) {
    r.kind = 0;
    r.p = u / d.T;
    r.t = u % d.T;
  } else if (u < d.P * d.T + d.T * d.N) {
    const int x = u - d.P * d.T;
    r.kind = 1;
    r.t = x / d.N;
    r.g = x % d.N;
  } else {
    r.kind = 2;
    r.t = u - d.P * d.T - d.T * d.N;
  }
  r.start = r.end = 0;
  return r;
}

__device__ __forceinline__ bool act(const Dims& d, int t, int g) {
  return d.active[(int64_t)t * d.N + g] != 0;
}

// player p (at frame t) belongs to group g
__device__ __forceinline__ bool in_group(const Dims& d, int t, int p, int g) {
  if (d.mem) return d.membership[((int64_t)t * d.N + g) * d.P + p] != 0;
  return d.labels[(int64_t)t * d.P + p] == (int64_t)g;
}

__device__ __forceinline__ bool share_group(const Dims& d, int t, int p, int o) {
  if (d.mem) {
    for (int g = 0; g < d.N; ++g)
      if (d.membership[((int64_t)t * d.N + g) * d.P + p] &&
          d.membership[((int64_t)t * d.N + g) * d.P + o])
        return true;
    return false;
  }
  return d.labels[(int64_t)t * d.P + p] == d.labels[(int64_t)t * d.P + o];
}

__device__ __forceinline__ bool global_only_at(const Dims& d, int t, int p) {
  return d.go[(int64_t)t * d.P + p] != 0;
}

// Unit-level edge predicate: the eleven edge sets of the dense mask
// (hier_masks.py:463-507 labels, :599-641 membership) minus the token-level
// inactive-local self edge.
__device__ bool unit_edge(const Dims& d, const Unit& q, const Unit& k) {
  if (q.kind == 3 || k.kind == 3) return false;
  const int qb = q.t / d.nblk, kb = k.t / d.nblk;
  const bool win = (kb <= qb) && (d.win == -1 || q.t - k.t < d.win);
  if (q.kind == 0) {
    if (k.kind == 0) {
      if (q.p == k.p) return win;
      if (!d.direct) return false;
      return (qb == kb) && share_group(d, q.t, q.p, k.p);
    }
    if (k.kind == 1) return win && act(d, k.t, k.g) && in_group(d, q.t, q.p, k.g);
    return win && (d.no_local || (d.mem && global_only_at(d, q.t, q.p)));
  }
  if (q.kind == 1) {
    if (!act(d, q.t, q.g)) return false;
    if (k.kind == 0) return win && in_group(d, q.t, k.p, q.g);
    if (k.kind == 1) return win && q.g == k.g && act(d, k.t, k.g);
    return win;
  }
  // global query
  if (k.kind == 1) return win && act(d, k.t, k.g);
  if (k.kind == 2) return win;
  return win && (d.no_local || (d.mem && global_only_at(d, k.t, k.p)));
}

__device__ __forceinline__ bool inactive_local(const Dims& d, const Unit& q) {
  return q.kind == 1 && !act(d, q.t, q.g);
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------

__global__ void dense_mask_kernel(Dims d, int64_t row0, int64_t nrows, uint8_t* out) {
  const int64_t total = nrows * d.S;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qi = row0 + e / d.S;
    const int64_t ki = e % d.S;
    const Unit q = unit_of_token(d, qi);
    const Unit k = unit_of_token(d, ki);
    bool m = unit_edge(d, q, k);
    if (!m && qi == ki && inactive_local(d, q)) m = true;
    out[e] = m ? 1 : 0;
  }
}

__global__ void unit_matrix_kernel(Dims d, uint8_t* M) {
  const int64_t total = (int64_t)d.U * d.U;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const Unit q = unit_of_index(d, (int)(e / d.U));
    const Unit k = unit_of_index(d, (int)(e % d.U));
    M[e] = unit_edge(d, q, k) ? 1 : 0;
  }
}

// class: 0 empty, 1 partial, 2 full (Flex semantics: padded rows/cols masked)
__global__ void block_classify_kernel(Dims d, const uint8_t* M, int nb, uint8_t* cls) {
  const int64_t total = (int64_t)nb * nb;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int qb = (int)(e / nb), kb = (int)(e % nb);
    const int64_t r0 = (int64_t)qb * 128, c0 = (int64_t)kb * 128;
    uint8_t c = 0;
    if (r0 < d.S && c0 < d.S) {
      const int64_t r1 = min(r0 + 128, d.S), c1 = min(c0 + 128, d.S);
      bool any = false, all = (r1 - r0 == 128) && (c1 - c0 == 128);
      for (int64_t i = r0; i < r1;) {
        const Unit q = unit_of_token(d, i);
        const int64_t qe = min(q.end, r1);
        for (int64_t j = c0; j < c1;) {
          const Unit k = unit_of_token(d, j);
          const bool m = M[(int64_t)q.u * d.U + k.u] != 0;
          any |= m;
          all &= m;
          j = min(k.end, c1);
        }
        if (inactive_local(d, q) && max(i, c0) < min(qe, c1)) any = true;
        i = qe;
      }
      c = any ? (all ? 2 : 1) : 0;
    }
    cls[e] = c;
  }
}

// one warp per query block: counts of partial / full blocks
__global__ void block_count_kernel(const uint8_t* cls, int nb, int32_t* kv_num,
                                   int32_t* full_num) {
  const int qb = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (qb >= nb) return;
  int np = 0, nf = 0;
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    const uint8_t c = kb < nb ? cls[(int64_t)qb * nb + kb] : 0;
    np += __popc(__ballot_sync(0xffffffffu, c == 1));
    nf += __popc(__ballot_sync(0xffffffffu, c == 2));
  }
  if (lane == 0) {
    kv_num[qb] = np;
    full_num[qb] = nf;
  }
}

// Exclusive scan of up to ~1e6 int32 counts by one block (used once per plan).
__global__ void scan_kernel(const int32_t* in, int n, int32_t* out, int32_t* total) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int32_t x = i < n ? in[i] : 0;
    int32_t v = x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) warp_sums[w] = v;
    __syncthreads();
    if (w == 0) {
      const int nw = blockDim.x / 32;
      int32_t s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      if (lane < nw) warp_sums[lane] = s;
    }
    __syncthreads();
    const int32_t prefix = carry + (w > 0 ? warp_sums[w - 1] : 0) + v - x;
    if (i < n) out[i] = prefix;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = prefix + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[n] = carry;
    if (total) *total = carry;
  }
}

// one warp per query block: ascending partial / full block lists
__global__ void block_fill_kernel(const uint8_t* cls, int nb, const int32_t* kv_off,
                                  int32_t* kv_idx, const int32_t* full_off,
                                  int32_t* full_idx) {
  const int qb = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (qb >= nb) return;
  int np = kv_off[qb], nf = full_off[qb];
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    const uint8_t c = kb < nb ? cls[(int64_t)qb * nb + kb] : 0;
    const unsigned bp = __ballot_sync(0xffffffffu, c == 1);
    const unsigned bf = __ballot_sync(0xffffffffu, c == 2);
    const unsigned lower = (1u << lane) - 1u;
    if (c == 1) kv_idx[np + __popc(bp & lower)] = kb;
    if (c == 2) full_idx[nf + __popc(bf & lower)] = kb;
    np += __popc(bp);
    nf += __popc(bf);
  }
}

// Query pairs: pair p holds query blocks 2p and 2p+1 (the attention kernel's
// two halves).  A key block is listed for the pair when either half sees it.
__device__ __forceinline__ uint8_t cls_at(const uint8_t* cls, int nb, int qb, int kb) {
  return (qb < nb && kb < nb) ? cls[(int64_t)qb * nb + kb] : 0;
}

// one warp per query pair: number of key blocks used by either half
__global__ void pair_count_kernel(const uint8_t* cls, int nb, int np, int32_t* cnt) {
  const int p = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (p >= np) return;
  int n = 0;
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    const bool any = (cls_at(cls, nb, 2 * p, kb) | cls_at(cls, nb, 2 * p + 1, kb)) != 0;
    n += __popc(__ballot_sync(0xffffffffu, any));
  }
  if (lane == 0) cnt[p] = n;
}

// one warp per query pair: the pair record and its ascending key-tile list
// (pool rows of the two 64-key halves, per-half mask selector: -1 full,
// -2 skip, otherwise the Flex partial-list index of that half's block)
__global__ void pair_plan_fill_kernel(Dims d, const uint8_t* cls, int nb, int np,
                                      const int32_t* kv_off, const int32_t* pair_off,
                                      const int32_t* page_table, int32_t* pairs,
                                      int32_t* kv_tiles) {
  const int p = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (p >= np) return;
  const int qb0 = 2 * p, qb1 = 2 * p + 1;
  if (lane == 0) {
    int32_t* rec = pairs + (int64_t)p * 8;
    rec[0] = qb0 * 128;
    rec[1] = (int32_t)min((int64_t)128, d.S - (int64_t)qb0 * 128);
    rec[2] = qb1 < nb ? qb1 * 128 : qb0 * 128;
    rec[3] = qb1 < nb ? (int32_t)min((int64_t)128, d.S - (int64_t)qb1 * 128) : 0;
    rec[4] = pair_off[p];
    rec[5] = pair_off[p + 1];
    rec[6] = 0;
    rec[7] = 0;
  }
  int pos = pair_off[p];
  int p0 = kv_off[qb0], p1 = qb1 < nb ? kv_off[qb1] : 0;
  for (int kb0 = 0; kb0 < nb; kb0 += 32) {
    const int kb = kb0 + lane;
    const uint8_t c0 = cls_at(cls, nb, qb0, kb), c1 = cls_at(cls, nb, qb1, kb);
    const unsigned ba = __ballot_sync(0xffffffffu, (c0 | c1) != 0);
    const unsigned b0 = __ballot_sync(0xffffffffu, c0 == 1);
    const unsigned b1 = __ballot_sync(0xffffffffu, c1 == 1);
    const unsigned lower = (1u << lane) - 1u;
    if ((c0 | c1) != 0) {
      int32_t* e = kv_tiles + (int64_t)(pos + __popc(ba & lower)) * 4;
      if (page_table) {
        e[0] = page_table[2 * kb] * 64;
        e[1] = page_table[2 * kb + 1] * 64;
      } else {
        e[0] = kb * 128;
        e[1] = kb * 128 + 64;
      }
      e[2] = c0 == 2 ? -1 : (c0 == 1 ? p0 + __popc(b0 & lower) : -2);
      e[3] = c1 == 2 ? -1 : (c1 == 1 ? p1 + __popc(b1 & lower) : -2);
    }
    pos += __popc(ba);
    p0 += __popc(b0);
    p1 += __popc(b1);
  }
}

__device__ __forceinline__ void set_bits(uint32_t (&w)[4], int a, int b) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int lo = max(a, 32 * i), hi = min(b, 32 * i + 32);
    if (lo < hi) {
      const int n = hi - lo;
      const uint32_t m = n == 32 ? 0xffffffffu : (((1u << n) - 1u) << (lo - 32 * i));
      w[i] |= m;
    }
  }
}

// One block (128 threads) per query block; thread = query row of the block.
// Mask index pi of a partial block equals its position in the Flex partial
// list (kv_idx), which is also the order plan_fill_kernel assigns.
__global__ void rowmask_kernel(Dims d, const uint8_t* M, const int32_t* kv_off,
                               const int32_t* kv_idx, uint4* row_masks) {
  const int qb = blockIdx.x;
  const int r = threadIdx.x;
  const int64_t qi = (int64_t)qb * 128 + r;
  const Unit q = unit_of_token(d, qi);
  const bool self = q.kind != 3 && inactive_local(d, q);
  for (int32_t pi = kv_off[qb]; pi < kv_off[qb + 1]; ++pi) {
    const int kb = kv_idx[pi];
    const int64_t c0 = (int64_t)kb * 128, c1 = min(c0 + 128, d.S);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (q.kind != 3) {
      for (int64_t j = c0; j < c1;) {
        const Unit k = unit_of_token(d, j);
        const int64_t je = min(k.end, c1);
        if (M[(int64_t)q.u * d.U + k.u]) set_bits(w, (int)(j - c0), (int)(je - c0));
        j = je;
      }
      if (self && qi >= c0 && qi < c1) set_bits(w, (int)(qi - c0), (int)(qi - c0 + 1));
    }
    row_masks[(int64_t)pi * 128 + r] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static int check_grouping(const hier_grouping* g) {
  if (!g) {
    set_error(HIER_EVALUE, "hier_grouping is NULL");
    return HIER_EVALUE;
  }
  if (g->P <= 0 || g->T <= 0 || g->L <= 0 || g->N <= 0 || g->KL < 0 || g->KG < 0 ||
      g->n_block <= 0) {
    set_error(HIER_EVALUE, "invalid hierarchical dims P=%d T=%d L=%d N=%d K_L=%d K_G=%d n=%d",
              g->P, g->T, g->L, g->N, g->KL, g->KG, g->n_block);
    return HIER_EVALUE;
  }
  if (g->membership_mode ? (!g->membership || !g->global_only) : !g->labels) {
    set_error(HIER_EVALUE, "grouping tensors missing for %s mode",
              g->membership_mode ? "membership" : "labels");
    return HIER_EVALUE;
  }
  if (!g->active) {
    set_error(HIER_EVALUE, "active_group tensor missing");
    return HIER_EVALUE;
  }
  const int64_t S = (int64_t)g->P * g->T * g->L + (int64_t)g->T * (g->N * g->KL + g->KG);
  if (S > (int64_t)INT32_MAX / 2) {
    set_error(HIER_EVALUE, "sequence too long for int32 plans: S=%lld", (long long)S);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

static int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace hier

using namespace hier;

extern "C" int hier_dense_mask(const hier_grouping* g, int64_t row0, int64_t nrows, uint8_t* out,
                               void* stream) {
  clear_error();
  int rc = check_grouping(g);
  if (rc) return rc;
  Dims d = make_dims(g);
  if (row0 < 0 || nrows < 0 || row0 + nrows > d.S) {
    set_error(HIER_EVALUE, "dense mask rows [%lld,%lld) outside [0,%lld)", (long long)row0,
              (long long)(row0 + nrows), (long long)d.S);
    return HIER_EVALUE;
  }
  if (nrows == 0) return HIER_OK;
  cudaStream_t s = (cudaStream_t)stream;
  dense_mask_kernel<<<grid_for(nrows * d.S, 256), 256, 0, s>>>(d, row0, nrows, out);
  HIER_CHECK_CUDA(cudaGetLastError(), "dense_mask_kernel launch");
  return HIER_OK;
}

extern "C" int hier_block_workspace_size(const hier_grouping* g, size_t* bytes) {
  clear_error();
  int rc = check_grouping(g);
  if (rc) return rc;
  Dims d = make_dims(g);
  const int64_t nb = (d.S + 127) / 128;
  const int64_t np = (nb + 1) / 2;
  *bytes = align256((size_t)d.U * d.U) + align256((size_t)(nb * nb)) +
           2 * align256((size_t)(np + 1) * sizeof(int32_t));
  return HIER_OK;
}

extern "C" int hier_block_mask_build(const hier_grouping* g, void* workspace, int32_t* kv_num,
                                     int32_t* kv_off, int32_t* kv_idx, int32_t* full_num,
                                     int32_t* full_off, int32_t* full_idx, int32_t* totals,
                                     void* stream) {
  clear_error();
  int rc = check_grouping(g);
  if (rc) return rc;
  Dims d = make_dims(g);
  const int nb = (int)((d.S + 127) / 128);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* M = (uint8_t*)workspace;
  uint8_t* cls = M + align256((size_t)d.U * d.U);
  unit_matrix_kernel<<<grid_for((int64_t)d.U * d.U, 256), 256, 0, s>>>(d, M);
  block_classify_kernel<<<grid_for((int64_t)nb * nb, 128), 128, 0, s>>>(d, M, nb, cls);
  block_count_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_num, full_num);
  scan_kernel<<<1, 1024, 0, s>>>(kv_num, nb, kv_off, totals);
  scan_kernel<<<1, 1024, 0, s>>>(full_num, nb, full_off, totals ? totals + 1 : nullptr);
  block_fill_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_off, kv_idx, full_off, full_idx);
  HIER_CHECK_CUDA(cudaGetLastError(), "block mask kernels launch");
  return HIER_OK;
}

extern "C" int hier_block_plan_build(const hier_grouping* g, void* workspace,
                                     const int32_t* kv_off, const int32_t* kv_idx,
                                     const int32_t* full_off, const int32_t* full_idx,
                                     const int32_t* page_table, int32_t* q_pairs,
                                     int32_t* kv_tiles, uint32_t* row_masks, int32_t* order,
                                     int32_t* n_kv_tiles, void* stream) {
  clear_error();
  int rc = check_grouping(g);
  if (rc) return rc;
  (void)full_off;
  (void)full_idx;
  Dims d = make_dims(g);
  const int nb = (int)((d.S + 127) / 128);
  const int np = (nb + 1) / 2;
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* M = (uint8_t*)workspace;
  uint8_t* cls = M + align256((size_t)d.U * d.U);
  int32_t* pair_cnt = (int32_t*)(cls + align256((size_t)nb * nb));
  int32_t* pair_off = (int32_t*)((uint8_t*)pair_cnt + align256((size_t)(np + 1) * sizeof(int32_t)));
  pair_count_kernel<<<(np + 7) / 8, 256, 0, s>>>(cls, nb, np, pair_cnt);
  scan_kernel<<<1, 1024, 0, s>>>(pair_cnt, np, pair_off, n_kv_tiles);
  pair_plan_fill_kernel<<<(np + 7) / 8, 256, 0, s>>>(d, cls, nb, np, kv_off, pair_off, page_table,
                                                     q_pairs, kv_tiles);
  if (row_masks) rowmask_kernel<<<nb, 128, 0, s>>>(d, M, kv_off, kv_idx, (uint4*)row_masks);
  if (order) order_by_work_kernel<8><<<grid_for(np, 128), 128, 0, s>>>(q_pairs, np, order);
  HIER_CHECK_CUDA(cudaGetLastError(), "block plan kernels launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Block plan of a caller's dense bool mask, or of no mask
// ---------------------------------------------------------------------------
//
// The reference's full-sequence attention also runs with a plain dense bool
// mask [S,S] (flash_attention(q, k, v, num_heads, mask=...),
// multics/models/attention.py:39-54) or with none.  The same 128x128 block
// plan is built from the mask bytes themselves: blocks are classified by
// reading every byte once (coalesced 128-byte row segments per warp), and
// partial blocks get per-row key bitmasks by warp ballots.  A NULL mask
// means every (query, key) pair inside [0,S)^2 is allowed.

namespace hier {

// Byte (r, c) of the mask as a bool; outside [0,S)^2 false.
__device__ __forceinline__ bool dense_at(const uint8_t* mask, int64_t ld, int64_t S, int64_t r,
                                         int64_t c) {
  if (r >= S || c >= S) return false;
  return mask ? mask[r * ld + c] != 0 : true;
}

// One 128-thread block per 128x128 block (grid-stride): each warp reads 32
// rows of the block, one 128-byte row segment per step (lane l: columns
// 4l..4l+3, one 32-bit load when the rows are 4-byte aligned).
__global__ void dense_classify_kernel(const uint8_t* mask, int64_t ld, int64_t S, int nb,
                                      bool vec4, uint8_t* cls) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int any_s[4], all_s[4];
  for (int64_t e = blockIdx.x; e < (int64_t)nb * nb; e += gridDim.x) {
    const int qb = (int)(e / nb), kb = (int)(e % nb);
    const int64_t r0 = (int64_t)qb * 128, c0 = (int64_t)kb * 128 + 4 * lane;
    bool any = false, all = true;
    for (int i = 0; i < 32; ++i) {
      const int64_t r = r0 + 32 * w + i;
      bool b[4];
      if (mask && vec4 && r < S && c0 + 3 < S) {
        const uint32_t x = *reinterpret_cast<const uint32_t*>(mask + r * ld + c0);
        b[0] = (x & 0xffu) != 0, b[1] = (x & 0xff00u) != 0;
        b[2] = (x & 0xff0000u) != 0, b[3] = (x & 0xff000000u) != 0;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = dense_at(mask, ld, S, r, c0 + j);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        any |= b[j];
        all &= b[j];
      }
    }
    any = __any_sync(0xffffffffu, any);
    all = __all_sync(0xffffffffu, all);
    if (lane == 0) {
      any_s[w] = any;
      all_s[w] = all;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const bool a = any_s[0] | any_s[1] | any_s[2] | any_s[3];
      const bool f = all_s[0] & all_s[1] & all_s[2] & all_s[3];
      cls[e] = a ? (f ? 2 : 1) : 0;
    }
    __syncthreads();
  }
}

// One 128-thread block per query block; warp w builds the bitmasks of rows
// 32w..32w+31 of every partial block of the row (lane l reads columns l,
// l+32, l+64, l+96; ballots give the four 32-bit words).
__global__ void dense_rowmask_kernel(const uint8_t* mask, int64_t ld, int64_t S,
                                     const int32_t* kv_off, const int32_t* kv_idx,
                                     uint4* row_masks) {
  const int qb = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int32_t pi = kv_off[qb]; pi < kv_off[qb + 1]; ++pi) {
    const int64_t c0 = (int64_t)kv_idx[pi] * 128;
    for (int i = 0; i < 32; ++i) {
      const int rr = 32 * w + i;
      const int64_t r = (int64_t)qb * 128 + rr;
      uint32_t word[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        word[j] = __ballot_sync(0xffffffffu, dense_at(mask, ld, S, r, c0 + 32 * j + lane));
      if (lane == 0) row_masks[(int64_t)pi * 128 + rr] = make_uint4(word[0], word[1], word[2], word[3]);
    }
  }
}

static int check_dense(const uint8_t* mask, int64_t S, int64_t ld) {
  if (S <= 0 || S > (int64_t)INT32_MAX / 2) {
    set_error(HIER_EVALUE, "dense mask plan: sequence length %lld out of range", (long long)S);
    return HIER_EVALUE;
  }
  if (mask && ld < S) {
    set_error(HIER_EVALUE, "dense mask row stride %lld is shorter than S=%lld", (long long)ld,
              (long long)S);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

}  // namespace hier

extern "C" int hier_dense_block_workspace_size(int64_t S, size_t* bytes) {
  clear_error();
  int rc = check_dense(nullptr, S, S);
  if (rc) return rc;
  const int64_t nb = (S + 127) / 128;
  const int64_t np = (nb + 1) / 2;
  *bytes = align256((size_t)(nb * nb)) + 2 * align256((size_t)(np + 1) * sizeof(int32_t));
  return HIER_OK;
}

extern "C" int hier_dense_block_mask_build(const uint8_t* mask, int64_t S, int64_t ld,
                                           void* workspace, int32_t* kv_num, int32_t* kv_off,
                                           int32_t* kv_idx, int32_t* full_num,
                                           int32_t* full_off, int32_t* full_idx,
                                           int32_t* totals, void* stream) {
  clear_error();
  int rc = check_dense(mask, S, ld);
  if (rc) return rc;
  const int nb = (int)((S + 127) / 128);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* cls = (uint8_t*)workspace;
  const bool vec4 = mask && ((uintptr_t)mask % 4 == 0) && (ld % 4 == 0);
  const int64_t blocks = (int64_t)nb * nb;
  dense_classify_kernel<<<(int)(blocks < 148 * 16 ? blocks : 148 * 16), 128, 0, s>>>(
      mask, ld, S, nb, vec4, cls);
  block_count_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_num, full_num);
  scan_kernel<<<1, 1024, 0, s>>>(kv_num, nb, kv_off, totals);
  scan_kernel<<<1, 1024, 0, s>>>(full_num, nb, full_off, totals ? totals + 1 : nullptr);
  block_fill_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_off, kv_idx, full_off, full_idx);
  HIER_CHECK_CUDA(cudaGetLastError(), "dense block mask kernels launch");
  return HIER_OK;
}

extern "C" int hier_dense_block_plan_build(const uint8_t* mask, int64_t S, int64_t ld,
                                           void* workspace, const int32_t* kv_off,
                                           const int32_t* kv_idx, int32_t* q_pairs,
                                           int32_t* kv_tiles, uint32_t* row_masks,
                                           int32_t* order, int32_t* n_kv_tiles, void* stream) {
  clear_error();
  int rc = check_dense(mask, S, ld);
  if (rc) return rc;
  const int nb = (int)((S + 127) / 128);
  const int np = (nb + 1) / 2;
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* cls = (uint8_t*)workspace;
  int32_t* pair_cnt = (int32_t*)(cls + align256((size_t)nb * nb));
  int32_t* pair_off = (int32_t*)((uint8_t*)pair_cnt + align256((size_t)(np + 1) * sizeof(int32_t)));
  Dims d;
  memset(&d, 0, sizeof(d));
  d.S = S;
  pair_count_kernel<<<(np + 7) / 8, 256, 0, s>>>(cls, nb, np, pair_cnt);
  scan_kernel<<<1, 1024, 0, s>>>(pair_cnt, np, pair_off, n_kv_tiles);
  pair_plan_fill_kernel<<<(np + 7) / 8, 256, 0, s>>>(d, cls, nb, np, kv_off, pair_off, nullptr,
                                                     q_pairs, kv_tiles);
  if (row_masks)
    dense_rowmask_kernel<<<nb, 128, 0, s>>>(mask, ld, S, kv_off, kv_idx, (uint4*)row_masks);
  if (order) order_by_work_kernel<8><<<grid_for(np, 128), 128, 0, s>>>(q_pairs, np, order);
  HIER_CHECK_CUDA(cudaGetLastError(), "dense block plan kernels launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Split-KV form of a query-pair plan
// ---------------------------------------------------------------------------
//
// Pair p becomes `chunks` pairs over consecutive parts of its key-tile list,
// flagged as partial rows in slot c (q_pairs[7] = 1 | c << 8): a plan whose
// pairs are few and long (one cached step: 21 pairs x heads, about 2.4
// waves of CTAs on 148 SMs) runs as shorter CTAs that balance across the
// SMs, and the slots are merged by log-sum-exp afterwards
// (hier_lse_gather_merge).

namespace hier {

__global__ void split_kv_kernel(const int4* in, int np, int chunks, int4* out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < np * chunks;
       i += gridDim.x * blockDim.x) {
    const int p = i / chunks, c = i % chunks;
    const int4 q = in[2 * p], k = in[2 * p + 1];
    const int len = k.y - k.x;
    const int b = k.x + (int)((int64_t)len * c / chunks);
    const int e = k.x + (int)((int64_t)len * (c + 1) / chunks);
    out[2 * i] = q;
    out[2 * i + 1] = make_int4(b, e, k.z, 1 | (c << 8));
  }
}

}  // namespace hier

extern "C" int hier_plan_split_kv(const int32_t* q_pairs, int32_t n_pairs, int32_t chunks,
                                  int32_t* out_pairs, int32_t* order, void* stream) {
  clear_error();
  if (n_pairs < 0 || chunks < 1 || chunks > 255 || (int64_t)n_pairs * chunks > INT32_MAX / 8) {
    set_error(HIER_EVALUE, "hier_plan_split_kv: %d pairs x %d chunks", n_pairs, chunks);
    return HIER_EVALUE;
  }
  if (n_pairs == 0) return HIER_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int n = n_pairs * chunks;
  split_kv_kernel<<<grid_for(n, 128), 128, 0, s>>>((const int4*)q_pairs, n_pairs, chunks,
                                                    (int4*)out_pairs);
  if (order) order_by_work_kernel<8><<<grid_for(n, 128), 128, 0, s>>>(out_pairs, n, order);
  HIER_CHECK_CUDA(cudaGetLastError(), "split_kv_kernel launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Plan of a batched attention under one mask shared by every batch entry
// ---------------------------------------------------------------------------
//
// The action branch of the reference's DiT block calls
// flash_attention(q, k, v, num_heads, mask) on B independent sequences with
// one bool mask [Lq, Lk] broadcast over the batch (multics/models/
// attention.py:39-54): the per-frame mouse attention (B = players x patches,
// Lq = Lk = frames, get_temporal_block_causal_mask, hier_masks.py:1152-1166;
// blocks.py:441-447,684-686), the keyboard cross-attention (B = players,
// Lq = frames x patches, Lk = frames x 12, the frame mask repeated,
// blocks.py:446-448,693-697) and their cached forms over a rolling window
// (blocks.py:256-375).  Query row b*Lq + i sees key row b*Lk + j iff
// mask[i, j].  Short sequences are packed: g = min(128/Lq, 128/Lk) batch
// entries (a "unit") share one 128-row query tile and one 128-key tile, with
// block-diagonal row masks.  Query tiles are paired two per CTA as in every
// plan; a pair's key tiles cover the key rows its query rows see (one range
// when both tiles are in the same unit, one range per tile otherwise).

namespace hier {

struct SharedMaskDims {
  int64_t B, Lq, Lk, ld;
  int64_t g;        // batch entries per unit
  int64_t nqt;      // query tiles per unit
  int64_t n_tiles;  // query tiles in all
  int64_t n_pairs;
  int64_t cap;      // kv_tiles entries (and mask pairs) reserved per pair
  int aligned;      // 128-row query tiles of the flat rows, key tiles on the 128-row grid
};

static int shared_mask_dims(int64_t B, int64_t Lq, int64_t Lk, int aligned, SharedMaskDims* d) {
  if (B < 1 || Lq < 1 || Lk < 1) {
    set_error(HIER_EVALUE, "shared-mask plan: B=%lld, Lq=%lld, Lk=%lld must be positive",
              (long long)B, (long long)Lq, (long long)Lk);
    return HIER_EVALUE;
  }
  // key rows are addressed with 24 bits (stream << 24 | row); 256 rows of
  // slack keep a tile's second half inside that range
  if (B * Lq > (int64_t)INT32_MAX / 2 || B * Lk > (int64_t)(1 << 24) - 256) {
    set_error(HIER_EVALUE, "shared-mask plan: %lld query rows / %lld key rows exceed the plan's "
              "row range", (long long)(B * Lq), (long long)(B * Lk));
    return HIER_EVALUE;
  }
  d->B = B, d->Lq = Lq, d->Lk = Lk, d->ld = Lk;
  const int64_t g = (Lq <= 128 && Lk <= 128) ? (128 / Lq < 128 / Lk ? 128 / Lq : 128 / Lk) : 1;
  d->g = g < B ? g : B;
  const int64_t units = (B + d->g - 1) / d->g;
  d->nqt = (d->g * Lq + 127) / 128;
  d->n_tiles = units * d->nqt;
  d->n_pairs = (d->n_tiles + 1) / 2;
  d->cap = 2 * ((d->g * Lk + 127) / 128);
  d->aligned = aligned != 0;
  if (d->aligned) {
    // one unit of every row: query tiles are the 128-row blocks of the flat
    // rows; a pair's 256 rows touch at most ceil(256/Lq) + 1 batch entries
    d->g = B;
    d->nqt = (B * Lq + 127) / 128;
    d->n_tiles = d->nqt;
    d->n_pairs = (d->n_tiles + 1) / 2;
    const int64_t span = ((256 + Lq - 1) / Lq + 1) * Lk;
    const int64_t all = (B * Lk + 127) / 128;
    d->cap = std::min(all, span / 128 + 2);
  }
  if (d->n_pairs * d->cap * 2 > (int64_t)INT32_MAX / 128) {
    set_error(HIER_EVALUE, "shared-mask plan: %lld pairs x %lld key tiles is too large",
              (long long)d->n_pairs, (long long)d->cap);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

// One 128-thread block per query pair; thread t owns row t of each tile.
__global__ void __launch_bounds__(128) shared_mask_plan_kernel(const uint8_t* __restrict__ mask,
                                                               SharedMaskDims d, int4* q_pairs,
                                                               int4* kv_tiles, uint4* masks) {
  const int64_t p = blockIdx.x;
  const int t = threadIdx.x;
  __shared__ int lo_s[2], hi_s[2], n_ent_s;
  int64_t q0[2], unit[2];
  int rows[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t tile = 2 * p + h;
    q0[h] = 0, rows[h] = 0, unit[h] = -1 - h;
    if (tile < d.n_tiles) {
      const int64_t u = tile / d.nqt, tt = tile % d.nqt;
      const int64_t ur = min(d.g * d.Lq, d.B * d.Lq - u * d.g * d.Lq);  // rows of the unit
      unit[h] = u;
      q0[h] = u * d.g * d.Lq + tt * 128;
      rows[h] = (int)min((int64_t)128, ur - tt * 128);
    }
  }
  if (rows[1] == 0) q0[1] = q0[0];
  if (t < 2) lo_s[t] = INT32_MAX, hi_s[t] = -1;
  if (t == 0) n_ent_s = 0;
  __syncthreads();
  // key rows seen by each query row: [b*Lk + first, b*Lk + last]
  int64_t rb[2], ri[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rb[h] = -1, ri[h] = 0;
    if (t < rows[h]) {
      const int64_t r = q0[h] + t;
      rb[h] = r / d.Lq, ri[h] = r - rb[h] * d.Lq;
      const uint8_t* mr = mask + ri[h] * d.ld;
      int64_t first = -1, last = -1;
      for (int64_t j = 0; j < d.Lk; ++j)
        if (mr[j]) {
          if (first < 0) first = j;
          last = j;
        }
      if (first >= 0) {
        atomicMin(&lo_s[h], (int)(rb[h] * d.Lk + first));
        atomicMax(&hi_s[h], (int)(rb[h] * d.Lk + last));
      }
    }
  }
  __syncthreads();
  // key ranges: one shared range, or one per tile
  int seg_lo[2] = {0, 0}, seg_hi[2] = {-1, -1}, seg_use[2] = {0, 0}, n_seg = 0;
  const bool has0 = hi_s[0] >= 0, has1 = hi_s[1] >= 0;
  if (has0 && has1 && unit[0] == unit[1]) {
    seg_lo[0] = min(lo_s[0], lo_s[1]), seg_hi[0] = max(hi_s[0], hi_s[1]), seg_use[0] = 3;
    n_seg = 1;
  } else if (d.aligned && (has0 || has1)) {
    seg_lo[0] = has0 ? (has1 ? min(lo_s[0], lo_s[1]) : lo_s[0]) : lo_s[1];
    seg_hi[0] = has0 ? (has1 ? max(hi_s[0], hi_s[1]) : hi_s[0]) : hi_s[1];
    seg_use[0] = (has0 ? 1 : 0) | (has1 ? 2 : 0);
    n_seg = 1;
  } else {
    if (has0) seg_lo[n_seg] = lo_s[0], seg_hi[n_seg] = hi_s[0], seg_use[n_seg++] = 1;
    if (has1) seg_lo[n_seg] = lo_s[1], seg_hi[n_seg] = hi_s[1], seg_use[n_seg++] = 2;
  }
  const int64_t kv_base = p * d.cap;
  if (d.aligned && n_seg) seg_lo[0] = seg_lo[0] / 128 * 128;  // key tiles on the 128-row grid
  for (int sgi = 0; sgi < n_seg; ++sgi) {
    for (int64_t ks = seg_lo[sgi]; ks <= seg_hi[sgi]; ks += 128) {
      const int e = n_ent_s;
      int sel[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        const bool on = (seg_use[sgi] >> h) & 1;
        if (on && t < rows[h]) {
          // keys of this row's batch entry inside [ks, ks + 128)
          const int64_t kb = rb[h] * d.Lk;
          const int64_t c_lo = max((int64_t)0, kb - ks);
          const int64_t c_hi = min((int64_t)128, kb + d.Lk - ks);
          const uint8_t* mr = mask + ri[h] * d.ld + (ks - kb);
          for (int64_t c = c_lo; c < c_hi; ++c)
            if (mr[c]) w[c >> 5] |= 1u << (c & 31);
        }
        const bool row_any = (w[0] | w[1] | w[2] | w[3]) != 0;
        const bool row_full = (w[0] & w[1] & w[2] & w[3]) == 0xffffffffu;
        const int any = __syncthreads_or(on && row_any);
        const int full = __syncthreads_and(!on || t >= rows[h] || row_full);
        const int64_t mi = (kv_base + e) * 2 + h;
        if (on && any && !full) masks[mi * 128 + t] = make_uint4(w[0], w[1], w[2], w[3]);
        sel[h] = !(on && any) ? -2 : (full ? -1 : (int)mi);
      }
      if (t == 0 && (sel[0] != -2 || sel[1] != -2)) {
        kv_tiles[kv_base + e] = make_int4((int)ks, (int)ks + 64, sel[0], sel[1]);
        n_ent_s = e + 1;
      }
      __syncthreads();
    }
  }
  if (t == 0) {
    q_pairs[2 * p] = make_int4((int)q0[0], rows[0], (int)q0[1], rows[1]);
    q_pairs[2 * p + 1] = make_int4((int)kv_base, (int)(kv_base + n_ent_s), 1, 0);
  }
}

}  // namespace hier

extern "C" int hier_shared_mask_plan_size(int64_t B, int64_t Lq, int64_t Lk, int32_t aligned,
                                          int32_t* n_pairs, int32_t* tiles_per_pair) {
  clear_error();
  SharedMaskDims d;
  int rc = shared_mask_dims(B, Lq, Lk, aligned, &d);
  if (rc) return rc;
  *n_pairs = (int32_t)d.n_pairs;
  *tiles_per_pair = (int32_t)d.cap;
  return HIER_OK;
}

extern "C" int hier_shared_mask_plan_build(const uint8_t* mask, int64_t ld, int64_t B, int64_t Lq,
                                           int64_t Lk, int32_t aligned, int32_t* q_pairs,
                                           int32_t* kv_tiles, uint32_t* tile_masks,
                                           int32_t* order, void* stream) {
  clear_error();
  SharedMaskDims d;
  int rc = shared_mask_dims(B, Lq, Lk, aligned, &d);
  if (rc) return rc;
  if (!mask || ld < Lk) {
    set_error(HIER_EVALUE, "shared-mask plan: mask is NULL or its row stride %lld < Lk=%lld",
              (long long)ld, (long long)Lk);
    return HIER_EVALUE;
  }
  d.ld = ld;
  cudaStream_t s = (cudaStream_t)stream;
  shared_mask_plan_kernel<<<(unsigned)d.n_pairs, 128, 0, s>>>(
      mask, d, (int4*)q_pairs, (int4*)kv_tiles, (uint4*)tile_masks);
  if (order)
    order_by_work_kernel<8><<<grid_for(d.n_pairs, 128), 128, 0, s>>>(q_pairs, (int)d.n_pairs,
                                                                     order);
  HIER_CHECK_CUDA(cudaGetLastError(), "shared-mask plan kernels launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free block classification: the scratch of hier_block_mask_build
// (unit matrix + block classes) lives in a fixed file-scope device array.
// Host code never dereferences or passes the array's name to a kernel: its
// device address is looked up once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
#include <mutex>

namespace hier {

static __device__ __align__(256) uint8_t g_static_scratch[HIER_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static std::mutex g_static_mu;
static void* g_static_ptr[kMaxDevices] = {};

static int static_scratch(void** out) {
  int dev = 0;
  HIER_CHECK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error(HIER_ERUNTIME, "device ordinal %d beyond the %d supported by the static scratch",
              dev, kMaxDevices);
    return HIER_ERUNTIME;
  }
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    HIER_CHECK_CUDA(cudaGetSymbolAddress(&p, g_static_scratch),
                    "cudaGetSymbolAddress(static scratch)");
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return HIER_OK;
}

}  // namespace hier

extern "C" int hier_block_mask_build_static(const hier_grouping* g, int32_t* kv_num,
                                            int32_t* kv_off, int32_t* kv_idx, int32_t* full_num,
                                            int32_t* full_off, int32_t* full_idx, int32_t* totals,
                                            void* stream) {
  clear_error();
  int rc = check_grouping(g);
  if (rc) return rc;
  Dims d = make_dims(g);
  const int nb = (int)((d.S + 127) / 128);
  const size_t m_bytes = align256((size_t)d.U * d.U);
  const size_t need = m_bytes + align256((size_t)nb * nb);
  if (need > (size_t)HIER_STATIC_SCRATCH_BYTES) {
    set_error(HIER_EVALUE,
              "hier_block_mask_build_static needs %zu bytes of scratch (U=%d units, %d blocks), "
              "more than its fixed %u-byte buffer; use hier_block_mask_build with a workspace",
              need, d.U, nb, (unsigned)HIER_STATIC_SCRATCH_BYTES);
    return HIER_EVALUE;
  }
  void* scratch = nullptr;
  rc = static_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* M = (uint8_t*)scratch;
  uint8_t* cls = M + m_bytes;
  unit_matrix_kernel<<<grid_for((int64_t)d.U * d.U, 256), 256, 0, s>>>(d, M);
  block_classify_kernel<<<grid_for((int64_t)nb * nb, 128), 128, 0, s>>>(d, M, nb, cls);
  block_count_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_num, full_num);
  scan_kernel<<<1, 1024, 0, s>>>(kv_num, nb, kv_off, totals);
  scan_kernel<<<1, 1024, 0, s>>>(full_num, nb, full_off, totals ? totals + 1 : nullptr);
  block_fill_kernel<<<(nb + 7) / 8, 256, 0, s>>>(cls, nb, kv_off, kv_idx, full_off, full_idx);
  HIER_CHECK_CUDA(cudaGetLastError(), "static block mask kernels launch");
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// Bounds check of an attention work plan before a launch.  Reads a table
// entry only after checking its index, so a corrupted plan cannot make the
// check itself read out of range.
// ---------------------------------------------------------------------------
namespace hier {

constexpr int kCheckMaxStreams = 32;

struct PlanCheckArgs {
  const int4* pairs;  // [n_pairs][2] int4
  int32_t n_pairs;
  const int4* kv_tiles;
  int64_t n_tiles, n_masks, q_rows_total;
  const int32_t* order;
  int32_t n_streams;
  int64_t stream_rows[kCheckMaxStreams];
};

// A 64-row key box: its stream exists (the kernel indexes its tensor maps by
// it) and it starts before the stream's end plus 64 rows (the second box of a
// block plan's last tile may start past the end; TMA reads such rows as 0).
__device__ __forceinline__ bool key_box_ok(const PlanCheckArgs& a, int32_t r) {
  if (r < 0) return false;
  const int s = r >> 24;
  return s < a.n_streams && (int64_t)(r & ((1 << 24) - 1)) < a.stream_rows[s] + 64;
}

__global__ void plan_check_kernel(PlanCheckArgs a, int32_t* status) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < a.n_pairs;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int4 pq = a.pairs[2 * p], pk = a.pairs[2 * p + 1];
    int bits = 0;
    const int qs[2] = {pq.x, pq.z}, qr[2] = {pq.y, pq.w};
    for (int h = 0; h < 2; ++h)
      if (qr[h] < 0 || qr[h] > 128 ||
          (qr[h] > 0 && (qs[h] < 0 || (int64_t)qs[h] + qr[h] > a.q_rows_total)))
        bits |= 2;
    if (pk.x < 0 || pk.y < pk.x || (int64_t)pk.y > a.n_tiles) {
      bits |= 1;
    } else {
      for (int e = pk.x; e < pk.y; ++e) {
        const int4 t = a.kv_tiles[e];
        const int sel[2] = {t.z, t.w};
        for (int h = 0; h < 2; ++h)
          if (sel[h] < -2 || (sel[h] >= 0 && (int64_t)sel[h] >= a.n_masks)) bits |= 4;
        if (!key_box_ok(a, t.x) || !key_box_ok(a, t.y)) bits |= 8;
      }
    }
    if (a.order && (a.order[p] < 0 || a.order[p] >= a.n_pairs)) bits |= 16;
    if (bits) atomicOr(status, bits);
  }
}

}  // namespace hier

extern "C" int hier_plan_check(const int32_t* q_pairs, int32_t n_pairs, const int32_t* kv_tiles,
                               int64_t n_tiles, int64_t n_masks, const int32_t* order,
                               int64_t q_rows_total, const int64_t* stream_rows,
                               int32_t n_streams, int32_t* status, void* stream) {
  clear_error();
  if (n_pairs < 0 || n_tiles < 0 || n_masks < 0 || q_rows_total < 0 || n_streams < 1 ||
      n_streams > kCheckMaxStreams || !stream_rows || !status ||
      (n_pairs > 0 && !q_pairs) || (n_tiles > 0 && !kv_tiles)) {
    set_error(HIER_EVALUE, "hier_plan_check: invalid arguments (pairs %d, tiles %lld, "
              "streams %d)", n_pairs, (long long)n_tiles, n_streams);
    return HIER_EVALUE;
  }
  PlanCheckArgs a{};
  a.pairs = (const int4*)q_pairs;
  a.n_pairs = n_pairs;
  a.kv_tiles = (const int4*)kv_tiles;
  a.n_tiles = n_tiles;
  a.n_masks = n_masks;
  a.q_rows_total = q_rows_total;
  a.order = order;
  a.n_streams = n_streams;
  for (int s = 0; s < n_streams; ++s) a.stream_rows[s] = stream_rows[s];
  cudaStream_t s = (cudaStream_t)stream;
  HIER_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int32_t), s), "plan check status clear");
  if (n_pairs > 0)
    plan_check_kernel<<<grid_for(n_pairs, 128), 128, 0, s>>>(a, status);
  HIER_CHECK_CUDA(cudaGetLastError(), "plan_check_kernel launch");
  return HIER_OK;
}
