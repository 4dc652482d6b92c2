// Device builders of the Tiled128 block layouts (HierTiledBlockLayout,
// multics/models/kernels/hier_tiled_attention.py:37-49), bit-exact:
//
//   * full sequence: build_hier_tiled_full_sequence_layouts (:244-429), one
//     layout per temporal block of n frames;
//   * cached step:   build_hier_tiled_cached_layout (:474-655).
//
// Per query segment the reference appends every candidate frame run of every
// stream (in a fixed order) to a dense slot list, each slot carrying the
// run's validity; the list is cut into 128-slot chunks, chunks without a
// valid slot are dropped and the last chunk is padded with (0, invalid)
// (_pack_layout, :182-241).  Here one CTA per (segment, layout) evaluates the
// candidates, scans their dense widths, flags the chunks that hold a valid
// slot and writes the kept chunks.  The same pass also builds the attention
// plan of the segment (its valid runs as 64-row key boxes, seg_plan.cuh), so
// the tiled attention entry points run on the tcgen05 kernel.

#include <limits.h>
#include <string.h>

#include "common.cuh"
#include "seg_plan.cuh"

namespace hier {
namespace {

using segplan::kThreads;
using segplan::SegSmem;
using segplan::block_scan;

constexpr int kTiledBlockM = 16;   // BLOCK_M of the reference layouts
constexpr int kTiledBlockN = 128;  // BLOCK_N (chunk size)
constexpr int kMaxCand = 2048;
constexpr int kMaxChunks = 8192;
constexpr int kStatusMissingFrame = 4;   // a query frame is missing from an agent cache
constexpr int kStatusTileOverflow = 2;

struct TDims {
  int mode;  // 0 full sequence, 1 cached
  int P, N, L, KL, KG, nb, win, direct;
  int T, R;            // full: frames, retention
  int n;               // query frames per layout (full: nb, cached: n_frames)
  int fa, fl, fg;      // cached: retained frames per stream
  int n_layouts, nA, nLs, n_seg;
  int pgA, pgL, pgG, npA, npL, npG;  // programs / attention pairs per segment kind
  int n_prog, n_pairs;               // per layout
  int use_glob_q;
  int64_t A, GS;       // full: agent rows, first global row; cached: local / global pool start
};

struct TSeg {
  int type, p, g, qrel, q0, ql;
};

__device__ __forceinline__ int64_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ bool temporal(const TDims& d, int64_t qf, int64_t kf) {
  if (floordiv(kf, d.nb) > floordiv(qf, d.nb)) return false;
  return d.win == -1 || (qf - kf) < d.win;
}

__device__ TSeg tseg_of(const TDims& d, int layout, int s) {
  TSeg r;
  r.p = r.g = 0;
  if (s < d.nA) {
    r.type = 0;
    r.p = s / d.n;
    r.qrel = s % d.n;
    r.ql = d.L;
  } else if (s < d.nA + d.nLs) {
    const int t = s - d.nA;
    r.type = 1;
    r.qrel = t / d.N;
    r.g = t % d.N;
    r.ql = d.KL;
  } else {
    r.type = 2;
    r.qrel = s - d.nA - d.nLs;
    r.ql = d.KG;
  }
  if (d.mode == 0) {
    const int qf = layout * d.n + r.qrel;
    r.q0 = r.type == 0   ? (r.p * d.T + qf) * d.L
           : r.type == 1 ? (int)(d.A + (int64_t)(qf * d.N + r.g) * d.KL)
                         : (int)(d.GS + (int64_t)qf * d.KG);
  } else {
    const int aq = d.P * d.n * d.L, lq = d.n * d.N * d.KL;
    r.q0 = r.type == 0   ? r.p * d.n * d.L + r.qrel * d.L
           : r.type == 1 ? aq + r.qrel * d.N * d.KL + r.g * d.KL
                         : aq + lq + r.qrel * d.KG;
  }
  return r;
}

struct Frames {  // cached-mode frame accessors
  const hier_tiled_grouping& g;
  const TDims& d;
  __device__ int64_t agent(int p, int fi) const { return g.agent_frames[p][(int64_t)fi * d.L]; }
  __device__ int64_t local(int gi, int fi) const { return g.local_frames[gi][(int64_t)fi * d.KL]; }
  __device__ int64_t glob(int fi) const { return g.global_frames[(int64_t)fi * d.KG]; }
  __device__ bool local_active(int gi, int fi) const {
    const uint8_t* a = g.local_active[gi] + (int64_t)fi * d.KL;
    for (int t = 0; t < d.KL; ++t)
      if (a[t]) return true;
    return false;
  }
  __device__ int64_t query(int qrel) const {
    return d.use_glob_q ? glob(d.fg - d.n + qrel) : agent(0, d.fa - d.n + qrel);
  }
};

// Number of candidate runs of a segment kind.
__device__ __forceinline__ int n_candidates(const TDims& d, int type, int Rb) {
  if (d.mode == 0) {
    if (type == 0) return Rb + (d.direct ? (d.P - 1) * d.n : 0) + d.N * Rb;
    if (type == 1) return d.P * Rb + 2 * Rb;
    return d.N * Rb + Rb;
  }
  if (type == 0) return d.fa + (d.direct ? (d.P - 1) * d.n : 0) + d.N * d.fl;
  if (type == 1) return d.P * d.fa + d.fl + d.fg;
  return d.N * d.fl + d.fg;
}

// Candidate c of a full-sequence segment (hier_tiled_attention.py:300-420):
// sets its first pool row, width and validity.
__device__ void full_candidate(const int64_t* labels, const uint8_t* active, const TDims& d,
                               const TSeg& sg, int bs, int ret0, int Rb, int c, int* base,
                               int* width, bool* valid) {
  const int qf = bs + sg.qrel;
  auto ab = [&](int p, int f) { return (p * d.T + f) * d.L; };
  auto lb = [&](int gi, int f) { return (int)(d.A + (int64_t)(f * d.N + gi) * d.KL); };
  auto gb = [&](int f) { return (int)(d.GS + (int64_t)f * d.KG); };
  auto lab = [&](int f, int p) { return labels[(int64_t)f * d.P + p]; };
  auto act = [&](int f, int gi) { return active[(int64_t)f * d.N + gi] != 0; };
  if (sg.type == 0) {
    if (c < Rb) {
      const int kf = ret0 + c;
      *base = ab(sg.p, kf), *width = d.L, *valid = temporal(d, qf, kf);
      return;
    }
    c -= Rb;
    if (d.direct) {
      if (c < (d.P - 1) * d.n) {
        const int slot = c / d.n, kr = c % d.n;
        const int o = slot < sg.p ? slot : slot + 1;
        const int kf = bs + kr;
        const bool same = lab(qf, o) == lab(qf, sg.p);
        *base = ab(o, kf), *width = d.L, *valid = same && (kf / d.nb == qf / d.nb);
        return;
      }
      c -= (d.P - 1) * d.n;
    }
    const int gi = c / Rb, kf = ret0 + c % Rb;
    const int64_t qg = lab(qf, sg.p);
    *base = lb(gi, kf), *width = d.KL;
    *valid = gi == qg && act(kf, gi) && temporal(d, qf, kf);
    return;
  }
  if (sg.type == 1) {
    const bool qa = act(qf, sg.g);
    if (c < d.P * Rb) {
      const int p = c / Rb, kf = ret0 + c % Rb;
      *base = ab(p, kf), *width = d.L;
      *valid = qa && lab(qf, p) == sg.g && temporal(d, qf, kf);
      return;
    }
    c -= d.P * Rb;
    if (c < Rb) {
      const int kf = ret0 + c;
      *base = lb(sg.g, kf), *width = d.KL, *valid = qa && act(kf, sg.g) && temporal(d, qf, kf);
      return;
    }
    const int kf = ret0 + c - Rb;
    *base = gb(kf), *width = d.KG, *valid = qa && temporal(d, qf, kf);
    return;
  }
  if (c < d.N * Rb) {
    const int gi = c / Rb, kf = ret0 + c % Rb;
    *base = lb(gi, kf), *width = d.KL, *valid = act(kf, gi) && temporal(d, qf, kf);
    return;
  }
  const int kf = ret0 + c - d.N * Rb;
  *base = gb(kf), *width = d.KG, *valid = temporal(d, qf, kf);
}

// Candidate c of a cached segment (hier_tiled_attention.py:556-650).
__device__ void cached_candidate(const hier_tiled_grouping& g, const TDims& d, const TSeg& sg,
                                 int c, int* base, int* width, bool* valid, int* missing) {
  const Frames F{g, d};
  const int64_t qf = F.query(sg.qrel);
  auto ab = [&](int p, int fi) { return (p * d.fa + fi) * d.L; };
  auto lb = [&](int gi, int fi) { return (int)(d.A + (int64_t)(gi * d.fl + fi) * d.KL); };
  auto gb = [&](int fi) { return (int)(d.GS + (int64_t)fi * d.KG); };
  auto lab = [&](int p) { return g.labels[(int64_t)sg.qrel * d.P + p]; };
  if (sg.type == 0) {
    if (c < d.fa) {
      *base = ab(sg.p, c), *width = d.L, *valid = temporal(d, qf, F.agent(sg.p, c));
      return;
    }
    c -= d.fa;
    if (d.direct) {
      if (c < (d.P - 1) * d.n) {
        const int slot = c / d.n, kr = c % d.n;
        const int o = slot < sg.p ? slot : slot + 1;
        const int64_t kf = F.query(kr);
        int fi = -1;  // position of kf in agent o's cache (last occurrence wins)
        for (int i = 0; i < d.fa; ++i)
          if (F.agent(o, i) == kf) fi = i;
        if (fi < 0) {
          *missing = 1;
          fi = 0;
        }
        const bool same = lab(o) == lab(sg.p);
        *base = ab(o, fi), *width = d.L;
        *valid = same && floordiv(kf, d.nb) == floordiv(qf, d.nb);
        return;
      }
      c -= (d.P - 1) * d.n;
    }
    const int gi = c / d.fl, fi = c % d.fl;
    *base = lb(gi, fi), *width = d.KL;
    *valid = gi == lab(sg.p) && F.local_active(gi, fi) && temporal(d, qf, F.local(gi, fi));
    return;
  }
  if (sg.type == 1) {
    const bool qa = g.active[(int64_t)sg.qrel * d.N + sg.g] != 0;
    if (c < d.P * d.fa) {
      const int p = c / d.fa, fi = c % d.fa;
      *base = ab(p, fi), *width = d.L;
      *valid = qa && lab(p) == sg.g && temporal(d, qf, F.agent(p, fi));
      return;
    }
    c -= d.P * d.fa;
    if (c < d.fl) {
      *base = lb(sg.g, c), *width = d.KL;
      *valid = qa && F.local_active(sg.g, c) && temporal(d, qf, F.local(sg.g, c));
      return;
    }
    c -= d.fl;
    *base = gb(c), *width = d.KG, *valid = qa && temporal(d, qf, F.glob(c));
    return;
  }
  if (c < d.N * d.fl) {
    const int gi = c / d.fl, fi = c % d.fl;
    *base = lb(gi, fi), *width = d.KL;
    *valid = F.local_active(gi, fi) && temporal(d, qf, F.local(gi, fi));
    return;
  }
  c -= d.N * d.fl;
  *base = gb(c), *width = d.KG, *valid = temporal(d, qf, F.glob(c));
}

struct ChunkSmem {
  int* flag;  // [kMaxChunks] kept flag, then rank of kept chunks
  int* list;  // [kMaxChunks] chunk of each rank
};

size_t tiled_smem_bytes(int C) {
  return (segplan::seg_smem_ints(C) + 2 * (size_t)kMaxChunks) * sizeof(int);
}

// Fill the candidates, analyse the attended runs and the dense chunks of one
// segment.  misc[0] = logical (attended) slots, [2] boxes, [4] dense slots,
// [5] kept chunks.
__device__ void analyse_tiled(const hier_tiled_grouping& g, const TDims& d, int layout,
                              const TSeg& sg, const SegSmem& m, const ChunkSmem& ch, int* C_out) {
  const int bs = layout * d.n, be = bs + d.n;
  const int ret0 = d.mode == 0 ? max(0, be - d.R) : 0;
  const int Rb = be - ret0;
  const int C = n_candidates(d, sg.type, Rb);
  *C_out = C;
  if (threadIdx.x == 0) m.misc[3] = 0;
  __syncthreads();
  int missing = 0;
  for (int c = threadIdx.x; c < C; c += kThreads) {
    int base = 0, width = 0;
    bool valid = false;
    if (d.mode == 0) full_candidate(g.labels, g.active, d, sg, bs, ret0, Rb, c, &base, &width, &valid);
    else cached_candidate(g, d, sg, c, &base, &width, &valid, &missing);
    m.dw[c] = width;
    m.pool[c] = base;
    m.key[c] = base;  // one pool (stream 0)
    m.w[c] = valid ? width : 0;
  }
  if (missing) atomicOr(&m.misc[3], kStatusMissingFrame);
  __syncthreads();
  // dense offsets
  int* wtmp = m.misc + 8;
  int carry = 0;
  for (int base = 0; base < C; base += kThreads) {
    const int c = base + threadIdx.x;
    const int v = c < C ? m.dw[c] : 0;
    const int incl = block_scan<false>(v, wtmp) + carry;
    if (c < C) m.doff[c] = incl - v;
    if (threadIdx.x == kThreads - 1) m.misc[16] = incl;
    __syncthreads();
    carry = m.misc[16];
    __syncthreads();
  }
  const int dense = carry;
  if (threadIdx.x == 0) m.doff[C] = dense;
  const int nch = (dense + kTiledBlockN - 1) / kTiledBlockN;
  for (int k = threadIdx.x; k < nch; k += kThreads) ch.flag[k] = 0;
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += kThreads) {
    if (m.w[c] == 0) continue;
    const int k0 = m.doff[c] / kTiledBlockN, k1 = (m.doff[c] + m.dw[c] - 1) / kTiledBlockN;
    for (int k = k0; k <= k1; ++k) ch.flag[k] = 1;
  }
  __syncthreads();
  carry = 0;
  for (int base = 0; base < nch; base += kThreads) {
    const int k = base + threadIdx.x;
    const int f = k < nch ? ch.flag[k] : 0;
    const int incl = block_scan<false>(f, wtmp) + carry;
    if (f) ch.list[incl - 1] = k;
    if (threadIdx.x == kThreads - 1) m.misc[16] = incl;
    __syncthreads();
    carry = m.misc[16];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    m.misc[4] = dense;
    m.misc[5] = carry;
  }
  __syncthreads();
  segplan::analyse_runs(m, C);  // attended runs -> boxes (misc[0..2])
}

__global__ void __launch_bounds__(kThreads)
    tiled_count_kernel(const hier_tiled_grouping g, const TDims d, int32_t* kv_count,
                       int32_t* n_boxes, int64_t* slots, int32_t* status) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, kMaxCand);
  const ChunkSmem ch{m.misc + segplan::kMiscInts, m.misc + segplan::kMiscInts + kMaxChunks};
  const int layout = blockIdx.y, s = blockIdx.x;
  const TSeg sg = tseg_of(d, layout, s);
  int C;
  analyse_tiled(g, d, layout, sg, m, ch, &C);
  if (threadIdx.x == 0) {
    const int gs = layout * d.n_seg + s;
    if (kv_count) kv_count[gs] = m.misc[5] * kTiledBlockN;
    if (n_boxes) n_boxes[gs] = m.misc[2];
    if (slots) {
      slots[2 * gs] = m.misc[0];
      slots[2 * gs + 1] = m.misc[4];
    }
    if (m.misc[3] && status) atomicOr(status, m.misc[3]);
  }
}

struct TiledOut {
  const int32_t* n_boxes;
  const int64_t* kv_off;
  const int32_t* kv_width;
  int32_t* prog_qbase;
  int32_t* prog_nq;
  int32_t* prog_seg;
  int32_t* kv_index;
  uint8_t* kv_valid;
  int32_t* q_pairs;
  int32_t* kv_tiles;
  uint32_t* tile_masks;
  int32_t tile_capacity;
  int32_t* status;
};

__global__ void __launch_bounds__(kThreads)
    tiled_build_kernel(const hier_tiled_grouping g, const TDims d, const TiledOut o) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, kMaxCand);
  const ChunkSmem ch{m.misc + segplan::kMiscInts, m.misc + segplan::kMiscInts + kMaxChunks};
  const int layout = blockIdx.y, s = blockIdx.x;
  const TSeg sg = tseg_of(d, layout, s);
  // programs of BLOCK_M rows
  if (o.prog_qbase && sg.ql > 0) {
    const int per = sg.type == 0 ? d.pgA : (sg.type == 1 ? d.pgL : d.pgG);
    const int base = layout * d.n_prog +
                     (sg.type == 0   ? s * d.pgA
                      : sg.type == 1 ? d.nA * d.pgA + (s - d.nA) * d.pgL
                                     : d.nA * d.pgA + d.nLs * d.pgL + (s - d.nA - d.nLs) * d.pgG);
    for (int i = threadIdx.x; i < per; i += kThreads) {
      o.prog_qbase[base + i] = sg.q0 + i * kTiledBlockM;
      o.prog_nq[base + i] = min(kTiledBlockM, sg.ql - i * kTiledBlockM);
      o.prog_seg[base + i] = s;
    }
  }
  int C;
  analyse_tiled(g, d, layout, sg, m, ch, &C);
  if (threadIdx.x == 0 && m.misc[3] && o.status) atomicOr(o.status, m.misc[3]);
  const int dense = m.misc[4], kept = m.misc[5];
  if (o.kv_index) {
    const int width = o.kv_width[layout];
    int32_t* row = o.kv_index + o.kv_off[layout] + (int64_t)s * width;
    uint8_t* vrow = o.kv_valid + o.kv_off[layout] + (int64_t)s * width;
    const int count = kept * kTiledBlockN;
    for (int t = threadIdx.x; t < width; t += kThreads) {
      int idx = 0;
      uint8_t v = 0;
      if (t < count) {
        const int pos = ch.list[t / kTiledBlockN] * kTiledBlockN + (t % kTiledBlockN);
        if (pos < dense) {
          int lo = 0, hi = C - 1;  // last candidate starting at or before pos: it holds pos
          while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (m.doff[mid] <= pos) lo = mid;
            else hi = mid - 1;
          }
          idx = m.pool[lo] + (pos - m.doff[lo]);
          v = m.w[lo] > 0;
        }
      }
      row[t] = idx;
      vrow[t] = v;
    }
  }
  if (!o.q_pairs) return;
  const int gs = layout * d.n_seg + s;
  const int tile_base = segplan::tile_base_of(o.n_boxes, gs, m.misc + 8);
  const int n_tiles = (m.misc[2] + 1) >> 1;
  if (tile_base + n_tiles > o.tile_capacity) {
    if (threadIdx.x == 0 && o.status) atomicOr(o.status, kStatusTileOverflow);
    return;
  }
  segplan::emit_plan(m, tile_base, o.kv_tiles, o.tile_masks);
  if (sg.ql > 0) {
    const int base = layout * d.n_pairs +
                     (sg.type == 0   ? s * d.npA
                      : sg.type == 1 ? d.nA * d.npA + (s - d.nA) * d.npL
                                     : d.nA * d.npA + d.nLs * d.npL + (s - d.nA - d.nLs) * d.npG);
    segplan::emit_pairs(sg.q0, sg.ql, base, tile_base, n_tiles, o.q_pairs);
  }
}

// ---------------------------------------------------------------------------
// Player-sharded full-sequence plan
// ---------------------------------------------------------------------------
using segplan::ceil_div;

int64_t boxes_of(int64_t runs, int width) {
  return width > 0 ? runs * ceil_div(width, segplan::kBoxRows) : 0;
}

int make_tdims(const hier_tiled_grouping* g, TDims* d, int64_t* tile_cap) {
  if (!g) {
    set_error(HIER_EVALUE, "hier_tiled_grouping is NULL");
    return HIER_EVALUE;
  }
  memset(d, 0, sizeof(*d));
  d->mode = g->mode;
  d->P = g->P, d->N = g->N, d->L = g->L, d->KL = g->KL, d->KG = g->KG;
  d->nb = g->n_block, d->win = g->local_attn, d->direct = g->direct != 0;
  if (g->mode != 0 && g->mode != 1) {
    set_error(HIER_EVALUE, "unknown tiled layout mode %d", g->mode);
    return HIER_EVALUE;
  }
  if (d->P <= 0 || d->N <= 0 || d->L <= 0 || d->KL < 0 || d->KG < 0 || d->nb <= 0 ||
      !g->labels || !g->active) {
    set_error(HIER_EVALUE, "invalid Tiled128 dims P=%d N=%d L=%d K_L=%d K_G=%d n=%d", d->P, d->N,
              d->L, d->KL, d->KG, d->nb);
    return HIER_EVALUE;
  }
  int64_t dense_max = 0, boxes_seg[3] = {0, 0, 0};
  int cand_max = 0;
  if (g->mode == 0) {
    d->T = g->T;
    const int T = d->T, n = d->nb, win = d->win;
    // hier_tiled_attention.py:262-270
    if (T <= 0 || T % n != 0) {
      set_error(HIER_EVALUE, "Tiled128 requires T %% n == 0, got T=%d, n=%d", T, n);
      return HIER_EVALUE;
    }
    if (win != -1 && win < n) {
      set_error(HIER_EVALUE, "Tiled128 requires local_attn_size=-1 or >=n, got %d, n=%d", win, n);
      return HIER_EVALUE;
    }
    d->R = win == -1 ? T : win + n;
    d->n = n;
    d->n_layouts = T / n;
    d->A = (int64_t)d->P * T * d->L;
    d->GS = d->A + (int64_t)T * d->N * d->KL;
    const int R = d->R < T ? d->R : T;
    const int64_t dl = (d->direct ? (int64_t)(d->P - 1) * n : 0);
    cand_max = max(R + (int)dl + d->N * R, max(d->P * R + 2 * R, d->N * R + R));
    dense_max = max((int64_t)R * d->L + dl * d->L + (int64_t)d->N * R * d->KL,
                    max((int64_t)d->P * R * d->L + (int64_t)R * (d->KL + d->KG),
                        (int64_t)d->N * R * d->KL + (int64_t)R * d->KG));
    boxes_seg[0] = boxes_of(R + dl, d->L) + boxes_of((int64_t)d->N * R, d->KL);
    boxes_seg[1] = boxes_of((int64_t)d->P * R, d->L) + boxes_of(R, d->KL) + boxes_of(R, d->KG);
    boxes_seg[2] = boxes_of((int64_t)d->N * R, d->KL) + boxes_of(R, d->KG);
    if (d->GS + (int64_t)T * d->KG > (1 << segplan::kStreamShift) - 1) {
      set_error(HIER_EVALUE, "sequence of %lld rows exceeds %d", (long long)(d->GS + (int64_t)T * d->KG),
                (1 << segplan::kStreamShift) - 1);
      return HIER_EVALUE;
    }
  } else {
    d->n = g->n_frames, d->fa = g->fa, d->fl = g->fl, d->fg = d->KG > 0 ? g->fg : 0;
    if (d->n <= 0 || d->fa <= 0 || d->fl <= 0) {
      set_error(HIER_EVALUE, "Tiled128 requires equal agent cache lengths");
      return HIER_EVALUE;
    }
    // hier_tiled_attention.py:537-539: query frames from the global cache when
    // K_G > 0, else from agent 0, with no fallback
    d->use_glob_q = d->KG > 0;
    if ((d->use_glob_q ? d->fg : d->fa) < d->n) {
      set_error(HIER_EVALUE, "Tiled128 cannot identify the current cached query frames");
      return HIER_EVALUE;
    }
    d->n_layouts = 1;
    d->A = (int64_t)d->P * d->fa * d->L;
    d->GS = d->A + (int64_t)d->N * d->fl * d->KL;
    const int64_t dl = d->direct ? (int64_t)(d->P - 1) * d->n : 0;
    cand_max = max(d->fa + (int)dl + d->N * d->fl, max(d->P * d->fa + d->fl + d->fg,
                                                       d->N * d->fl + d->fg));
    dense_max = max((int64_t)(d->fa + dl) * d->L + (int64_t)d->N * d->fl * d->KL,
                    max((int64_t)d->P * d->fa * d->L + (int64_t)d->fl * d->KL +
                            (int64_t)d->fg * d->KG,
                        (int64_t)d->N * d->fl * d->KL + (int64_t)d->fg * d->KG));
    boxes_seg[0] = boxes_of(d->fa + dl, d->L) + boxes_of((int64_t)d->N * d->fl, d->KL);
    boxes_seg[1] = boxes_of((int64_t)d->P * d->fa, d->L) + boxes_of(d->fl, d->KL) +
                   boxes_of(d->fg, d->KG);
    boxes_seg[2] = boxes_of((int64_t)d->N * d->fl, d->KL) + boxes_of(d->fg, d->KG);
    if (d->GS + (int64_t)d->fg * d->KG > (1 << segplan::kStreamShift) - 1) {
      set_error(HIER_EVALUE, "cached pool exceeds %d rows", (1 << segplan::kStreamShift) - 1);
      return HIER_EVALUE;
    }
  }
  if (cand_max > kMaxCand || ceil_div((int)dense_max, kTiledBlockN) > kMaxChunks) {
    set_error(HIER_EVALUE, "Tiled128 segment too large for the builder (%d runs, %lld slots)",
              cand_max, (long long)dense_max);
    return HIER_EVALUE;
  }
  d->nA = d->P * d->n;
  d->nLs = d->n * d->N;
  d->n_seg = d->nA + d->nLs + d->n;
  d->pgA = ceil_div(d->L, kTiledBlockM);
  d->pgL = ceil_div(d->KL, kTiledBlockM);
  d->pgG = ceil_div(d->KG, kTiledBlockM);
  d->npA = segplan::pairs_for_rows(d->L);
  d->npL = segplan::pairs_for_rows(d->KL);
  d->npG = segplan::pairs_for_rows(d->KG);
  d->n_prog = d->nA * d->pgA + d->nLs * d->pgL + d->n * d->pgG;
  d->n_pairs = d->nA * d->npA + d->nLs * d->npL + d->n * d->npG;
  const int64_t cap = (int64_t)d->n_layouts *
                      (d->nA * ((boxes_seg[0] + 1) / 2) + d->nLs * ((boxes_seg[1] + 1) / 2) +
                       d->n * ((boxes_seg[2] + 1) / 2));
  if (cap > INT32_MAX / 4) {
    set_error(HIER_EVALUE, "Tiled128 plan too large");
    return HIER_EVALUE;
  }
  *tile_cap = cap;
  return HIER_OK;
}

}  // namespace
}  // namespace hier

using namespace hier;

extern "C" int hier_tiled_sizes(const hier_tiled_grouping* g, hier_tiled_sizes_t* out) {
  clear_error();
  TDims d;
  int64_t cap;
  int rc = make_tdims(g, &d, &cap);
  if (rc) return rc;
  if (!out) {
    set_error(HIER_EVALUE, "sizes output is NULL");
    return HIER_EVALUE;
  }
  out->n_layouts = d.n_layouts;
  out->n_seg = d.n_seg;
  out->n_prog = d.n_prog;
  out->n_pairs = d.n_pairs;
  out->tile_capacity = (int32_t)cap;
  out->q_rows = d.mode == 0 ? d.GS + (int64_t)d.T * d.KG
                            : (int64_t)d.P * d.n * d.L + (int64_t)d.n * (d.N * d.KL + d.KG);
  return HIER_OK;
}

extern "C" int hier_tiled_count(const hier_tiled_grouping* g, int32_t* kv_count, int32_t* n_boxes,
                                int64_t* slots, int32_t* status, void* stream) {
  clear_error();
  TDims d;
  int64_t cap;
  int rc = make_tdims(g, &d, &cap);
  if (rc) return rc;
  const size_t sm = tiled_smem_bytes(kMaxCand);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(tiled_count_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(tiled_count_kernel)");
  tiled_count_kernel<<<dim3(d.n_seg, d.n_layouts), kThreads, sm, (cudaStream_t)stream>>>(
      *g, d, kv_count, n_boxes, slots, status);
  HIER_CHECK_CUDA(cudaGetLastError(), "tiled_count_kernel launch");
  return HIER_OK;
}

extern "C" int hier_tiled_build(const hier_tiled_grouping* g, const int32_t* n_boxes,
                                const int64_t* kv_off, const int32_t* kv_width,
                                int32_t* prog_qbase, int32_t* prog_nq, int32_t* prog_seg,
                                int32_t* kv_index, uint8_t* kv_valid, int32_t* q_pairs,
                                int32_t* kv_tiles, uint32_t* tile_masks, int32_t tile_capacity,
                                int32_t* order, int32_t* status, void* stream) {
  clear_error();
  TDims d;
  int64_t cap;
  int rc = make_tdims(g, &d, &cap);
  if (rc) return rc;
  if ((prog_qbase != nullptr) != (prog_nq != nullptr) ||
      (prog_qbase != nullptr) != (prog_seg != nullptr) ||
      (kv_index != nullptr) != (kv_valid != nullptr) ||
      (kv_index && (!kv_off || !kv_width)) ||
      (q_pairs && (!kv_tiles || !tile_masks || !n_boxes))) {
    set_error(HIER_EVALUE, "incomplete Tiled128 output groups");
    return HIER_EVALUE;
  }
  TiledOut o;
  o.n_boxes = n_boxes;
  o.kv_off = kv_off;
  o.kv_width = kv_width;
  o.prog_qbase = prog_qbase;
  o.prog_nq = prog_nq;
  o.prog_seg = prog_seg;
  o.kv_index = kv_index;
  o.kv_valid = kv_valid;
  o.q_pairs = q_pairs;
  o.kv_tiles = kv_tiles;
  o.tile_masks = tile_masks;
  o.tile_capacity = tile_capacity;
  o.status = status;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t sm = tiled_smem_bytes(kMaxCand);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(tiled_build_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(tiled_build_kernel)");
  tiled_build_kernel<<<dim3(d.n_seg, d.n_layouts), kThreads, sm, s>>>(*g, d, o);
  HIER_CHECK_CUDA(cudaGetLastError(), "tiled_build_kernel launch");
  const int np = d.n_pairs * d.n_layouts;
  if (q_pairs && order && np > 0) {
    order_by_work_kernel<8><<<(np + 127) / 128, 128, 0, s>>>(q_pairs, np, order);
    HIER_CHECK_CUDA(cudaGetLastError(), "order_by_work_kernel launch");
  }
  return HIER_OK;
}
