// Device builders for one cached (rolling key/value cache) step of the
// hierarchical attention:
//
//   * the segment metadata of _build_metadata
//     (multics/models/kernels/hier_segmented_attention.py:156-395), bit-exact:
//     per homogeneous query segment (player x query frame: L rows; query frame
//     x group: K_L rows; query frame: K_G rows) the ascending-order list of
//     pool indices it attends to, plus the block_m programs;
//   * the attention plan of the same segments for hier_attn_fwd_streams: the
//     key list of a segment is a concatenation of contiguous runs of one
//     stream's rows (an agent, local-hub or global cache), covered by 64-row
//     key boxes read straight from that stream; two boxes make a 128-key
//     tile, and a tile whose boxes are not both full gets a per-key mask;
//   * the packed varlen plan of _get_varlen_plan
//     (multics/models/kernels/hier_packed_attention.py:32-102).
//
// One CTA builds one segment.  The segment's candidate runs (one per cached
// frame of every stream) are enumerated in the reference's order, each is
// tested by the same predicates as the reference, and block-wide scans turn
// the selected widths into key offsets, merged runs and box offsets.

#include <limits.h>
#include <string.h>

#include "common.cuh"
#include "seg_plan.cuh"

namespace hier {
namespace {

using segplan::kBoxRows;
using segplan::kStreamShift;
using segplan::kThreads;
using segplan::SegSmem;
using segplan::block_scan;

constexpr int kMaxCand = 2048;  // frames of all streams together

// status bits written by the builders
constexpr int kStatusBadFrame = 1;     // membership / global_only frame out of range
constexpr int kStatusTileOverflow = 2; // plan larger than the tile capacity

struct CDims {
  int P, N, L, KL, KG, n, nb, win, direct, no_local, mem, fa, fl, fg, T_mem;
  int nA, nLs, n_seg;  // agent segments, local-hub segments, all segments
  int cA, cL, cG, C;   // candidate runs: agent frames, local frames, global frames
  int gstream;         // stream index of the global cache
  int npA, npL, npG;   // attention pairs per segment of each kind
  int bm, pgA, pgL, pgG;  // block_m and programs per segment of each kind
  int use_glob_q;      // query frames come from the global cache (else agent 0)
};

struct Seg {
  int type;  // 0 player rows, 1 local-hub rows, 2 global-hub rows
  int p, g, qrel, q0, ql;
};

__device__ __forceinline__ int64_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q;
}

// _temporal (hier_segmented_attention.py:115-120)
__device__ __forceinline__ bool temporal(const CDims& d, int64_t qf, int64_t kf) {
  if (floordiv(kf, d.nb) > floordiv(qf, d.nb)) return false;
  return d.win == -1 || (qf - kf) < d.win;
}

// Frame of a cached frame row = the frame id of its first token (_frame_list,
// hier_segmented_attention.py:123-124).
__device__ __forceinline__ int64_t agent_frame(const hier_cached_grouping& g, const CDims& d,
                                               int p, int fi) {
  return g.agent_frames[p][(int64_t)fi * d.L];
}
__device__ __forceinline__ int64_t local_frame(const hier_cached_grouping& g, const CDims& d,
                                               int gi, int fi) {
  return g.local_frames[gi][(int64_t)fi * d.KL];
}
__device__ __forceinline__ int64_t global_frame(const hier_cached_grouping& g, const CDims& d,
                                                int fi) {
  return g.global_frames[(int64_t)fi * d.KG];
}
// _active_frames (:127-128): a local frame is active if any of its tokens is.
__device__ __forceinline__ bool local_frame_active(const hier_cached_grouping& g, const CDims& d,
                                                   int gi, int fi) {
  const uint8_t* a = g.local_active[gi] + (int64_t)fi * d.KL;
  for (int t = 0; t < d.KL; ++t)
    if (a[t]) return true;
  return false;
}
// The newest n_frames entries are the query frames (:261-267).
__device__ __forceinline__ int64_t query_frame(const hier_cached_grouping& g, const CDims& d,
                                               int qrel) {
  return d.use_glob_q ? global_frame(g, d, d.fg - d.n + qrel)
                      : agent_frame(g, d, 0, d.fa - d.n + qrel);
}

__device__ __forceinline__ bool mem_at(const hier_cached_grouping& g, const CDims& d, int64_t f,
                                       int gi, int p, int* bad) {
  if (f < 0 || f >= d.T_mem) {
    *bad = 1;
    return false;
  }
  return g.membership[(f * d.N + gi) * d.P + p] != 0;
}
__device__ __forceinline__ bool global_only_at(const hier_cached_grouping& g, const CDims& d,
                                               int64_t f, int p, int* bad) {
  if (f < 0 || f >= d.T_mem) {
    *bad = 1;
    return false;
  }
  return g.global_only[f * d.P + p] != 0;
}
__device__ __forceinline__ int64_t label_of(const hier_cached_grouping& g, const CDims& d,
                                            int qrel, int p) {
  return g.labels[(int64_t)qrel * d.P + p];
}

__device__ Seg seg_of(const CDims& d, int s) {
  Seg r;
  r.p = r.g = 0;
  const int aq = d.P * d.n * d.L, lq = d.n * d.N * d.KL;
  if (s < d.nA) {
    r.type = 0;
    r.p = s / d.n;
    r.qrel = s % d.n;
    r.q0 = r.p * d.n * d.L + r.qrel * d.L;
    r.ql = d.L;
  } else if (s < d.nA + d.nLs) {
    const int t = s - d.nA;
    r.type = 1;
    r.qrel = t / d.N;
    r.g = t % d.N;
    r.q0 = aq + r.qrel * d.N * d.KL + r.g * d.KL;
    r.ql = d.KL;
  } else {
    r.type = 2;
    r.qrel = s - d.nA - d.nLs;
    r.q0 = aq + lq + r.qrel * d.KG;
    r.ql = d.KG;
  }
  return r;
}

// Candidate run c of segment sg: returns its width if the segment attends to
// it (0 otherwise) and its stream-packed row and pool index.  Candidate order
// is the reference's append order (hier_segmented_attention.py:271-368):
//   player rows:  own agent frames, other agents (direct edges), owned local
//                 groups, global frames;
//   local rows:   member agents, the group's local frames, global frames;
//   global rows:  local frames of every group, global frames, agents.
__device__ int candidate(const hier_cached_grouping& g, const CDims& d, const Seg& sg, int64_t qf,
                         int c, int* key, int* pool, int* bad) {
  int kind, idx;
  if (sg.type == 2) {
    if (c < d.cL) {
      kind = 1;
      idx = c;
    } else if (c < d.cL + d.cG) {
      kind = 2;
      idx = c - d.cL;
    } else {
      kind = 0;
      idx = c - d.cL - d.cG;
    }
  } else if (c < d.cA) {
    kind = 0;
    idx = c;
  } else if (c < d.cA + d.cL) {
    kind = 1;
    idx = c - d.cA;
  } else {
    kind = 2;
    idx = c - d.cA - d.cL;
  }
  if (kind == 0) {
    const int slot = idx / d.fa, fi = idx % d.fa;
    int o = slot;
    if (sg.type == 0) o = slot == 0 ? sg.p : (slot - 1 < sg.p ? slot - 1 : slot);
    const int64_t kf = agent_frame(g, d, o, fi);
    bool sel = false;
    if (sg.type == 0) {
      if (o == sg.p) {
        sel = temporal(d, qf, kf);
      } else if (d.direct) {
        bool share = false;
        if (d.mem) {
          for (int gi = 0; gi < d.N && !share; ++gi)
            share = mem_at(g, d, qf, gi, sg.p, bad) && mem_at(g, d, qf, gi, o, bad);
        } else {
          share = label_of(g, d, sg.qrel, o) == label_of(g, d, sg.qrel, sg.p);
        }
        if (share && floordiv(kf, d.nb) == floordiv(qf, d.nb)) {
          bool in_q = false;
          for (int r = 0; r < d.n && !in_q; ++r) in_q = query_frame(g, d, r) == kf;
          sel = in_q;
        }
      }
    } else if (sg.type == 1) {
      const bool inside = d.mem ? mem_at(g, d, qf, sg.g, o, bad)
                                : label_of(g, d, sg.qrel, o) == sg.g;
      sel = g.q_active[sg.qrel * d.N + sg.g] && inside && temporal(d, qf, kf);
    } else {
      sel = temporal(d, qf, kf) && (d.no_local || (d.mem && global_only_at(g, d, kf, o, bad)));
    }
    *key = (o << kStreamShift) | (fi * d.L);
    *pool = (o * d.fa + fi) * d.L;
    return sel ? d.L : 0;
  }
  if (kind == 1) {
    const int gi = idx / d.fl, fi = idx % d.fl;
    bool sel;
    if (sg.type == 0) {
      sel = d.mem ? mem_at(g, d, qf, gi, sg.p, bad) : label_of(g, d, sg.qrel, sg.p) == gi;
    } else if (sg.type == 1) {
      sel = gi == sg.g && g.q_active[sg.qrel * d.N + sg.g];
    } else {
      sel = true;
    }
    sel = sel && local_frame_active(g, d, gi, fi) && temporal(d, qf, local_frame(g, d, gi, fi));
    *key = ((d.P + gi) << kStreamShift) | (fi * d.KL);
    *pool = d.P * d.fa * d.L + (gi * d.fl + fi) * d.KL;
    return sel ? d.KL : 0;
  }
  const int fi = idx;
  bool sel = temporal(d, qf, global_frame(g, d, fi));
  if (sg.type == 0)
    sel = sel && (d.no_local || (d.mem && global_only_at(g, d, qf, sg.p, bad)));
  else if (sg.type == 1)
    sel = sel && g.q_active[sg.qrel * d.N + sg.g];
  *key = (d.gstream << kStreamShift) | (fi * d.KG);
  *pool = d.P * d.fa * d.L + d.N * d.fl * d.KL + fi * d.KG;
  return sel ? d.KG : 0;
}

size_t seg_smem_bytes(int C) { return segplan::seg_smem_ints(C) * sizeof(int); }

// Evaluate the segment's candidate runs into m.w / m.key / m.pool, then
// derive its key offsets, merged runs and boxes.
__device__ void analyse_segment(const hier_cached_grouping& g, const CDims& d, const Seg& sg,
                                const SegSmem& m) {
  if (threadIdx.x == 0) m.misc[3] = 0;
  __syncthreads();
  const int64_t qf = query_frame(g, d, sg.qrel);
  int bad = 0;
  for (int c = threadIdx.x; c < d.C; c += kThreads) {
    int key = 0, pool = 0;
    m.w[c] = candidate(g, d, sg, qf, c, &key, &pool, &bad);
    m.key[c] = key;
    m.pool[c] = pool;
  }
  if (bad) atomicOr(&m.misc[3], 1);
  __syncthreads();
  segplan::analyse_runs(m, d.C);
}

__global__ void __launch_bounds__(kThreads)
    cached_count_kernel(const hier_cached_grouping g, const CDims d, int32_t* kv_count,
                        int32_t* n_boxes, int32_t* status) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, d.C);
  const int s = blockIdx.x;
  const Seg sg = seg_of(d, s);
  analyse_segment(g, d, sg, m);
  if (threadIdx.x == 0) {
    if (kv_count) kv_count[s] = m.misc[0];
    if (n_boxes) n_boxes[s] = m.misc[2];
    if (m.misc[3] && status) atomicOr(status, kStatusBadFrame);
  }
}

struct BuildOut {
  int32_t* prog_qbase;
  int32_t* prog_nq;
  int32_t* prog_seg;
  int32_t* kv_index;
  int32_t kv_width;
  int32_t* q_pairs;
  int32_t* kv_tiles;
  uint32_t* tile_masks;
  int32_t tile_capacity;
  const int32_t* n_boxes;
  int32_t* status;
};

__global__ void __launch_bounds__(kThreads)
    cached_build_kernel(const hier_cached_grouping g, const CDims d, const BuildOut o) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, d.C);
  const int s = blockIdx.x;
  const Seg sg = seg_of(d, s);
  // programs (block_m rows each)
  if (o.prog_qbase && sg.ql > 0) {
    const int per = sg.type == 0 ? d.pgA : (sg.type == 1 ? d.pgL : d.pgG);
    const int base = sg.type == 0   ? s * d.pgA
                     : sg.type == 1 ? d.nA * d.pgA + (s - d.nA) * d.pgL
                                    : d.nA * d.pgA + d.nLs * d.pgL + (s - d.nA - d.nLs) * d.pgG;
    for (int i = threadIdx.x; i < per; i += kThreads) {
      o.prog_qbase[base + i] = sg.q0 + i * d.bm;
      o.prog_nq[base + i] = min(d.bm, sg.ql - i * d.bm);
      o.prog_seg[base + i] = s;
    }
  }
  analyse_segment(g, d, sg, m);
  const int total = m.misc[0], n_box = m.misc[2];
  if (threadIdx.x == 0 && m.misc[3] && o.status) atomicOr(o.status, kStatusBadFrame);
  // kv_index row (zero padded), one warp per candidate run
  if (o.kv_index) {
    int32_t* row = o.kv_index + (int64_t)s * o.kv_width;
    const int lane = threadIdx.x & 31;
    for (int c = threadIdx.x >> 5; c < d.C; c += kThreads / 32) {
      const int wc = m.w[c];
      if (wc == 0) continue;
      const int off = m.off[c], p0 = m.pool[c];
      for (int i = lane; i < wc; i += 32) row[off + i] = p0 + i;
    }
    for (int i = total + threadIdx.x; i < o.kv_width; i += kThreads) row[i] = 0;
  }
  if (!o.q_pairs) return;
  // tiles at the exclusive scan of the counted boxes, or at a fixed stride
  // per segment (the capacity bound of one segment) without a count
  const int tile_base = o.n_boxes ? segplan::tile_base_of(o.n_boxes, s, m.misc + 8)
                                  : s * (o.tile_capacity / d.n_seg);
  const int n_tiles = (n_box + 1) >> 1;
  if (tile_base + n_tiles > o.tile_capacity) {
    if (threadIdx.x == 0 && o.status) atomicOr(o.status, kStatusTileOverflow);
    return;
  }
  segplan::emit_plan(m, tile_base, o.kv_tiles, o.tile_masks);
  if (sg.ql > 0) {
    const int base = sg.type == 0   ? s * d.npA
                     : sg.type == 1 ? d.nA * d.npA + (s - d.nA) * d.npL
                                    : d.nA * d.npA + d.nLs * d.npL + (s - d.nA - d.nLs) * d.npG;
    segplan::emit_pairs(sg.q0, sg.ql, base, tile_base, n_tiles, o.q_pairs);
  }
}

// ---------------------------------------------------------------------------
// Packed hub plan
// ---------------------------------------------------------------------------
//
// A local-hub segment has K_L query rows (16 at the released shape) and the
// longest key list of the step (its members' whole cached history), and
// the segments of one group at the n query frames see almost the same keys
// (the same members and frames; only the window edge differs).  So the
// attention plan packs them: pack g holds the rows of group g at every query
// frame (n*K_L rows, frame-major), pack N the global-hub rows of every
// frame; a pack's key list is the union of its frames' candidate runs and
// its tiles carry per-row masks (row f*K_L + s sees the keys its frame's
// segment attends to).  The packed rows are read through the attention
// kernel's second query tensor and written back through its output row map.
// The per-segment metadata (_build_metadata's contract) is unchanged.

__host__ __device__ inline int pack_count(const CDims& d) {
  if (d.no_local || d.n * d.KL > 128 || d.n * d.KG > 128) return 0;
  return d.N + (d.KG > 0 ? 1 : 0);
}

// Pack j: its type (1 local, 2 global), group, rows per frame.
__device__ __forceinline__ void pack_of(const CDims& d, int j, int* type, int* gi, int* rpf) {
  *type = j < d.N ? 1 : 2;
  *gi = j < d.N ? j : 0;
  *rpf = j < d.N ? d.KL : d.KG;
}

// Union of the pack's frames' candidate runs into m (w, key, pool) with the
// frames that select each candidate in fsel (bit qrel), then runs and boxes.
__device__ void analyse_pack(const hier_cached_grouping& g, const CDims& d, int j,
                             const SegSmem& m, int* fsel) {
  if (threadIdx.x == 0) m.misc[3] = 0;
  __syncthreads();
  int type, gi, rpf;
  pack_of(d, j, &type, &gi, &rpf);
  int bad = 0;
  for (int c = threadIdx.x; c < d.C; c += kThreads) {
    int w = 0, fs = 0, key = 0, pool = 0;
    for (int qrel = 0; qrel < d.n; ++qrel) {
      const Seg sg = seg_of(d, type == 1 ? d.nA + qrel * d.N + gi : d.nA + d.nLs + qrel);
      const int wc = candidate(g, d, sg, query_frame(g, d, qrel), c, &key, &pool, &bad);
      if (wc > 0) {
        w = wc;
        fs |= 1 << qrel;
      }
    }
    m.w[c] = w;
    m.key[c] = key;
    m.pool[c] = pool;
    fsel[c] = fs;
  }
  if (bad) atomicOr(&m.misc[3], 1);
  __syncthreads();
  segplan::analyse_runs(m, d.C);
}

__global__ void __launch_bounds__(kThreads)
    cached_pack_count_kernel(const hier_cached_grouping g, const CDims d, int32_t* n_boxes,
                             int32_t* status) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, d.C);
  analyse_pack(g, d, blockIdx.x, m, m.dw);
  if (threadIdx.x == 0) {
    n_boxes[blockIdx.x] = m.misc[2];
    if (m.misc[3] && status) atomicOr(status, kStatusBadFrame);
  }
}

struct PackOut {
  const int32_t* n_boxes;  // per pack
  int32_t tile_base;       // first kv_tiles row of the packs
  int32_t tile_end;        // capacity end
  int32_t mask_base;       // first 128-row mask (index in 128-entry units)
  int32_t q2_row0;         // query row of the first packed row
  int32_t pair_base;       // first q_pairs row of the packs
  int32_t* q_pairs;
  int32_t* kv_tiles;
  uint32_t* tile_masks;
  int32_t* status;
};

__global__ void __launch_bounds__(kThreads)
    cached_pack_build_kernel(const hier_cached_grouping g, const CDims d, const PackOut o) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, d.C);
  const int j = blockIdx.x;
  int* fsel = m.dw;
  int* sel_c = m.doff;  // selected candidates in key order
  analyse_pack(g, d, j, m, fsel);
  int type, gi, rpf;
  pack_of(d, j, &type, &gi, &rpf);
  // selected candidates in order (their key offsets m.off ascend)
  {
    int* wtmp = m.misc + 8;
    int* carry = m.misc + 16;
    int run = 0;
    for (int base = 0; base < d.C; base += kThreads) {
      const int c = base + threadIdx.x;
      const int f = (c < d.C && m.w[c] > 0) ? 1 : 0;
      const int incl = segplan::block_scan<false>(f, wtmp) + run;
      if (f) sel_c[incl - 1] = c;
      if (threadIdx.x == kThreads - 1) carry[0] = incl;
      __syncthreads();
      run = carry[0];
      __syncthreads();
    }
    if (threadIdx.x == 0) m.misc[4] = run;
    __syncthreads();
  }
  const int n_sel = m.misc[4], n_runs = m.misc[1], n_box = m.misc[2];
  const int n_tiles = (n_box + 1) >> 1;
  int tb = 0;  // tiles of the packs before j (a fixed stride without counts)
  if (o.n_boxes)
    for (int i = threadIdx.x; i < j; i += kThreads) tb += (o.n_boxes[i] + 1) >> 1;
  tb = segplan::block_scan<false>(tb, m.misc + 8);
  __shared__ int tb_s;
  if (threadIdx.x == kThreads - 1)
    tb_s = o.n_boxes ? tb : j * ((o.tile_end - o.tile_base) / pack_count(d));
  __syncthreads();
  const int tile0 = o.tile_base + tb_s;
  if (tile0 + n_tiles > o.tile_end) {
    if (threadIdx.x == 0 && o.status) atomicOr(o.status, kStatusTileOverflow);
    return;
  }
  const int mask0 = o.mask_base + tb_s;  // this pack's first 128-row mask
  const int rows = d.n * rpf;
  // key rows of the boxes and the tile selectors
  for (int b = threadIdx.x; b < 2 * n_tiles; b += kThreads) {
    const int t = b >> 1, slot = b & 1;
    const int bb = b < n_box ? b : b - 1;  // odd count: the last tile repeats its first box
    const int r = segplan::run_of_box(m, n_runs, bb);
    o.kv_tiles[(int64_t)(tile0 + t) * 4 + slot] = m.rk[r] + kBoxRows * (bb - m.rb[r]);
    if (slot == 0) {
      o.kv_tiles[(int64_t)(tile0 + t) * 4 + 2] = mask0 + t;
      o.kv_tiles[(int64_t)(tile0 + t) * 4 + 3] = -2;
    }
  }
  // per-row masks: one item per (tile, box, frame) computes the frame's two
  // words and writes them to the frame's rows
  uint4* masks = reinterpret_cast<uint4*>(o.tile_masks);
  for (int it = threadIdx.x; it < n_tiles * 2 * d.n; it += kThreads) {
    const int t = it / (2 * d.n), rem = it % (2 * d.n), slot = rem / d.n, f = rem % d.n;
    const int b = 2 * t + slot;
    uint32_t w0 = 0u, w1 = 0u;
    if (b < n_box) {
      const int r = segplan::run_of_box(m, n_runs, b);
      const int kofs0 = m.rf[r] + kBoxRows * (b - m.rb[r]);
      const int valid = min(kBoxRows, m.rf[r + 1] - kofs0);
      int lo = 0, hi = n_sel - 1;  // last selected candidate starting at or before kofs0
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (m.off[sel_c[mid]] <= kofs0) lo = mid;
        else hi = mid - 1;
      }
      for (int jj = lo; jj < n_sel; ++jj) {
        const int c = sel_c[jj];
        const int a0 = m.off[c];
        if (a0 >= kofs0 + valid) break;
        if (!((fsel[c] >> f) & 1)) continue;
        const int s0 = max(a0, kofs0) - kofs0, s1 = min(a0 + m.w[c], kofs0 + valid) - kofs0;
        for (int k = s0; k < s1; ++k) {
          if (k < 32) w0 |= 1u << k;
          else w1 |= 1u << (k - 32);
        }
      }
    }
    for (int rr = f * rpf; rr < (f + 1) * rpf; ++rr) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(masks + (int64_t)(mask0 + t) * 128 + rr);
      dst[2 * slot] = w0;
      dst[2 * slot + 1] = w1;
    }
  }
  for (int it = threadIdx.x; it < n_tiles * (128 - rows); it += kThreads) {
    const int t = it / (128 - rows), rr = rows + it % (128 - rows);
    masks[(int64_t)(mask0 + t) * 128 + rr] = make_uint4(0u, 0u, 0u, 0u);
  }
  if (threadIdx.x == 0) {
    int row0 = 0;
    for (int i = 0; i < j; ++i) row0 += d.n * (i < d.N ? d.KL : d.KG);
    int32_t* q = o.q_pairs + (int64_t)(o.pair_base + j) * 8;
    q[0] = o.q2_row0 + row0;
    q[1] = rows;
    q[2] = o.q2_row0 + row0;
    q[3] = 0;
    q[4] = tile0;
    q[5] = tile0 + n_tiles;
    q[6] = 1;  // 128-row masks
    q[7] = 0;
  }
}

int ceil_div(int a, int b) { return (a + b - 1) / b; }

int make_dims(const hier_cached_grouping* g, int32_t block_m, CDims* d) {
  if (!g) {
    set_error(HIER_EVALUE, "hier_cached_grouping is NULL");
    return HIER_EVALUE;
  }
  if (g->P <= 0 || g->N < 0 || g->L <= 0 || g->KL < 0 || g->KG < 0 || g->n_frames <= 0 ||
      g->n_block <= 0 || g->fa <= 0 || g->fl < 0 || g->fg < 0) {
    set_error(HIER_EVALUE,
              "invalid cached dims P=%d N=%d L=%d K_L=%d K_G=%d n=%d n_block=%d frames=(%d,%d,%d)",
              g->P, g->N, g->L, g->KL, g->KG, g->n_frames, g->n_block, g->fa, g->fl, g->fg);
    return HIER_EVALUE;
  }
  // hier_segmented_attention.py:217-229
  if (g->no_local) {
    if (g->KL != 0 || g->fl != 0) {
      set_error(HIER_EVALUE, "hier_no_local_hub metadata requires K_L=0 and empty local caches");
      return HIER_EVALUE;
    }
  } else if (g->N <= 0 || g->fl <= 0) {
    set_error(HIER_EVALUE, "segmented hierarchical attention requires equal local cache lengths");
    return HIER_EVALUE;
  }
  if (g->membership_mode && (!g->membership || !g->global_only)) {
    set_error(HIER_EVALUE, "membership metadata requires global_only");
    return HIER_EVALUE;
  }
  if (!g->membership_mode && !g->labels) {
    set_error(HIER_EVALUE, "labels are required without membership");
    return HIER_EVALUE;
  }
  const int n_local_streams = g->no_local ? 0 : g->N;
  if (g->P + n_local_streams + 1 > HIER_MAX_KV_STREAMS) {
    set_error(HIER_EVALUE, "%d players + %d groups exceed %d key/value streams", g->P,
              n_local_streams, HIER_MAX_KV_STREAMS);
    return HIER_EVALUE;
  }
  const bool use_glob_q = g->KG > 0 && g->fg >= g->n_frames;
  if (!use_glob_q && g->fa < g->n_frames) {
    set_error(HIER_EVALUE, "segmented hierarchical attention cannot identify the current query frames");
    return HIER_EVALUE;
  }
  d->P = g->P;
  d->N = g->N;
  d->L = g->L;
  d->KL = g->KL;
  d->KG = g->KG;
  d->n = g->n_frames;
  d->nb = g->n_block;
  d->win = g->local_attn;
  d->direct = g->direct != 0;
  d->no_local = g->no_local != 0;
  d->mem = g->membership_mode != 0;
  d->fa = g->fa;
  d->fl = g->no_local ? 0 : g->fl;
  d->fg = g->KG > 0 ? g->fg : 0;
  d->T_mem = g->T_mem;
  d->nA = d->P * d->n;
  d->nLs = d->no_local ? 0 : d->n * d->N;
  d->n_seg = d->nA + d->nLs + d->n;
  d->cA = d->P * d->fa;
  d->cL = d->N * d->fl;
  d->cG = d->fg;
  d->C = d->cA + d->cL + d->cG;
  d->gstream = d->P + n_local_streams;
  d->use_glob_q = use_glob_q;
  d->npA = ceil_div(ceil_div(d->L, 128), 2);
  d->npL = ceil_div(ceil_div(d->KL, 128), 2);
  d->npG = ceil_div(ceil_div(d->KG, 128), 2);
  d->bm = block_m > 0 ? block_m : 1;
  d->pgA = ceil_div(d->L, d->bm);
  d->pgL = ceil_div(d->KL, d->bm);
  d->pgG = ceil_div(d->KG, d->bm);
  if (d->C > kMaxCand) {
    set_error(HIER_EVALUE, "%d cached frame runs exceed the builder limit %d", d->C, kMaxCand);
    return HIER_EVALUE;
  }
  const int64_t rows[3] = {(int64_t)d->fa * d->L, (int64_t)d->fl * d->KL, (int64_t)d->fg * d->KG};
  for (int i = 0; i < 3; ++i) {
    if (rows[i] >= (1 << kStreamShift)) {
      set_error(HIER_EVALUE, "a cache of %lld rows exceeds %d", (long long)rows[i],
                (1 << kStreamShift) - 1);
      return HIER_EVALUE;
    }
  }
  const int64_t pool = (int64_t)d->P * d->fa * d->L + (int64_t)d->N * d->fl * d->KL + rows[2];
  if (pool > INT32_MAX) {
    set_error(HIER_EVALUE, "key/value pool too large for int32 indices");
    return HIER_EVALUE;
  }
  return HIER_OK;
}

// ---------------------------------------------------------------------------
// varlen plan
// ---------------------------------------------------------------------------

// cu_q / cu_k over the active segments (qn > 0 and kv_count > 0) and the
// plan's scalars; one CTA.
__global__ void __launch_bounds__(kThreads)
    varlen_offsets_kernel(const int32_t* prog_nq, const int32_t* kv_count, int n_seg,
                          int32_t* cu_q, int32_t* cu_k, int64_t* q_dst, int64_t* k_dst,
                          unsigned long long* minmax, int64_t* scalars) {
  __shared__ int scratch[40];
  int cq = 0, ck = 0, cact = 0, mq = 0, mk = 0;
  if (threadIdx.x == 0) {
    cu_q[0] = 0;
    cu_k[0] = 0;
    minmax[0] = ~0ull;
    minmax[1] = 0ull;
  }
  for (int base = 0; base < n_seg; base += kThreads) {
    const int s = base + threadIdx.x;
    const bool act = s < n_seg && prog_nq[s] > 0 && kv_count[s] > 0;
    const int nq = act ? prog_nq[s] : 0, nk = act ? kv_count[s] : 0;
    const int iq = block_scan<false>(nq, scratch) + cq;
    const int ik = block_scan<false>(nk, scratch) + ck;
    const int ia = block_scan<false>(act ? 1 : 0, scratch) + cact;
    const int xq = block_scan<true>(nq, scratch);
    const int xk = block_scan<true>(nk, scratch);
    if (act) {
      cu_q[ia] = iq;
      cu_k[ia] = ik;
    }
    if (s < n_seg) {  // per-segment destinations (-1: inactive)
      q_dst[s] = act ? iq - nq : -1;
      k_dst[s] = act ? ik - nk : -1;
    }
    if (threadIdx.x == kThreads - 1) {
      scratch[32] = iq;
      scratch[33] = ik;
      scratch[34] = ia;
      scratch[35] = xq;
      scratch[36] = xk;
    }
    __syncthreads();
    cq = scratch[32];
    ck = scratch[33];
    cact = scratch[34];
    mq = max(mq, scratch[35]);
    mk = max(mk, scratch[36]);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    scalars[0] = mq;
    scalars[1] = mk;
    scalars[4] = cact;
  }
}

// q_index / k_index (and the int32 page table) per active segment; one CTA
// per segment; min / max key index by atomics on scalars[2..3].
__global__ void __launch_bounds__(kThreads)
    varlen_fill_kernel(const int32_t* prog_qbase, const int32_t* prog_nq, const int32_t* kv_index,
                       int kv_width, const int32_t* kv_count, const int64_t* q_dst,
                       const int64_t* k_dst, int64_t* q_index, int64_t* k_index,
                       int32_t* page_indices, unsigned long long* minmax) {
  const int s = blockIdx.x;
  if (q_dst[s] < 0) return;
  const int nq = prog_nq[s], nk = kv_count[s], q0 = prog_qbase[s];
  for (int i = threadIdx.x; i < nq; i += kThreads) q_index[q_dst[s] + i] = q0 + i;
  const int32_t* row = kv_index + (int64_t)s * kv_width;
  int lo = INT_MAX, hi = INT_MIN;
  for (int i = threadIdx.x; i < nk; i += kThreads) {
    const int v = row[i];
    k_index[k_dst[s] + i] = v;
    if (page_indices) page_indices[k_dst[s] + i] = v;
    lo = min(lo, v);
    hi = max(hi, v);
  }
  // indices are non-negative: min via atomicMin, max via atomicMax
  if (lo != INT_MAX) atomicMin(&minmax[0], (unsigned long long)lo);
  if (hi != INT_MIN) atomicMax(&minmax[1], (unsigned long long)hi);
}

__global__ void varlen_finish_kernel(const unsigned long long* minmax, int64_t* scalars) {
  if (scalars[4] == 0) {
    scalars[2] = 0;
    scalars[3] = -1;
  } else {
    scalars[2] = (int64_t)minmax[0];
    scalars[3] = (int64_t)minmax[1];
  }
}

}  // namespace
}  // namespace hier

using namespace hier;

extern "C" int hier_cached_sizes(const hier_cached_grouping* g, int32_t block_m,
                                 hier_cached_sizes_t* out) {
  clear_error();
  CDims d;
  int rc = make_dims(g, block_m, &d);
  if (rc) return rc;
  if (!out) {
    set_error(HIER_EVALUE, "sizes output is NULL");
    return HIER_EVALUE;
  }
  out->n_seg = d.n_seg;
  out->n_prog = d.nA * d.pgA + d.nLs * d.pgL + d.n * d.pgG;
  out->n_pairs = d.nA * d.npA + d.nLs * d.npL + d.n * d.npG;
  out->n_streams = d.gstream + 1;
  out->n_cand = d.C;
  out->q_rows = d.P * d.n * d.L + d.n * (d.N * d.KL + d.KG);
  // every candidate run as its own boxes bounds the merged-run boxes
  const int64_t boxes_per_seg = (int64_t)d.cA * ceil_div(d.L, kBoxRows) +
                                (int64_t)d.cL * (d.KL > 0 ? ceil_div(d.KL, kBoxRows) : 0) +
                                (int64_t)d.cG * (d.KG > 0 ? ceil_div(d.KG, kBoxRows) : 0);
  const int64_t cap = (int64_t)d.n_seg * ((boxes_per_seg + 1) / 2);
  if (cap > INT32_MAX / 4) {
    set_error(HIER_EVALUE, "cached plan too large");
    return HIER_EVALUE;
  }
  out->tile_capacity = (int32_t)cap;
  out->pool_rows = (int64_t)d.P * d.fa * d.L + (int64_t)d.N * d.fl * d.KL + (int64_t)d.fg * d.KG;
  return HIER_OK;
}

extern "C" int hier_cached_count(const hier_cached_grouping* g, int32_t* kv_count,
                                 int32_t* n_boxes, int32_t* status, void* stream) {
  clear_error();
  CDims d;
  int rc = make_dims(g, 1, &d);
  if (rc) return rc;
  const size_t sm = seg_smem_bytes(d.C);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(cached_count_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(cached_count_kernel)");
  cached_count_kernel<<<d.n_seg, kThreads, sm, (cudaStream_t)stream>>>(*g, d, kv_count, n_boxes,
                                                                       status);
  HIER_CHECK_CUDA(cudaGetLastError(), "cached_count_kernel launch");
  return HIER_OK;
}

extern "C" int hier_cached_build(const hier_cached_grouping* g, int32_t block_m,
                                 const int32_t* n_boxes, int32_t* prog_qbase, int32_t* prog_nq,
                                 int32_t* prog_seg, int32_t* kv_index, int32_t kv_width,
                                 int32_t* q_pairs, int32_t* kv_tiles, uint32_t* tile_masks,
                                 int32_t tile_capacity, int32_t* order, int32_t* status,
                                 void* stream) {
  clear_error();
  CDims d;
  int rc = make_dims(g, block_m, &d);
  if (rc) return rc;
  if (block_m <= 0) {
    set_error(HIER_EVALUE, "block_m must be positive; got %d", block_m);
    return HIER_EVALUE;
  }
  if ((prog_qbase != nullptr) != (prog_nq != nullptr) ||
      (prog_qbase != nullptr) != (prog_seg != nullptr)) {
    set_error(HIER_EVALUE, "program outputs must be given together");
    return HIER_EVALUE;
  }
  if (q_pairs && (!kv_tiles || !tile_masks)) {
    set_error(HIER_EVALUE, "attention plan outputs need kv_tiles and tile_masks");
    return HIER_EVALUE;
  }
  if (kv_index && kv_width <= 0) {
    set_error(HIER_EVALUE, "kv_index needs a positive row width");
    return HIER_EVALUE;
  }
  BuildOut o;
  o.prog_qbase = prog_qbase;
  o.prog_nq = prog_nq;
  o.prog_seg = prog_seg;
  o.kv_index = kv_index;
  o.kv_width = kv_width;
  o.q_pairs = q_pairs;
  o.kv_tiles = kv_tiles;
  o.tile_masks = tile_masks;
  o.tile_capacity = tile_capacity;
  o.n_boxes = n_boxes;
  o.status = status;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t sm = seg_smem_bytes(d.C);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(cached_build_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(cached_build_kernel)");
  cached_build_kernel<<<d.n_seg, kThreads, sm, s>>>(*g, d, o);
  HIER_CHECK_CUDA(cudaGetLastError(), "cached_build_kernel launch");
  const int np = d.nA * d.npA + d.nLs * d.npL + d.n * d.npG;
  if (q_pairs && order && np > 0) {
    order_by_work_kernel<8><<<(np + 127) / 128, 128, 0, s>>>(q_pairs, np, order);
    HIER_CHECK_CUDA(cudaGetLastError(), "order_by_work_kernel launch");
  }
  return HIER_OK;
}

extern "C" int hier_varlen_workspace_size(int32_t n_seg, size_t* bytes) {
  clear_error();
  if (n_seg < 0 || !bytes) {
    set_error(HIER_EVALUE, "invalid segment count %d", n_seg);
    return HIER_EVALUE;
  }
  *bytes = (size_t)n_seg * 2 * sizeof(int64_t) + 2 * sizeof(unsigned long long);
  return HIER_OK;
}

extern "C" int hier_varlen_plan_build(const int32_t* prog_qbase, const int32_t* prog_nq,
                                      const int32_t* kv_index, int32_t kv_width,
                                      const int32_t* kv_count, int32_t n_seg, void* workspace,
                                      int64_t* q_index, int64_t* k_index, int32_t* cu_q,
                                      int32_t* cu_k, int32_t* page_indices, int64_t* scalars,
                                      void* stream) {
  clear_error();
  if (n_seg < 0 || kv_width <= 0 || !workspace || !scalars || !cu_q || !cu_k) {
    set_error(HIER_EVALUE, "invalid varlen plan arguments (segments=%d, width=%d)", n_seg,
              kv_width);
    return HIER_EVALUE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int64_t* q_dst = reinterpret_cast<int64_t*>(workspace);
  int64_t* k_dst = q_dst + n_seg;
  unsigned long long* minmax = reinterpret_cast<unsigned long long*>(k_dst + n_seg);
  varlen_offsets_kernel<<<1, kThreads, 0, s>>>(prog_nq, kv_count, n_seg, cu_q, cu_k, q_dst, k_dst,
                                               minmax, scalars);
  HIER_CHECK_CUDA(cudaGetLastError(), "varlen_offsets_kernel launch");
  if (n_seg > 0) {
    varlen_fill_kernel<<<n_seg, kThreads, 0, s>>>(prog_qbase, prog_nq, kv_index, kv_width,
                                                  kv_count, q_dst, k_dst, q_index, k_index,
                                                  page_indices, minmax);
    HIER_CHECK_CUDA(cudaGetLastError(), "varlen_fill_kernel launch");
  }
  varlen_finish_kernel<<<1, 1, 0, s>>>(minmax, scalars);
  HIER_CHECK_CUDA(cudaGetLastError(), "varlen_finish_kernel launch");
  return HIER_OK;
}

extern "C" int hier_cached_pack_sizes(const hier_cached_grouping* g,
                                      hier_cached_pack_sizes_t* out) {
  clear_error();
  CDims d;
  int rc = make_dims(g, 1, &d);
  if (rc) return rc;
  if (!out) {
    set_error(HIER_EVALUE, "pack sizes output is NULL");
    return HIER_EVALUE;
  }
  out->n_packs = pack_count(d);
  out->q2_rows = out->n_packs ? d.n * (d.N * d.KL + d.KG) : 0;
  out->agent_pairs = d.nA * d.npA;
  const int64_t boxes = (int64_t)d.cA * ceil_div(d.L, kBoxRows) +
                        (int64_t)d.cL * (d.KL > 0 ? ceil_div(d.KL, kBoxRows) : 0) +
                        (int64_t)d.cG * (d.KG > 0 ? ceil_div(d.KG, kBoxRows) : 0);
  const int64_t cap = (int64_t)out->n_packs * ((boxes + 1) / 2);
  if (cap > INT32_MAX / 512) {
    set_error(HIER_EVALUE, "packed hub plan too large");
    return HIER_EVALUE;
  }
  out->tile_capacity = (int32_t)cap;
  return HIER_OK;
}

extern "C" int hier_cached_pack_count(const hier_cached_grouping* g, int32_t* n_boxes,
                                      int32_t* status, void* stream) {
  clear_error();
  CDims d;
  int rc = make_dims(g, 1, &d);
  if (rc) return rc;
  const int np = pack_count(d);
  if (np == 0) return HIER_OK;
  const size_t sm = seg_smem_bytes(d.C);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(cached_pack_count_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(cached_pack_count_kernel)");
  cached_pack_count_kernel<<<np, kThreads, sm, (cudaStream_t)stream>>>(*g, d, n_boxes, status);
  HIER_CHECK_CUDA(cudaGetLastError(), "cached_pack_count_kernel launch");
  return HIER_OK;
}

extern "C" int hier_cached_pack_build(const hier_cached_grouping* g, const int32_t* n_boxes,
                                      int32_t tile_base, int32_t tile_end, int32_t mask_base,
                                      int32_t q2_row0, int32_t* q_pairs, int32_t* kv_tiles,
                                      uint32_t* tile_masks, int32_t* order, int32_t* status,
                                      void* stream) {
  clear_error();
  CDims d;
  int rc = make_dims(g, 1, &d);
  if (rc) return rc;
  const int np = pack_count(d);
  if (np == 0) return HIER_OK;
  if (!q_pairs || !kv_tiles || !tile_masks || tile_base < 0 || tile_end < tile_base ||
      mask_base < 0 || q2_row0 < 0) {
    set_error(HIER_EVALUE, "hier_cached_pack_build: invalid outputs or offsets");
    return HIER_EVALUE;
  }
  PackOut o;
  o.n_boxes = n_boxes;
  o.tile_base = tile_base;
  o.tile_end = tile_end;
  o.mask_base = mask_base;
  o.q2_row0 = q2_row0;
  o.pair_base = d.nA * d.npA;
  o.q_pairs = q_pairs;
  o.kv_tiles = kv_tiles;
  o.tile_masks = tile_masks;
  o.status = status;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t sm = seg_smem_bytes(d.C);
  HIER_CHECK_CUDA(cudaFuncSetAttribute(cached_pack_build_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm),
                  "cudaFuncSetAttribute(cached_pack_build_kernel)");
  cached_pack_build_kernel<<<np, kThreads, sm, s>>>(*g, d, o);
  HIER_CHECK_CUDA(cudaGetLastError(), "cached_pack_build_kernel launch");
  const int total = o.pair_base + np;
  if (order) {
    order_by_work_kernel<8><<<(total + 127) / 128, 128, 0, s>>>(q_pairs, total, order);
    HIER_CHECK_CUDA(cudaGetLastError(), "order_by_work_kernel launch");
  }
  return HIER_OK;
}
