// Attention plan of one shard (a rank holding the rows of some players and
// computing some 256-row strips of them), and, with a single shard, of the
// whole full-sequence layer.
//
// Query rows of the shard (a row space over two query tensors):
//   [0, own_rows)               the rows of its local players, in slot order
//                               (slot, frame, patch);
//   [own_rows, V)               every hub row, group-major: local hub (g, f, slot)
//                               at own_rows + (g*T + f)*K_L + slot, then global
//                               hub (f, slot) at own_rows + T*N*K_L + f*K_G + slot;
//   [V + o, V + o + n_hp*T*K_L) per hub-partial player p (those the shard
//                               computes hub partials for) and frame t the K_L
//                               local-hub rows of p's group at t (second query
//                               tensor; V = own_rows + hub_rows, o =
//                               hub_partial_row0, the shard's slot in a buffer
//                               shared by the ranks).
// Key/value streams: 0 = the shard's player rows, 1 = the hub rows (same
// order as above), and for a remote group-mate unit (o, f) the
// stream-packed first row remote_key[o*T + f].
//
// A hub row's attention is split by key set into partial rows merged from
// their log-sum-exp: per member player p of its group, the row of the third
// block over p's frames (on the rank that owns p), and over the hub tokens
// the row of the second block (on the rank with hub_keys).  Each partial
// then needs exactly one player's history, which keeps its tiles dense when
// groups change from frame to frame.
//
// Query pairs are two consecutive 128-row tiles of one query block:
//   * the shard's strips of a local player's T*L rows (256 rows each);
//   * a player's T*K_L hub-partial rows, cut into 256-row strips;
//   * one group's T*K_L local-hub rows, or the T*K_G global-hub rows (hub
//     keys only; on the hub_keys rank).
// Per pair one CTA enumerates the key units any of its rows may attend to,
// keeps those with an edge from some row, merges consecutive rows of a
// stream into runs, covers the runs with 64-row key boxes (two per 128-key
// tile) and evaluates, per tile and query row, the 128-bit key mask from the
// unit-level edges of the hierarchical mask (labels grouping):
//   player p, frame t -> own frame f:      temporal(t, f)
//                     -> player o, frame f: direct, same block, same group at t
//                     -> local hub (g, f):  temporal, active(f, g), g = group of p at t
//   local hub (g, t)  -> player (o, f):     temporal, o in g at t      (g active at t)
//                     -> local hub (g, f):  temporal, active(f, g)
//                     -> global f:          temporal
//                     (an inactive local hub attends to itself only)
//   global t          -> local hub (g, f):  temporal, active(f, g)
//                     -> global f:          temporal
// (multics/models/hier_masks.py:364-507, the edge sets of the dense mask).
// A tile is full for a half when every row of the half sees every key, is
// skipped by a half whose rows see none of its keys, and otherwise carries a
// 128-row mask for that half.  A first pass counts key tiles and masks per
// pair (the caller sizes the tables from the totals); the second writes the
// plan.  Pairs of hub rows are flagged in q_pairs[7] (partial rows).

#include <limits.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "seg_plan.cuh"

namespace hier {
namespace {

using segplan::kThreads;
using segplan::SegSmem;
using segplan::block_scan;

constexpr int kMaxCand = 2048;
constexpr int kMaxPages = 32768;     // pages of the paged stream (bitmap bits)
constexpr int kMaxPairPages = 2048;  // pages one pair's keys may touch
constexpr int kPageRows = 64;
constexpr int kStatusPageOverflow = 32;
constexpr int kStripRows = 256;
constexpr int kStatusTileOverflow = 2;
constexpr int kStatusMissingRemote = 8;
constexpr int kStatusMaskOverflow = 16;
constexpr int kSelSkip = -2;

struct SDims {
  int P, T, L, N, KL, KG, nb, win, direct;
  int n_local, hub_keys;
  int player[HIER_SHARD_MAX_LOCAL];     // local player slot -> absolute player
  int strip0[HIER_SHARD_MAX_LOCAL];     // this shard's strips of that player
  int strip_pre[HIER_SHARD_MAX_LOCAL + 1];  // exclusive prefix of the strip counts
  int hp_player[HIER_SHARD_MAX_LOCAL];  // hub-partial player k -> local slot
  int n_hp_players, n_strips;
  int hp_row0;         // offset of this shard's hub-partial rows in the partial-row space
  int nps;             // 256-row strips of one player's rows
  int nph;             // hub-partial strips per hub-partial player
  int npl, npg;        // hub-key pairs per group, global hub-key pairs (hub_keys rank)
  int n_hh;            // hub-key pairs of this shard
  int hh0;             // its first hub-key pair (in the order of all hub-key pairs)
  int n_pairs;         // all pairs: player strips, hub-partial strips, hub-key pairs
  int nf_mate;         // mate frames enumerated per player strip
  int c_player, c_hub; // candidates per player strip / hub-key pair
  int own_rows, hub_rows;
  const int* page_table;  // stream 0 paged (NULL: in place)
  int n_pages;
};

__device__ __forceinline__ int fdiv(int a, int b) {
  int q = a / b;
  return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ bool temporal(const SDims& d, int qf, int kf) {
  if (fdiv(kf, d.nb) > fdiv(qf, d.nb)) return false;
  return d.win == -1 || (qf - kf) < d.win;
}

// Unit codes (stored per candidate): kind << 24 | id << 12 | frame.
constexpr int kUnitPlayer = 0, kUnitLocal = 1, kUnitGlobal = 2;
__device__ __forceinline__ int unit_code(int kind, int id, int f) {
  return (kind << 24) | (id << 12) | f;
}

constexpr int kPairPlayer = 0, kPairLocal = 1, kPairGlobal = 2, kPairHubOfPlayer = 3;

struct Pair {
  int kind;    // kPair*: player strip, local / global hub-key pair, hub-partial strip
  int id;      // player (absolute) or group
  int j0;      // first row within the block of rows (player / group / global)
  int n0, n1;  // rows of the two halves
  int q0;      // first row of the shard
  int unit;    // rows per query unit: L, K_L or K_G
  int f_lo, f_hi;
  int mf0, nfr;  // strips: first frame and number of frames of mate candidates
};

__device__ Pair pair_of(const SDims& d, int i) {
  Pair r;
  int rows;
  const int n_hp = d.n_hp_players * d.nph;
  if (i < d.n_strips) {
    int slot = 0;
    while (slot + 1 < d.n_local && d.strip_pre[slot + 1] <= i) ++slot;
    r.kind = kPairPlayer;
    r.id = d.player[slot];
    r.j0 = kStripRows * (d.strip0[slot] + i - d.strip_pre[slot]);
    rows = d.T * d.L;
    r.unit = d.L;
    r.q0 = slot * rows + r.j0;
  } else if ((i -= d.n_strips) < n_hp) {
    const int k = i / d.nph;
    r.kind = kPairHubOfPlayer;
    r.id = d.player[d.hp_player[k]];
    r.j0 = kStripRows * (i % d.nph);
    rows = d.T * d.KL;
    r.unit = d.KL;
    r.q0 = d.own_rows + d.hub_rows + d.hp_row0 + k * rows + r.j0;
  } else if ((i = i - n_hp + d.hh0) < d.N * d.npl) {
    const int h = i;
    r.kind = kPairLocal;
    r.id = h / d.npl;
    r.j0 = kStripRows * (h % d.npl);
    rows = d.T * d.KL;
    r.unit = d.KL;
    r.q0 = d.own_rows + r.id * rows + r.j0;
  } else {
    const int h = i - d.N * d.npl;
    r.kind = kPairGlobal;
    r.id = 0;
    r.j0 = kStripRows * h;
    rows = d.T * d.KG;
    r.unit = d.KG;
    r.q0 = d.own_rows + d.T * d.N * d.KL + r.j0;
  }
  r.n0 = min(128, rows - r.j0);
  r.n1 = max(0, min(128, rows - r.j0 - 128));
  r.f_lo = r.j0 / r.unit;
  r.f_hi = (r.j0 + r.n0 + r.n1 - 1) / r.unit;
  r.mf0 = fdiv(r.f_lo, d.nb) * d.nb;
  r.nfr = min(d.T, (fdiv(r.f_hi, d.nb) + 1) * d.nb) - r.mf0;
  return r;
}

__device__ __forceinline__ int label(const hier_shard_desc& g, int t, int p) {
  return (int)g.labels[(int64_t)t * g.P + p];
}
__device__ __forceinline__ bool active(const hier_shard_desc& g, int t, int gi) {
  return g.active[(int64_t)t * g.N + gi] != 0;
}

// Unit-level edge from a query row (pair kind, id, frame t) to key unit u.
__device__ bool edge(const hier_shard_desc& g, const SDims& d, int qkind, int qid, int t,
                     int u) {
  const int kind = u >> 24, id = (u >> 12) & 0xfff, f = u & 0xfff;
  if (qkind == kPairHubOfPlayer)  // local hub of qid's group at t -> qid's frames
    return kind == kUnitPlayer && id == qid && temporal(d, t, f) &&
           active(g, t, label(g, t, qid));
  if (qkind == kPairPlayer) {
    if (kind == kUnitPlayer) {
      if (id == qid) return temporal(d, t, f);
      return d.direct && fdiv(f, d.nb) == fdiv(t, d.nb) && label(g, t, id) == label(g, t, qid);
    }
    if (kind == kUnitLocal) return temporal(d, t, f) && active(g, f, id) && label(g, t, qid) == id;
    return false;
  }
  if (qkind == kPairLocal) {
    if (!active(g, t, qid)) return false;
    if (kind == kUnitPlayer) return temporal(d, t, f) && label(g, t, id) == qid;
    if (kind == kUnitLocal) return temporal(d, t, f) && id == qid && active(g, f, qid);
    return temporal(d, t, f);
  }
  if (kind == kUnitPlayer) return false;
  if (kind == kUnitLocal) return temporal(d, t, f) && active(g, f, id);
  return temporal(d, t, f);
}

// Local row slot of player o (-1: not held by this shard).
__device__ __forceinline__ int local_slot(const SDims& d, int o) {
  for (int i = 0; i < d.n_local; ++i)
    if (d.player[i] == o) return i;
  return -1;
}

// Candidate c of a pair: unit code, stream-packed first key row and width
// (0 for an unused slot).  *remote marks a remote mate frame, whose key is
// remote_key[o*T + f] (-1 when the shard has no slot for it).
__device__ void candidate(const hier_shard_desc& g, const SDims& d, const Pair& pr, int c,
                          int* code, int* key, int* width, bool* remote) {
  *remote = false;
  const int s1 = 1 << segplan::kStreamShift;
  auto player_key = [&](int o, int f) {
    return local_slot(d, o) * d.T * d.L + f * d.L;
  };
  if (pr.kind == kPairHubOfPlayer) {  // the player's frames
    *code = unit_code(kUnitPlayer, pr.id, c);
    *key = player_key(pr.id, c);
    *width = d.L;
    return;
  }
  if (pr.kind == kPairPlayer) {
    if (c < d.T) {  // own frames
      *code = unit_code(kUnitPlayer, pr.id, c);
      *key = player_key(pr.id, c);
      *width = d.L;
      return;
    }
    c -= d.T;
    if (c < (d.P - 1) * d.nf_mate) {  // group-mate frames of the rows' blocks
      const int oi = c / d.nf_mate, k = c % d.nf_mate;
      const int o = oi < pr.id ? oi : oi + 1;
      const int f = pr.mf0 + k;
      if (k >= pr.nfr || f >= d.T) {
        *code = unit_code(kUnitPlayer, o, 0);
        *key = 0;
        *width = 0;
        return;
      }
      *code = unit_code(kUnitPlayer, o, f);
      *width = d.L;
      if (local_slot(d, o) >= 0) {
        *key = player_key(o, f);
      } else {
        *key = g.remote_key[o * d.T + f];
        *remote = true;
      }
      return;
    }
    c -= (d.P - 1) * d.nf_mate;
    const int gi = c / d.T, f = c % d.T;  // local hubs, group-major
    *code = unit_code(kUnitLocal, gi, f);
    *key = s1 | ((gi * d.T + f) * d.KL);
    *width = d.KL;
    return;
  }
  if (c < d.T * d.N) {  // hub-key pairs: hub units only
    const int gi = c / d.T, f = c % d.T;
    *code = unit_code(kUnitLocal, gi, f);
    *key = s1 | ((gi * d.T + f) * d.KL);
    *width = d.KL;
    return;
  }
  const int f = c - d.T * d.N;
  *code = unit_code(kUnitGlobal, 0, f);
  *key = s1 | (d.T * d.N * d.KL + f * d.KG);
  *width = d.KG;
}

// Does some row of the pair attend to unit u (the inactive-local self edge
// included)?
__device__ bool pair_sees(const hier_shard_desc& g, const SDims& d, const Pair& pr, int u) {
  for (int t = pr.f_lo; t <= pr.f_hi; ++t) {
    if (edge(g, d, pr.kind, pr.id, t, u)) return true;
    if (pr.kind == kPairLocal && !active(g, t, pr.id) && u == unit_code(kUnitLocal, pr.id, t))
      return true;
  }
  return false;
}

// Page bitmap and page list of the paged stream, after the run analysis.
__device__ __forceinline__ uint32_t* page_bitmap(int* smem_i) {
  return reinterpret_cast<uint32_t*>(smem_i + segplan::seg_smem_ints(kMaxCand));
}
__device__ __forceinline__ int* page_list(int* smem_i) {
  return smem_i + segplan::seg_smem_ints(kMaxCand) + kMaxPages / 32;
}

// Paged stream 0: the boxes become the distinct pages the stream-0 runs
// touch (ascending), numbered first; the other runs' boxes follow in run
// order (m.rb recomputed, zero boxes for stream-0 runs).  m.misc[7] = pages.
__device__ void page_boxes(const SDims& d, const SegSmem& m, int* smem_i, int* status) {
  uint32_t* bm = page_bitmap(smem_i);
  int* pl = page_list(smem_i);
  const int words = (d.n_pages + 31) / 32;
  for (int i = threadIdx.x; i < words; i += kThreads) bm[i] = 0u;
  __syncthreads();
  const int n_runs = m.misc[1];
  for (int r = threadIdx.x; r < n_runs; r += kThreads) {
    const int k = m.rk[r];
    if ((k >> segplan::kStreamShift) != 0) continue;
    const int row = k & ((1 << segplan::kStreamShift) - 1);
    const int len = m.rf[r + 1] - m.rf[r];
    for (int p = row / kPageRows; p <= (row + len - 1) / kPageRows; ++p)
      atomicOr(bm + p / 32, 1u << (p % 32));
  }
  __syncthreads();
  int* wtmp = m.misc + 8;
  int carry = 0;
  for (int base = 0; base < words; base += kThreads) {
    const int i = base + threadIdx.x;
    const uint32_t w = i < words ? bm[i] : 0u;
    const int incl = block_scan<false>(__popc(w), wtmp) + carry;
    int pos = incl - __popc(w);
    for (uint32_t x = w; x; x &= x - 1, ++pos)
      if (pos < kMaxPairPages) pl[pos] = 32 * i + __ffs(x) - 1;
    if (threadIdx.x == kThreads - 1) m.misc[21] = incl;
    __syncthreads();
    carry = m.misc[21];
    __syncthreads();
  }
  int n_paged = carry;
  if (n_paged > kMaxPairPages) {
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusPageOverflow);
    n_paged = kMaxPairPages;
  }
  // boxes of the other streams' runs, after the pages
  int cb = 0;
  for (int base = 0; base < n_runs; base += kThreads) {
    const int r = base + threadIdx.x;
    int nbx = 0;
    if (r < n_runs && (m.rk[r] >> segplan::kStreamShift) != 0)
      nbx = (m.rf[r + 1] - m.rf[r] + segplan::kBoxRows - 1) / segplan::kBoxRows;
    const int incl = block_scan<false>(nbx, wtmp) + cb;
    if (r < n_runs) m.rb[r] = n_paged + incl - nbx;
    if (threadIdx.x == kThreads - 1) m.misc[21] = incl;
    __syncthreads();
    cb = m.misc[21];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    m.rb[n_runs] = n_paged + cb;
    m.misc[2] = n_paged + cb;
    m.misc[7] = n_paged;
  }
  __syncthreads();
}

// 64 mask bits of one query row (frame t) over page `page` of the paged
// stream: each key row's bit is the unit-level edge to its own unit.
__device__ uint64_t page_bits(const hier_shard_desc& g, const SDims& d, const Pair& pr, int t,
                              int page) {
  const int TL = d.T * d.L;
  const int r0 = page * kPageRows, end = min(r0 + kPageRows, d.own_rows);
  uint64_t bits = 0;
  for (int r = r0; r < end;) {
    const int slot = r / TL, f = (r % TL) / d.L;
    const int e = min(end, slot * TL + (f + 1) * d.L);
    if (edge(g, d, pr.kind, pr.id, t, unit_code(kUnitPlayer, d.player[slot], f))) {
      const int a = r - r0, b = e - r0;
      const uint64_t hi = b >= 64 ? ~0ull : ((1ull << b) - 1ull);
      bits |= hi & ~((1ull << a) - 1ull);
    }
    r = e;
  }
  return bits;
}

// Candidates, runs and boxes of pair pr (all threads); m.pool holds unit
// codes, m.dw / m.doff the attended candidates and their key offsets.
__device__ void analyse_pair(const hier_shard_desc& g, const SDims& d, const Pair& pr,
                             const SegSmem& m, int* smem_i, int* status) {
  const int C = pr.kind == kPairPlayer ? d.c_player : pr.kind == kPairHubOfPlayer ? d.T : d.c_hub;
  int missing = 0;
  for (int c = threadIdx.x; c < C; c += kThreads) {
    int code, key, width;
    bool remote;
    candidate(g, d, pr, c, &code, &key, &width, &remote);
    bool seen = width > 0 && pair_sees(g, d, pr, code);
    if (seen && remote && key < 0) {
      missing = 1;
      seen = false;
    }
    m.w[c] = seen ? width : 0;
    m.key[c] = seen ? key : 0;
    m.pool[c] = code;
  }
  if (missing && status) atomicOr(status, kStatusMissingRemote);
  __syncthreads();
  segplan::analyse_runs(m, C);
  if (threadIdx.x == 0) m.misc[7] = 0;
  __syncthreads();
  if (d.page_table) page_boxes(d, m, smem_i, status);
  // compact list of attended candidates with their key offsets
  int* wtmp = m.misc + 8;
  int carry = 0;
  for (int base = 0; base < C; base += kThreads) {
    const int c = base + threadIdx.x;
    const int f = (c < C && m.w[c] > 0) ? 1 : 0;
    const int incl = block_scan<false>(f, wtmp) + carry;
    if (f) {
      m.dw[incl - 1] = c;
      m.doff[incl - 1] = m.off[c];
    }
    if (threadIdx.x == kThreads - 1) m.misc[20] = incl;
    __syncthreads();
    carry = m.misc[20];
    __syncthreads();
  }
  if (threadIdx.x == 0) m.misc[6] = carry;
  __syncthreads();
}

// 64 mask bits of one query row (frame t, slot within its unit) over the
// box of `valid` keys starting at key offset k0 of the pair's key list.
__device__ uint64_t box_bits(const hier_shard_desc& g, const SDims& d, const Pair& pr,
                             const SegSmem& m, int t, int slot, int k0, int valid) {
  const int n_att = m.misc[6];
  int lo = 0, hi = n_att - 1;  // last attended candidate starting at or before k0
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (m.doff[mid] <= k0) lo = mid;
    else hi = mid - 1;
  }
  const bool self_only = pr.kind == kPairLocal && !active(g, t, pr.id);
  uint64_t bits = 0;
  int pos = 0;
  for (int a = lo; pos < valid && a < n_att; ++a) {
    const int c = m.dw[a];
    const int end = min(valid, m.doff[a] + m.w[c] - k0);
    if (end <= pos) continue;
    const int u = m.pool[c];
    if (!self_only) {
      if (edge(g, d, pr.kind, pr.id, t, u)) {
        const uint64_t hi_bits = end >= 64 ? ~0ull : ((1ull << end) - 1ull);
        bits |= hi_bits & ~((1ull << pos) - 1ull);
      }
    } else if (u == unit_code(kUnitLocal, pr.id, t)) {
      const int self = m.doff[a] + slot - k0;  // the row's own token
      if (self >= pos && self < end) bits |= 1ull << self;
    }
    pos = end;
  }
  return bits;
}

// Walks the pair's key tiles with one thread per (half, row): per tile the
// selector of each half and, for a masked half, the row's 128-bit mask.
// kWrite = false only counts the masked halves.
template <bool kWrite>
__device__ int emit_tiles(const hier_shard_desc& g, const SDims& d, const Pair& pr,
                          const SegSmem& m, int* smem_i, int tile_base, int mask_base,
                          int32_t* kv_tiles, uint32_t* tile_masks) {
  const int n_runs = m.misc[1], n_box = m.misc[2], n_tiles = (n_box + 1) >> 1;
  const int n_paged = m.misc[7];
  const int* pl = page_list(smem_i);
  const int h = threadIdx.x >> 7, r = threadIdx.x & 127;
  const int nrow = h ? pr.n1 : pr.n0;
  const bool row_ok = r < nrow;
  const int j = pr.j0 + 128 * h + r;
  const int t = row_ok ? j / pr.unit : 0, slot = row_ok ? j % pr.unit : 0;
  int n_mask = 0;
  for (int i = 0; i < n_tiles; ++i) {
    int key[2], k0[2], valid[2], page[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int b = 2 * i + s;
      const int bb = b < n_box ? b : b - 1;  // odd count: the last tile repeats a box, masked
      page[s] = -1;
      if (bb < n_paged) {  // one physical page of the paged stream
        page[s] = pl[bb];
        key[s] = d.page_table[page[s]] * kPageRows;
        k0[s] = 0;
        valid[s] = b < n_box ? kPageRows : 0;
      } else {
        const int ru = segplan::run_of_box(m, n_runs, bb);
        const int k = bb - m.rb[ru];
        key[s] = m.rk[ru] + segplan::kBoxRows * k;
        k0[s] = m.rf[ru] + segplan::kBoxRows * k;
        valid[s] = b < n_box ? min(segplan::kBoxRows, m.rf[ru + 1] - k0[s]) : 0;
      }
    }
    uint64_t bits[2] = {0ull, 0ull};
    if (row_ok) {
#pragma unroll
      for (int s = 0; s < 2; ++s)
        bits[s] = page[s] >= 0 ? (valid[s] ? page_bits(g, d, pr, t, page[s]) : 0ull)
                               : box_bits(g, d, pr, m, t, slot, k0[s], valid[s]);
    }
    const bool all = (bits[0] & bits[1]) == ~0ull;
    const bool some = (bits[0] | bits[1]) != 0ull;
    const int full0 = __syncthreads_and(h == 1 || !row_ok || all);
    const int full1 = __syncthreads_and(h == 0 || !row_ok || all);
    const int any0 = __syncthreads_or(h == 0 && row_ok && some);
    const int any1 = __syncthreads_or(h == 1 && row_ok && some);
    const bool masked0 = any0 && !full0, masked1 = any1 && !full1;
    const int mi = mask_base + n_mask + (h ? (masked0 ? 1 : 0) : 0);
    const bool masked_h = h ? masked1 : masked0;
    if (kWrite) {
      const int sel = !(h ? any1 : any0) ? kSelSkip : masked_h ? mi : -1;
      const int64_t ti = tile_base + i;
      if (r == 0) {
        if (h == 0) {
          kv_tiles[ti * 4 + 0] = key[0];
          kv_tiles[ti * 4 + 1] = key[1];
        }
        kv_tiles[ti * 4 + 2 + h] = sel;
      }
      if (masked_h) {
        uint32_t* dst = tile_masks + ((int64_t)mi * 128 + r) * 4;
        dst[0] = (uint32_t)bits[0];
        dst[1] = (uint32_t)(bits[0] >> 32);
        dst[2] = (uint32_t)bits[1];
        dst[3] = (uint32_t)(bits[1] >> 32);
      }
    }
    n_mask += (masked0 ? 1 : 0) + (masked1 ? 1 : 0);
  }
  return n_mask;
}

size_t plan_smem_bytes() {
  return (segplan::seg_smem_ints(kMaxCand) + kMaxPages / 32 + kMaxPairPages + 32) * sizeof(int);
}


__global__ void __launch_bounds__(kThreads)
    pair_count_kernel(const hier_shard_desc g, const SDims d, int32_t* counts, int32_t* totals,
                      int32_t* status) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, kMaxCand);
  const Pair pr = pair_of(d, blockIdx.x);
  analyse_pair(g, d, pr, m, smem_i, status);
  const int n_mask = emit_tiles<false>(g, d, pr, m, smem_i, 0, 0, nullptr, nullptr);
  if (threadIdx.x == 0) {
    const int n_tiles = (m.misc[2] + 1) >> 1;
    counts[2 * blockIdx.x] = n_tiles;
    counts[2 * blockIdx.x + 1] = n_mask;
    atomicAdd(totals, n_tiles);
    atomicAdd(totals + 1, n_mask);
  }
}

__global__ void __launch_bounds__(kThreads)
    pair_build_kernel(const hier_shard_desc g, const SDims d, const int32_t* counts,
                      int32_t* q_pairs, int32_t* kv_tiles, int32_t tile_capacity,
                      uint32_t* tile_masks, int64_t mask_capacity, int32_t* status) {
  extern __shared__ int smem_i[];
  const SegSmem m = segplan::seg_smem(smem_i, kMaxCand);
  const int pi = blockIdx.x;
  const Pair pr = pair_of(d, pi);
  // tile and mask bases: exclusive sums over the earlier pairs
  int tb = 0, mb = 0;
  for (int i = threadIdx.x; i < pi; i += kThreads) {
    tb += counts[2 * i];
    mb += counts[2 * i + 1];
  }
  tb = block_scan<false>(tb, m.misc + 8);
  __shared__ int bases[2];
  if (threadIdx.x == kThreads - 1) bases[0] = tb;
  __syncthreads();
  mb = block_scan<false>(mb, m.misc + 8);
  if (threadIdx.x == kThreads - 1) bases[1] = mb;
  __syncthreads();
  const int tile_base = bases[0], mask_base = bases[1];
  analyse_pair(g, d, pr, m, smem_i, nullptr);
  const int n_tiles = (m.misc[2] + 1) >> 1;
  if (n_tiles != counts[2 * pi] || tile_base + n_tiles > tile_capacity ||
      (int64_t)mask_base + counts[2 * pi + 1] > mask_capacity) {
    if (threadIdx.x == 0) {
      if (status)
        atomicOr(status, tile_base + n_tiles > tile_capacity ? kStatusTileOverflow
                                                             : kStatusMaskOverflow);
      // still a well-formed record: an empty pair, so that ordering and an
      // attention launch over this plan read no key tile outside the table
      int32_t* rec = q_pairs + (int64_t)pi * 8;
      rec[0] = pr.q0;
      rec[1] = pr.n0;
      rec[2] = pr.q0 + 128;
      rec[3] = pr.n1;
      rec[4] = 0;
      rec[5] = 0;
      rec[6] = 1;
      rec[7] = pr.kind == kPairPlayer ? 0 : 1;
    }
    return;
  }
  emit_tiles<true>(g, d, pr, m, smem_i, tile_base, mask_base, kv_tiles, tile_masks);
  if (threadIdx.x == 0) {
    int32_t* rec = q_pairs + (int64_t)pi * 8;
    rec[0] = pr.q0;
    rec[1] = pr.n0;
    rec[2] = pr.q0 + 128;
    rec[3] = pr.n1;
    rec[4] = tile_base;
    rec[5] = tile_base + n_tiles;
    rec[6] = 1;                                // 128-row masks
    rec[7] = pr.kind == kPairPlayer ? 0 : 1;  // hub rows: partial rows
  }
}

int make_sdims(const hier_shard_desc* g, SDims* d) {
  if (!g) {
    set_error(HIER_EVALUE, "hier_shard_desc is NULL");
    return HIER_EVALUE;
  }
  memset(d, 0, sizeof(*d));
  d->P = g->P, d->T = g->T, d->L = g->L, d->N = g->N, d->KL = g->KL, d->KG = g->KG;
  d->nb = g->n_block, d->win = g->local_attn, d->direct = g->direct != 0;
  if (d->P <= 0 || d->T <= 0 || d->L <= 0 || d->N <= 0 || d->KL < 0 || d->KG < 0 ||
      d->nb <= 0 || !g->labels || !g->active) {
    set_error(HIER_EVALUE, "invalid shard dims P=%d T=%d L=%d N=%d K_L=%d K_G=%d n=%d", d->P,
              d->T, d->L, d->N, d->KL, d->KG, d->nb);
    return HIER_EVALUE;
  }
  if (d->win != -1 && d->win <= 0) {
    set_error(HIER_EVALUE, "local_attn must be -1 or positive, got %d", d->win);
    return HIER_EVALUE;
  }
  if (d->P > 4095 || d->N > 4095 || d->T > 4095) {
    set_error(HIER_EVALUE, "shard plan supports at most 4095 players, groups and frames");
    return HIER_EVALUE;
  }
  if (g->n_local <= 0 || g->n_local > HIER_SHARD_MAX_LOCAL) {
    set_error(HIER_EVALUE, "a shard holds 1..%d players; got %d", HIER_SHARD_MAX_LOCAL,
              g->n_local);
    return HIER_EVALUE;
  }
  if (d->direct && !g->remote_key) {
    set_error(HIER_EVALUE, "direct player edges need the remote unit table");
    return HIER_EVALUE;
  }
  d->n_local = g->n_local, d->hub_keys = g->hub_keys != 0;
  const int nps_all = (int)(((int64_t)d->T * d->L + kStripRows - 1) / kStripRows);
  d->strip_pre[0] = 0;
  for (int i = 0; i < d->n_local; ++i) {
    const int o = g->local_player[i];
    if (o < 0 || o >= d->P) {
      set_error(HIER_EVALUE, "local player %d out of range [0, %d)", o, d->P);
      return HIER_EVALUE;
    }
    for (int j = 0; j < i; ++j)
      if (g->local_player[j] == o) {
        set_error(HIER_EVALUE, "player %d listed twice in a shard", o);
        return HIER_EVALUE;
      }
    const int b = g->strip_begin[i], e = g->strip_end[i];
    if (b < 0 || e < b || e > nps_all) {
      set_error(HIER_EVALUE, "strips [%d, %d) of player %d outside [0, %d)", b, e, o, nps_all);
      return HIER_EVALUE;
    }
    d->player[i] = o;
    d->strip0[i] = b;
    d->strip_pre[i + 1] = d->strip_pre[i] + (e - b);
    if (g->hub_partials[i]) d->hp_player[d->n_hp_players++] = i;
  }
  d->n_strips = d->strip_pre[d->n_local];
  if (g->hub_partial_row0 < 0) {
    set_error(HIER_EVALUE, "negative hub-partial row offset %d", g->hub_partial_row0);
    return HIER_EVALUE;
  }
  d->hp_row0 = g->hub_partial_row0;
  const int64_t own_rows = (int64_t)d->n_local * d->T * d->L;
  const int64_t hub_rows = (int64_t)d->T * (d->N * d->KL + d->KG);
  if (own_rows >= (1 << segplan::kStreamShift) || hub_rows >= (1 << segplan::kStreamShift)) {
    set_error(HIER_EVALUE, "shard of %lld player rows / %lld hub rows exceeds %d",
              (long long)own_rows, (long long)hub_rows, (1 << segplan::kStreamShift) - 1);
    return HIER_EVALUE;
  }
  d->own_rows = (int)own_rows;
  d->hub_rows = (int)hub_rows;
  d->page_table = g->page_table;
  d->n_pages = g->page_table ? g->n_pages : 0;
  if (g->page_table) {
    if (g->n_local != g->P) {
      set_error(HIER_EVALUE, "paged player rows need a single shard holding all %d players", g->P);
      return HIER_EVALUE;
    }
    if ((int64_t)g->n_pages * kPageRows < own_rows || g->n_pages > kMaxPages) {
      set_error(HIER_EVALUE, "page table of %d pages for %lld player rows (at most %d pages)",
                g->n_pages, (long long)own_rows, kMaxPages);
      return HIER_EVALUE;
    }
  }
  auto cdiv = [](int64_t a, int64_t b) { return (int)((a + b - 1) / b); };
  d->nps = cdiv((int64_t)d->T * d->L, kStripRows);
  d->nph = d->KL > 0 ? cdiv((int64_t)d->T * d->KL, kStripRows) : 0;
  d->npl = d->KL > 0 ? cdiv((int64_t)d->T * d->KL, kStripRows) : 0;
  d->npg = d->KG > 0 ? cdiv((int64_t)d->T * d->KG, kStripRows) : 0;
  {
    const int all = d->N * d->npl + d->npg;
    const int first = g->hub_key_count > 0 ? std::min(std::max(g->hub_key_first, 0), all) : 0;
    const int cnt = g->hub_key_count > 0 ? std::min(g->hub_key_count, all - first) : all;
    d->hh0 = d->hub_keys ? first : 0;
    d->n_hh = d->hub_keys ? cnt : 0;
  }
  d->n_pairs = d->n_strips + d->n_hp_players * d->nph + d->n_hh;
  if ((int64_t)own_rows + hub_rows + d->hp_row0 + (int64_t)d->n_hp_players * d->T * d->KL >
      INT_MAX / 2) {
    set_error(HIER_EVALUE, "shard query rows exceed the row range");
    return HIER_EVALUE;
  }
  // mate frames of the blocks a strip's rows touch (the same for every player)
  int nf = 0;
  for (int i = 0; i < d->nps; ++i) {
    const int j0 = kStripRows * i, rows = (int)std::min<int64_t>(kStripRows, (int64_t)d->T * d->L - j0);
    const int f_lo = j0 / d->L, f_hi = (j0 + rows - 1) / d->L;
    const int bs = (f_lo / d->nb) * d->nb, be = std::min(d->T, (f_hi / d->nb + 1) * d->nb);
    nf = std::max(nf, be - bs);
  }
  d->nf_mate = d->direct ? nf : 0;
  d->c_player = d->T + (d->P - 1) * d->nf_mate + d->T * d->N;
  d->c_hub = d->T * d->N + d->T;
  if (d->c_player > kMaxCand || d->c_hub > kMaxCand) {
    set_error(HIER_EVALUE, "shard too large for the plan builder (%d / %d key units per pair)",
              d->c_player, d->c_hub);
    return HIER_EVALUE;
  }
  return HIER_OK;
}

int set_smem(const void* k) {
  HIER_CHECK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)plan_smem_bytes()),
                  "cudaFuncSetAttribute(shard plan kernels)");
  return HIER_OK;
}

}  // namespace
}  // namespace hier

using namespace hier;

extern "C" int hier_shard_sizes(const hier_shard_desc* g, hier_shard_sizes_t* out) {
  clear_error();
  if (!out) {
    set_error(HIER_EVALUE, "sizes output is NULL");
    return HIER_EVALUE;
  }
  SDims d;
  int rc = make_sdims(g, &d);
  if (rc) return rc;
  memset(out, 0, sizeof(*out));
  out->n_pairs = d.n_pairs;
  out->n_player_pairs = d.n_strips;
  out->n_counts = 2 * d.n_pairs;
  out->own_rows = d.own_rows;
  out->hub_rows = d.hub_rows;
  out->hub_partial_rows = (int64_t)d.n_hp_players * d.T * d.KL;
  return HIER_OK;
}

extern "C" int hier_shard_count(const hier_shard_desc* g, int32_t* counts, int32_t* totals,
                                int32_t* status, void* stream) {
  clear_error();
  SDims d;
  int rc = make_sdims(g, &d);
  if (rc) return rc;
  if (!counts || !totals) {
    set_error(HIER_EVALUE, "shard count outputs missing");
    return HIER_EVALUE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  HIER_CHECK_CUDA(cudaMemsetAsync(totals, 0, 2 * sizeof(int32_t), s), "cudaMemsetAsync(totals)");
  if (d.n_pairs == 0) return HIER_OK;
  if ((rc = set_smem((const void*)pair_count_kernel))) return rc;
  pair_count_kernel<<<d.n_pairs, kThreads, plan_smem_bytes(), s>>>(*g, d, counts, totals, status);
  HIER_CHECK_CUDA(cudaGetLastError(), "pair_count_kernel launch");
  return HIER_OK;
}

extern "C" int hier_shard_build(const hier_shard_desc* g, const int32_t* counts,
                                int32_t* q_pairs, int32_t* kv_tiles, int32_t tile_capacity,
                                uint32_t* tile_masks, int64_t mask_capacity, int32_t* order,
                                int32_t* status, void* stream) {
  clear_error();
  SDims d;
  int rc = make_sdims(g, &d);
  if (rc) return rc;
  if (!counts || !q_pairs || !kv_tiles || !tile_masks) {
    set_error(HIER_EVALUE, "shard plan outputs missing");
    return HIER_EVALUE;
  }
  if (d.n_pairs == 0) return HIER_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if ((rc = set_smem((const void*)pair_build_kernel))) return rc;
  pair_build_kernel<<<d.n_pairs, kThreads, plan_smem_bytes(), s>>>(
      *g, d, counts, q_pairs, kv_tiles, tile_capacity, tile_masks, mask_capacity, status);
  HIER_CHECK_CUDA(cudaGetLastError(), "pair_build_kernel launch");
  if (order) {  // every pair by descending work: the long hub-partial strips start early
    order_by_work_kernel<8><<<(d.n_pairs + 127) / 128, 128, 0, s>>>(q_pairs, d.n_pairs, order);
    HIER_CHECK_CUDA(cudaGetLastError(), "order_by_work_kernel launch");
  }
  return HIER_OK;
}
