// Trie-constrained beam search kernels for sm_100a.
//
// A request is searched by one thread-block cluster ("team") of 1 to 16 CTAs
// that stays on the request for all its steps (persistent grid, requests
// strided over teams).  Team-wide counters and the merged radix histogram live
// in the shared memory of the team's rank-0 CTA and are updated with
// distributed-shared-memory atomics; the phases of a step are separated by
// hardware cluster barriers.  The reference launches one cooperative grid per
// request and separates each step's expansion, pruning and history save with
// 2-3 grid-wide syncs (lib/marisa/grimoire/trie/tbs-kernels.cu:476-594).
// Small batches use large teams (latency), large batches 1-CTA teams
// (throughput).
//
// Per step t of a request:
//   1. every CTA stages row t (ids ascending, log-probs, original columns;
//      sorted once by row_prep_kernel) in its shared memory;
//   2. expand:
//      - in-link beams, one thread each: the next tail cell is the only
//        allowed token; look it up in the sorted row (tbs-kernels.cu:324-371);
//      - branching beams: a task table of (parent, 128 items) drained by all
//        warps of the team; an item is a child whose label is looked up in the
//        row (small fan-out), or a proposal that probes the parent's hash
//        table (large fan-out) or binary-searches its child labels
//        (tbs-kernels.cu:210-322); found children ("hits") are resolved in one
//        bulk round that gathers their flags and link offsets;
//      - thresholds: logp > token_threshold and score + logp > sent_threshold,
//        compared in f64 (tbs-kernels.cu:229-231);
//      - children go to the step's candidate list and, when they end a key,
//        to the result pool;
//   3. select: exact top-beams[t] of the candidates in the pinned order
//      (logp_norm, node, depth, score), an 11-bit MSD radix select over the
//      192-bit key starting after the bits all candidates share; survivors
//      become the next step's beams and append (parent, token) history;
//   4. trim the result pool to the final beam the same way.
// After the last step the pool is sorted and written ascending with each
// sequence rebuilt from the history (tbs-kernels.cu:393-474).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include <cstdlib>

#include "cuda_util.hpp"
#include "tbs_kernel.cuh"

namespace cg = cooperative_groups;

namespace ftb {
namespace {

constexpr uint32_t kTailTerm = 0xFFFFFFFFu;
constexpr int kWarps = kSearchThreads / 32;
constexpr int kRadixBits = 11;
constexpr int kRadixBins = 1 << kRadixBits;
constexpr int kKeyBits = 192;
constexpr int kNodeFlagTerminal = 1;
constexpr int kNodeFlagLink = 2;
constexpr int kNodeFlagHashed = 4;     // plain nodes
constexpr int kNodeFlagLinkEnds1 = 4;  // link nodes

// ------------------------------------------------------------- keys
// Monotone map of an f64 to u64 (-0.0 folded onto +0.0).
__device__ __forceinline__ uint64_t orderable(double d) {
  uint64_t u = (uint64_t)__double_as_longlong(d);
  if ((u << 1) == 0) u = 0;
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

struct Key3 {
  uint64_t w[3];  // w[0] most significant
};

__device__ __forceinline__ Key3 cand_key(const Cand &c, double factor, uint32_t depth) {
  Key3 k;
  k.w[0] = orderable(c.score * factor);
  k.w[1] = ((uint64_t)c.node << 32) | ((uint64_t)(depth & 0xFFFFu) << 16);
  k.w[2] = orderable(c.score);
  return k;
}

__device__ __forceinline__ int key_cmp(const Key3 &a, const Key3 &b) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
  }
  return 0;
}

__device__ __forceinline__ uint64_t low_mask(int width) { return width >= 64 ? ~0ull : ((1ull << width) - 1); }

// `width` bits starting `from_top` bits below the most significant bit.
__device__ __forceinline__ uint32_t key_bits(const Key3 &k, int from_top, int width) {
  const int wi = from_top >> 6, o = from_top & 63;
  const int avail = 64 - o;
  if (width <= avail) return (uint32_t)((k.w[wi] >> (avail - width)) & low_mask(width));
  const int rest = width - avail;
  const uint64_t hi = k.w[wi] & low_mask(avail);
  const uint64_t lo = k.w[wi + 1] >> (64 - rest);
  return (uint32_t)((hi << rest) | lo);
}

__device__ __forceinline__ void key_set_bits(Key3 &k, int from_top, int width, uint64_t v) {
  const int wi = from_top >> 6, o = from_top & 63;
  const int avail = 64 - o;
  if (width <= avail) {
    const int sh = avail - width;
    k.w[wi] = (k.w[wi] & ~(low_mask(width) << sh)) | ((v & low_mask(width)) << sh);
    return;
  }
  const int rest = width - avail;
  k.w[wi] = (k.w[wi] & ~low_mask(avail)) | ((v >> rest) & low_mask(avail));
  const int sh = 64 - rest;
  k.w[wi + 1] = (k.w[wi + 1] & ~(low_mask(rest) << sh)) | ((v & low_mask(rest)) << sh);
}

// ------------------------------------------- loads of team-written data
// Candidates, hits, beams, pool entries and history are written by any CTA of
// the team and read by another after a cluster barrier; they are loaded
// through L2 (ld.global.cg) so that no SM can see a line it cached earlier.
__device__ __forceinline__ Cand ld_cand(const Cand *p) {
  Cand c;
  c.score = __ldcg(&p->score);
  const uint2 a = __ldcg(reinterpret_cast<const uint2 *>(&p->node));
  const uint2 b = __ldcg(reinterpret_cast<const uint2 *>(&p->parent));
  c.node = a.x;
  c.aux = a.y;
  c.parent = b.x;
  c.token = b.y;
  return c;
}

__device__ __forceinline__ Beam ld_beam(const Beam *p) {
  Beam b;
  b.score = __ldcg(&p->score);
  const uint2 a = __ldcg(reinterpret_cast<const uint2 *>(&p->node));
  b.node = a.x;
  b.off = a.y;
  return b;
}

__device__ __forceinline__ Hit ld_hit(const Hit *p) {
  const uint2 a = __ldcg(reinterpret_cast<const uint2 *>(p));
  return Hit{a.x, a.y};
}

__device__ __forceinline__ Hist ld_hist(const Hist *p) {
  const uint2 a = __ldcg(reinterpret_cast<const uint2 *>(p));
  return Hist{a.x, a.y};
}

// ---------------------------------------------------------- team state
// Authoritative in the team's rank-0 CTA; other CTAs reach it through
// distributed shared memory.
struct TeamState {
  uint32_t n_in, n_br;          // beams of the current step: in-link / branching
  uint32_t n_sel;               // beams written for the next step (capped at its width)
  uint32_t n_in_new, n_br_new;  // ... of which in-link / branching
  uint32_t n_next;              // candidates of this step
  uint32_t pool_n;              // pool entries kept from earlier steps
  uint32_t pool_end;            // pool entries after this step's appends
  uint32_t n_hits;              // lookup hits of this step
  uint32_t n_compact;           // pool compaction counter
  uint32_t eq_taken;
  uint32_t cur;                 // current beam buffer
  uint32_t pad0;
  uint64_t sel_pushes;          // pushes to the pool so far (early exit)
  uint32_t key_min;             // range of the top 32 bits of the candidates' first key word
  uint32_t key_max;
  Key3 sel_prefix;
  Key3 sel_mask;
  uint32_t sel_rem;
  int sel_ge;                   // 1: every key >= prefix is taken
  uint32_t hist[2][kRadixBins]; // merged histograms (double-buffered)
  unsigned long long t_exp, t_sel, t_ovh, t_start;
};

// Per-CTA state.
struct LocalState {
  uint32_t hist[kRadixBins];
  uint32_t warp_sums[kWarps];
  uint32_t n_tasks;
  uint32_t sel_digit, sel_above;
  // snapshots of team values, taken after a barrier
  uint32_t n_in, n_br, cur, n_next, pool_end, pool_n, hits_lo, hits_hi;
  uint64_t sel_pushes;
  uint32_t key_min, key_max;
  Key3 sel_prefix;
  uint32_t sel_rem;
  int sel_ge;
};

// Task table of a chunk of branching parents, in dynamic shared memory.
struct BranchTable {
  uint4 *info;      // c0, fan-out, hash base, mode | lg << 8
  double *score;    // parent score
  uint32_t *start;  // first task of each parent
};

// Row of the current step, in dynamic shared memory.
struct RowView {
  uint32_t *id;
  float *lp;
  uint32_t *orig;
  uint32_t K;
};

struct Ctx {
  const SearchParams *p;
  SlotView slot;
  TeamState *T;   // rank 0's team state (distributed shared memory)
  LocalState *S;  // this CTA's state
  RowView row;
  const Beam *cur;
  uint32_t step;   // t
  double f_next;   // length-norm factor of the candidates' depth (t + 1)
  uint32_t rank;   // CTA rank in the team
  uint32_t cs;     // team size (CTAs)
  __device__ uint32_t gtid() const { return rank * blockDim.x + threadIdx.x; }
  __device__ uint32_t gthreads() const { return cs * blockDim.x; }
};

__device__ __forceinline__ void team_sync() { cg::this_cluster().sync(); }

// Records the first failed self-check (one writer wins).
__device__ void report(const Ctx &c, uint32_t code, uint32_t n, uint32_t k, uint32_t got) {
  atomicOr(c.p->status, kStatusSelection);
  if (c.p->debug && atomicCAS(c.p->debug, 0u, code) == 0u) {
    c.p->debug[1] = c.step;
    c.p->debug[2] = n;
    c.p->debug[3] = k;
    c.p->debug[4] = got;
    c.p->debug[5] = c.cs;
    c.p->debug[6] = (uint32_t)c.S->sel_ge;
    c.p->debug[7] = c.S->sel_rem;
  }
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// First index in the sorted row whose id >= x.
__device__ __forceinline__ uint32_t row_lower_bound(const RowView &r, uint32_t x) {
  uint32_t lo = 0, n = r.K;
  while (n > 0) {
    const uint32_t half = n >> 1;
    if (r.id[lo + half] < x) {
      lo += half + 1;
      n -= half + 1;
    } else {
      n = half;
    }
  }
  return lo;
}

// Warp-aggregated append on a (possibly remote) counter: this thread's slot.
__device__ __forceinline__ uint32_t append_slot(uint32_t *counter) {
  cg::coalesced_group g = cg::coalesced_threads();
  uint32_t base = 0;
  if (g.thread_rank() == 0) base = atomicAdd(counter, (uint32_t)g.size());
  base = g.shfl(base, 0);
  return base + g.thread_rank();
}

__device__ __forceinline__ void push_next(const Ctx &c, double score, uint32_t node, uint32_t off, uint32_t parent,
                                          uint32_t token) {
  {
    // Track the range of the first key word so the selection can skip the
    // bits every candidate shares.
    cg::coalesced_group g = cg::coalesced_threads();
    const uint32_t k1 = (uint32_t)(orderable(score * c.f_next) >> 32);
    const uint32_t mn = cg::reduce(g, k1, cg::less<uint32_t>());
    const uint32_t mx = cg::reduce(g, k1, cg::greater<uint32_t>());
    if (g.thread_rank() == 0) {
      atomicMin(&c.T->key_min, mn);
      atomicMax(&c.T->key_max, mx);
    }
  }
  const uint32_t i = append_slot(&c.T->n_next);
  if (i < c.p->cand_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = off;
    v.parent = parent;
    v.token = token;
    c.slot.next[i] = v;
  } else {
    atomicOr(c.p->status, kStatusCandOverflow);
  }
}

__device__ __forceinline__ void push_pool(const Ctx &c, double score, uint32_t node, uint32_t parent,
                                          uint32_t token) {
  const uint32_t i = append_slot(&c.T->pool_end);
  if (i < c.p->pool_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = c.step + 1;  // depth
    v.parent = parent;
    v.token = token;
    c.slot.pool[i] = v;
  } else {
    atomicOr(c.p->status, kStatusPoolOverflow);
  }
}

// Is the string finished after consuming tail cell `off`?
__device__ __forceinline__ bool tail_ends_at(const TrieView &t, uint32_t off, bool &ok) {
  if (t.tail_end) {
    ok = off < t.tail_size;
    return ok ? ((__ldg(t.tail_end + (off >> 6)) >> (off & 63)) & 1ull) : true;
  }
  ok = (uint64_t)off + 1 < t.tail_size;
  return ok ? (__ldg(t.tail + off + 1) == kTailTerm) : true;
}

// ------------------------------------------------------- block scans
__device__ __forceinline__ uint32_t block_exclusive_sum(uint32_t v, LocalState *S) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= (uint32_t)o) inc += y;
  }
  if (lane == 31) S->warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < (uint32_t)kWarps ? S->warp_sums[lane] : 0;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= (uint32_t)o) wi += y;
    }
    if (lane < (uint32_t)kWarps) S->warp_sums[lane] = wi - w;  // exclusive
  }
  __syncthreads();
  const uint32_t r = S->warp_sums[warp] + inc - v;
  __syncthreads();
  return r;
}

// ------------------------------------------------------------ expansion
__device__ void expand_inlink(const Ctx &c) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t n_in = c.S->n_in;
  for (uint32_t i = c.gtid(); i < n_in; i += c.gthreads()) {
    const Beam b = ld_beam(c.cur + i);
    const uint32_t off = b.off;
    if ((uint64_t)off >= t.tail_size || (uint64_t)b.node >= t.num_nodes) {
      atomicOr(c.p->status, kStatusTailBounds);
      continue;
    }
    const uint32_t tok = __ldg(t.tail + off);
    bool ok;
    const bool end = tail_ends_at(t, off, ok);
    if (!ok) {
      atomicOr(c.p->status, kStatusTailBounds);
      continue;
    }
    const uint32_t lo = row_lower_bound(c.row, tok);
    if (lo >= c.row.K || c.row.id[lo] != tok) continue;
    uint32_t hi = lo + 1;
    while (hi < c.row.K && c.row.id[hi] == tok) ++hi;
    for (uint32_t m = lo; m < hi; ++m) {
      // Duplicate ids: each reference thread keeps its first match only
      // (matches are in original column order within an equal-id run).
      bool first = true;
      for (uint32_t m2 = lo; m2 < m; ++m2)
        if ((c.row.orig[m2] % kRefBlock) == (c.row.orig[m] % kRefBlock)) first = false;
      if (!first) continue;
      const double lp = (double)c.row.lp[m];
      if (lp <= tt || b.score + lp <= st) continue;
      const double score = b.score + lp;
      if (end) {
        if (__ldg(t.flags + b.node) & kNodeFlagTerminal) push_pool(c, score, b.node, i, tok);
      } else {
        push_next(c, score, b.node, off + 1, i, tok);
      }
    }
  }
}

// Expansion mode of a branching parent.
constexpr uint32_t kModeScan = 0;  // every child looks its label up in the row
constexpr uint32_t kModeHash = 1;  // every proposal probes the parent's hash table
constexpr uint32_t kModeBin = 2;   // every proposal binary-searches the child labels
constexpr uint32_t kItemsPerLane = kTaskItems / 32;

// The shorter side is iterated; a large fan-out uses the node's hash table
// (one probe per proposal), or a binary search when it has none.
__device__ __forceinline__ uint32_t pick_mode(uint32_t d, uint32_t K, uint8_t f) {
  if (d <= 2u * K + 32u) return kModeScan;
  if (f & kNodeFlagHashed) return kModeHash;
  return kModeBin;
}

// Records a child found for parent q (chunk-local) and sorted-row column m.
__device__ __forceinline__ void push_hit(const Ctx &c, uint32_t child, uint32_t q, uint32_t m) {
  const uint32_t i = append_slot(&c.T->n_hits);
  if (i < c.p->cand_cap) {
    c.slot.hits[i] = Hit{child, (q << 16) | m};
  } else {
    atomicOr(c.p->status, kStatusCandOverflow);
  }
}

// Lookup tasks.  All loads of a lane's items are issued before any is used.
__device__ __forceinline__ void task_scan(const Ctx &c, uint32_t c0, uint32_t d, uint32_t first_item, double score,
                                          uint32_t q) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t lane = threadIdx.x & 31;
  uint32_t lab[kItemsPerLane];
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t i = first_item + 32u * k + lane;
    lab[k] = i < d ? __ldg(t.first_label + c0 + i) : 0u;
  }
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t i = first_item + 32u * k + lane;
    if (i >= d) continue;
    for (uint32_t m = row_lower_bound(c.row, lab[k]); m < c.row.K && c.row.id[m] == lab[k]; ++m) {
      const double lp = (double)c.row.lp[m];
      if (lp <= tt || score + lp <= st) continue;
      push_hit(c, c0 + i, q, m);
    }
  }
}

__device__ __forceinline__ void task_hash(const Ctx &c, uint32_t base, uint32_t lg, uint32_t first_item, double score,
                                          uint32_t q) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t mask = (1u << lg) - 1u;
  uint32_t x[kItemsPerLane], h[kItemsPerLane];
  uint2 slot[kItemsPerLane];
  bool on[kItemsPerLane];
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t m = first_item + 32u * k + lane;
    on[k] = false;
    x[k] = 0;
    h[k] = 0;
    if (m < c.row.K) {
      const double lp = (double)c.row.lp[m];
      x[k] = c.row.id[m];
      on[k] = !(lp <= tt || score + lp <= st);
    }
    if (on[k]) {
      h[k] = (x[k] * 2654435761u) >> (32 - lg);
      slot[k] = __ldg(t.hash + base + h[k]);
    }
  }
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    if (!on[k]) continue;
    uint2 sl = slot[k];
    uint32_t hk = h[k];
    while (sl.y != 0 && sl.x != x[k]) {
      hk = (hk + 1) & mask;
      sl = __ldg(t.hash + base + hk);
    }
    if (sl.y != 0) push_hit(c, sl.y, q, first_item + 32u * k + lane);
  }
}

__device__ __forceinline__ void task_bin(const Ctx &c, uint32_t c0, uint32_t d, uint32_t first_item, double score,
                                         uint32_t q) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t *labs = t.first_label + c0;
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t m = first_item + 32u * k + lane;
    if (m >= c.row.K) continue;
    const double lp = (double)c.row.lp[m];
    if (lp <= tt || score + lp <= st) continue;
    const uint32_t xv = c.row.id[m];
    uint32_t lo = 0, n = d;
    while (n > 0) {
      const uint32_t half = n >> 1;
      if (__ldg(labs + lo + half) < xv) {
        lo += half + 1;
        n -= half + 1;
      } else {
        n = half;
      }
    }
    if (lo < d && __ldg(labs + lo) == xv) push_hit(c, c0 + lo, q, m);
  }
}

// Turns hits [lo, hi) into candidates: one flags/link_off gather per hit,
// issued for two hits at a time (tbs-kernels.cu:295-317).
__device__ void resolve_hits(const Ctx &c, const BranchTable &bt, uint32_t c_first, uint32_t lo_hit, uint32_t hi_hit) {
  const TrieView &t = c.p->trie;
  const uint32_t beam_cap = c.p->beam_cap;
  const uint32_t stride = c.gthreads();
  for (uint32_t i0 = lo_hit + c.gtid(); i0 < hi_hit; i0 += 2 * stride) {
    Hit hv[2];
    uint8_t f[2];
    uint32_t lo[2];
    bool ok[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t i = i0 + k * stride;
      ok[k] = i < hi_hit;
      if (ok[k]) {
        hv[k] = ld_hit(c.slot.hits + i);
        const uint32_t ch = (uint64_t)hv[k].child < t.num_nodes ? hv[k].child : 0u;
        f[k] = __ldg(t.flags + ch);
        lo[k] = __ldg(t.link_off + ch);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (!ok[k]) continue;
      const uint32_t q = hv[k].qm >> 16, m = hv[k].qm & 0xFFFFu;
      if (q >= kParentChunk || m >= c.row.K || (uint64_t)hv[k].child >= t.num_nodes) {
        report(c, 3, q, m, hv[k].child);
        continue;
      }
      const double score = bt.score[q] + (double)c.row.lp[m];
      const uint32_t token = c.row.id[m];
      const uint32_t parent_idx = beam_cap - 1 - (c_first + q);
      const uint32_t child = hv[k].child;
      if (!(f[k] & kNodeFlagLink)) {
        push_next(c, score, child, kNoOffset, parent_idx, token);
        if (f[k] & kNodeFlagTerminal) push_pool(c, score, child, parent_idx, token);
      } else if (f[k] & kNodeFlagLinkEnds1) {
        // The link's string ended with its first token (tbs-kernels.cu:310-313).
        if (f[k] & kNodeFlagTerminal) push_pool(c, score, child, parent_idx, token);
      } else {
        push_next(c, score, child, lo[k] + 1, parent_idx, token);
      }
    }
  }
}

// Branching beams, per chunk of parents: every CTA builds the same task table
// of (parent, 128 items); the team's warps drain it doing lookups only; then
// all threads of the team resolve the hits.  A heavy parent is spread over
// every warp of the team, and the dependent gathers of the matches happen in
// one bulk round.
__device__ void expand_branch(const Ctx &c, const BranchTable &bt) {
  const TrieView &t = c.p->trie;
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t n_br = c.S->n_br;
  const uint32_t K = c.row.K;
  const uint32_t beam_cap = c.p->beam_cap;
  for (uint32_t c_first = 0; c_first < n_br; c_first += kParentChunk) {
    const uint32_t m = min(kParentChunk, n_br - c_first);
    uint32_t my_tasks[kParentChunk / kSearchThreads];
#pragma unroll
    for (uint32_t r = 0; r < kParentChunk / kSearchThreads; ++r) {
      const uint32_t q = threadIdx.x * (kParentChunk / kSearchThreads) + r;
      my_tasks[r] = 0;
      if (q >= m) continue;
      const uint32_t idx = beam_cap - 1 - (c_first + q);
      const Beam b = ld_beam(c.cur + idx);
      uint4 info = make_uint4(0, 0, 0, 0);
      if ((uint64_t)b.node >= t.num_nodes) {
        atomicOr(c.p->status, kStatusNodeBounds);
      } else {
        const uint32_t c0 = __ldg(t.child_begin + b.node);
        const uint32_t c1 = __ldg(t.child_begin + b.node + 1);
        const uint32_t d = c1 > c0 ? c1 - c0 : 0;
        uint8_t f = 0;
        uint32_t hbase = 0;
        if (d > 2u * K + 32u) {
          f = __ldg(t.flags + b.node);
          if (f & kNodeFlagHashed) hbase = __ldg(t.link_off + b.node);
        }
        const uint32_t mode = pick_mode(d, K, f);
        const uint32_t items = (d == 0) ? 0u : (mode == kModeScan ? d : K);
        info = make_uint4(c0, d, hbase, mode | ((uint32_t)(f >> 3) << 8));
        my_tasks[r] = (items + kTaskItems - 1) / kTaskItems;
      }
      bt.info[q] = info;
      bt.score[q] = b.score;
    }
    uint32_t sum = 0;
#pragma unroll
    for (uint32_t r = 0; r < kParentChunk / kSearchThreads; ++r) sum += my_tasks[r];
    uint32_t pre = block_exclusive_sum(sum, c.S);
#pragma unroll
    for (uint32_t r = 0; r < kParentChunk / kSearchThreads; ++r) {
      const uint32_t q = threadIdx.x * (kParentChunk / kSearchThreads) + r;
      if (q < m) bt.start[q] = pre;
      pre += my_tasks[r];
    }
    if (threadIdx.x == blockDim.x - 1) c.S->n_tasks = pre;
    __syncthreads();
    const uint32_t total = c.S->n_tasks;
    const uint32_t team_warps = c.cs * kWarps;
    for (uint32_t task = c.rank * kWarps + warp; task < total; task += team_warps) {
      uint32_t lo = 0, n = m;  // last parent whose first task <= task
      while (n > 1) {
        const uint32_t half = n >> 1;
        if (bt.start[lo + half] <= task) {
          lo += half;
          n -= half;
        } else {
          n = half;
        }
      }
      const uint4 info = bt.info[lo];
      const double score = bt.score[lo];
      const uint32_t first_item = (task - bt.start[lo]) * kTaskItems;
      const uint32_t mode = info.w & 0xFFu;
      if (mode == kModeScan) {
        task_scan(c, info.x, info.y, first_item, score, lo);
      } else if (mode == kModeHash) {
        task_hash(c, info.z, info.w >> 8, first_item, score, lo);
      } else {
        task_bin(c, info.x, info.y, first_item, score, lo);
      }
    }
    team_sync();  // every hit of the chunk is written
    if (threadIdx.x == 0) {
      c.S->hits_lo = c.S->hits_hi;
      c.S->hits_hi = min(c.T->n_hits, (uint32_t)c.p->cand_cap);
    }
    __syncthreads();
    // The next chunk's hits must not be appended before every CTA has taken
    // its snapshot of this chunk's end.
    if (c_first + kParentChunk < n_br) team_sync();
    resolve_hits(c, bt, c_first, c.S->hits_lo, c.S->hits_hi);
    __syncthreads();  // the task table is rebuilt for the next chunk
  }
}

// ------------------------------------------------------------- selection
// Exact top-k threshold over n candidates by the 192-bit key, computed by the
// whole team: each CTA histograms its share of the keys and adds it into rank
// 0's merged histogram; rank 0 picks the digit.  `start` leading bits of the
// first key word are common to all n keys (equal to those of `common_w0`).
// On return every CTA's LocalState holds the threshold: with sel_ge every key
// >= sel_prefix is taken (exactly k of them), otherwise keys > sel_prefix plus
// sel_rem keys equal to it.
template <bool kPoolKeys>
__device__ void team_radix_select(const Ctx &c, const Cand *v, uint32_t n, uint32_t k, uint32_t depth_const,
                                  int start, uint64_t common_w0) {
  TeamState *T = c.T;
  LocalState *S = c.S;
  const double *factor = c.p->factor;
  if (c.rank == 0) {
    for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) T->hist[0][b] = 0;
    if (threadIdx.x == 0) {
      const uint64_t m0 = start >= 64 ? ~0ull : (start == 0 ? 0ull : ~0ull << (64 - start));
      T->sel_prefix = Key3{{common_w0 & m0, 0, 0}};
      T->sel_mask = Key3{{m0, 0, 0}};
      T->sel_rem = k;
      T->sel_ge = 0;
      T->eq_taken = 0;
    }
  }
  team_sync();
  int buf = 0;
  for (int from_top = start; from_top < kKeyBits; from_top += kRadixBits) {
    const int width = min(kRadixBits, kKeyBits - from_top);
    for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) S->hist[b] = 0;
    const Key3 P = T->sel_prefix, M = T->sel_mask;
    __syncthreads();
    for (uint32_t i = c.gtid(); i < n; i += c.gthreads()) {
      const Cand cv = ld_cand(v + i);
      const uint32_t depth = kPoolKeys ? min(cv.aux, c.step + 1) : depth_const;
      const Key3 key = cand_key(cv, factor[depth], depth);
      if ((key.w[0] & M.w[0]) == P.w[0] && (key.w[1] & M.w[1]) == P.w[1] && (key.w[2] & M.w[2]) == P.w[2])
        atomicAdd(&S->hist[key_bits(key, from_top, width)], 1u);
    }
    __syncthreads();
    if (c.cs == 1) {
      for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) T->hist[buf][b] = S->hist[b];
    } else {
      for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x)
        if (S->hist[b]) atomicAdd(&T->hist[buf][b], S->hist[b]);
    }
    team_sync();
    if (c.rank == 0) {
      // Bins from the top: thread i owns bins 2047-4i .. 2044-4i.
      constexpr int kPer = kRadixBins / kSearchThreads;
      uint32_t mine[kPer];
      uint32_t sum = 0;
#pragma unroll
      for (int q = 0; q < kPer; ++q) {
        mine[q] = T->hist[buf][kRadixBins - 1 - kPer * threadIdx.x - q];
        sum += mine[q];
      }
      const uint32_t rem = T->sel_rem;
      const uint32_t above = block_exclusive_sum(sum, S);
      if (above < rem && rem <= above + sum) {
        uint32_t acc = above;
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
          if (acc + mine[q] >= rem) {
            S->sel_digit = kRadixBins - 1 - kPer * threadIdx.x - q;
            S->sel_above = acc;
            break;
          }
          acc += mine[q];
        }
      }
      for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) T->hist[buf ^ 1][b] = 0;
      if (threadIdx.x == blockDim.x - 1 && above + sum < rem) S->sel_digit = 0xFFFFFFFFu;
      __syncthreads();
      if (threadIdx.x == 0 && S->sel_digit == 0xFFFFFFFFu) {
        // Fewer keys match the prefix than remain to be taken: the key range
        // was wrong.  Report it and take everything at or above the prefix.
        atomicOr(c.p->status, kStatusSelection);
        T->sel_ge = 1;
      } else if (threadIdx.x == 0) {
        const uint32_t d = S->sel_digit;
        T->sel_rem = rem - S->sel_above;
        key_set_bits(T->sel_prefix, from_top, width, d);
        key_set_bits(T->sel_mask, from_top, width, low_mask(width));
        if (T->hist[buf][d] == T->sel_rem) T->sel_ge = 1;
      }
    }
    team_sync();
    if (T->sel_ge) break;
    buf ^= 1;
  }
  if (threadIdx.x == 0) {
    S->sel_prefix = T->sel_prefix;
    S->sel_rem = T->sel_rem;
    S->sel_ge = T->sel_ge;
  }
  __syncthreads();
}

// Is `key` among the selected?  Equal keys beyond the threshold count are
// indistinguishable beams, so which of them are taken does not matter.
__device__ __forceinline__ bool is_selected(const Ctx &c, const Key3 &key) {
  const int r = key_cmp(key, c.S->sel_prefix);
  if (c.S->sel_ge) return r >= 0;  // the prefix has its free bits at zero
  if (r > 0) return true;
  if (r < 0) return false;
  return atomicAdd(&c.T->eq_taken, 1u) < c.S->sel_rem;
}

// Makes the selected candidates the beams of step t+1.
__device__ void materialize_next(const Ctx &c, uint32_t n, uint32_t k, Beam *out_beams) {
  const uint32_t depth = c.step + 1;
  const double f = c.p->factor[depth];
  const bool all = n <= k;
  if (k == 0) return;
  if (!all) {
    const uint32_t lo = c.S->key_min, hi = c.S->key_max;
    const int common = (lo == hi) ? 32 : __clz((int)(lo ^ hi));
    team_radix_select<false>(c, c.slot.next, n, k, depth, common, (uint64_t)lo << 32);
  }
  const uint32_t beam_cap = c.p->beam_cap;
  Hist *hist = c.slot.hist + (uint64_t)depth * beam_cap;
  for (uint32_t i = c.gtid(); i < n; i += c.gthreads()) {
    const Cand v = ld_cand(c.slot.next + i);
    if (!all && !is_selected(c, cand_key(v, f, depth))) continue;
    // In-link beams fill the buffer from the front, branching beams from the
    // back; the capped total keeps the two from ever overlapping.
    if (atomicAdd(&c.T->n_sel, 1u) >= k) {
      atomicOr(c.p->status, kStatusSelection);
      continue;
    }
    const bool in_link = v.aux != kNoOffset;
    const uint32_t idx = in_link ? atomicAdd(&c.T->n_in_new, 1u) : beam_cap - 1 - atomicAdd(&c.T->n_br_new, 1u);
    Beam b;
    b.score = v.score;
    b.node = v.node;
    b.off = v.aux;
    out_beams[idx] = b;
    hist[idx] = Hist{v.parent, v.token};
  }
}

// Trims the pool to its best `k` entries; returns the entries kept.
__device__ uint32_t trim_pool(const Ctx &c, uint32_t n, uint32_t k) {
  if (n <= k) return n;
  team_radix_select<true>(c, c.slot.pool, n, k, 0, 0, 0);
  if (c.rank == 0 && threadIdx.x == 0) c.T->n_compact = 0;
  team_sync();
  for (uint32_t i = c.gtid(); i < n; i += c.gthreads()) {
    const Cand v = ld_cand(c.slot.pool + i);
    if (v.aux == 0 || v.aux > c.step + 1) {
      report(c, 4, i, v.aux, c.step);
      continue;
    }
    if (!is_selected(c, cand_key(v, c.p->factor[v.aux], v.aux))) continue;
    const uint32_t j = atomicAdd(&c.T->n_compact, 1u);
    if (j < k) c.slot.pool_tmp[j] = v;
  }
  team_sync();
  const uint32_t got = c.T->n_compact;
  if (got != k && c.rank == 0 && threadIdx.x == 0) report(c, 2, n, k, got);
  const uint32_t kept = min(got, k);
  for (uint32_t i = c.gtid(); i < kept; i += c.gthreads()) c.slot.pool[i] = ld_cand(c.slot.pool_tmp + i);
  return kept;
}

// Sorts the final pool (descending) and writes the ascending result (rank 0).
__device__ void write_result(const SearchParams &p, const SlotView &slot, uint32_t n, uint32_t req, uint8_t *dyn) {
  uint32_t P2 = 1;
  while (P2 < n) P2 <<= 1;
  ulonglong2 *items = reinterpret_cast<ulonglong2 *>(dyn);
  for (uint32_t i = threadIdx.x; i < P2; i += blockDim.x) {
    ulonglong2 it = make_ulonglong2(0, 0);
    if (i < n) {
      const Cand v = ld_cand(slot.pool + i);
      it.x = orderable(v.score * p.factor[min(v.aux, p.out_stride)]);
      it.y = ((uint64_t)v.node << 32) | ((uint64_t)(v.aux & 0xFFFFu) << 16) | (uint64_t)i;
    }
    items[i] = it;
  }
  __syncthreads();
  // Bitonic sort, descending.
  for (uint32_t kk = 2; kk <= P2; kk <<= 1) {
    for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
      for (uint32_t i = threadIdx.x; i < P2; i += blockDim.x) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
          const ulonglong2 a = items[i], b = items[ixj];
          const bool a_less = (a.x < b.x) || (a.x == b.x && a.y < b.y);
          const bool desc = (i & kk) == 0;
          if (a_less == desc) {
            items[i] = b;
            items[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const uint32_t cap = p.out_cap, stride = p.out_stride;
  for (uint32_t s = threadIdx.x; s < n; s += blockDim.x) {
    const uint32_t idx = (uint32_t)(items[s].y & 0xFFFFu);
    const Cand v = ld_cand(slot.pool + idx);
    const uint32_t o = n - 1 - s;
    const uint64_t slot_o = (uint64_t)req * cap + o;
    uint32_t depth = v.aux;
    if (depth == 0 || depth > stride) {
      atomicOr(p.status, kStatusSelection);
      depth = 0;
    }
    p.out_lpn[slot_o] = depth ? v.score * p.factor[depth] : 0.0;
    p.out_len[slot_o] = depth;
    uint32_t *tok = p.out_tok + slot_o * stride;
    if (depth) tok[depth - 1] = v.token;
    uint32_t j = v.parent;
    for (uint32_t st = depth ? depth - 1 : 0; st >= 1; --st) {
      if (j >= p.beam_cap) {
        atomicOr(p.status, kStatusSelection);
        break;
      }
      const Hist h = ld_hist(slot.hist + (uint64_t)st * p.beam_cap + j);
      tok[st - 1] = h.token;
      j = h.parent;
    }
  }
  if (threadIdx.x == 0) p.out_count[req] = n;
}

__device__ void search_request(const SearchParams &p, uint32_t req, const SlotView &slot, TeamState *T,
                               LocalState *S, uint32_t rank, uint32_t cs, uint8_t *dyn) {
  const ReqMeta meta = p.meta[req];
  const uint32_t L = meta.L, K = meta.K;
  const uint32_t *beams = p.beams + meta.beams_off;
  const bool leader = rank == 0 && threadIdx.x == 0;
  if (leader) {
    T->t_start = global_ns();
    T->t_exp = T->t_sel = T->t_ovh = 0;
  }
  if (L == 0) {
    if (leader) {
      p.out_count[req] = 0;
      atomicOr(p.status, kStatusBadRequest);
    }
    return;
  }
  const uint32_t final_beam = beams[L - 1];
  if (final_beam == 0) {
    if (leader) p.out_count[req] = 0;
    return;
  }
  // Device-resident batches are not validated on the host: refuse widths
  // beyond the workspace instead of writing past it.
  bool bad = final_beam > p.out_cap || L > p.out_stride;
  for (uint32_t t = threadIdx.x; t < L; t += blockDim.x) bad |= beams[t] > p.beam_cap;
  if (__syncthreads_or(bad)) {
    if (leader) {
      p.out_count[req] = 0;
      atomicOr(p.status, kStatusBadRequest);
    }
    return;
  }
  const uint32_t beam_cap = p.beam_cap;
  if (leader) {
    Beam root;
    root.score = 0.0;
    root.node = 0;
    root.off = kNoOffset;
    slot.beams[0][beam_cap - 1] = root;
    T->n_in = 0;
    T->n_br = 1;
    T->cur = 0;
    T->pool_n = 0;
    T->sel_pushes = 0;
  }
  RowView row;
  row.id = reinterpret_cast<uint32_t *>(dyn);
  row.lp = reinterpret_cast<float *>(dyn + sizeof(uint32_t) * K);
  row.orig = reinterpret_cast<uint32_t *>(dyn + 2 * sizeof(uint32_t) * K);
  row.K = K;
  BranchTable bt;
  {
    uint8_t *tb = dyn + ((12u * K + 15u) & ~15u);
    bt.info = reinterpret_cast<uint4 *>(tb);
    bt.score = reinterpret_cast<double *>(tb + sizeof(uint4) * kParentChunk);
    bt.start = reinterpret_cast<uint32_t *>(tb + (sizeof(uint4) + sizeof(double)) * kParentChunk);
  }
  team_sync();

  for (uint32_t t = 0; t < L; ++t) {
    unsigned long long t0 = 0;
    if (leader) t0 = global_ns();
    if (threadIdx.x == 0) {
      S->n_in = min(T->n_in, beam_cap);
      S->n_br = min(T->n_br, beam_cap - S->n_in);
      S->cur = T->cur & 1u;
      S->sel_pushes = T->sel_pushes;
      S->pool_n = T->pool_n;
      S->hits_lo = S->hits_hi = 0;
    }
    __syncthreads();
    if (S->n_in + S->n_br == 0 || (p.early_exit && S->sel_pushes >= final_beam)) break;
    const uint64_t rbase = meta.rows_off + (uint64_t)t * K;
    for (uint32_t j = threadIdx.x; j < K; j += blockDim.x) {
      row.id[j] = p.row_id[rbase + j];
      row.lp[j] = p.row_lp[rbase + j];
      row.orig[j] = p.row_orig[rbase + j];
    }
    if (leader) {
      T->n_next = 0;
      T->pool_end = T->pool_n;
      T->n_sel = 0;
      T->n_in_new = 0;
      T->n_br_new = 0;
      T->n_hits = 0;
      T->key_min = 0xFFFFFFFFu;
      T->key_max = 0u;
    }
    team_sync();
    unsigned long long t1 = 0;
    if (leader) t1 = global_ns();

    Ctx c;
    c.p = &p;
    c.slot = slot;
    c.T = T;
    c.S = S;
    c.row = row;
    c.cur = slot.beams[S->cur];
    c.step = t;
    c.f_next = p.factor[t + 1];
    c.rank = rank;
    c.cs = cs;
    expand_inlink(c);
    expand_branch(c, bt);
    team_sync();
    unsigned long long t2 = 0;
    if (leader) t2 = global_ns();

    if (threadIdx.x == 0) {
      S->n_next = min(T->n_next, (uint32_t)p.cand_cap);
      S->pool_end = min(T->pool_end, (uint32_t)p.pool_cap);
      S->key_min = T->key_min;
      S->key_max = T->key_max;
    }
    __syncthreads();
    const uint32_t n_next = S->n_next, pool_end = S->pool_end, pool_before = S->pool_n;
    materialize_next(c, n_next, beams[t], slot.beams[S->cur ^ 1]);
    team_sync();
    const uint32_t kept = trim_pool(c, pool_end, final_beam);
    team_sync();
    if (leader) {
      T->sel_pushes += (uint64_t)(pool_end - pool_before);
      T->pool_n = kept;
      uint32_t n_in_new = T->n_in_new, n_br_new = T->n_br_new;
      const uint32_t want = min(n_next, beams[t]);
      if (T->n_sel != want || n_in_new + n_br_new != want) {
        report(c, 1, n_next, beams[t], T->n_sel);
        n_in_new = n_br_new = 0;  // the beam buffer is not trustworthy: stop
      }
      T->n_in = n_in_new;
      T->n_br = n_br_new;
      T->cur ^= 1;
      const unsigned long long t3 = global_ns();
      T->t_ovh += t1 - t0;
      T->t_exp += t2 - t1;
      T->t_sel += t3 - t2;
    }
    team_sync();
  }
  if (rank == 0) {
    unsigned long long t4 = 0;
    if (threadIdx.x == 0) {
      t4 = global_ns();
      S->pool_n = T->pool_n;
    }
    __syncthreads();
    write_result(p, slot, S->pool_n, req, dyn);
    if (threadIdx.x == 0 && p.out_phase_ms) {
      const unsigned long long t5 = global_ns();
      double *ph = p.out_phase_ms + (uint64_t)req * 5;
      ph[0] = T->t_exp * 1e-6;
      ph[1] = 0.0;  // validation is fused into expansion
      ph[2] = T->t_sel * 1e-6;
      ph[3] = (T->t_ovh + (t5 - t4)) * 1e-6;
      ph[4] = (t5 - T->t_start) * 1e-6;
    }
  }
}

__global__ void __launch_bounds__(kSearchThreads, 1) tbs_search_kernel(const SearchParams p) {
  extern __shared__ __align__(16) uint8_t dyn[];
  __shared__ TeamState team_state;
  __shared__ LocalState local_state;
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t cs = cluster.num_blocks();
  const uint32_t rank = cluster.block_rank();
  TeamState *T = cluster.map_shared_rank(&team_state, 0);
  const uint32_t team = blockIdx.x / cs, n_teams = gridDim.x / cs;
  const SlotView slot = p.slots[team];
  for (uint32_t req = team; req < p.n_req; req += n_teams) {
    search_request(p, req, slot, T, &local_state, rank, cs, dyn);
    team_sync();  // rank 0's state is reused by the next request
  }
}

// Sorts each row by (id, original column) so the search can binary-search it;
// rows that are already strictly ascending are copied as they are.
__global__ void row_prep_kernel(const ReqMeta *meta, const uint32_t *ids, const float *lps, uint32_t *out_id,
                                float *out_lp, uint32_t *out_orig, uint32_t n_req) {
  extern __shared__ __align__(16) uint8_t dyn[];
  uint64_t *keys = reinterpret_cast<uint64_t *>(dyn);
  const uint32_t r = blockIdx.y, t = blockIdx.x;
  if (r >= n_req) return;
  const ReqMeta m = meta[r];
  if (t >= m.L) return;
  const uint32_t K = m.K;
  const uint64_t base = m.rows_off + (uint64_t)t * K;
  bool ok = true;
  for (uint32_t j = threadIdx.x; j + 1 < K; j += blockDim.x)
    if (ids[base + j] >= ids[base + j + 1]) ok = false;
  if (__syncthreads_and(ok)) {
    for (uint32_t j = threadIdx.x; j < K; j += blockDim.x) {
      out_id[base + j] = ids[base + j];
      out_lp[base + j] = lps[base + j];
      out_orig[base + j] = j;
    }
    return;
  }
  uint32_t P2 = 1;
  while (P2 < K) P2 <<= 1;
  for (uint32_t j = threadIdx.x; j < P2; j += blockDim.x)
    keys[j] = j < K ? (((uint64_t)ids[base + j] << 32) | j) : ~0ull;
  __syncthreads();
  for (uint32_t kk = 2; kk <= P2; kk <<= 1) {
    for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
      for (uint32_t i = threadIdx.x; i < P2; i += blockDim.x) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = keys[i], b = keys[ixj];
          const bool up = (i & kk) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (uint32_t j = threadIdx.x; j < K; j += blockDim.x) {
    const uint32_t o = (uint32_t)(keys[j] & 0xFFFFFFFFu);
    out_id[base + j] = (uint32_t)(keys[j] >> 32);
    out_lp[base + j] = lps[base + o];
    out_orig[base + j] = o;
  }
}

}  // namespace

size_t search_smem_bytes(uint32_t max_topk, uint32_t max_final_beam) {
  uint32_t P2 = 1;
  while (P2 < max_final_beam) P2 <<= 1;
  const size_t row = (((size_t)max_topk * 12 + 15) & ~size_t(15)) +
                     (size_t)kParentChunk * (sizeof(uint4) + sizeof(double) + sizeof(uint32_t));
  const size_t sort = (size_t)P2 * 16;
  return std::max<size_t>(std::max(row, sort), 16);
}

int configure_search_kernel(size_t smem_bytes) {
  CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
  CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  CUDA_TRY(cudaFuncSetAttribute(row_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tbs_search_kernel, kSearchThreads, smem_bytes));
  int dev = 0, sms = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return std::max(per_sm, 1) * sms;
}

int ensure_search_smem(size_t search_smem, size_t prep_smem) {
  cudaFuncAttributes a;
  CUDA_TRY(cudaFuncGetAttributes(&a, tbs_search_kernel));
  if ((size_t)a.maxDynamicSharedSizeBytes < search_smem)
    CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)search_smem));
  CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  CUDA_TRY(cudaFuncGetAttributes(&a, row_prep_kernel));
  if ((size_t)a.maxDynamicSharedSizeBytes < prep_smem)
    CUDA_TRY(cudaFuncSetAttribute(row_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tbs_search_kernel, kSearchThreads, search_smem));
  int dev = 0, sms = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return std::max(per_sm, 1) * sms;
}

int max_search_clusters(int cluster_size, size_t smem_bytes) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_size, 1, 1);
  cfg.blockDim = dim3(kSearchThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cluster_size;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, (void *)tbs_search_kernel, &cfg));
  return n;
}

int pick_cluster_size(uint32_t n, size_t smem_bytes, int *max_teams) {
  int dev = 0, sms = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int cs = 1;
  if (const char *e = getenv("FT_CLUSTER_SIZE")) {
    cs = atoi(e);
    if (cs < 1 || cs > 16 || (cs & (cs - 1))) cs = 1;
  } else {
    const int want = n ? sms / (int)n : sms;
    while (cs * 2 <= 16 && cs * 2 <= want) cs *= 2;
  }
  for (;; cs /= 2) {
    const int teams = max_search_clusters(cs, smem_bytes);
    if (teams >= 1 || cs == 1) {
      *max_teams = std::max(teams, 1);
      return cs;
    }
  }
}

void launch_search(const SearchParams &p, uint32_t max_K, uint32_t max_L, size_t smem_bytes, int grid,
                   cudaStream_t stream, int cluster_size) {
  if (p.n_req == 0) return;
  uint32_t P2 = 1;
  while (P2 < max_K) P2 <<= 1;
  dim3 pg(max_L, p.n_req);
  row_prep_kernel<<<pg, 256, (size_t)P2 * 8, stream>>>(p.meta, p.topk_id, p.topk_logp, p.row_id, p.row_lp,
                                                       p.row_orig, p.n_req);
  CUDA_TRY(cudaGetLastError());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid * cluster_size, 1, 1);
  cfg.blockDim = dim3(kSearchThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cluster_size;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  CUDA_TRY(cudaLaunchKernelEx(&cfg, tbs_search_kernel, p));
}

}  // namespace ftb
