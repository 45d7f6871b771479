// Trie-constrained beam search kernel for sm_100a.
//
// A request is searched by one thread-block cluster ("team") of 1 to 16 CTAs
// that stays on the request for all its steps (persistent grid, requests
// strided over teams).  Team counters live in the shared memory of the team's
// rank-0 CTA and are updated with distributed-shared-memory atomics; radix
// histograms stay in each CTA's own shared memory and are read remotely; the
// phases of a step are separated by hardware cluster barriers.  The reference
// launches one cooperative grid per request and separates each step's
// expansion, pruning and history save with 2-3 grid-wide syncs
// (lib/marisa/grimoire/trie/tbs-kernels.cu:476-594).  Small batches use large
// teams (latency), large batches one-CTA teams (throughput).
//
// Per step t of a request:
//   1. every CTA stages row t (ids ascending, log-probs, original columns)
//      in its shared memory, straight from the caller's top-k arrays; a row
//      that is not in id order is bitonic-sorted by (id, column) there;
//   2. expand:
//      - in-link beams, one thread each: the next tail cell is the only
//        allowed token; look it up in the sorted row (tbs-kernels.cu:324-371);
//      - branching beams: a task table of (parent, 128 items) drained by all
//        warps of the team; an item is a child whose record is loaded and its
//        label looked up in the row (small fan-out), or a proposal that probes
//        the parent's hash table (large fan-out) or binary-searches its child
//        labels (tbs-kernels.cu:210-322), then loads what it found;
//      - thresholds: logp > token_threshold and score + logp > sent_threshold,
//        compared in f64 (tbs-kernels.cu:229-231);
//      - children go to the step's candidate list and, when they end a key,
//        to the result pool (one warp-wide reservation per task);
//   3. select: exact top-beams[t] of the candidates in the pinned order
//      (logp_norm, node, depth, score), an 11-bit MSD radix select over the
//      192-bit key starting after the bits all candidates share (its first
//      pass bins logp_norm linearly when the values span a wide range);
//      survivors become the next step's beams and append (parent, token)
//      history;
//   4. trim the result pool to the final beam the same way when the next
//      step could overflow it.
// After the last step the pool is sorted and written ascending with each
// sequence rebuilt from the history (tbs-kernels.cu:393-474), and with each
// result's key id when asked.
//
// The same file holds the batched key lookups over the same device image:
// lookup_kernel (token sequence -> key id) and reverse_lookup_kernel (key id
// -> token sequence, over parents derived by parents_kernel).
#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

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
// Bounded waits on helper clusters (on the GPU's global timer), the longest
// sleep between two polls of a helper waiting for its leader, and the fewest
// tasks for which a step is opened to helpers.
constexpr unsigned long long kHelpWaitNs = 20000000ull;  // 20 ms
constexpr uint32_t kHelpMaxSleepNs = 1024;
constexpr uint32_t kHelpMinTasks = 1024;

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

// The same key from a candidate's first 16 bytes (score in .x/.y, node in .z).
__device__ __forceinline__ Key3 head_key(const uint4 h, double factor, uint32_t depth) {
  const double score = __hiloint2double((int)h.y, (int)h.x);
  Key3 k;
  k.w[0] = orderable(score * factor);
  k.w[1] = ((uint64_t)h.z << 32) | ((uint64_t)(depth & 0xFFFFu) << 16);
  k.w[2] = orderable(score);
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
// Candidates, beams, pool entries and history are written by any CTA of
// the team and read by another after a cluster barrier; they are loaded
// through L2 (ld.global.cg) so that no SM can see a line it cached earlier.
__device__ __forceinline__ Cand ld_cand(const Cand *p) {
  const uint4 a = __ldcg(reinterpret_cast<const uint4 *>(p));
  const uint4 b = __ldcg(reinterpret_cast<const uint4 *>(p) + 1);
  Cand c;
  c.score = __hiloint2double((int)a.y, (int)a.x);
  c.node = a.z;
  c.aux = a.w;
  c.parent = b.x;
  c.token = b.y;
  c.c0 = b.z;
  c.dw = b.w;
  return c;
}

// The first 16 bytes of a candidate (score, node, aux): all a selection key
// needs.  The second half (parent, token, c0, dw) is loaded only for the
// candidates that are kept.
__device__ __forceinline__ uint4 ld_cand_head(const Cand *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ Cand cand_from(const uint4 a, const Cand *p) {
  const uint4 b = __ldcg(reinterpret_cast<const uint4 *>(p) + 1);
  Cand c;
  c.score = __hiloint2double((int)a.y, (int)a.x);
  c.node = a.z;
  c.aux = a.w;
  c.parent = b.x;
  c.token = b.y;
  c.c0 = b.z;
  c.dw = b.w;
  return c;
}

__device__ __forceinline__ Beam ld_beam(const Beam *p) {
  const uint2 *q = reinterpret_cast<const uint2 *>(p);
  const uint2 a = __ldcg(q), b = __ldcg(q + 1), d = __ldcg(q + 2);
  Beam r;
  r.score = __hiloint2double((int)a.y, (int)a.x);
  r.node = b.x;
  r.off = b.y;
  r.c0 = d.x;
  r.dw = d.y;
  return r;
}

__device__ __forceinline__ uint32_t rec_flags(uint32_t dw) { return dw >> 24; }

// Key id of a terminal node: terminal nodes before it (louds-trie.cc:56-72).
__device__ __forceinline__ uint32_t key_id(const TrieView &t, uint32_t node) {
  const uint4 r = __ldg(t.term_rank + (node >> 6));
  const uint64_t bits = ((uint64_t)r.w << 32) | r.z;
  const uint32_t o = node & 63u;
  return r.x + (uint32_t)__popcll(o ? bits & ((1ull << o) - 1) : 0ull);
}

__device__ __forceinline__ Hist ld_hist(const Hist *p) {
  const uint2 a = __ldcg(reinterpret_cast<const uint2 *>(p));
  return Hist{a.x, a.y};
}

// ---------------------------------------------------------- team state
constexpr int kSuperBins = kRadixBins / 32;  // 64 super-bins of 32 radix bins
constexpr uint32_t kMaxTeam = 16;            // CTAs per team (non-portable cluster size)
// Counters of one step.  Two sets alternate by step parity: the set of step
// t is read by every CTA after the barrier that closes step t, so the leader
// clears it again only after the next step's expansion barrier.
struct StepCounters {
  uint32_t n_sel;     // beams written for the next step (capped at its width)
  uint32_t n_in_new;  // ... of which in-link
  uint32_t n_br_new;  // ... of which branching
  uint32_t eq_taken;  // keys equal to the selection threshold taken so far
  uint32_t n_tasks_new;  // branch tasks of the next step, summed from the branching beams' fan-outs
};

// Authoritative in the team's rank-0 CTA; other CTAs reach it through
// distributed shared memory.
// The expansion counters (xc, pool) are used from here in a request without
// helper clusters, from the slot's HelpState in a request with them.
struct alignas(16) TeamState {
  StepCounters cnt[2];
  ExpCounters xc[2];
  PoolCounters pool;
  uint32_t n_compact;      // entries written by the last pool trim
  uint32_t eq_taken_trim;
  uint32_t pad;
  unsigned long long removed;     // pool entries dropped by trims so far
  unsigned long long t_exp, t_sel, t_ovh, t_start;
};

// Per-CTA state; every CTA of a team derives the same values.
// The radix histograms are double-buffered by pass parity: every CTA reads
// every other CTA's histogram of a pass after that pass's barrier, and a
// buffer is rewritten two passes later, after the next barrier.
struct alignas(16) LocalState {
  uint32_t hist[2][kRadixBins];
  uint32_t super[2][kSuperBins];
  uint32_t part[kMaxTeam * kSuperBins];  // per-rank super-bins / bins of a pass
  uint32_t sel_sb, sel_above;
  uint32_t warp_sums[kWarps];
  uint32_t n_tasks;
  uint32_t n_in, n_br, n_next, pool_end;
  uint32_t key_min, key_max, pool_key_min, pool_key_max;
  unsigned long long pushes;
  Key3 sel_prefix;
  Key3 sel_mask;
  uint32_t sel_rem;
  int sel_ge;
  uint32_t pass;  // radix passes run by the team in this request
  uint32_t out_total;               // tokens of the request's result (compact output)
  unsigned long long out_base;      // their first slot
  uint32_t stop;
  // Value pass of a selection (see team_radix_select): keys fall in bins
  // floor((v - sel_lo) * sel_scale) of their first word's value v.  With
  // sel_in_bin set, keys above bin sel_bin are taken, keys below it are not,
  // and the bit-level threshold above decides among the keys in it.
  double sel_lo, sel_scale;
  uint32_t sel_bin;
  int sel_in_bin;
  int sel_value;  // the selection starts with a value pass
  int sel_next;   // first key bit of the bit passes after the value pass
  uint32_t help_step;   // helper CTA: the step it works on next (kHelpStop: none)
  uint32_t help_epoch;  // the request's helper epoch
  uint32_t pool_base;   // the pool's end at this step's start
  uint32_t pool_add;    // added to pool slots from Ctx::xp (an open step appends after pool_base)
  uint32_t est_tasks;   // this step's branch tasks as the last selection counted them
  uint32_t help_open;   // this step is shared with helper clusters
};
// hist is read as uint4, super and part as uint2 (also over DSMEM).
static_assert(offsetof(LocalState, hist) % 16 == 0 && (sizeof(uint32_t) * kRadixBins) % 16 == 0,
              "LocalState::hist must stay 16-byte aligned");
static_assert(offsetof(LocalState, super) % 8 == 0 && offsetof(LocalState, part) % 8 == 0 &&
                  (sizeof(uint32_t) * kSuperBins) % 8 == 0,
              "LocalState::super and part must stay 8-byte aligned");

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
  TeamState *T;        // rank 0's team state (distributed shared memory)
  StepCounters *cnt;   // this step's counters (in T)
  LocalState *S;       // this CTA's state
  RowView row;
  const Beam *cur;
  uint32_t step;   // t
  double f_next;   // length-norm factor of the candidates' depth (t + 1)
  uint32_t rank;   // CTA rank in the team
  uint32_t cs;     // team size (CTAs)
  // Counters every expanding CTA appends to (this step's set and the
  // pool's): in the leader team's shared memory, or in the slot's HelpState
  // when the request has helper clusters.  help: set while a step is shared
  // with helpers; T == nullptr on a helper CTA.
  ExpCounters *xc;
  PoolCounters *xp;
  HelpState *help;
  // Ranges of this thread's pushes (top 32 bits of the first key word),
  // folded into the team's at the end of expansion.
  mutable uint32_t kmin, kmax, pkmin, pkmax;
  __device__ uint32_t gtid() const { return rank * blockDim.x + threadIdx.x; }
  __device__ uint32_t gthreads() const { return cs * blockDim.x; }
};

// Team barrier: a hardware cluster barrier (release/acquire at cluster
// scope), or a CTA barrier for a one-CTA team (about 10x cheaper).
__device__ __forceinline__ void team_sync(uint32_t cs) {
  if (cs > 1) {
    cg::this_cluster().sync();
  } else {
    __syncthreads();
  }
}

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

// Folds the key ranges of a warp's pushes into the team's (lane 0 issues one
// remote atomic per bound).
__device__ __forceinline__ void publish_ranges(const Ctx &c) {
  uint32_t a = c.kmin, b = c.kmax, d = c.pkmin, e = c.pkmax;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = min(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
    b = max(b, __shfl_xor_sync(0xFFFFFFFFu, b, o));
    d = min(d, __shfl_xor_sync(0xFFFFFFFFu, d, o));
    e = max(e, __shfl_xor_sync(0xFFFFFFFFu, e, o));
  }
  const uint32_t lane = threadIdx.x & 31;
  if (a <= b) {
    if (lane == 0) atomicMin(&c.xc->key_min, a);
    if (lane == 1) atomicMax(&c.xc->key_max, b);
  }
  if (d <= e) {
    if (lane == 2) atomicMin(&c.xp->pool_key_min, d);
    if (lane == 3) atomicMax(&c.xp->pool_key_max, e);
  }
}

__device__ __forceinline__ void push_next(const Ctx &c, double score, uint32_t node, uint32_t off, uint32_t parent,
                                          uint32_t token, uint32_t c0, uint32_t dw) {
  // The range of the first key word lets the selection skip the bits every
  // candidate shares.
  const uint32_t k32 = (uint32_t)(orderable(score * c.f_next) >> 32);
  c.kmin = min(c.kmin, k32);
  c.kmax = max(c.kmax, k32);
  const uint32_t i = append_slot(&c.xc->n_next);
  if (i < c.p->cand_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = off;
    v.parent = parent;
    v.token = token;
    v.c0 = c0;
    v.dw = dw;
    c.slot.next[i] = v;
  } else {
    atomicOr(c.p->status, kStatusCandOverflow);
  }
}

// kHelp (here and down the emission chain): the helper instance, where an
// open step's pool slots are offset by S->pool_add; elsewhere the offset is 0.
template <bool kHelp>
__device__ __forceinline__ void push_pool(const Ctx &c, double score, uint32_t node, uint32_t parent,
                                          uint32_t token) {
  const uint32_t k32 = (uint32_t)(orderable(score * c.f_next) >> 32);
  c.pkmin = min(c.pkmin, k32);
  c.pkmax = max(c.pkmax, k32);
  const uint32_t i = (kHelp ? c.S->pool_add : 0u) + append_slot(&c.xp->pool_end);
  if (i < c.p->pool_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = c.step + 1;  // depth
    v.parent = parent;
    v.token = token;
    v.c0 = 0;
    v.dw = 0;
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
template <bool kHelp>
__device__ void expand_inlink(const Ctx &c) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t n_in = c.S->n_in;
  // Beam i goes to CTA i % cs, and within it round-robin over the warps
  // first, so that every warp holds about the same share of this chain of
  // dependent loads and then takes fewer branch tasks (handed out on demand).
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (uint32_t j = lane * kWarps + warp;; j += blockDim.x) {
    const uint32_t i = j * c.cs + c.rank;
    if (i >= n_in) break;
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
        if (rec_flags(b.dw) & kNodeFlagTerminal) push_pool<kHelp>(c, score, b.node, i, tok);
      } else {
        push_next(c, score, b.node, off + 1, i, tok, b.c0, b.dw);
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
__device__ __forceinline__ uint32_t pick_mode(uint32_t d, uint32_t K, uint32_t f) {
  if (d <= 2u * K + 32u) return kModeScan;
  if (f & kNodeFlagHashed) return kModeHash;
  return kModeBin;
}

// What a matched child yields (tbs-kernels.cu:295-317): a candidate unless it
// is a link child whose string ends with its first token; a pool entry if it
// ends a key there (a terminal plain child, or a terminal link child whose
// string ends with its first token).
__device__ __forceinline__ void classify(uint32_t f, bool &next, bool &pool) {
  const bool link = f & kNodeFlagLink, ends1 = link && (f & kNodeFlagLinkEnds1);
  next = !ends1;
  pool = (f & kNodeFlagTerminal) && (!link || ends1);
}

// Reserves `n` consecutive slots per lane from a team counter with one atomic
// for the whole warp; returns this lane's first slot.  Called by all 32 lanes.
__device__ __forceinline__ uint32_t warp_reserve(uint32_t *counter, uint32_t n) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t inc = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= (uint32_t)o) inc += y;
  }
  const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
  uint32_t base = 0;
  if (lane == 0 && total) base = atomicAdd(counter, total);
  return __shfl_sync(0xFFFFFFFFu, base, 0) + inc - n;
}

// Two reservations at once (called by all 32 lanes): lanes 0 and 1 issue
// their atomics in the same instruction, so the warp waits for one round
// trip instead of two.
__device__ __forceinline__ void warp_reserve2(uint32_t *ca, uint32_t na, uint32_t *cb, uint32_t nb, uint32_t &ba,
                                              uint32_t &bb) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t ia = na, ib = nb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t ya = __shfl_up_sync(0xFFFFFFFFu, ia, o);
    const uint32_t yb = __shfl_up_sync(0xFFFFFFFFu, ib, o);
    if (lane >= (uint32_t)o) {
      ia += ya;
      ib += yb;
    }
  }
  const uint32_t ta = __shfl_sync(0xFFFFFFFFu, ia, 31), tb = __shfl_sync(0xFFFFFFFFu, ib, 31);
  uint32_t *ctr = lane == 0 ? ca : cb;
  const uint32_t tot = lane == 0 ? ta : tb;
  uint32_t base = 0;
  if (lane < 2 && tot) base = atomicAdd(ctr, tot);
  ba = __shfl_sync(0xFFFFFFFFu, base, 0) + ia - na;
  bb = __shfl_sync(0xFFFFFFFFu, base, 1) + ib - nb;
}

__device__ __forceinline__ void write_next(const Ctx &c, uint32_t idx, double score, uint32_t node, uint32_t aux,
                                           uint32_t parent, uint32_t token, uint32_t c0, uint32_t dw) {
  const uint32_t k32 = (uint32_t)(orderable(score * c.f_next) >> 32);
  c.kmin = min(c.kmin, k32);
  c.kmax = max(c.kmax, k32);
  if (idx < c.p->cand_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = aux;
    v.parent = parent;
    v.token = token;
    v.c0 = c0;
    v.dw = dw;
    c.slot.next[idx] = v;
  } else {
    atomicOr(c.p->status, kStatusCandOverflow);
  }
}

template <bool kHelp>
__device__ __forceinline__ void write_pool(const Ctx &c, uint32_t idx, double score, uint32_t node, uint32_t parent,
                                           uint32_t token) {
  if (kHelp) idx += c.S->pool_add;
  const uint32_t k32 = (uint32_t)(orderable(score * c.f_next) >> 32);
  c.pkmin = min(c.pkmin, k32);
  c.pkmax = max(c.pkmax, k32);
  if (idx < c.p->pool_cap) {
    Cand v;
    v.score = score;
    v.node = node;
    v.aux = c.step + 1;  // depth
    v.parent = parent;
    v.token = token;
    v.c0 = 0;
    v.dw = 0;
    c.slot.pool[idx] = v;
  } else {
    atomicOr(c.p->status, kStatusPoolOverflow);
  }
}

// A task's matches: (item k, row column m) pairs, each with the child's record.
// `visit(k, m)` is called for every pair whose log-prob passes the thresholds.
// The warp counts its candidates and pool entries first, reserves them with
// one atomic each, then writes them.
template <bool kHelp, class Pairs>
__device__ __forceinline__ void emit_task(const Ctx &c, double pscore, uint32_t parent_idx, const uint32_t child[4],
                                          const uint4 rec[4], Pairs &&pairs) {
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  uint32_t nn = 0, np = 0;
  pairs([&](uint32_t k, uint32_t m) {
    const double lp = (double)c.row.lp[m];
    if (lp <= tt || pscore + lp <= st) return;
    bool nx, pl;
    classify(rec[k].w >> 24, nx, pl);
    nn += nx;
    np += pl;
  });
  uint32_t bn, bp;
  warp_reserve2(&c.xc->n_next, nn, &c.xp->pool_end, np, bn, bp);
  if (nn + np == 0) return;
  pairs([&](uint32_t k, uint32_t m) {
    const double lp = (double)c.row.lp[m];
    if (lp <= tt || pscore + lp <= st) return;
    const double score = pscore + lp;
    const uint32_t token = c.row.id[m];
    const uint4 &r = rec[k];
    bool nx, pl;
    classify(r.w >> 24, nx, pl);
    const bool link = (r.w >> 24) & kNodeFlagLink;
    if (nx) write_next(c, bn++, score, child[k], link ? r.y + 1 : r.y, parent_idx, token, r.z, r.w);
    if (pl) write_pool<kHelp>(c, bp++, score, child[k], parent_idx, token);
  });
}

// Lower bounds of four ids in the sorted row, advanced in lockstep (branch
// free, the same number of steps for all).
__device__ __forceinline__ void row_lower_bound4(const RowView &r, const uint32_t x[4], uint32_t pos[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) pos[k] = 0;
  if (r.K == 0) return;
  for (uint32_t n = r.K; n > 1;) {
    const uint32_t half = n >> 1;
    uint32_t v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = r.id[pos[k] + half - 1];
#pragma unroll
    for (int k = 0; k < 4; ++k) pos[k] = v[k] < x[k] ? pos[k] + half : pos[k];
    n -= half;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (r.id[pos[k]] < x[k]) ++pos[k];
}

// Lookup tasks (called by all 32 lanes of a warp): a lane's four items issue
// each round of loads before using any.
template <bool kHelp>
__device__ __forceinline__ void task_scan(const Ctx &c, uint32_t c0, uint32_t d, uint32_t first_item, double score,
                                          uint32_t parent_idx) {
  const TrieView &t = c.p->trie;
  const uint32_t lane = threadIdx.x & 31;
  uint4 rec[kItemsPerLane];
  uint32_t child[kItemsPerLane], x[kItemsPerLane], mlo[kItemsPerLane];
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t i = first_item + 32u * k + lane;
    child[k] = c0 + i;
    rec[k] = i < d ? __ldg(t.node + c0 + i) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) x[k] = rec[k].x;
  row_lower_bound4(c.row, x, mlo);
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t i = first_item + 32u * k + lane;
    if (i >= d || mlo[k] >= c.row.K || c.row.id[mlo[k]] != x[k]) mlo[k] = c.row.K;
  }
  emit_task<kHelp>(c, score, parent_idx, child, rec, [&](auto &&fn) {
#pragma unroll
    for (uint32_t k = 0; k < kItemsPerLane; ++k)
      for (uint32_t m = mlo[k]; m < c.row.K && c.row.id[m] == x[k]; ++m) fn(k, m);
  });
}

template <bool kHelp>
__device__ __forceinline__ void task_hash(const Ctx &c, uint32_t base, uint32_t lg, uint32_t first_item, double score,
                                          uint32_t parent_idx) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t size = 1u << lg, mask = size - 1u;
  // The table must lie inside the hash array (base and lg are the same for
  // the whole warp's task, so the early return is warp-uniform).
  if (lg > 31 || (uint64_t)base + size > t.hash_slots) {
    if (lane == 0) atomicOr(c.p->status, kStatusNodeBounds);
    return;
  }
  uint32_t x[kItemsPerLane], h[kItemsPerLane], child[kItemsPerLane];
  uint4 rec[kItemsPerLane];
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
    child[k] = 0;
    rec[k] = make_uint4(0, 0, 0, 0);
    if (!on[k]) continue;
    uint2 sl = slot[k];
    uint32_t hk = h[k];
    // Load <= 1/2 means an empty slot ends every probe of a valid table; a
    // full table (an inconsistent image) ends after `size` probes instead.
    for (uint32_t probe = 1; sl.y != 0 && sl.x != x[k]; ++probe) {
      if (probe >= size) {
        atomicOr(c.p->status, kStatusNodeBounds);
        sl.y = 0;
        break;
      }
      hk = (hk + 1) & mask;
      sl = __ldg(t.hash + base + hk);
    }
    child[k] = sl.y;
    if ((uint64_t)child[k] >= t.num_nodes) {
      atomicOr(c.p->status, kStatusNodeBounds);
      child[k] = 0;
    }
    if (child[k] != 0) rec[k] = __ldg(t.node + child[k]);
  }
  emit_task<kHelp>(c, score, parent_idx, child, rec, [&](auto &&fn) {
#pragma unroll
    for (uint32_t k = 0; k < kItemsPerLane; ++k)
      if (child[k] != 0) fn(k, first_item + 32u * k + lane);
  });
}

template <bool kHelp>
__device__ __forceinline__ void task_bin(const Ctx &c, uint32_t c0, uint32_t d, uint32_t first_item, double score,
                                         uint32_t parent_idx) {
  const TrieView &t = c.p->trie;
  const double tt = c.p->token_threshold, st = c.p->sent_threshold;
  const uint32_t lane = threadIdx.x & 31;
  // Labels are the first word of each 16-byte record.
  const uint32_t *labs = reinterpret_cast<const uint32_t *>(t.node + c0);
  uint32_t x[kItemsPerLane], pos[kItemsPerLane], child[kItemsPerLane];
  uint4 rec[kItemsPerLane];
  bool on[kItemsPerLane];
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    const uint32_t m = first_item + 32u * k + lane;
    on[k] = false;
    x[k] = 0;
    pos[k] = 0;
    if (m < c.row.K) {
      const double lp = (double)c.row.lp[m];
      x[k] = c.row.id[m];
      on[k] = !(lp <= tt || score + lp <= st);
    }
  }
  // Branch-free lower bounds in lockstep: every item of the task searches the
  // same d labels, so all take the same number of steps.
  for (uint32_t n = d; n > 1;) {
    const uint32_t half = n >> 1;
    uint32_t v[kItemsPerLane];
#pragma unroll
    for (uint32_t k = 0; k < kItemsPerLane; ++k) v[k] = __ldg(labs + 4u * (pos[k] + half - 1));
#pragma unroll
    for (uint32_t k = 0; k < kItemsPerLane; ++k) pos[k] = v[k] < x[k] ? pos[k] + half : pos[k];
    n -= half;
  }
#pragma unroll
  for (uint32_t k = 0; k < kItemsPerLane; ++k) {
    child[k] = 0;
    rec[k] = make_uint4(0, 0, 0, 0);
    if (on[k] && d > 0) {
      uint32_t q = pos[k];
      if (__ldg(labs + 4u * q) < x[k]) ++q;
      if (q < d && __ldg(labs + 4u * q) == x[k]) child[k] = c0 + q;
    }
    if (child[k] != 0) rec[k] = __ldg(t.node + child[k]);
  }
  emit_task<kHelp>(c, score, parent_idx, child, rec, [&](auto &&fn) {
#pragma unroll
    for (uint32_t k = 0; k < kItemsPerLane; ++k)
      if (child[k] != 0) fn(k, first_item + 32u * k + lane);
  });
}

// Branching beams, per chunk of parents: every CTA builds the same task table
// of (parent, 128 items) and the team's warps drain it, each task doing its
// lookups and the gathers of what they found.  A heavy parent is spread over
// every warp of the team; no team barrier is needed between chunks.
// Task `task` of the current chunk: its parent (the last one whose first
// task is <= task).
__device__ __forceinline__ uint32_t task_parent(const BranchTable &bt, uint32_t m, uint32_t task) {
  uint32_t lo = 0, n = m;
  while (n > 1) {
    const uint32_t half = n >> 1;
    if (bt.start[lo + half] <= task) {
      lo += half;
      n -= half;
    } else {
      n = half;
    }
  }
  return lo;
}

// Builds the task table of one chunk of m branching parents starting at
// c_first (every CTA builds the same one): per parent its child range, mode
// and first task.  Returns the chunk's task count.
__device__ uint32_t build_table(const Ctx &c, const BranchTable &bt, uint32_t c_first, uint32_t m) {
  const TrieView &t = c.p->trie;
  const uint32_t K = c.row.K;
  const uint32_t beam_cap = c.p->beam_cap;
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
      // The beam carries its node's child range and flags.
      const uint32_t c0 = b.c0;
      uint32_t d = b.dw & kFanoutMask;
      if (d == kFanoutMask) {
        const uint32_t end = (uint64_t)b.node + 1 < t.num_nodes ? __ldg(t.node + b.node + 1).z
                                                               : (uint32_t)t.num_nodes;
        d = end > c0 ? end - c0 : 0;
      }
      if ((uint64_t)c0 + d > t.num_nodes) {
        atomicOr(c.p->status, kStatusNodeBounds);
        d = 0;
      }
      const uint32_t f = rec_flags(b.dw);
      const uint32_t mode = pick_mode(d, K, f);
      const uint32_t items = (d == 0) ? 0u : (mode == kModeScan ? d : K);
      info = make_uint4(c0, d, b.off, mode | ((f >> 3) << 8));
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
  return c.S->n_tasks;
}

// One task of the chunk (called by all 32 lanes of a warp).
template <bool kHelp>
__device__ __forceinline__ void run_task(const Ctx &c, const BranchTable &bt, uint32_t c_first, uint32_t m,
                                         uint32_t task) {
  const uint32_t lo = task_parent(bt, m, task);
  const uint4 info = bt.info[lo];
  const double score = bt.score[lo];
  const uint32_t first_item = (task - bt.start[lo]) * kTaskItems;
  const uint32_t mode = info.w & 0xFFu;
  const uint32_t parent_idx = c.p->beam_cap - 1 - (c_first + lo);
  if (mode == kModeScan) {
    task_scan<kHelp>(c, info.x, info.y, first_item, score, parent_idx);
  } else if (mode == kModeHash) {
    task_hash<kHelp>(c, info.z, info.w >> 8, first_item, score, parent_idx);
  } else {
    task_bin<kHelp>(c, info.x, info.y, first_item, score, parent_idx);
  }
}

__device__ __forceinline__ uint32_t vld(const uint32_t *p) { return *reinterpret_cast<const volatile uint32_t *>(p); }
__device__ __forceinline__ unsigned long long vld64(const unsigned long long *p) {
  return *reinterpret_cast<const volatile unsigned long long *>(p);
}
__device__ __forceinline__ void vst(uint32_t *p, uint32_t v) { *reinterpret_cast<volatile uint32_t *>(p) = v; }
__device__ __forceinline__ void vst64(unsigned long long *p, unsigned long long v) {
  *reinterpret_cast<volatile unsigned long long *>(p) = v;
}

// Branching beams of a step, chunk by chunk (kParentChunk parents each).
// Every warp runs task `wid` first (no wait); the tasks beyond the team's
// warps are handed out on demand from the team's counter: a warp asks for its
// next task before it runs the current one, so the round trip overlaps the
// task, and a warp that drew cheap tasks takes more.  Later chunks (beam
// widths above 1024) go round-robin.
// A step opened to helper clusters (c.help, helper instance): all tasks of the
// first chunk come from the step's claim counter in the HelpState, shared by
// the leader team's CTAs (which wait until rank 0 has armed the step) and the
// helpers' (which run only this chunk, started after the step's `go`).  Each
// warp counts the tasks it ran into `done` (a helper after publishing its key
// ranges, behind a fence); rank 0 of the leader then waits until every task
// handed out has finished.  A claim at or beyond the task count ends a warp's
// share; a helper that started late may have built its table from a later
// step's beams, so it bounds claims by the count the leader published, once
// known (before then the step is open and its table is right).
template <bool kHelp>
__device__ void expand_branch(const Ctx &c, const BranchTable &bt) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t n_br = c.S->n_br;
  const uint32_t team_warps = c.cs * kWarps;
  const uint32_t wid = c.rank * kWarps + (threadIdx.x >> 5);
  const bool helper = c.T == nullptr;
  for (uint32_t c_first = 0; c_first < n_br; c_first += kParentChunk) {
    const uint32_t m = min(kParentChunk, n_br - c_first);
    const uint32_t total = build_table(c, bt, c_first, m);
    const bool claimed = kHelp && c.help && c_first == 0;
    const uint32_t lim = total;
    if (kHelp && claimed) {
      if (threadIdx.x == 0 && !helper) {
        // Claim only once this CTA sees the step armed (bounded wait).
        const unsigned long long deadline = global_ns() + kHelpWaitNs;
        while (vld(help_word(c.help, kHelpArm, c.step)) != c.S->help_epoch) {
          if (global_ns() > deadline) {
            atomicOr(c.p->status, kStatusHelp);
            break;
          }
          __nanosleep(32);
        }
        __threadfence();
        if (c.rank == 0) vst(help_word(c.help, kHelpTotal, c.step), total);
      }
      __syncthreads();
    }
    const uint32_t n_dyn = (!claimed && c_first == 0 && total > team_warps) ? total - team_warps : 0u;
    uint32_t task = wid;
    if (kHelp && claimed) {
      uint32_t v = 0;
      if (lane == 0) {
        v = atomicAdd(help_word(c.help, kHelpClaim, c.step), 1u);
        if (helper) {
          const uint32_t pt = vld(help_word(c.help, kHelpTotal, c.step));
          if (pt != 0xFFFFFFFFu && v >= pt) v = 0xFFFFFFFFu;
        }
      }
      task = __shfl_sync(0xFFFFFFFFu, v, 0);
    }
    uint32_t mine = 0;
    while (task < lim) {
      uint32_t nxt = 0xFFFFFFFFu;
      if (lane == 0) {
        if (kHelp && claimed) {
          nxt = atomicAdd(help_word(c.help, kHelpClaim, c.step), 1u);
        } else if (n_dyn) {
          nxt = atomicAdd(&c.xc->task_next, 1u);
        }
      }
      run_task<kHelp>(c, bt, c_first, m, task);
      ++mine;
      if (kHelp && claimed) {
        if (helper && lane == 0) {
          const uint32_t pt = vld(help_word(c.help, kHelpTotal, c.step));
          if (pt != 0xFFFFFFFFu && nxt >= pt) nxt = 0xFFFFFFFFu;
        }
        task = __shfl_sync(0xFFFFFFFFu, nxt, 0);
      } else if (n_dyn) {
        const uint32_t v = __shfl_sync(0xFFFFFFFFu, nxt, 0);
        task = v < n_dyn ? team_warps + v : total;
      } else {
        task += team_warps;
      }
    }
    if (kHelp && claimed) {
      if (helper) {
        publish_ranges(c);
        __threadfence();
        __syncwarp();
      }
      if (lane == 0 && mine) atomicAdd(help_word(c.help, kHelpDone, c.step), mine);
      if (!helper && c.rank == 0 && threadIdx.x == 0) {
        const unsigned long long deadline = global_ns() + kHelpWaitNs;
        while (vld(help_word(c.help, kHelpDone, c.step)) < total) {
          if (global_ns() > deadline) {
            atomicOr(c.p->status, kStatusHelp);
            break;
          }
          __nanosleep(32);
        }
        __threadfence();
      }
    }
    __syncthreads();  // the task table is rebuilt for the next chunk
  }
}

// The f64 whose orderable() image is w0 (-0.0 comes back as +0.0).
__device__ __forceinline__ double key_value(uint64_t w0) {
  const uint64_t u = (w0 >> 63) ? (w0 & 0x7FFFFFFFFFFFFFFFull) : ~w0;
  return __longlong_as_double((long long)u);
}

// Bin of `key` in a value pass: floor((v - lo) * scale) of its first word's
// value, clamped to the radix bins.  Non-decreasing in the key.  Rounded
// explicitly (no fused multiply-add), so that every thread that bins the same
// key gets the same bin.
__device__ __forceinline__ uint32_t value_bin(const Key3 &key, double lo, double scale) {
  const double x = __dmul_rn(__dsub_rn(key_value(key.w[0]), lo), scale);
  if (!(x >= 0.0)) return 0;
  if (x >= (double)(kRadixBins - 1)) return kRadixBins - 1;
  return (uint32_t)x;
}

constexpr int kPassBits = 0;       // `width` key bits at `from_top`, keys matching P under M
constexpr int kPassValue = 1;      // value bins of every key
constexpr int kPassBitsInBin = 2;  // as kPassBits, among the keys in value bin `bin`
// Value passes are used when the keys share fewer leading bits than this:
// then a bit pass would mostly separate binades (sign and exponent bits).
constexpr int kValuePassMaxCommon = 24;

// One radix pass of a selection.
struct RadixPass {
  Key3 P, M;
  int from_top, width;
  int kind;
  uint32_t bin;
  double lo, scale;
};

// Counts `key` in its bin of the current pass if it takes part in it.
__device__ __forceinline__ void hist_add(const Key3 &key, const RadixPass &rp, uint32_t *hist) {
  if (rp.kind == kPassValue) {
    atomicAdd(&hist[value_bin(key, rp.lo, rp.scale)], 1u);
    return;
  }
  if ((key.w[0] & rp.M.w[0]) == rp.P.w[0] && (key.w[1] & rp.M.w[1]) == rp.P.w[1] &&
      (key.w[2] & rp.M.w[2]) == rp.P.w[2] &&
      (rp.kind != kPassBitsInBin || value_bin(key, rp.lo, rp.scale) == rp.bin))
    atomicAdd(&hist[key_bits(key, rp.from_top, rp.width)], 1u);
}

// ------------------------------------------------------------- selection
// Exact top-k threshold over n candidates by the 192-bit key, computed by the
// whole team with one cluster barrier per radix pass.  Each CTA histograms
// its share of the keys that match the current prefix into its own shared
// memory (2048 bins, buffer pass % 2) and sums them into 64 super-bins.  After
// the barrier every CTA derives the same digit from the team's histograms:
// warp r reads rank r's super-bins (one DSMEM load per lane, all ranks in
// parallel), warp 0 sums and scans them; then the same for the 32 bins of the
// super-bin that holds the rem-th key.  Nothing is merged with atomics.
// `start` leading bits of the first key word are common to all n keys (equal
// to those of common_hi << 32); the top 32 bits of every first key word lie
// in [common_hi, key_hi].  On return every CTA's LocalState holds the
// threshold: with sel_ge every key >= sel_prefix is taken (exactly k of them),
// otherwise keys > sel_prefix plus sel_rem keys equal to it.
// With `value_first` and a short common prefix, the first pass is a value
// pass: 2048 bins linear in the first word's value over the keys' range, so
// that the threshold bin usually holds a few keys (a bit pass there would
// mostly separate binades).  When that bin holds exactly the keys still
// needed, the selection ends; otherwise bit passes continue among the keys of
// that bin, from the leading bits its value range shares (the range is
// widened by a whole bin on each side, far beyond the rounding of the bin
// arithmetic, which is below 2^-40 of a bin here).
// `add_keys(pass, hist)` histograms (hist_add) this thread's keys, from
// memory or from registers.
template <class AddKeys>
__device__ void team_radix_select(const Ctx &c, uint32_t k, int start, uint32_t common_hi, uint32_t key_hi,
                                  bool value_first, AddKeys &&add_keys) {
  LocalState *S = c.S;
  const uint32_t cs = c.cs;
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // this CTA may still be testing keys against the previous threshold
  if (threadIdx.x == 0) {
    const uint64_t m0 = start >= 32 ? 0xFFFFFFFF00000000ull : (start == 0 ? 0ull : ~0ull << (64 - start));
    S->sel_prefix = Key3{{((uint64_t)common_hi << 32) & m0, 0, 0}};
    S->sel_mask = Key3{{m0, 0, 0}};
    S->sel_rem = k;
    S->sel_ge = 0;
    S->sel_in_bin = 0;
    S->sel_value = 0;
    S->sel_bin = 0;
    S->sel_lo = 0.0;
    S->sel_scale = 0.0;
    if (value_first && start < kValuePassMaxCommon) {
      // Every key's value lies in [lo, hi] (orderable() is monotone).
      const double lo = key_value((uint64_t)common_hi << 32);
      const double hi = key_value(((uint64_t)key_hi << 32) | 0xFFFFFFFFull);
      const double scale = (double)kRadixBins / (hi - lo);
      if (hi > lo && scale > 0.0 && scale < 1e300) {
        S->sel_lo = lo;
        S->sel_scale = scale;
        S->sel_value = 1;
      }
    }
  }
  __syncthreads();
  bool value = S->sel_value != 0;
  for (int from_top = start; value || from_top < kKeyBits;) {
    const int width = value ? kRadixBits : min(kRadixBits, kKeyBits - from_top);
    const uint32_t buf = S->pass & 1u;
    uint32_t *hist = S->hist[buf];
    uint32_t *super = S->super[buf];
    RadixPass rp;
    rp.P = S->sel_prefix;
    rp.M = S->sel_mask;
    rp.from_top = from_top;
    rp.width = width;
    rp.kind = value ? kPassValue : (S->sel_in_bin ? kPassBitsInBin : kPassBits);
    rp.bin = S->sel_bin;
    rp.lo = S->sel_lo;
    rp.scale = S->sel_scale;
    add_keys(rp, hist);
    __syncthreads();
    {
      // Super-bin sums: thread i sums bins 4i..4i+3; 8 lanes make a super-bin.
      const uint4 q = *reinterpret_cast<const uint4 *>(hist + 4 * threadIdx.x);
      uint32_t s4 = q.x + q.y + q.z + q.w;
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 1);
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 2);
      s4 += __shfl_xor_sync(0xFFFFFFFFu, s4, 4);
      if ((threadIdx.x & 7) == 0) super[threadIdx.x >> 3] = s4;
    }
    team_sync(cs);
    {
      // The other buffer was last read (over DSMEM) before the barrier above:
      // clear it for the next pass, which the barriers below order before
      // that pass's adds.
      uint32_t *other = S->hist[buf ^ 1u];
      for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) other[b] = 0;
    }
    uint32_t *part = S->part;
    if (warp < cs) {
      const uint2 pv = *reinterpret_cast<const uint2 *>(cluster.map_shared_rank(super, warp) + 2 * lane);
      *reinterpret_cast<uint2 *>(part + warp * kSuperBins + 2 * lane) = pv;
    }
    __syncthreads();
    if (warp == 0) {
      const uint32_t rem = S->sel_rem;
      // Lane l holds super-bins 63-2l (upper) and 62-2l (lower).
      uint32_t hi_s = 0, lo_s = 0;
      // Unrolled so that the team's loads are all in flight at once.
#pragma unroll
      for (uint32_t r = 0; r < kMaxTeam; ++r) {
        if (r < cs) {
          const uint2 pv = *reinterpret_cast<const uint2 *>(part + r * kSuperBins + kSuperBins - 2 - 2 * lane);
          hi_s += pv.y;
          lo_s += pv.x;
        }
      }
      uint32_t inc = hi_s + lo_s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= (uint32_t)o) inc += y;
      }
      const uint32_t excl = inc - hi_s - lo_s;
      const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
      const uint32_t who = __ffs(__ballot_sync(0xFFFFFFFFu, excl < rem && rem <= inc));  // 1-based, 0 if none
      uint32_t sb = 0xFFFFFFFFu, sb_above = 0;
      if (who != 0 && total >= rem) {
        const uint32_t w = who - 1;
        const uint32_t e = __shfl_sync(0xFFFFFFFFu, excl, w);
        const uint32_t h = __shfl_sync(0xFFFFFFFFu, hi_s, w);
        const bool upper = rem <= e + h;
        sb = upper ? kSuperBins - 1 - 2 * w : kSuperBins - 2 - 2 * w;
        sb_above = upper ? e : e + h;
      }
      if (lane == 0) {
        S->sel_sb = sb;
        S->sel_above = sb_above;
      }
    }
    __syncthreads();
    const uint32_t sb = S->sel_sb;
    if (sb != 0xFFFFFFFFu && warp < cs) part[warp * 32 + lane] = cluster.map_shared_rank(hist, warp)[sb * 32 + 31 - lane];
    __syncthreads();
    if (warp == 0) {
      const uint32_t rem = S->sel_rem;
      uint32_t digit = 0xFFFFFFFFu, above = 0, count = 0;
      if (sb != 0xFFFFFFFFu) {
        // Lane l holds bin sb*32 + 31 - l (descending).
        uint32_t bv = 0;
#pragma unroll
        for (uint32_t r = 0; r < kMaxTeam; ++r)
          if (r < cs) bv += part[r * 32 + lane];
        uint32_t binc = bv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, binc, o);
          if (lane >= (uint32_t)o) binc += y;
        }
        const uint32_t bexcl = binc - bv;
        const uint32_t sb_above = S->sel_above;
        const uint32_t need = rem - sb_above;
        const uint32_t who2 = __ffs(__ballot_sync(0xFFFFFFFFu, bexcl < need && need <= binc));
        if (who2 != 0) {
          const uint32_t w2 = who2 - 1;
          digit = sb * 32 + 31 - w2;
          above = sb_above + __shfl_sync(0xFFFFFFFFu, bexcl, w2);
          count = __shfl_sync(0xFFFFFFFFu, bv, w2);
        }
      }
      if (lane == 0) {
        S->pass += 1;
        if (digit == 0xFFFFFFFFu) {
          // Fewer keys match the prefix than remain to be taken: the key range
          // was wrong.  Report it and take everything at or above the prefix.
          atomicOr(c.p->status, kStatusSelection);
          S->sel_ge = 1;
        } else if (value) {
          S->sel_in_bin = 1;
          S->sel_bin = digit;
          S->sel_rem = rem - above;
          if (count == S->sel_rem) {
            // Every key of the bin is taken.
            S->sel_ge = 1;
            S->sel_prefix = Key3{{0, 0, 0}};
            S->sel_mask = Key3{{0, 0, 0}};
          } else {
            const double w = 1.0 / S->sel_scale;
            const uint64_t a = orderable(S->sel_lo + ((double)digit - 1.0) * w);
            const uint64_t b = orderable(S->sel_lo + ((double)digit + 2.0) * w);
            const int s2 = a == b ? 64 : __clzll((long long)(a ^ b));
            const uint64_t m = s2 == 0 ? 0ull : (s2 >= 64 ? ~0ull : ~0ull << (64 - s2));
            S->sel_prefix = Key3{{a & m, 0, 0}};
            S->sel_mask = Key3{{m, 0, 0}};
            S->sel_next = s2;
          }
        } else {
          S->sel_rem = rem - above;
          key_set_bits(S->sel_prefix, from_top, width, digit);
          key_set_bits(S->sel_mask, from_top, width, low_mask(width));
          if (count == S->sel_rem) S->sel_ge = 1;
        }
      }
    }
    __syncthreads();
    if (S->sel_ge) break;
    if (value) {
      from_top = S->sel_next;
      value = false;
    } else {
      from_top += kRadixBits;
    }
  }
}

// Is `key` among the selected?  Equal keys beyond the threshold count are
// indistinguishable beams, so which of them are taken does not matter.
__device__ __forceinline__ bool is_selected(const Ctx &c, const Key3 &key, uint32_t *eq_taken) {
  if (c.S->sel_in_bin) {
    const uint32_t b = value_bin(key, c.S->sel_lo, c.S->sel_scale);
    if (b != c.S->sel_bin) return b > c.S->sel_bin;
  }
  const int r = key_cmp(key, c.S->sel_prefix);
  if (c.S->sel_ge) return r >= 0;  // the prefix has its free bits at zero
  if (r > 0) return true;
  if (r < 0) return false;
  return atomicAdd(eq_taken, 1u) < c.S->sel_rem;
}

__device__ __forceinline__ int common_bits(uint32_t lo, uint32_t hi) {
  return lo == hi ? 32 : __clz((int)(lo ^ hi));
}

// Appends a selected candidate to the beams of step t+1 and its history.
// In-link beams fill the buffer from the front, branching beams from the
// back; the capped total keeps the two from overlapping.  The converged
// threads reserve together: one thread issues the three counter atomics back
// to back (one round trip) for all of them.
template <bool kCount>
__device__ __forceinline__ void take_beam(const Ctx &c, const Cand &v, uint32_t k, Beam *out_beams, Hist *hist) {
  const uint32_t act = __activemask();
  const uint32_t lane = threadIdx.x & 31;
  const bool link = rec_flags(v.dw) & kNodeFlagLink;
  const uint32_t m_in = __ballot_sync(act, link);
  const uint32_t m_br = act & ~m_in;
  const uint32_t leader = __ffs(act) - 1;
  uint32_t n_tasks = 0;
  if (kCount) {
    // This beam's branch tasks at the next step, as the task table will
    // count them (an escaped fan-out is large: one task per 128 proposals).
    const uint32_t d = v.dw & kFanoutMask, K = c.row.K;
    const uint32_t items = (link || d == 0) ? 0u : (d <= 2u * K + 32u ? d : K);
    n_tasks = __reduce_add_sync(act, (items + kTaskItems - 1) / kTaskItems);
  }
  uint32_t b_sel = 0, b_in = 0, b_br = 0;
  if (lane == leader) {
    b_sel = atomicAdd(&c.cnt->n_sel, (uint32_t)__popc(act));
    if (m_in) b_in = atomicAdd(&c.cnt->n_in_new, (uint32_t)__popc(m_in));
    if (m_br) b_br = atomicAdd(&c.cnt->n_br_new, (uint32_t)__popc(m_br));
    if (n_tasks) atomicAdd(&c.cnt->n_tasks_new, n_tasks);
  }
  b_sel = __shfl_sync(act, b_sel, leader);
  b_in = __shfl_sync(act, b_in, leader);
  b_br = __shfl_sync(act, b_br, leader);
  const uint32_t below = (1u << lane) - 1u;
  if (b_sel + (uint32_t)__popc(act & below) >= k) {
    atomicOr(c.p->status, kStatusSelection);
    return;
  }
  const uint32_t beam_cap = c.p->beam_cap;
  const uint32_t j = link ? b_in + __popc(m_in & below) : b_br + __popc(m_br & below);
  if (j >= beam_cap) {
    atomicOr(c.p->status, kStatusSelection);
    return;
  }
  const uint32_t idx = link ? j : beam_cap - 1 - j;
  Beam b;
  b.score = v.score;
  b.node = v.node;
  b.off = v.aux;
  b.c0 = v.c0;
  b.dw = v.dw;
  out_beams[idx] = b;
  hist[idx] = Hist{v.parent, v.token};
}

// Makes the selected candidates the beams of step t+1 (kCount: and sums their
// branch tasks for the next step, when c.count_tasks).
template <bool kCount>
__device__ void materialize_next(const Ctx &c, uint32_t n, uint32_t k, Beam *out_beams) {
  const uint32_t depth = c.step + 1;
  const double f = c.p->factor[depth];
  if (k == 0) return;
  const Cand *next = c.slot.next;
  Hist *hist = c.slot.hist + (uint64_t)depth * c.p->beam_cap;
  const int start = common_bits(c.S->key_min, c.S->key_max);
  if (n > k && n <= c.gthreads()) {
    // One candidate per thread at most: it stays in registers through every
    // radix pass and the final test, so nothing is read twice.
    const uint32_t i = c.gtid();
    const bool have = i < n;
    Cand v = {};
    Key3 key = {};
    if (have) {
      v = ld_cand(next + i);
      key = cand_key(v, f, depth);
    }
    team_radix_select(c, k, start, c.S->key_min, c.S->key_max, true, [&](const RadixPass &rp, uint32_t *h) {
      if (have) hist_add(key, rp, h);
    });
    if (have && is_selected(c, key, &c.cnt->eq_taken)) take_beam<kCount>(c, v, k, out_beams, hist);
    return;
  }
  const bool all = n <= k;
  const uint32_t G = c.gthreads();
  if (!all)
    team_radix_select(c, k, start, c.S->key_min, c.S->key_max, true, [&](const RadixPass &rp, uint32_t *h) {
      // Four candidates' loads in flight before any is counted.
      uint32_t i = c.gtid();
      for (; i + 3 * G < n; i += 4 * G) {
        uint4 a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = ld_cand_head(next + i + u * G);
#pragma unroll
        for (int u = 0; u < 4; ++u) hist_add(head_key(a[u], f, depth), rp, h);
      }
      for (; i < n; i += G) hist_add(head_key(ld_cand_head(next + i), f, depth), rp, h);
    });
  for (uint32_t i = c.gtid(); i < n; i += G) {
    const uint4 a = ld_cand_head(next + i);
    if (!all && !is_selected(c, head_key(a, f, depth), &c.cnt->eq_taken)) continue;
    take_beam<kCount>(c, cand_from(a, next + i), k, out_beams, hist);
  }
}

// Writes the best k of the n pool entries to pool_tmp (the team's
// n_compact counts them).
__device__ void trim_pool(const Ctx &c, uint32_t n, uint32_t k) {
  const Cand *pool = c.slot.pool;
  const double *factor = c.p->factor;
  const uint32_t max_depth = c.step + 1;
  team_radix_select(c, k, common_bits(c.S->pool_key_min, c.S->pool_key_max), c.S->pool_key_min,
                    c.S->pool_key_max, true, [&](const RadixPass &rp, uint32_t *h) {
                      for (uint32_t i = c.gtid(); i < n; i += c.gthreads()) {
                        const Cand cv = ld_cand(pool + i);
                        const uint32_t d = min(cv.aux, max_depth);
                        hist_add(cand_key(cv, factor[d], d), rp, h);
                      }
                    });
  for (uint32_t i = c.gtid(); i < n; i += c.gthreads()) {
    const Cand v = ld_cand(c.slot.pool + i);
    if (v.aux == 0 || v.aux > c.step + 1) {
      report(c, 4, i, v.aux, c.step);
      continue;
    }
    if (!is_selected(c, cand_key(v, c.p->factor[v.aux], v.aux), &c.T->eq_taken_trim)) continue;
    const uint32_t j = append_slot(&c.T->n_compact);
    if (j < k) c.slot.pool_tmp[j] = v;
  }
}

// Sorts the final pool (descending) and writes the ascending result (rank 0).
// With p.tok_total set, each request's tokens are written contiguously (beam
// by beam in output order) at an offset it reserves from that counter, stored
// in p.out_tok_base; otherwise beam o of request r starts at slot (r*cap + o)
// of p.out_tok with stride p.out_stride.
__device__ void write_result(const SearchParams &p, const SlotView &slot, const Cand *pool, uint32_t n, uint32_t req,
                             uint8_t *dyn, LocalState *S) {
  uint32_t P2 = 1;
  while (P2 < n) P2 <<= 1;
  ulonglong2 *items = reinterpret_cast<ulonglong2 *>(dyn);
  for (uint32_t i = threadIdx.x; i < P2; i += blockDim.x) {
    ulonglong2 it = make_ulonglong2(0, 0);
    if (i < n) {
      const Cand v = ld_cand(pool + i);
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
  const bool compact = p.tok_total != nullptr;
  uint64_t tok_base = 0;
  if (compact) {
    // Output beam o = n-1-s starts after the tokens of every beam s' > s.
    // items[s].x (the sort key, no longer needed) takes the length, then
    // the offset.
    for (uint32_t s = threadIdx.x; s < n; s += blockDim.x) {
      const uint32_t d = ld_cand(pool + (uint32_t)(items[s].y & 0xFFFFu)).aux;
      items[s].x = (d == 0 || d > stride) ? 0 : d;
    }
    __syncthreads();
    const uint32_t per = (n + blockDim.x - 1) / blockDim.x;
    const uint32_t s0 = min(n, threadIdx.x * per), s1 = min(n, s0 + per);
    uint32_t mine = 0;
    for (uint32_t s = s0; s < s1; ++s) mine += (uint32_t)items[s].x;
    uint32_t run = block_exclusive_sum(mine, S);
    if (threadIdx.x == blockDim.x - 1) S->out_total = run + mine;  // the request's token total
    __syncthreads();
    const uint32_t total = S->out_total;
    for (uint32_t s = s0; s < s1; ++s) {
      const uint32_t len = (uint32_t)items[s].x;
      items[s].x = total - run - len;
      run += len;
    }
    if (threadIdx.x == 0) {
      const uint64_t b = total ? atomicAdd(reinterpret_cast<unsigned long long *>(p.tok_total), (unsigned long long)total) : 0ull;
      p.out_tok_base[req] = b;
      S->out_base = b;
    }
    __syncthreads();
    tok_base = S->out_base;
  }
  for (uint32_t s = threadIdx.x; s < n; s += blockDim.x) {
    const uint32_t idx = (uint32_t)(items[s].y & 0xFFFFu);
    const Cand v = ld_cand(pool + idx);
    const uint32_t o = n - 1 - s;
    const uint64_t slot_o = (uint64_t)req * cap + o;
    uint32_t depth = v.aux;
    if (depth == 0 || depth > stride) {
      atomicOr(p.status, kStatusSelection);
      depth = 0;
    }
    p.out_lpn[slot_o] = depth ? v.score * p.factor[depth] : 0.0;
    p.out_len[slot_o] = depth;
    if (p.out_key)
      p.out_key[slot_o] = (uint64_t)v.node < p.trie.num_nodes ? key_id(p.trie, v.node) : 0xFFFFFFFFu;
    uint32_t *tok = compact ? p.out_tok + tok_base + items[s].x : p.out_tok + slot_o * stride;
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

// Stages a row of the caller's top-k arrays in shared memory, ordered by
// (id, original column): rows already in non-decreasing id order are copied
// (equal ids keep their column order), others are bitonic-sorted through
// `scratch` (P2(K) u64 keys, the task table's space).
__device__ void stage_row(const SearchParams &p, const RowView &row, uint64_t rbase, uint64_t *scratch) {
  const uint32_t K = row.K;
  const uint32_t *gid = p.topk_id + rbase;
  const float *glp = p.topk_logp + rbase;
  bool ok = true;
  for (uint32_t j = threadIdx.x; j < K; j += blockDim.x) {
    const uint32_t id = __ldg(gid + j);
    row.id[j] = id;
    row.lp[j] = __ldg(glp + j);
    row.orig[j] = j;
    if (j + 1 < K && id > __ldg(gid + j + 1)) ok = false;
  }
  if (__syncthreads_and(ok)) return;
  uint32_t P2 = 1;
  while (P2 < K) P2 <<= 1;
  for (uint32_t j = threadIdx.x; j < P2; j += blockDim.x)
    scratch[j] = j < K ? (((uint64_t)row.id[j] << 32) | j) : ~0ull;
  __syncthreads();
  for (uint32_t kk = 2; kk <= P2; kk <<= 1) {
    for (uint32_t j = kk >> 1; j > 0; j >>= 1) {
      for (uint32_t i = threadIdx.x; i < P2; i += blockDim.x) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = scratch[i], b = scratch[ixj];
          const bool up = (i & kk) == 0;
          if ((a > b) == up) {
            scratch[i] = b;
            scratch[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (uint32_t j = threadIdx.x; j < K; j += blockDim.x) {
    const uint32_t o = (uint32_t)(scratch[j] & 0xFFFFFFFFu);
    row.id[j] = (uint32_t)(scratch[j] >> 32);
    row.lp[j] = __ldg(glp + o);
    row.orig[j] = o;
  }
  __syncthreads();
}

__device__ void reset_counters(StepCounters *s) {
  s->n_sel = 0;
  s->n_in_new = 0;
  s->n_br_new = 0;
  s->eq_taken = 0;
  s->n_tasks_new = 0;
}

__device__ void reset_exp(ExpCounters *x) {
  x->n_next = 0;
  x->key_min = 0xFFFFFFFFu;
  x->key_max = 0;
  x->task_next = 0;
}

__device__ void reset_pool(PoolCounters *x) {
  x->pool_end = 0;
  x->pool_key_min = 0xFFFFFFFFu;
  x->pool_key_max = 0;
}

// One request, searched by the whole team.  Cluster barriers per step: one
// after expansion, one per radix pass of the selection, one after the next
// beams are written (plus the passes of a pool trim when the next step could
// overflow the pool).
// Splits the dynamic shared memory into the staged row and the task table.
__device__ __forceinline__ void carve(uint8_t *dyn, uint32_t K, RowView &row, BranchTable &bt) {
  row.id = reinterpret_cast<uint32_t *>(dyn);
  row.lp = reinterpret_cast<float *>(dyn + sizeof(uint32_t) * K);
  row.orig = reinterpret_cast<uint32_t *>(dyn + 2 * sizeof(uint32_t) * K);
  row.K = K;
  uint8_t *tb = dyn + ((12u * K + 15u) & ~15u);
  bt.info = reinterpret_cast<uint4 *>(tb);
  bt.score = reinterpret_cast<double *>(tb + sizeof(uint4) * kParentChunk);
  bt.start = reinterpret_cast<uint32_t *>(tb + (sizeof(uint4) + sizeof(double)) * kParentChunk);
}

// `epoch` names this request of this launch; `kord` is the request's
// ordinal among its slot's requests in this launch (helper bookkeeping).
template <bool kHelp>
__device__ void search_request(const SearchParams &p, uint32_t req, const SlotView &slot, TeamState *T,
                               LocalState *S, uint32_t rank, uint32_t cs, uint8_t *dyn, uint32_t epoch,
                               uint32_t kord) {
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
    const uint4 r = __ldg(p.trie.node);  // the root (node 0) is never a link node
    Beam root;
    root.score = 0.0;
    root.node = 0;
    root.off = r.y;
    root.c0 = r.z;
    root.dw = r.w;
    slot.beams[0][beam_cap - 1] = root;
    reset_counters(&T->cnt[0]);
    reset_counters(&T->cnt[1]);
    reset_exp(&T->xc[0]);
    reset_exp(&T->xc[1]);
    reset_pool(&T->pool);
    T->n_compact = 0;
    T->eq_taken_trim = 0;
    T->removed = 0;
  }
  // Helper clusters: the counters they share live in the slot's HelpState.
  // Its per-step words are re-armed only when every helper of this slot's
  // previous request in this launch has left that request (bounded wait; a
  // launch's first request has none, and every earlier launch has ended).
  // The HelpState's counters are clear between open steps (set so at
  // allocation, cleared by the leader after each open step); a step's claim,
  // done and total words are re-armed when the step opens.
  HelpState *const H = (kHelp && p.helpers && slot.help) ? slot.help : nullptr;
  if (H && leader && kord > 0) {
    __threadfence();
    const uint32_t q = (kord & 1u) ^ 1u;
    const unsigned long long deadline = global_ns() + kHelpWaitNs;
    while (vld(&H->left[q]) != vld(&H->joined[q])) {
      if (global_ns() > deadline) {
        atomicOr(p.status, kStatusHelp);
        break;
      }
      __nanosleep(32);
    }
  }
  if (threadIdx.x == 0) S->help_epoch = epoch;
  if (threadIdx.x == 0) S->pass = 0;
  // Both histogram buffers start clear; afterwards each pass clears the
  // buffer of the pass after it (team_radix_select).
  for (uint32_t b = threadIdx.x; b < 2 * kRadixBins; b += blockDim.x) (&S->hist[0][0])[b] = 0;
  RowView row;
  BranchTable bt;
  carve(dyn, K, row, bt);
  team_sync(cs);

  Ctx c;
  c.p = &p;
  c.slot = slot;
  c.T = T;
  c.S = S;
  c.row = row;
  c.rank = rank;
  c.cs = cs;
  c.help = nullptr;
  c.xp = &T->pool;
  if (threadIdx.x == 0) S->pool_add = 0;
  bool trimmed = false;  // the previous step left its pool survivors in pool_tmp
  uint32_t prev_want = 0;
  for (uint32_t t = 0; t < L; ++t) {
    const uint32_t par = t & 1u;
    unsigned long long t0 = 0;
    if (leader) t0 = global_ns();
    c.step = t;
    c.cnt = &T->cnt[par];
    c.xc = &T->xc[par];
    c.help = nullptr;
    if (threadIdx.x == 0) {
      if (t == 0) {
        S->n_in = 0;
        S->n_br = 1;
        S->stop = 0;
      } else {
        // Counters of step t-1 are final after the barrier that closed it.
        const StepCounters *pc = &T->cnt[par ^ 1u];
        const uint32_t sel = pc->n_sel, n_in = pc->n_in_new, n_br = pc->n_br_new;
        S->stop = 0;
        if (sel != prev_want || n_in + n_br != prev_want || (trimmed && T->n_compact != final_beam)) {
          // The beam buffer or the pool is not trustworthy: stop.
          if (rank == 0) report(c, 1, prev_want, sel, n_in + n_br);
          S->stop = 1;
        }
        S->n_in = min(n_in, beam_cap);
        S->n_br = min(n_br, beam_cap - S->n_in);
        S->est_tasks = pc->n_tasks_new;
      }
      S->pool_base = vld(&c.xp->pool_end);
      S->pushes = (unsigned long long)S->pool_base + T->removed;
      // A step whose branching beams bring many tasks (summed by the last
      // selection) is opened to the helpers; every CTA decides alike and
      // rank 0 publishes it.  Its counters move to the HelpState: pool
      // entries go after the pool's end at the step's start (pool_base), the
      // HelpState's pool counter is zero between open steps, and the leader
      // folds it back after the step's expansion barrier.
      const bool go_on = !(S->stop || S->n_in + S->n_br == 0 || (p.early_exit && S->pushes >= final_beam));
      S->help_open = (H && go_on && t > 0 && S->est_tasks >= kHelpMinTasks && t < H->steps) ? 1u : 0u;
      S->pool_add = S->help_open ? S->pool_base : 0u;
      if (S->help_open && rank == 0) {
        // Re-arm the step's words, the arm word last: the team's CTAs claim
        // only once they see it, and by then the other words are visible;
        // helpers see them through the fence before `go`.
        *help_word(H, kHelpClaim, t) = 0;
        *help_word(H, kHelpDone, t) = 0;
        *help_word(H, kHelpTotal, t) = 0xFFFFFFFFu;
        *help_word(H, kHelpNbr, t) = S->n_br;
        H->pool.base = S->pool_base;
        __threadfence();
        vst(help_word(H, kHelpArm, t), epoch);
        __threadfence();
        vst64(&H->go, ((unsigned long long)epoch << 32) | t);
      }
    }
    __syncthreads();
    if (S->help_open) {
      c.help = H;
      c.xc = &H->xc[par];
      c.xp = &H->pool;
    }
    if (trimmed) {
      // Survivors of the previous step's trim go back to the pool's front;
      // this step appends behind them, and the pool is next read after the
      // expansion barrier.
      for (uint32_t i = c.gtid(); i < final_beam; i += c.gthreads()) slot.pool[i] = ld_cand(slot.pool_tmp + i);
      trimmed = false;
    }
    if (S->stop || S->n_in + S->n_br == 0 || (p.early_exit && S->pushes >= final_beam)) break;
    stage_row(p, row, meta.rows_off + (uint64_t)t * K, reinterpret_cast<uint64_t *>(bt.info));
    __syncthreads();
    unsigned long long t1 = 0;
    if (leader) t1 = global_ns();

    c.cur = slot.beams[par];
    c.f_next = p.factor[t + 1];
    c.kmin = c.pkmin = 0xFFFFFFFFu;
    c.kmax = c.pkmax = 0;
    expand_inlink<kHelp>(c);
    expand_branch<kHelp>(c, bt);
    publish_ranges(c);
    team_sync(cs);
    unsigned long long t2 = 0;
    if (leader) t2 = global_ns();

    if (threadIdx.x == 0) {
      S->n_next = min(vld(&c.xc->n_next), (uint32_t)p.cand_cap);
      S->key_min = vld(&c.xc->key_min);
      S->key_max = vld(&c.xc->key_max);
      if (c.help) {
        // An open step's pool entries were counted in the HelpState.
        S->pool_end = min(S->pool_base + vld(&H->pool.pool_end), (uint32_t)p.pool_cap);
        S->pool_key_min = min(vld(&T->pool.pool_key_min), vld(&H->pool.pool_key_min));
        S->pool_key_max = max(vld(&T->pool.pool_key_max), vld(&H->pool.pool_key_max));
      } else {
        S->pool_end = min(vld(&c.xp->pool_end), (uint32_t)p.pool_cap);
        S->pool_key_min = vld(&c.xp->pool_key_min);
        S->pool_key_max = vld(&c.xp->pool_key_max);
      }
    }
    __syncthreads();
    // Every CTA has read step t-1's counters and the last trim's count
    // (before the barrier above).
    if (leader) {
      reset_counters(&T->cnt[par ^ 1u]);
      reset_exp(&T->xc[par ^ 1u]);
      if (c.help) {
        // Every CTA has read the open step's counters (above): fold the
        // pool's into the team's and clear the HelpState's for the next open
        // step.
        T->pool.pool_end = S->pool_end;
        T->pool.pool_key_min = S->pool_key_min;
        T->pool.pool_key_max = S->pool_key_max;
        reset_pool(&H->pool);
        reset_exp(&H->xc[par]);
      }
      T->n_compact = 0;
      T->eq_taken_trim = 0;
    }
    c.xp = &T->pool;
    if (threadIdx.x == 0) S->pool_add = 0;
    const uint32_t n_next = S->n_next, pool_end = S->pool_end;
    materialize_next<kHelp>(c, n_next, beams[t], slot.beams[par ^ 1u]);
    prev_want = min(n_next, beams[t]);
    // Trim the pool only when the next step's appends (at most K per beam)
    // could overflow it.
    if (t + 1 < L && pool_end > final_beam &&
        (uint64_t)pool_end + (uint64_t)prev_want * K > p.pool_cap) {
      trim_pool(c, pool_end, final_beam);
      if (leader) {
        T->removed += pool_end - final_beam;
        c.xp->pool_end = final_beam;
      }
      trimmed = true;
    }
    team_sync(cs);
    if (leader) {
      const unsigned long long t3 = global_ns();
      T->t_ovh += t1 - t0;
      T->t_exp += t2 - t1;
      T->t_sel += t3 - t2;
    }
  }
  // The pool survivors copied back at the last step start must land before
  // the final trim reads the pool.
  team_sync(cs);
  // The helpers are done with this request.
  if (H && leader) vst64(&H->go, ((unsigned long long)epoch << 32) | kHelpStop);
  const unsigned long long t4 = leader ? global_ns() : 0ull;
  if (threadIdx.x == 0) {
    S->pool_end = min(vld(&c.xp->pool_end), (uint32_t)p.pool_cap);
    S->pool_key_min = vld(&c.xp->pool_key_min);
    S->pool_key_max = vld(&c.xp->pool_key_max);
  }
  __syncthreads();
  if (leader) {
    // Every CTA read the last trim's count before the barrier above.
    T->n_compact = 0;
    T->eq_taken_trim = 0;
  }
  const uint32_t n_pool = S->pool_end;
  const Cand *out_pool = slot.pool;
  uint32_t n_out = n_pool;
  if (n_pool > final_beam) {
    c.step = L - 1;  // pool depths are at most L
    trim_pool(c, n_pool, final_beam);
    team_sync(cs);
    out_pool = slot.pool_tmp;
    n_out = final_beam;
    if (threadIdx.x == 0) S->n_next = T->n_compact;
    __syncthreads();
    if (S->n_next != final_beam) {
      if (leader) report(c, 2, n_pool, final_beam, S->n_next);
      n_out = min(S->n_next, final_beam);
    }
  }
  if (rank == 0) {
    write_result(p, slot, out_pool, n_out, req, dyn, S);
    if (threadIdx.x == 0 && p.out_phase_ms) {
      const unsigned long long t5 = global_ns();
      double *ph = p.out_phase_ms + (uint64_t)req * 5;
      ph[0] = T->t_exp * 1e-6;
      ph[1] = 0.0;  // validation is fused into expansion
      ph[2] = (T->t_sel + (t5 - t4)) * 1e-6;
      ph[3] = T->t_ovh * 1e-6;
      ph[4] = (t5 - T->t_start) * 1e-6;
    }
  }
}

// A helper CTA's share of a request: for every step the leader opens (its
// `go` word), stage the step's row, build the same task table from the
// step's beams and run tasks from the step's claim counter; then publish the
// candidates' key ranges and count the tasks done (after a fence, so the
// leader sees the candidates once it sees the count).  Waits are bounded: a
// helper whose leader never opens a step, or is not resident, gives up and
// the leader runs every task itself.  It registers in joined[kpar] before
// reading `go` and in left[kpar] when it leaves.
__device__ void help_request(const SearchParams &p, uint32_t req, const SlotView &slot, LocalState *S,
                             uint8_t *dyn, uint32_t epoch, uint32_t kpar) {
  HelpState *const H = slot.help;
  const ReqMeta meta = p.meta[req];
  const uint32_t L = meta.L, K = meta.K;
  if (threadIdx.x == 0) {
    atomicAdd(&H->joined[kpar], 1u);
    __threadfence();
  }
  RowView row;
  BranchTable bt;
  carve(dyn, K, row, bt);
  Ctx c;
  c.p = &p;
  c.slot = slot;
  c.T = nullptr;
  c.cnt = nullptr;
  c.S = S;
  c.row = row;
  c.rank = 0;
  c.cs = 1;
  c.help = H;
  c.xp = &H->pool;
  if (threadIdx.x == 0) S->help_epoch = epoch;
  uint32_t t_next = 0;
  for (;;) {
    if (threadIdx.x == 0) {
      uint32_t got = kHelpStop;
      const unsigned long long deadline = global_ns() + kHelpWaitNs;
      // Polls back off (up to ~1 us between them): idle helpers must not
      // crowd the L2 slice that holds `go` while their leader works.
      uint32_t nap = 32;
      while (global_ns() < deadline) {
        const unsigned long long g = vld64(&H->go);
        const uint32_t ge = (uint32_t)(g >> 32);
        if (ge == epoch) {
          const uint32_t st = (uint32_t)g;
          if (st == kHelpStop) break;
          if (st >= t_next) {
            got = st;
            break;
          }
        } else if ((ge >> 16) == (epoch >> 16) && (ge & 0xFFFFu) > (epoch & 0xFFFFu)) {
          break;  // the leader has moved on to a later request of this launch
        }
        __nanosleep(nap);
        nap = min(2 * nap, kHelpMaxSleepNs);
      }
      __threadfence();
      S->help_step = got;
    }
    __syncthreads();
    const uint32_t t = S->help_step;
    if (t == kHelpStop || t >= L || t >= H->steps) break;
    t_next = t + 1;
    const uint32_t par = t & 1u;
    c.step = t;
    c.cur = slot.beams[par];
    c.f_next = p.factor[t + 1];
    c.xc = &H->xc[par];
    c.kmin = c.pkmin = 0xFFFFFFFFu;
    c.kmax = c.pkmax = 0;
    stage_row(p, row, meta.rows_off + (uint64_t)t * K, reinterpret_cast<uint64_t *>(bt.info));
    if (threadIdx.x == 0) {
      S->n_br = min(kParentChunk, min(vld(help_word(H, kHelpNbr, t)), p.beam_cap));
      S->pool_add = vld(&H->pool.base);
    }
    __syncthreads();
    expand_branch<true>(c, bt);  // the first chunk only, from the step's claim counter
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&H->left[kpar], 1u);
  }
}

// Two instances: one CTA per SM with up to 128 registers per thread (all
// launches with teams of 2-16 CTAs, and batches the SMs can hold one request
// each), and two CTAs per SM at 64 registers per thread (batches larger than
// the SM count, where twice the requests in flight hide more latency than the
// spills cost).
// kHelp: the instance that runs launches with helper clusters (the one-CTA
// instance only); the other instances compile none of that code.
template <int kMinBlocks, bool kHelp>
__global__ void __launch_bounds__(kSearchThreads, kMinBlocks) tbs_search_kernel(const SearchParams p) {
  extern __shared__ __align__(16) uint8_t dyn[];
  __shared__ TeamState team_state;
  __shared__ LocalState local_state;
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t cs = cluster.num_blocks();
  const uint32_t rank = cluster.block_rank();
  TeamState *T = cluster.map_shared_rank(&team_state, 0);
  // Clusters come in groups of 1 + helpers: the first of a group leads its
  // slot's requests, the others help with their expansion.
  const uint32_t per = p.helpers + 1;
  const uint32_t team = blockIdx.x / cs, n_groups = (gridDim.x / cs) / per;
  const uint32_t group = team / per, role = team % per;
  const SlotView slot = p.slots[group];
  if (role != 0 && (!kHelp || slot.help == nullptr)) return;
  uint32_t k = 0;
  for (uint32_t req = group; req < p.n_req; req += n_groups, ++k) {
    const uint32_t epoch = (p.launch_seq << 16) | (req & 0xFFFFu);
    if (role == 0) {
      search_request<kHelp>(p, req, slot, T, &local_state, rank, cs, dyn, epoch, k);
      // Every path out of the request ends its helpers' wait.
      if (kHelp && p.helpers && slot.help && rank == 0 && threadIdx.x == 0)
        vst64(&slot.help->go, ((unsigned long long)epoch << 32) | kHelpStop);
      team_sync(cs);  // rank 0's state is reused by the next request
    } else if (kHelp) {
      help_request(p, req, slot, &local_state, dyn, epoch, k & 1u);
    }
  }
}

// ------------------------------------------------------------- lookup
// Node reached from `node` by label x, or 0 (the root is nobody's child).
__device__ __forceinline__ uint32_t find_child(const TrieView &t, uint32_t node, uint32_t x, uint32_t *status) {
  const uint4 r = __ldg(t.node + node);
  const uint32_t f = rec_flags(r.w), c0 = r.z;
  uint32_t d = r.w & kFanoutMask;
  if (d == kFanoutMask) {
    const uint32_t end = (uint64_t)node + 1 < t.num_nodes ? __ldg(t.node + node + 1).z : (uint32_t)t.num_nodes;
    d = end > c0 ? end - c0 : 0;
  }
  if (d == 0) return 0;
  if ((uint64_t)c0 + d > t.num_nodes) {
    atomicOr(status, kStatusNodeBounds);
    return 0;
  }
  if (!(f & kNodeFlagLink) && (f & kNodeFlagHashed)) {
    // The node's open-addressing table (load <= 1/2: an empty slot ends every probe).
    const uint32_t lg = f >> 3, size = 1u << lg, mask = size - 1u;
    if ((uint64_t)r.y + size > t.hash_slots) {
      atomicOr(status, kStatusNodeBounds);
      return 0;
    }
    uint32_t h = (x * 2654435761u) >> (32 - lg);
    for (uint32_t probe = 0; probe < size; ++probe) {
      const uint2 sl = __ldg(t.hash + r.y + h);
      if (sl.y == 0) return 0;
      if (sl.x == x) return sl.y < t.num_nodes ? sl.y : 0u;
      h = (h + 1) & mask;
    }
    return 0;
  }
  // Child labels are sorted: binary search (the first word of each record).
  const uint32_t *labs = reinterpret_cast<const uint32_t *>(t.node + c0);
  uint32_t lo = 0, n = d;
  while (n > 0) {
    const uint32_t half = n >> 1;
    if (__ldg(labs + 4ull * (lo + half)) < x) {
      lo += half + 1;
      n -= half + 1;
    } else {
      n = half;
    }
  }
  return lo < d && __ldg(labs + 4ull * lo) == x ? c0 + lo : 0u;
}

// Key ids of n token sequences (reference LoudsTrie::lookup,
// louds-trie.cc:56-72, with the find_child walk of :764-808): one thread per
// key walks from the root; a link child matches its whole tail string.
__global__ void __launch_bounds__(256) lookup_kernel(const TrieView t, const uint32_t *tokens,
                                                     const uint64_t *offsets, uint32_t n, uint64_t total_tokens,
                                                     uint32_t *out, uint32_t *status) {
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t s = offsets[k], e = offsets[k + 1];
    uint32_t id = 0xFFFFFFFFu;
    if (s > e || e > total_tokens) {
      atomicOr(status, kStatusBadRequest);
      out[k] = id;
      continue;
    }
    uint32_t node = 0;
    bool found = t.num_nodes > 0;
    for (uint64_t pos = s; found && pos < e;) {
      const uint32_t child = find_child(t, node, tokens[pos], status);
      if (child == 0) {
        found = false;
        break;
      }
      ++pos;
      const uint4 cr = __ldg(t.node + child);
      const uint32_t cf = rec_flags(cr.w);
      if ((cf & kNodeFlagLink) && !(cf & kNodeFlagLinkEnds1)) {
        // The rest of the link's string, after its first token (the label).
        uint32_t off = cr.y + 1;
        for (;;) {
          bool ok;
          const bool end = tail_ends_at(t, off, ok);
          if (!ok) {
            atomicOr(status, kStatusTailBounds);
            found = false;
            break;
          }
          if (pos >= e || __ldg(t.tail + off) != tokens[pos]) {
            found = false;
            break;
          }
          ++pos;
          ++off;
          if (end) break;
        }
      }
      node = child;
    }
    if (found && (rec_flags(__ldg(t.node + node).w) & kNodeFlagTerminal)) id = key_id(t, node);
    out[k] = id;
  }
}

// Parent of every node (LOUDS numbers children after their parent, so
// parent[c] < c): each node writes itself into its children's entries.
__global__ void __launch_bounds__(256) parents_kernel(const TrieView t, uint32_t *parent, uint32_t *status) {
  for (uint64_t p = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; p < t.num_nodes;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint4 r = __ldg(t.node + p);
    const uint32_t c0 = r.z;
    uint64_t d = r.w & kFanoutMask;
    if (d == kFanoutMask) {
      const uint64_t end = p + 1 < t.num_nodes ? (uint64_t)__ldg(t.node + p + 1).z : t.num_nodes;
      d = end > c0 ? end - c0 : 0;
    }
    if (d == 0) continue;
    if ((uint64_t)c0 + d > t.num_nodes || c0 <= p) {
      atomicOr(status, kStatusNodeBounds);
      continue;
    }
    for (uint64_t c = c0; c < (uint64_t)c0 + d; ++c) parent[c] = (uint32_t)p;
  }
}

// Tokens a node contributes to its keys: its label, or a link node's whole
// tail string (which starts with the label).  Returns the count (0 and a
// status bit on a tail inconsistency); writes them to `out` when non-null.
__device__ __forceinline__ uint32_t node_tokens(const TrieView &t, uint32_t m, uint32_t *out, uint32_t *status) {
  const uint4 r = __ldg(t.node + m);
  if (!(rec_flags(r.w) & kNodeFlagLink)) {
    if (out) out[0] = r.x;
    return 1;
  }
  uint32_t n = 0;
  for (uint32_t off = r.y;; ++off) {
    bool ok;
    const bool end = tail_ends_at(t, off, ok);
    if (!ok) {
      atomicOr(status, kStatusTailBounds);
      return 0;
    }
    if (out) out[n] = __ldg(t.tail + off);
    ++n;
    if (end) return n;
  }
}

// Token sequences of key ids (reference LoudsTrie::reverse_lookup,
// louds-trie.cc:179-210): the id-th terminal node is found in the
// terminal-rank directory, then the walk to the root collects each node's
// tokens, back to front.  out_len[k] = the key's length (0xFFFFFFFF: not a
// key id); its tokens are written when they fit in max_len.
__global__ void __launch_bounds__(256) reverse_lookup_kernel(const TrieView t, const uint32_t *parent,
                                                             uint64_t num_keys, const uint32_t *ids, uint32_t n,
                                                             uint32_t max_len, uint32_t *out_tok, uint32_t *out_len,
                                                             uint32_t *status) {
  const uint64_t blocks = (t.num_nodes + 63) / 64;
  for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t id = ids[k];
    if ((uint64_t)id >= num_keys || blocks == 0) {
      out_len[k] = 0xFFFFFFFFu;
      continue;
    }
    // Last block whose count of earlier terminals is <= id holds the id-th.
    uint64_t lo = 0, cnt = blocks;
    while (cnt > 1) {
      const uint64_t half = cnt >> 1;
      if (__ldg(t.term_rank + lo + half).x <= id) {
        lo += half;
        cnt -= half;
      } else {
        cnt = half;
      }
    }
    const uint4 b = __ldg(t.term_rank + lo);
    uint64_t bits = ((uint64_t)b.w << 32) | b.z;
    for (uint32_t r = id - b.x; r > 0 && bits; --r) bits &= bits - 1;
    if (!bits || b.x > id) {
      atomicOr(status, kStatusNodeBounds);
      out_len[k] = 0xFFFFFFFFu;
      continue;
    }
    const uint32_t node = (uint32_t)(lo * 64 + (uint64_t)(__ffsll((long long)bits) - 1));
    // Length, then the tokens back to front.
    uint64_t len = 0;
    bool ok = true;
    for (uint32_t m = node; m != 0;) {
      const uint32_t c = node_tokens(t, m, nullptr, status);
      const uint32_t up = parent[m];
      if (c == 0 || up >= m) {
        ok = false;
        break;
      }
      len += c;
      m = up;
    }
    if (!ok || len > 0xFFFFFFFEull) {
      atomicOr(status, kStatusNodeBounds);
      out_len[k] = 0xFFFFFFFFu;
      continue;
    }
    out_len[k] = (uint32_t)len;
    if (len > max_len) continue;
    uint32_t *dst = out_tok + k * (uint64_t)max_len;
    uint64_t pos = len;
    for (uint32_t m = node; m != 0; m = parent[m]) {
      const uint32_t c = node_tokens(t, m, nullptr, status);
      pos -= c;
      node_tokens(t, m, dst + pos, status);
    }
  }
}

}  // namespace

size_t search_smem_bytes(uint32_t max_topk, uint32_t max_final_beam) {
  uint32_t P2 = 1;
  while (P2 < max_final_beam) P2 <<= 1;
  uint32_t PK = 1;
  while (PK < max_topk) PK <<= 1;
  // Row, then the task table (which also holds the sort keys of an unsorted row).
  const size_t row = (((size_t)max_topk * 12 + 15) & ~size_t(15)) +
                     std::max<size_t>((size_t)kParentChunk * (sizeof(uint4) + sizeof(double) + sizeof(uint32_t)),
                                      (size_t)PK * 8);
  const size_t sort = (size_t)P2 * 16;
  return std::max<size_t>(std::max(row, sort), 16);
}

template <int kMinBlocks, bool kHelp>
static int raise_smem(size_t search_smem) {
  cudaFuncAttributes a;
  CUDA_TRY(cudaFuncGetAttributes(&a, tbs_search_kernel<kMinBlocks, kHelp>));
  if ((size_t)a.maxDynamicSharedSizeBytes < search_smem)
    CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel<kMinBlocks, kHelp>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)search_smem));
  CUDA_TRY(cudaFuncSetAttribute(tbs_search_kernel<kMinBlocks, kHelp>,
                                cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tbs_search_kernel<kMinBlocks, kHelp>,
                                                         kSearchThreads, search_smem));
  return per_sm;
}

// Launch-planning answers of the driver, per device: the SM count, and how
// many teams (or, for the two-CTAs-per-SM instance, CTAs per SM) fit for a
// team size and dynamic shared-memory size.  They do not change while the
// process runs, and asking the driver again on every search call would add
// its cost to every synchronous search.  Callers raise the kernels'
// shared-memory limit (ensure_search_smem) before planning a launch with
// that size, so a remembered answer is never one taken under a lower limit.
namespace {
struct PlanCache {
  std::mutex mu;
  std::map<int, int> sms;                                   // device -> SMs
  std::map<std::tuple<int, int, size_t>, int> clusters;     // (device, team size, smem) -> teams
  std::map<std::pair<int, size_t>, int> dense_per_sm;       // (device, smem) -> CTAs per SM
};
PlanCache &plan_cache() {
  static PlanCache c;
  return c;
}
}  // namespace

static int sm_count() {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  PlanCache &pc = plan_cache();
  {
    std::lock_guard<std::mutex> lock(pc.mu);
    auto it = pc.sms.find(dev);
    if (it != pc.sms.end()) return it->second;
  }
  int sms = 0;
  CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  std::lock_guard<std::mutex> lock(pc.mu);
  pc.sms[dev] = sms;
  return sms;
}

int ensure_search_smem(size_t search_smem) {
  const int one = raise_smem<1, false>(search_smem), two = raise_smem<2, false>(search_smem);
  raise_smem<1, true>(search_smem);
  return std::max(std::max(one, two), 1) * sm_count();
}

int max_search_clusters(int cluster_size, size_t smem_bytes) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  PlanCache &pc = plan_cache();
  const auto key = std::make_tuple(dev, cluster_size, smem_bytes);
  {
    std::lock_guard<std::mutex> lock(pc.mu);
    auto it = pc.clusters.find(key);
    if (it != pc.clusters.end()) return it->second;
  }
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
  CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, (void *)tbs_search_kernel<1, false>, &cfg));
  std::lock_guard<std::mutex> lock(pc.mu);
  pc.clusters[key] = n;
  return n;
}

SearchLaunch plan_search(uint32_t n, size_t smem_bytes) {
  const int sms = sm_count();
  SearchLaunch l;
  int cs = 1;
  bool forced = false;
  if (const char *e = getenv("FT_CLUSTER_SIZE")) {
    cs = atoi(e);
    if (cs < 1 || cs > 16 || (cs & (cs - 1))) cs = 1;
    forced = true;
  } else {
    const int want = n ? sms / (int)n : sms;
    while (cs * 2 <= 16 && cs * 2 <= want) cs *= 2;
  }
  // Halve the team until the whole batch is resident at once: clusters of
  // 16 CTAs need 16 free SMs of one GPC, so fewer of them fit than SMs / 16,
  // and a request left for a second wave doubles the batch's time.
  for (;; cs /= 2) {
    const int teams = max_search_clusters(cs, smem_bytes);
    if ((teams >= 1 && (forced || teams >= (int)n)) || cs == 1) {
      l.cluster_size = cs;
      l.max_teams = std::max(teams, 1);
      break;
    }
  }
  l.dense = 0;
  bool dense_ok = l.cluster_size == 1 && n > (uint32_t)sms;
  if (const char *e = getenv("FT_DENSE")) dense_ok = l.cluster_size == 1 && atoi(e) != 0;
  if (dense_ok) {
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    PlanCache &pc = plan_cache();
    int per_sm = -1;
    {
      std::lock_guard<std::mutex> lock(pc.mu);
      auto it = pc.dense_per_sm.find({dev, smem_bytes});
      if (it != pc.dense_per_sm.end()) per_sm = it->second;
    }
    if (per_sm < 0) {
      CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tbs_search_kernel<2, false>, kSearchThreads,
                                                             smem_bytes));
      std::lock_guard<std::mutex> lock(pc.mu);
      pc.dense_per_sm[{dev, smem_bytes}] = per_sm;
    }
    if (per_sm >= 2) {
      l.dense = 1;
      l.max_teams = per_sm * sms;
    }
  }
  return l;
}

namespace {
struct L2Window {
  size_t persist = 0;  // persisting L2 bytes set aside (0: none)
  size_t max_window = 0;
};
std::mutex g_l2_mu;
std::map<int, L2Window> g_l2;

L2Window l2_window(int device) {
  std::lock_guard<std::mutex> lock(g_l2_mu);
  auto it = g_l2.find(device);
  return it == g_l2.end() ? L2Window{} : it->second;
}
}  // namespace

size_t reserve_l2_persisting(int device) {
  std::lock_guard<std::mutex> lock(g_l2_mu);
  auto it = g_l2.find(device);
  if (it != g_l2.end()) return it->second.persist;
  L2Window w;
  // Opt-in: measured neutral at batch 1 and 9-12% slower at batches of
  // hundreds, where the carve-out takes L2 from the candidate buffers.
  const char *e = getenv("FT_L2_PERSIST");
  if (e && atoi(e) != 0) {
    int max_persist = 0, max_window = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, device));
    CUDA_TRY(cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, device));
    if (max_persist > 0 && max_window > 0) {
      // A limit of this process's context, released with it.
      CUDA_TRY(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, (size_t)max_persist));
      CUDA_TRY(cudaDeviceGetLimit(&w.persist, cudaLimitPersistingL2CacheSize));
      w.max_window = (size_t)max_window;
    }
  }
  g_l2[device] = w;
  return w.persist;
}

int search_grid(SearchParams &p, uint32_t n, uint32_t n_slots, const SearchLaunch &l, bool can_help) {
  static std::atomic<uint32_t> seq{1};  // epochs are never 0, the words' value at allocation
  const uint32_t teams = (uint32_t)std::max(l.max_teams, 1);
  const uint32_t groups = std::max<uint32_t>(1u, std::min(std::min(n, n_slots), teams));
  uint32_t helpers = 0;
  if (can_help && !l.dense && n < 65536u) {
    helpers = std::min<uint32_t>(kMaxHelpers, teams / groups - 1u);
    if (const char *e = getenv("FT_HELPERS")) helpers = std::min<uint32_t>(helpers, (uint32_t)std::max(atoi(e), 0));
  }
  p.n_groups = groups;
  p.helpers = helpers;
  uint32_t ls = seq.fetch_add(1u) & 0xFFFFu;
  if (ls == 0) ls = seq.fetch_add(1u) & 0xFFFFu;
  p.launch_seq = ls;
  return (int)(groups * (helpers + 1u));
}

void launch_search(const SearchParams &p, size_t smem_bytes, int grid, cudaStream_t stream, const SearchLaunch &l) {
  if (p.n_req == 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid * l.cluster_size, 1, 1);
  cfg.blockDim = dim3(kSearchThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = l.cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The upper levels of the trie (the first node records: LOUDS numbers
  // nodes level by level) stay in the persisting part of L2.
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  const L2Window w = l2_window(dev);
  if (w.persist > 0) {
    const size_t bytes = std::min<size_t>({(size_t)p.trie.num_nodes * sizeof(uint4), w.max_window, w.persist});
    if (bytes > 0) {
      attr[1].id = cudaLaunchAttributeAccessPolicyWindow;
      attr[1].val.accessPolicyWindow.base_ptr = const_cast<uint4 *>(p.trie.node);
      attr[1].val.accessPolicyWindow.num_bytes = bytes;
      attr[1].val.accessPolicyWindow.hitRatio = 1.0f;
      attr[1].val.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
      attr[1].val.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
      cfg.numAttrs = 2;
    }
  }
  if (l.dense) {
    CUDA_TRY(cudaLaunchKernelEx(&cfg, tbs_search_kernel<2, false>, p));
  } else if (p.helpers) {
    CUDA_TRY(cudaLaunchKernelEx(&cfg, tbs_search_kernel<1, true>, p));
  } else {
    CUDA_TRY(cudaLaunchKernelEx(&cfg, tbs_search_kernel<1, false>, p));
  }
}

void launch_lookup(const TrieView &t, const uint32_t *tokens, const uint64_t *offsets, uint32_t n,
                   uint64_t total_tokens, uint32_t *out, uint32_t *status, cudaStream_t stream) {
  if (n == 0) return;
  const uint32_t blocks = std::min<uint32_t>((n + 255) / 256, (uint32_t)sm_count() * 8u);
  lookup_kernel<<<blocks, 256, 0, stream>>>(t, tokens, offsets, n, total_tokens, out, status);
  CUDA_TRY(cudaGetLastError());
}

void launch_parents(const TrieView &t, uint32_t *parent, uint32_t *status, cudaStream_t stream) {
  if (t.num_nodes == 0) return;
  const uint64_t want = (t.num_nodes + 255) / 256;
  const uint32_t blocks = (uint32_t)std::min<uint64_t>(want, (uint64_t)sm_count() * 8u);
  parents_kernel<<<blocks, 256, 0, stream>>>(t, parent, status);
  CUDA_TRY(cudaGetLastError());
}

void launch_reverse_lookup(const TrieView &t, const uint32_t *parent, uint64_t num_keys, const uint32_t *ids,
                           uint32_t n, uint32_t max_len, uint32_t *out_tok, uint32_t *out_len, uint32_t *status,
                           cudaStream_t stream) {
  if (n == 0) return;
  const uint32_t blocks = std::min<uint32_t>((n + 255) / 256, (uint32_t)sm_count() * 8u);
  reverse_lookup_kernel<<<blocks, 256, 0, stream>>>(t, parent, num_keys, ids, n, max_len, out_tok, out_len, status);
  CUDA_TRY(cudaGetLastError());
}

}  // namespace ftb
