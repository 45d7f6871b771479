// Shared declarations of the TBS search kernels (device side) and the host
// launcher.  See tbs_kernel.cu for the algorithm.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "device_trie.hpp"

namespace ftb {

constexpr int kSearchThreads = 512;          // threads per search CTA
constexpr int kRefBlock = 512;               // threads per CTA of the reference kernel
                                             // (tbs-kernels.cu:10): in-link matches are
                                             // taken first-per-residue-class of this size

// Candidate produced by expansion (32 bytes).
//   next-candidates: aux = tail offset of the next token for a link node (an
//                    in-link beam), the hash base for a hashed plain node;
//                    c0 / dw = the node record's child range and flags, so
//                    the next step needs no further load to expand it
//   pool entries:    aux = depth
struct alignas(16) Cand {
  double score;
  uint32_t node;
  uint32_t aux;
  uint32_t parent;  // index of the parent beam in the step's beam array
  uint32_t token;
  uint32_t c0;
  uint32_t dw;
};

// A live beam (24 bytes).  In-link iff its node is a link node.
struct Beam {
  double score;
  uint32_t node;
  uint32_t off;  // next tail cell (in-link beam) or hash base (hashed plain node)
  uint32_t c0;
  uint32_t dw;
};

// History record of the beam at index i of step s: its parent's index at
// step s-1 and its last token.
struct Hist {
  uint32_t parent;
  uint32_t token;
};

// Per-request metadata (element offsets into the packed batch arrays).
struct ReqMeta {
  uint32_t L;
  uint32_t K;
  uint64_t beams_off;  // into beams[]
  uint64_t rows_off;   // into topk_id[] / topk_logp[] and the sorted-row workspace
};

struct TrieView {
  const uint4 *node;
  const uint4 *term_rank;    // key-id directory, see device_trie.hpp
  const uint32_t *tail;
  const uint64_t *tail_end;  // nullptr for a text tail
  const uint2 *hash;         // per-node child tables {label, child}, see device_trie.hpp
  uint64_t num_nodes;
  uint64_t tail_size;
  uint64_t hash_slots;
};

inline TrieView make_trie_view(const DeviceTrie &d) {
  TrieView v;
  v.node = reinterpret_cast<const uint4 *>(d.node);
  v.term_rank = reinterpret_cast<const uint4 *>(d.term_rank);
  v.tail = d.tail;
  v.tail_end = d.binary_tail ? d.tail_end : nullptr;
  v.hash = reinterpret_cast<const uint2 *>(d.hash);
  v.num_nodes = d.num_nodes;
  v.tail_size = d.tail_size;
  v.hash_slots = d.hash_slots;
  return v;
}

// Branching parents are expanded in chunks of this many parents (their task
// table lives in shared memory behind the staged row).
constexpr uint32_t kParentChunk = 1024;
// Items (children or proposals) per expansion task: four per lane.
constexpr uint32_t kTaskItems = 128;

// State a request's leader team shares with its helper CTAs (global memory,
// one per slot).  `go` = (epoch << 32) | step: the step the leader opened for
// helpers, or kHelpStop when the request is over; the epoch names the launch
// and request, so a value left by an earlier request or launch is never taken
// for the current one.  The counters are the ones every expanding CTA appends
// to, by step parity, and the result pool's; in a request without helpers the
// same counters live in the leader team's shared memory.
// Counters every CTA that expands a step appends to (one set per step
// parity), and the result pool's.
struct ExpCounters {
  uint32_t n_next;     // candidates appended
  uint32_t key_min;    // range of the top 32 bits of the candidates' first key word
  uint32_t key_max;
  uint32_t task_next;  // branch tasks handed out on demand
};
struct PoolCounters {
  uint32_t pool_end;      // pool entries (append counter)
  uint32_t pool_key_min;  // range of the top 32 bits of the pool entries' first key word
  uint32_t pool_key_max;
  uint32_t base;          // HelpState copy: where an open step's appends start in the pool
};

// joined[q] / left[q] count helper CTAs that entered / left requests whose
// ordinal in the slot has parity q: the leader re-arms the per-step counters
// for a request only when every helper of the request before it has left.
// The per-step arrays follow the struct (help_word()), `steps` long each.
struct alignas(16) HelpState {
  unsigned long long go;
  uint32_t joined[2], left[2];
  uint32_t steps, pad0, pad1, pad2;
  ExpCounters xc[2];
  PoolCounters pool;
};
// Per step t (arrays after the struct, help_words()): claim = branch tasks
// handed out; done = tasks finished; total = the step's task count
// (0xFFFFFFFF until the leader has built its table); nbr = branching beams of
// the step; arm = the epoch of the request that last opened the step (the
// leader writes it after the other words; its CTAs claim only once they see
// it, helpers only after `go`).
constexpr uint32_t kHelpClaim = 0, kHelpDone = 1, kHelpTotal = 2, kHelpNbr = 3, kHelpArm = 4;
__host__ __device__ inline uint32_t *help_word(HelpState *h, uint32_t which, uint32_t t) {
  return reinterpret_cast<uint32_t *>(h + 1) + (size_t)which * h->steps + t;
}
__host__ __device__ inline size_t help_state_bytes(uint64_t steps) {
  return (sizeof(HelpState) + 5 * 4 * steps + 15) & ~size_t(15);
}
constexpr uint32_t kHelpStop = 0xFFFFFFFFu;
// Most helper clusters one request gets.
constexpr uint32_t kMaxHelpers = 8;
// Helper clusters pay off only where a step can hold many branch tasks (a
// step is opened to them at 1024 tasks, one task per 128 proposals of a
// large node): rows of at least kHelpMinTopk proposals and beams of at least
// kHelpMinBeam.  Elsewhere the kernel instance without helper code runs.
constexpr uint32_t kHelpMinTopk = 512;
constexpr uint32_t kHelpMinBeam = 256;
inline bool helpers_pay(uint32_t topk, uint32_t max_beam) {
  return topk >= kHelpMinTopk && max_beam >= kHelpMinBeam;
}

// Device workspace of one search slot (one in-flight request).
//   pool_cap = beam_cap + 2 * beam_cap * max_topk: a step appends at most
//   (its beams) * K pool entries, so the pool is trimmed to the final beam
//   width only when the next step could overflow it.
struct SlotView {
  Cand *next;        // [cand_cap]: this step's candidates
  Cand *pool;        // [pool_cap]: result pool (entries that end a key)
  Cand *pool_tmp;    // [beam_cap]: survivors of a pool trim
  Beam *beams[2];    // [beam_cap] each; in-link beams from the front, branching from the back
  Hist *hist;        // [(max_outpos + 1) * beam_cap]
  HelpState *help;   // helper state and its per-step arrays, or null (no helpers)
};

struct SearchParams {
  TrieView trie;
  const ReqMeta *meta;
  const uint32_t *beams;
  const uint32_t *topk_id;
  const float *topk_logp;
  const double *factor;     // [max L + 1]: (6 / (5 + depth)) ^ length_norm
  // workspace
  SlotView *slots;
  uint64_t cand_cap;
  uint64_t pool_cap;
  uint32_t beam_cap;
  uint32_t n_req;
  uint32_t n_slots;
  // Requests in flight at once (one slot each) and helper clusters per
  // request: cluster g of the grid serves slot g / (helpers + 1), as its
  // leader when g % (helpers + 1) == 0.  helpers = 0: every cluster leads.
  uint32_t n_groups;
  uint32_t helpers;
  uint32_t launch_seq;  // distinct per launch (helper epochs)
  // search parameters
  double token_threshold;
  double sent_threshold;
  int early_exit;
  // outputs
  uint32_t out_cap;
  uint32_t out_stride;
  uint32_t *out_count;
  double *out_lpn;
  uint32_t *out_len;
  uint32_t *out_tok;
  uint32_t *out_key;     // [n_req][out_cap] key ids of the result beams, or nullptr
  double *out_phase_ms;  // [n_req][5] or nullptr
  uint64_t *tok_total;   // compact token output: running token count, or nullptr (strided output)
  uint64_t *out_tok_base;  // compact token output: [n_req] first token of each request
  uint32_t *status;      // device status word (bit flags, see kStatus*)
  uint32_t *debug;       // [8]: first failed self-check (code, step, n, k, got, team, ge, rem)
};

constexpr uint32_t kStatusCandOverflow = 1u;
constexpr uint32_t kStatusPoolOverflow = 2u;
constexpr uint32_t kStatusTailBounds = 4u;
constexpr uint32_t kStatusNodeBounds = 8u;
constexpr uint32_t kStatusBadRequest = 16u;
constexpr uint32_t kStatusSelection = 32u;  // a selection did not select exactly k
constexpr uint32_t kStatusHelp = 64u;       // a bounded wait on helper clusters ran out

// Shared-memory bytes the search kernel needs for a given max K / max final beam.
size_t search_smem_bytes(uint32_t max_topk, uint32_t max_final_beam);

// How a batch is launched: teams of `cluster_size` CTAs (thread-block
// clusters), at most `max_teams` resident at once; `dense` selects the
// two-CTAs-per-SM kernel instance (one-CTA teams, batches larger than the SM
// count).  FT_CLUSTER_SIZE and FT_DENSE override the choice.
struct SearchLaunch {
  int cluster_size;
  int max_teams;
  int dense;
};

// Teams (clusters) to launch for n requests on `n_slots` slots and helper
// clusters per request: when fewer requests than resident teams are in
// flight, each request's leader team gets up to kMaxHelpers helper clusters
// (only with helper state in the workspace: `can_help`).  Fills
// p.n_groups / p.helpers and returns the number of teams.
int search_grid(SearchParams &p, uint32_t n, uint32_t n_slots, const SearchLaunch &l, bool can_help);

// Team size for a batch of n requests: the largest power of two <= 16 with
// n teams fitting on the device.
SearchLaunch plan_search(uint32_t n, size_t smem_bytes);

// Enqueues the search kernel on `stream`: `grid` teams, one per in-flight
// request (requests beyond `grid` are taken by teams that finish).
// Key ids of n token sequences in device memory (key i is
// tokens[offsets[i], offsets[i+1])) into out (0xFFFFFFFF: not a key), on
// `stream`; bad offsets and trie inconsistencies set bits of *status.
void launch_lookup(const TrieView &t, const uint32_t *tokens, const uint64_t *offsets, uint32_t n,
                   uint64_t total_tokens, uint32_t *out, uint32_t *status, cudaStream_t stream);

// parent[c] for every node c (parent[0] = 0), on `stream`.
void launch_parents(const TrieView &t, uint32_t *parent, uint32_t *status, cudaStream_t stream);

// Token sequences of n key ids (see reverse_lookup_kernel), on `stream`:
// out_len[k] = length of key ids[k] (0xFFFFFFFF: not a key id); its tokens go
// to out_tok[k * max_len ...] when the length is at most max_len.
void launch_reverse_lookup(const TrieView &t, const uint32_t *parent, uint64_t num_keys, const uint32_t *ids,
                           uint32_t n, uint32_t max_len, uint32_t *out_tok, uint32_t *out_len, uint32_t *status,
                           cudaStream_t stream);

// With FT_L2_PERSIST=1, sets aside the device's persisting L2 (once per
// device and process) for the access-policy window every search launch then
// puts on the upper levels of its trie; returns the bytes set aside (0: off).
size_t reserve_l2_persisting(int device);

void launch_search(const SearchParams &p, size_t smem_bytes, int grid, cudaStream_t stream, const SearchLaunch &l);

// Teams of `cluster_size` CTAs that can be resident at once.
int max_search_clusters(int cluster_size, size_t smem_bytes);

// Raises (never lowers) the dynamic shared-memory limit of both search kernel
// instances on the current device; returns max resident search CTAs for
// `search_smem` (of the denser instance).
int ensure_search_smem(size_t search_smem);

}  // namespace ftb
