/*
 * TEST INFRASTRUCTURE ONLY - not part of the product.
 *
 * CPU restatement of the reference FlashTrie trie-constrained beam search
 * (TBS) as its GPU kernel defines it (lib/marisa/grimoire/trie/tbs-kernels.cu),
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as
 * the checker.  It reads the reference trie file format itself and walks the
 * reference's own succinct structures (LOUDS select0/rank1, bases/extras,
 * link_extras, text/binary tail), so it shares no code with the engine it
 * checks.
 *
 * Pinning: the restatement is checked against golden vectors produced by the
 * unmodified reference (its CPU `tbs`, built from its own sources by
 * oracle/ref.mk) in tests/golden/.  The reference's GPU and CPU paths differ
 * (link-node handling, early exit, tie order); the golden tests compare on
 * the requests where they agree and report the rest.
 *
 * Ordering is pinned where the reference leaves it open: candidates rank by
 * logp_norm (f64) descending, then node id descending, then depth descending,
 * then raw score descending.  Output lists are ascending in that order.
 */
#ifndef FT_TBS_ORACLE_H_
#define FT_TBS_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_trie oracle_trie;

#define ORACLE_MAX_STEPS 256

/* Per-request counters; `bytes_alg` is the algorithmic byte count the
 * engine's roofline divides by its time: K*8 per step (the row); 32 per
 * in-link parent (its tail cells) and 32 more when its link ends (terminal
 * flag); 32 per branching parent (child range) plus
 * 32*min(ceil(d/8)+1, K*ceil(log2(d+1))) for its child labels; 32 per matched
 * child (flags) and 64 more per matched link child (link offset, next tail
 * cells); 64 per candidate or pool entry (written, then read at selection);
 * 12 + 4*len per output beam. */
typedef struct {
  uint32_t steps_run;
  uint64_t parents_inlink[ORACLE_MAX_STEPS];
  uint64_t parents_branch[ORACLE_MAX_STEPS];
  uint64_t degree_sum[ORACLE_MAX_STEPS];
  uint64_t next_pushes[ORACLE_MAX_STEPS];
  uint64_t sel_pushes[ORACLE_MAX_STEPS];
  uint64_t bytes_alg;
  /* selections whose cut fell between candidates with equal logp_norm (the
   * reference leaves the order of such ties open) */
  uint32_t ties_at_cut;
} oracle_stats;

/* Load a trie file. Returns 0 on success, negative on error (message in err). */
int oracle_load(const char *path, oracle_trie **out, char *err, int errlen);
void oracle_free(oracle_trie *t);
uint64_t oracle_num_nodes(const oracle_trie *t);
uint64_t oracle_num_keys(const oracle_trie *t);

/* Is `key` (len labels) a key of the trie?  (reference LoudsTrie::lookup) */
int oracle_lookup(const oracle_trie *t, const uint32_t *key, uint32_t len);
/* Key id of `key` (reference LoudsTrie::lookup: the rank of its terminal node
 * among terminal nodes), or -1 if it is not a key. */
int64_t oracle_lookup_id(const oracle_trie *t, const uint32_t *key, uint32_t len);

/*
 * One search request.  Rows are topk_id/topk_logp[L][K] row-major.
 * Output: up to out_cap beams, ascending; tokens of beam i at
 * out_tok[i*out_stride ...], length out_len[i].
 * Returns 0 on success, -1 bad arguments, -2 out_cap/out_stride too small,
 * -3 out of memory.
 */
int oracle_tbs(const oracle_trie *t, uint32_t L, uint32_t K, const uint32_t *beams,
               const uint32_t *topk_id, const float *topk_logp, float token_logp_threshold,
               double sent_logp_threshold, double length_norm, int early_exit, uint32_t out_cap,
               uint32_t out_stride, uint32_t *out_n, double *out_lpn, uint32_t *out_len,
               uint32_t *out_tok, oracle_stats *stats);

#ifdef __cplusplus
}
#endif

#endif
