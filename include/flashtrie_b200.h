/*
 * flashtrie_b200 - C ABI of the B200 trie-constrained beam search (TBS) engine.
 *
 * This is the drop-in boundary for the reference FlashTrie TBS path: every
 * entry point below replaces one call the reference's pybind11 module
 * `flashtrie` (tools/bindings.cpp) makes into `marisa::Trie`
 * (include/marisa/trie.h).  Plain pointers and sizes only; no exceptions
 * cross the ABI.  Every function returns FT_OK (0) or a negative FT_ERR_*
 * code; ft_last_error() gives the message of the calling thread's last
 * failure.
 *
 * Memory layout conventions:
 *   - a request has L decoding positions (L = len(beams)) and K proposals per
 *     position; rows are stored row-major: topk_id[t*K + j], topk_logp[t*K + j];
 *   - results are ascending by logp_norm, like the reference output
 *     (lib/marisa/grimoire/trie/tbs-kernels.cu:415-421).
 */
#ifndef FLASHTRIE_B200_H_
#define FLASHTRIE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  -1..-10 mirror marisa_error_code (include/marisa/base.h:79-91). */
#define FT_OK 0
#define FT_ERR_STATE (-1)    /* MARISA_STATE_ERROR: no trie, no workspace, ...   */
#define FT_ERR_NULL (-2)     /* MARISA_NULL_ERROR                                */
#define FT_ERR_BOUND (-3)    /* MARISA_BOUND_ERROR                               */
#define FT_ERR_RANGE (-4)    /* MARISA_RANGE_ERROR                               */
#define FT_ERR_CODE (-5)     /* MARISA_CODE_ERROR: bad config flags              */
#define FT_ERR_SIZE (-7)     /* MARISA_SIZE_ERROR: trie exceeds format limits    */
#define FT_ERR_MEMORY (-8)   /* MARISA_MEMORY_ERROR / device allocation failed   */
#define FT_ERR_IO (-9)       /* MARISA_IO_ERROR                                  */
#define FT_ERR_FORMAT (-10)  /* MARISA_FORMAT_ERROR                              */
#define FT_ERR_INVALID_ARG (-20) /* request violates the workspace limits        */
#define FT_ERR_CUDA (-21)        /* a CUDA runtime call failed                   */
#define FT_ERR_DEVICE (-22)      /* the search kernel reported a bad trie access */

typedef struct ft_trie ft_trie;

typedef struct {
  uint64_t num_keys;   /* Trie::num_keys   (include/marisa/trie.h:51)  */
  uint64_t num_nodes;  /* Trie::num_nodes  (include/marisa/trie.h:52)  */
  uint64_t num_tries;  /* Trie::num_tries  (include/marisa/trie.h:50)  */
  uint64_t total_size; /* Trie::total_size (include/marisa/trie.h:59)  */
  uint64_t io_size;    /* Trie::io_size    (include/marisa/trie.h:60)  */
  uint32_t tail_mode;  /* Trie::tail_mode  (include/marisa/trie.h:54)  */
  uint32_t node_order; /* Trie::node_order (include/marisa/trie.h:55)  */
} ft_trie_info;

/* One request, host memory (TbsInput inputs, include/marisa/tbs_input.h:7-12). */
typedef struct {
  uint32_t num_outpos;        /* L = len(beams)                       */
  uint32_t topk;              /* K, proposals per position            */
  const uint32_t *beams;      /* [L] beam width per position           */
  const uint32_t *topk_id;    /* [L*K] token ids                       */
  const float *topk_logp;     /* [L*K] token log-probabilities         */
} ft_request;

/* One result, host memory (TbsInput outputs, include/marisa/tbs_input.h:13-25).
 * The caller provides capacity >= beams[L-1] and stride >= L. */
typedef struct {
  uint32_t capacity;          /* in: beams the arrays can hold               */
  uint32_t stride;            /* in: token slots per beam                    */
  uint32_t num_beams;         /* out                                         */
  uint32_t reserved;
  double *logp_norm;          /* out: [capacity], ascending                  */
  uint32_t *lengths;          /* out: [capacity]                             */
  uint32_t *tokens;           /* out: [capacity*stride], beam i at i*stride  */
  double phase_ms[5];         /* out: expansion, validation, selection,
                                 overhead, kernel (tbs_input.h:19-25)        */
  uint32_t *key_ids;          /* out, optional ([capacity], NULL: not written):
                                 the key id of each beam, as LoudsTrie::lookup
                                 reports it (louds-trie.cc:56-72; no
                                 counterpart in the reference's TbsInput)    */
} ft_result;

/* Search parameters shared by a batch (tools/bindings.cpp:71-78). */
typedef struct {
  float token_logp_threshold;
  float reserved;
  double sent_logp_threshold;
  double length_norm;
  int32_t early_exit;
  int32_t reserved2;
} ft_search_params;

/* Last error message of the calling thread ("" if none). */
const char *ft_last_error(void);

/* marisa::Trie::Trie() (include/marisa/trie.h:21), bound at tools/bindings.cpp:28 */
int ft_trie_create(ft_trie **out);
/* marisa::Trie::~Trie(); frees host and device state */
void ft_trie_destroy(ft_trie *trie);

/* marisa::Trie::load (include/marisa/trie.h:29), bound at tools/bindings.cpp:29 */
int ft_trie_load(ft_trie *trie, const char *path);
/* marisa::Trie::mmap (include/marisa/trie.h:26), bound at tools/bindings.cpp:30 */
int ft_trie_mmap(ft_trie *trie, const char *path);
/* build_from_list (tools/bindings.cpp:10-22): keys as a flat token array plus
 * num_rows+1 offsets; flags 1 | TEXT_TAIL | LABEL_ORDER | NORMAL_CACHE */
int ft_trie_build(ft_trie *trie, const uint32_t *tokens, const uint64_t *offsets, uint64_t num_rows);
/* marisa::Trie::save (include/marisa/trie.h:32), bound at tools/bindings.cpp:36 */
int ft_trie_save(const ft_trie *trie, const char *path);
/* marisa::Trie::clear (include/marisa/trie.h:62), bound at tools/bindings.cpp:37 */
int ft_trie_clear(ft_trie *trie);
/* num_keys / num_nodes / num_tries / total_size / io_size
 * (tools/bindings.cpp:32-35) */
int ft_trie_get_info(const ft_trie *trie, ft_trie_info *out);

/* marisa::Trie::init_tbs_gpu (include/marisa/trie.h:40-44), bound at
 * tools/bindings.cpp:38-43.  Uploads the trie to the current CUDA device and
 * sizes the search workspace. */
int ft_trie_init_tbs_gpu(ft_trie *trie, uint64_t max_batch_size, uint64_t max_num_topk,
                         uint64_t max_num_outpos, uint64_t max_num_out_beams,
                         uint64_t max_num_out_tokens, uint64_t max_num_inter_beams,
                         uint64_t radix_topk_threshold);
/* marisa::Trie::get_max_batch_size (include/marisa/trie.h:45) */
int ft_trie_get_max_batch_size(const ft_trie *trie, uint64_t *out);

/* marisa::Trie::tbs_gpu_batched (include/marisa/trie.h:48), bound as
 * bs_tbs_gpu at tools/bindings.cpp:71-119, and marisa::Trie::tbs_gpu
 * (trie.h:47) for n == 1.  Host buffers in and out; copies, kernel and
 * synchronisation happen inside the call. */
int ft_tbs_batch(ft_trie *trie, const ft_request *requests, uint32_t n,
                 const ft_search_params *params, ft_result *results);

/*
 * Device-resident batch (no counterpart in the reference, which always stages
 * host buffers): the same search on inputs already in device memory, written
 * to device outputs, on a caller stream.  Layout of the inputs for n
 * requests with a common L and K:
 *   beams     u32 [n][L]
 *   topk_id   u32 [n][L][K]
 *   topk_logp f32 [n][L][K]
 * Every pointer of a non-empty batch except out_key must be set (the rows
 * only when K > 0); a NULL one is refused with FT_ERR_NULL before any launch.
 * Outputs, per request i, with cap = max final beam and stride = L:
 *   out_count u32 [n]            number of beams
 *   out_lpn   f64 [n][cap]       ascending logp_norm
 *   out_len   u32 [n][cap]
 *   out_tok   u32 [n][cap][L]
 *   out_key   u32 [n][cap]       key ids (optional, NULL: not written)
 * `stream` is a cudaStream_t (0 = default stream).  The call returns after
 * enqueueing; completion is observed with stream synchronisation.
 */
typedef struct {
  uint32_t n;
  uint32_t num_outpos;
  uint32_t topk;
  uint32_t out_capacity;
  const uint32_t *beams;
  const uint32_t *topk_id;
  const float *topk_logp;
  uint32_t *out_count;
  double *out_lpn;
  uint32_t *out_len;
  uint32_t *out_tok;
  uint32_t *out_key;
} ft_device_batch;

int ft_tbs_batch_device(ft_trie *trie, const ft_device_batch *batch,
                        const ft_search_params *params, void *stream);

/*
 * Replaces LoudsTrie::lookup (lib/marisa/grimoire/trie/louds-trie.cc:56-72)
 * for a batch, on the device: key i is tokens[offsets[i] .. offsets[i+1]) and
 * out_ids[i] receives its key id (the id ft_result.key_ids reports), or
 * 0xFFFFFFFF when it is not a key of the trie.  tokens (total_tokens entries),
 * offsets (n + 1 entries) and out_ids (n entries) are device pointers; the
 * lookup runs on `stream` and the call returns without waiting.  Requires
 * ft_trie_init_tbs_gpu.  Offsets that decrease or pass total_tokens give
 * 0xFFFFFFFF for that key and set a bit of the device status word.
 */
int ft_lookup_batch_device(ft_trie *trie, uint32_t n, const uint32_t *tokens, const uint64_t *offsets,
                           uint64_t total_tokens, uint32_t *out_ids, void *stream);

/*
 * Replaces LoudsTrie::reverse_lookup (lib/marisa/grimoire/trie/louds-trie.cc:179-210)
 * for a batch, on the device: out_len[i] receives the length of the key whose
 * id is ids[i] (0xFFFFFFFF when ids[i] is not a key id), and its tokens go to
 * out_tokens[i * max_len ...] when that length is at most max_len.  ids (n),
 * out_tokens (n * max_len) and out_len (n) are device pointers; the lookup
 * runs on `stream` and the call returns without waiting.  Requires
 * ft_trie_init_tbs_gpu; the first call derives every node's parent (4 bytes
 * per node, freed with the workspace) and waits for that once.
 */
int ft_reverse_lookup_batch_device(ft_trie *trie, uint32_t n, const uint32_t *ids, uint32_t max_len,
                                   uint32_t *out_tokens, uint32_t *out_len, void *stream);

/* Status word of the device-resident searches and lookups since the last call
 * (0 = clean; the word is cleared by reading it); non-zero bits name the
 * checks that failed inside the kernel. */
int ft_trie_device_status(ft_trie *trie, uint32_t *status);

/*
 * No counterpart in the reference.  The same search as ft_tbs_batch_device,
 * for callers that cannot allocate device memory while they search: code whose
 * host framework owns every device allocation, or request threads that must
 * not stall on cudaMalloc/cudaFree.  It allocates nothing; its scratch is a
 * fixed 8 MiB array in the library, which every GPU that loads the library
 * keeps until exit.  The trie must already be on the device
 * (ft_trie_init_tbs_gpu); the caller passes device inputs and outputs as for
 * ft_tbs_batch_device, with every beam width at most out_capacity.  Batches
 * whose scratch would exceed 8 MiB are rejected with FT_ERR_INVALID_ARG.
 * The first call on a device looks up the array's address; make it before any
 * stream capture.  Calls are serialised per device; each reads the kernel's
 * status word back on `stream` and synchronises `stream` before it returns,
 * so no call can be made inside a stream capture.  All calls share the array, so searches whose GPU work overlapped would race.
 */
int ft_tbs_batch_device_noalloc(ft_trie *trie, const ft_device_batch *batch,
                                const ft_search_params *params, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHTRIE_B200_H_ */
