// ft_tbs_batch_device_noalloc: the device-resident search for callers that
// cannot allocate device memory at search time.
//
// Who needs it: code that runs inside a host framework that owns every device
// allocation (an inference server's memory pool, a plugin whose host forbids
// cudaMalloc on its request path), and latency-critical request threads where a
// cudaMalloc/cudaFree (which synchronises the device and can stall for
// milliseconds) is not acceptable.  Such callers upload the trie once at start-up
// (ft_trie_init_tbs_gpu) and afterwards only pass input and output buffers.
//
// The search's scratch memory (candidates, result pool, beams, history,
// request metadata and the status word) lives in the file-scope array
// below: a fixed kNoAllocScratchBytes that every GPU which loads this library
// keeps until the process exits.  Nothing here calls cudaMalloc, cudaFree or any
// allocating routine.
//
// Rules for callers:
//   * The first call on a device resolves the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.
//   * All calls share the one array, and it keeps the last call's contents
//     (each call clears the status word it reads; everything else is written
//     before it is read).  The entry point serialises its own calls per device;
//     every call reads the status word back on the caller's stream and
//     synchronises that stream before it returns.  Calls whose GPU work
//     overlapped would race on the array.
//   * A batch whose scratch would exceed kNoAllocScratchBytes is rejected with
//     FT_ERR_INVALID_ARG; every beam width must be at most out_capacity.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>

#include "../../../include/flashtrie_b200.h"
#include "cuda_util.hpp"
#include "device_trie.hpp"
#include "tbs_kernel.cuh"

namespace ftb {
std::shared_ptr<DeviceTrie> device_trie_of(ft_trie *t);
void set_last_error(const std::string &m);
const char *missing_device_batch_field(const ft_device_batch &b);
}  // namespace ftb

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr uint32_t kNoAllocMaxOutpos = 255;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Byte offsets of the scratch regions for one call.
struct Layout {
  size_t status, meta, factor, slots, slot0, slot_bytes;
  size_t cand, pool, pool_tmp, beams0, beams1, hist;  // within a slot
  size_t total;
};

Layout plan(uint32_t n, uint32_t L, uint32_t K, uint32_t B, uint32_t n_slots) {
  Layout a;
  size_t o = 0;
  a.status = o;
  o = align256(o + 16);
  a.meta = o;
  o = align256(o + sizeof(ftb::ReqMeta) * n);
  a.factor = o;
  o = align256(o + 8ull * (L + 1));
  a.slots = o;
  o = align256(o + sizeof(ftb::SlotView) * n_slots);
  size_t s = 0;
  a.cand = s;
  s = align256(s + sizeof(ftb::Cand) * (size_t)B * K);
  a.pool = s;
  s = align256(s + sizeof(ftb::Cand) * ((size_t)B + 2 * (size_t)B * K));
  a.pool_tmp = s;
  s = align256(s + sizeof(ftb::Cand) * B);
  a.beams0 = s;
  s = align256(s + sizeof(ftb::Beam) * B);
  a.beams1 = s;
  s = align256(s + sizeof(ftb::Beam) * B);
  a.hist = s;
  s = align256(s + sizeof(ftb::Hist) * (size_t)(L + 1) * B);
  a.slot_bytes = s;
  a.slot0 = o;
  a.total = o + s * n_slots;
  return a;
}

struct FactorTable {
  double f[kNoAllocMaxOutpos + 1];
};

// Writes the per-call metadata into the scratch array (kernel parameters
// carry the values, so no host staging buffer is needed).
__global__ void noalloc_setup_kernel(Layout a, uint32_t n, uint32_t L, uint32_t K, uint32_t n_slots,
                                     FactorTable ft) {
  unsigned char *base = g_noalloc_scratch;
  ftb::ReqMeta *meta = reinterpret_cast<ftb::ReqMeta *>(base + a.meta);
  double *factor = reinterpret_cast<double *>(base + a.factor);
  ftb::SlotView *slots = reinterpret_cast<ftb::SlotView *>(base + a.slots);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
    meta[i] = ftb::ReqMeta{L, K, (uint64_t)i * L, (uint64_t)i * L * K};
  for (uint32_t d = threadIdx.x; d <= L; d += blockDim.x) factor[d] = ft.f[d];
  for (uint32_t s = threadIdx.x; s < n_slots; s += blockDim.x) {
    unsigned char *sb = base + a.slot0 + (size_t)s * a.slot_bytes;
    ftb::SlotView v;
    v.next = reinterpret_cast<ftb::Cand *>(sb + a.cand);
    v.pool = reinterpret_cast<ftb::Cand *>(sb + a.pool);
    v.pool_tmp = reinterpret_cast<ftb::Cand *>(sb + a.pool_tmp);
    v.beams[0] = reinterpret_cast<ftb::Beam *>(sb + a.beams0);
    v.beams[1] = reinterpret_cast<ftb::Beam *>(sb + a.beams1);
    v.hist = reinterpret_cast<ftb::Hist *>(sb + a.hist);
    v.help = nullptr;  // no helper clusters in this search
    slots[s] = v;
  }
  if (threadIdx.x == 0) *reinterpret_cast<uint32_t *>(base + a.status) = 0;  // status starts clean
}

std::mutex g_mu[kMaxDevices];
void *g_addr[kMaxDevices];

// Device address of the scratch array on the current device, resolved once.
unsigned char *scratch_address(int dev) {
  if (!g_addr[dev]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) ftb::throw_cuda(e, "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
    g_addr[dev] = ptr;
  }
  return static_cast<unsigned char *>(g_addr[dev]);
}

}  // namespace

extern "C" int ft_tbs_batch_device_noalloc(ft_trie *trie, const ft_device_batch *b, const ft_search_params *prm,
                                           void *stream_ptr) {
  try {
    if (!trie || !b || !prm) {
      ftb::set_last_error("MARISA_NULL_ERROR: NULL argument");
      return FT_ERR_NULL;
    }
    if (const char *field = ftb::missing_device_batch_field(*b)) {
      ftb::set_last_error(std::string("MARISA_NULL_ERROR: device batch field ") + field + " is NULL");
      return FT_ERR_NULL;
    }
    std::shared_ptr<ftb::DeviceTrie> dt = ftb::device_trie_of(trie);
    if (!dt) {
      ftb::set_last_error("MARISA_STATE_ERROR: upload the trie with init_tbs_gpu before searching");
      return FT_ERR_STATE;
    }
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices || dev != dt->device) {
      ftb::set_last_error("no-allocation search: the current device is not the trie's device");
      return FT_ERR_STATE;
    }
    const uint32_t n = b->n, L = b->num_outpos, K = b->topk, B = b->out_capacity;
    if (n == 0) return FT_OK;
    if (L == 0 || L > kNoAllocMaxOutpos || K > 8192 || B == 0 || B > 8192) {
      ftb::set_last_error("no-allocation search: needs 1 <= L <= 255, K <= 8192, 1 <= out_capacity <= 8192");
      return FT_ERR_INVALID_ARG;
    }
    // As many slots (concurrent requests) as the scratch holds, at least one.
    Layout one = plan(n, L, K, B, 1);
    if (one.total > kNoAllocScratchBytes) {
      ftb::set_last_error("no-allocation search: this batch needs " + std::to_string(one.total) +
                          " bytes of scratch; the fixed scratch is " + std::to_string(kNoAllocScratchBytes) +
                          " bytes (8 MiB) - use ft_tbs_batch_device for larger batches");
      return FT_ERR_INVALID_ARG;
    }
    uint32_t n_slots = std::max<uint32_t>(
        1, std::min<uint32_t>(n, (uint32_t)((kNoAllocScratchBytes - one.slot0) / one.slot_bytes)));
    Layout a = plan(n, L, K, B, n_slots);
    while (a.total > kNoAllocScratchBytes && n_slots > 1) a = plan(n, L, K, B, --n_slots);

    std::lock_guard<std::mutex> lock(g_mu[dev]);
    unsigned char *base = scratch_address(dev);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    FactorTable ft;
    std::memset(&ft, 0, sizeof(ft));
    for (uint32_t d = 0; d <= L; ++d) ft.f[d] = std::pow(6.0 / (5.0 + (double)d), prm->length_norm);
    const size_t smem = ftb::search_smem_bytes(K, B);
    const int max_ctas = ftb::ensure_search_smem(smem);
    noalloc_setup_kernel<<<1, 256, 0, stream>>>(a, n, L, K, n_slots, ft);
    CUDA_TRY(cudaGetLastError());

    ftb::SearchParams sp;
    std::memset(&sp, 0, sizeof(sp));
    sp.trie = ftb::make_trie_view(*dt);
    sp.meta = reinterpret_cast<const ftb::ReqMeta *>(base + a.meta);
    sp.beams = b->beams;
    sp.topk_id = b->topk_id;
    sp.topk_logp = b->topk_logp;
    sp.factor = reinterpret_cast<const double *>(base + a.factor);
    sp.slots = reinterpret_cast<ftb::SlotView *>(base + a.slots);
    sp.cand_cap = (uint64_t)B * K;
    sp.pool_cap = (uint64_t)B + 2 * (uint64_t)B * K;
    sp.beam_cap = B;
    sp.n_req = n;
    sp.n_slots = n_slots;
    sp.token_threshold = (double)prm->token_logp_threshold;
    sp.sent_threshold = prm->sent_logp_threshold;
    sp.early_exit = prm->early_exit ? 1 : 0;
    sp.out_cap = B;
    sp.out_stride = L;
    sp.out_count = b->out_count;
    sp.out_lpn = b->out_lpn;
    sp.out_len = b->out_len;
    sp.out_tok = b->out_tok;
    sp.out_key = b->out_key;
    sp.out_phase_ms = nullptr;
    sp.status = reinterpret_cast<uint32_t *>(base + a.status);
    sp.debug = nullptr;
    const ftb::SearchLaunch plan = ftb::plan_search(n, smem);
    const int grid = (int)std::min<uint32_t>(std::min<uint32_t>(n_slots, (uint32_t)max_ctas), (uint32_t)plan.max_teams);
    ftb::launch_search(sp, smem, grid, stream, plan);
    // The status word comes back on the caller's stream (pageable
    // destination: the copy completes before the synchronisation returns).
    uint32_t status = 0;
    CUDA_TRY(cudaMemcpyAsync(&status, base + a.status, 4, cudaMemcpyDeviceToHost, stream));
    CUDA_TRY(cudaStreamSynchronize(stream));
    if (status != 0) {
      char hex[16];
      std::snprintf(hex, sizeof(hex), "%x", status);
      ftb::set_last_error(std::string("no-allocation search: the kernel reported status 0x") + hex +
                          " (a beam width above out_capacity, or an inconsistent trie image)");
      return FT_ERR_DEVICE;
    }
    ftb::set_last_error("");
    return FT_OK;
  } catch (const ftb::CudaError &e) {
    ftb::set_last_error(e.what());
    return FT_ERR_CUDA;
  } catch (const std::exception &e) {
    ftb::set_last_error(e.what());
    return FT_ERR_DEVICE;
  }
}
