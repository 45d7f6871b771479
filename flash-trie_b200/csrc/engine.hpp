// Search engine: owns the device workspace sized by init_tbs_gpu and runs
// batches either from host buffers (packing, one H2D copy, kernels, one D2H
// copy) or from device-resident buffers on a caller stream.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/flashtrie_b200.h"
#include "device/device_trie.hpp"
#include "device/tbs_kernel.cuh"

namespace ftb {

// Workspace limits, the arguments of init_tbs_gpu
// (lib/marisa/grimoire/trie/tbs-kernels.cu:599-648).
struct EngineLimits {
  uint64_t max_batch = 1;
  uint64_t max_topk = 1024;
  uint64_t max_outpos = 64;
  uint64_t max_out_beams = 8192;
  uint64_t max_out_tokens = 8192 * 64;
  uint64_t max_inter_beams = 1024 * 1024;
  uint64_t radix_topk_threshold = 1024;
};

// Hard limits of the kernel (shared-memory row staging and result sort).
constexpr uint64_t kMaxTopk = 8192;
constexpr uint64_t kMaxBeams = 8192;
constexpr uint64_t kMaxOutpos = 65535;
// Result tokens of a host-buffer batch come back in one copy with the headers
// up to this size, else in a second copy of just the tokens produced.
constexpr size_t kOneCopyTokenBytes = 256 * 1024;

class InvalidArgument : public std::runtime_error {
 public:
  explicit InvalidArgument(const std::string &m) : std::runtime_error(m) {}
};

// Name of the first device pointer of a non-empty batch that is NULL but
// must not be (out_key is optional; the rows may be NULL only when K = 0),
// or nullptr when every required pointer is set.  Both device entry points
// refuse such a batch before anything is launched.
const char *missing_device_batch_field(const ft_device_batch &b);

class Engine {
 public:
  Engine(std::shared_ptr<DeviceTrie> trie, const EngineLimits &lim);
  ~Engine();
  Engine(const Engine &) = delete;
  Engine &operator=(const Engine &) = delete;

  const EngineLimits &limits() const { return lim_; }
  void search_host(const ft_request *reqs, uint32_t n, const ft_search_params &prm, ft_result *out);
  void search_device(const ft_device_batch &b, const ft_search_params &prm, cudaStream_t stream);
  uint32_t read_status();
  // Key ids of n token sequences in device memory, on `stream` (bad offsets
  // and trie inconsistencies go to the same status word as search_device).
  void lookup_device(uint32_t n, const uint32_t *tokens, const uint64_t *offsets, uint64_t total_tokens,
                     uint32_t *out_ids, cudaStream_t stream);
  // Token sequences of n key ids in device memory, on `stream`; the first
  // call derives the nodes' parents (4 bytes per node, kept with the workspace).
  void reverse_lookup_device(uint32_t n, const uint32_t *ids, uint32_t max_len, uint32_t *out_tokens,
                             uint32_t *out_len, cudaStream_t stream);

 private:
  struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
  };
  void *dalloc(size_t bytes);
  void release();
  void validate_request(const ft_request &r) const;
  void fill_params(SearchParams &sp, const ft_search_params &prm, uint32_t n_req) const;

  std::shared_ptr<DeviceTrie> trie_;
  EngineLimits lim_;
  int device_ = -1;
  int max_ctas_ = 1;
  uint32_t n_slots_ = 1;
  size_t smem_ = 0;
  std::vector<DevBuf> allocs_;
  // device workspace
  SlotView *d_slots_ = nullptr;
  uint32_t *d_status_dev_ = nullptr;  // device path: accumulates until read
  uint32_t *d_debug_ = nullptr;       // first failed kernel self-check
  uint32_t *d_parent_ = nullptr;      // parent of every node, derived at the first reverse lookup
  // host-buffer path staging, on device and pinned host: a call's inputs
  // [meta | factor | beams | ids | logp], then its outputs [status, token total |
  // count | phase | lpn | len | key | token base | tok]
  uint8_t *d_io_ = nullptr;
  uint8_t *h_io_ = nullptr;
  size_t in_bytes_ = 0, out_bytes_ = 0;
  // device-path meta/factor staging
  uint8_t *d_dmeta_ = nullptr;
  uint8_t *h_dmeta_ = nullptr;
  size_t dmeta_bytes_ = 0;
  // shape and length norm of what d_dmeta_ holds (n = 0: nothing yet)
  uint32_t dmeta_L_ = 0, dmeta_K_ = 0, dmeta_n_ = 0;
  double dmeta_ln_ = 0.0;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t dmeta_done_ = nullptr;
  std::mutex mu_;
};

}  // namespace ftb
