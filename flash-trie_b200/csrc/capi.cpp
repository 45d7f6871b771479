// extern "C" entry points of libftcore (declared in include/flashtrie_b200.h).
// Each wraps the C++ implementation, turns exceptions into status codes and
// keeps the message for ft_last_error().
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>

#include "../../include/flashtrie_b200.h"
#include "device/cuda_util.hpp"
#include "device/device_trie.hpp"
#include "engine.hpp"
#include "host/marisa_image.hpp"

struct ft_trie {
  std::unique_ptr<ftb::LoudsLevel> image;
  std::shared_ptr<ftb::DeviceTrie> dev;
  std::unique_ptr<ftb::Engine> engine;
  std::mutex mu;
};

namespace ftb {
// Device image of a trie handle (nullptr before init_tbs_gpu); used by the
// no-allocation entry point in device/noalloc.cu.
std::shared_ptr<DeviceTrie> device_trie_of(ft_trie *t) {
  if (!t) return nullptr;
  std::lock_guard<std::mutex> lock(t->mu);
  return t->dev;
}
void set_last_error(const std::string &m);
}  // namespace ftb

namespace {

thread_local std::string g_last_error;

int host_threads() {
  const unsigned n = std::thread::hardware_concurrency();
  return (int)std::max(1u, std::min(n, 64u));
}

int code_of(ftb::ErrorKind k) {
  switch (k) {
    case ftb::ErrorKind::kState: return FT_ERR_STATE;
    case ftb::ErrorKind::kNull: return FT_ERR_NULL;
    case ftb::ErrorKind::kBound: return FT_ERR_BOUND;
    case ftb::ErrorKind::kRange: return FT_ERR_RANGE;
    case ftb::ErrorKind::kCode: return FT_ERR_CODE;
    case ftb::ErrorKind::kReset: return FT_ERR_STATE;
    case ftb::ErrorKind::kSize: return FT_ERR_SIZE;
    case ftb::ErrorKind::kMemory: return FT_ERR_MEMORY;
    case ftb::ErrorKind::kIO: return FT_ERR_IO;
    case ftb::ErrorKind::kFormat: return FT_ERR_FORMAT;
  }
  return FT_ERR_STATE;
}

template <typename F>
int guarded(F &&f) {
  try {
    f();
    g_last_error.clear();
    return FT_OK;
  } catch (const ftb::FormatError &e) {
    g_last_error = e.what();
    return code_of(e.kind());
  } catch (const ftb::InvalidArgument &e) {
    g_last_error = e.what();
    return FT_ERR_INVALID_ARG;
  } catch (const ftb::CudaError &e) {
    g_last_error = e.what();
    return FT_ERR_CUDA;
  } catch (const std::bad_alloc &) {
    g_last_error = "MARISA_MEMORY_ERROR: std::bad_alloc";
    return FT_ERR_MEMORY;
  } catch (const std::exception &e) {
    g_last_error = e.what();
    return FT_ERR_DEVICE;
  }
}

void require_trie(const ft_trie *t) {
  if (t == nullptr) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: trie handle is NULL");
  if (!t->image) ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: trie_.get() == NULL");
}

void drop_device(ft_trie *t) {
  t->engine.reset();
  t->dev.reset();
}

}  // namespace

void ftb::set_last_error(const std::string &m) { g_last_error = m; }

extern "C" {

const char *ft_last_error(void) { return g_last_error.c_str(); }

int ft_trie_create(ft_trie **out) {
  return guarded([&] {
    if (!out) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: out is NULL");
    *out = new ft_trie();
  });
}

void ft_trie_destroy(ft_trie *trie) { delete trie; }

int ft_trie_load(ft_trie *trie, const char *path) {
  return guarded([&] {
    if (!trie || !path) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: NULL argument");
    std::unique_ptr<ftb::LoudsLevel> img = ftb::read_image_file(path);
    std::lock_guard<std::mutex> lock(trie->mu);
    drop_device(trie);
    trie->image = std::move(img);
  });
}

int ft_trie_mmap(ft_trie *trie, const char *path) {
  return guarded([&] {
    if (!trie || !path) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: NULL argument");
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) ftb::fail(ftb::ErrorKind::kIO, std::string("MARISA_IO_ERROR: failed to open file: ") + path);
    struct stat st;
    if (::fstat(fd, &st) != 0) {
      ::close(fd);
      ftb::fail(ftb::ErrorKind::kIO, std::string("MARISA_IO_ERROR: failed to stat file: ") + path);
    }
    const size_t n = (size_t)st.st_size;
    void *p = n ? ::mmap(nullptr, n, PROT_READ, MAP_SHARED, fd, 0) : nullptr;
    ::close(fd);
    if (n && p == MAP_FAILED) ftb::fail(ftb::ErrorKind::kIO, std::string("MARISA_IO_ERROR: failed to map file: ") + path);
    std::unique_ptr<ftb::LoudsLevel> img;
    try {
      img = ftb::read_image(static_cast<const uint8_t *>(p), n);
    } catch (...) {
      if (n) ::munmap(p, n);
      throw;
    }
    if (n) ::munmap(p, n);
    std::lock_guard<std::mutex> lock(trie->mu);
    drop_device(trie);
    trie->image = std::move(img);
  });
}

int ft_trie_build(ft_trie *trie, const uint32_t *tokens, const uint64_t *offsets, uint64_t num_rows) {
  return guarded([&] {
    if (!trie || !offsets || (!tokens && num_rows && offsets[num_rows] != 0))
      ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: NULL argument");
    for (uint64_t i = 0; i < num_rows; ++i)
      if (offsets[i + 1] < offsets[i]) ftb::fail(ftb::ErrorKind::kRange, "MARISA_RANGE_ERROR: offsets must not decrease");
    std::unique_ptr<ftb::LoudsLevel> img = ftb::build_image(tokens, offsets, num_rows, host_threads());
    std::lock_guard<std::mutex> lock(trie->mu);
    drop_device(trie);
    trie->image = std::move(img);
  });
}

int ft_trie_save(const ft_trie *trie, const char *path) {
  return guarded([&] {
    require_trie(trie);
    if (!path) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: filename is NULL");
    ftb::write_image_file(*trie->image, path);
  });
}

int ft_trie_clear(ft_trie *trie) {
  return guarded([&] {
    if (!trie) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: trie handle is NULL");
    std::lock_guard<std::mutex> lock(trie->mu);
    drop_device(trie);
    trie->image.reset();
  });
}

int ft_trie_get_info(const ft_trie *trie, ft_trie_info *out) {
  return guarded([&] {
    require_trie(trie);
    if (!out) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: out is NULL");
    const ftb::LoudsLevel &lv = *trie->image;
    out->num_keys = lv.num_keys();
    out->num_nodes = lv.num_nodes();
    out->num_tries = lv.num_tries();
    out->total_size = lv.total_size();
    out->io_size = 16 + lv.io_size_body();
    out->tail_mode = lv.tail_mode();
    out->node_order = lv.node_order();
  });
}

int ft_trie_init_tbs_gpu(ft_trie *trie, uint64_t max_batch_size, uint64_t max_num_topk, uint64_t max_num_outpos,
                         uint64_t max_num_out_beams, uint64_t max_num_out_tokens, uint64_t max_num_inter_beams,
                         uint64_t radix_topk_threshold) {
  return guarded([&] {
    require_trie(trie);
    std::lock_guard<std::mutex> lock(trie->mu);
    trie->engine.reset();
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (!trie->dev || trie->dev->device != dev) {
      auto d = std::make_shared<ftb::DeviceTrie>();
      d->upload(*trie->image, host_threads());
      trie->dev = std::move(d);
    }
    ftb::EngineLimits lim;
    lim.max_batch = max_batch_size;
    lim.max_topk = max_num_topk;
    lim.max_outpos = max_num_outpos;
    lim.max_out_beams = max_num_out_beams;
    lim.max_out_tokens = max_num_out_tokens;
    lim.max_inter_beams = max_num_inter_beams;
    lim.radix_topk_threshold = radix_topk_threshold;
    trie->engine.reset(new ftb::Engine(trie->dev, lim));
  });
}

int ft_trie_get_max_batch_size(const ft_trie *trie, uint64_t *out) {
  return guarded([&] {
    require_trie(trie);
    if (!out) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: out is NULL");
    *out = trie->engine ? trie->engine->limits().max_batch : 0;
  });
}

int ft_tbs_batch(ft_trie *trie, const ft_request *requests, uint32_t n, const ft_search_params *params,
                 ft_result *results) {
  return guarded([&] {
    require_trie(trie);
    if ((!requests || !results) && n) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: NULL argument");
    if (!params) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: params is NULL");
    if (!trie->engine)
      ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: init_tbs_gpu must be called before a GPU search");
    trie->engine->search_host(requests, n, *params, results);
  });
}

int ft_tbs_batch_device(ft_trie *trie, const ft_device_batch *batch, const ft_search_params *params, void *stream) {
  return guarded([&] {
    require_trie(trie);
    if (!batch || !params) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: NULL argument");
    if (const char *field = ftb::missing_device_batch_field(*batch))
      ftb::fail(ftb::ErrorKind::kNull, std::string("MARISA_NULL_ERROR: device batch field ") + field + " is NULL");
    if (!trie->engine)
      ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: init_tbs_gpu must be called before a GPU search");
    trie->engine->search_device(*batch, *params, static_cast<cudaStream_t>(stream));
  });
}

int ft_lookup_batch_device(ft_trie *trie, uint32_t n, const uint32_t *tokens, const uint64_t *offsets,
                           uint64_t total_tokens, uint32_t *out_ids, void *stream) {
  return guarded([&] {
    require_trie(trie);
    if (!trie->engine)
      ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: init_tbs_gpu must be called before a GPU lookup");
    trie->engine->lookup_device(n, tokens, offsets, total_tokens, out_ids, static_cast<cudaStream_t>(stream));
  });
}

int ft_reverse_lookup_batch_device(ft_trie *trie, uint32_t n, const uint32_t *ids, uint32_t max_len,
                                   uint32_t *out_tokens, uint32_t *out_len, void *stream) {
  return guarded([&] {
    require_trie(trie);
    if (!trie->engine)
      ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: init_tbs_gpu must be called before a GPU lookup");
    trie->engine->reverse_lookup_device(n, ids, max_len, out_tokens, out_len, static_cast<cudaStream_t>(stream));
  });
}

int ft_trie_device_status(ft_trie *trie, uint32_t *status) {
  return guarded([&] {
    require_trie(trie);
    if (!status) ftb::fail(ftb::ErrorKind::kNull, "MARISA_NULL_ERROR: status is NULL");
    if (!trie->engine) ftb::fail(ftb::ErrorKind::kState, "MARISA_STATE_ERROR: no GPU workspace");
    *status = trie->engine->read_status();
  });
}

}  // extern "C"
