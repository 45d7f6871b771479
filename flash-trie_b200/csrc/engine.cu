#include "engine.hpp"

#include <omp.h>

#include <cmath>
#include <cstring>
#include <string>

#include "device/cuda_util.hpp"

namespace ftb {

namespace {

inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// (6 / (5 + depth)) ^ length_norm for depth 0..max_L, computed on the host so
// device scores are bit-identical to a host computation of the reference
// formula (lib/marisa/grimoire/trie/beam-state.h:24-26).
void fill_factor(double *f, uint32_t max_L, double length_norm) {
  for (uint32_t d = 0; d <= max_L; ++d) f[d] = std::pow(6.0 / (5.0 + (double)d), length_norm);
}

}  // namespace

void *Engine::dalloc(size_t bytes) {
  void *p = nullptr;
  bytes = std::max<size_t>(align16(bytes), 16);
  CUDA_TRY(cudaMalloc(&p, bytes));
  allocs_.push_back(DevBuf{p, bytes});
  return p;
}

Engine::Engine(std::shared_ptr<DeviceTrie> trie, const EngineLimits &lim) : trie_(std::move(trie)), lim_(lim) {
  if (lim.max_batch == 0) throw InvalidArgument("init_tbs_gpu: max_batch_size must be >= 1");
  if (lim.max_topk == 0 || lim.max_topk > kMaxTopk)
    throw InvalidArgument("init_tbs_gpu: max_num_topk must be in [1, " + std::to_string(kMaxTopk) + "]");
  if (lim.max_outpos == 0 || lim.max_outpos > kMaxOutpos)
    throw InvalidArgument("init_tbs_gpu: max_num_outpos must be in [1, " + std::to_string(kMaxOutpos) + "]");
  if (lim.max_out_beams == 0 || lim.max_out_beams > kMaxBeams)
    throw InvalidArgument("init_tbs_gpu: max_num_out_beams must be in [1, " + std::to_string(kMaxBeams) + "]");
  CUDA_TRY(cudaGetDevice(&device_));
  smem_ = search_smem_bytes((uint32_t)lim.max_topk, (uint32_t)lim.max_out_beams);
  max_ctas_ = ensure_search_smem(smem_);
  n_slots_ = (uint32_t)std::min<uint64_t>(lim.max_batch, (uint64_t)max_ctas_);

  const uint64_t B = lim.max_out_beams, K = lim.max_topk, L = lim.max_outpos, NB = lim.max_batch;
  const uint64_t cand_cap = B * K, pool_cap = B + 2 * B * K;
  try {
    std::vector<SlotView> slots(n_slots_);
    for (uint32_t s = 0; s < n_slots_; ++s) {
      slots[s].next = (Cand *)dalloc(sizeof(Cand) * cand_cap);
      slots[s].pool = (Cand *)dalloc(sizeof(Cand) * pool_cap);
      slots[s].pool_tmp = (Cand *)dalloc(sizeof(Cand) * B);
      slots[s].beams[0] = (Beam *)dalloc(sizeof(Beam) * B);
      slots[s].beams[1] = (Beam *)dalloc(sizeof(Beam) * B);
      slots[s].hist = (Hist *)dalloc(sizeof(Hist) * (L + 1) * B);
      // Helper state: zeroed (no epoch, no helper inside), then its step count.
      const size_t hb = help_state_bytes(L);
      slots[s].help = (HelpState *)dalloc(hb);
      CUDA_TRY(cudaMemset(slots[s].help, 0, hb));
      HelpState hs;
      std::memset(&hs, 0, sizeof(hs));
      hs.steps = (uint32_t)L;
      for (int q = 0; q < 2; ++q) hs.xc[q].key_min = 0xFFFFFFFFu;  // clear: empty key ranges
      hs.pool.pool_key_min = 0xFFFFFFFFu;
      CUDA_TRY(cudaMemcpy(slots[s].help, &hs, sizeof(hs), cudaMemcpyHostToDevice));
    }
    d_slots_ = (SlotView *)dalloc(sizeof(SlotView) * n_slots_);
    CUDA_TRY(cudaMemcpy(d_slots_, slots.data(), sizeof(SlotView) * n_slots_, cudaMemcpyHostToDevice));
    d_status_dev_ = (uint32_t *)dalloc(16);
    CUDA_TRY(cudaMemset(d_status_dev_, 0, 16));
    d_debug_ = (uint32_t *)dalloc(64);
    CUDA_TRY(cudaMemset(d_debug_, 0, 64));

    // One staging buffer per side: a call's inputs, then its outputs (whose
    // first 16 bytes, the status and token-total words, travel with the
    // inputs so that the one host-to-device copy also clears them).
    in_bytes_ = align16(sizeof(ReqMeta) * NB) + align16(8 * (L + 1)) + align16(4 * NB * L) + 2 * align16(4 * NB * L * K);
    out_bytes_ = 16 + align16(4 * NB) + align16(8 * 5 * NB) + align16(8 * NB * B) + 2 * align16(4 * NB * B) +
                 align16(8 * NB) +
                 align16(4 * NB * B * L);
    d_io_ = (uint8_t *)dalloc(in_bytes_ + out_bytes_);
    CUDA_TRY(cudaMallocHost(&h_io_, in_bytes_ + out_bytes_));
    dmeta_bytes_ = align16(sizeof(ReqMeta) * NB) + align16(8 * (L + 1));
    d_dmeta_ = (uint8_t *)dalloc(dmeta_bytes_);
    CUDA_TRY(cudaMallocHost(&h_dmeta_, dmeta_bytes_));
    CUDA_TRY(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    CUDA_TRY(cudaEventCreateWithFlags(&dmeta_done_, cudaEventDisableTiming));
  } catch (...) {
    release();
    throw;
  }
}

Engine::~Engine() { release(); }

void Engine::release() {
  int prev = -1;
  cudaGetDevice(&prev);
  if (device_ >= 0) cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  for (auto &a : allocs_) cudaFree(a.p);
  allocs_.clear();
  if (h_io_) cudaFreeHost(h_io_);
  if (h_dmeta_) cudaFreeHost(h_dmeta_);
  if (dmeta_done_) cudaEventDestroy(dmeta_done_);
  if (stream_) cudaStreamDestroy(stream_);
  h_io_ = h_dmeta_ = nullptr;
  stream_ = nullptr;
  dmeta_done_ = nullptr;
  if (prev >= 0) cudaSetDevice(prev);
}

void Engine::validate_request(const ft_request &r) const {
  if (r.num_outpos == 0) throw InvalidArgument("tbs: beams must not be empty");
  if (r.num_outpos > lim_.max_outpos)
    throw InvalidArgument("tbs: len(beams) = " + std::to_string(r.num_outpos) + " exceeds max_num_outpos = " +
                          std::to_string(lim_.max_outpos));
  if (r.topk > lim_.max_topk)
    throw InvalidArgument("tbs: top-k row length " + std::to_string(r.topk) + " exceeds max_num_topk = " +
                          std::to_string(lim_.max_topk));
  for (uint32_t t = 0; t < r.num_outpos; ++t)
    if (r.beams[t] > lim_.max_out_beams)
      throw InvalidArgument("tbs: beam width " + std::to_string(r.beams[t]) + " exceeds max_num_out_beams = " +
                            std::to_string(lim_.max_out_beams));
}

void Engine::fill_params(SearchParams &sp, const ft_search_params &prm, uint32_t n_req) const {
  std::memset(&sp, 0, sizeof(sp));
  sp.trie = make_trie_view(*trie_);
  sp.slots = d_slots_;
  sp.cand_cap = lim_.max_out_beams * lim_.max_topk;
  sp.pool_cap = lim_.max_out_beams + 2 * lim_.max_out_beams * lim_.max_topk;
  sp.beam_cap = (uint32_t)lim_.max_out_beams;
  sp.n_req = n_req;
  sp.n_slots = n_slots_;
  // The reference binds token_logp_threshold as float and compares it as a
  // double (tools/bindings.cpp:50, beam-search-state.h:158).
  sp.token_threshold = (double)prm.token_logp_threshold;
  sp.sent_threshold = prm.sent_logp_threshold;
  sp.early_exit = prm.early_exit ? 1 : 0;
  sp.debug = d_debug_;  // the caller sets sp.status
}

void Engine::search_host(const ft_request *reqs, uint32_t n, const ft_search_params &prm, ft_result *out) {
  std::lock_guard<std::mutex> lock(mu_);
  if (n > lim_.max_batch)
    throw InvalidArgument("bs_tbs_gpu: batch_size " + std::to_string(n) + " exceeds max_batch_size = " +
                          std::to_string(lim_.max_batch));
  uint32_t max_L = 0, max_K = 1, cap = 1, max_beam = 0;
  uint64_t sum_L = 0, sum_LK = 0;
  for (uint32_t i = 0; i < n; ++i) {
    validate_request(reqs[i]);
    for (uint32_t t = 0; t < reqs[i].num_outpos; ++t) max_beam = std::max(max_beam, reqs[i].beams[t]);
    if (out[i].capacity < reqs[i].beams[reqs[i].num_outpos - 1] || out[i].stride < reqs[i].num_outpos)
      throw InvalidArgument("tbs: result buffer too small");
    max_L = std::max(max_L, reqs[i].num_outpos);
    max_K = std::max(max_K, reqs[i].topk);
    cap = std::max(cap, reqs[i].beams[reqs[i].num_outpos - 1]);
    sum_L += reqs[i].num_outpos;
    sum_LK += (uint64_t)reqs[i].num_outpos * reqs[i].topk;
  }
  for (uint32_t i = 0; i < n; ++i) {
    out[i].num_beams = 0;
    for (int k = 0; k < 5; ++k) out[i].phase_ms[k] = 0.0;
  }
  if (n == 0) return;
  CUDA_TRY(cudaSetDevice(device_));

  // Pack [meta | factor | beams | ids | logp] into pinned memory.
  const size_t o_meta = 0, o_fac = align16(sizeof(ReqMeta) * n), o_beams = o_fac + align16(8 * (max_L + 1)),
               o_ids = o_beams + align16(4 * sum_L), o_lp = o_ids + align16(4 * sum_LK),
               in_used = o_lp + align16(4 * sum_LK);
  ReqMeta *meta = reinterpret_cast<ReqMeta *>(h_io_ + o_meta);
  fill_factor(reinterpret_cast<double *>(h_io_ + o_fac), max_L, prm.length_norm);
  uint32_t *hb = reinterpret_cast<uint32_t *>(h_io_ + o_beams);
  uint32_t *hid = reinterpret_cast<uint32_t *>(h_io_ + o_ids);
  float *hlp = reinterpret_cast<float *>(h_io_ + o_lp);
  uint64_t bo = 0, ro = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const ft_request &r = reqs[i];
    meta[i] = ReqMeta{r.num_outpos, r.topk, bo, ro};
    bo += r.num_outpos;
    ro += (uint64_t)r.num_outpos * r.topk;
  }
  // Large batches are copied into the pinned buffer by several threads.
  const int pack_threads = sum_LK * 8 > (4u << 20) ? std::min(16, omp_get_max_threads()) : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(pack_threads)
  for (int64_t i = 0; i < (int64_t)n; ++i) {
    const ft_request &r = reqs[i];
    std::memcpy(hb + meta[i].beams_off, r.beams, 4ull * r.num_outpos);
    const uint64_t lk = (uint64_t)r.num_outpos * r.topk;
    if (lk) {
      std::memcpy(hid + meta[i].rows_off, r.topk_id, 4 * lk);
      std::memcpy(hlp + meta[i].rows_off, r.topk_logp, 4 * lk);
    }
  }
  // Output region [status, token total | count | phase | lpn | len | key | token base | tok] for
  // this batch, right after the inputs; tokens are written compactly (each request's at the base
  // it reserves), so only the tokens actually produced need to come back.  The status and
  // token-total words go down zeroed with the inputs.
  uint8_t *const d_out = d_io_ + in_used, *const h_out = h_io_ + in_used;
  std::memset(h_out, 0, 16);
  CUDA_TRY(cudaMemcpyAsync(d_io_, h_io_, in_used + 16, cudaMemcpyHostToDevice, stream_));

  const uint32_t stride = max_L;
  bool want_keys = false;
  for (uint32_t i = 0; i < n; ++i) want_keys |= out[i].key_ids != nullptr;
  const size_t q_count = 16, q_phase = q_count + align16(4 * n), q_lpn = q_phase + align16(8 * 5 * n),
               q_len = q_lpn + align16(8ull * n * cap), q_key = q_len + align16(4ull * n * cap),
               q_base = q_key + (want_keys ? align16(4ull * n * cap) : 0), q_tok = q_base + align16(8ull * n),
               tok_bytes_max = 4ull * n * cap * stride;

  SearchParams sp;
  fill_params(sp, prm, n);
  sp.status = reinterpret_cast<uint32_t *>(d_out);
  sp.meta = reinterpret_cast<const ReqMeta *>(d_io_ + o_meta);
  sp.factor = reinterpret_cast<const double *>(d_io_ + o_fac);
  sp.beams = reinterpret_cast<const uint32_t *>(d_io_ + o_beams);
  sp.topk_id = reinterpret_cast<const uint32_t *>(d_io_ + o_ids);
  sp.topk_logp = reinterpret_cast<const float *>(d_io_ + o_lp);
  sp.out_cap = cap;
  sp.out_stride = stride;
  sp.out_count = reinterpret_cast<uint32_t *>(d_out + q_count);
  sp.out_phase_ms = reinterpret_cast<double *>(d_out + q_phase);
  sp.out_lpn = reinterpret_cast<double *>(d_out + q_lpn);
  sp.out_len = reinterpret_cast<uint32_t *>(d_out + q_len);
  sp.out_tok = reinterpret_cast<uint32_t *>(d_out + q_tok);
  sp.out_key = want_keys ? reinterpret_cast<uint32_t *>(d_out + q_key) : nullptr;
  sp.tok_total = reinterpret_cast<uint64_t *>(d_out + 8);
  sp.out_tok_base = reinterpret_cast<uint64_t *>(d_out + q_base);
  const SearchLaunch plan = plan_search(n, smem_);
  const int grid = search_grid(sp, n, n_slots_, plan, helpers_pay(max_K, max_beam));
  launch_search(sp, smem_, grid, stream_, plan);
  // Small batches: everything in one copy.  Large ones: the headers first,
  // then only the tokens produced.
  const bool two_phase = tok_bytes_max > kOneCopyTokenBytes;
  CUDA_TRY(cudaMemcpyAsync(h_out, d_out, two_phase ? q_tok : q_tok + tok_bytes_max, cudaMemcpyDeviceToHost,
                           stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  const uint64_t tok_total = *reinterpret_cast<const uint64_t *>(h_out + 8);
  if (tok_total * 4 > tok_bytes_max) throw std::runtime_error("tbs: the search kernel reported an invalid token total");
  if (two_phase && tok_total) {
    CUDA_TRY(cudaMemcpyAsync(h_out + q_tok, d_out + q_tok, 4 * tok_total, cudaMemcpyDeviceToHost, stream_));
    CUDA_TRY(cudaStreamSynchronize(stream_));
  }

  const uint32_t status = *reinterpret_cast<const uint32_t *>(h_out);
  if (status != 0) {
    uint32_t dbg[8] = {0};
    CUDA_TRY(cudaMemcpy(dbg, d_debug_, sizeof(dbg), cudaMemcpyDeviceToHost));
    std::string d;
    for (int i = 0; i < 8; ++i) d += (i ? "," : "") + std::to_string(dbg[i]);
    throw std::runtime_error("tbs: the search kernel reported a failed self-check (status " + std::to_string(status) +
                             ", detail " + d + ")");
  }
  const uint32_t *hcount = reinterpret_cast<const uint32_t *>(h_out + q_count);
  const double *hphase = reinterpret_cast<const double *>(h_out + q_phase);
  const double *hlpn = reinterpret_cast<const double *>(h_out + q_lpn);
  const uint32_t *hlen = reinterpret_cast<const uint32_t *>(h_out + q_len);
  const uint64_t *hbase = reinterpret_cast<const uint64_t *>(h_out + q_base);
  const uint32_t *hkey = reinterpret_cast<const uint32_t *>(h_out + q_key);
  const uint32_t *htok = reinterpret_cast<const uint32_t *>(h_out + q_tok);
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t nb = hcount[i];
    ft_result &r = out[i];
    r.num_beams = nb;
    for (int k = 0; k < 5; ++k) r.phase_ms[k] = hphase[5 * i + k];
    uint64_t off = nb ? hbase[i] : 0;
    for (uint32_t b = 0; b < nb; ++b) {
      const uint64_t s = (uint64_t)i * cap + b;
      r.logp_norm[b] = hlpn[s];
      const uint32_t len = hlen[s];
      if (len > r.stride || off + len > tok_total)
        throw std::runtime_error("tbs: the search kernel returned an inconsistent result layout");
      r.lengths[b] = len;
      if (r.key_ids) r.key_ids[b] = hkey[s];
      std::memcpy(r.tokens + (uint64_t)b * r.stride, htok + off, 4ull * len);
      off += len;
    }
  }
}

const char *missing_device_batch_field(const ft_device_batch &b) {
  if (b.n == 0) return nullptr;
  if (!b.beams) return "beams";
  if (b.topk && !b.topk_id) return "topk_id";
  if (b.topk && !b.topk_logp) return "topk_logp";
  if (!b.out_count) return "out_count";
  if (!b.out_lpn) return "out_lpn";
  if (!b.out_len) return "out_len";
  if (!b.out_tok) return "out_tok";
  return nullptr;
}

void Engine::search_device(const ft_device_batch &b, const ft_search_params &prm, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(mu_);
  if (b.n > lim_.max_batch)
    throw InvalidArgument("batch of " + std::to_string(b.n) + " exceeds max_batch_size = " +
                          std::to_string(lim_.max_batch));
  if (b.num_outpos == 0 || b.num_outpos > lim_.max_outpos || b.topk > lim_.max_topk)
    throw InvalidArgument("device batch shape exceeds the workspace limits");
  if (b.n == 0) return;
  CUDA_TRY(cudaSetDevice(device_));
  const uint32_t L = b.num_outpos, K = b.topk;
  // The meta table depends only on the shape, the factor table only on the
  // length norm: a call like the last one (whose copy has landed, as the
  // event says) reuses what is on the device.  The factors sit after room
  // for max_batch meta records, so a smaller batch of the same shape reuses
  // a prefix of the meta table.
  CUDA_TRY(cudaEventSynchronize(dmeta_done_));
  const size_t o_fac = align16(sizeof(ReqMeta) * lim_.max_batch);
  if (!(dmeta_L_ == L && dmeta_K_ == K && dmeta_n_ >= b.n &&
        std::memcmp(&dmeta_ln_, &prm.length_norm, sizeof(double)) == 0)) {
    ReqMeta *meta = reinterpret_cast<ReqMeta *>(h_dmeta_);
    for (uint32_t i = 0; i < b.n; ++i) meta[i] = ReqMeta{L, K, (uint64_t)i * L, (uint64_t)i * L * K};
    fill_factor(reinterpret_cast<double *>(h_dmeta_ + o_fac), L, prm.length_norm);
    CUDA_TRY(cudaMemcpyAsync(d_dmeta_, h_dmeta_, sizeof(ReqMeta) * b.n, cudaMemcpyHostToDevice, stream));
    CUDA_TRY(cudaMemcpyAsync(d_dmeta_ + o_fac, h_dmeta_ + o_fac, 8 * (L + 1), cudaMemcpyHostToDevice, stream));
    CUDA_TRY(cudaEventRecord(dmeta_done_, stream));
    dmeta_L_ = L;
    dmeta_K_ = K;
    dmeta_n_ = b.n;
    dmeta_ln_ = prm.length_norm;
  }

  SearchParams sp;
  fill_params(sp, prm, b.n);
  sp.meta = reinterpret_cast<const ReqMeta *>(d_dmeta_);
  sp.factor = reinterpret_cast<const double *>(d_dmeta_ + o_fac);
  sp.beams = b.beams;
  sp.topk_id = b.topk_id;
  sp.topk_logp = b.topk_logp;
  sp.out_cap = b.out_capacity;
  sp.out_stride = L;
  sp.out_count = b.out_count;
  sp.out_lpn = b.out_lpn;
  sp.out_len = b.out_len;
  sp.out_tok = b.out_tok;
  sp.out_key = b.out_key;
  sp.out_phase_ms = nullptr;
  sp.status = d_status_dev_;
  const SearchLaunch plan = plan_search(b.n, smem_);
  // The beam widths are in device memory: the output capacity (at least the
  // final width) stands in for them.
  const int grid = search_grid(sp, b.n, n_slots_, plan, helpers_pay(b.topk, b.out_capacity));
  launch_search(sp, smem_, grid, stream, plan);
}

void Engine::lookup_device(uint32_t n, const uint32_t *tokens, const uint64_t *offsets, uint64_t total_tokens,
                           uint32_t *out_ids, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(mu_);
  if (n == 0) return;
  if (!tokens && total_tokens) throw InvalidArgument("lookup: tokens is NULL");
  if (!offsets || !out_ids) throw InvalidArgument("lookup: offsets and out_ids must not be NULL");
  CUDA_TRY(cudaSetDevice(device_));
  launch_lookup(make_trie_view(*trie_), tokens, offsets, n, total_tokens, out_ids, d_status_dev_, stream);
}

void Engine::reverse_lookup_device(uint32_t n, const uint32_t *ids, uint32_t max_len, uint32_t *out_tokens,
                                   uint32_t *out_len, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(mu_);
  if (n == 0) return;
  if (!ids || !out_len || (max_len && !out_tokens))
    throw InvalidArgument("reverse_lookup: ids, out_len and out_tokens must not be NULL");
  CUDA_TRY(cudaSetDevice(device_));
  const TrieView tv = make_trie_view(*trie_);
  if (!d_parent_) {
    uint32_t *p = (uint32_t *)dalloc(sizeof(uint32_t) * std::max<uint64_t>(trie_->num_nodes, 1));
    CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(uint32_t) * std::max<uint64_t>(trie_->num_nodes, 1), stream_));
    launch_parents(tv, p, d_status_dev_, stream_);
    CUDA_TRY(cudaStreamSynchronize(stream_));
    d_parent_ = p;
  }
  launch_reverse_lookup(tv, d_parent_, trie_->num_keys, ids, n, max_len, out_tokens, out_len, d_status_dev_, stream);
}

uint32_t Engine::read_status() {
  std::lock_guard<std::mutex> lock(mu_);
  uint32_t s = 0;
  CUDA_TRY(cudaSetDevice(device_));
  CUDA_TRY(cudaDeviceSynchronize());
  CUDA_TRY(cudaMemcpy(&s, d_status_dev_, 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemset(d_status_dev_, 0, 4));
  return s;
}

}  // namespace ftb
