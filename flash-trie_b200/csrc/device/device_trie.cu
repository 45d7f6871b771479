#include <cuda_runtime.h>
#include <omp.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "cuda_util.hpp"
#include "device_trie.hpp"
#include "tbs_kernel.cuh"

namespace ftb {

void build_hash_index(HostDeviceImage &out, int num_threads);

void derive_device_image(const LoudsLevel &lv, HostDeviceImage &out, int num_threads) {
  if (lv.next) fail(ErrorKind::kState, "MARISA_STATE_ERROR: the GPU search needs a single-trie dictionary (num_tries == 1)");
  if (lv.node_order() != kLabelOrder)
    fail(ErrorKind::kState, "MARISA_STATE_ERROR: the GPU search needs a label-ordered trie (MARISA_LABEL_ORDER)");
  const uint64_t N = lv.num_nodes();
  if (lv.louds.size < 4 || lv.louds.size != 2 * N + 2 || lv.louds.num_1s != N)
    fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: inconsistent LOUDS bit vector");
  if (lv.terminal.size < N || lv.link.size < N || lv.bases.size() != N || lv.extras.size < N)
    fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: node arrays shorter than the node count");
  if (N >= 0xFFFFFFFFull) fail(ErrorKind::kSize, "MARISA_SIZE_ERROR: too many nodes");
  out.num_nodes = N;
  out.binary_tail = lv.binary_tail();
  const uint64_t T = lv.tail.size();
  if (out.binary_tail) {
    if (lv.tail_end_flags.size != T || T == 0 || !lv.tail_end_flags.get(T - 1))
      fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: binary tail end flags do not close the tail");
  } else if (T != 0 && lv.tail[T - 1] != kTailTerminal) {
    fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: text tail does not end with a terminator");
  }

  // child_begin[n] = select0(n) - n: enumerate the zeros of the LOUDS bits.
  out.child_begin.assign(N + 1, 0);
  {
    uint64_t k = 0;  // zeros seen so far
    const uint64_t nbits = lv.louds.size;
    for (uint64_t u = 0; u < lv.louds.units.size() && k <= N; ++u) {
      uint64_t z = ~lv.louds.units[u];
      const uint64_t base = u * 64;
      if (base + 64 > nbits) z &= (nbits - base >= 64) ? ~0ull : ((1ull << (nbits - base)) - 1);
      while (z && k <= N) {
        const uint64_t pos = base + (uint64_t)__builtin_ctzll(z);
        z &= z - 1;
        out.child_begin[k] = (uint32_t)(pos - k);
        ++k;
      }
    }
    if (k <= N || out.child_begin[0] != 1 || out.child_begin[N] != N)
      fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: LOUDS child ranges are inconsistent");
  }

  out.first_label.assign(N, 0);
  out.link_off.assign(N, 0);
  out.flags.assign(N, 0);
  // Link ids are ranks over the link bits; compute per-chunk starting ranks so
  // the chunks can run in parallel.
  const uint64_t chunk = 1 << 20;
  const uint64_t nchunks = (N + chunk - 1) / chunk;
  std::vector<uint64_t> link_rank(nchunks + 1, 0);
  for (uint64_t c = 0; c < nchunks; ++c) link_rank[c + 1] = lv.link.rank1(std::min(N, (c + 1) * chunk));
  if (link_rank[nchunks] > lv.link_extras.size)
    fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: fewer link extras than link nodes");
  bool bad = false;
#pragma omp parallel for schedule(dynamic, 1) num_threads(num_threads) reduction(|| : bad)
  for (int64_t c = 0; c < (int64_t)nchunks; ++c) {
    uint64_t link_id = link_rank[c];
    const uint64_t end = std::min(N, (uint64_t)(c + 1) * chunk);
    for (uint64_t n = (uint64_t)c * chunk; n < end; ++n) {
      uint8_t f = lv.terminal.get(n) ? kNodeTerminal : 0;
      if (lv.link.get(n)) {
        f |= kNodeLink;
        const uint64_t off = lv.link_offset(n, link_id++);
        // The kernel reads tail[off] and tail[off + 1] (text) or tail[off]
        // and the end bit at off (binary); the terminator / end bit that
        // closes the tail bounds every later step of the walk.
        if (out.binary_tail ? (off >= T) : (off + 1 >= T)) {
          bad = true;
        } else {
          out.first_label[n] = lv.tail[off];
          const bool ends1 = out.binary_tail ? lv.tail_end_flags.get(off) : lv.tail[off + 1] == kTailTerminal;
          if (ends1) f |= kNodeLinkEnds1;
        }
        out.link_off[n] = (uint32_t)off;
      } else {
        out.first_label[n] = lv.label(n);
      }
      out.flags[n] = f;
    }
  }
  if (bad) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: link offset outside the tail");
  // Children of a node must be sorted by first label for the binary search
  // (label order); reject anything else rather than search it wrongly.
  bool unsorted = false;
#pragma omp parallel for schedule(static) num_threads(num_threads) reduction(|| : unsorted)
  for (int64_t n = 0; n < (int64_t)N; ++n) {
    const uint32_t b = out.child_begin[n], e = out.child_begin[n + 1];
    if (e < b || e > N) {
      unsorted = true;
      continue;
    }
    for (uint32_t c = b + 1; c < e; ++c)
      if (out.first_label[c - 1] >= out.first_label[c]) unsorted = true;
  }
  if (unsorted)
    fail(ErrorKind::kFormat,
         "MARISA_FORMAT_ERROR: children are not in ascending label order (the GPU search binary-searches them)");
  build_hash_index(out, num_threads);
}

void build_hash_index(HostDeviceImage &out, int num_threads) {
  const uint64_t N = out.num_nodes;
  std::vector<uint32_t> heavy;
  for (uint64_t n = 0; n < N; ++n) {
    const uint32_t d = out.child_begin[n + 1] - out.child_begin[n];
    if (d >= kHashMinDegree && !(out.flags[n] & kNodeLink)) heavy.push_back((uint32_t)n);
  }
  std::vector<uint64_t> base(heavy.size());
  std::vector<uint32_t> lgs(heavy.size());
  uint64_t total = 0;
  size_t used = 0;
  for (; used < heavy.size(); ++used) {
    const uint32_t n = heavy[used];
    const uint64_t d = out.child_begin[n + 1] - out.child_begin[n];
    uint32_t lg = 1;
    while ((1ull << lg) < 2 * d) ++lg;
    if (lg > 31 || total + (1ull << lg) >= 0xFFFFFFFFull) break;  // offsets must fit link_off
    base[used] = total;
    lgs[used] = lg;
    total += 1ull << lg;
  }
  out.hash.assign(2 * total, 0);
#pragma omp parallel for schedule(dynamic, 64) num_threads(num_threads)
  for (int64_t i = 0; i < (int64_t)used; ++i) {
    const uint32_t n = heavy[i];
    const uint32_t lg = lgs[i];
    const uint64_t mask = (1ull << lg) - 1;
    uint32_t *tab = out.hash.data() + 2 * base[i];
    for (uint32_t c = out.child_begin[n]; c < out.child_begin[n + 1]; ++c) {
      const uint32_t lab = out.first_label[c];
      uint64_t h = hash_slot(lab, lg);
      while (tab[2 * h + 1] != 0) h = (h + 1) & mask;
      tab[2 * h] = lab;
      tab[2 * h + 1] = c;
    }
    out.link_off[n] = (uint32_t)base[i];
    out.flags[n] = (uint8_t)(out.flags[n] | kNodeHashed | (lg << 3));
  }
}

void pack_node_records(const HostDeviceImage &img, std::vector<uint32_t> &out, int num_threads) {
  const uint64_t N = img.num_nodes;
  out.assign(4 * N, 0);
#pragma omp parallel for schedule(static) num_threads(num_threads)
  for (int64_t n = 0; n < (int64_t)N; ++n) {
    const uint32_t c0 = img.child_begin[n], d = img.child_begin[n + 1] - c0;
    uint32_t *r = out.data() + 4 * n;
    r[0] = img.first_label[n];
    r[1] = img.link_off[n];
    r[2] = c0;
    r[3] = ((uint32_t)img.flags[n] << 24) | std::min(d, kFanoutMask);
  }
}

DeviceTrie::~DeviceTrie() { release(); }

void DeviceTrie::release() {
  if (device >= 0) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaFree(node);
    cudaFree(term_rank);
    cudaFree(tail);
    cudaFree(tail_end);
    cudaFree(hash);
    if (prev >= 0) cudaSetDevice(prev);
  }
  node = term_rank = tail = nullptr;
  tail_end = nullptr;
  hash = nullptr;
  hash_slots = 0;
  num_keys = 0;
  device = -1;
  bytes = 0;
}

template <typename T>
static T *upload_array(const T *src, uint64_t count, uint64_t &bytes) {
  T *dst = nullptr;
  const uint64_t b = std::max<uint64_t>(count, 1) * sizeof(T) + 16;  // slack: vectorised tail reads
  CUDA_TRY(cudaMalloc(&dst, b));
  CUDA_TRY(cudaMemset(dst, 0, b));
  if (count) CUDA_TRY(cudaMemcpy(dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
  bytes += b;
  return dst;
}

void DeviceTrie::upload(const LoudsLevel &lv, int num_threads) {
  HostDeviceImage img;
  derive_device_image(lv, img, num_threads);
  release();
  CUDA_TRY(cudaGetDevice(&device));
  num_nodes = img.num_nodes;
  tail_size = lv.tail.size();
  binary_tail = img.binary_tail;
  try {
    {
      std::vector<uint32_t> rec;
      pack_node_records(img, rec, num_threads);
      node = upload_array(rec.data(), rec.size(), bytes);
    }
    {
      // Key-id directory over the terminal flags.
      const uint64_t blocks = (num_nodes + 63) / 64;
      if (lv.terminal.units.size() < blocks) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: terminal flags too short");
      std::vector<uint32_t> tr(4 * blocks, 0);
      uint64_t cum = 0;
      for (uint64_t b = 0; b < blocks; ++b) {
        uint64_t bits = lv.terminal.units[b];
        const uint64_t valid = num_nodes - b * 64;
        if (valid < 64) bits &= (1ull << valid) - 1;
        tr[4 * b] = (uint32_t)cum;
        tr[4 * b + 2] = (uint32_t)bits;
        tr[4 * b + 3] = (uint32_t)(bits >> 32);
        cum += (uint64_t)__builtin_popcountll(bits);
      }
      if (cum >= 0xFFFFFFFFull) fail(ErrorKind::kSize, "MARISA_SIZE_ERROR: too many keys for 32-bit key ids");
      num_keys = cum;
      term_rank = upload_array(tr.data(), tr.size(), bytes);
    }
    tail = upload_array(lv.tail.data(), lv.tail.size(), bytes);
    if (binary_tail) tail_end = upload_array(lv.tail_end_flags.units.data(), lv.tail_end_flags.units.size(), bytes);
    hash = upload_array(img.hash.data(), img.hash.size(), bytes);
    hash_slots = img.hash.size() / 2;
    reserve_l2_persisting(device);
  } catch (...) {
    release();
    throw;
  }
}

}  // namespace ftb
