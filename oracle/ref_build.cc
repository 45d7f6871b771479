// Builds a trie file with the UNMODIFIED reference builder (marisa::Keyset +
// marisa::Trie::build + save, linked from the reference's own sources by
// oracle/ref.mk) from a flat key list:
//
//   ref_build <tokens.u32> <offsets.u64> <out.bin>
//
// tokens.u32  : raw little-endian uint32 labels of all keys, concatenated
// offsets.u64 : raw little-endian uint64, n+1 entries, key i is
//               tokens[offsets[i] .. offsets[i+1])
//
// The keys are pushed and built exactly as the reference's pybind
// `Trie.build(token_rows)` does (tools/bindings.cpp:10-22: one push_back per
// row, flags 1 | MARISA_DEFAULT_TAIL | MARISA_LABEL_ORDER |
// MARISA_DEFAULT_CACHE), without the Python list of lists that binding needs,
// which does not fit in memory at 10^8+ keys.
//
// Test and benchmark infrastructure only: bench.py's reference arm builds the
// trie it searches with this program, so that arm runs the reference's code
// alone; the product never runs it.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include <marisa.h>

namespace {

bool read_file(const char *path, std::vector<char> *out) {
  std::FILE *f = std::fopen(path, "rb");
  if (f == nullptr) return false;
  std::fseek(f, 0, SEEK_END);
  const long size = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  out->resize(static_cast<std::size_t>(size));
  const std::size_t got = size > 0 ? std::fread(out->data(), 1, out->size(), f) : 0;
  std::fclose(f);
  return got == out->size();
}

}  // namespace

int main(int argc, char **argv) {
  if (argc != 4) {
    std::fprintf(stderr, "usage: %s <tokens.u32> <offsets.u64> <out.bin>\n", argv[0]);
    return 2;
  }
  std::vector<char> tok_raw, off_raw;
  if (!read_file(argv[1], &tok_raw) || !read_file(argv[2], &off_raw)) {
    std::fprintf(stderr, "ref_build: cannot read the key files\n");
    return 3;
  }
  if (tok_raw.size() % 4 != 0 || off_raw.size() % 8 != 0 || off_raw.size() < 8) {
    std::fprintf(stderr, "ref_build: key files have the wrong size\n");
    return 3;
  }
  const auto *tok = reinterpret_cast<const marisa::UInt32 *>(tok_raw.data());
  const auto *off = reinterpret_cast<const std::uint64_t *>(off_raw.data());
  const std::size_t n = off_raw.size() / 8 - 1;
  const std::size_t n_tok = tok_raw.size() / 4;
  if (off[0] != 0 || off[n] != n_tok) {
    std::fprintf(stderr, "ref_build: offsets do not cover the tokens\n");
    return 3;
  }
  const auto t0 = std::chrono::steady_clock::now();
  try {
    marisa::Keyset keyset;
    for (std::size_t i = 0; i < n; ++i) {
      if (off[i + 1] < off[i] || off[i + 1] > n_tok) {
        std::fprintf(stderr, "ref_build: offsets are not monotone at key %zu\n", i);
        return 3;
      }
      keyset.push_back(tok + off[i], static_cast<std::size_t>(off[i + 1] - off[i]));
    }
    // The token arrays are no longer needed once the keyset holds its copy.
    std::vector<char>().swap(tok_raw);
    std::vector<char>().swap(off_raw);
    marisa::Trie trie;
    trie.build(keyset, 1 | MARISA_DEFAULT_TAIL | MARISA_LABEL_ORDER | MARISA_DEFAULT_CACHE);
    trie.save(argv[3]);
    const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::printf("{\"keys\": %zu, \"num_keys\": %zu, \"nodes\": %zu, \"io_size\": %zu, \"build_s\": %.3f}\n",
                n, trie.num_keys(), trie.num_nodes(), trie.io_size(), s);
  } catch (const marisa::Exception &ex) {
    std::fprintf(stderr, "ref_build: %s\n", ex.what());
    return 4;
  }
  return 0;
}
