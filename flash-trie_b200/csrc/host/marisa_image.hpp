// In-memory model of a MARISA (FlashTrie) trie file: the succinct structures
// exactly as they are serialised, so that load -> save reproduces the input
// byte for byte and a freshly built trie serialises to the same bytes as the
// reference builder.
//
// Serialised layout (all little-endian, every "Vector" is a u64 byte count
// followed by the payload zero-padded to 8 bytes):
//   header        16 bytes "We love Marisa.\0"   (grimoire/trie/header.h:38-41)
//   louds         BitVector                      (louds-trie.cc:748-762 order)
//   terminal      BitVector
//   link          BitVector
//   bases         Vector<u16>
//   extras        FlatVector
//   link_extras   FlatVector
//   tail          Vector<u32> buf + BitVector end_flags (tail.cc:316-319)
//   [next trie]   same record again without header (multi-trie files only)
//   cache         Vector<12-byte Cache>          (cache.h:75-81)
//   num_l1_nodes  u32
//   config flags  u32
// BitVector = Vector<u64> units, u32 size, u32 num_1s, Vector<RankIndex(12B)>,
//   Vector<u32> select0s, Vector<u32> select1s   (vector/bit-vector.h:219-226)
// FlatVector = Vector<u64> units, u32 value_size, u32 mask, u64 size
//   (vector/flat-vector.h:175-180)
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace ftb {

// Error categories mirror marisa_error_code (include/marisa/base.h:79-91) so the
// C-ABI can report the same class of failure the reference throws.
enum class ErrorKind { kState, kNull, kBound, kRange, kCode, kReset, kSize, kMemory, kIO, kFormat };

class FormatError : public std::runtime_error {
 public:
  FormatError(ErrorKind kind, const std::string &msg) : std::runtime_error(msg), kind_(kind) {}
  ErrorKind kind() const { return kind_; }

 private:
  ErrorKind kind_;
};

[[noreturn]] void fail(ErrorKind kind, const std::string &msg);

// Config flags (include/marisa/base.h:100-157).
constexpr uint32_t kNumTriesMask = 0x0007F;
constexpr uint32_t kCacheLevelMask = 0x00F80;
constexpr uint32_t kTailModeMask = 0x0F000;
constexpr uint32_t kNodeOrderMask = 0xF0000;
constexpr uint32_t kNormalCache = 0x00200;
constexpr uint32_t kTextTail = 0x01000;
constexpr uint32_t kBinaryTail = 0x02000;
constexpr uint32_t kLabelOrder = 0x10000;
constexpr uint32_t kWeightOrder = 0x20000;
constexpr uint32_t kTailTerminal = 0xFFFFFFFFu;  // tail.cc:11

// 12-byte rank directory entry: absolute rank of each 512-bit block plus the
// seven 64-bit sub-block offsets packed into 7+8+8+9 / 9+9+9 bits
// (vector/rank-index.h:10-76).
struct RankEntry {
  uint32_t abs = 0;
  uint32_t rel_lo = 0;
  uint32_t rel_hi = 0;
  uint32_t rel(int k) const;  // k in 1..7
  void set_rel(int k, uint32_t v);
};
static_assert(sizeof(RankEntry) == 12, "RankEntry must serialise as 12 bytes");

struct BitVec {
  std::vector<uint64_t> units;
  uint64_t size = 0;
  uint64_t num_1s = 0;
  std::vector<RankEntry> ranks;
  std::vector<uint32_t> select0s;
  std::vector<uint32_t> select1s;

  bool get(uint64_t i) const { return (units[i >> 6] >> (i & 63)) & 1u; }
  void push_back(bool bit);
  // Builds the rank directory and the select samples (bit-vector.cc:733-859).
  void build_index(bool enable_select0, bool enable_select1);
  uint64_t rank1(uint64_t i) const;
  uint64_t select0(uint64_t i) const;
  uint64_t select1(uint64_t i) const;
  uint64_t total_size() const;
  uint64_t io_size() const;
};

struct FlatVec {
  std::vector<uint64_t> units;
  uint32_t value_size = 0;
  uint32_t mask = 0;
  uint64_t size = 0;

  uint32_t get(uint64_t i) const {
    const uint64_t pos = i * value_size;
    const uint64_t u = pos >> 6, off = pos & 63;
    if (off + value_size <= 64) return (uint32_t)(units[u] >> off) & mask;
    return (uint32_t)((units[u] >> off) | (units[u + 1] << (64 - off))) & mask;
  }
  // Packs `values` with the minimum bit width (flat-vector.h:95-131).
  void build(const std::vector<uint32_t> &values);
  uint64_t total_size() const { return units.size() * 8; }
  uint64_t io_size() const;
};

struct CacheEntry {
  uint32_t parent = 0;
  uint32_t child = 0;
  uint32_t value = 0;  // float weight during build, packed label/link afterwards
};
static_assert(sizeof(CacheEntry) == 12, "CacheEntry must serialise as 12 bytes");

struct LoudsLevel {
  BitVec louds;
  BitVec terminal;
  BitVec link;
  std::vector<uint16_t> bases;
  FlatVec extras;
  FlatVec link_extras;
  std::vector<uint32_t> tail;
  BitVec tail_end_flags;  // empty for a text tail
  std::unique_ptr<LoudsLevel> next;
  std::vector<CacheEntry> cache;
  uint32_t num_l1_nodes = 0;
  uint32_t config_flags = 0;

  uint64_t num_nodes() const { return louds.size / 2 - 1; }  // louds-trie.h:55-57
  uint64_t num_keys() const { return terminal.num_1s; }
  uint32_t num_tries() const { return config_flags & kNumTriesMask; }
  uint32_t tail_mode() const { return config_flags & kTailModeMask; }
  uint32_t node_order() const { return config_flags & kNodeOrderMask; }
  bool binary_tail() const { return tail_end_flags.size != 0; }
  uint32_t label(uint64_t node) const {
    return (uint32_t)bases[node] | (extras.get(node) << 16);  // louds-trie.cc:1047-1053
  }
  uint64_t link_offset(uint64_t node, uint64_t link_id) const {
    return (uint32_t)bases[node] | (link_extras.get(link_id) << 16);  // louds-trie.cc:1036-1039
  }
  uint64_t total_size() const;
  uint64_t io_size_body() const;
};

// A complete trie (header + top level).
struct MarisaImage {
  std::unique_ptr<LoudsLevel> top;

  bool empty_handle() const { return !top; }
  uint64_t io_size() const { return 16 + top->io_size_body(); }
};

// Serialisation.  `read_image` validates everything it can without trusting
// the file (sizes against the remaining bytes, bit counts against units).
std::unique_ptr<LoudsLevel> read_image(const uint8_t *data, size_t size);
std::unique_ptr<LoudsLevel> read_image_file(const std::string &path);
std::vector<uint8_t> write_image(const LoudsLevel &top);
void write_image_file(const LoudsLevel &top, const std::string &path);

// Builder: same structure as `Trie.build(token_rows)` in the reference
// (tools/bindings.cpp:10-22): one trie, text tail (switching to a binary tail
// when a link string contains 0xFFFFFFFF), label order, normal cache.
// `rows` are given as a flat token array plus num_rows+1 offsets.
std::unique_ptr<LoudsLevel> build_image(const uint32_t *tokens, const uint64_t *offsets,
                                        uint64_t num_rows, int num_threads);

}  // namespace ftb
