// Reader, writer and index builder for the MARISA trie file format.
// The byte layout is documented in marisa_image.hpp; every field, width and
// padding rule below follows the reference serialisation so files round-trip.
#include "marisa_image.hpp"

#include <algorithm>
#include <cstring>
#include <fstream>
#include <iterator>

namespace ftb {

void fail(ErrorKind kind, const std::string &msg) { throw FormatError(kind, msg); }

// ---------------------------------------------------------------- RankEntry
// Bit positions of the packed sub-block counts (vector/rank-index.h:19-76).
static const int kRelShift[8] = {0, 0, 7, 15, 23, 0, 9, 18};
static const uint32_t kRelMask[8] = {0, 0x7Fu, 0xFFu, 0xFFu, 0x1FFu, 0x1FFu, 0x1FFu, 0x1FFu};

uint32_t RankEntry::rel(int k) const {
  const uint32_t w = k <= 4 ? rel_lo : rel_hi;
  return (w >> kRelShift[k]) & kRelMask[k];
}

void RankEntry::set_rel(int k, uint32_t v) {
  uint32_t &w = k <= 4 ? rel_lo : rel_hi;
  w = (w & ~(kRelMask[k] << kRelShift[k])) | ((v & kRelMask[k]) << kRelShift[k]);
}

// ------------------------------------------------------------------ BitVec
void BitVec::push_back(bool bit) {
  if (size == 0xFFFFFFFFull) fail(ErrorKind::kSize, "MARISA_SIZE_ERROR: bit vector exceeds 2^32-1 bits");
  if (size == 64 * units.size()) units.push_back(0);
  if (bit) {
    units[size >> 6] |= 1ull << (size & 63);
    ++num_1s;
  }
  ++size;
}

// Position of the i-th (0-based) set bit of `w`, plus `base`.
static inline uint64_t nth_set_bit(uint64_t w, uint64_t i, uint64_t base) {
  for (uint64_t k = 0; k < i; ++k) w &= w - 1;
  return base + (uint64_t)__builtin_ctzll(w);
}

void BitVec::build_index(bool enable_select0, bool enable_select1) {
  const uint64_t num_bits = size;
  ranks.assign(num_bits / 512 + ((num_bits % 512) != 0 ? 1 : 0) + 1, RankEntry());
  select0s.clear();
  select1s.clear();
  uint64_t zeros = 0, ones = 0;
  for (uint64_t u = 0; u < units.size(); ++u) {
    const uint64_t bit_id = u * 64;
    const uint64_t rid = bit_id / 512;
    const int sub = (int)((bit_id / 64) % 8);
    if (sub == 0) {
      ranks[rid].abs = (uint32_t)ones;
    } else {
      ranks[rid].set_rel(sub, (uint32_t)(ones - ranks[rid].abs));
    }
    const uint64_t w = units[u];
    const uint64_t w1 = (uint64_t)__builtin_popcountll(w);
    if (enable_select0) {
      const uint64_t remaining = num_bits - bit_id;
      const uint64_t w0 = std::min<uint64_t>(remaining, 64) - w1;
      const uint64_t want = (512 - (zeros % 512)) % 512;  // next multiple of 512 zeros
      if (w0 > want) select0s.push_back((uint32_t)nth_set_bit(~w, want, bit_id));
      zeros += w0;
    }
    if (enable_select1) {
      const uint64_t want = (512 - (ones % 512)) % 512;
      if (w1 > want) select1s.push_back((uint32_t)nth_set_bit(w, want, bit_id));
    }
    ones += w1;
  }
  if ((num_bits % 512) != 0) {
    // Remaining sub-blocks of the last block carry the final count.
    const uint64_t rid = (num_bits - 1) / 512;
    const int last_sub = (int)(((num_bits - 1) / 64) % 8);
    for (int k = last_sub + 1; k <= 7; ++k) ranks[rid].set_rel(k, (uint32_t)(ones - ranks[rid].abs));
  }
  ranks.back().abs = (uint32_t)ones;
  if (enable_select0) select0s.push_back((uint32_t)num_bits);
  if (enable_select1) select1s.push_back((uint32_t)num_bits);
}

uint64_t BitVec::rank1(uint64_t i) const {
  const RankEntry &r = ranks[i / 512];
  uint64_t off = r.abs;
  const int sub = (int)((i / 64) % 8);
  if (sub) off += r.rel(sub);
  const uint64_t m = (i & 63) ? ((1ull << (i & 63)) - 1) : 0;
  return off + (uint64_t)__builtin_popcountll(units[i / 64] & m);
}

// select0/select1 by binary search over the rank directory; used only on the
// host (building and validation), so clarity beats the sampled fast path.
uint64_t BitVec::select0(uint64_t i) const {
  uint64_t lo = 0, hi = ranks.size() - 1;  // zeros before block b = b*512 - abs
  while (lo + 1 < hi) {
    const uint64_t mid = (lo + hi) / 2;
    if (mid * 512 - ranks[mid].abs <= i) lo = mid; else hi = mid;
  }
  uint64_t rem = i - (lo * 512 - ranks[lo].abs);
  for (uint64_t u = lo * 8; u < units.size(); ++u) {
    const uint64_t valid = std::min<uint64_t>(64, size - u * 64);
    uint64_t w = ~units[u];
    if (valid < 64) w &= (1ull << valid) - 1;
    const uint64_t c = (uint64_t)__builtin_popcountll(w);
    if (rem < c) return nth_set_bit(w, rem, u * 64);
    rem -= c;
  }
  fail(ErrorKind::kBound, "MARISA_BOUND_ERROR: select0 out of range");
}

uint64_t BitVec::select1(uint64_t i) const {
  uint64_t lo = 0, hi = ranks.size() - 1;
  while (lo + 1 < hi) {
    const uint64_t mid = (lo + hi) / 2;
    if (ranks[mid].abs <= i) lo = mid; else hi = mid;
  }
  uint64_t rem = i - ranks[lo].abs;
  for (uint64_t u = lo * 8; u < units.size(); ++u) {
    const uint64_t c = (uint64_t)__builtin_popcountll(units[u]);
    if (rem < c) return nth_set_bit(units[u], rem, u * 64);
    rem -= c;
  }
  fail(ErrorKind::kBound, "MARISA_BOUND_ERROR: select1 out of range");
}

static inline uint64_t vec_io(uint64_t bytes) { return 8 + ((bytes + 7) & ~7ull); }

uint64_t BitVec::total_size() const {
  return units.size() * 8 + ranks.size() * 12 + select0s.size() * 4 + select1s.size() * 4;
}
uint64_t BitVec::io_size() const {
  return vec_io(units.size() * 8) + 8 + vec_io(ranks.size() * 12) + vec_io(select0s.size() * 4) +
         vec_io(select1s.size() * 4);
}

// ----------------------------------------------------------------- FlatVec
void FlatVec::build(const std::vector<uint32_t> &values) {
  uint32_t max_value = 0;
  for (uint32_t v : values) max_value = std::max(max_value, v);
  uint32_t vs = 0;
  while (max_value != 0) {
    ++vs;
    max_value >>= 1;
  }
  uint64_t n_units = values.empty() ? 0 : 1;
  if (vs != 0) n_units = ((uint64_t)vs * values.size() + 63) / 64;
  units.assign(n_units, 0);
  value_size = vs;
  mask = vs ? (0xFFFFFFFFu >> (32 - vs)) : 0;
  size = values.size();
  for (uint64_t i = 0; i < values.size(); ++i) {
    const uint64_t pos = i * vs, u = pos >> 6, off = pos & 63;
    const uint64_t v = values[i] & mask;
    units[u] |= v << off;
    if (off + vs > 64) units[u + 1] |= v >> (64 - off);
  }
}

uint64_t FlatVec::io_size() const { return vec_io(units.size() * 8) + 4 + 4 + 8; }

// --------------------------------------------------------------- LoudsLevel
uint64_t LoudsLevel::total_size() const {
  return louds.total_size() + terminal.total_size() + link.total_size() + bases.size() * 2 +
         extras.total_size() + link_extras.total_size() + tail.size() * 4 + tail_end_flags.total_size() +
         (next ? next->total_size() : 0) + cache.size() * 12;
}

uint64_t LoudsLevel::io_size_body() const {
  return louds.io_size() + terminal.io_size() + link.io_size() + vec_io(bases.size() * 2) + extras.io_size() +
         link_extras.io_size() + vec_io(tail.size() * 4) + tail_end_flags.io_size() +
         (next ? next->io_size_body() : 0) + vec_io(cache.size() * 12) + 8;
}

// ------------------------------------------------------------------ reading
namespace {

constexpr char kHeader[16] = "We love Marisa.";

struct Cursor {
  const uint8_t *p;
  size_t left;

  void need(uint64_t n) {
    if (n > left) fail(ErrorKind::kIO, "MARISA_IO_ERROR: unexpected end of trie data");
  }
  template <typename T>
  T scalar() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    left -= sizeof(T);
    return v;
  }
  template <typename T>
  void vec(std::vector<T> &out) {
    const uint64_t bytes = scalar<uint64_t>();
    if (bytes % sizeof(T) != 0) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: vector size is not a multiple of its element");
    need(bytes);
    out.resize(bytes / sizeof(T));
    if (bytes) std::memcpy(out.data(), p, bytes);
    p += bytes;
    left -= bytes;
    const uint64_t pad = (8 - bytes % 8) % 8;
    need(pad);
    p += pad;
    left -= pad;
  }
  void bitvec(BitVec &bv) {
    vec(bv.units);
    bv.size = scalar<uint32_t>();
    bv.num_1s = scalar<uint32_t>();
    if (bv.num_1s > bv.size) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: bit vector has more 1s than bits");
    if (bv.units.size() * 64 < bv.size) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: bit vector units too short");
    vec(bv.ranks);
    vec(bv.select0s);
    vec(bv.select1s);
  }
  void flatvec(FlatVec &fv) {
    vec(fv.units);
    fv.value_size = scalar<uint32_t>();
    if (fv.value_size > 32) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: flat vector value size > 32");
    fv.mask = scalar<uint32_t>();
    fv.size = scalar<uint64_t>();
    if ((__uint128_t)fv.size * fv.value_size > (__uint128_t)fv.units.size() * 64)
      fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: flat vector units too short");
  }
};

void check_config(uint32_t flags) {
  // Config::parse (grimoire/trie/config.h:57-144).
  if (flags & ~0xFFFFFu) fail(ErrorKind::kCode, "MARISA_CODE_ERROR: undefined config flags");
  switch (flags & kCacheLevelMask) {
    case 0: case 0x80: case 0x100: case 0x200: case 0x400: case 0x800: break;
    default: fail(ErrorKind::kCode, "MARISA_CODE_ERROR: undefined cache level");
  }
  switch (flags & kTailModeMask) {
    case 0: case kTextTail: case kBinaryTail: break;
    default: fail(ErrorKind::kCode, "MARISA_CODE_ERROR: undefined tail mode");
  }
  switch (flags & kNodeOrderMask) {
    case 0: case kLabelOrder: case kWeightOrder: break;
    default: fail(ErrorKind::kCode, "MARISA_CODE_ERROR: undefined node order");
  }
}

void read_level(Cursor &c, LoudsLevel &lv) {
  c.bitvec(lv.louds);
  c.bitvec(lv.terminal);
  c.bitvec(lv.link);
  c.vec(lv.bases);
  c.flatvec(lv.extras);
  c.flatvec(lv.link_extras);
  c.vec(lv.tail);
  c.bitvec(lv.tail_end_flags);
  // louds-trie.cc:730-733: a level with links but no tail stores its link
  // strings in a nested trie.
  if (lv.link.num_1s != 0 && lv.tail.empty()) {
    lv.next.reset(new LoudsLevel());
    read_level(c, *lv.next);
  }
  c.vec(lv.cache);
  lv.num_l1_nodes = c.scalar<uint32_t>();
  lv.config_flags = c.scalar<uint32_t>();
  check_config(lv.config_flags);
}

// Writes bytes exactly as grimoire::io::Writer does: vectors padded with zeros.
struct Sink {
  std::vector<uint8_t> out;
  template <typename T>
  void scalar(T v) {
    const uint8_t *b = reinterpret_cast<const uint8_t *>(&v);
    out.insert(out.end(), b, b + sizeof(T));
  }
  template <typename T>
  void vec(const std::vector<T> &v) {
    const uint64_t bytes = v.size() * sizeof(T);
    scalar<uint64_t>(bytes);
    const uint8_t *b = reinterpret_cast<const uint8_t *>(v.data());
    if (bytes) out.insert(out.end(), b, b + bytes);
    out.insert(out.end(), (8 - bytes % 8) % 8, 0);
  }
  void bitvec(const BitVec &bv) {
    vec(bv.units);
    scalar<uint32_t>((uint32_t)bv.size);
    scalar<uint32_t>((uint32_t)bv.num_1s);
    vec(bv.ranks);
    vec(bv.select0s);
    vec(bv.select1s);
  }
  void flatvec(const FlatVec &fv) {
    vec(fv.units);
    scalar<uint32_t>(fv.value_size);
    scalar<uint32_t>(fv.mask);
    scalar<uint64_t>(fv.size);
  }
  void level(const LoudsLevel &lv) {
    bitvec(lv.louds);
    bitvec(lv.terminal);
    bitvec(lv.link);
    vec(lv.bases);
    flatvec(lv.extras);
    flatvec(lv.link_extras);
    vec(lv.tail);
    bitvec(lv.tail_end_flags);
    if (lv.next) level(*lv.next);
    vec(lv.cache);
    scalar<uint32_t>(lv.num_l1_nodes);
    scalar<uint32_t>(lv.config_flags);
  }
};

}  // namespace

std::unique_ptr<LoudsLevel> read_image(const uint8_t *data, size_t size) {
  Cursor c{data, size};
  c.need(16);
  if (std::memcmp(c.p, kHeader, 16) != 0) fail(ErrorKind::kFormat, "MARISA_FORMAT_ERROR: bad trie header");
  c.p += 16;
  c.left -= 16;
  std::unique_ptr<LoudsLevel> lv(new LoudsLevel());
  read_level(c, *lv);
  return lv;
}

std::unique_ptr<LoudsLevel> read_image_file(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(ErrorKind::kIO, "MARISA_IO_ERROR: failed to open file: " + path);
  f.seekg(0, std::ios::end);
  const std::streamoff n = f.tellg();
  if (n < 0) fail(ErrorKind::kIO, "MARISA_IO_ERROR: failed to size file: " + path);
  f.seekg(0, std::ios::beg);
  std::vector<uint8_t> buf((size_t)n);
  if (n && !f.read(reinterpret_cast<char *>(buf.data()), n))
    fail(ErrorKind::kIO, "MARISA_IO_ERROR: failed to read file: " + path);
  return read_image(buf.data(), buf.size());
}

std::vector<uint8_t> write_image(const LoudsLevel &top) {
  Sink s;
  s.out.reserve(16 + top.io_size_body());
  s.out.insert(s.out.end(), kHeader, kHeader + 16);
  s.level(top);
  return std::move(s.out);
}

void write_image_file(const LoudsLevel &top, const std::string &path) {
  const std::vector<uint8_t> bytes = write_image(top);
  std::ofstream f(path, std::ios::binary | std::ios::trunc);
  if (!f) fail(ErrorKind::kIO, "MARISA_IO_ERROR: failed to open file: " + path);
  f.write(reinterpret_cast<const char *>(bytes.data()), (std::streamsize)bytes.size());
  if (!f) fail(ErrorKind::kIO, "MARISA_IO_ERROR: failed to write file: " + path);
}

}  // namespace ftb
