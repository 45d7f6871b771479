// Trie builder producing the same MARISA structures (and therefore the same
// file bytes) as the reference `Trie.build(token_rows)` for label values
// below 2^31.
//
// Build steps and the reference code each one must agree with:
//   1. sort the keys lexicographically, a proper prefix before its
//      extensions (algorithm/sort.h:80-190 orders keys this way whenever
//      every label is below 2^31; it compares labels as signed ints);
//   2. breadth-first LOUDS construction with Patricia "links" for edges whose
//      whole key range shares the next labels (louds-trie.cc:477-588);
//   3. terminal flags by node id (louds-trie.cc:405-435);
//   4. suffix-merged tail of the link strings (tail.cc:185-228);
//   5. link offsets split into bases (low 16 bits) and link_extras
//      (louds-trie.cc:462-473), label extras, and the node cache
//      (louds-trie.cc:645-694).
// The implementation is this project's own: flat index arrays, a vector-backed
// FIFO, parallel sorts on packed label prefixes, and a parallel tail merge.
#include <algorithm>
#include <cfloat>
#include <cstring>
#include <numeric>
#include <parallel/algorithm>

#include "marisa_image.hpp"

namespace ftb {
namespace {

struct KeyRef {
  const uint32_t *p;
  uint32_t len;
  uint32_t terminal;  // node id where the key ends (set by the BFS)
};

// A key while the keys are sorted.  The order is lexicographic on u32
// labels, a prefix before its extensions.  The first two labels, packed as
// (l0 << 32) | l1 with zeros where the key is shorter, decide most
// comparisons without reading the labels: a key shorter than two labels sorts
// no later than any key with the same packed labels (it is a prefix of them
// or equal to them), and equal packed labels fall through to the full
// comparison.
struct SortKey {
  uint64_t head;
  const uint32_t *p;
  uint32_t len;
};

inline bool sort_key_less(const SortKey &a, const SortKey &b) {
  if (a.head != b.head) return a.head < b.head;
  const uint32_t n = std::min(a.len, b.len);
  for (uint32_t i = 0; i < n; ++i)
    if (a.p[i] != b.p[i]) return a.p[i] < b.p[i];
  return a.len < b.len;
}

inline bool key_equal(const KeyRef &a, const KeyRef &b) {
  return a.len == b.len && std::memcmp(a.p, b.p, (size_t)a.len * 4) == 0;
}

// A link string, compared from its last label backwards (tail entries are
// sorted as reversed strings so that a suffix sorts right before the strings
// it is a suffix of; tail.cc:185-201).
struct TailEntry {
  const uint32_t *p;  // first label
  uint32_t len;       // at least 2: a link spans two or more labels
  uint32_t id;        // index in BFS link order
  uint64_t last2;     // last two labels, (p[len-1] << 32) | p[len-2]
};

// Strings whose last two labels differ are ordered by `last2` alone.
inline bool reversed_less(const TailEntry &a, const TailEntry &b) {
  if (a.last2 != b.last2) return a.last2 < b.last2;
  const uint32_t n = std::min(a.len, b.len);
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t x = a.p[a.len - 1 - i], y = b.p[b.len - 1 - i];
    if (x != y) return x < y;
  }
  return a.len < b.len;
}

struct Range {
  uint64_t begin, end;
  uint32_t key_pos;
};

// Cache slot for (parent, label) (louds-trie.cc:1024-1026).
inline uint64_t cache_slot(uint64_t parent, uint32_t label, uint64_t mask) {
  return (parent ^ (parent << 5) ^ label) & mask;
}

}  // namespace

std::unique_ptr<LoudsLevel> build_image(const uint32_t *tokens, const uint64_t *offsets, uint64_t num_rows,
                                        int num_threads) {
  std::unique_ptr<LoudsLevel> lv(new LoudsLevel());
  if (num_threads < 1) num_threads = 1;

  // ---- 1. sort keys ---------------------------------------------------
  // Sorted through a temporary array carrying the packed labels; the sorted
  // keys are allocated after the sort has released its scratch memory.
  std::vector<KeyRef> keys;
  {
    std::vector<SortKey> sk(num_rows);
    for (uint64_t i = 0; i < num_rows; ++i) {
      const uint64_t len = offsets[i + 1] - offsets[i];
      if (len > 0xFFFFFFFFull) fail(ErrorKind::kSize, "MARISA_SIZE_ERROR: key longer than 2^32-1 labels");
      const uint32_t *p = tokens + offsets[i];
      sk[i] = SortKey{len == 0 ? 0 : ((uint64_t)p[0] << 32) | (len > 1 ? p[1] : 0u), p, (uint32_t)len};
    }
    if (num_threads > 1 && num_rows > 100000) {
      __gnu_parallel::sort(sk.begin(), sk.end(), sort_key_less,
                           __gnu_parallel::multiway_mergesort_tag((__gnu_parallel::_ThreadIndex)num_threads));
    } else {
      std::sort(sk.begin(), sk.end(), sort_key_less);
    }
    keys.resize(num_rows);
    for (uint64_t i = 0; i < num_rows; ++i) keys[i] = KeyRef{sk[i].p, sk[i].len, 0};
  }
  uint64_t num_unique = num_rows ? 1 : 0;
  for (uint64_t i = 1; i < num_rows; ++i)
    if (!key_equal(keys[i - 1], keys[i])) ++num_unique;

  // ---- cache sizing (louds-trie.cc:658-666) -----------------------------
  uint64_t cache_size = 256;
  while (cache_size < num_unique / kNormalCache) cache_size *= 2;
  const uint64_t cache_mask = cache_size - 1;
  std::vector<float> cache_weight(cache_size, FLT_MIN);
  lv->cache.assign(cache_size, CacheEntry());

  // ---- 2. breadth-first LOUDS -------------------------------------------
  BitVec &louds = lv->louds;
  std::vector<uint16_t> &bases = lv->bases;
  std::vector<uint32_t> extras_vals;
  std::vector<uint8_t> is_link;
  std::vector<TailEntry> links;  // link strings in BFS order
  louds.push_back(true);
  louds.push_back(false);
  bases.push_back(0);
  extras_vals.push_back(0);
  is_link.push_back(0);

  std::vector<Range> fifo;
  fifo.reserve(num_rows + 16);
  fifo.push_back(Range{0, num_rows, 0});
  std::vector<Range> children;
  std::vector<double> child_w;
  for (uint64_t head = 0; head < fifo.size(); ++head) {
    const uint64_t node_id = head;  // ranges are dequeued in node-id order
    Range r = fifo[head];
    while (r.begin < r.end && keys[r.begin].len == r.key_pos) keys[r.begin++].terminal = (uint32_t)node_id;
    if (r.begin == r.end) {
      louds.push_back(false);
      continue;
    }
    // Split by the label at key_pos; weights count keys (each key weighs 1).
    children.clear();
    child_w.clear();
    uint64_t start = r.begin;
    for (uint64_t i = r.begin + 1; i < r.end; ++i) {
      if (keys[i - 1].p[r.key_pos] != keys[i].p[r.key_pos]) {
        children.push_back(Range{start, i, r.key_pos});
        child_w.push_back((double)(i - start));
        start = i;
      }
    }
    children.push_back(Range{start, r.end, r.key_pos});
    child_w.push_back((double)(r.end - start));
    if (node_id == 0) lv->num_l1_nodes = (uint32_t)children.size();

    for (size_t c = 0; c < children.size(); ++c) {
      Range &w = children[c];
      // Extend the edge while every key of the range agrees, stopping at the
      // end of the shortest (first) key.
      uint32_t kp = w.key_pos + 1;
      const KeyRef &first = keys[w.begin];
      while (kp < first.len) {
        uint64_t j = w.begin + 1;
        for (; j < w.end; ++j)
          if (keys[j - 1].p[kp] != keys[j].p[kp]) break;
        if (j < w.end) break;
        ++kp;
      }
      const uint64_t child_id = bases.size();
      const uint32_t label = first.p[w.key_pos];
      const float weight = (float)child_w[c];
      const uint64_t slot = cache_slot(node_id, label, cache_mask);
      if (weight > cache_weight[slot]) {
        lv->cache[slot].parent = (uint32_t)node_id;
        lv->cache[slot].child = (uint32_t)child_id;
        cache_weight[slot] = weight;
      }
      if (kp == w.key_pos + 1) {
        bases.push_back((uint16_t)(label & 0xFFFF));
        extras_vals.push_back(label >> 16);
        is_link.push_back(0);
      } else {
        bases.push_back(0);
        extras_vals.push_back(0);
        is_link.push_back(1);
        const uint32_t *lp = first.p + w.key_pos;
        const uint32_t ll = kp - w.key_pos;
        links.push_back(TailEntry{lp, ll, (uint32_t)links.size(), ((uint64_t)lp[ll - 1] << 32) | lp[ll - 2]});
      }
      w.key_pos = kp;
      fifo.push_back(w);
      louds.push_back(true);
    }
    louds.push_back(false);
  }
  louds.push_back(false);
  const uint64_t num_nodes = bases.size();
  fifo = std::vector<Range>();

  // ---- 3. terminal flags ------------------------------------------------
  {
    std::vector<uint8_t> term(num_nodes, 0);
    for (const KeyRef &k : keys) term[k.terminal] = 1;
    for (uint64_t n = 0; n < num_nodes; ++n) lv->terminal.push_back(term[n] != 0);
    lv->terminal.push_back(false);
  }
  keys = std::vector<KeyRef>();

  // ---- 4. tail of link strings --------------------------------------------
  // A link string holding the text terminator needs a binary tail.
  bool binary = false;
#pragma omp parallel for schedule(static, 4096) num_threads(num_threads) reduction(|| : binary)
  for (int64_t k = 0; k < (int64_t)links.size(); ++k) {
    const TailEntry &e = links[k];
    for (uint32_t i = 0; i < e.len; ++i)
      if (e.p[i] == kTailTerminal) {
        binary = true;
        break;
      }
  }
  std::vector<uint32_t> link_off(links.size(), 0);
  {
    std::vector<TailEntry> sorted(links);
    if (num_threads > 1 && sorted.size() > 100000) {
      __gnu_parallel::sort(sorted.begin(), sorted.end(), reversed_less,
                           __gnu_parallel::multiway_mergesort_tag((__gnu_parallel::_ThreadIndex)num_threads));
    } else {
      std::sort(sorted.begin(), sorted.end(), reversed_less);
    }
    // Walking the sorted strings from the last, each string either shares the
    // cells of the one walked just before it (when it is a suffix of it) or
    // is appended to the tail.  Which strings are suffixes of their successor
    // is decided for all at once; an appended string's position is the total
    // length appended after it; a suffix lies inside the nearest appended
    // string after it (suffixes chain), ending where that string ends.
    const uint64_t m = sorted.size();
    const uint64_t term = binary ? 0 : 1;
    std::vector<uint8_t> suffix(m, 0);
#pragma omp parallel for schedule(static, 4096) num_threads(num_threads)
    for (int64_t k = 0; k < (int64_t)m - 1; ++k) {
      const TailEntry &cur = sorted[k], &nx = sorted[k + 1];
      uint32_t match = 0;
      while (match < cur.len && match < nx.len && nx.p[nx.len - 1 - match] == cur.p[cur.len - 1 - match]) ++match;
      suffix[k] = match == cur.len;
    }
    std::vector<uint32_t> pos(m);
    uint64_t total = 0;
    for (uint64_t k = m; k > 0; --k) {
      if (suffix[k - 1]) continue;
      pos[k - 1] = (uint32_t)total;
      total += sorted[k - 1].len + term;
      if (total > 0xFFFFFFFFull) fail(ErrorKind::kSize, "MARISA_SIZE_ERROR: tail exceeds 2^32-1 labels");
    }
    {
      uint64_t owner = m ? m - 1 : 0;
      for (uint64_t k = m; k > 0; --k) {
        if (!suffix[k - 1]) owner = k - 1;
        link_off[sorted[k - 1].id] = (uint32_t)(pos[owner] + sorted[owner].len - sorted[k - 1].len);
      }
    }
    std::vector<uint32_t> &buf = lv->tail;
    buf.resize(total);
#pragma omp parallel for schedule(static, 4096) num_threads(num_threads)
    for (int64_t k = 0; k < (int64_t)m; ++k) {
      if (suffix[k]) continue;
      std::memcpy(buf.data() + pos[k], sorted[k].p, 4ull * sorted[k].len);
      if (!binary) buf[pos[k] + sorted[k].len] = kTailTerminal;
    }
    if (binary) {
      for (uint64_t k = m; k > 0; --k) {
        if (suffix[k - 1]) continue;
        for (uint32_t j = 1; j < sorted[k - 1].len; ++j) lv->tail_end_flags.push_back(false);
        lv->tail_end_flags.push_back(true);
      }
    }
  }

  // ---- 5. links, extras, cache, indexes -----------------------------------
  for (uint64_t n = 0; n < num_nodes; ++n) lv->link.push_back(is_link[n] != 0);
  lv->link.build_index(false, false);
  std::vector<uint32_t> link_hi(links.size());
  {
    uint64_t li = 0;
    for (uint64_t n = 0; n < num_nodes; ++n) {
      if (!is_link[n]) continue;
      bases[n] = (uint16_t)(link_off[li] & 0xFFFF);
      link_hi[li] = link_off[li] >> 16;
      ++li;
    }
  }
  lv->extras.build(extras_vals);
  lv->link_extras.build(link_hi);

  for (uint64_t s = 0; s < cache_size; ++s) {
    CacheEntry &e = lv->cache[s];
    uint32_t bits;
    std::memcpy(&bits, &cache_weight[s], 4);
    if (e.child != 0) {
      // Cache::set_base / set_extra (cache.h:35-45): base in the low 16 bits,
      // extra shifted above it (truncated to 32 bits), bit 31 marks a link.
      const uint64_t child = e.child;
      const bool lnk = is_link[child] != 0;
      const uint64_t extra = lnk ? link_hi[lv->link.rank1(child)] : extras_vals[child];
      bits = (bits & ~0xFFFFu) | bases[child];
      bits = (uint32_t)((bits & 0xFFFFu) | (extra << 16));
      if (lnk) bits |= 0x80000000u;
    } else {
      e.parent = 0xFFFFFFFFu;
      e.child = 0xFFFFFFFFu;
    }
    e.value = bits;
  }

  lv->louds.build_index(true, true);
  lv->terminal.build_index(false, true);
  lv->config_flags = 1u | (binary ? kBinaryTail : kTextTail) | kLabelOrder;
  return lv;
}

}  // namespace ftb
