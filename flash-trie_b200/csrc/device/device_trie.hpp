// Device image of a trie: the arrays the search kernel gathers from, derived
// once from the MARISA structures at upload time and never written to disk.
//
// The reference kernel walks the succinct structures directly: select0 over
// the LOUDS bits for a parent's child range (3-5 dependent gathers), rank1 +
// link_extras + tail to learn a link child's first label inside every binary
// search probe (lib/marisa/grimoire/trie/tbs-kernels.cu:210-278).  On B200
// the search is bound by chains of dependent random gathers, so the image
// spends HBM to make everything the search needs about a node one 16-byte
// load:
//   node[n] = {label, aux, c0, flags << 24 | fan-out}
//     label   the label of a plain node, or the first tail token of a link
//             node, so the children of a node are one run of records sorted
//             by label (LOUDS numbers siblings consecutively);
//     aux     tail offset of a link node's string; first slot of the node's
//             hash table for a hashed plain node; 0 otherwise;
//     c0      first child (= select0(n) - n); children are [c0, c0 + fan-out);
//     flags   bit0 terminal, bit1 link; bit2 on a link node: its string ends
//             after the first token (the child that consumes it cannot
//             continue); bit2 on a plain node: it has a hash table (bits 3-7:
//             log2 of the table size);
//     fan-out min(number of children, 0xFFFFFF); 0xFFFFFF means "at least
//             that many": the range then ends at node[n + 1].c0 (or N).
//   term_rank per 64 nodes {u32 terminal nodes before the block, u32 0, u64 the
//             block's terminal bits}: a key's id is the rank of its terminal
//             node among terminal nodes (LoudsTrie::lookup, louds-trie.cc:56-72),
//             one 16-byte load;
//   tail      u32 cells as stored in the file (0xFFFFFFFF terminates a string
//             in a text tail); tail_end: end bits of a binary tail.
//   hash      per-node open-addressing tables for plain (non-link) nodes with
//             at least kHashMinDegree children: slots {label, child} (child 0 =
//             empty), 2^lg slots at load <= 1/2.  A proposal then costs one
//             probe instead of a log2(fan-out) binary search.
#pragma once

#include <cstdint>
#include <vector>

#include "../host/marisa_image.hpp"

namespace ftb {

constexpr uint8_t kNodeTerminal = 1;
constexpr uint8_t kNodeLink = 2;
constexpr uint8_t kNodeHashed = 4;      // plain nodes
constexpr uint8_t kNodeLinkEnds1 = 4;   // link nodes
constexpr uint32_t kHashMinDegree = 64;
constexpr uint32_t kFanoutMask = 0xFFFFFFu;  // fan-out field of a node record

// Slot of a child in its parent's hash table.
inline uint32_t hash_slot(uint32_t label, uint32_t lg) { return (label * 2654435761u) >> (32 - lg); }

struct HostDeviceImage {
  uint64_t num_nodes = 0;
  std::vector<uint32_t> child_begin;
  std::vector<uint32_t> first_label;
  std::vector<uint32_t> link_off;
  std::vector<uint8_t> flags;
  std::vector<uint32_t> hash;  // pairs: label, child
  bool binary_tail = false;
};

// Derives and validates the arrays above (throws FormatError on any
// inconsistency that could send the kernel out of bounds).
void derive_device_image(const LoudsLevel &lv, HostDeviceImage &out, int num_threads);

void pack_node_records(const HostDeviceImage &img, std::vector<uint32_t> &out, int num_threads);

// Device-resident trie; owns its allocations.
struct DeviceTrie {
  int device = -1;
  uint64_t num_nodes = 0;
  uint64_t tail_size = 0;
  bool binary_tail = false;
  uint32_t *node = nullptr;  // [4 * num_nodes]: {label, aux, c0, flags << 24 | fan-out}
  uint32_t *term_rank = nullptr;  // [4 * ceil(num_nodes / 64)], see above
  uint32_t *tail = nullptr;
  uint64_t *tail_end = nullptr;
  uint32_t *hash = nullptr;
  uint64_t hash_slots = 0;
  uint64_t num_keys = 0;  // terminal nodes
  uint64_t bytes = 0;

  DeviceTrie() = default;
  DeviceTrie(const DeviceTrie &) = delete;
  DeviceTrie &operator=(const DeviceTrie &) = delete;
  ~DeviceTrie();
  void release();
  // Uploads the image of `lv` to the current device.
  void upload(const LoudsLevel &lv, int num_threads);
};

}  // namespace ftb
