// Layout of the split-KV receive buffers in NVLink peer memory (csrc/peer_exchange.cu), shared
// with the attention merge that writes into them (csrc/tree_attn.cu).
//
// Receive buffer: [counters: 256 bytes, u32 per rank][parity 0: O, m, l][parity 1: O, m, l],
// with O [world][rows][128] f32 and m, l [world][rows] f32.  Call e (epochs start at 1) uses
// parity e & 1.
#pragma once

#include <cstddef>
#include <cstdint>

namespace ddt {
namespace peer {

constexpr int kMaxWorld = 8;  // ranks of one node
constexpr int kHeadDim = 128;

struct Layout {
  size_t o[2], m[2], l[2], total;
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

inline Layout layout(int64_t world, int64_t rows) {
  Layout L;
  size_t off = 256;  // counters
  for (int p = 0; p < 2; ++p) {
    L.o[p] = off;
    off = align256(off + sizeof(float) * static_cast<size_t>(world * rows * kHeadDim));
    L.m[p] = off;
    off = align256(off + sizeof(float) * static_cast<size_t>(world * rows));
    L.l[p] = off;
    off = align256(off + sizeof(float) * static_cast<size_t>(world * rows));
  }
  L.total = off;
  return L;
}

// Where one rank's partial of one call goes: slot `rank` of every rank's buffer, and the
// counter `rank` of each, bumped once by the last CTA of the writing grid (ticket).
struct Push {
  unsigned char* base[kMaxWorld];
  int world;  // 0: no push
  int rank;
  unsigned long long o_off, m_off, l_off;
  unsigned int* ticket;
};

}  // namespace peer
}  // namespace ddt
