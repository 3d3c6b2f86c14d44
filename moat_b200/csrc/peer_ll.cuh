// Exchange-buffer layout and the 8-byte "low-latency" words of the tensor-parallel
// exchanges, shared by the exchange kernels (peer.cu) and the GEMM whose epilogue
// stores its rows straight into the exchange buffers (gemm.cu).
//
// A word is 4 bytes of payload and 4 bytes holding the epoch of the call that wrote
// it, stored and loaded as one 8-byte transaction, so a receiver that reads a word
// carrying the current epoch has its payload too.
//
// Exchange buffer (one per rank, zeroed at creation):
//   [0, 16384)      channel 1 (argmax): [2 parities][kPeerMaxRanks][kPeerMaxRows] keys,
//                   each two words (low and high 32 bits of the 64-bit key)
//   [16384, ...)    channel 0 (row joins): [2 parities][kPeerMaxRanks][slot_elems / 2]
//                   words, two fp16 per word; row n, column c of rank src's rows at
//                   element (parity * kPeerMaxRanks + src) * slot_elems + n * D + c
#pragma once

#include <stdint.h>

namespace mb {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerMaxRows = 64;
constexpr size_t kPeerKeyOff = 0;
constexpr size_t kPeerRowOff = 16384;
static_assert(kPeerKeyOff + 2 * kPeerMaxRanks * kPeerMaxRows * 2 * sizeof(uint2) <= kPeerRowOff, "layout");

// One low-latency word: payload and epoch in a single 8-byte store / load.
__device__ __forceinline__ void st_ll(uint2* p, uint32_t payload, uint32_t epoch) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(payload), "r"(epoch) : "memory");
}

__device__ __forceinline__ uint2 ld_ll(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// First word of rank src's channel-0 slot of parity par in an exchange buffer.
__device__ __forceinline__ uint2* peer_row_slot(uint8_t* buf, int par, int src, int64_t slot_elems) {
  return reinterpret_cast<uint2*>(buf + kPeerRowOff) + (static_cast<int64_t>(par) * kPeerMaxRanks + src) * slot_elems / 2;
}

}  // namespace mb
