// Shared pieces of the tensor-core attention kernels: tile geometry, the
// partition-layout slot decode and the 128-byte shared-memory swizzle.
#pragma once
#include "attn.cuh"
#include "sm100.cuh"

namespace pe {
namespace attn_tc {

constexpr int HD = 128;  // head dim
constexpr int TQ = 128;  // query rows per tile
constexpr int TK = 128;  // keys per tile
constexpr uint32_t TILE_BYTES = 128 * HD * 2;  // one 128 x 128 bf16 tile = two 64-column chunks
constexpr uint32_t CHUNK = TILE_BYTES / 2;      // 16 KB: 128 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct PartGeom {
  int S, a0, a1, km1;  // km1 = K - 1 (0 when K == 1)
};

// anchor / depth of slot s in the partition layout (reference partition.py:41-55)
__device__ __forceinline__ void decode(const PartGeom& g, int s, int& i, int& d) {
  if (s < g.a1 || g.km1 == 0) {
    i = s;
    d = 0;
  } else {
    const int t = s - g.a1;
    i = g.a0 + t / g.km1;
    d = 1 + t % g.km1;
  }
}

// byte offset of 16-byte unit u (0..7) of row r inside a 128B-swizzled chunk
// (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B on a 1024 B-aligned base)
__device__ __forceinline__ uint32_t swz(int r, int u) {
  return (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4));
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace attn_tc
}  // namespace pe
