// Rotary-embedding arithmetic shared by the fused rotations (the q|k|v GEMM
// epilogue, the attention backward's dQ store and dK cast): half-split pairs
// (x[p], x[p + hd/2]) rotated by bf16 cos / sin from a per-row table written by
// pe_rope_table, each product and sum rounded to bf16 like the reference's
// element-wise bf16 ops (src/pe/nn.py:44-49) and like rope.cu's kernels, so the
// fused and unfused paths give identical bits.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace pe {

__device__ __forceinline__ float rb16(float x) { return round_to<__nv_bfloat16>(x); }

// forward: (a, b) -> (a c - b s, b c + a s); inverse (the transpose, for gradients):
// (a, b) -> (a c + b s, b c - a s).  a, b, c, s are bf16 values held in fp32.
__device__ __forceinline__ void rope_rotate_pair(float& a, float& b, float c, float s,
                                                 bool inverse) {
  float ya, yb;
  if (!inverse) {
    ya = rb16(rb16(a * c) + rb16(-b * s));
    yb = rb16(rb16(b * c) + rb16(a * s));
  } else {
    ya = rb16(rb16(a * c) + rb16(b * s));
    yb = rb16(rb16(b * c) - rb16(a * s));
  }
  a = ya;
  b = yb;
}

// n (a multiple of 8) consecutive bf16 values from a 16-byte aligned address, as fp32
template <int N>
__device__ __forceinline__ void load_bf16_f32(const __nv_bfloat16* p, float* out) {
#pragma unroll
  for (int q = 0; q < N / 8; ++q) {
    const uint4 u = reinterpret_cast<const uint4*>(p)[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      out[q * 8 + 2 * j] = f.x;
      out[q * 8 + 2 * j + 1] = f.y;
    }
  }
}

}  // namespace pe
