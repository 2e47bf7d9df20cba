// Feature ingestion fused with the drafter's feature RMSNorm (reference
// src/pe/drafter.py:129-130: `features.to(dtype)`, viewed as [n, F / H, H], then one
// RMSNorm with a shared weight over each H-wide block).
//
// The step feeds each stacked segment the real prefix rows [0, a1) of the sequence's
// features, so a pass of S segments reads the prefix rows S times.  Instead of casting
// the shard to the run dtype and gathering those rows into a new buffer first, the
// forward kernel reads every output row straight from the shard through the token
// map (`src_tok`), rounds each element to the run dtype (the reference's cast) and
// normalises: one read of the source rows it needs and one write of the normalised
// rows.  The backward needs only the weight gradient (features take no gradient):
// sum over rows of dy * x * rstd, with x re-read from the shard the same way -- no dx
// is written.
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"

namespace pe {
namespace {

// 8 consecutive elements of the source row as fp32 (16- or 32-byte aligned)
__device__ __forceinline__ void load8_src(const __half* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load8_src(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load8_src(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

template <typename T>
__device__ __forceinline__ void load8_w(const T* p, float* f) {
  if constexpr (sizeof(T) == 2) {
    load8_src(reinterpret_cast<const __nv_bfloat16*>(p), f);
  } else {
    load8_src(reinterpret_cast<const float*>(p), f);
  }
}

// the source row of output row o: token src_tok[o / nfl] (o / nfl without a map),
// block o % nfl of width H
template <typename TX>
__device__ __forceinline__ const TX* src_row(const TX* x, int64_t ldx, const int64_t* src_tok,
                                             int nfl, int64_t H, int64_t o) {
  const int64_t t = o / nfl;
  const int64_t tok = src_tok ? src_tok[t] : t;
  return x + tok * ldx + (o - t * nfl) * H;
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += sh[i];
  return t;
}

// one block per output row, thread t owns columns [8 t, 8 t + 8) (blockDim = H / 8)
template <typename TX, typename T>
__global__ void feature_norm_fwd_kernel(int64_t orows, int64_t H, int nfl, const TX* __restrict__ x,
                                        int64_t ldx, const int64_t* __restrict__ src_tok,
                                        const T* __restrict__ w, T* __restrict__ y, int64_t ldy,
                                        float* __restrict__ rstd, float eps) {
  __shared__ float sh[32];
  const int64_t o = blockIdx.x;
  const int64_t c = (int64_t)threadIdx.x * 8;
  float f[8];
  load8_src(src_row(x, ldx, src_tok, nfl, H, o) + c, f);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    f[k] = round_to<T>(f[k]);  // the reference's features.to(dtype)
    ss += f[k] * f[k];
  }
  const float r = rsqrtf(block_sum(ss, sh) / (float)H + eps);
  if (threadIdx.x == 0 && rstd) rstd[o] = r;
  float g[8];
  load8_w(w + c, g);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = (f[k] * r) * g[k];
  store8(y + o * ldy + c, f);
}

// dw_partial[b, c] = sum over the rows block b visits of dy[o, c] * x[o, c] * rstd[o]
template <typename TX, typename T>
__global__ void feature_norm_dw_kernel(int64_t orows, int64_t H, int nfl, const T* __restrict__ dy,
                                       int64_t lddy, const TX* __restrict__ x, int64_t ldx,
                                       const int64_t* __restrict__ src_tok,
                                       const float* __restrict__ rstd,
                                       float* __restrict__ dw_partial) {
  const int64_t c = (int64_t)threadIdx.x * 8;
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  for (int64_t o = blockIdx.x; o < orows; o += gridDim.x) {
    float a[8], b[8];
    load8_w(dy + o * lddy + c, a);
    load8_src(src_row(x, ldx, src_tok, nfl, H, o) + c, b);
    const float rr = rstd[o];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] += a[k] * (round_to<T>(b[k]) * rr);
  }
  store8(dw_partial + (int64_t)blockIdx.x * H + c, acc);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename F>
int dispatch_src(int x_dtype, F&& f) {
  if (x_dtype == PE_F16) return f(static_cast<const __half*>(nullptr));
  if (x_dtype == PE_BF16) return f(static_cast<const __nv_bfloat16*>(nullptr));
  if (x_dtype == PE_F32) return f(static_cast<const float*>(nullptr));
  set_error("feature norm: unsupported source dtype code %d", x_dtype);
  return PE_ERR_ARG;
}

int check_shape(int x_dtype, int64_t tokens, int nfl, int64_t H, const void* x, int64_t ldx) {
  // one thread per 8 columns, whole warps: H a multiple of 256 up to 8192
  PE_CHECK_ARG(tokens >= 0 && nfl >= 1 && H >= 256 && H % 256 == 0 && H <= 8192,
               "feature norm: H must be a multiple of 256 up to 8192 (got %lld)", (long long)H);
  PE_CHECK_ARG(ldx >= nfl * H && ldx % 8 == 0 && al16(x),
               "feature norm: source rows must hold nfl * H elements, 16-byte aligned");
  PE_CHECK_ARG(x_dtype == PE_F16 || x_dtype == PE_BF16 || x_dtype == PE_F32,
               "feature norm: source dtype code %d not F16/BF16/F32", x_dtype);
  return PE_OK;
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_feature_norm_fwd(int x_dtype, int dtype, int64_t tokens, int nfl, int64_t H,
                                   const void* x, int64_t ldx, const int64_t* src_tok,
                                   const void* w, void* y, int64_t ldy, float* rstd, float eps,
                                   void* stream) {
  int rc = check_shape(x_dtype, tokens, nfl, H, x, ldx);
  if (rc) return rc;
  PE_CHECK_ARG(ldy >= H && ldy % 8 == 0 && al16(y) && al16(w),
               "feature norm: output rows must be 16-byte aligned");
  const int64_t orows = tokens * nfl;
  if (orows == 0) return PE_OK;
  PE_CHECK_ARG(orows <= 0x7fffffffll, "feature norm: too many rows");
  return PE_DISPATCH(dtype, T, [&] {
    return dispatch_src(x_dtype, [&](auto tag) {
      using TX = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
      feature_norm_fwd_kernel<TX, T><<<(unsigned)orows, (unsigned)(H / 8), 0, as_stream(stream)>>>(
          orows, H, nfl, static_cast<const TX*>(x), ldx, src_tok, static_cast<const T*>(w),
          static_cast<T*>(y), ldy, rstd, eps);
      PE_LAUNCHED();
      return PE_OK;
    });
  });
}

extern "C" int pe_feature_norm_dw(int x_dtype, int dtype, int64_t tokens, int nfl, int64_t H,
                                  const void* dy, int64_t lddy, const void* x, int64_t ldx,
                                  const int64_t* src_tok, const float* rstd, float* dw_partial,
                                  void* stream) {
  int rc = check_shape(x_dtype, tokens, nfl, H, x, ldx);
  if (rc) return rc;
  PE_CHECK_ARG(lddy >= H && lddy % 8 == 0 && al16(dy) && al16(dw_partial),
               "feature norm: dy rows must be 16-byte aligned");
  const int64_t orows = tokens * nfl;
  const int64_t nblk = pe_rmsnorm_bwd_blocks(orows);
  if (orows == 0) {
    PE_CUDA_TRY(cudaMemsetAsync(dw_partial, 0, nblk * H * 4, as_stream(stream)));
    return PE_OK;
  }
  return PE_DISPATCH(dtype, T, [&] {
    return dispatch_src(x_dtype, [&](auto tag) {
      using TX = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
      feature_norm_dw_kernel<TX, T><<<(unsigned)nblk, (unsigned)(H / 8), 0, as_stream(stream)>>>(
          orows, H, nfl, static_cast<const T*>(dy), lddy, static_cast<const TX*>(x), ldx, src_tok,
          rstd, dw_partial);
      PE_LAUNCHED();
      return PE_OK;
    });
  });
}
