// Small memory-bound pieces of the drafter input and MLP: embedding gather,
// broadcast of the shared prediction-slot input, SwiGLU (reference
// src/pe/nn.py:99-100, src/pe/drafter.py:126-137), row scatter/gather for the
// loss-slot compaction, column sums for the shared-input backward, casts.
#include <cooperative_groups.h>

#include "common.cuh"

namespace pe {
namespace {

namespace cg = cooperative_groups;

template <typename T>
__global__ void embed_rows_kernel(int64_t rows, int64_t H, const int64_t* __restrict__ ids,
                                  const T* __restrict__ embed, T* __restrict__ out, int64_t ldo) {
  const int64_t r = blockIdx.y;
  const int64_t id = ids[r];
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < H;
       c += (int64_t)gridDim.x * blockDim.x)
    out[r * ldo + c] = embed[id * H + c];
}

template <typename T>
__global__ void fill_rows_kernel(int64_t rows, int64_t H, const T* __restrict__ vec,
                                 T* __restrict__ out, int64_t ldo) {
  const int64_t total = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H, c = i - r * H;
    out[r * ldo + c] = vec[c];
  }
}

// sigmoid(x) = 1 / (1 + e^-x).  bf16 storage: from the hardware exp2 and reciprocal
// approximations (a few ulp in fp32, before the result is rounded to bf16) -- the
// gate|up GEMM's fused SwiGLU epilogue evaluates the same expression, so the fused and
// element-wise paths give the same bits.  fp32 storage: the accurate expf and division.
template <typename T>
__device__ __forceinline__ float sigmoid_t(float x) {
  if constexpr (sizeof(T) == 2) {
    return __fdividef(1.0f, 1.0f + __expf(-x));
  } else {
    return 1.0f / (1.0f + expf(-x));
  }
}
__device__ __forceinline__ float sigmoidf_(float x) { return sigmoid_t<__nv_bfloat16>(x); }

template <typename T>
__global__ void swiglu_fwd_kernel(int64_t rows, int64_t I, const T* __restrict__ gu, int64_t ldgu,
                                  T* __restrict__ a, int64_t lda) {
  const int64_t total = rows * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / I, c = i - r * I;
    const float g = to_f(gu[r * ldgu + c]);
    const float u = to_f(gu[r * ldgu + I + c]);
    const float act = round_to<T>(g * sigmoid_t<T>(g));
    a[r * lda + c] = from_f<T>(act * u);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(int64_t rows, int64_t I, const T* __restrict__ da, int64_t ldda,
                                  const T* __restrict__ gu, int64_t ldgu, T* __restrict__ dgu,
                                  int64_t lddgu) {
  const int64_t total = rows * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / I, c = i - r * I;
    const float d = to_f(da[r * ldda + c]);
    const float g = to_f(gu[r * ldgu + c]);
    const float u = to_f(gu[r * ldgu + I + c]);
    const float s = sigmoid_t<T>(g);
    const float act = round_to<T>(g * s);
    const float dact = round_to<T>(d * u);
    dgu[r * lddgu + I + c] = from_f<T>(d * act);
    dgu[r * lddgu + c] = from_f<T>(dact * (s * (1.0f + g * (1.0f - s))));
  }
}

// Vectorised SwiGLU for bf16 rows with I % 8 == 0: 8 columns (16 B) per thread,
// blockIdx.y = row, so no per-element index division.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

__global__ void swiglu_fwd_vec_kernel(int64_t I, const __nv_bfloat16* __restrict__ gu,
                                      int64_t ldgu, __nv_bfloat16* __restrict__ a, int64_t lda) {
  const int64_t r = blockIdx.y;
  const int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= I) return;
  float g[8], u[8], o[8];
  load8(gu + r * ldgu + c, g);
  load8(gu + r * ldgu + I + c, u);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = round_to<__nv_bfloat16>(g[i] * sigmoidf_(g[i])) * u[i];
  store8(a + r * lda + c, o);
}

__global__ void swiglu_bwd_vec_kernel(int64_t I, const __nv_bfloat16* __restrict__ da,
                                      int64_t ldda, const __nv_bfloat16* __restrict__ gu,
                                      int64_t ldgu, __nv_bfloat16* __restrict__ dgu,
                                      int64_t lddgu) {
  const int64_t r = blockIdx.y;
  const int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= I) return;
  float d[8], g[8], u[8], dg[8], du[8];
  load8(da + r * ldda + c, d);
  load8(gu + r * ldgu + c, g);
  load8(gu + r * ldgu + I + c, u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float s = sigmoidf_(g[i]);
    const float act = round_to<__nv_bfloat16>(g[i] * s);
    const float dact = round_to<__nv_bfloat16>(d[i] * u[i]);
    du[i] = d[i] * act;
    dg[i] = dact * (s * (1.0f + g[i] * (1.0f - s)));
  }
  store8(dgu + r * lddgu + c, dg);
  store8(dgu + r * lddgu + I + c, du);
}

bool vec8_ok(const void* p, int64_t ld) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ld % 8 == 0;
}

// out[c] (+)= sum_r x[r, c]; 32 columns per block, 8 row lanes, fixed order.
template <typename T>
__global__ void rowsum_cols_kernel(int64_t rows, int64_t H, const T* __restrict__ x, int64_t ldx,
                                   float* __restrict__ out, int accumulate) {
  __shared__ float red[8][33];
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < H)
    for (int64_t r = threadIdx.y; r < rows; r += 8) s += to_f(x[r * ldx + c]);
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < H) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][threadIdx.x];
    out[c] = accumulate ? out[c] + t : t;
  }
}

// Column sums over several row ranges of x (16-byte loads, H % 8 == 0): a cluster of
// kSplit blocks shares one 128-column slab, block k of the cluster taking every
// kSplit-th group of 16 rows of every range; each block sums its 16 row lanes in a fixed
// order and block 0 of the cluster adds the kSplit block sums, read from the others'
// shared memory, in rank order.  Deterministic, and 8x the blocks of one block per slab.
constexpr int kRowsumSplit = 8;
constexpr int kRowsumRanges = 16;
struct RowRanges {
  int n;
  int64_t begin[kRowsumRanges], end[kRowsumRanges];
};

__device__ __forceinline__ void load8f(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void load8f(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename T>
__global__ void __cluster_dims__(1, kRowsumSplit, 1) __launch_bounds__(256)
    rowsum_ranges_kernel(const __grid_constant__ RowRanges rr, int64_t H,
                         const T* __restrict__ x, int64_t ldx, float* __restrict__ out) {
  __shared__ float red[16][129];
  __shared__ float part[128];
  cg::cluster_group cluster = cg::this_cluster();
  const int lane16 = threadIdx.x & 15, rl = threadIdx.x >> 4;
  const int64_t c = (int64_t)blockIdx.x * 128 + lane16 * 8;
  const int rank = (int)cluster.block_rank();
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (c < H) {
    const int64_t step = 16 * kRowsumSplit;
    for (int g = 0; g < rr.n; ++g) {
      int64_t r = rr.begin[g] + rank * 16 + rl;
      const int64_t e = rr.end[g];
      // two rows' loads in flight per iteration
      for (; r + step < e; r += 2 * step) {
        float a[8], b[8];
        load8f(x + r * ldx + c, a);
        load8f(x + (r + step) * ldx + c, b);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += a[i] + b[i];
      }
      if (r < e) {
        float a[8];
        load8f(x + r * ldx + c, a);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += a[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[rl][lane16 * 8 + i] = acc[i];
  __syncthreads();
  if (threadIdx.x < 128) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) t += red[i][threadIdx.x];
    part[threadIdx.x] = t;
  }
  cluster.sync();  // every block's part[] is written
  if (rank == 0 && threadIdx.x < 128) {
    const int64_t col = (int64_t)blockIdx.x * 128 + threadIdx.x;
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kRowsumSplit; ++k) t += cluster.map_shared_rank(part, k)[threadIdx.x];
    if (col < H) out[col] = t;
  }
  cluster.sync();  // block 0 has read the others' part[] before they exit
}

template <typename T>
__global__ void move_rows_kernel(int64_t rows, int64_t H, const int64_t* __restrict__ idx,
                                 const T* __restrict__ src, int64_t lds, T* __restrict__ dst,
                                 int64_t ldd, int scatter) {
  const int64_t r = blockIdx.y;
  const int64_t s_row = scatter ? r : idx[r];
  const int64_t d_row = scatter ? idx[r] : r;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < H;
       c += (int64_t)gridDim.x * blockDim.x)
    dst[d_row * ldd + c] = src[s_row * lds + c];
}

// Row moves in 16-byte units (rows whose bytes and strides are multiples of 16):
// dst row d(r) = src row s(r) with mode 0 gather (s = idx[r], d = r), 1 scatter
// (s = r, d = idx[r]), 2 broadcast (s = 0, the source stride 0).  Thread = one
// 16-byte unit of a row; blockIdx.y walks the rows.
__global__ void move_rows16_kernel(int64_t rows, int n16, const int64_t* __restrict__ idx,
                                   const uint4* __restrict__ src, int64_t lds16,
                                   uint4* __restrict__ dst, int64_t ldd16, int mode) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n16) return;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t s = mode == 0 ? idx[r] : (mode == 1 ? r : 0);
    const int64_t d = mode == 1 ? idx[r] : r;
    dst[d * ldd16 + c] = src[s * lds16 + c];
  }
}

// true (and the 16-byte row geometry filled in) when every row start is 16-byte aligned
bool rows16(int64_t H, size_t es, const void* a, int64_t lda, const void* b, int64_t ldb,
            int& n16, int64_t& lda16, int64_t& ldb16) {
  const int64_t bytes = H * (int64_t)es;
  if (bytes % 16 || (lda * (int64_t)es) % 16 || (ldb * (int64_t)es) % 16 ||
      (reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(b) & 15u) ||
      bytes / 16 > (1 << 30))
    return false;
  n16 = (int)(bytes / 16);
  lda16 = lda * (int64_t)es / 16;
  ldb16 = ldb * (int64_t)es / 16;
  return true;
}

int launch_rows16(int64_t rows, int n16, const int64_t* idx, const void* src, int64_t lds16,
                  void* dst, int64_t ldd16, int mode, cudaStream_t st) {
  constexpr int kT = 128;
  dim3 grid((unsigned)ceil_div((int64_t)n16, (int64_t)kT),
            (unsigned)(rows < 32768 ? rows : 32768));
  move_rows16_kernel<<<grid, kT, 0, st>>>(rows, n16, idx, static_cast<const uint4*>(src), lds16,
                                          static_cast<uint4*>(dst), ldd16, mode);
  PE_LAUNCHED();
  return PE_OK;
}

template <typename T>
__global__ void cast_kernel(int64_t n, const float* __restrict__ x, T* __restrict__ y) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f<T>(x[i]);
}

unsigned grid_for(int64_t n, int threads) {
  int64_t g = ceil_div(n, threads);
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_embed_rows(int dtype, int64_t rows, int64_t H, const int64_t* ids,
                             const void* embed, void* out, int64_t ldo, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0 && ldo >= H, "embed_rows: bad shape");
  if (rows == 0) return PE_OK;
  {
    int n16;
    int64_t le16, lo16;
    if ((dtype == PE_F32 || dtype == PE_BF16) &&
        rows16(H, dtype == PE_F32 ? 4 : 2, embed, H, out, ldo, n16, le16, lo16))
      return launch_rows16(rows, n16, ids, embed, le16, out, lo16, 0, as_stream(stream));
  }
  PE_CHECK_ARG(rows <= 65535, "embed_rows: rows > 65535");
  dim3 grid((unsigned)ceil_div(H, 256 * 4), (unsigned)rows);
  return PE_DISPATCH(dtype, T, [&] {
    embed_rows_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(rows, H, ids, (const T*)embed,
                                                              (T*)out, ldo);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_fill_rows(int dtype, int64_t rows, int64_t H, const void* vec, void* out,
                            int64_t ldo, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0 && ldo >= H, "fill_rows: bad shape");
  if (rows == 0) return PE_OK;
  {
    int n16;
    int64_t lv16, lo16;
    if ((dtype == PE_F32 || dtype == PE_BF16) &&
        rows16(H, dtype == PE_F32 ? 4 : 2, vec, 0, out, ldo, n16, lv16, lo16))
      return launch_rows16(rows, n16, nullptr, vec, 0, out, lo16, 2, as_stream(stream));
  }
  return PE_DISPATCH(dtype, T, [&] {
    fill_rows_kernel<T><<<grid_for(rows * H, 256), 256, 0, as_stream(stream)>>>(
        rows, H, (const T*)vec, (T*)out, ldo);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_swiglu_fwd(int dtype, int64_t rows, int64_t I, const void* gu, int64_t ldgu,
                             void* a, int64_t lda, void* stream) {
  PE_CHECK_ARG(rows >= 0 && I > 0 && ldgu >= 2 * I && lda >= I, "swiglu_fwd: bad shape");
  if (rows == 0) return PE_OK;
  if (dtype == PE_BF16 && I % 8 == 0 && rows <= 65535 && vec8_ok(gu, ldgu) && vec8_ok(a, lda)) {
    dim3 grid((unsigned)ceil_div(I / 8, 256), (unsigned)rows);
    swiglu_fwd_vec_kernel<<<grid, 256, 0, as_stream(stream)>>>(
        I, (const __nv_bfloat16*)gu, ldgu, (__nv_bfloat16*)a, lda);
    PE_LAUNCHED();
    return PE_OK;
  }
  return PE_DISPATCH(dtype, T, [&] {
    swiglu_fwd_kernel<T><<<grid_for(rows * I, 256), 256, 0, as_stream(stream)>>>(
        rows, I, (const T*)gu, ldgu, (T*)a, lda);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_swiglu_bwd(int dtype, int64_t rows, int64_t I, const void* da, int64_t ldda,
                             const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                             void* stream) {
  PE_CHECK_ARG(rows >= 0 && I > 0 && ldgu >= 2 * I && lddgu >= 2 * I && ldda >= I,
               "swiglu_bwd: bad shape");
  if (rows == 0) return PE_OK;
  if (dtype == PE_BF16 && I % 8 == 0 && rows <= 65535 && vec8_ok(da, ldda) && vec8_ok(gu, ldgu) &&
      vec8_ok(dgu, lddgu)) {
    dim3 grid((unsigned)ceil_div(I / 8, 256), (unsigned)rows);
    swiglu_bwd_vec_kernel<<<grid, 256, 0, as_stream(stream)>>>(
        I, (const __nv_bfloat16*)da, ldda, (const __nv_bfloat16*)gu, ldgu, (__nv_bfloat16*)dgu,
        lddgu);
    PE_LAUNCHED();
    return PE_OK;
  }
  return PE_DISPATCH(dtype, T, [&] {
    swiglu_bwd_kernel<T><<<grid_for(rows * I, 256), 256, 0, as_stream(stream)>>>(
        rows, I, (const T*)da, ldda, (const T*)gu, ldgu, (T*)dgu, lddgu);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_rowsum_cols_ranges(int dtype, int nranges, const int64_t* ranges, int64_t H,
                                     const void* x, int64_t ldx, float* out, void* stream) {
  PE_CHECK_ARG(nranges >= 1 && nranges <= kRowsumRanges && ranges != nullptr,
               "rowsum_cols_ranges: 1 to %d row ranges (got %d)", kRowsumRanges, nranges);
  PE_CHECK_ARG(H > 0 && ldx >= H, "rowsum_cols_ranges: bad shape");
  RowRanges rr{};
  rr.n = nranges;
  for (int g = 0; g < nranges; ++g) {
    PE_CHECK_ARG(ranges[2 * g] >= 0 && ranges[2 * g + 1] >= ranges[2 * g],
                 "rowsum_cols_ranges: range %d is [%lld, %lld)", g, (long long)ranges[2 * g],
                 (long long)ranges[2 * g + 1]);
    rr.begin[g] = ranges[2 * g];
    rr.end[g] = ranges[2 * g + 1];
  }
  const size_t esz = dtype == PE_F32 ? 4 : 2;
  const bool vec = (dtype == PE_BF16 || dtype == PE_F32) && H % 8 == 0 &&
                   (ldx * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  if (!vec) {
    // one range at a time on the scalar kernel, the sums added in range order
    for (int g = 0; g < nranges; ++g) {
      const int64_t rows = rr.end[g] - rr.begin[g];
      const uint8_t* xg = static_cast<const uint8_t*>(x) + (size_t)rr.begin[g] * ldx * esz;
      int rc = PE_DISPATCH(dtype, T, [&] {
        rowsum_cols_kernel<T><<<(unsigned)ceil_div(H, 32), dim3(32, 8), 0, as_stream(stream)>>>(
            rows, H, (const T*)xg, ldx, out, g > 0 ? 1 : 0);
        PE_LAUNCHED();
        return PE_OK;
      });
      if (rc) return rc;
    }
    return PE_OK;
  }
  const dim3 grid((unsigned)ceil_div(H, 128), kRowsumSplit);
  if (dtype == PE_BF16)
    rowsum_ranges_kernel<__nv_bfloat16><<<grid, 256, 0, as_stream(stream)>>>(
        rr, H, static_cast<const __nv_bfloat16*>(x), ldx, out);
  else
    rowsum_ranges_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(
        rr, H, static_cast<const float*>(x), ldx, out);
  PE_LAUNCHED();
  return PE_OK;
}

extern "C" int pe_rowsum_cols(int dtype, int64_t rows, int64_t H, const void* x, int64_t ldx,
                              float* out, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0 && ldx >= H, "rowsum_cols: bad shape");
  if (rows > 0) {
    const int64_t range[2] = {0, rows};
    return pe_rowsum_cols_ranges(dtype, 1, range, H, x, ldx, out, stream);
  }
  return PE_DISPATCH(dtype, T, [&] {
    rowsum_cols_kernel<T><<<(unsigned)ceil_div(H, 32), dim3(32, 8), 0, as_stream(stream)>>>(
        rows, H, (const T*)x, ldx, out, 0);
    PE_LAUNCHED();
    return PE_OK;
  });
}

static int move_rows(int dtype, int64_t rows, int64_t H, const int64_t* idx, const void* src,
                     int64_t lds, void* dst, int64_t ldd, int scatter, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0 && lds >= H && ldd >= H, "scatter/gather rows: bad shape");
  if (rows == 0) return PE_OK;
  {
    int n16;
    int64_t ls16, ld16;
    if ((dtype == PE_F32 || dtype == PE_BF16) &&
        rows16(H, dtype == PE_F32 ? 4 : 2, src, lds, dst, ldd, n16, ls16, ld16))
      return launch_rows16(rows, n16, idx, src, ls16, dst, ld16, scatter ? 1 : 0,
                           as_stream(stream));
  }
  PE_CHECK_ARG(rows <= 65535, "scatter/gather rows: rows > 65535");
  dim3 grid((unsigned)ceil_div(H, 256 * 4), (unsigned)rows);
  return PE_DISPATCH(dtype, T, [&] {
    move_rows_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(rows, H, idx, (const T*)src, lds,
                                                             (T*)dst, ldd, scatter);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_scatter_rows(int dtype, int64_t rows, int64_t H, const int64_t* idx,
                               const void* src, int64_t lds, void* dst, int64_t ldd,
                               void* stream) {
  return move_rows(dtype, rows, H, idx, src, lds, dst, ldd, 1, stream);
}

extern "C" int pe_gather_rows(int dtype, int64_t rows, int64_t H, const int64_t* idx,
                              const void* src, int64_t lds, void* dst, int64_t ldd,
                              void* stream) {
  return move_rows(dtype, rows, H, idx, src, lds, dst, ldd, 0, stream);
}

extern "C" int pe_cast_f32(int dtype, int64_t n, const float* x, void* y, void* stream) {
  PE_CHECK_ARG(n >= 0, "cast: bad size");
  if (n == 0) return PE_OK;
  return PE_DISPATCH(dtype, T, [&] {
    cast_kernel<T><<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(n, x, (T*)y);
    PE_LAUNCHED();
    return PE_OK;
  });
}
