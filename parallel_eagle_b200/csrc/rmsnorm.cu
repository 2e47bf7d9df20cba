// RMSNorm forward/backward (reference src/pe/nn.py:16-26) and the column
// reduction that turns per-block weight-gradient partials into dw.
//
// One warp per row.  The vector path moves 8 elements (16 B of bf16) per lane
// per access, so a warp touches 512 contiguous bytes per instruction; rows of a
// few KB stay in L1 between the two passes.  HBM traffic per row: forward reads
// x once and writes y (+4 B rstd); backward reads dy, x (+residual) once and
// writes dx.
#include "common.cuh"

namespace pe {
namespace {

constexpr int kWarps = 8;

template <typename T, int VEC>
struct Vec;
template <typename T>
struct Vec<T, 1> {
  __device__ __forceinline__ static void load(const T* p, float* f) { f[0] = to_f(p[0]); }
  __device__ __forceinline__ static void store(T* p, const float* f) { p[0] = from_f<T>(f[0]); }
};
template <>
struct Vec<__nv_bfloat16, 8> {
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float* f) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, const float* f) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec<float, 8> {
  __device__ __forceinline__ static void load(const float* p, float* f) {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ __forceinline__ static void store(float* p, const float* f) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

template <typename T, int VEC>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_kernel(int64_t rows, int64_t H, const T* __restrict__ x, int64_t ldx,
                   const T* __restrict__ w, T* __restrict__ y, int64_t ldy,
                   float* __restrict__ rstd, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * ldx;
  T* yr = y + row * ldy;
  float ss = 0.f;
  for (int64_t c = (int64_t)lane * VEC; c < H; c += 32 * VEC) {
    float f[VEC];
    Vec<T, VEC>::load(xr + c, f);
#pragma unroll
    for (int i = 0; i < VEC; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)H + eps);
  if (lane == 0 && rstd) rstd[row] = r;
  for (int64_t c = (int64_t)lane * VEC; c < H; c += 32 * VEC) {
    float f[VEC], g[VEC];
    Vec<T, VEC>::load(xr + c, f);
    Vec<T, VEC>::load(w + c, g);
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = (f[i] * r) * g[i];
    Vec<T, VEC>::store(yr + c, f);
  }
}

// bf16 rows of up to 4096 columns (H % 8 == 0): one warp per row keeps the whole
// row in registers (16-byte chunks), so x is read from HBM exactly once.
constexpr int kFwdRegChunks = 16;

__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_fwd_reg_kernel(int64_t rows, int64_t H, const __nv_bfloat16* __restrict__ x,
                       int64_t ldx, const __nv_bfloat16* __restrict__ w,
                       __nv_bfloat16* __restrict__ y, int64_t ldy, float* __restrict__ rstd,
                       float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int ngroups = (int)(H / 8);
  const __nv_bfloat16* xr = x + row * ldx;
  __nv_bfloat16* yr = y + row * ldy;
  uint4 raw[kFwdRegChunks];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kFwdRegChunks; ++i) {
    const int gi = lane + 32 * i;
    if (gi < ngroups) raw[i] = *reinterpret_cast<const uint4*>(xr + gi * 8);
  }
#pragma unroll
  for (int i = 0; i < kFwdRegChunks; ++i) {
    const int gi = lane + 32 * i;
    if (gi < ngroups) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)H + eps);
  if (lane == 0 && rstd) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < kFwdRegChunks; ++i) {
    const int gi = lane + 32 * i;
    if (gi < ngroups) {
      float f[8], g[8];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 t = __bfloat1622float2(h[k]);
        f[2 * k] = t.x;
        f[2 * k + 1] = t.y;
      }
      Vec<__nv_bfloat16, 8>::load(w + gi * 8, g);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = (f[k] * r) * g[k];
      Vec<__nv_bfloat16, 8>::store(yr + gi * 8, f);
    }
  }
}

template <typename T, int VEC>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_kernel(int64_t rows, int64_t H, const T* __restrict__ dy, int64_t lddy,
                   const T* __restrict__ x, int64_t ldx, const T* __restrict__ w,
                   const float* __restrict__ rstd, T* dx, int64_t lddx, const T* res,
                   int64_t ldres, float* __restrict__ dw_partial) {
  extern __shared__ float sdw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (dw_partial) {
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) sdw[c] = 0.f;
    __syncthreads();
  }
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const T* dyr = dy + row * lddy;
    const T* xr = x + row * ldx;
    const float r = rstd[row];
    float s = 0.f;
    for (int64_t c = (int64_t)lane * VEC; c < H; c += 32 * VEC) {
      float a[VEC], b[VEC], g[VEC];
      Vec<T, VEC>::load(dyr + c, a);
      Vec<T, VEC>::load(xr + c, b);
      Vec<T, VEC>::load(w + c, g);
#pragma unroll
      for (int i = 0; i < VEC; ++i) s += (a[i] * g[i]) * b[i];
    }
    s = warp_sum(s);
    const float coef = s * r * r * r / (float)H;
    T* dxr = dx + row * lddx;
    const T* rr = res ? res + row * ldres : nullptr;
    for (int64_t c = (int64_t)lane * VEC; c < H; c += 32 * VEC) {
      float a[VEC], b[VEC], g[VEC], o[VEC];
      Vec<T, VEC>::load(dyr + c, a);
      Vec<T, VEC>::load(xr + c, b);
      Vec<T, VEC>::load(w + c, g);
      if (rr) {
        Vec<T, VEC>::load(rr + c, o);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) o[i] += r * (a[i] * g[i]) - b[i] * coef;
      Vec<T, VEC>::store(dxr + c, o);
      if (dw_partial) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) atomicAdd(&sdw[c + i], a[i] * (b[i] * r));
      }
    }
  }
  if (dw_partial) {
    __syncthreads();
    float* out = dw_partial + (int64_t)blockIdx.x * H;
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) out[c] = sdw[c];
  }
}

// Backward for rows whose width is a multiple of 256 (up to 4096): lane l owns
// the 8 contiguous columns c*256 + 8l.. of every 256-column chunk c, so the
// weight-gradient partial stays in registers across all rows a warp handles and
// the block reduces it through shared memory once at the end (no per-element
// shared-memory atomics).  Two passes over each row; the second re-reads dy and x
// from L1.
constexpr int kMaxChunks = 16;

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_chunked_kernel(int64_t rows, int64_t H, int nch, const T* __restrict__ dy,
                           int64_t lddy, const T* __restrict__ x, int64_t ldx,
                           const T* __restrict__ w, const float* __restrict__ rstd, T* dx,
                           int64_t lddx, const T* res, int64_t ldres,
                           float* __restrict__ dw_partial) {
  extern __shared__ float sdw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[kMaxChunks][8];
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[i][k] = 0.f;
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const T* dyr = dy + row * lddy;
    const T* xr = x + row * ldx;
    const float r = rstd[row];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      if (i < nch) {
        const int64_t c = (int64_t)i * 256 + lane * 8;
        float a[8], b[8], g[8];
        Vec<T, 8>::load(dyr + c, a);
        Vec<T, 8>::load(xr + c, b);
        Vec<T, 8>::load(w + c, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += (a[k] * g[k]) * b[k];
      }
    }
    s = warp_sum(s);
    const float coef = s * r * r * r / (float)H;
    T* dxr = dx + row * lddx;
    const T* rr = res ? res + row * ldres : nullptr;
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      if (i < nch) {
        const int64_t c = (int64_t)i * 256 + lane * 8;
        float a[8], b[8], g[8], o[8];
        Vec<T, 8>::load(dyr + c, a);
        Vec<T, 8>::load(xr + c, b);
        Vec<T, 8>::load(w + c, g);
        if (rr) {
          Vec<T, 8>::load(rr + c, o);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o[k] += r * (a[k] * g[k]) - b[k] * coef;
          acc[i][k] += a[k] * (b[k] * r);
        }
        Vec<T, 8>::store(dxr + c, o);
      }
    }
  }
  if (dw_partial) {
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) sdw[c] = 0.f;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      if (i < nch) {
#pragma unroll
        for (int k = 0; k < 8; ++k) atomicAdd(&sdw[i * 256 + lane * 8 + k], acc[i][k]);
      }
    }
    __syncthreads();
    float* out = dw_partial + (int64_t)blockIdx.x * H;
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) out[c] = sdw[c];
  }
}

// Backward over tiles of kTileRows rows, persistent blocks.  Per tile: one warp
// per row reduces s = sum_c dy w x into the row coefficient; then the block walks
// the tile row by row with thread t owning 8 contiguous columns (coalesced 16-byte
// accesses), writing dx and keeping those columns' dW partial in 8 registers
// across every tile it visits.  The second read of the tile's dy / x comes from
// L2: a block's tile is a few hundred KB and only ~2 blocks per SM are in flight.
constexpr int kTileRows = 16;
constexpr int kTiledThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kTiledThreads)
rmsnorm_bwd_tiled_kernel(int64_t rows, int64_t H, const T* __restrict__ dy, int64_t lddy,
                         const T* __restrict__ x, int64_t ldx, const T* __restrict__ w,
                         const float* __restrict__ rstd, T* dx, int64_t lddx, const T* res,
                         int64_t ldres, float* __restrict__ dw_partial) {
  __shared__ float s_coef[kTileRows], s_rstd[kTileRows];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ngroups = (int)(H / 8);
  const int64_t ntiles = (rows + kTileRows - 1) / kTileRows;
  // this thread's column groups: threadIdx.x, + blockDim.x (at most 2 for H <= 4096)
  constexpr int kMaxGroups = 2;
  float acc[kMaxGroups][8];
#pragma unroll
  for (int q = 0; q < kMaxGroups; ++q)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[q][k] = 0.f;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t r0 = t * kTileRows;
    const int nr = (int)((rows - r0) < kTileRows ? (rows - r0) : kTileRows);
    for (int i = warp; i < nr; i += kTiledThreads / 32) {
      const int64_t r = r0 + i;
      const T* dyr = dy + r * lddy;
      const T* xr = x + r * ldx;
      // all of the row's loads issue before the first multiply-add (fully unrolled,
      // H <= 16 * 32 * 8): the row costs one memory latency, not one per chunk
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int gi = lane + 32 * i;
        if (gi < ngroups) {
          float a[8], b[8], g[8];
          Vec<T, 8>::load(dyr + gi * 8, a);
          Vec<T, 8>::load(xr + gi * 8, b);
          Vec<T, 8>::load(w + gi * 8, g);
#pragma unroll
          for (int k = 0; k < 8; ++k) s += (a[k] * g[k]) * b[k];
        }
      }
      s = warp_sum(s);
      if (lane == 0) {
        const float rr = rstd[r];
        s_rstd[i] = rr;
        s_coef[i] = s * rr * rr * rr / (float)H;
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kMaxGroups; ++q) {
      const int gi = threadIdx.x + q * kTiledThreads;
      if (gi < ngroups) {
        const int64_t c = (int64_t)gi * 8;
        float g[8];
        Vec<T, 8>::load(w + c, g);
#pragma unroll 4
        for (int i = 0; i < nr; ++i) {
          const int64_t r = r0 + i;
          float a[8], b[8], o[8];
          Vec<T, 8>::load(dy + r * lddy + c, a);
          Vec<T, 8>::load(x + r * ldx + c, b);
          if (res) {
            Vec<T, 8>::load(res + r * ldres + c, o);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = 0.f;
          }
          const float rr = s_rstd[i], cf = s_coef[i];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            o[k] += rr * (a[k] * g[k]) - b[k] * cf;
            acc[q][k] += a[k] * (b[k] * rr);
          }
          Vec<T, 8>::store(dx + r * lddx + c, o);
        }
      }
    }
    __syncthreads();
  }
  if (dw_partial) {
#pragma unroll
    for (int q = 0; q < kMaxGroups; ++q) {
      const int gi = threadIdx.x + q * kTiledThreads;
      if (gi < ngroups) Vec<float, 8>::store(dw_partial + (int64_t)blockIdx.x * H + gi * 8, acc[q]);
    }
  }
}

// bf16 backward for rows of H = 512 W columns (W <= 8), one block of W warps per row at
// a time: lane l of warp v owns columns 8 (32 (2 v + i) + l) .. + 8 for i = 0, 1, so each
// thread holds two 16-byte chunks of dy, x and the residual (all loads of a row issued
// together: one DRAM round trip per row) and the block adds its warps' parts of
// sum(dy w x) through shared memory (one barrier per row; the slots alternate with the
// row parity).  Every thread keeps the weight-gradient partial of its 16 columns in
// registers across all the rows its block visits and writes it once into the block's
// row of dw_partial -- no per-row shared-memory traffic.  Two blocks per SM (the
// persistent grid's size) at <= 146 registers: 14 warps per SM at H = 3584, against 8
// for the one-warp-per-row kernel below.
template <int W>
__global__ void __launch_bounds__(W * 32, 2)
rmsnorm_bwd_rowblock_kernel(int64_t rows, const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                            const __nv_bfloat16* __restrict__ x, int64_t ldx,
                            const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                            __nv_bfloat16* dx, int64_t lddx, const __nv_bfloat16* res,
                            int64_t ldres, float* __restrict__ dw_partial) {
  constexpr int H = W * 512;
  __shared__ float s_part[2][W];  // [row parity][warp]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = ((2 * warp) * 32 + lane) * 8, c1 = c0 + 256;
  float g[16];
  Vec<__nv_bfloat16, 8>::load(w + c0, g);
  Vec<__nv_bfloat16, 8>::load(w + c1, g + 8);
  float dwacc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) dwacc[k] = 0.f;
  int parity = 0;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x, parity ^= 1) {
    const uint4 a0 = *reinterpret_cast<const uint4*>(dy + r * lddy + c0);
    const uint4 a1 = *reinterpret_cast<const uint4*>(dy + r * lddy + c1);
    const uint4 b0 = *reinterpret_cast<const uint4*>(x + r * ldx + c0);
    const uint4 b1 = *reinterpret_cast<const uint4*>(x + r * ldx + c1);
    uint4 o0 = make_uint4(0, 0, 0, 0), o1 = o0;
    if (res) {
      o0 = *reinterpret_cast<const uint4*>(res + r * ldres + c0);
      o1 = *reinterpret_cast<const uint4*>(res + r * ldres + c1);
    }
    const float rr = rstd[r];
    float fa[16], fb[16];
    Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&a0), fa);
    Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&a1), fa + 8);
    Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&b0), fb);
    Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&b1), fb + 8);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) sum += (fa[k] * g[k]) * fb[k];
    sum = warp_sum(sum);
    if (lane == 0) s_part[parity][warp] = sum;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int v = 0; v < W; ++v) tot += s_part[parity][v];
    const float cf = tot * rr * rr * rr / (float)H;
    float fo[16];
    if (res) {
      Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&o0), fo);
      Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&o1), fo + 8);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) fo[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      fo[k] += rr * (fa[k] * g[k]) - fb[k] * cf;
      dwacc[k] += fa[k] * (fb[k] * rr);
    }
    Vec<__nv_bfloat16, 8>::store(dx + r * lddx + c0, fo);
    Vec<__nv_bfloat16, 8>::store(dx + r * lddx + c1, fo + 8);
  }
  if (dw_partial) {
    Vec<float, 8>::store(dw_partial + (int64_t)blockIdx.x * H + c0, dwacc);
    Vec<float, 8>::store(dw_partial + (int64_t)blockIdx.x * H + c1, dwacc + 8);
  }
}

template <int W>
int launch_bwd_rowblock(int64_t nblk, int64_t rows, const void* dy, int64_t lddy, const void* x,
                        int64_t ldx, const void* w, const float* rstd, void* dx, int64_t lddx,
                        const void* res, int64_t ldres, float* dw_partial, cudaStream_t st) {
  rmsnorm_bwd_rowblock_kernel<W><<<(unsigned)nblk, W * 32, 0, st>>>(
      rows, (const __nv_bfloat16*)dy, lddy, (const __nv_bfloat16*)x, ldx,
      (const __nv_bfloat16*)w, rstd, (__nv_bfloat16*)dx, lddx, (const __nv_bfloat16*)res, ldres,
      dw_partial);
  PE_LAUNCHED();
  return PE_OK;
}

// bf16 backward for rows of H = 256 m <= 4096 columns: one warp per row holds the
// row's dy and x in registers (16-byte chunks; lane l owns columns 8 (32 i + l) ..
// + 8 of chunk i), so each is read from HBM once and no second pass touches L2;
// the residual is loaded once the row coefficient is known.  The weight-gradient
// partial of each warp lives in its own shared-memory row (no atomics) and the
// block sums its warps' rows at the end.  Four warps per block, two blocks per SM:
// the row registers cost ~200 per thread.
constexpr int kRowRegWarps = 4;
constexpr int kRowRegChunks = 16;

__global__ void __launch_bounds__(kRowRegWarps * 32, 2)
rmsnorm_bwd_rowreg_kernel(int64_t rows, int H, const __nv_bfloat16* __restrict__ dy,
                          int64_t lddy, const __nv_bfloat16* __restrict__ x, int64_t ldx,
                          const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                          __nv_bfloat16* dx, int64_t lddx, const __nv_bfloat16* res,
                          int64_t ldres, float* __restrict__ dw_partial) {
  extern __shared__ float sdw[];  // [kRowRegWarps][H] when dw_partial
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nch = H / 256;
  float* mydw = sdw + (int64_t)warp * H;
  if (dw_partial)
    for (int c = lane * 4; c < H; c += 128)
      *reinterpret_cast<float4*>(mydw + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();
  const int64_t step = (int64_t)gridDim.x * kRowRegWarps;
  for (int64_t r = (int64_t)blockIdx.x * kRowRegWarps + warp; r < rows; r += step) {
    const __nv_bfloat16* dyr = dy + r * lddy;
    const __nv_bfloat16* xr = x + r * ldx;
    uint4 a[kRowRegChunks], b[kRowRegChunks];
#pragma unroll
    for (int i = 0; i < kRowRegChunks; ++i) {
      if (i < nch) {
        const int c = (i * 32 + lane) * 8;
        a[i] = *reinterpret_cast<const uint4*>(dyr + c);
        b[i] = *reinterpret_cast<const uint4*>(xr + c);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kRowRegChunks; ++i) {
      if (i < nch) {
        float fa[8], fb[8], g[8];
        Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&a[i]), fa);
        Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&b[i]), fb);
        Vec<__nv_bfloat16, 8>::load(w + (i * 32 + lane) * 8, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += (fa[k] * g[k]) * fb[k];
      }
    }
    s = warp_sum(s);
    const float rr = rstd[r];
    const float cf = s * rr * rr * rr / (float)H;
    uint4 o[kRowRegChunks];
    if (res) {
      const __nv_bfloat16* rrow = res + r * ldres;
#pragma unroll
      for (int i = 0; i < kRowRegChunks; ++i)
        if (i < nch) o[i] = *reinterpret_cast<const uint4*>(rrow + (i * 32 + lane) * 8);
    }
    __nv_bfloat16* dxr = dx + r * lddx;
#pragma unroll
    for (int i = 0; i < kRowRegChunks; ++i) {
      if (i < nch) {
        const int c = (i * 32 + lane) * 8;
        float fa[8], fb[8], g[8], fo[8];
        Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&a[i]), fa);
        Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&b[i]), fb);
        Vec<__nv_bfloat16, 8>::load(w + c, g);
        if (res) {
          Vec<__nv_bfloat16, 8>::load(reinterpret_cast<const __nv_bfloat16*>(&o[i]), fo);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) fo[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) fo[k] += rr * (fa[k] * g[k]) - fb[k] * cf;
        Vec<__nv_bfloat16, 8>::store(dxr + c, fo);
        if (dw_partial) {
          float4* d4 = reinterpret_cast<float4*>(mydw + c);
          float4 p = d4[0], q = d4[1];
          p.x += fa[0] * (fb[0] * rr); p.y += fa[1] * (fb[1] * rr);
          p.z += fa[2] * (fb[2] * rr); p.w += fa[3] * (fb[3] * rr);
          q.x += fa[4] * (fb[4] * rr); q.y += fa[5] * (fb[5] * rr);
          q.z += fa[6] * (fb[6] * rr); q.w += fa[7] * (fb[7] * rr);
          d4[0] = p;
          d4[1] = q;
        }
      }
    }
  }
  if (dw_partial) {
    __syncthreads();
    float* out = dw_partial + (int64_t)blockIdx.x * H;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < kRowRegWarps; ++k) t += sdw[k * H + c];
      out[c] = t;
    }
  }
}

// out[c] = (acc ? out[c] : 0) + sum_b partial[b, c]; fixed summation order.
template <typename T>
__global__ void colsum_kernel(int64_t nblk, int64_t H, const float* __restrict__ partial,
                              T* out, int accumulate) {
  __shared__ float red[8][33];
  const int64_t c = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < H)
    for (int64_t b = threadIdx.y; b < nblk; b += 8) s += partial[b * H + c];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && c < H) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][threadIdx.x];
    if (accumulate) t += to_f(out[c]);
    out[c] = from_f<T>(t);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_rmsnorm_fwd(int dtype, int64_t rows, int64_t H, const void* x, int64_t ldx,
                              const void* w, void* y, int64_t ldy, float* rstd, float eps,
                              void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0 && ldx >= H && ldy >= H, "rmsnorm_fwd: bad shape");
  if (rows == 0) return PE_OK;
  const bool vec = H % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && aligned16(x) && aligned16(y) &&
                   aligned16(w);
  dim3 grid((unsigned)ceil_div(rows, kWarps));
  if (vec && dtype == PE_BF16 && H <= (int64_t)kFwdRegChunks * 32 * 8) {
    rmsnorm_fwd_reg_kernel<<<grid, kWarps * 32, 0, as_stream(stream)>>>(
        rows, H, (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy,
        rstd, eps);
    PE_LAUNCHED();
    return PE_OK;
  }
  return PE_DISPATCH(dtype, T, [&] {
    if (vec)
      rmsnorm_fwd_kernel<T, 8><<<grid, kWarps * 32, 0, as_stream(stream)>>>(
          rows, H, (const T*)x, ldx, (const T*)w, (T*)y, ldy, rstd, eps);
    else
      rmsnorm_fwd_kernel<T, 1><<<grid, kWarps * 32, 0, as_stream(stream)>>>(
          rows, H, (const T*)x, ldx, (const T*)w, (T*)y, ldy, rstd, eps);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int64_t pe_rmsnorm_bwd_blocks(int64_t rows) {
  // persistent backward: two blocks per SM (every kernel below keeps that many
  // resident, so no block starts after another finished), one tile of rows at least
  const int64_t cap = 2 * (int64_t)sm_count();
  int64_t b = ceil_div(rows, kTileRows);
  return b < 1 ? 1 : (b > cap ? cap : b);
}

extern "C" int pe_rmsnorm_bwd(int dtype, int64_t rows, int64_t H, const void* dy, int64_t lddy,
                              const void* x, int64_t ldx, const void* w, const float* rstd,
                              void* dx, int64_t lddx, const void* residual, int64_t ldres,
                              float* dw_partial, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0, "rmsnorm_bwd: bad shape");
  PE_CHECK_ARG(!dw_partial || H * 4 <= 200 * 1024, "rmsnorm_bwd: H too large for dw staging");
  const int64_t nblk = pe_rmsnorm_bwd_blocks(rows);
  if (rows == 0) {
    if (dw_partial) PE_CUDA_TRY(cudaMemsetAsync(dw_partial, 0, nblk * H * 4, as_stream(stream)));
    return PE_OK;
  }
  const bool vec = H % 8 == 0 && lddy % 8 == 0 && ldx % 8 == 0 && lddx % 8 == 0 &&
                   (!residual || ldres % 8 == 0) && aligned16(dy) && aligned16(x) &&
                   aligned16(w) && aligned16(dx) && (!residual || aligned16(residual));
  const size_t smem = dw_partial ? (size_t)H * 4 : 0;
  if (vec && dtype == PE_BF16 && H % 512 == 0 && H <= 4096) {
    cudaStream_t st = as_stream(stream);
#define PE_RB(Wn)                                                                            \
  case Wn:                                                                                   \
    return launch_bwd_rowblock<Wn>(nblk, rows, dy, lddy, x, ldx, w, rstd, dx, lddx, residual, \
                                   ldres, dw_partial, st);
    switch (H / 512) {
      PE_RB(1) PE_RB(2) PE_RB(3) PE_RB(4) PE_RB(5) PE_RB(6) PE_RB(7) PE_RB(8)
      default: break;
    }
#undef PE_RB
  }
  if (vec && dtype == PE_BF16 && H % 256 == 0 && H <= 256 * kRowRegChunks) {
    const size_t sm_rr = dw_partial ? (size_t)kRowRegWarps * H * 4 : 0;
    if (sm_rr > 48 * 1024)
      PE_CUDA_TRY(cudaFuncSetAttribute(rmsnorm_bwd_rowreg_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_rr));
    rmsnorm_bwd_rowreg_kernel<<<(unsigned)nblk, kRowRegWarps * 32, sm_rr, as_stream(stream)>>>(
        rows, (int)H, (const __nv_bfloat16*)dy, lddy, (const __nv_bfloat16*)x, ldx,
        (const __nv_bfloat16*)w, rstd, (__nv_bfloat16*)dx, lddx,
        (const __nv_bfloat16*)residual, ldres, dw_partial);
    PE_LAUNCHED();
    return PE_OK;
  }
  if (vec && H <= 8 * 2 * kTiledThreads) {
    return PE_DISPATCH(dtype, T, [&] {
      rmsnorm_bwd_tiled_kernel<T><<<(unsigned)nblk, kTiledThreads, 0, as_stream(stream)>>>(
          rows, H, (const T*)dy, lddy, (const T*)x, ldx, (const T*)w, rstd, (T*)dx, lddx,
          (const T*)residual, ldres, dw_partial);
      PE_LAUNCHED();
      return PE_OK;
    });
  }
  const bool chunked = vec && H % 256 == 0 && H / 256 <= kMaxChunks;
  if (chunked) {
    return PE_DISPATCH(dtype, T, [&] {
      auto kern = rmsnorm_bwd_chunked_kernel<T>;
      if (smem > 48 * 1024)
        PE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      kern<<<(unsigned)nblk, kWarps * 32, smem, as_stream(stream)>>>(
          rows, H, (int)(H / 256), (const T*)dy, lddy, (const T*)x, ldx, (const T*)w, rstd,
          (T*)dx, lddx, (const T*)residual, ldres, dw_partial);
      PE_LAUNCHED();
      return PE_OK;
    });
  }
  return PE_DISPATCH(dtype, T, [&] {
    auto kern = vec ? rmsnorm_bwd_kernel<T, 8> : rmsnorm_bwd_kernel<T, 1>;
    if (smem > 48 * 1024)
      PE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<(unsigned)nblk, kWarps * 32, smem, as_stream(stream)>>>(
        rows, H, (const T*)dy, lddy, (const T*)x, ldx, (const T*)w, rstd, (T*)dx, lddx,
        (const T*)residual, ldres, dw_partial);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_colsum_f32(int dtype, int64_t nblk, int64_t H, const float* partial, void* dw,
                             int accumulate, void* stream) {
  PE_CHECK_ARG(nblk > 0 && H > 0, "colsum: bad shape");
  return PE_DISPATCH(dtype, T, [&] {
    colsum_kernel<T><<<(unsigned)ceil_div(H, 32), dim3(32, 8), 0, as_stream(stream)>>>(
        nblk, H, partial, (T*)dw, accumulate);
    PE_LAUNCHED();
    return PE_OK;
  });
}
