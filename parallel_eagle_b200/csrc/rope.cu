// Half-split rotary embedding applied in place (reference src/pe/nn.py:29-49).
//
// Each thread rotates one (d, d + hd/2) pair of one head of one row.  The
// angle is pos * inv_freq with inv_freq = 1 / theta^(2p/hd), both in fp32 like
// the reference's cache; cos/sin are rounded to the storage type before use,
// and each product/sum is rounded like the reference's element-wise ops.
// Memory bound: one read and one write of the rotated columns.
#include "common.cuh"

namespace pe {
namespace {

template <typename T>
__global__ void rope_kernel(int64_t rows, int heads, int hd, T* x, int64_t ldx,
                            const int64_t* __restrict__ pos, float theta, int inverse) {
  const int half = hd >> 1;
  const int64_t pairs_per_row = (int64_t)heads * half;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * pairs_per_row) return;
  const int64_t row = idx / pairs_per_row;
  const int64_t rem = idx - row * pairs_per_row;
  const int h = (int)(rem / half);
  const int p = (int)(rem - (int64_t)h * half);
  const float expo = (float)(2 * p) / (float)hd;
  const float inv_freq = 1.0f / powf(theta, expo);
  const float ang = (float)pos[row] * inv_freq;
  float s, c;
  sincosf(ang, &s, &c);
  c = round_to<T>(c);
  s = round_to<T>(s);
  T* base = x + row * ldx + (int64_t)h * hd;
  const float a = to_f(base[p]);
  const float b = to_f(base[p + half]);
  float ya, yb;
  if (!inverse) {
    // y1 = x1*c + (-x2)*s ; y2 = x2*c + x1*s
    ya = round_to<T>(round_to<T>(a * c) + round_to<T>(-b * s));
    yb = round_to<T>(round_to<T>(b * c) + round_to<T>(a * s));
  } else {
    // transpose of the rotation: dx1 = dy1*c + dy2*s ; dx2 = dy2*c - dy1*s
    ya = round_to<T>(round_to<T>(a * c) + round_to<T>(b * s));
    yb = round_to<T>(round_to<T>(b * c) - round_to<T>(a * s));
  }
  base[p] = from_f<T>(ya);
  base[p + half] = from_f<T>(yb);
}

// One thread per (row, pair): the angle, cos and sin are computed once and applied
// to the pair in every head of the row (q and k heads share positions).  Threads of
// a warp cover consecutive pairs, so each head's two half-rows are read and
// written as contiguous segments.
template <typename T>
__global__ void rope_rowpair_kernel(int64_t rows, int heads, int hd, T* x, int64_t ldx,
                                    const int64_t* __restrict__ pos, float theta, int inverse) {
  const int half = hd >> 1;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * half) return;
  const int64_t row = idx / half;
  const int p = (int)(idx - row * half);
  const float inv_freq = 1.0f / powf(theta, (float)(2 * p) / (float)hd);
  float s, c;
  sincosf((float)pos[row] * inv_freq, &s, &c);
  c = round_to<T>(c);
  s = round_to<T>(s);
  T* base = x + row * ldx + p;
  for (int h = 0; h < heads; ++h) {
    T* hp = base + (int64_t)h * hd;
    const float a = to_f(hp[0]);
    const float b = to_f(hp[half]);
    float ya, yb;
    if (!inverse) {
      ya = round_to<T>(round_to<T>(a * c) + round_to<T>(-b * s));
      yb = round_to<T>(round_to<T>(b * c) + round_to<T>(a * s));
    } else {
      ya = round_to<T>(round_to<T>(a * c) + round_to<T>(b * s));
      yb = round_to<T>(round_to<T>(b * c) - round_to<T>(a * s));
    }
    hp[0] = from_f<T>(ya);
    hp[half] = from_f<T>(yb);
  }
}

// rotate 8 consecutive pairs (a: first half-row, b: second) in place
__device__ __forceinline__ void rot8(uint4& ua, uint4& ub, const float* cs, const float* sn,
                                     int inverse) {
  using T = __nv_bfloat16;
  __nv_bfloat162* a2 = reinterpret_cast<__nv_bfloat162*>(&ua);
  __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&ub);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __bfloat1622float2(a2[i]), b = __bfloat1622float2(b2[i]);
    const float c0 = cs[2 * i], c1 = cs[2 * i + 1], s0 = sn[2 * i], s1 = sn[2 * i + 1];
    float ya0, ya1, yb0, yb1;
    if (!inverse) {
      ya0 = round_to<T>(round_to<T>(a.x * c0) + round_to<T>(-b.x * s0));
      ya1 = round_to<T>(round_to<T>(a.y * c1) + round_to<T>(-b.y * s1));
      yb0 = round_to<T>(round_to<T>(b.x * c0) + round_to<T>(a.x * s0));
      yb1 = round_to<T>(round_to<T>(b.y * c1) + round_to<T>(a.y * s1));
    } else {
      ya0 = round_to<T>(round_to<T>(a.x * c0) + round_to<T>(b.x * s0));
      ya1 = round_to<T>(round_to<T>(a.y * c1) + round_to<T>(b.y * s1));
      yb0 = round_to<T>(round_to<T>(b.x * c0) - round_to<T>(a.x * s0));
      yb1 = round_to<T>(round_to<T>(b.y * c1) - round_to<T>(a.y * s1));
    }
    a2[i] = __floats2bfloat162_rn(ya0, ya1);
    b2[i] = __floats2bfloat162_rn(yb0, yb1);
  }
}

// bf16, half-width a multiple of 8: one thread per (row, 8 consecutive pairs); the
// block's inverse frequencies once in shared memory, the 8 angles' cos / sin once
// per thread, then every head's two 16-byte half-row segments, four heads' loads
// in flight before their rotations and stores.
__global__ void rope_vec8_kernel(int64_t rows, int heads, int hd, __nv_bfloat16* x, int64_t ldx,
                                 const int64_t* __restrict__ pos, float theta, int inverse) {
  using T = __nv_bfloat16;
  constexpr int kBatch = 4;
  extern __shared__ float s_inv_freq[];  // [hd / 2], the same powf as per element
  const int half = hd >> 1;
  const int groups = half >> 3;
  for (int p = threadIdx.x; p < half; p += blockDim.x)
    s_inv_freq[p] = 1.0f / powf(theta, (float)(2 * p) / (float)hd);
  __syncthreads();
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * groups) return;
  const int64_t row = idx / groups;
  const int p0 = (int)(idx - row * groups) * 8;
  T* base = x + row * ldx + p0;
  // the first batch's loads go out before the angle arithmetic
  uint4 ua[kBatch], ub[kBatch];
  const int nb = heads < kBatch ? heads : kBatch;
#pragma unroll
  for (int q = 0; q < kBatch; ++q) {
    if (q < nb) {
      ua[q] = *reinterpret_cast<const uint4*>(base + (int64_t)q * hd);
      ub[q] = *reinterpret_cast<const uint4*>(base + (int64_t)q * hd + half);
    }
  }
  const float pr = (float)pos[row];
  float cs[8], sn[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float sv, cv;
    sincosf(pr * s_inv_freq[p0 + k], &sv, &cv);
    cs[k] = round_to<T>(cv);
    sn[k] = round_to<T>(sv);
  }
  for (int h = 0; h < heads; h += kBatch) {
    const int n = heads - h < kBatch ? heads - h : kBatch;
    if (h > 0) {
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        if (q < n) {
          const T* hp = base + (int64_t)(h + q) * hd;
          ua[q] = *reinterpret_cast<const uint4*>(hp);
          ub[q] = *reinterpret_cast<const uint4*>(hp + half);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      if (q < n) {
        rot8(ua[q], ub[q], cs, sn, inverse);
        T* hp = base + (int64_t)(h + q) * hd;
        *reinterpret_cast<uint4*>(hp) = ua[q];
        *reinterpret_cast<uint4*>(hp + half) = ub[q];
      }
    }
  }
}

// cos / sin table for the fused rotations: row r holds cos(pos_r * f_p) for the hd/2
// pairs p, then sin(pos_r * f_p), each rounded to the storage type -- the same
// angle and rounding as every rotation kernel above, so a rotation that reads the
// table is bit-identical to rope_vec8_kernel.
template <typename T>
__global__ void rope_table_kernel(int64_t rows, int hd, const int64_t* __restrict__ pos,
                                  float theta, T* __restrict__ cs, int64_t ld) {
  const int half = hd >> 1;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * half) return;
  const int64_t row = idx / half;
  const int p = (int)(idx - row * half);
  const float inv_freq = 1.0f / powf(theta, (float)(2 * p) / (float)hd);
  float sv, cv;
  sincosf((float)pos[row] * inv_freq, &sv, &cv);
  cs[row * ld + p] = from_f<T>(cv);
  cs[row * ld + half + p] = from_f<T>(sv);
}

// Rotation from a pe_rope_table table (same arithmetic as the kernels above), one
// thread per (row, pair) over every head of the row: the generic form of the fused
// rotations, for operands the fused kernels do not take.
template <typename T>
__global__ void rope_apply_table_kernel(int64_t rows, int heads, int hd, T* x, int64_t ldx,
                                        const T* __restrict__ cs, int64_t cs_ld, int inverse) {
  const int half = hd >> 1;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * half) return;
  const int64_t row = idx / half;
  const int p = (int)(idx - row * half);
  const float c = to_f(cs[row * cs_ld + p]);
  const float s = to_f(cs[row * cs_ld + half + p]);
  T* base = x + row * ldx + p;
  for (int h = 0; h < heads; ++h) {
    T* hp = base + (int64_t)h * hd;
    const float a = to_f(hp[0]);
    const float b = to_f(hp[half]);
    float ya, yb;
    if (!inverse) {
      ya = round_to<T>(round_to<T>(a * c) + round_to<T>(-b * s));
      yb = round_to<T>(round_to<T>(b * c) + round_to<T>(a * s));
    } else {
      ya = round_to<T>(round_to<T>(a * c) + round_to<T>(b * s));
      yb = round_to<T>(round_to<T>(b * c) - round_to<T>(a * s));
    }
    hp[0] = from_f<T>(ya);
    hp[half] = from_f<T>(yb);
  }
}

}  // namespace

int rope_apply_table(int dtype, int64_t rows, int heads, int hd, void* x, int64_t ldx,
                     const void* cs, int64_t cs_ld, int inverse, cudaStream_t st) {
  PE_CHECK_ARG(rows >= 0 && heads > 0 && hd > 0 && hd % 2 == 0 && cs_ld >= hd,
               "rope (table): bad shape");
  if (rows == 0) return PE_OK;
  const int64_t total = rows * (hd / 2);
  return PE_DISPATCH(dtype, T, [&] {
    rope_apply_table_kernel<T><<<(unsigned)ceil_div(total, 256), 256, 0, st>>>(
        rows, heads, hd, (T*)x, ldx, (const T*)cs, cs_ld, inverse);
    PE_LAUNCHED();
    return PE_OK;
  });
}

}  // namespace pe

using namespace pe;

extern "C" int pe_rope_table(int dtype, int64_t rows, int head_dim, const int64_t* pos,
                             float theta, void* cs, int64_t ld, void* stream) {
  PE_CHECK_ARG(rows >= 0 && head_dim > 0 && head_dim % 2 == 0, "rope table: bad shape");
  PE_CHECK_ARG(ld >= head_dim, "rope table: ld < head_dim");
  if (rows == 0) return PE_OK;
  const int64_t total = rows * (head_dim / 2);
  return PE_DISPATCH(dtype, T, [&] {
    rope_table_kernel<T><<<(unsigned)ceil_div(total, 256), 256, 0, as_stream(stream)>>>(
        rows, head_dim, pos, theta, (T*)cs, ld);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_rope(int dtype, int64_t rows, int heads, int head_dim, void* x, int64_t ldx,
                       const int64_t* pos, float theta, int inverse, void* stream) {
  PE_CHECK_ARG(rows >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0,
               "rope: bad shape");
  PE_CHECK_ARG(ldx >= (int64_t)heads * head_dim, "rope: ldx too small");
  if (rows == 0) return PE_OK;
  const int threads = 256;
  const bool vec8 = dtype == PE_BF16 && (head_dim / 2) % 8 == 0 && ldx % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
  if (vec8) {
    const int64_t total = rows * (head_dim / 16);
    rope_vec8_kernel<<<(unsigned)ceil_div(total, threads), threads,
                       (size_t)(head_dim / 2) * sizeof(float), as_stream(stream)>>>(
        rows, heads, head_dim, (__nv_bfloat16*)x, ldx, pos, theta, inverse);
    PE_LAUNCHED();
    return PE_OK;
  }
  if (heads >= 4) {
    const int64_t total = rows * (head_dim / 2);
    return PE_DISPATCH(dtype, T, [&] {
      rope_rowpair_kernel<T><<<(unsigned)ceil_div(total, threads), threads, 0, as_stream(stream)>>>(
          rows, heads, head_dim, (T*)x, ldx, pos, theta, inverse);
      PE_LAUNCHED();
      return PE_OK;
    });
  }
  const int64_t total = rows * heads * (head_dim / 2);
  return PE_DISPATCH(dtype, T, [&] {
    rope_kernel<T><<<(unsigned)ceil_div(total, threads), threads, 0, as_stream(stream)>>>(
        rows, heads, head_dim, (T*)x, ldx, pos, theta, inverse);
    PE_LAUNCHED();
    return PE_OK;
  });
}
