// Per-row log-softmax + top-k of draft logits: the selection step of the
// drafter's tree / chain proposals (reference src/pe/decode/tree.py:33-41 and
// src/pe/decode/chain.py:22-23, i.e. log_softmax(logits.float()) then topk /
// argmax per prediction depth).
//
// One CTA per row.  Pass 1 reduces the row maximum m and s = sum exp(z - m) in
// fp32; the log-probability of column v is lp_v = (z_v - m) - log(s), the same
// two roundings torch's log_softmax applies (with raw = 1 the ranking value is the
// logit itself, as for argmax, and pass 1 is skipped).  Pass 2 picks the k best columns
// in k rounds: round r takes the first column after the previous winner in the
// order (lp descending, column ascending) -- a scan of the row from L2 per
// round, with no per-thread candidate lists, so k is limited only by the
// caller's buffers.  The row (at most a vocabulary of ~150K bf16) stays in L2
// across the rounds.
#include <cfloat>

#include "common.cuh"

namespace pe {
namespace {

constexpr int kThreads = 512;

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// (value, column) ordered by value descending, then column ascending; NaN ranks
// above every number, as in torch.topk / torch.argmax (an all-NaN row therefore
// yields its first columns, never an out-of-range index)
struct Cand {
  float v;
  int64_t i;
};
__device__ __forceinline__ bool before(const Cand& a, const Cand& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (!an && a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}

__device__ Cand block_best(Cand c, Cand* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Cand x;
    x.v = __shfl_xor_sync(0xffffffffu, c.v, o);
    x.i = __shfl_xor_sync(0xffffffffu, c.i, o);
    if (before(x, c)) c = x;
  }
  if (lane == 0) red[warp] = c;
  __syncthreads();
  if (warp == 0) {
    c = lane < kThreads / 32 ? red[lane] : Cand{-INFINITY, INT64_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Cand x;
      x.v = __shfl_xor_sync(0xffffffffu, c.v, o);
      x.i = __shfl_xor_sync(0xffffffffu, c.i, o);
      if (before(x, c)) c = x;
    }
    if (lane == 0) red[0] = c;
  }
  __syncthreads();
  const Cand out = red[0];
  __syncthreads();  // red is reused by the next round
  return out;
}

__device__ float block_reduce(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float x = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, x) : v + x;
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? red[lane] : (is_max ? -INFINITY : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float x = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, x) : v + x;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float out = red[0];
  __syncthreads();
  return out;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
topk_logprobs_kernel(int64_t V, const T* __restrict__ logits, int64_t ld, int k, int raw,
                     int64_t* __restrict__ idx, float* __restrict__ val) {
  __shared__ Cand cred[kThreads / 32];
  __shared__ float fred[kThreads / 32];
  const T* z = logits + (int64_t)blockIdx.x * ld;
  float m = 0.f, logs = 0.f;
  if (!raw) {
    m = -INFINITY;
    for (int64_t v = threadIdx.x; v < V; v += kThreads) m = fmaxf(m, load_f(z + v));
    m = block_reduce(m, fred, true);
    float s = 0.f;
    for (int64_t v = threadIdx.x; v < V; v += kThreads) s += expf(load_f(z + v) - m);
    s = block_reduce(s, fred, false);
    logs = logf(s);
  }
  Cand prev{__int_as_float(0x7fffffff), -1};  // a NaN at column -1: everything comes after it
  for (int r = 0; r < k; ++r) {
    Cand best{-INFINITY, INT64_MAX};
    for (int64_t v = threadIdx.x; v < V; v += kThreads) {
      const float x = load_f(z + v);
      const Cand c{raw ? x : (x - m) - logs, v};
      if (before(prev, c) && before(c, best)) best = c;
    }
    best = block_best(best, cred);
    if (threadIdx.x == 0) {
      idx[(int64_t)blockIdx.x * k + r] = best.i;
      val[(int64_t)blockIdx.x * k + r] = best.v;
    }
    prev = best;
  }
}

__device__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const double out = red[0];
  __syncthreads();
  return out;
}

// q = softmax(z / T) per row in fp32 (reference src/pe/decode/chain.py:50:
// torch.softmax(logits.float() / temperature)): the division first, then the row
// maximum, s = sum exp(x - m) and q_v = exp(x_v - m) / s, in torch's order.  The
// ~150K-term row sum is accumulated in fp64 and rounded once, so s is the correctly
// rounded sum of the fp32 exponentials whatever the reduction order.
template <typename T>
__global__ void __launch_bounds__(kThreads)
softmax_rows_kernel(int64_t V, const T* __restrict__ logits, int64_t ld, float temperature,
                    float* __restrict__ q, int64_t ldq) {
  __shared__ float fred[kThreads / 32];
  __shared__ double dred[kThreads / 32];
  const T* z = logits + (int64_t)blockIdx.x * ld;
  float* out = q + (int64_t)blockIdx.x * ldq;
  float m = -INFINITY;
  for (int64_t v = threadIdx.x; v < V; v += kThreads) m = fmaxf(m, load_f(z + v) / temperature);
  m = block_reduce(m, fred, true);
  double sd = 0.0;
  for (int64_t v = threadIdx.x; v < V; v += kThreads)
    sd += (double)expf(load_f(z + v) / temperature - m);
  const float s = (float)block_sum_d(sd, dred);
  for (int64_t v = threadIdx.x; v < V; v += kThreads)
    out[v] = expf(load_f(z + v) / temperature - m) / s;
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_softmax_rows(int dtype, int64_t rows, int64_t V, const void* logits,
                               int64_t ld, float temperature, float* q, int64_t ldq,
                               void* stream) {
  PE_CHECK_ARG(rows >= 0 && V >= 1 && ld >= V && ldq >= V,
               "softmax_rows: need V >= 1, ld >= V and ldq >= V");
  PE_CHECK_ARG(temperature > 0.f && temperature <= FLT_MAX,
               "softmax_rows: temperature must be positive and finite");
  PE_CHECK_ARG(rows <= 0x7fffffff, "softmax_rows: too many rows");
  if (rows == 0) return PE_OK;
  PE_CHECK_ARG(logits && q, "softmax_rows: null pointer");
  cudaStream_t st = as_stream(stream);
  return PE_DISPATCH(dtype, T, [&] {
    softmax_rows_kernel<T><<<(unsigned)rows, kThreads, 0, st>>>(V, (const T*)logits, ld,
                                                                temperature, q, ldq);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_topk_logprobs(int dtype, int64_t rows, int64_t V, const void* logits,
                                int64_t ld, int k, int raw, int64_t* idx, float* val,
                                void* stream) {
  PE_CHECK_ARG(rows >= 0 && V >= 1 && ld >= V && k >= 1 && k <= V,
               "topk_logprobs: need V >= 1, ld >= V and 1 <= k <= V");
  PE_CHECK_ARG(rows <= 0x7fffffff, "topk_logprobs: too many rows");
  if (rows == 0) return PE_OK;
  PE_CHECK_ARG(logits && idx && val, "topk_logprobs: null pointer");
  cudaStream_t st = as_stream(stream);
  return PE_DISPATCH(dtype, T, [&] {
    topk_logprobs_kernel<T><<<(unsigned)rows, kThreads, 0, st>>>(V, (const T*)logits, ld, k, raw,
                                                                 idx, val);
    PE_LAUNCHED();
    return PE_OK;
  });
}
