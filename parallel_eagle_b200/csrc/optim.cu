// Gradient clipping by global norm and AdamW over a flat parameter buffer
// (reference src/pe/train.py:158-159: clip_grad_norm_(params, 1.0) then
// torch.optim.AdamW.step(); decoupled weight decay, bias-corrected moments).
// Both are single memory-bound passes; moments are kept in fp32.
#include "common.cuh"

namespace pe {
namespace {

template <typename T>
__global__ void sumsq_kernel(int64_t n, const T* __restrict__ g, float* out) {
  __shared__ float sh[32];
  float s = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = to_f(g[i]);
    s += x * x;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

template <typename T>
__global__ void adamw_kernel(int64_t n, T* __restrict__ p, const T* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v,
                             const float* __restrict__ sumsq, float max_norm, float lr, float b1,
                             float b2, float eps, float wd, float bc1, float bc2_sqrt) {
  float coef = 1.f;
  if (sumsq && max_norm > 0.f) {
    const float norm = sqrtf(sumsq[0]);
    coef = fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float step_size = lr / bc1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = to_f(g[i]) * coef;
    float pi = to_f(p[i]);
    pi *= 1.f - lr * wd;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    pi -= step_size * mi / denom;
    p[i] = from_f<T>(pi);
  }
}

// Deterministic sum of squares: block b of a fixed grid reduces elements b * 256 + t,
// strided by the grid, in a fixed order and writes partials[b] (no atomics), then one
// block adds the partials in a fixed order.  Every rank of a data-parallel job holding
// the same gradient therefore computes the same bits -- the clip coefficient, and so
// the update, cannot drift apart between replicas.
template <typename T>
__global__ void sumsq_partials_kernel(int64_t n, const T* __restrict__ g, float* __restrict__ part) {
  __shared__ float sh[32];
  float s = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = to_f(g[i]);
    s += x * x;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) part[blockIdx.x] = t;
  }
}

__global__ void sum_f32_kernel(int64_t n, const float* __restrict__ x, float* out, int accumulate) {
  __shared__ float sh[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) out[0] = accumulate ? out[0] + t : t;
  }
}

unsigned grid_for(int64_t n) {
  int64_t g = ceil_div(n, 256);
  const int64_t cap = (int64_t)sm_count() * 8;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_sumsq(int dtype, int64_t n, const void* g, float* sumsq_out, void* stream) {
  PE_CHECK_ARG(n >= 0, "sumsq: bad size");
  if (n == 0) return PE_OK;
  return PE_DISPATCH(dtype, T, [&] {
    sumsq_kernel<T><<<grid_for(n), 256, 0, as_stream(stream)>>>(n, (const T*)g, sumsq_out);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_sumsq_partials(int dtype, int64_t n, const void* g, float* partials,
                                 int64_t nblk, void* stream) {
  PE_CHECK_ARG(n >= 0 && nblk >= 1 && nblk <= 65535, "sumsq_partials: bad size / block count");
  return PE_DISPATCH(dtype, T, [&] {
    sumsq_partials_kernel<T><<<(unsigned)nblk, 256, 0, as_stream(stream)>>>(n, (const T*)g,
                                                                             partials);
    PE_LAUNCHED();
    return PE_OK;
  });
}

extern "C" int pe_sum_f32(int64_t n, const float* x, float* out, int accumulate, void* stream) {
  PE_CHECK_ARG(n >= 0, "sum_f32: bad size");
  sum_f32_kernel<<<1, 1024, 0, as_stream(stream)>>>(n, x, out, accumulate);
  PE_LAUNCHED();
  return PE_OK;
}

extern "C" int pe_adamw_step(int dtype, int64_t n, void* p, const void* g, float* m, float* v,
                             const float* sumsq, float max_norm, float lr, float beta1,
                             float beta2, float eps, float weight_decay, int64_t step,
                             void* stream) {
  PE_CHECK_ARG(n >= 0 && step >= 1, "adamw: bad size/step");
  if (n == 0) return PE_OK;
  const float bc1 = 1.f - powf(beta1, (float)step);
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  return PE_DISPATCH(dtype, T, [&] {
    adamw_kernel<T><<<grid_for(n), 256, 0, as_stream(stream)>>>(
        n, (T*)p, (const T*)g, m, v, sumsq, max_norm, lr, beta1, beta2, eps, weight_decay, bc1,
        bc2_sqrt);
    PE_LAUNCHED();
    return PE_OK;
  });
}
