// RMSNorm backward with the weight gradient, for callers that cannot allocate.
//
// pe_rmsnorm_bwd needs a caller-provided fp32 buffer for its per-block dW
// partial sums.  Some callers have no way to provide one: a host that owns the
// device's whole memory budget and forbids its plugins to allocate, or a caller
// that must not put cudaMalloc / cudaFree (which synchronise the device) on its
// hot path.  This entry point keeps those partials in a fixed array that lives in
// the library's own device memory instead, so the caller passes only inputs and
// outputs.
//
// The array (kNoAllocBlocks x kNoAllocMaxH floats = 2 MiB) is a file-scope
// __device__ variable: every GPU that loads the library holds it until the
// process exits.  Its device address is looked up once per device, on the first
// call made with that device current; make that first call before any stream
// capture.  All calls share the one array and it keeps the last call's partials,
// so calls that overlap on the GPU (concurrent streams, or several host threads
// on one device) race; serialise them.  Every call rewrites all the partial rows
// it later reads, so no clearing is needed between calls.
#include <atomic>

#include "common.cuh"

namespace pe {
namespace {

constexpr int kNoAllocBlocks = 64;     // partial rows (one per CTA)
constexpr int64_t kNoAllocMaxH = 8192;  // widest row the array holds
constexpr int kWarps = 8;

static __device__ __align__(256) float g_dw_scratch[kNoAllocBlocks * kNoAllocMaxH];

// Per device: the device address of g_dw_scratch (nullptr until looked up).
// Per-device cache of the array's device address.  Concurrent first calls may both
// look it up; each stores the same address, and the atomic keeps the store whole.
static std::atomic<float*> g_scratch_ptr[64];
// one partial row per CTA is staged in shared memory: within the default 48 KiB
static_assert(kNoAllocMaxH * sizeof(float) <= 48 * 1024, "partial row exceeds static smem");

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
rmsnorm_bwd_scratch_kernel(int64_t rows, int64_t H, const T* __restrict__ dy, int64_t lddy,
                           const T* __restrict__ x, int64_t ldx, const T* __restrict__ w,
                           const float* __restrict__ rstd, T* dx, int64_t lddx, const T* res,
                           int64_t ldres, float* __restrict__ partial) {
  extern __shared__ float sdw[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t c = threadIdx.x; c < H; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  for (int64_t row = (int64_t)blockIdx.x * kWarps + warp; row < rows;
       row += (int64_t)gridDim.x * kWarps) {
    const T* dyr = dy + row * lddy;
    const T* xr = x + row * ldx;
    const float r = rstd[row];
    float s = 0.f;
    for (int64_t c = lane; c < H; c += 32) s += (to_f(dyr[c]) * to_f(w[c])) * to_f(xr[c]);
    s = warp_sum(s);
    const float coef = s * r * r * r / (float)H;
    T* dxr = dx + row * lddx;
    const T* rr = res ? res + row * ldres : nullptr;
    for (int64_t c = lane; c < H; c += 32) {
      const float a = to_f(dyr[c]), b = to_f(xr[c]);
      float o = rr ? to_f(rr[c]) : 0.f;
      o += r * (a * to_f(w[c])) - b * coef;
      dxr[c] = from_f<T>(o);
      atomicAdd(&sdw[c], a * (b * r));
    }
  }
  __syncthreads();
  // every CTA rewrites its whole partial row, so no stale values survive a call
  float* out = partial + (int64_t)blockIdx.x * H;
  for (int64_t c = threadIdx.x; c < H; c += blockDim.x) out[c] = sdw[c];
}

template <typename T>
__global__ void dw_from_scratch_kernel(int nblk, int64_t H, const float* __restrict__ partial,
                                       T* dw, int accumulate) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float t = 0.f;
  for (int b = 0; b < nblk; ++b) t += partial[(int64_t)b * H + c];
  if (accumulate) t += to_f(dw[c]);
  dw[c] = from_f<T>(t);
}

int scratch_for_current_device(float** out) {
  int dev = 0;
  PE_CUDA_TRY(cudaGetDevice(&dev));
  PE_CHECK_ARG(dev >= 0 && dev < 64, "rmsnorm_bwd_noalloc: device index %d out of range", dev);
  float* cached = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (cached == nullptr) {
    void* p = nullptr;
    PE_CUDA_TRY(cudaGetSymbolAddress(&p, g_dw_scratch));
    cached = static_cast<float*>(p);
    g_scratch_ptr[dev].store(cached, std::memory_order_release);
  }
  *out = cached;
  return PE_OK;
}

}  // namespace
}  // namespace pe

using namespace pe;

// No counterpart in the reference: the same computation as pe_rmsnorm_bwd followed
// by pe_colsum_f32, without any caller-provided workspace.
extern "C" int pe_rmsnorm_bwd_noalloc(int dtype, int64_t rows, int64_t H, const void* dy,
                                      int64_t lddy, const void* x, int64_t ldx, const void* w,
                                      const float* rstd, void* dx, int64_t lddx,
                                      const void* residual, int64_t ldres, void* dw,
                                      int accumulate, void* stream) {
  PE_CHECK_ARG(rows >= 0 && H > 0, "rmsnorm_bwd_noalloc: bad shape");
  PE_CHECK_ARG(H <= kNoAllocMaxH,
               "rmsnorm_bwd_noalloc: H = %lld exceeds the built-in scratch limit of %lld "
               "columns; use pe_rmsnorm_bwd with a caller-provided workspace",
               (long long)H, (long long)kNoAllocMaxH);
  PE_CHECK_ARG(lddy >= H && ldx >= H && lddx >= H && (!residual || ldres >= H),
               "rmsnorm_bwd_noalloc: row stride smaller than H");
  PE_CHECK_ARG(dw != nullptr, "rmsnorm_bwd_noalloc: dw is required");
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  int64_t nb = ceil_div(rows, 4 * kWarps);
  const int nblk = (int)(nb < 1 ? 1 : (nb > kNoAllocBlocks ? kNoAllocBlocks : nb));
  const size_t smem = (size_t)H * 4;
  cudaStream_t st = as_stream(stream);
  return PE_DISPATCH(dtype, T, [&] {
    auto kern = rmsnorm_bwd_scratch_kernel<T>;
    kern<<<nblk, kWarps * 32, smem, st>>>(rows, H, (const T*)dy, lddy, (const T*)x, ldx,
                                          (const T*)w, rstd, (T*)dx, lddx, (const T*)residual,
                                          ldres, scratch);
    PE_LAUNCHED();
    dw_from_scratch_kernel<T><<<(unsigned)ceil_div(H, 256), 256, 0, st>>>(nblk, H, scratch,
                                                                         (T*)dw, accumulate);
    PE_LAUNCHED();
    return PE_OK;
  });
}
