// Self-test of the bounded-wait unwind path that every tensor-core kernel of this
// library relies on.  One warp allocates TMEM as the kernels do, then one thread
// waits with sm100::mbar_wait on an mbarrier that nothing ever arrives at.  The
// wait gives up after `limit_ns`, records its code in the caller's status word,
// and the warp frees its TMEM and returns -- the same steps a real kernel takes
// when a TMA copy or an MMA it waits on never completes.  No copy or MMA is in
// flight, so the wait running out leaves nothing behind on the device.
#include "common.cuh"
#include "sm100.cuh"

namespace pe {
namespace {

constexpr int kProbeCode = 901;

__global__ void __launch_bounds__(32, 1)
    wait_probe_kernel(uint64_t limit_ns, int* status, int* waited_out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_slot;
  sm100::tmem_alloc(&tmem_slot, 32);
  sm100::tmem_relinquish();
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_barrier_init();
  }
  sm100::tc_fence_before();
  __syncwarp();
  sm100::tc_fence_after();
  bool ok = true;
  if (threadIdx.x == 0) ok = sm100::mbar_wait(&bar, 0, status, kProbeCode, limit_ns);
  __syncwarp();
  sm100::tc_fence_before();
  sm100::tmem_dealloc(tmem_slot, 32);
  if (threadIdx.x == 0) waited_out[0] = ok ? 0 : 1;
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" int pe_wait_probe(uint64_t limit_ns, int32_t* status, int32_t* waited_out,
                             void* stream) {
  PE_CHECK_ARG(limit_ns >= 1000ull && limit_ns <= 10000000000ull,
               "wait probe: limit_ns must be within [1 us, 10 s], got %llu",
               (unsigned long long)limit_ns);
  PE_CHECK_ARG(status != nullptr && waited_out != nullptr,
               "wait probe: status and waited_out must be device int32 words");
  wait_probe_kernel<<<1, 32, 0, as_stream(stream)>>>(limit_ns, status, waited_out);
  PE_LAUNCHED();
  return PE_OK;
}
