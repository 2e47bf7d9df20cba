// Library-wide state: thread-local error message, launch counter, device queries.
#include "common.cuh"

#include <mutex>

namespace pe {

static thread_local std::string g_last_error;
static int64_t g_launches = 0;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int64_t& launch_counter() { return g_launches; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {
constexpr int kMaxDev = 64, kSlots = 4, kEvents = 32;
std::mutex g_stream_mu;
cudaStream_t g_streams[kMaxDev][kSlots];
cudaEvent_t g_events[kMaxDev][kEvents];
}  // namespace

cudaStream_t side_stream(int slot) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev || slot < 0 ||
      slot >= kSlots)
    return nullptr;
  std::lock_guard<std::mutex> lk(g_stream_mu);
  if (!g_streams[dev][slot]) {
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    g_streams[dev][slot] = s;
  }
  return g_streams[dev][slot];
}

cudaEvent_t pool_event(int i) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev || i < 0 || i >= kEvents)
    return nullptr;
  std::lock_guard<std::mutex> lk(g_stream_mu);
  if (!g_events[dev][i]) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    g_events[dev][i] = e;
  }
  return g_events[dev][i];
}

}  // namespace pe

extern "C" const char* pe_last_error(void) { return pe::g_last_error.c_str(); }
extern "C" int pe_version(void) { return 1; }
extern "C" int64_t pe_launch_count(void) { return pe::launch_counter(); }
