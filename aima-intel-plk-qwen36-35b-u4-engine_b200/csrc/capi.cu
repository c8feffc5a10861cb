// capi.cu — library-level entry points: version, status strings, PDL switch.

#include <atomic>

#include "common.cuh"
#include "launch.cuh"
#include "u4_stream.cuh"

namespace iq36 {
static std::atomic<int> g_pdl{1};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
}  // namespace iq36

extern "C" const char* iq36_version(void) { return "iq36-b200 0.1.0 sm_100a"; }

extern "C" const char* iq36_status_string(int status) {
  switch (status) {
    case IQ36_OK: return "ok";
    case IQ36_ERR_ARG: return "invalid argument (null pointer or bad enum)";
    case IQ36_ERR_SHAPE: return "unsupported or inconsistent shape";
    case IQ36_ERR_ALIGN: return "pointer alignment requirement violated";
    case IQ36_ERR_WORKSPACE: return "workspace missing or too small";
    case IQ36_ERR_CUDA: return "CUDA runtime error at launch";
    case IQ36_ERR_TIMEOUT: return "bounded device wait expired";
    case IQ36_ERR_DEVICE: return "device-side check failed";
    default: return "unknown status";
  }
}

extern "C" void iq36_set_pdl(int enabled) { iq36::g_pdl.store(enabled ? 1 : 0); }

namespace iq36 {
int attn_wait_timeouts(int* count, int reset);
int gemm_wait_timeouts(int* count, int reset);
int moe_wait_timeouts(int* count, int reset);
int tp_wait_timeouts(int* count, int reset);
int delta_wait_timeouts(int* count, int reset);
}

extern "C" int iq36_wait_timeouts(int32_t* count, int32_t reset) {
  if (count == nullptr) return IQ36_ERR_ARG;
  int c = 0, a = 0, g = 0, m = 0, t = 0, d = 0;
  int st = iq36::stream_wait_timeouts(&c, reset);
  if (st == IQ36_OK) st = iq36::attn_wait_timeouts(&a, reset);
  if (st == IQ36_OK) st = iq36::gemm_wait_timeouts(&g, reset);
  if (st == IQ36_OK) st = iq36::moe_wait_timeouts(&m, reset);
  if (st == IQ36_OK) st = iq36::tp_wait_timeouts(&t, reset);
  if (st == IQ36_OK) st = iq36::delta_wait_timeouts(&d, reset);
  *count = c + a + g + m + t + d;
  return st;
}
