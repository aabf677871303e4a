// knx_api.cu — library-level entry points (version, device check, status strings).
#include "knx_common.cuh"

extern "C" int knx_version(void) { return 10000; }

extern "C" int knx_device_ok(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

extern "C" const char* knx_status_string(int status) {
  switch (status) {
    case KNX_OK: return "ok";
    case KNX_E_INVALID: return "invalid argument (size, dtype or flag)";
    case KNX_E_ALIGN: return "pointer or stride alignment violated";
    case KNX_E_WORKSPACE: return "workspace missing or too small";
    case KNX_E_LAUNCH: return "kernel launch failed";
    case KNX_E_UNSUPPORTED: return "shape outside the supported range";
    case KNX_E_DEVICE: return "device is not sm_100 or a CUDA call failed";
    default: return "unknown status";
  }
}

// ---- per-device launch set-up -----------------------------------------------------------------
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace knx {
namespace {
std::mutex g_setup_mu;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  cache[dev] = n > 0 ? n : 148;
  return cache[dev];
}

int set_max_dyn_smem(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KNX_E_DEVICE;
  static std::map<std::tuple<const void*, int>, int> done;  // (kernel, device) -> bytes set
  std::lock_guard<std::mutex> lk(g_setup_mu);
  const auto key = std::make_tuple(func, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return KNX_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return KNX_E_DEVICE;
  done[key] = bytes;
  return KNX_OK;
}
}  // namespace knx

// ---- stage profiling ------------------------------------------------------------------------

namespace knx {
namespace prof {
static bool g_on = false;
static int g_max = 0, g_calls = 0;
static std::vector<cudaEvent_t> g_ev;  // [g_max][KNX_PROF_STAGES + 1]

void mark(int call, int slot, cudaStream_t s) {
  if (!g_on || call < 0 || call >= g_max) return;
  cudaEventRecord(g_ev[static_cast<size_t>(call) * (KNX_PROF_STAGES + 1) + slot], s);
}
int begin_call() {
  if (!g_on || g_calls >= g_max) return -1;
  return g_calls++;
}
}  // namespace prof
}  // namespace knx

extern "C" int knx_prof_start(int max_calls) {
  using namespace knx::prof;
  if (max_calls <= 0 || max_calls > 100000) return KNX_E_INVALID;
  for (auto e : g_ev) cudaEventDestroy(e);
  g_ev.assign(static_cast<size_t>(max_calls) * (KNX_PROF_STAGES + 1), nullptr);
  for (auto& e : g_ev)
    if (cudaEventCreate(&e) != cudaSuccess) return KNX_E_DEVICE;
  g_max = max_calls;
  g_calls = 0;
  g_on = true;
  return KNX_OK;
}

extern "C" int knx_prof_stop(float* stage_ms, int n_stages, int* ncalls) {
  using namespace knx::prof;
  g_on = false;
  if (ncalls) *ncalls = g_calls;
  for (int s = 0; s < n_stages; ++s) stage_ms[s] = 0.f;
  for (int c = 0; c < g_calls; ++c) {
    for (int s = 0; s < KNX_PROF_STAGES && s < n_stages; ++s) {
      cudaEvent_t a = g_ev[static_cast<size_t>(c) * (KNX_PROF_STAGES + 1) + s];
      cudaEvent_t b = g_ev[static_cast<size_t>(c) * (KNX_PROF_STAGES + 1) + s + 1];
      if (cudaEventSynchronize(b) != cudaSuccess) return KNX_E_DEVICE;
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, a, b) != cudaSuccess) return KNX_E_DEVICE;
      stage_ms[s] += ms;
    }
  }
  g_calls = 0;
  return KNX_OK;
}
