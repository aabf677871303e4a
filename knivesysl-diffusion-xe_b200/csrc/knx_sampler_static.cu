// knx_sampler_static.cu — the fused sampler pass with its scratch in a fixed device array, for
// callers that must not allocate device memory when they sample.
//
// Who cannot allocate, and why: a host runtime reached over the C ABI (Go, Java, JavaScript) owns
// no CUDA allocator and would otherwise have to create, size and keep alive a workspace buffer
// across calls; serving loops that freeze their device memory after warm-up cannot allocate inside
// the step, and cudaMalloc/cudaFree there could also synchronise the device.  This entry point
// takes no workspace: the sampler's scratch (per-chunk partial row states, per-row tickets and
// Gumbel bounds, the work counter) lives in `g_sampler_scratch`, a file-scope array of this
// library's device image, and nothing here allocates.
//
// Rules (also in include/knx.h):
//   * size limit KNX_SAMPLER_STATIC_SCRATCH_BYTES (1 MiB).  The scratch a call needs is
//     knx_sampler_workspace_size(rows, V) (32 B per row chunk — 8 chunks per row at V = 262144 —
//     plus 8 B per row and 512 B); 256 x 262144 needs about 67 KB and the limit admits 3,969
//     rows at that V.  A larger call is rejected with KNX_E_WORKSPACE before anything is launched.
//   * set-up: the first call on each device looks the array's device address up with
//     cudaGetSymbolAddress while that device is current, checks the result and caches it; make that
//     first call before any stream capture begins.
//   * what starts at zero: the row tickets, the per-row bounds and the work counter, cleared by an
//     async memset in stream order at every call (inside knx_sampler_fused); the partial states
//     are always written before they are read.
//   * one array per device: two calls that can run at the same time on one device (different
//     streams, or host threads without ordering between them) race on the scratch and corrupt each
//     other's results.  Calls issued one after another on one stream are safe.
#include <mutex>

#include "knx_common.cuh"

namespace {

static __device__ __align__(256) uint8_t g_sampler_scratch[KNX_SAMPLER_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of this device's scratch array (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return KNX_E_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sampler_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return KNX_E_DEVICE;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return KNX_OK;
}

}  // namespace

extern "C" int knx_sampler_fused_static(const float* logits, int64_t rows, int64_t V,
                                        float temperature, int64_t seed, float* entropy,
                                        int64_t* samp, int64_t* amax, void* stream) {
  if (rows < 0 || V <= 0 || V > 0x7fffffffLL || rows > (1LL << 31)) return KNX_E_INVALID;
  if (knx_sampler_workspace_size(rows, V) > KNX_SAMPLER_STATIC_SCRATCH_BYTES)
    return KNX_E_WORKSPACE;
  if (rows == 0) return KNX_OK;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != KNX_OK) return rc;
  return knx_sampler_fused(logits, rows, V, temperature, seed, entropy, samp, amax, scratch,
                           KNX_SAMPLER_STATIC_SCRATCH_BYTES, stream);
}
