// hyena_prefill_noalloc: the prefill entry point for callers that cannot
// allocate device memory.
//
// hyena_prefill needs a caller-provided workspace for the LI (HCL) kind: the
// range table and the carried modal states of the chunked scan.  Some callers
// have no way to provide one: a host program in another language that reaches
// this library only through the C ABI and has no CUDA allocator of its own, or
// a serving loop that may not call cudaMalloc once it runs, because cudaMalloc
// can synchronise the device and its memory budget was fixed at start-up.
// This entry point takes the
// same arguments minus the workspace and uses a fixed scratch array that lives
// in this library's device memory instead.
//
// Limits and contract:
//   * the scratch is NOALLOC_SCRATCH_BYTES (32 MiB) on every GPU that loads the
//     library, held until the process exits.  The LI prefill needs one (H, 16)
//     fp32 modal state per segment plus a few for splitting long segments
//     (256 KiB each at H = 4096); a step needing more (beyond ~120 segments at
//     H = 4096) is rejected with HYENA_ERR_INVALID;
//   * the first call on a device looks the array's device address up (once per
//     device, with that device current); make that first call before any
//     stream capture.  The address is cached per device ordinal for the life of
//     the process and belongs to that device's primary context (the one the
//     CUDA runtime uses): callers that make another context current, or reset
//     the device (cudaDeviceReset), must not use this entry point afterwards;
//   * every call shares the one array and leaves its contents behind: nothing in
//     it needs to start at zero (the range table and every carried state are
//     written before they are read), but two calls whose kernels overlap on the
//     GPU (different streams, or different host threads) race on it.  Serialise
//     them on one stream.
#include <mutex>

#include "common.cuh"

namespace hb {

size_t hcl_workspace_size(int H, int T, int nseg);

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static void* g_noalloc_ptr[NOALLOC_MAX_DEVICES];
static std::mutex g_noalloc_mu;

// The device address of the scratch array on the current device.  Host code
// cannot pass `g_noalloc_scratch` itself: in host code that name is a host-side
// stand-in, not a device address.
static int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(HYENA_ERR_CUDA, std::string("hyena_prefill_noalloc: cudaGetDevice: ") +
                                    cudaGetErrorString(e));
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
    return fail(HYENA_ERR_UNSUPPORTED, "hyena_prefill_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(HYENA_ERR_CUDA, std::string("hyena_prefill_noalloc: cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return HYENA_OK;
}

}  // namespace hb

extern "C" int hyena_prefill_noalloc(const hyena_layer_params* p, const hyena_prefill_args* a,
                                     void* stream) {
  using namespace hb;
  if (p == nullptr || a == nullptr)
    return fail(HYENA_ERR_INVALID, "hyena_prefill_noalloc: null params or args");
  const size_t need = hyena_prefill_workspace_size(p, a->T, a->num_segments);
  if (need > NOALLOC_SCRATCH_BYTES)
    return fail(HYENA_ERR_INVALID,
                "hyena_prefill_noalloc: this prefill needs " + std::to_string(need) +
                    " bytes of scratch but the fixed scratch holds " +
                    std::to_string(NOALLOC_SCRATCH_BYTES) +
                    " (32 MiB); split the step or use hyena_prefill with a workspace");
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
  }
  return hyena_prefill(p, a, scratch, need > 0 ? NOALLOC_SCRATCH_BYTES : 0, stream);
}
