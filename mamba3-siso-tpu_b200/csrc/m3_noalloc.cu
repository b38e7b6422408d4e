// m3_siso_bwd_noalloc: the backward entry point for callers that cannot allocate device
// memory.
//
// m3_siso_bwd needs a workspace (the recomputed chunk-start states), which its caller
// allocates.  Some callers cannot: code running under an allocator it does not own (an
// XLA custom call registered without a workspace buffer, a plugin inside a host
// application that hands it only its inputs and outputs), or a serving process that
// forbids device allocation after start-up so that memory use stays fixed.  This entry
// point takes the same arguments, ignores `workspace` / `workspace_bytes`, and uses a
// fixed scratch array compiled into the library instead.  It calls no cudaMalloc,
// cudaFree or other allocating routine.
//
// Limits and sharing:
//  * the scratch holds kNoAllocScratchBytes (64 MiB); calls whose
//    m3_siso_bwd_workspace_size() is larger are rejected with M3_ERR_WORKSPACE;
//  * every GPU that loads the library keeps this array resident until the process exits;
//  * all calls on a device share the one array: calls that can overlap on the GPU (on
//    different streams, or from different host threads) race on it and must be
//    serialised by the caller;
//  * the kernel writes every scratch element before reading it, so nothing needs to be
//    cleared between calls (the array keeps the last call's contents);
//  * the first call on each device resolves the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call before any
//    stream capture begins.  The address is cached per device together with the id of
//    the CUDA context it was resolved in: if the device's primary context is destroyed
//    and re-created (cudaDeviceReset), the next call resolves it again, so that call
//    too must come before any capture;
//  * `stream` must belong to the current device (a stream of another device gets
//    M3_ERR_ARG: the scratch address is the current device's).
#include <cuda.h>

#include <mutex>

#include "m3_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

// Id of the current CUDA context (unique for the life of the process), through the driver
// entry points the runtime hands out; 0 if they are unavailable.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {  // under g_mu
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault) == cudaSuccess) get_current = (GetCurrent)f;
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault) == cudaSuccess) get_id = (GetId)f;
    looked_up = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of g_scratch on the current device, resolved once per device and CUDA
// context.  In host code `g_scratch` names a host-side shadow, not device memory, so it is
// never passed to a kernel directly.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return m3::set_error(M3_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return m3::set_error(M3_ERR_ARG, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_scratch_ptr[dev] || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p)
      return m3::set_error(M3_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = current_context_id();  // the lookup may have created the context
  }
  *out = g_scratch_ptr[dev];
  return M3_OK;
}

}  // namespace

extern "C" size_t m3_siso_bwd_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int m3_siso_bwd_noalloc(const M3BwdArgs* args, void* stream) {
  if (!args) return m3::set_error(M3_ERR_ARG, "args is NULL");
  const M3Dims& d = args->dims;
  if (d.batch <= 0 || d.seqlen <= 0 || d.nheads <= 0 || d.state_dim <= 0 || d.headdim <= 0 || d.n_angles <= 0 ||
      d.chunk <= 0)
    return m3::set_error(M3_ERR_SHAPE, "all dims must be positive");
  if (stream) {
    int cur = 0, sdev = 0;
    if (cudaGetDevice(&cur) != cudaSuccess || cudaStreamGetDevice((cudaStream_t)stream, &sdev) != cudaSuccess)
      return m3::set_error(M3_ERR_ARG, "m3_siso_bwd_noalloc: cannot query the stream's device");
    if (sdev != cur)
      return m3::set_error(M3_ERR_ARG, "m3_siso_bwd_noalloc: the stream belongs to device " + std::to_string(sdev) +
                                           ", not the current device " + std::to_string(cur));
  }
  const size_t need = m3_siso_bwd_workspace_size(&args->dims);
  if (need > kNoAllocScratchBytes)
    return m3::set_error(M3_ERR_WORKSPACE,
                         "m3_siso_bwd_noalloc: this problem needs " + std::to_string(need) +
                             " bytes of scratch, more than the built-in " + std::to_string(kNoAllocScratchBytes) +
                             " bytes; call m3_siso_bwd with a caller-allocated workspace instead");
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != M3_OK) return rc;
  M3BwdArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  a.states_ready = 0;  // the library's own scratch never holds a forward's saved states
  return m3_siso_bwd(&a, stream);
}
