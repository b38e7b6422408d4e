// Launcher of the generic forward kernel.
#include "m3_fwd_simt.cuh"
#include "m3_internal.h"

namespace m3 {

template <int N, int P, typename T, bool MMB>
static int run_fwd(const M3FwdArgs& a, cudaStream_t s) {
  auto* kern = fwd_simt_kernel<N, P, T, MMB>;
  const size_t smem = FwdSmem<N, P>::bytes;
  static bool attr_done[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("fwd: cudaFuncSetAttribute");
    attr_done[dev] = true;
  }
  kern<<<a.dims.batch * a.dims.nheads, kSimtThreads, smem, s>>>(a);
  return check_launch("m3_siso_fwd");
}

int launch_fwd_simt(const M3FwdArgs& a, cudaStream_t s) {
  const bool mmb = a.policy == M3_POLICY_BF16;
  const bool bf = a.io_dtype == M3_DTYPE_BF16;
#define X(N_, P_)                                                                  \
  if (bf) return mmb ? run_fwd<N_, P_, __nv_bfloat16, true>(a, s) : run_fwd<N_, P_, __nv_bfloat16, false>(a, s); \
  return mmb ? run_fwd<N_, P_, float, true>(a, s) : run_fwd<N_, P_, float, false>(a, s);
  M3_DISPATCH_NP(a.dims.state_dim, a.dims.headdim, X);
#undef X
}

}  // namespace m3
