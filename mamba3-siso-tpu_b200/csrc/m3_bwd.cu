// Launcher of the generic backward kernel.
#include "m3_bwd_simt.cuh"
#include "m3_internal.h"

namespace m3 {

size_t bwd_workspace_bytes(const M3Dims& d) {
  const size_t simt = sizeof(float) * (bwd_ws_state_floats(d) + bwd_ws_phi_floats(d)) + 256;
  const size_t tcw = (d.seqlen % 128 == 0) ? bwd_tc_workspace_bytes(d) : 0;
  return simt > tcw ? simt : tcw;
}

template <int N, int P, typename T, bool MMB>
static int run_bwd(const M3BwdArgs& a, cudaStream_t s) {
  auto* kern = bwd_simt_kernel<N, P, T, MMB>;
  const size_t smem = BwdSmem<N, P>::bytes;
  static bool attr_done[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("bwd: cudaFuncSetAttribute");
    attr_done[dev] = true;
  }
  kern<<<a.dims.batch * a.dims.nheads, kSimtThreads, smem, s>>>(a);
  return check_launch("m3_siso_bwd");
}

int launch_bwd_simt(const M3BwdArgs& a, cudaStream_t s) {
  const bool mmb = a.policy == M3_POLICY_BF16;
  const bool bf = a.io_dtype == M3_DTYPE_BF16;
#define X(N_, P_)                                                                  \
  if (bf) return mmb ? run_bwd<N_, P_, __nv_bfloat16, true>(a, s) : run_bwd<N_, P_, __nv_bfloat16, false>(a, s); \
  return mmb ? run_bwd<N_, P_, float, true>(a, s) : run_bwd<N_, P_, float, false>(a, s);
  M3_DISPATCH_NP(a.dims.state_dim, a.dims.headdim, X);
#undef X
}

}  // namespace m3
