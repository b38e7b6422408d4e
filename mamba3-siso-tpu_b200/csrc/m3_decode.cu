// Launcher of the decode kernel.
#include "m3_decode.cuh"
#include "m3_internal.h"

namespace m3 {

template <int N, int P, typename T, bool MMB>
static int run_decode(const M3DecodeArgs& a, cudaStream_t s) {
  decode_kernel<N, P, T, MMB><<<a.batch * a.nheads, kDecThreads, 0, s>>>(a);
  return check_launch("m3_siso_decode");
}

int launch_decode(const M3DecodeArgs& a, cudaStream_t s) {
  const bool mmb = a.policy == M3_POLICY_BF16;
  const bool bf = a.io_dtype == M3_DTYPE_BF16;
#define X(N_, P_)                                                                  \
  if (bf) return mmb ? run_decode<N_, P_, __nv_bfloat16, true>(a, s) : run_decode<N_, P_, __nv_bfloat16, false>(a, s); \
  return mmb ? run_decode<N_, P_, float, true>(a, s) : run_decode<N_, P_, float, false>(a, s);
  M3_DISPATCH_NP(a.state_dim, a.headdim, X);
#undef X
}

}  // namespace m3
