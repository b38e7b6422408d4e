// Launcher of the decode kernel.
#include "m3_decode.cuh"
#include "m3_internal.h"

namespace m3 {

template <int N, int P, typename T, bool MMB, bool FUSED>
static int run_decode_v(const M3DecodeArgs& a, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  static int sms[64] = {};
  static bool attr[64] = {};
  if (dev < 0 || dev >= 64) return set_error(M3_ERR_LAUNCH, "device index out of range");
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  if (!attr[dev]) {
    if (cudaFuncSetAttribute(decode_kernel<N, P, T, MMB, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)DecSmem<N, P>::kBytes) != cudaSuccess)
      return check_launch("m3_siso_decode: cudaFuncSetAttribute");
    attr[dev] = true;
  }
  const int items = a.batch * a.nheads;
  const int grid = items < sms[dev] * kDecCtasPerSm ? items : sms[dev] * kDecCtasPerSm;
  decode_kernel<N, P, T, MMB, FUSED><<<grid, kDecThreads, DecSmem<N, P>::kBytes, s>>>(a);
  return check_launch("m3_siso_decode");
}

template <int N, int P, typename T, bool MMB>
static int run_decode(const M3DecodeArgs& a, cudaStream_t s) {
  const bool fused = a.q_norm_w != nullptr || a.scalar_dtype == M3_DTYPE_BF16;
  return fused ? run_decode_v<N, P, T, MMB, true>(a, s) : run_decode_v<N, P, T, MMB, false>(a, s);
}

int read_decode_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_m3_dec_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_m3_dec_error, &zero, sizeof(int));
  }
  return v;
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
