// Launchers of the forward kernels: the tcgen05 tensor-core kernel for the production
// shape, the generic CUDA-core kernel for everything else.
#include "m3_fwd_simt.cuh"
#include "m3_fwd_tc.cuh"
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

static bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static bool fwd_tc_eligible(const M3FwdArgs& a) {
  const M3Dims& d = a.dims;
  if (!(d.state_dim == tc::kN && d.headdim == tc::kP && a.io_dtype == M3_DTYPE_BF16 && a.policy == M3_POLICY_BF16))
    return false;
  if (d.chunk % tc::kC != 0 || d.seqlen % tc::kC != 0 || d.n_angles > 64 || d.n_angles % 8 != 0) return false;
  // 16-byte vector access to rows of q, k, v, z, y; 8-byte to the bias / angle pairs
  auto rows_ok = [](const void* p, const M3Strides& s, bool bhl) {
    if (!p) return true;
    return al16(p) && s.b % 8 == 0 && s.l % 8 == 0 && (!bhl || s.h % 8 == 0);
  };
  if (!rows_ok(a.q, a.q_st, false) || !rows_ok(a.k, a.k_st, false) || !rows_ok(a.v, a.v_st, true) ||
      !rows_ok(a.z, a.z_st, true) || !rows_ok(a.y, a.y_st, true))
    return false;
  if (((uintptr_t)a.q_bias & 7u) || ((uintptr_t)a.k_bias & 7u)) return false;
  if (a.raw && (!al16(a.angles) || (a.ang_st.b % 4) || (a.ang_st.l % 4))) return false;
  if (!a.raw && !al16(a.phi)) return false;
  if (a.ybar && !al16(a.ybar)) return false;
  return true;
}

static int run_fwd_tc(const M3FwdArgs& a, cudaStream_t s) {
  auto* kern = a.raw ? tc::fwd_tc_kernel<true> : tc::fwd_tc_kernel<false>;
  static bool attr_done[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[a.raw][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes) != cudaSuccess)
      return check_launch("fwd_tc: cudaFuncSetAttribute");
    attr_done[a.raw][dev] = true;
  }
  const int nseq = a.dims.batch * a.dims.nheads;
  kern<<<(nseq + 1) / 2, tc::kThreads, tc::kSmemBytes, s>>>(a);
  return check_launch("m3_siso_fwd (tensor core)");
}

int launch_fwd(const M3FwdArgs& a, cudaStream_t s) {
  const bool tc_ok = fwd_tc_eligible(a);
  if (a.kernel == M3_KERNEL_TENSORCORE && !tc_ok)
    return set_error(M3_ERR_UNSUPPORTED,
                     "tensor-core forward needs bf16 I/O, bf16 policy, N=128, P=64, chunk % 128 == 0, "
                     "n_angles a multiple of 8 and <= 64, and 16-byte aligned rows");
  if (tc_ok && a.kernel != M3_KERNEL_GENERIC) return run_fwd_tc(a, s);
  const bool mmb = a.policy == M3_POLICY_BF16;
  const bool bf = a.io_dtype == M3_DTYPE_BF16;
#define X(N_, P_)                                                                  \
  if (bf) return mmb ? run_fwd<N_, P_, __nv_bfloat16, true>(a, s) : run_fwd<N_, P_, __nv_bfloat16, false>(a, s); \
  return mmb ? run_fwd<N_, P_, float, true>(a, s) : run_fwd<N_, P_, float, false>(a, s);
  M3_DISPATCH_NP(a.dims.state_dim, a.dims.headdim, X);
#undef X
}

int read_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_m3_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_m3_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace m3

#ifdef M3_TC_TIMING
extern "C" int m3_debug_tc_timing(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, m3::g_m3_tc_timing, sizeof(unsigned long long) * 8);
  if (reset) {
    unsigned long long z[8] = {};
    cudaMemcpyToSymbol(m3::g_m3_tc_timing, z, sizeof(z));
  }
  return 0;
}
#endif
