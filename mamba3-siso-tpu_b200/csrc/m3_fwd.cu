// Launchers of the forward kernels: the tcgen05 tensor-core kernel for the production
// shape, the generic CUDA-core kernel for everything else.
#include "m3_fwd_simt.cuh"
#include "m3_fwd_tc.cuh"
#include "m3_fwd_ws.cuh"
#include "m3_bwd_tc.cuh"
#include "m3_internal.h"

#include <algorithm>

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

static size_t tc_tiles_bytes(const M3Dims& d);

// `states`: the states-only sweep; `save`: a full forward that also writes them
static int run_fwd_tc(const M3FwdArgs& a, cudaStream_t s, const tc::TcStates* states = nullptr,
                      const tc::TcStates* save = nullptr) {
  const int mode = (a.raw ? 1 : 0) + (states ? 2 : 0);
  decltype(&tc::fwd_tc_kernel<true, false>) kerns[4] = {tc::fwd_tc_kernel<false, false>, tc::fwd_tc_kernel<true, false>,
                                                         tc::fwd_tc_kernel<false, true>, tc::fwd_tc_kernel<true, true>};
  auto* kern = kerns[mode];
  static bool attr_done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[mode][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes) != cudaSuccess)
      return check_launch("fwd_tc: cudaFuncSetAttribute");
    attr_done[mode][dev] = true;
  }
  const int nseq = a.dims.batch * a.dims.nheads;
  const tc::TcStates so = states ? *states : save ? *save : tc::TcStates{nullptr, nullptr};
  kern<<<(nseq + 1) / 2, tc::kThreads, tc::kSmemBytes, s>>>(a, so);
  return check_launch("m3_siso_fwd (tensor core)");
}

// The backward's recompute sweep: chunk-start state tiles and angle carries only.
static bool fwd_ws_eligible(const M3FwdArgs& a, bool states_only);
static int run_fwd_ws(const M3FwdArgs& a, cudaStream_t s, uint8_t* tiles, float* phis, bool states_only);

int launch_fwd_states_tc(const M3FwdArgs& a, uint8_t* tiles, float* phis, cudaStream_t s) {
  if (fwd_ws_eligible(a, true)) return run_fwd_ws(a, s, tiles, phis, true);
  const tc::TcStates st{tiles, phis};
  return run_fwd_tc(a, s, &st);
}

// ---- warp-specialised TMA-fed forward ---------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// bf16 tensor with dims (inner..outer) and element strides of the outer dims; boxes of
// 64 inner elements x 128 rows (SWIZZLE_128B: one 128-byte row per token).
static bool make_map(CUtensorMap* m, const void* ptr, int rank, const uint64_t* dims, const int64_t* strides) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t gd[4], gs[3];
  cuuint32_t box[4], es[4];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    box[i] = i == 0 ? 64u : i == 1 ? 128u : 1u;
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gs[i] = (cuuint64_t)strides[i] * 2u;
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(ptr), gd, gs, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool fwd_ws_eligible(const M3FwdArgs& a, bool states_only) {
  if (a.kernel == M3_KERNEL_GENERIC || a.kernel == M3_KERNEL_TENSORCORE_V1) return false;
  if (!a.raw || (!states_only && !a.y) || a.ybar || a.chunk_states) return false;
  if (!fwd_tc_eligible(a)) return false;
  return al16(a.q_bias) && al16(a.k_bias);
}

size_t fwd_workspace_bytes(const M3Dims& d) {
  return ((size_t)d.batch * d.seqlen * d.n_angles * sizeof(float) + 255) & ~(size_t)255;
}

static int sm_count() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && n[dev]) return n[dev];
  int c = 148;
  cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) n[dev] = c;
  return c;
}

static int run_fwd_ws(const M3FwdArgs& a, cudaStream_t s, uint8_t* tiles, float* phis, bool states_only) {
  const M3Dims& d = a.dims;
  CUtensorMap tq, tk, tv, tz, ty;
  const uint64_t dq[3] = {(uint64_t)d.state_dim, (uint64_t)d.seqlen, (uint64_t)d.batch};
  const int64_t sq[2] = {a.q_st.l, a.q_st.b}, sk[2] = {a.k_st.l, a.k_st.b};
  const uint64_t dv[4] = {(uint64_t)d.headdim, (uint64_t)d.seqlen, (uint64_t)d.nheads, (uint64_t)d.batch};
  const int64_t sv[3] = {a.v_st.l, a.v_st.h, a.v_st.b}, sy[3] = {a.y_st.l, a.y_st.h, a.y_st.b};
  const int64_t sz[3] = {a.z_st.l, a.z_st.h, a.z_st.b};
  if (!make_map(&tq, a.q, 3, dq, sq) || !make_map(&tk, a.k, 3, dq, sk) || !make_map(&tv, a.v, 4, dv, sv) ||
      !make_map(&ty, states_only ? a.v : a.y, 4, dv, states_only ? sv : sy) || !make_map(&tz, a.z ? a.z : a.v, 4, dv, a.z ? sz : sv))
    return set_error(M3_ERR_LAUNCH, "m3_siso_fwd: cuTensorMapEncodeTiled failed");
  const bool pre = a.fwd_workspace && a.fwd_workspace_bytes >= fwd_workspace_bytes(d) &&
                   ((uintptr_t)a.fwd_workspace % 256) == 0;
  ws::Extra ex{nullptr, tiles, phis, d.batch * d.nheads};
  const int nsm = sm_count();
  if (pre) {
    float* T = (float*)a.fwd_workspace;
    if (!a.fwd_workspace_ready) {
      const size_t n4 = (size_t)d.batch * d.seqlen * (d.n_angles / 4);
      const int blocks = (int)std::min<size_t>((n4 + 255) / 256, (size_t)nsm * 8);
      ws::angle_rate_kernel<<<blocks, 256, 0, s>>>(a.angles, a.ang_st, d.batch, d.seqlen, d.n_angles, T);
      int rc = check_launch("m3_siso_fwd (angle rates)");
      if (rc != M3_OK) return rc;
    }
    ex.T = T;
  }
  decltype(&ws::fwd_ws_kernel<true, false>) kerns[4] = {ws::fwd_ws_kernel<false, false>, ws::fwd_ws_kernel<true, false>,
                                                         ws::fwd_ws_kernel<false, true>, ws::fwd_ws_kernel<true, true>};
  const int mode = (pre ? 1 : 0) + (states_only ? 2 : 0);
  auto* kern = kerns[mode];
  static bool attr_done[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[mode][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ws::kSmemBytes) != cudaSuccess)
      return check_launch("fwd_ws: cudaFuncSetAttribute");
    attr_done[mode][dev] = true;
  }
  const int grid = std::min(nsm, ex.nunits);
  kern<<<grid, ws::kThreads, ws::kSmemBytes, s>>>(a, tq, tk, tv, tz, ty, ex);
  return check_launch("m3_siso_fwd (tensor core, warp-specialised)");
}

bool fwd_tc_eligible_public(const M3FwdArgs& a) { return fwd_tc_eligible(a); }
bool fwd_saves_states(const M3FwdArgs& a) { return a.kernel != M3_KERNEL_GENERIC && fwd_tc_eligible(a); }

int launch_fwd(const M3FwdArgs& a, cudaStream_t s) {
  const bool tc_ok = fwd_tc_eligible(a);
  if ((a.kernel == M3_KERNEL_TENSORCORE || a.kernel == M3_KERNEL_TENSORCORE_V1) && !tc_ok)
    return set_error(M3_ERR_UNSUPPORTED,
                     "tensor-core forward needs bf16 I/O, bf16 policy, N=128, P=64, chunk % 128 == 0, "
                     "n_angles a multiple of 8 and <= 64, and 16-byte aligned rows");
  if (!a.y) {  // final state only: the states-only variant of the tensor-core kernel
    if (!tc_ok || a.kernel == M3_KERNEL_GENERIC)
      return set_error(M3_ERR_UNSUPPORTED, "y == NULL (final state only) needs the tensor-core forward");
    if (fwd_ws_eligible(a, true)) return run_fwd_ws(a, s, nullptr, nullptr, true);
    const tc::TcStates none{nullptr, nullptr};
    return run_fwd_tc(a, s, &none);
  }
  if (tc_ok && a.kernel != M3_KERNEL_GENERIC) {
    uint8_t* tiles = nullptr;
    float* phis = nullptr;
    if (a.bwd_states) {  // the backward workspace's state region: tiles, then angle carries
      tiles = (uint8_t*)a.bwd_states;
      phis = (float*)(tiles + tc_tiles_bytes(a.dims));
    }
    if (fwd_ws_eligible(a, false)) return run_fwd_ws(a, s, tiles, phis, false);
    if (tiles) {
      const tc::TcStates save{tiles, phis};
      return run_fwd_tc(a, s, nullptr, &save);
    }
    return run_fwd_tc(a, s);
  }
  const bool mmb = a.policy == M3_POLICY_BF16;
  const bool bf = a.io_dtype == M3_DTYPE_BF16;
#define X(N_, P_)                                                                  \
  if (bf) return mmb ? run_fwd<N_, P_, __nv_bfloat16, true>(a, s) : run_fwd<N_, P_, __nv_bfloat16, false>(a, s); \
  return mmb ? run_fwd<N_, P_, float, true>(a, s) : run_fwd<N_, P_, float, false>(a, s);
  M3_DISPATCH_NP(a.dims.state_dim, a.dims.headdim, X);
#undef X
}

// ---- backward on tensor cores ------------------------------------------------------------
static size_t tc_tiles_bytes(const M3Dims& d) {  // also the offset of the angle carries
  return (size_t)d.batch * d.nheads * (d.seqlen / tc::kC + 1) * 16384u;
}
static size_t tc_phis_bytes(const M3Dims& d) {
  return (size_t)d.batch * d.nheads * (d.seqlen / tc::kC) * d.n_angles * sizeof(float);
}
size_t bwd_tc_workspace_bytes(const M3Dims& d) {
  return tc_tiles_bytes(d) + tc_phis_bytes(d) + (size_t)d.batch * d.nheads * tcb::kScratchBytes + 256;
}

bool bwd_tc_eligible(const M3BwdArgs& a) {
  M3FwdArgs f{};
  f.dims = a.dims;
  f.io_dtype = a.io_dtype;
  f.policy = a.policy;
  f.raw = a.raw;
  f.phi = a.phi;
  f.q = a.q; f.k = a.k; f.v = a.v; f.z = a.z;
  f.q_st = a.q_st; f.k_st = a.k_st; f.v_st = a.v_st; f.z_st = a.z_st;
  f.angles = a.angles; f.ang_st = a.ang_st;
  f.q_bias = a.q_bias; f.k_bias = a.k_bias;
  if (!fwd_tc_eligible(f)) return false;
  auto rows_ok = [](const void* p, const M3Strides& s) {
    return al16(p) && s.b % 8 == 0 && s.l % 8 == 0 && s.h % 8 == 0;
  };
  if (!rows_ok(a.dy, a.dy_st)) return false;
  if (!al16(a.dq) || !al16(a.dk) || !al16(a.dv) || (a.dz && !al16(a.dz)) || !al16(a.dangles)) return false;
  for (const M3Strides* st : {&a.dv_st, &a.dz_st})  // 8-byte (bf16) / 16-byte (f32) row pieces
    if (st->b % 8 || st->h % 8 || st->l % 8) return false;
  return true;
}

int launch_bwd_tc(const M3BwdArgs& a, cudaStream_t s) {
  const M3Dims& d = a.dims;
  uint8_t* ws = (uint8_t*)a.workspace;
  uint8_t* tiles = ws;
  float* phis = (float*)(ws + tc_tiles_bytes(d));
  float* scratch = (float*)(ws + tc_tiles_bytes(d) + tc_phis_bytes(d));
  // sweep 1: recompute the chunk-start states (forward kernel, states-only mode)
  M3FwdArgs f{};
  f.dims = d;
  f.io_dtype = a.io_dtype;
  f.policy = a.policy;
  f.raw = a.raw;
  f.a_floor = a.a_floor;
  f.q = a.q; f.k = a.k; f.v = a.v;
  f.q_st = a.q_st; f.k_st = a.k_st; f.v_st = a.v_st;
  f.dt_raw = a.dt_raw; f.a_raw = a.a_raw; f.trap_raw = a.trap_raw; f.raw_st = a.raw_st;
  f.angles = a.angles; f.ang_st = a.ang_st; f.dt_bias = a.dt_bias;
  f.adt = a.adt; f.gamma = a.gamma; f.scale = a.scale; f.phi = a.phi;
  f.q_bias = a.q_bias; f.k_bias = a.k_bias; f.d_skip = a.d_skip;
  f.seed_ssm = a.seed_ssm; f.seed_k = a.seed_k; f.seed_v = a.seed_v; f.seed_phi = a.seed_phi;
  f.seed_coef = a.seed_coef;
  if (!a.states_ready) {  // else a forward on the same inputs already wrote them
    const int rc = launch_fwd_states_tc(f, tiles, phis, s);
    if (rc != M3_OK) return rc;
  }
  if (a.seed_ssm) {
    cudaMemsetAsync(a.dseed_k, 0, (size_t)d.batch * d.nheads * d.state_dim * sizeof(float), s);
    cudaMemsetAsync(a.dseed_v, 0, (size_t)d.batch * d.nheads * d.headdim * sizeof(float), s);
  }
  auto* kern = a.raw ? tcb::bwd_tc_kernel<true> : tcb::bwd_tc_kernel<false>;
  static bool attr_done[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[a.raw ? 1 : 0][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tcb::kSmemBytes) != cudaSuccess)
      return check_launch("bwd_tc: cudaFuncSetAttribute");
    attr_done[a.raw ? 1 : 0][dev] = true;
  }
  kern<<<d.batch * d.nheads, tcb::kThreads, tcb::kSmemBytes, s>>>(a, tiles, phis, scratch);
  return check_launch("m3_siso_bwd (tensor core)");
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
  cudaMemcpyFromSymbol(out, m3::g_m3_tc_timing, sizeof(unsigned long long) * 24);
  if (reset) {
    unsigned long long z[24] = {};
    cudaMemcpyToSymbol(m3::g_m3_tc_timing, z, sizeof(z));
  }
  return 0;
}
#endif

#ifdef M3_WS_TIMING
extern "C" int m3_debug_ws_timing(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, m3::ws::g_ws_wait, sizeof(unsigned long long) * 256);
  if (reset) {
    static unsigned long long z[256] = {};
    cudaMemcpyToSymbol(m3::ws::g_ws_wait, z, sizeof(z));
  }
  return 0;
}
#endif
