// extern "C" entry points of libm3siso.so: argument validation (the counterpart of the
// reference's ValueErrors), stride defaults, output zeroing, dispatch.
#include <cstring>
#include <string>

#include "m3_internal.h"

namespace m3 {

static thread_local std::string g_err;

int set_error(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(M3_ERR_LAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  return M3_OK;
}

bool supported_np(int n, int p) {
  return (n == 16 && p == 16) || (n == 32 && p == 16) || (n == 32 && p == 32) || (n == 64 && p == 64) ||
         (n == 128 && p == 64);
}

static bool zero(const M3Strides& s) { return s.b == 0 && s.h == 0 && s.l == 0; }

// (B, L, X) tensors (q, k, angles): default b = L*X, l = X
static void def_blx(M3Strides& s, const M3Dims& d, int x) {
  if (zero(s)) s = M3Strides{(int64_t)d.seqlen * x, 0, x};
}
// (B, H, L, P) tensors
static void def_bhlp(M3Strides& s, const M3Dims& d) {
  if (zero(s)) s = M3Strides{(int64_t)d.nheads * d.seqlen * d.headdim, (int64_t)d.seqlen * d.headdim, d.headdim};
}
// (B, L, H) raw scalar streams
static void def_blh(M3Strides& s, const M3Dims& d) {
  if (zero(s)) s = M3Strides{(int64_t)d.seqlen * d.nheads, 1, d.nheads};
}

static int check_dims(const M3Dims& d, int sub) {
  if (d.batch <= 0 || d.seqlen <= 0 || d.nheads <= 0 || d.state_dim <= 0 || d.headdim <= 0 || d.n_angles <= 0)
    return set_error(M3_ERR_SHAPE, "all dims must be positive");
  if (d.chunk <= 0 || d.chunk % 64 != 0)
    return set_error(M3_ERR_UNSUPPORTED, "chunk must be a positive multiple of 64, got " + std::to_string(d.chunk));
  if (d.seqlen % d.chunk != 0)
    return set_error(M3_ERR_SHAPE, "seqlen (" + std::to_string(d.seqlen) + ") must be a multiple of chunk (" +
                                       std::to_string(d.chunk) + "); pad the sequence before calling");
  if (d.seqlen % sub != 0) return set_error(M3_ERR_SHAPE, "seqlen must be a multiple of the sub-chunk");
  if (d.n_angles > d.state_dim / 2)
    return set_error(M3_ERR_SHAPE, "n_angles (" + std::to_string(d.n_angles) + ") exceeds state_dim // 2 (" +
                                       std::to_string(d.state_dim / 2) + ")");
  if (d.n_angles > 64) return set_error(M3_ERR_UNSUPPORTED, "n_angles > 64");
  if (!supported_np(d.state_dim, d.headdim))
    return set_error(M3_ERR_UNSUPPORTED, "unsupported (state_dim, headdim) = (" + std::to_string(d.state_dim) +
                                             ", " + std::to_string(d.headdim) + ")");
  return M3_OK;
}

static int check_enums(int io, int pol) {
  if (io != M3_DTYPE_F32 && io != M3_DTYPE_BF16) return set_error(M3_ERR_ARG, "io_dtype must be F32 or BF16");
  if (pol != M3_POLICY_F32 && pol != M3_POLICY_BF16) return set_error(M3_ERR_ARG, "policy must be F32 or BF16");
  return M3_OK;
}

template <class Args>
static int check_common_inputs(const Args& a) {
  if (!a.q || !a.k || !a.v || !a.q_bias || !a.k_bias) return set_error(M3_ERR_ARG, "q, k, v, q_bias, k_bias are required");
  if (a.raw != 0 && a.raw != 1) return set_error(M3_ERR_ARG, "raw must be 0 or 1");
  if (a.raw) {
    if (!a.dt_raw || !a.a_raw || !a.trap_raw || !a.angles || !a.dt_bias)
      return set_error(M3_ERR_ARG, "raw boundary needs dt_raw, a_raw, trap_raw, angles and dt_bias");
  } else {
    if (!a.adt || !a.gamma || !a.scale || !a.phi)
      return set_error(M3_ERR_ARG, "preprocessed boundary needs adt, gamma, scale and phi");
  }
  const bool any = a.seed_ssm || a.seed_k || a.seed_v;
  const bool all = a.seed_ssm && a.seed_k && a.seed_v && (a.raw || a.seed_coef);
  if (any && !all)
    return set_error(M3_ERR_ARG, "seed_ssm, seed_k, seed_v and seed_coef must be given together");
  if (!a.raw && a.seed_coef && !a.seed_ssm)
    return set_error(M3_ERR_ARG, "seed_ssm, seed_k, seed_v and seed_coef must be given together");
  return M3_OK;
}

}  // namespace m3

using namespace m3;

extern "C" {

const char* m3_last_error(void) { return g_err.c_str(); }

int m3_version(void) { return 1; }

int m3_rms_norm(const void* x, int64_t x_row_stride, const void* weight, void* y, int64_t y_row_stride, int64_t rows,
                int32_t dim, float eps, int32_t x_dtype, int32_t w_dtype, float* rstd, void* stream) {
  if (!x || !weight || !y) return m3::set_error(M3_ERR_ARG, "m3_rms_norm: NULL pointer");
  if (rows < 0 || dim <= 0 || x_row_stride < dim || y_row_stride < dim)
    return m3::set_error(M3_ERR_SHAPE, "m3_rms_norm: bad rows / dim / strides");
  if ((x_dtype != M3_DTYPE_BF16 && x_dtype != M3_DTYPE_F32) || (w_dtype != M3_DTYPE_BF16 && w_dtype != M3_DTYPE_F32))
    return m3::set_error(M3_ERR_UNSUPPORTED, "m3_rms_norm: dtype must be bf16 or f32");
  if (rows == 0) return M3_OK;
  return m3::launch_rms_norm(x, x_row_stride, weight, y, y_row_stride, rows, dim, eps, x_dtype, w_dtype, rstd,
                             (cudaStream_t)stream);
}

int m3_rms_norm_bwd(const void* x, int64_t x_row_stride, const void* weight, const float* rstd, const void* dy,
                    int64_t dy_row_stride, void* dx, int64_t dx_row_stride, float* dweight, int64_t rows, int32_t dim,
                    int32_t x_dtype, int32_t w_dtype, void* stream) {
  if (!x || !weight || !rstd || !dy || !dx || !dweight) return m3::set_error(M3_ERR_ARG, "m3_rms_norm_bwd: NULL pointer");
  if (rows < 0 || dim <= 0 || dim > 2048 || x_row_stride < dim || dy_row_stride < dim || dx_row_stride < dim)
    return m3::set_error(M3_ERR_SHAPE, "m3_rms_norm_bwd: bad rows / dim (<= 2048) / strides");
  if ((x_dtype != M3_DTYPE_BF16 && x_dtype != M3_DTYPE_F32) || (w_dtype != M3_DTYPE_BF16 && w_dtype != M3_DTYPE_F32))
    return m3::set_error(M3_ERR_UNSUPPORTED, "m3_rms_norm_bwd: dtype must be bf16 or f32");
  if (rows == 0) return M3_OK;
  return m3::launch_rms_norm_bwd(x, x_row_stride, weight, rstd, dy, dy_row_stride, dx, dx_row_stride, dweight, rows,
                                 dim, x_dtype, w_dtype, (cudaStream_t)stream);
}

int m3_copy2d_async(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t height,
                    void* stream) {
  if (!dst || !src) return m3::set_error(M3_ERR_ARG, "m3_copy2d_async: NULL pointer");
  if (width > dpitch || width > spitch) return m3::set_error(M3_ERR_SHAPE, "m3_copy2d_async: width exceeds a pitch");
  if (width == 0 || height == 0) return M3_OK;
  const cudaError_t e =
      cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault, (cudaStream_t)stream);
  if (e != cudaSuccess) return m3::set_error(M3_ERR_LAUNCH, std::string("m3_copy2d_async: ") + cudaGetErrorString(e));
  return M3_OK;
}

size_t m3_gemv_scratch_floats(int32_t m, int32_t k, int32_t n) {
  if (m <= 0 || k <= 0 || n <= 0) return 0;
  const int mp = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
  return (size_t)m3::gemv_ksplit(m, k, n) * mp * n;
}

int m3_gemv_bf16(const M3GemvArgs* args, void* stream) {
  if (!args) return m3::set_error(M3_ERR_ARG, "m3_gemv_bf16: args is NULL");
  const M3GemvArgs& a = *args;
  if (!a.x || !a.w || !a.out || !a.scratch || !a.tickets || (a.x_mode == 1 && !a.norm_w))
    return m3::set_error(M3_ERR_ARG, "m3_gemv_bf16: NULL pointer");
  if (a.m <= 0 || a.m > 8 || a.k <= 0 || a.n <= 0 || a.n % 8 || a.w_ld % 8 || a.w_ld < a.n || a.out_ld < a.n ||
      a.x_ld < (a.x_mode == 2 ? 2 * (int64_t)a.k : a.k) || (a.residual && a.r_ld < a.n))
    return m3::set_error(M3_ERR_SHAPE, "m3_gemv_bf16: bad m (1..8) / k / n (multiple of 8) / leading dimensions");
  if (a.x_mode < 0 || a.x_mode > 2) return m3::set_error(M3_ERR_ARG, "m3_gemv_bf16: x_mode must be 0, 1 or 2");
  if (((uintptr_t)a.w) % 16) return m3::set_error(M3_ERR_ARG, "m3_gemv_bf16: w must be 16-byte aligned");
  return m3::launch_gemv(a, (cudaStream_t)stream);
}

int m3_gated_act_bf16(const void* x, int64_t x_row_stride, void* out, int64_t out_row_stride, int64_t rows,
                      int32_t k, void* stream) {
  if (!x || !out) return m3::set_error(M3_ERR_ARG, "m3_gated_act_bf16: NULL pointer");
  if (rows < 0 || k <= 0 || k % 8 || x_row_stride % 8 || out_row_stride % 8 || x_row_stride < 2 * (int64_t)k ||
      out_row_stride < k || ((uintptr_t)x) % 16 || ((uintptr_t)out) % 16)
    return m3::set_error(M3_ERR_SHAPE, "m3_gated_act_bf16: k and strides must be multiples of 8, rows 16-byte aligned");
  if (rows == 0) return M3_OK;
  return m3::launch_gated_act(x, x_row_stride, out, out_row_stride, rows, k, (cudaStream_t)stream);
}

int m3_sample_tokens(const M3SampleArgs* args, void* stream) {
  if (!args) return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: args is NULL");
  const M3SampleArgs& a = *args;
  if (!a.logits || !a.out_token || (a.vocab > 184320 && !a.scratch))
    return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: NULL pointer");
  if (a.batch < 0 || a.vocab <= 0 || a.vocab >= 8388608 || a.logits_ld < a.vocab || (a.probs_out && a.probs_ld < a.vocab))
    return m3::set_error(M3_ERR_SHAPE, "m3_sample_tokens: bad batch / vocab / leading dimension");
  if (a.logits_dtype != M3_DTYPE_F32 && a.logits_dtype != M3_DTYPE_BF16)
    return m3::set_error(M3_ERR_UNSUPPORTED, "m3_sample_tokens: logits must be f32 or bf16");
  if (!(a.temperature > 0.f) || !(a.rep_penalty > 0.f) || !(a.top_p >= 0.f))
    return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: temperature and rep_penalty must be > 0, top_p >= 0");
  if (a.window && (!a.window_state || !a.seen_count || a.rep_window <= 0))
    return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: a window needs window_state, seen_count and rep_window > 0");
  if (a.n_stop < 0 || (a.n_stop > 0 && !a.stop_ids)) return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: stop ids");
  if (a.history && (!a.counter || a.history_cap <= 0))
    return m3::set_error(M3_ERR_ARG, "m3_sample_tokens: history needs a counter and history_cap > 0");
  if (a.batch == 0) return M3_OK;
  return m3::launch_sample(a, (cudaStream_t)stream);
}

int m3_device_error(int reset) {
  const int f = read_device_error(reset), d = read_decode_error(reset), g = read_gemm_error(reset);
  return f != 0 ? f : d != 0 ? d : g;
}

static void fwd_defaults(M3FwdArgs& a) {
  def_blx(a.q_st, a.dims, a.dims.state_dim);
  def_blx(a.k_st, a.dims, a.dims.state_dim);
  def_bhlp(a.v_st, a.dims);
  def_bhlp(a.z_st, a.dims);
  def_bhlp(a.y_st, a.dims);
  def_blh(a.raw_st, a.dims);
  def_blx(a.ang_st, a.dims, a.dims.n_angles);
}

int m3_siso_fwd_saves_states(const M3FwdArgs* args) {
  if (!args) return 0;
  M3FwdArgs a = *args;
  if (check_enums(a.io_dtype, a.policy) != M3_OK || check_dims(a.dims, 64) != M3_OK) return 0;
  fwd_defaults(a);
  return fwd_saves_states(a) ? 1 : 0;
}

int m3_siso_fwd(const M3FwdArgs* args, void* stream) {
  g_err.clear();
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  M3FwdArgs a = *args;
  int rc;
  if ((rc = check_enums(a.io_dtype, a.policy)) != M3_OK) return rc;
  if ((rc = check_dims(a.dims, 64)) != M3_OK) return rc;
  if ((rc = check_common_inputs(a)) != M3_OK) return rc;
  if (!a.final_ssm || !a.final_k || !a.final_v) return set_error(M3_ERR_ARG, "final_ssm, final_k, final_v are required");
  if (a.chunk_states && a.chunk_states_dtype != M3_DTYPE_F32 && a.chunk_states_dtype != M3_DTYPE_BF16)
    return set_error(M3_ERR_ARG, "chunk_states_dtype must be F32 or BF16");
  fwd_defaults(a);
  if (a.kernel < M3_KERNEL_AUTO || a.kernel > M3_KERNEL_TENSORCORE_V1)
    return set_error(M3_ERR_ARG, "kernel must be AUTO, GENERIC, TENSORCORE or TENSORCORE_V1");
  if (a.fwd_workspace && ((uintptr_t)a.fwd_workspace) % 256 != 0)
    return set_error(M3_ERR_ARG, "fwd_workspace must be 256-byte aligned");
  if (a.bwd_states && a.bwd_states_bytes < bwd_workspace_bytes(a.dims))
    return set_error(M3_ERR_WORKSPACE, "bwd_states is smaller than m3_siso_bwd_workspace_size");
  if (a.bwd_states && ((uintptr_t)a.bwd_states) % 256 != 0)
    return set_error(M3_ERR_ARG, "bwd_states must be 256-byte aligned");
  return launch_fwd(a, (cudaStream_t)stream);
}

size_t m3_siso_fwd_workspace_size(const M3Dims* dims) {
  if (!dims) return 0;
  return fwd_workspace_bytes(*dims);
}

size_t m3_siso_bwd_workspace_size(const M3Dims* dims) {
  if (!dims) return 0;
  return bwd_workspace_bytes(*dims);
}

int m3_siso_bwd(const M3BwdArgs* args, void* stream) {
  g_err.clear();
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  M3BwdArgs a = *args;
  if (a.grad_dtype != M3_DTYPE_F32 && a.grad_dtype != M3_DTYPE_BF16)
    return set_error(M3_ERR_ARG, "grad_dtype must be F32 or BF16");
  int rc;
  if ((rc = check_enums(a.io_dtype, a.policy)) != M3_OK) return rc;
  if ((rc = check_dims(a.dims, 32)) != M3_OK) return rc;
  if ((rc = check_common_inputs(a)) != M3_OK) return rc;
  if (!a.dy || !a.dq || !a.dk || !a.dv || !a.dq_bias || !a.dk_bias)
    return set_error(M3_ERR_ARG, "dy, dq, dk, dv, dq_bias, dk_bias are required");
  if (a.z && !a.dz) return set_error(M3_ERR_ARG, "dz is required when z is given");
  if (a.d_skip && !a.dd_skip) return set_error(M3_ERR_ARG, "dd_skip is required when d_skip is given");
  if (a.raw) {
    if (!a.ddt_raw || !a.da_raw || !a.dtrap_raw || !a.dangles || !a.ddt_bias)
      return set_error(M3_ERR_ARG, "raw boundary needs ddt_raw, da_raw, dtrap_raw, dangles, ddt_bias");
    if (a.seed_phi && !a.dseed_phi) return set_error(M3_ERR_ARG, "dseed_phi is required when seed_phi is given");
  } else {
    if (!a.dadt || !a.dgamma || !a.dscale || !a.dphi)
      return set_error(M3_ERR_ARG, "preprocessed boundary needs dadt, dgamma, dscale, dphi");
  }
  if (a.seed_ssm && (!a.dseed_ssm || !a.dseed_k || !a.dseed_v || (!a.raw && !a.dseed_coef)))
    return set_error(M3_ERR_ARG, "seed gradients are required when a seed is given");
  const size_t need = bwd_workspace_bytes(a.dims);
  if (!a.workspace || a.workspace_bytes < need)
    return set_error(M3_ERR_WORKSPACE, "workspace of " + std::to_string(need) + " bytes required");
  if (((uintptr_t)a.workspace) % 256 != 0) return set_error(M3_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  def_blx(a.q_st, a.dims, a.dims.state_dim);
  def_blx(a.k_st, a.dims, a.dims.state_dim);
  def_bhlp(a.v_st, a.dims);
  def_bhlp(a.z_st, a.dims);
  def_bhlp(a.dy_st, a.dims);
  def_bhlp(a.dv_st, a.dims);
  def_bhlp(a.dz_st, a.dims);
  def_blh(a.raw_st, a.dims);
  def_blx(a.ang_st, a.dims, a.dims.n_angles);
  cudaStream_t s = (cudaStream_t)stream;
  const M3Dims& d = a.dims;
  // outputs accumulated with atomics start at zero
  const size_t bln = (size_t)d.batch * d.seqlen * d.state_dim * sizeof(float);
  cudaMemsetAsync(a.dq, 0, bln, s);
  cudaMemsetAsync(a.dk, 0, bln, s);
  cudaMemsetAsync(a.dq_bias, 0, (size_t)d.nheads * d.state_dim * sizeof(float), s);
  cudaMemsetAsync(a.dk_bias, 0, (size_t)d.nheads * d.state_dim * sizeof(float), s);
  if (a.d_skip) cudaMemsetAsync(a.dd_skip, 0, (size_t)d.nheads * sizeof(float), s);
  if (a.raw) {
    cudaMemsetAsync(a.ddt_bias, 0, (size_t)d.nheads * sizeof(float), s);
    cudaMemsetAsync(a.dangles, 0, (size_t)d.batch * d.seqlen * d.n_angles * sizeof(float), s);
  }
  if ((rc = check_launch("m3_siso_bwd: zeroing")) != M3_OK) return rc;
  if (a.kernel < M3_KERNEL_AUTO || a.kernel > M3_KERNEL_TENSORCORE)
    return set_error(M3_ERR_ARG, "kernel must be AUTO, GENERIC or TENSORCORE");
  const bool tc_ok = bwd_tc_eligible(a);
  if (a.kernel == M3_KERNEL_TENSORCORE && !tc_ok)
    return set_error(M3_ERR_UNSUPPORTED,
                     "tensor-core backward needs the raw boundary, bf16 I/O, bf16 policy, N=128, P=64, "
                     "chunk % 128 == 0, n_angles a multiple of 8 and <= 64, and 16-byte aligned rows");
  if (tc_ok && a.kernel != M3_KERNEL_GENERIC) return launch_bwd_tc(a, s);
  return launch_bwd_simt(a, s);
}

int m3_siso_decode(const M3DecodeArgs* args, void* stream) {
  g_err.clear();
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  M3DecodeArgs a = *args;
  int rc;
  if ((rc = check_enums(a.io_dtype, a.policy)) != M3_OK) return rc;
  if (a.batch <= 0 || a.nheads <= 0 || a.state_dim <= 0 || a.headdim <= 0 || a.n_angles <= 0)
    return set_error(M3_ERR_SHAPE, "all dims must be positive");
  if (a.n_angles > a.state_dim / 2) return set_error(M3_ERR_SHAPE, "n_angles exceeds state_dim // 2");
  if (!supported_np(a.state_dim, a.headdim))
    return set_error(M3_ERR_UNSUPPORTED, "unsupported (state_dim, headdim) = (" + std::to_string(a.state_dim) +
                                             ", " + std::to_string(a.headdim) + ")");
  if (!a.q || !a.k || !a.v || !a.angles || !a.q_bias || !a.k_bias || !a.ssm || !a.state_k || !a.state_v || !a.phi ||
      !a.y)
    return set_error(M3_ERR_ARG, "q, k, v, angles, biases, state buffers and y are required");
  if (a.raw) {
    if (!a.dt_raw || !a.a_raw || !a.trap_raw || !a.dt_bias)
      return set_error(M3_ERR_ARG, "raw decode needs dt_raw, a_raw, trap_raw, dt_bias");
  } else if (!a.adt || !a.dt || !a.lam) {
    return set_error(M3_ERR_ARG, "decode needs adt, dt, lam");
  }
  if (((uintptr_t)a.ssm) % 16 != 0) return set_error(M3_ERR_ARG, "ssm must be 16-byte aligned");
  if (a.scalar_dtype != M3_DTYPE_F32 && a.scalar_dtype != M3_DTYPE_BF16)
    return set_error(M3_ERR_UNSUPPORTED, "scalar_dtype must be f32 or bf16");
  if ((a.q_norm_w == nullptr) != (a.k_norm_w == nullptr))
    return set_error(M3_ERR_ARG, "q_norm_w and k_norm_w go together");
  if (a.qk_stride_b == 0) a.qk_stride_b = a.state_dim;
  if (a.vz_stride_b == 0) a.vz_stride_b = (int64_t)a.nheads * a.headdim;
  if (a.raw_stride_b == 0) a.raw_stride_b = a.nheads;
  if (a.ang_stride_b == 0) a.ang_stride_b = a.n_angles;
  return launch_decode(a, (cudaStream_t)stream);
}

}  // extern "C"
