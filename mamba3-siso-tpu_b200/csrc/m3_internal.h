// Host-side internals shared by the translation units of libm3siso.so.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "m3_siso.h"

namespace m3 {

// Records a thread-local error message and returns `code`.
int set_error(int code, const std::string& msg);
// Checks the launch that was just issued.
int check_launch(const char* what);

// Supported (N, P) pairs of the generic kernels.
bool supported_np(int n, int p);

int launch_fwd(const M3FwdArgs& a, cudaStream_t s);
int read_device_error(int reset);
int read_decode_error(int reset);
int read_gemm_error(int reset);
int launch_rms_norm(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int dim, float eps,
                    int x_dtype, int w_dtype, float* rstd, cudaStream_t s);
int launch_rms_norm_bwd(const void* x, int64_t xs, const void* w, const float* rstd, const void* dy, int64_t dys,
                        void* dx, int64_t dxs, float* dw, int64_t rows, int dim, int x_dtype, int w_dtype,
                        cudaStream_t s);
int launch_fwd_states_tc(const M3FwdArgs& a, uint8_t* tiles, float* phis, cudaStream_t s);
bool fwd_tc_eligible_public(const M3FwdArgs& a);
bool fwd_saves_states(const M3FwdArgs& a);
size_t bwd_tc_workspace_bytes(const M3Dims& d);
bool bwd_tc_eligible(const M3BwdArgs& a);
int launch_bwd_tc(const M3BwdArgs& a, cudaStream_t s);
int launch_bwd_simt(const M3BwdArgs& a, cudaStream_t s);
int launch_decode(const M3DecodeArgs& a, cudaStream_t s);
size_t bwd_workspace_bytes(const M3Dims& d);
size_t fwd_workspace_bytes(const M3Dims& d);
int launch_sample(const M3SampleArgs& a, cudaStream_t s);
int launch_gemv(const M3GemvArgs& a, cudaStream_t s);
int launch_gated_act(const void* x, int64_t xs, void* out, int64_t os, int64_t rows, int k, cudaStream_t s);
int gemv_ksplit(int m, int k, int n);

}  // namespace m3

// Instantiate `FN<N, P, T, MMB>` for the supported shapes; `call` is a lambda-like macro
// argument receiving the instantiated function.  Returns M3_ERR_UNSUPPORTED otherwise.
#define M3_DISPATCH_NP(n, p, X)                          \
  do {                                                   \
    if ((n) == 16 && (p) == 16) { X(16, 16); }           \
    else if ((n) == 32 && (p) == 16) { X(32, 16); }      \
    else if ((n) == 32 && (p) == 32) { X(32, 32); }      \
    else if ((n) == 64 && (p) == 64) { X(64, 64); }      \
    else if ((n) == 128 && (p) == 64) { X(128, 64); }    \
    else return m3::set_error(M3_ERR_UNSUPPORTED, "unsupported (state_dim, headdim) = (" + \
                              std::to_string(n) + ", " + std::to_string(p) + ")"); \
  } while (0)
