// XLA FFI handlers over libm3siso.so: the jax.ffi registration of the three kernels, so the
// reference's JAX callers (kernel_fwd.siso_forward, kernel_bwd.siso_backward,
// kernel_decode.decode_step: mamba3_pallas/kernel_fwd.py:204-388, kernel_bwd.py:534-669,
// kernel_decode.py:252-471) can call them in place of their pallas_call.
//
// Build (on a machine with jaxlib, which ships the XLA FFI headers):
//   nvcc -std=c++17 -O2 -Xcompiler -fPIC -shared -I<repo>/include \
//        -I$(python -c "import jax.ffi; print(jax.ffi.include_dir())") \
//        m3_ffi.cc -L<repo>/mamba3-siso-tpu_b200/mamba3_b200/_lib -lm3siso -o libm3ffi.so
//
// Every handler runs its kernel on the stream XLA hands it and allocates nothing: the
// backward uses m3_siso_bwd_noalloc (its scratch is a fixed array inside libm3siso.so), as
// a custom call has only its operands and results.  Errors come back as
// ffi::Error::InvalidArgument carrying m3_last_error().
#if __has_include("xla/ffi/api/ffi.h")
#include <cuda_runtime.h>

#include <cstdint>

#include "m3_siso.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

int32_t io_of(const ffi::AnyBuffer& b) { return b.element_type() == ffi::BF16 ? M3_DTYPE_BF16 : M3_DTYPE_F32; }

ffi::Error status(int rc) {
  return rc == M3_OK ? ffi::Error::Success() : ffi::Error::InvalidArgument(m3_last_error());
}

// Preprocessed boundary forward (siso_forward): q, k (B, L, N); v, z (B, H, L, P);
// adt, gamma, scale (B, H, L); phi (B, H, L, Nr).
ffi::Error SisoFwd(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer z,
                   ffi::Buffer<ffi::F32> adt, ffi::Buffer<ffi::F32> gamma, ffi::Buffer<ffi::F32> scale,
                   ffi::Buffer<ffi::F32> phi, ffi::Buffer<ffi::F32> q_bias, ffi::Buffer<ffi::F32> k_bias,
                   ffi::Buffer<ffi::F32> d_skip, int32_t chunk, int32_t policy, ffi::Result<ffi::AnyBuffer> y,
                   ffi::Result<ffi::Buffer<ffi::F32>> fs, ffi::Result<ffi::Buffer<ffi::F32>> fk,
                   ffi::Result<ffi::Buffer<ffi::F32>> fv) {
  const auto qd = q.dimensions(), vd = v.dimensions(), pd = phi.dimensions();
  M3FwdArgs a{};
  a.dims = M3Dims{(int32_t)qd[0], (int32_t)qd[1], (int32_t)vd[1], (int32_t)qd[2], (int32_t)vd[3], (int32_t)pd[3],
                  chunk};
  a.io_dtype = io_of(q);
  a.policy = policy;
  a.q = q.untyped_data();
  a.k = k.untyped_data();
  a.v = v.untyped_data();
  a.z = z.untyped_data();
  a.adt = adt.typed_data();
  a.gamma = gamma.typed_data();
  a.scale = scale.typed_data();
  a.phi = phi.typed_data();
  a.q_bias = q_bias.typed_data();
  a.k_bias = k_bias.typed_data();
  a.d_skip = d_skip.typed_data();
  a.y = y->untyped_data();
  a.final_ssm = fs->typed_data();
  a.final_k = fk->typed_data();
  a.final_v = fv->typed_data();
  return status(m3_siso_fwd(&a, stream));
}

// Preprocessed boundary backward (siso_backward) without a workspace operand.
ffi::Error SisoBwd(cudaStream_t stream, ffi::AnyBuffer dy, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                   ffi::AnyBuffer z, ffi::Buffer<ffi::F32> adt, ffi::Buffer<ffi::F32> gamma,
                   ffi::Buffer<ffi::F32> scale, ffi::Buffer<ffi::F32> phi, ffi::Buffer<ffi::F32> q_bias,
                   ffi::Buffer<ffi::F32> k_bias, ffi::Buffer<ffi::F32> d_skip, int32_t chunk, int32_t policy,
                   ffi::Result<ffi::Buffer<ffi::F32>> dq, ffi::Result<ffi::Buffer<ffi::F32>> dk,
                   ffi::Result<ffi::Buffer<ffi::F32>> dv, ffi::Result<ffi::Buffer<ffi::F32>> dz,
                   ffi::Result<ffi::Buffer<ffi::F32>> dadt, ffi::Result<ffi::Buffer<ffi::F32>> dgamma,
                   ffi::Result<ffi::Buffer<ffi::F32>> dscale, ffi::Result<ffi::Buffer<ffi::F32>> dphi,
                   ffi::Result<ffi::Buffer<ffi::F32>> dq_bias, ffi::Result<ffi::Buffer<ffi::F32>> dk_bias,
                   ffi::Result<ffi::Buffer<ffi::F32>> dd_skip) {
  const auto qd = q.dimensions(), vd = v.dimensions(), pd = phi.dimensions();
  M3BwdArgs a{};
  a.dims = M3Dims{(int32_t)qd[0], (int32_t)qd[1], (int32_t)vd[1], (int32_t)qd[2], (int32_t)vd[3], (int32_t)pd[3],
                  chunk};
  a.io_dtype = io_of(q);
  a.policy = policy;
  a.dy = dy.untyped_data();
  a.q = q.untyped_data();
  a.k = k.untyped_data();
  a.v = v.untyped_data();
  a.z = z.untyped_data();
  a.adt = adt.typed_data();
  a.gamma = gamma.typed_data();
  a.scale = scale.typed_data();
  a.phi = phi.typed_data();
  a.q_bias = q_bias.typed_data();
  a.k_bias = k_bias.typed_data();
  a.d_skip = d_skip.typed_data();
  a.dq = dq->typed_data();
  a.dk = dk->typed_data();
  a.dv = dv->typed_data();
  a.dz = dz->typed_data();
  a.dadt = dadt->typed_data();
  a.dgamma = dgamma->typed_data();
  a.dscale = dscale->typed_data();
  a.dphi = dphi->typed_data();
  a.dq_bias = dq_bias->typed_data();
  a.dk_bias = dk_bias->typed_data();
  a.dd_skip = dd_skip->typed_data();
  return status(m3_siso_bwd_noalloc(&a, stream));
}

// One decode step (decode_step); the state buffers are aliased in -> out by the caller
// (input_output_aliases), as the reference donates them.
ffi::Error SisoDecode(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer z,
                      ffi::Buffer<ffi::F32> adt, ffi::Buffer<ffi::F32> dt, ffi::Buffer<ffi::F32> lam,
                      ffi::Buffer<ffi::F32> angles, ffi::Buffer<ffi::F32> q_bias, ffi::Buffer<ffi::F32> k_bias,
                      ffi::Buffer<ffi::F32> d_skip, ffi::Buffer<ffi::F32> ssm, ffi::Buffer<ffi::F32> sk,
                      ffi::Buffer<ffi::F32> sv, ffi::Buffer<ffi::F32> sphi, int32_t policy,
                      ffi::Result<ffi::AnyBuffer> y, ffi::Result<ffi::Buffer<ffi::F32>> ssm_out,
                      ffi::Result<ffi::Buffer<ffi::F32>> k_out, ffi::Result<ffi::Buffer<ffi::F32>> v_out,
                      ffi::Result<ffi::Buffer<ffi::F32>> phi_out) {
  const auto qd = q.dimensions(), vd = v.dimensions(), ad = angles.dimensions();
  (void)ssm;
  (void)sk;
  (void)sv;
  (void)sphi;  // aliased with the results: the kernel updates them in place
  M3DecodeArgs a{};
  a.batch = (int32_t)qd[0];
  a.state_dim = (int32_t)qd[1];
  a.nheads = (int32_t)vd[1];
  a.headdim = (int32_t)vd[2];
  a.n_angles = (int32_t)ad[1];
  a.io_dtype = io_of(q);
  a.policy = policy;
  a.q = q.untyped_data();
  a.k = k.untyped_data();
  a.v = v.untyped_data();
  a.z = z.untyped_data();
  a.adt = adt.typed_data();
  a.dt = dt.typed_data();
  a.lam = lam.typed_data();
  a.angles = angles.typed_data();
  a.q_bias = q_bias.typed_data();
  a.k_bias = k_bias.typed_data();
  a.d_skip = d_skip.typed_data();
  a.ssm = ssm_out->typed_data();
  a.state_k = k_out->typed_data();
  a.state_v = v_out->typed_data();
  a.phi = phi_out->typed_data();
  a.y = y->untyped_data();
  return status(m3_siso_decode(&a, stream));
}

}  // namespace

#define M3_F32 ffi::Buffer<ffi::F32>
XLA_FFI_DEFINE_HANDLER_SYMBOL(kM3SisoFwd, SisoFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Attr<int32_t>("chunk").Attr<int32_t>("policy")
                                  .Ret<ffi::AnyBuffer>().Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>());
XLA_FFI_DEFINE_HANDLER_SYMBOL(kM3SisoBwd, SisoBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Attr<int32_t>("chunk").Attr<int32_t>("policy")
                                  .Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>()
                                  .Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>()
                                  .Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>());
XLA_FFI_DEFINE_HANDLER_SYMBOL(kM3SisoDecode, SisoDecode,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>().Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>().Arg<M3_F32>()
                                  .Attr<int32_t>("policy")
                                  .Ret<ffi::AnyBuffer>().Ret<M3_F32>().Ret<M3_F32>().Ret<M3_F32>()
                                  .Ret<M3_F32>());
#undef M3_F32
#endif  // __has_include("xla/ffi/api/ffi.h")
