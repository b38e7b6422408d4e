// Shared device helpers for the Mamba-3 SISO kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "m3_siso.h"

namespace m3 {

constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 6.28318530717958647692f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kSimtThreads = 256;  // block size of the generic CUDA-core kernels

template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void stg(T* p, float x);
template <> __device__ __forceinline__ void stg<float>(float* p, float x) { *p = x; }
template <> __device__ __forceinline__ void stg<__nv_bfloat16>(__nv_bfloat16* p, float x) {
  *p = __float2bfloat16_rn(x);
}

// Round-to-nearest-even through bf16: the matmul-operand cast of the BF16 policy
// (mamba3_pallas/kernel_fwd.py:139-141).
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <bool MMB> __device__ __forceinline__ float mmr(float x) { return MMB ? bf16r(x) : x; }

// softplus(x) = max(x, 0) + log1p(exp(-|x|))  (jax.nn.softplus, reference.py:186)
__device__ __forceinline__ float softplusf(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
// heavy_tail(x) = max(x,0) + 1/(1 - min(x,0))  (reference.py:202-209)
__device__ __forceinline__ float heavy_tail(float x) { return fmaxf(x, 0.f) + 1.f / (1.f - fminf(x, 0.f)); }
// phi - 2 pi floor(phi / 2 pi)  (reference.py:156)
__device__ __forceinline__ float wrap2pi(float x) { return x - kTwoPi * floorf(x / kTwoPi); }

// Packed fp32x2 arithmetic (sm_100 FFMA2 / FADD2 / FMUL2): one instruction per two
// lanes of work, each component rounded exactly as its scalar counterpart.
__device__ __forceinline__ float2 f2(float x, float y) { return make_float2(x, y); }
__device__ __forceinline__ float2 f2s(float x) { return make_float2(x, x); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// the two bf16 halves of a packed word as fp32 (exact)
__device__ __forceinline__ float2 bf2f(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f2bf(float2 v) {
  __nv_bfloat162 t = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<uint32_t*>(&t);
}

// Eight consecutive floats with one 256-bit load (sm_100; the address is 32-byte aligned).
__device__ __forceinline__ void ldg8(const float* p, float (&v)[8]) {
  asm volatile("ld.global.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}

// sin / cos of an angle in [0, 2 pi) through the SFU (accurate on [-pi, pi]).
__device__ __forceinline__ void sincos_wrapped(float x, float* s, float* c) {
  if (x >= kPi) x -= kTwoPi;
  __sincosf(x, s, c);
}

// 2^x on the SFU (relative error ~2^-22; flushes subnormal results to zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// phi - 2 pi floor(phi / 2 pi) with a reciprocal multiply instead of a division.
__device__ __forceinline__ float wrap_fast(float x) {
  return x - kTwoPi * floorf(x * 0.15915494309189535f);
}

// 1/x on the SFU (rcp.approx: about 1 ulp; flushes subnormals).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// tanh from exp2 and the SFU reciprocal: |error| ~ 1e-7 absolute and unbiased, so the
// cumulative angle does not drift (tanh.approx's 2^-11 would).
__device__ __forceinline__ float tanh_acc(float x) {
  const float e = ex2(2.f * kLog2e * fminf(fabsf(x), 15.f));
  const float t = 1.f - 2.f * rcp_approx(e + 1.f);
  return copysignf(t, x);
}

// sigmoid of two values on the SFU (exp2 and reciprocal; ~1e-7 relative), for the
// bf16-output gate of the tensor-core kernels.
__device__ __forceinline__ float2 sigmoid2(float2 z) {
  const float2 m = mul2(z, f2s(-kLog2e));
  const float2 d = add2(f2(ex2(m.x), ex2(m.y)), f2s(1.f));
  return f2(rcp_approx(d.x), rcp_approx(d.y));
}
__device__ __forceinline__ float2 silu2(float2 z) { return mul2(z, sigmoid2(z)); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Inclusive scan over the 32 lanes of a warp.
__device__ __forceinline__ float warp_inclusive_scan(float x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

// Output-tile geometry for an (M x NC) block computed by NT threads: thread (ty, tx)
// owns rows ty + RY*i and columns tx + RX*j (strided so neighbouring lanes touch
// neighbouring shared-memory banks).
template <int M, int NC, int NT>
struct Tile {
  static constexpr int RX = NC < 16 ? NC : 16;
  static constexpr int RY = NT / RX;
  static constexpr int TM = M / RY;
  static constexpr int TN = NC / RX;
  static_assert(NT % RX == 0, "tile");
  static_assert(M % RY == 0 && TM >= 1, "tile rows");
  static_assert(NC % RX == 0, "tile cols");
};

}  // namespace m3
