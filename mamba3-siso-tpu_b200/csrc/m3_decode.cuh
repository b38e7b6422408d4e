// Single-token decode step (mamba3_pallas/kernel_decode.py:56-233, reference.py:442-490):
//
//   phi' = wrap(phi + tanh(angles) pi dt)                 per head (dt is per head)
//   q~, k~ = R(phi') (q + q_bias), R(phi') (k + k_bias)
//   S'   = alpha S + beta v_prev k_prev^T + gamma v k~^T,  alpha = exp(adt),
//          beta = alpha dt (1 - lam), gamma = dt lam
//   y    = (S' q~ + D v) * silu(z)
//
// A bandwidth-bound read-modify-write of the (P, N) fp32 state, which is touched once.
// One CTA per (b, h).  A preamble computes, once per CTA, the rotated q~ / k~ columns and
// the per-row coefficients beta v_prev, gamma v and the gate into shared memory; then the
// state streams through in whole rows (a warp instruction covers 32 consecutive float4
// of the state, one 512-byte row at N = 128) with packed fp32x2 arithmetic, and the
// readout S' q~ is a shuffle reduction over the lanes of a row.  The state, k, v and phi
// buffers are updated in place.
#pragma once

#include "m3_common.cuh"

namespace m3 {

constexpr int kDecThreads = 256;

template <int N, int P, typename T, bool MMB>
__global__ void __launch_bounds__(kDecThreads, 4) decode_kernel(const M3DecodeArgs a) {
  static_assert(N <= 128 && P <= 128 && N % 4 == 0, "decode tiling");
  constexpr int LPR = N / 4;              // lanes (float4 columns) per state row
  constexpr int NF4 = P * N / 4;          // float4 of one (b, h) state
  constexpr int EPT = (NF4 + kDecThreads - 1) / kDecThreads;
  constexpr int H2 = N / 2;
  __shared__ __align__(16) float s_q[N], s_k[N], s_kp[N];  // q~ (readout-rounded), k~, previous k~
  __shared__ float s_bv[P], s_gv[P], s_dv[P], s_gate[P];  // beta v_prev, gamma v, D v, silu(z)
  __shared__ float s_ph[64];
  const int tid = threadIdx.x;
  const int H = a.nheads, Nr = a.n_angles;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const size_t bh = (size_t)b * H + h;

  // ---- the state: every load in flight first ---------------------------------------------
  float4* st4 = reinterpret_cast<float4*>(a.ssm + bh * P * N);
  float4 S[EPT];
#pragma unroll
  for (int m = 0; m < EPT; ++m) {
    const int i = tid + kDecThreads * m;
    if (i < NF4) S[m] = __ldcs(st4 + i);
  }

  // ---- scalars (raw == 1 fuses model.py:274-277) -----------------------------------
  float adt, dt, lam;
  if (a.raw) {
    const size_t o = (size_t)b * a.raw_stride_b + h;
    dt = softplusf(a.dt_raw[o] + a.dt_bias[h]);
    adt = fminf(-heavy_tail(a.a_raw[o]), -a.a_floor) * dt;
    lam = sigmoidf_(a.trap_raw[o]);
  } else {
    adt = a.adt[bh];
    dt = a.dt[bh];
    lam = a.lam[bh];
  }
  const float alpha = expf(adt);
  const float beta = alpha * dt * (1.f - lam);
  const float gamma = dt * lam;

  // ---- preamble: advanced angles; per-row coefficients -------------------------------------
  if (tid < Nr)
    s_ph[tid] = wrap_fast(a.phi[bh * Nr + tid] + tanh_acc(a.angles[(size_t)b * a.ang_stride_b + tid]) * kPi * dt);
  if (tid >= 128 && tid < 128 + P) {
    const int p = tid - 128;
    const T* vrow = (const T*)a.v + (size_t)b * a.vz_stride_b + (size_t)h * P;
    const float vc = ld(vrow + p);
    const float vp = a.state_v[bh * P + p];
    s_bv[p] = beta * vp;
    s_gv[p] = gamma * vc;
    s_dv[p] = a.d_skip ? a.d_skip[h] * vc : 0.f;
    float gate = 1.f;
    if (a.z) {
      const float zz = ld((const T*)a.z + (size_t)b * a.vz_stride_b + (size_t)h * P + p);
      gate = zz * sigmoidf_(zz);
    }
    s_gate[p] = gate;
    a.state_v[bh * P + p] = vc;
  }
  __syncthreads();
  // rotary columns: x cos + rot_half(x) sin, rot_half = [-hi, lo]  (layout.py:375-398)
  if (tid < N) {
    const int n = tid, j = n < H2 ? n : n - H2;
    const T* q = (const T*)a.q + (size_t)b * a.qk_stride_b;
    const T* k = (const T*)a.k + (size_t)b * a.qk_stride_b;
    const float u = ld(q + n) + a.q_bias[h * N + n];
    const float w = ld(k + n) + a.k_bias[h * N + n];
    float qv = u, kv = w;
    if (j < Nr) {
      const int mm = n < H2 ? n + H2 : n - H2;  // the pair partner
      const float um = ld(q + mm) + a.q_bias[h * N + mm];
      const float wm = ld(k + mm) + a.k_bias[h * N + mm];
      float sn, cs;
      sincos_wrapped(s_ph[j], &sn, &cs);
      const float sgn = n < H2 ? -1.f : 1.f;
      qv = u * cs + sgn * um * sn;
      kv = w * cs + sgn * wm * sn;
    }
    s_q[n] = mmr<MMB>(qv);
    s_k[n] = kv;
    s_kp[n] = a.state_k[bh * N + n];
    a.state_k[bh * N + n] = kv;
  }
  if (tid < Nr) a.phi[bh * Nr + tid] = s_ph[tid];  // nobody reads the old phi any more
  __syncthreads();

  // ---- S' = alpha S + (beta v_prev) k_prev^T + (gamma v) k~^T; y = (S' q~ + D v) silu(z) -----
  const int c4 = tid % LPR;
  const float4 q4 = *reinterpret_cast<const float4*>(s_q + 4 * c4);
  const float4 k4 = *reinterpret_cast<const float4*>(s_k + 4 * c4);
  const float4 kp4 = *reinterpret_cast<const float4*>(s_kp + 4 * c4);
  const float2 al2 = f2s(alpha);
  T* yrow = (T*)a.y + bh * P;
#pragma unroll
  for (int m = 0; m < EPT; ++m) {
    const int i = tid + kDecThreads * m;
    if (NF4 % kDecThreads != 0 && i >= NF4) break;  // NF4 % 32 == 0: whole warps stop together
    const int p = i / LPR;
    const float2 bv = f2s(s_bv[p]), gv = f2s(s_gv[p]);
    const float2 s01 = fma2(al2, f2(S[m].x, S[m].y), fma2(bv, f2(kp4.x, kp4.y), mul2(gv, f2(k4.x, k4.y))));
    const float2 s23 = fma2(al2, f2(S[m].z, S[m].w), fma2(bv, f2(kp4.z, kp4.w), mul2(gv, f2(k4.z, k4.w))));
    __stcs(st4 + i, make_float4(s01.x, s01.y, s23.x, s23.y));
    float2 r01 = s01, r23 = s23;
    if (MMB) {  // bf16 readout operands (kernel_decode.py, BF16 policy)
      r01 = bf2f(f2bf(s01));
      r23 = bf2f(f2bf(s23));
    }
    const float2 pr = fma2(r23, f2(q4.z, q4.w), mul2(r01, f2(q4.x, q4.y)));
    float part = pr.x + pr.y;
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (c4 == 0) stg<T>(yrow + p, (part + s_dv[p]) * s_gate[p]);
  }
}

}  // namespace m3
