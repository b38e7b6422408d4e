// Single-token decode step (mamba3_pallas/kernel_decode.py:56-233, reference.py:442-490):
//
//   phi' = wrap(phi + tanh(angles) pi dt)                 per head (dt is per head)
//   q~, k~ = R(phi') (q + q_bias), R(phi') (k + k_bias)
//   S'   = alpha S + beta v_prev k_prev^T + gamma v k~^T,  alpha = exp(adt),
//          beta = alpha dt (1 - lam), gamma = dt lam
//   y    = (S' q~ + D v) * silu(z)
//
// A bandwidth-bound read-modify-write of the (P, N) fp32 state, which is touched once:
// one CTA per (b, h), each warp owns P / 8 state rows, each lane N / 32 consecutive
// columns loaded as one 128-bit vector; the readout S' q~ is a warp-shuffle reduction
// per row.  The state, k, v and phi buffers are updated in place.
#pragma once

#include "m3_common.cuh"

namespace m3 {

constexpr int kDecThreads = 256;

template <int N>
struct DecVec {
  static constexpr int V = N >= 32 ? N / 32 : 1;      // columns per lane
  static constexpr int LANES = N >= 32 ? 32 : N;      // active lanes per row
};

template <int V> struct F4 { float x[V]; };

// The state is read once and written once per step: stream it past L1 / L2 residency
// (evict-first loads, streaming stores).
template <int V>
__device__ __forceinline__ F4<V> ldv(const float* p) {
  F4<V> r;
  if constexpr (V == 4) {
    float4 t = __ldcs(reinterpret_cast<const float4*>(p));
    r.x[0] = t.x; r.x[1] = t.y; r.x[2] = t.z; r.x[3] = t.w;
  } else if constexpr (V == 2) {
    float2 t = *reinterpret_cast<const float2*>(p);
    r.x[0] = t.x; r.x[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) r.x[i] = p[i];
  }
  return r;
}

template <int V>
__device__ __forceinline__ void stv(float* p, const F4<V>& r) {
  if constexpr (V == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(r.x[0], r.x[1], r.x[2], r.x[3]));
  } else if constexpr (V == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r.x[0], r.x[1]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = r.x[i];
  }
}

template <int N, int P, typename T, bool MMB>
__global__ void __launch_bounds__(kDecThreads, 4) decode_kernel(const M3DecodeArgs a) {
  constexpr int V = DecVec<N>::V, LANES = DecVec<N>::LANES, H2 = N / 2;
  constexpr int NW = kDecThreads / 32;
  constexpr int RPW = (P + NW - 1) / NW;  // rows per warp
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.nheads, Nr = a.n_angles;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const size_t bh = (size_t)b * H + h;
  const bool active = lane < LANES;
  const int n0 = lane * V;

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

  // ---- the state rows this warp owns: issue every load first ---------------------------
  float* srow = a.ssm + bh * P * N;
  F4<V> S[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int p = warp * RPW + r;
    if (active && p < P) S[r] = ldv<V>(srow + (size_t)p * N + n0);
  }

  // ---- rotary angle advance and rotation of this lane's columns ----------------------
  const T* q = (const T*)a.q + (size_t)b * a.qk_stride_b;
  const T* k = (const T*)a.k + (size_t)b * a.qk_stride_b;
  float qr[V], kr[V], kp[V];
  float phi_new[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int n = n0 + i;
    qr[i] = kr[i] = kp[i] = phi_new[i] = 0.f;
    if (!active) continue;
    const int j = n < H2 ? n : n - H2;
    const float u = ld(q + n) + a.q_bias[h * N + n];
    const float w = ld(k + n) + a.k_bias[h * N + n];
    float qv = u, kv = w;
    if (j < Nr) {
      const float ph = wrap_fast(a.phi[bh * Nr + j] + tanh_acc(a.angles[(size_t)b * a.ang_stride_b + j]) * kPi * dt);
      phi_new[i] = ph;
      const int m = n < H2 ? n + H2 : n - H2;  // the pair partner
      const float um = ld(q + m) + a.q_bias[h * N + m];
      const float wm = ld(k + m) + a.k_bias[h * N + m];
      float sn, cs;
      sincos_wrapped(ph, &sn, &cs);
      // x cos + rot_half(x) sin, rot_half = [-hi, lo]  (layout.py:375-398)
      const float sgn = n < H2 ? -1.f : 1.f;
      qv = u * cs + sgn * um * sn;
      kv = w * cs + sgn * wm * sn;
    }
    qr[i] = qv;
    kr[i] = kv;
    kp[i] = a.state_k[bh * N + n];
  }

  const T* vrow = (const T*)a.v + (size_t)b * a.vz_stride_b + (size_t)h * P;
  const T* zrow = a.z ? (const T*)a.z + (size_t)b * a.vz_stride_b + (size_t)h * P : nullptr;
  float yv[RPW];
  float vcur[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int p = warp * RPW + r;
    yv[r] = 0.f;
    vcur[r] = 0.f;
    if (p >= P) continue;
    const float vp = a.state_v[bh * P + p];
    const float vc = ld(vrow + p);
    vcur[r] = vc;
    float part = 0.f;
    if (active) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float s = alpha * S[r].x[i] + beta * vp * kp[i] + gamma * vc * kr[i];
        S[r].x[i] = s;
        part = fmaf(mmr<MMB>(s), mmr<MMB>(qr[i]), part);
      }
    }
    yv[r] = warp_sum(part);
  }
  // All reads of the carried k/v/phi are done before anyone overwrites them.
  __syncthreads();

#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int p = warp * RPW + r;
    if (p >= P) continue;
    if (active) stv<V>(srow + (size_t)p * N + n0, S[r]);
    if (lane == 0) {
      float o = yv[r];
      if (a.d_skip) o += a.d_skip[h] * vcur[r];
      if (zrow) {
        const float zz = ld(zrow + p);
        o *= zz * sigmoidf_(zz);
      }
      stg<T>((T*)a.y + bh * P + p, o);
      a.state_v[bh * P + p] = vcur[r];
    }
  }
  if (warp == 0 && active) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int n = n0 + i;
      a.state_k[bh * N + n] = kr[i];
      if (n < Nr) a.phi[bh * Nr + n] = phi_new[i];
    }
  }
}

}  // namespace m3
