// Generic (CUDA-core) backward of the chunked scan.  One CTA per (b, h):
//
//  sweep 1 (forward):  recompute the state at every 32-token sub-chunk start into the
//                      workspace (the forward saves no residuals), plus the rotary
//                      angle carry at each sub-chunk start for the raw boundary;
//  sweep 2 (reverse):  per sub-chunk, with g = dy silu(z) and the adjoint G carried in
//                      shared memory (mamba3_pallas/kernel_bwd.py:10-19, 103-355):
//     Wm   = tril_strict((q~ khat^T) exp2(min(A_i - A_j, 0)))
//     dM   = tril_strict((g v^T)     exp2(min(A_i - A_j, 0)))
//     ybar = exp2(A) (q~ S^T) + Wm v + (D + gamma u.w) v      (recomputed, for dz)
//     dq~  = dM khat + exp2(A) (g S)
//     dkhat= dM^T q~ + exp2(A_last - A) (v G)
//     dv   = Wm^T g + exp2(A_last - A) (khat G^T) + (D + gamma u.w) g
//     G   <- exp2(A_last) G + (exp2(A) g)^T q~
//     dA_t = q~_t.dq~_t - khat_t.dkhat_t, plus the A_last term on every position after
//            the suffix sum (kernel_bwd.py:264-285)
//  followed by the rotation pullback, the head reduction of dq/dk (atomic adds into the
//  head-shared (B, L, N) gradients; kernel_bwd.py:292-333), the epilogue of
//  kernel_bwd.py:592-651 (dgamma, dD, dfinal_* injection, seed gradients) and, on the
//  raw boundary, the autodiff of reference.preprocess (softplus / heavy-tail / sigmoid /
//  trapezoid shift / cumulative angles; reference.py:104-199).
#pragma once

#include "m3_chunk_common.cuh"

namespace m3 {

// dv / dz element in the requested gradient dtype (the struct's pointers are float*)
__device__ __forceinline__ void store_grad(float* base, size_t i, float v, int32_t dtype) {
  if (dtype == M3_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16(v);
  else
    base[i] = v;
}

constexpr int kBwdSub = 32;

template <int N, int P>
struct BwdSmem {
  static constexpr int CS = kBwdSub, H2 = N / 2, NT = kSimtThreads;
  static constexpr int qs = 0;
  static constexpr int ks = qs + CS * (N + 1);
  static constexpr int vs = ks + CS * (N + 1);
  static constexpr int gs = vs + CS * (P + 1);
  static constexpr int st = gs + CS * (P + 1);
  static constexpr int Gs = st + P * (N + 1);
  static constexpr int sW = Gs + P * (N + 1);
  static constexpr int sM = sW + CS * (CS + 1);
  static constexpr int dqs = sM + CS * (CS + 1);
  static constexpr int dks = dqs + CS * (N + 1);
  static constexpr int phis = dks + CS * (N + 1);
  static constexpr int dph = phis + CS * H2;
  static constexpr int adt = dph + CS * H2;
  static constexpr int gam = adt + CS;
  static constexpr int scl = gam + CS;
  static constexpr int A = scl + CS;
  static constexpr int av = A + CS;
  static constexpr int uw = av + CS;
  static constexpr int dqkd = uw + CS;
  static constexpr int dg = dqkd + CS;
  static constexpr int dA = dg + CS;
  static constexpr int dsc = dA + CS;
  static constexpr int dth = dsc + CS;
  static constexpr int dtv = dth + CS;       // CS + 1
  static constexpr int lamv = dtv + CS + 1;  // CS + 1
  static constexpr int carry = lamv + CS + 1;
  static constexpr int dcarry = carry + H2;
  static constexpr int dqb = dcarry + H2;
  static constexpr int dkb = dqb + N;
  static constexpr int part = dkb + N;
  static constexpr int red = part + NT;
  static constexpr int total = red + 64;
  static constexpr size_t bytes = sizeof(float) * (size_t)total;
};

// Sum over the block; every thread gets the total.  `red` needs 33 floats.
__device__ __forceinline__ float block_sum(float x, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  x = warp_sum(x);
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    float y = lane < nw ? red[lane] : 0.f;
    y = warp_sum(y);
    if (lane == 0) red[32] = y;
  }
  __syncthreads();
  return red[32];
}

__host__ __device__ inline size_t bwd_ws_state_floats(const M3Dims& d) {
  return (size_t)d.batch * d.nheads * (d.seqlen / kBwdSub) * d.headdim * d.state_dim;
}
__host__ __device__ inline size_t bwd_ws_phi_floats(const M3Dims& d) {
  return (size_t)d.batch * d.nheads * (d.seqlen / kBwdSub) * d.n_angles;
}

template <int N, int P, typename T, bool MMB>
__global__ void __launch_bounds__(kSimtThreads) bwd_simt_kernel(const M3BwdArgs a) {
  using SM = BwdSmem<N, P>;
  constexpr int CS = kBwdSub, NT = kSimtThreads, H2 = N / 2;
  extern __shared__ float sm[];
  float* qs = sm + SM::qs;
  float* ks = sm + SM::ks;
  float* vs = sm + SM::vs;
  float* gs = sm + SM::gs;
  float* st = sm + SM::st;
  float* Gs = sm + SM::Gs;
  float* sW = sm + SM::sW;
  float* sM = sm + SM::sM;
  float* dqs = sm + SM::dqs;
  float* dks = sm + SM::dks;
  float* phis = sm + SM::phis;
  float* dph = sm + SM::dph;
  float* adts = sm + SM::adt;
  float* gam = sm + SM::gam;
  float* scl = sm + SM::scl;
  float* A = sm + SM::A;
  float* av = sm + SM::av;
  float* uw = sm + SM::uw;
  float* dqkd = sm + SM::dqkd;
  float* dg = sm + SM::dg;
  float* dA = sm + SM::dA;
  float* dsc = sm + SM::dsc;
  float* dth = sm + SM::dth;
  float* dtv = sm + SM::dtv;
  float* lamv = sm + SM::lamv;
  float* carry = sm + SM::carry;
  float* dcarry = sm + SM::dcarry;
  float* dqb = sm + SM::dqb;
  float* dkb = sm + SM::dkb;
  float* part = sm + SM::part;
  float* red = sm + SM::red;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.dims.nheads, L = a.dims.seqlen, Nr = a.dims.n_angles;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const size_t bh = (size_t)b * H + h;
  const int nsub = L / CS;
  const T* q = (const T*)a.q;
  const T* k = (const T*)a.k;
  const T* v = (const T*)a.v;
  const T* z = (const T*)a.z;
  const T* dy = (const T*)a.dy;
  const float Dh = a.d_skip ? a.d_skip[h] : 0.f;
  float* ws_state = (float*)a.workspace + bh * (size_t)nsub * P * N;
  float* ws_phi = (float*)a.workspace + bwd_ws_state_floats(a.dims) + bh * (size_t)nsub * Nr;

  // Rotate rows 0..CS-1 of the sub-chunk: ks = khat (and qs = q~ when `with_q`), both
  // unrounded fp32; uw / dg per row.  Warp per row, lane per rotary pair.
  auto rotate_rows = [&](int t0, bool with_q) {
    for (int i = warp; i < CS; i += NT / 32) {
      const int t = t0 + i;
      const T* qrow = q + (size_t)b * a.q_st.b + (size_t)t * a.q_st.l;
      const T* krow = k + (size_t)b * a.k_st.b + (size_t)t * a.k_st.l;
      float uwp = 0.f;
      for (int j = lane; j < H2; j += 32) {
        const float wlo = ld(krow + j) + a.k_bias[h * N + j];
        const float whi = ld(krow + j + H2) + a.k_bias[h * N + j + H2];
        float cs = 1.f, sn = 0.f;
        if (j < Nr) {
          const float ph = a.raw ? phis[i * H2 + j] : a.phi[(bh * L + t) * Nr + j];
          sincosf(ph, &sn, &cs);
        }
        ks[i * (N + 1) + j] = (wlo * cs - whi * sn) * scl[i];
        ks[i * (N + 1) + j + H2] = (whi * cs + wlo * sn) * scl[i];
        if (with_q) {
          const float ulo = ld(qrow + j) + a.q_bias[h * N + j];
          const float uhi = ld(qrow + j + H2) + a.q_bias[h * N + j + H2];
          qs[i * (N + 1) + j] = ulo * cs - uhi * sn;
          qs[i * (N + 1) + j + H2] = uhi * cs + ulo * sn;
          uwp += ulo * wlo + uhi * whi;
        }
      }
      if (with_q) {
        uwp = warp_sum(uwp);
        if (lane == 0) {
          uw[i] = uwp;
          dg[i] = uwp * gam[i] + Dh;
        }
      }
    }
  };
  auto load_pc = [&](const T* base, const M3Strides& s, int t0, float* dst) {
    for (int idx = tid; idx < CS * P; idx += NT) {
      const int i = idx / P, p = idx % P;
      dst[i * (P + 1) + p] = ld(base + (size_t)b * s.b + (size_t)h * s.h + (size_t)(t0 + i) * s.l + p);
    }
  };

  // ======================= sweep 1: chunk-start states ===========================
  float coef = 0.f, dt0 = 0.f, lam0 = 0.f;
  if (a.seed_ssm) {
    if (a.raw) {
      const size_t o = (size_t)b * a.raw_st.b + (size_t)h * a.raw_st.h;
      dt0 = softplusf(a.dt_raw[o] + a.dt_bias[h]);
      lam0 = sigmoidf_(a.trap_raw[o]);
      coef = dt0 * (1.f - lam0);
    } else {
      coef = a.seed_coef[bh];
    }
  }
  for (int idx = tid; idx < P * N; idx += NT) {
    const int p = idx / N, n = idx % N;
    float s0 = 0.f;
    if (a.seed_ssm) s0 = a.seed_ssm[bh * P * N + idx] + coef * a.seed_v[bh * P + p] * a.seed_k[bh * N + n];
    st[p * (N + 1) + n] = s0;
  }
  if (a.raw)
    for (int r = tid; r < Nr; r += NT) carry[r] = a.seed_phi ? a.seed_phi[bh * Nr + r] : 0.f;
  __syncthreads();
  for (int sc = 0; sc < nsub; ++sc) {
    const int t0 = sc * CS;
    if (a.raw)
      for (int r = tid; r < Nr; r += NT) ws_phi[(size_t)sc * Nr + r] = carry[r];
    prep_scalars<CS, NT>(a, b, h, t0, adts, gam, scl, A, dtv, lamv, av);
    if (a.raw) phi_scan<CS, NT>(a, b, t0, dtv, phis, H2, carry, part);
    rotate_rows(t0, false);
    load_pc(v, a.v_st, t0, vs);
    for (int idx = tid; idx < P * N; idx += NT) ws_state[(size_t)sc * P * N + idx] = st[(idx / N) * (N + 1) + idx % N];
    __syncthreads();
    {
      const float Al = A[CS - 1];
      for (int idx = tid; idx < CS * P; idx += NT) {
        const int i = idx / P, p = idx % P;
        gs[i * (P + 1) + p] = mmr<MMB>(vs[i * (P + 1) + p] * exp2f(Al - A[i]));
      }
    }
    __syncthreads();
    {
      using TL = Tile<P, N, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
#pragma unroll 4
      for (int s = 0; s < CS; ++s) {
        float va[TL::TM], kb[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) va[i] = gs[s * (P + 1) + ty + TL::RY * i];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) kb[j] = mmr<MMB>(ks[s * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(va[i], kb[j], acc[i][j]);
      }
      const float eAl = exp2f(A[CS - 1]);
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          float* sp = st + (ty + TL::RY * i) * (N + 1) + tx + TL::RX * j;
          *sp = *sp * eAl + acc[i][j];
        }
    }
    __syncthreads();
  }

  // ======================= sweep 2: reverse adjoint scan ==========================
  for (int idx = tid; idx < P * N; idx += NT)
    Gs[(idx / N) * (N + 1) + idx % N] = a.dfinal_ssm ? a.dfinal_ssm[bh * P * N + idx] : 0.f;
  for (int r = tid; r < H2; r += NT) dcarry[r] = (a.raw && a.dfinal_phi && r < Nr) ? a.dfinal_phi[bh * Nr + r] : 0.f;
  for (int n = tid; n < N; n += NT) dqb[n] = dkb[n] = 0.f;
  float dD_acc = 0.f, ddtb_acc = 0.f;  // thread-private partials, reduced at the end
  __syncthreads();

  for (int sc = nsub - 1; sc >= 0; --sc) {
    const int t0 = sc * CS;
    prep_scalars<CS, NT>(a, b, h, t0, adts, gam, scl, A, dtv, lamv, av);
    if (a.raw) {
      for (int r = tid; r < Nr; r += NT) carry[r] = ws_phi[(size_t)sc * Nr + r];
      __syncthreads();
      phi_scan<CS, NT>(a, b, t0, dtv, phis, H2, carry, part);
    }
    for (int idx = tid; idx < P * N; idx += NT) st[(idx / N) * (N + 1) + idx % N] = ws_state[(size_t)sc * P * N + idx];
    rotate_rows(t0, true);
    load_pc(v, a.v_st, t0, vs);
    // g = dy silu(z)  (kernel_bwd.py:186-196)
    for (int idx = tid; idx < CS * P; idx += NT) {
      const int i = idx / P, p = idx % P, t = t0 + i;
      float g = ld(dy + (size_t)b * a.dy_st.b + (size_t)h * a.dy_st.h + (size_t)t * a.dy_st.l + p);
      if (z) {
        const float zz = ld(z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)t * a.z_st.l + p);
        g *= zz * sigmoidf_(zz);
      }
      gs[i * (P + 1) + p] = g;
    }
    __syncthreads();
    // dqk_diag_t = g_t . v_t
    for (int i = warp; i < CS; i += NT / 32) {
      float x = 0.f;
      for (int p = lane; p < P; p += 32) x += gs[i * (P + 1) + p] * vs[i * (P + 1) + p];
      x = warp_sum(x);
      if (lane == 0) dqkd[i] = x;
    }
    // Wm and dM (kernel_bwd.py:205-220)
    {
      using TL = Tile<CS, CS, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float aw[TL::TM][TL::TN] = {}, am[TL::TM][TL::TN] = {};
      for (int n = 0; n < N; ++n) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(qs[(ty + TL::RY * i) * (N + 1) + n]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(ks[(tx + TL::RX * j) * (N + 1) + n]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) aw[i][j] = fmaf(x[i], y[j], aw[i][j]);
      }
      for (int p = 0; p < P; ++p) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(gs[(ty + TL::RY * i) * (P + 1) + p]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(vs[(tx + TL::RX * j) * (P + 1) + p]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) am[i][j] = fmaf(x[i], y[j], am[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          const int ti = ty + TL::RY * i, sj = tx + TL::RX * j;
          const bool low = ti > sj;
          const float dec = exp2f(fminf(A[ti] - A[sj], 0.f));
          sW[ti * (CS + 1) + sj] = low ? mmr<MMB>(aw[i][j] * dec) : 0.f;
          sM[ti * (CS + 1) + sj] = low ? mmr<MMB>(am[i][j] * dec) : 0.f;
        }
    }
    __syncthreads();

    const float Al = A[CS - 1];
    // ybar (recomputed) -> dz  (kernel_bwd.py:186-196)
    if (z) {
      using TL = Tile<CS, P, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
      for (int n = 0; n < N; ++n) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(qs[(ty + TL::RY * i) * (N + 1) + n]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(st[(tx + TL::RX * j) * (N + 1) + n]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const float e = exp2f(A[ty + TL::RY * i]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) acc[i][j] *= e;
      }
      for (int s = 0; s < CS; ++s) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = sW[(ty + TL::RY * i) * (CS + 1) + s];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(vs[s * (P + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const int ti = ty + TL::RY * i, t = t0 + ti;
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          const int p = tx + TL::RX * j;
          const float ybar = acc[i][j] + dg[ti] * vs[ti * (P + 1) + p];
          const float dyv = ld(dy + (size_t)b * a.dy_st.b + (size_t)h * a.dy_st.h + (size_t)t * a.dy_st.l + p);
          const float zz = ld(z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)t * a.z_st.l + p);
          const float sg = sigmoidf_(zz);
          store_grad(a.dz, (size_t)b * a.dz_st.b + (size_t)h * a.dz_st.h + (size_t)t * a.dz_st.l + p,
                     dyv * ybar * sg * (1.f + zz * (1.f - sg)), a.grad_dtype);
        }
      }
    }
    // dq~ = dM khat + exp2(A) (g S)  -> dqs
    {
      using TL = Tile<CS, N, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
      for (int p = 0; p < P; ++p) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(gs[(ty + TL::RY * i) * (P + 1) + p]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(st[p * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const float e = exp2f(A[ty + TL::RY * i]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) acc[i][j] *= e;
      }
      for (int s = 0; s < CS; ++s) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = sM[(ty + TL::RY * i) * (CS + 1) + s];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(ks[s * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) dqs[(ty + TL::RY * i) * (N + 1) + tx + TL::RX * j] = acc[i][j];
    }
    // dkhat = dM^T q~ + exp2(A_last - A) (v G)  -> dks ; A_last term part 2
    float alast_part = 0.f;
    {
      using TL = Tile<CS, N, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
      for (int p = 0; p < P; ++p) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(vs[(ty + TL::RY * i) * (P + 1) + p]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(Gs[p * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const int si = ty + TL::RY * i;
        const float e = exp2f(Al - A[si]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          acc[i][j] *= e;
          alast_part += ks[si * (N + 1) + tx + TL::RX * j] * acc[i][j];
        }
      }
      for (int t = 0; t < CS; ++t) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = sM[t * (CS + 1) + ty + TL::RY * i];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(qs[t * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) dks[(ty + TL::RY * i) * (N + 1) + tx + TL::RX * j] = acc[i][j];
    }
    // dv = Wm^T g + exp2(A_last - A) (khat G^T) + coeff g   -> global
    {
      using TL = Tile<CS, P, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
      for (int n = 0; n < N; ++n) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(ks[(ty + TL::RY * i) * (N + 1) + n]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(Gs[(tx + TL::RX * j) * (N + 1) + n]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const float e = exp2f(Al - A[ty + TL::RY * i]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) acc[i][j] *= e;
      }
      for (int t = 0; t < CS; ++t) {
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = sW[t * (CS + 1) + ty + TL::RY * i];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(gs[t * (P + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const int si = ty + TL::RY * i, t = t0 + si;
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          const int p = tx + TL::RX * j;
          float o = acc[i][j] + dg[si] * gs[si * (P + 1) + p];
          if (t == L - 1 && a.dfinal_v) o += a.dfinal_v[bh * P + p];
          store_grad(a.dv, (size_t)b * a.dv_st.b + (size_t)h * a.dv_st.h + (size_t)t * a.dv_st.l + p, o,
                     a.grad_dtype);
        }
      }
    }
    // sum(G * S) for the A_last term (kernel_bwd.py:280-282)
    float gsum = 0.f;
    for (int idx = tid; idx < P * N; idx += NT) {
      const int o = (idx / N) * (N + 1) + idx % N;
      gsum += Gs[o] * st[o];
    }
    const float alast_term = exp2f(Al) * block_sum(gsum, red) + block_sum(alast_part, red);

    // G <- exp2(A_last) G + (exp2(A) g)^T q~   (kernel_bwd.py:346-350)
    {
      using TL = Tile<P, N, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
      for (int t = 0; t < CS; ++t) {
        const float e = exp2f(A[t]);
        float x[TL::TM], y[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) x[i] = mmr<MMB>(e * gs[t * (P + 1) + ty + TL::RY * i]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) y[j] = mmr<MMB>(qs[t * (N + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
      }
      const float eAl = exp2f(Al);
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          float* gp = Gs + (ty + TL::RY * i) * (N + 1) + tx + TL::RX * j;
          *gp = *gp * eAl + acc[i][j];
        }
    }

    // ---- per-row pullback: rotation, head sums, dscale, dphi, dA (kernel_bwd.py:264-333)
    for (int i = warp; i < CS; i += NT / 32) {
      const int t = t0 + i;
      const T* qrow = q + (size_t)b * a.q_st.b + (size_t)t * a.q_st.l;
      const T* krow = k + (size_t)b * a.k_st.b + (size_t)t * a.k_st.l;
      const float dgm = dqkd[i] * gam[i];
      float dsp = 0.f, dap = 0.f;
      for (int j = lane; j < H2; j += 32) {
        const float ulo = ld(qrow + j) + a.q_bias[h * N + j];
        const float uhi = ld(qrow + j + H2) + a.q_bias[h * N + j + H2];
        const float wlo = ld(krow + j) + a.k_bias[h * N + j];
        const float whi = ld(krow + j + H2) + a.k_bias[h * N + j + H2];
        float cs = 1.f, sn = 0.f;
        if (j < Nr) {
          const float ph = a.raw ? phis[i * H2 + j] : a.phi[(bh * L + t) * Nr + j];
          sincosf(ph, &sn, &cs);
        }
        const float qlo = ulo * cs - uhi * sn, qhi = uhi * cs + ulo * sn;
        const float klo = wlo * cs - whi * sn, khi = whi * cs + wlo * sn;
        const float dqlo = dqs[i * (N + 1) + j], dqhi = dqs[i * (N + 1) + j + H2];
        const float dhlo = dks[i * (N + 1) + j], dhhi = dks[i * (N + 1) + j + H2];
        float dklo = dhlo * scl[i], dkhi = dhhi * scl[i];
        if (t == L - 1 && a.dfinal_k) {
          dklo += a.dfinal_k[bh * N + j];
          dkhi += a.dfinal_k[bh * N + j + H2];
        }
        // R^T = R(-phi): pull the cotangents back through the rotation.
        const float dulo = dqlo * cs + dqhi * sn + dgm * wlo;
        const float duhi = dqhi * cs - dqlo * sn + dgm * whi;
        const float dwlo = dklo * cs + dkhi * sn + dgm * ulo;
        const float dwhi = dkhi * cs - dklo * sn + dgm * uhi;
        dsp += dhlo * klo + dhhi * khi;
        dap += qlo * dqlo + qhi * dqhi - (ks[i * (N + 1) + j] * dhlo + ks[i * (N + 1) + j + H2] * dhhi);
        if (j < Nr) {
          const float dp = (dqhi * qlo - dqlo * qhi) + (dkhi * klo - dklo * khi);
          if (a.raw) dph[i * H2 + j] = dp;
          else a.dphi[(bh * L + t) * Nr + j] = dp;
        }
        float* dqrow = a.dq + ((size_t)b * L + t) * N;
        float* dkrow = a.dk + ((size_t)b * L + t) * N;
        atomicAdd(dqrow + j, dulo);
        atomicAdd(dqrow + j + H2, duhi);
        atomicAdd(dkrow + j, dwlo);
        atomicAdd(dkrow + j + H2, dwhi);
        atomicAdd(dqb + j, dulo);
        atomicAdd(dqb + j + H2, duhi);
        atomicAdd(dkb + j, dwlo);
        atomicAdd(dkb + j + H2, dwhi);
      }
      dsp = warp_sum(dsp);
      dap = warp_sum(dap);
      if (lane == 0) {
        dsc[i] = dsp;
        dA[i] = dap;
      }
    }
    __syncthreads();

    // ---- dtheta suffix sums and the angle gradient (raw boundary; reference.py:152-157)
    if (a.raw) {
      for (int r = tid; r < Nr; r += NT) {
        float run = dcarry[r];
        for (int i = CS - 1; i >= 0; --i) {
          const int t = t0 + i;
          run += dph[i * H2 + r];
          const float th = tanhf(a.angles[(size_t)b * a.ang_st.b + (size_t)t * a.ang_st.l + r]);
          atomicAdd(a.dangles + ((size_t)b * L + t) * Nr + r, run * kPi * dtv[i] * (1.f - th * th));
          dph[i * H2 + r] = run * th * kPi;  // this angle's share of d dt_t
        }
        dcarry[r] = run;
      }
      __syncthreads();
      for (int i = warp; i < CS; i += NT / 32) {
        float x = 0.f;
        for (int r = lane; r < Nr; r += 32) x += dph[i * H2 + r];
        x = warp_sum(x);
        if (lane == 0) dth[i] = x;
      }
      __syncthreads();
    }

    // ---- per-token scalar gradients -------------------------------------------------
    if (warp == 0) {
      // dadt = suffix_sum(dA) + A_last term (kernel_bwd.py:264-285)
      const float x = lane < CS ? dA[lane] : 0.f;
      const float incl = warp_inclusive_scan(x);
      const float tot = __shfl_sync(0xffffffffu, incl, 31);
      const float dadt = tot - incl + x + alast_term;
      if (lane < CS) {
        const int i = lane, t = t0 + i;
        const float dgam = dqkd[i] * uw[i];
        if (a.d_skip) dD_acc += dqkd[i];
        if (!a.raw) {
          a.dadt[bh * L + t] = dadt;
          a.dgamma[bh * L + t] = dgam;
          a.dscale[bh * L + t] = dsc[i];
        } else {
          // autodiff of preprocess (reference.py:104-131, 186-199)
          const float dt = dtv[i], lam = lamv[i];
          const float dsp = i > 0 ? dsc[i - 1] : 0.f;  // i == 0 gets it from the earlier sub-chunk's step
          const float ddt = (dgam + dsc[i]) * lam + dsp * (1.f - lam) + dadt * av[i] + dth[i];
          const float dlam = (dgam + dsc[i]) * dt - dsp * dt;
          const size_t o = (size_t)b * a.raw_st.b + (size_t)t * a.raw_st.l + (size_t)h * a.raw_st.h;
          const float sg = sigmoidf_(a.dt_raw[o] + a.dt_bias[h]);
          const size_t od = ((size_t)b * L + t) * H + h;
          a.ddt_raw[od] = ddt * sg;
          ddtb_acc += ddt * sg;
          const float ar = a.a_raw[o];
          const bool open = -heavy_tail(ar) < -a.a_floor;
          const float htp = ar >= 0.f ? 1.f : 1.f / ((1.f - ar) * (1.f - ar));
          a.da_raw[od] = open ? -(dadt * dt) * htp : 0.f;
          a.dtrap_raw[od] = dlam * lam * (1.f - lam);
          if (i == CS - 1 && t + 1 < L) {
            // scale_t reaches dt/lam of t+1, the first token of the next sub-chunk,
            // whose gradients were written one step earlier by this block.
            const float dtn = dtv[CS], lamn = lamv[CS];
            const size_t on = o + a.raw_st.l;
            const size_t odn = od + H;
            const float sgn = sigmoidf_(a.dt_raw[on] + a.dt_bias[h]);
            const float e_dt = dsc[i] * (1.f - lamn) * sgn;
            a.ddt_raw[odn] += e_dt;
            ddtb_acc += e_dt;
            a.dtrap_raw[odn] += -dsc[i] * dtn * lamn * (1.f - lamn);
          }
        }
      }
    }
    __syncthreads();
  }

  // ======================= seeds and per-head reductions ==========================
  if (a.seed_ssm) {
    // S0 = seed_ssm + coef v_prev k_prev^T  (kernel_bwd.py:636-646)
    double dcoef_d = 0.0;  // a long cancelling sum: accumulate in double
    for (int idx = tid; idx < P * N; idx += NT) {
      const int p = idx / N, n = idx % N;
      const float g = Gs[p * (N + 1) + n];
      a.dseed_ssm[bh * P * N + idx] = g;
      dcoef_d += (double)g * a.seed_v[bh * P + p] * a.seed_k[bh * N + n];
    }
    float dcoef = (float)dcoef_d;
    for (int n = tid; n < N; n += NT) {
      float x = 0.f;
      for (int p = 0; p < P; ++p) x += Gs[p * (N + 1) + n] * a.seed_v[bh * P + p];
      a.dseed_k[bh * N + n] = coef * x;
    }
    for (int p = tid; p < P; p += NT) {
      float x = 0.f;
      for (int n = 0; n < N; ++n) x += Gs[p * (N + 1) + n] * a.seed_k[bh * N + n];
      a.dseed_v[bh * P + p] = coef * x;
    }
    dcoef = block_sum(dcoef, red);
    if (tid == 0) {
      if (!a.raw) {
        a.dseed_coef[bh] = dcoef;
      } else {
        const size_t o = (size_t)b * a.raw_st.b + (size_t)h * a.raw_st.h;
        const size_t od = (size_t)b * L * H + h;
        const float sg = sigmoidf_(a.dt_raw[o] + a.dt_bias[h]);
        const float e_dt = dcoef * (1.f - lam0) * sg;
        a.ddt_raw[od] += e_dt;
        ddtb_acc += e_dt;
        a.dtrap_raw[od] += -dcoef * dt0 * lam0 * (1.f - lam0);
      }
    }
  }
  if (a.raw && a.dseed_phi)
    for (int r = tid; r < Nr; r += NT) a.dseed_phi[bh * Nr + r] = dcarry[r];
  __syncthreads();
  for (int n = tid; n < N; n += NT) {
    atomicAdd(a.dq_bias + h * N + n, dqb[n]);
    atomicAdd(a.dk_bias + h * N + n, dkb[n]);
  }
  const float dD_tot = block_sum(dD_acc, red);
  const float ddtb_tot = block_sum(ddtb_acc, red);
  if (tid == 0) {
    if (a.d_skip) atomicAdd(a.dd_skip + h, dD_tot);
    if (a.raw) atomicAdd(a.ddt_bias + h, ddtb_tot);
  }
}

}  // namespace m3
