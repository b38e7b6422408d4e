// Generic (CUDA-core) chunked forward scan.  One CTA per (b, h) walks its sequence in
// 64-token sub-chunks, carrying the fp32 state in shared memory.  Covers every
// supported (N, P), both I/O dtypes and both matmul policies; the bf16 policy rounds
// the same operands the reference kernel does (mamba3_pallas/kernel_fwd.py:139-187),
// so its contractions are exact bf16 x bf16 products accumulated in fp32.
//
// Per sub-chunk (local A_t = sum_{i<=t} adt_i log2 e), following
// mamba3_pallas/kernel_fwd.py:113-187 and reference.py:382-410:
//   ybar = exp2(A) (q~ S^T) + tril_strict(q~ khat^T exp2(min(A_i - A_j, 0))) v
//          + (D + gamma u.w) v
//   S   <- exp2(A_last) S + (v exp2(A_last - A))^T khat
// The sub-chunk length is an internal tiling choice: the recurrence is chunk-invariant
// (convert.py:219-222 of the reference states the same), only rounding differs.
#pragma once

#include "m3_chunk_common.cuh"

namespace m3 {

constexpr int kSub = 64;  // tokens per internal sub-chunk

template <int N, int P>
struct FwdSmem {
  static constexpr int H2 = N / 2;
  static constexpr int qs = 0;                              // kSub x (N+1)
  static constexpr int ks = qs + kSub * (N + 1);            // kSub x (N+1)
  static constexpr int vs = ks + kSub * (N + 1);            // kSub x (P+1)
  static constexpr int vsc = vs + kSub * (P + 1);           // kSub x (P+1)
  static constexpr int st = vsc + kSub * (P + 1);           // P x (N+1)
  static constexpr int sS = st + P * (N + 1);               // kSub x (kSub+1)
  static constexpr int phis = sS + kSub * (kSub + 1);       // kSub x H2
  static constexpr int A = phis + kSub * H2;                // kSub
  static constexpr int gam = A + kSub;                      // kSub
  static constexpr int scl = gam + kSub;                    // kSub
  static constexpr int dg = scl + kSub;                     // kSub
  static constexpr int adt = dg + kSub;                     // kSub
  static constexpr int dtv = adt + kSub;                    // kSub + 1
  static constexpr int lamv = dtv + kSub + 1;               // kSub + 1
  static constexpr int carry = lamv + kSub + 1;             // H2
  static constexpr int part = carry + H2;                   // kSimtThreads
  static constexpr int av = part + kSimtThreads;            // kSub
  static constexpr int total = av + kSub;
  static constexpr size_t bytes = sizeof(float) * (size_t)total;
};

template <int N, int P, typename T, bool MMB>
__global__ void __launch_bounds__(kSimtThreads) fwd_simt_kernel(const M3FwdArgs a) {
  using S = FwdSmem<N, P>;
  constexpr int NT = kSimtThreads, H2 = N / 2;
  extern __shared__ float sm[];
  float* qs = sm + S::qs;
  float* ks = sm + S::ks;
  float* vs = sm + S::vs;
  float* vsc = sm + S::vsc;
  float* st = sm + S::st;
  float* sS = sm + S::sS;
  float* phis = sm + S::phis;
  float* A = sm + S::A;
  float* gam = sm + S::gam;
  float* scl = sm + S::scl;
  float* dg = sm + S::dg;
  float* adts = sm + S::adt;
  float* dtv = sm + S::dtv;
  float* lamv = sm + S::lamv;
  float* carry = sm + S::carry;
  float* part = sm + S::part;
  float* av = sm + S::av;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.dims.nheads, L = a.dims.seqlen, Nr = a.dims.n_angles;
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int bh = b * H + h;
  const T* q = (const T*)a.q;
  const T* k = (const T*)a.k;
  const T* v = (const T*)a.v;
  const T* z = (const T*)a.z;
  T* y = (T*)a.y;
  const float Dh = a.d_skip ? a.d_skip[h] : 0.f;
  const int chunk_sub = a.dims.chunk / kSub;

  // ---- state init, seeded with the carried (k, v) pair's beta term --------------
  // (kernel_fwd.py:96-111, reference.py:353-360)
  float coef = 0.f;
  if (a.seed_ssm) {
    if (a.raw) {
      const float dt0 = softplusf(a.dt_raw[b * a.raw_st.b + h * a.raw_st.h] + a.dt_bias[h]);
      const float lam0 = sigmoidf_(a.trap_raw[b * a.raw_st.b + h * a.raw_st.h]);
      coef = dt0 * (1.f - lam0);
    } else {
      coef = a.seed_coef[bh];
    }
  }
  for (int idx = tid; idx < P * N; idx += NT) {
    const int p = idx / N, n = idx % N;
    float s0 = 0.f;
    if (a.seed_ssm)
      s0 = a.seed_ssm[(size_t)bh * P * N + idx] + coef * a.seed_v[(size_t)bh * P + p] * a.seed_k[(size_t)bh * N + n];
    st[p * (N + 1) + n] = s0;
  }
  if (a.raw)
    for (int r = tid; r < Nr; r += NT) carry[r] = a.seed_phi ? a.seed_phi[(size_t)bh * Nr + r] : 0.f;
  __syncthreads();

  const int nsub = L / kSub;
  for (int sc = 0; sc < nsub; ++sc) {
    const int t0 = sc * kSub;
    prep_scalars<kSub, NT>(a, b, h, t0, adts, gam, scl, A, dtv, lamv, av);
    if (a.raw) phi_scan<kSub, NT>(a, b, t0, dtv, phis, H2, carry, part);

    // ---- bias, rotate, scale (kernel_fwd.py:125-141) -------------------------------
    for (int i = warp; i < kSub; i += NT / 32) {
      const int t = t0 + i;
      const T* qrow = q + (size_t)b * a.q_st.b + (size_t)t * a.q_st.l;
      const T* krow = k + (size_t)b * a.k_st.b + (size_t)t * a.k_st.l;
      const float sc_t = scl[i];
      float uw = 0.f;
      for (int j = lane; j < H2; j += 32) {
        const float ulo = ld(qrow + j) + a.q_bias[h * N + j];
        const float uhi = ld(qrow + j + H2) + a.q_bias[h * N + j + H2];
        const float wlo = ld(krow + j) + a.k_bias[h * N + j];
        const float whi = ld(krow + j + H2) + a.k_bias[h * N + j + H2];
        uw += ulo * wlo + uhi * whi;
        float qlo = ulo, qhi = uhi, klo = wlo, khi = whi;
        if (j < Nr) {
          const float ph = a.raw ? phis[i * H2 + j] : a.phi[((size_t)bh * L + t) * Nr + j];
          float sn, cs;
          sincosf(ph, &sn, &cs);
          qlo = ulo * cs - uhi * sn;
          qhi = uhi * cs + ulo * sn;
          klo = wlo * cs - whi * sn;
          khi = whi * cs + wlo * sn;
        }
        qs[i * (N + 1) + j] = mmr<MMB>(qlo);
        qs[i * (N + 1) + j + H2] = mmr<MMB>(qhi);
        ks[i * (N + 1) + j] = mmr<MMB>(klo * sc_t);
        ks[i * (N + 1) + j + H2] = mmr<MMB>(khi * sc_t);
        if (t == L - 1) {  // final k is rotated but unscaled (kernel_fwd.py:192-201)
          a.final_k[(size_t)bh * N + j] = klo;
          a.final_k[(size_t)bh * N + j + H2] = khi;
        }
      }
      uw = warp_sum(uw);
      if (lane == 0) dg[i] = uw * gam[i] + Dh;
    }
    for (int idx = tid; idx < kSub * P; idx += NT) {
      const int i = idx / P, p = idx % P;
      vs[i * (P + 1) + p] = ld(v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h + (size_t)(t0 + i) * a.v_st.l + p);
    }
    __syncthreads();

    // ---- masked intra-chunk scores (kernel_fwd.py:155-163) ---------------------------
    {
      using TL = Tile<kSub, kSub, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
#pragma unroll 4
      for (int n = 0; n < N; ++n) {
        float qa[TL::TM], kb[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) qa[i] = qs[(ty + TL::RY * i) * (N + 1) + n];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) kb[j] = ks[(tx + TL::RX * j) * (N + 1) + n];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(qa[i], kb[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i)
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          const int ti = ty + TL::RY * i, sj = tx + TL::RX * j;
          float val = 0.f;
          if (ti > sj) val = mmr<MMB>(acc[i][j] * exp2f(fminf(A[ti] - A[sj], 0.f)));
          sS[ti * (kSub + 1) + sj] = val;
        }
    }
    __syncthreads();

    // ---- output: inter + intra + diagonal/skip, gate (kernel_fwd.py:143-180) --------
    {
      using TL = Tile<kSub, P, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
#pragma unroll 4
      for (int n = 0; n < N; ++n) {
        float qa[TL::TM], sb[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) qa[i] = qs[(ty + TL::RY * i) * (N + 1) + n];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) sb[j] = mmr<MMB>(st[(tx + TL::RX * j) * (N + 1) + n]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(qa[i], sb[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const float e = exp2f(A[ty + TL::RY * i]);
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) acc[i][j] *= e;
      }
#pragma unroll 4
      for (int s = 0; s < kSub; ++s) {
        float sa[TL::TM], vb[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) sa[i] = sS[(ty + TL::RY * i) * (kSub + 1) + s];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) vb[j] = mmr<MMB>(vs[s * (P + 1) + tx + TL::RX * j]);
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(sa[i], vb[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < TL::TM; ++i) {
        const int ti = ty + TL::RY * i, t = t0 + ti;
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) {
          const int p = tx + TL::RX * j;
          float o = acc[i][j] + dg[ti] * vs[ti * (P + 1) + p];
          if (a.ybar) a.ybar[((size_t)bh * L + t) * P + p] = o;
          if (z) {
            const float zz = ld(z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)t * a.z_st.l + p);
            o *= zz * sigmoidf_(zz);
          }
          stg<T>(y + (size_t)b * a.y_st.b + (size_t)h * a.y_st.h + (size_t)t * a.y_st.l + p, o);
        }
      }
    }
    // chunk-start state residual (kernel_fwd.py:174) and the decayed v of the update
    if (a.chunk_states && sc % chunk_sub == 0) {
      const int c = sc / chunk_sub, nc = L / a.dims.chunk;
      const size_t base = (((size_t)bh * nc) + c) * P * N;
      for (int idx = tid; idx < P * N; idx += NT) {
        const float s0 = st[(idx / N) * (N + 1) + idx % N];
        if (a.chunk_states_dtype == M3_DTYPE_BF16)
          ((__nv_bfloat16*)a.chunk_states)[base + idx] = __float2bfloat16_rn(s0);
        else
          ((float*)a.chunk_states)[base + idx] = s0;
      }
    }
    {
      const float Al = A[kSub - 1];
      for (int idx = tid; idx < kSub * P; idx += NT) {
        const int i = idx / P, p = idx % P;
        vsc[i * (P + 1) + p] = mmr<MMB>(vs[i * (P + 1) + p] * exp2f(Al - A[i]));
      }
    }
    __syncthreads();

    // ---- advance the state (kernel_fwd.py:182-187) -----------------------------------
    {
      using TL = Tile<P, N, NT>;
      const int tx = tid % TL::RX, ty = tid / TL::RX;
      float acc[TL::TM][TL::TN] = {};
#pragma unroll 4
      for (int s = 0; s < kSub; ++s) {
        float va[TL::TM], kb[TL::TN];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i) va[i] = vsc[s * (P + 1) + ty + TL::RY * i];
#pragma unroll
        for (int j = 0; j < TL::TN; ++j) kb[j] = ks[s * (N + 1) + tx + TL::RX * j];
#pragma unroll
        for (int i = 0; i < TL::TM; ++i)
#pragma unroll
          for (int j = 0; j < TL::TN; ++j) acc[i][j] = fmaf(va[i], kb[j], acc[i][j]);
      }
      const float eAl = exp2f(A[kSub - 1]);
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

  // ---- final state (kernel_fwd.py:189-201) ---------------------------------------------
  for (int idx = tid; idx < P * N; idx += NT) a.final_ssm[(size_t)bh * P * N + idx] = st[(idx / N) * (N + 1) + idx % N];
  for (int p = tid; p < P; p += NT)
    a.final_v[(size_t)bh * P + p] = ld(v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h + (size_t)(L - 1) * a.v_st.l + p);
  if (a.final_phi) {
    for (int r = tid; r < Nr; r += NT)
      a.final_phi[(size_t)bh * Nr + r] = a.raw ? phis[(kSub - 1) * H2 + r] : a.phi[((size_t)bh * L + L - 1) * Nr + r];
  }
}

}  // namespace m3
