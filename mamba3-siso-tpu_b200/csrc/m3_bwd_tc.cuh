// Tensor-core (tcgen05 / TMEM) backward for the production shape: bf16 I/O and bf16
// matmul operands, N = 128, P = 64, 128-token chunks, raw (fused-preprocess) boundary.
//
// The chunk-start states are recomputed first by the forward kernel's states-only mode
// (bf16 tiles in the layout used below, plus the rotary-angle carries); nothing is read
// from the forward's residuals.  Then one CTA (256 threads) per (b, h) walks the chunks in
// reverse with the adjoint G of the chunk's end state in registers (fp32), per chunk
// (kernel_bwd.py:10-34, 103-355; A_t the prefix of adt log2 e inside the chunk):
//
//   round 1  Wm  = q~ khat^T         dM = g v^T            Yi = q~ S^T
//   CUDA     one decay mask exp2(min(A_i - A_j, 0)), strict lower triangle, for both
//   round 2  Ya  = Wm v              dv_a = Wm^T g         dv_b = khat G^T
//            dq~ = dM khat + (e^A g) S                      dkhat = dM^T q~ + vd G
//   CUDA     ybar -> dz, dv, rotation pullback (fp32, recomputed angles), head-summed
//            dq / dk, bias and angle adjoints, the autodiff of the preprocessing
//   round 3  dG^T = q~^T (e^A g);    G <- exp2(A_last) G + dG
//
// with vd = v exp2(A_last - A) and e^A g folded into bf16 operands.  The A_last term of
// dadt is sum(G o S_next): every occurrence of A_last scales the chunk's end state
// S_next = exp2(A_last) S + vd^T khat, so its adjoint is exactly that inner product.
#pragma once

#include "m3_chunk_common.cuh"
#include "m3_fwd_tc.cuh"
#include "m3_umma.cuh"

namespace m3 {
namespace tcb {

using tc::bf16hi;
using tc::bf16lo;
using tc::pack8;

constexpr int kN = 128, kP = 64, kC = 128, kThreads = 256;
// tile offsets (bytes); everything from kK on is free once round 2 has completed
constexpr uint32_t kQ = 0, kGe = 32768, kSt = 49152, kGt = 65536, kK = 81920, kWm = 114688, kDM = 147456,
                   kV = 180224, kVd = 196608, kG = 212992, kTiles = 229376;
// scratch inside tiles while they are not live
constexpr uint32_t kScrDt = kWm, kScrScl = kWm + 512, kScrUw = kWm + 1024, kScrQkd = kWm + 5120;   // prep
constexpr uint32_t kScrPart = kGt, kScrDtb = kGt + 2048, kScrTh = kGt + 2560;                     // epilogue
constexpr uint32_t kAng = kDM;  // this chunk's raw angles [128][64] fp32, 16-byte chunks XOR-swizzled by row (P0-P1)
constexpr uint32_t kStDv = kDM, kStDz = kV;  // dv / dz rows [128][64] fp32 on their way out (after round 2)
constexpr uint32_t kDu = kK, kDw = kDM;  // fp32 [128][128] each, column index XOR-swizzled by row

// per-sequence global scratch: phi then dphi [64][128] fp32, tanh(angles) [64][128] fp32,
// raw q and k rows as 16-byte column groups [16][128] (all token-contiguous, so coalesced)
constexpr size_t kScratchBytes = 2 * 64 * kC * sizeof(float) + 2 * 16 * kC * 16;

struct Small {
  uint64_t mbar[3];
  uint32_t tmem;
  float alast;
  float wtot[4];
  float red[8];
  float A[128];
  float bias[2 * kN];  // the head's q_bias, k_bias
};
constexpr size_t kSmemBytes = kTiles + 2048 + 1024;  // tiles + Small (<= 2 KB) + alignment slack
static_assert(sizeof(Small) <= 2048, "Small must fit its 2 KB slot");

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Sum over the CTA (every thread gets the total).
__device__ __forceinline__ float cta_sum(float x, Small* sm_) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  x = warp_sum(x);
  __syncthreads();
  if (lane == 0) sm_->red[warp] = x;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += sm_->red[w];
  __syncthreads();
  return t;
}

// Inclusive suffix scan over the 32 lanes of a warp (lane l gets sum of lanes >= l).
__device__ __forceinline__ float warp_suffix_scan(float x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += y;
  }
  return x;
}

// RAW: the fused raw boundary (dt / A / trap streams and angles in, their gradients out);
// otherwise the reference's preprocessed boundary (adt, gamma, scale, phi in; dadt,
// dgamma, dscale, dphi, dseed_coef out: kernel_bwd.py:534-669).
template <bool RAW>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_tc_kernel(const M3BwdArgs a, const uint8_t* __restrict__ tiles, const float* __restrict__ phis,
                  float* __restrict__ scratch) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  Small* ss = reinterpret_cast<Small*>(sm + kTiles);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = tid & 127, half = tid >> 7;  // token / state row and column half
  const int H = a.dims.nheads, L = a.dims.seqlen, Nr = a.dims.n_angles;
  const int seq = blockIdx.x, b = seq / H, h = seq % H;
  const size_t bh = (size_t)seq;
  const int nchunk = L / kC;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
  const __nv_bfloat16* q = (const __nv_bfloat16*)a.q;
  const __nv_bfloat16* k = (const __nv_bfloat16*)a.k;
  const __nv_bfloat16* v = (const __nv_bfloat16*)a.v;
  const __nv_bfloat16* z = (const __nv_bfloat16*)a.z;
  const __nv_bfloat16* dy = (const __nv_bfloat16*)a.dy;
  const float Dh = a.d_skip ? a.d_skip[h] : 0.f;
  const float dtb = RAW ? a.dt_bias[h] : 0.f;
  float* phs = scratch + (size_t)blockIdx.x * (kScratchBytes / sizeof(float));  // [64][128]: phi, then dphi
  float* ths = phs + 64 * kC;                                                     // [64][128]: tanh(angles)
  uint4* rqs = reinterpret_cast<uint4*>(ths + 64 * kC);                            // [16][128]: raw q
  uint4* rks = rqs + 16 * kC;                                                      // [16][128]: raw k

  if (warp == 0) umma::tmem_alloc(&ss->tmem, 512);
  ss->bias[tid] = tid < kN ? a.q_bias[h * kN + tid] : a.k_bias[h * kN + tid - kN];
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) umma::mbar_init(&ss->mbar[i], 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = ss->tmem;
  const uint32_t aQ = umma::smem_u32(sm + kQ), aGe = umma::smem_u32(sm + kGe), aSt = umma::smem_u32(sm + kSt);
  const uint32_t aGt = umma::smem_u32(sm + kGt), aK = umma::smem_u32(sm + kK), aWm = umma::smem_u32(sm + kWm);
  const uint32_t aDM = umma::smem_u32(sm + kDM), aV = umma::smem_u32(sm + kV), aVd = umma::smem_u32(sm + kVd);
  const uint32_t aG = umma::smem_u32(sm + kG);
  bool ok = true;

  // ---- adjoint of the final state: G^T[n = t][p = 32 half + i] (fp32, registers) ------
  float G[32];
#pragma unroll
  for (int i = 0; i < 32; ++i)
    G[i] = a.dfinal_ssm ? a.dfinal_ssm[(bh * kP + 32 * half + i) * kN + t] : 0.f;
  float dcarry8[8];  // adjoint of this warp's rotary-angle carry
#pragma unroll
  for (int r = 0; r < 8; ++r)
    dcarry8[r] = (RAW && a.dfinal_phi && 8 * warp + r < Nr) ? a.dfinal_phi[bh * Nr + 8 * warp + r] : 0.f;
  {
    // A_last term of the last chunk: sum(G o S_final); S_final is tile `nchunk`
    const uint8_t* sf = tiles + (bh * (nchunk + 1) + nchunk) * 16384u;
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 u = *reinterpret_cast<const uint4*>(sf + umma::sw128_off(t, 4 * half + j));
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) part += G[8 * j + 2 * e] * bf16lo(w4[e]) + G[8 * j + 2 * e + 1] * bf16hi(w4[e]);
    }
    const float tot = cta_sum(part, ss);
    if (tid == 0) ss->alast = tot;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(sm + kGt + umma::sw128_off(t, 4 * half + j)) = pack8(G + 8 * j);
  }
  float2 bias01 = f2s(0.f), bias23 = f2s(0.f);  // bias column sums (see the row pass)
  float dD_acc = 0.f, ddtb_acc = 0.f;
  __syncthreads();

  // Raw tiles of chunk cc (cp.async).  k, v and the angles go to tiles that are free once the
  // previous chunk's head-sum pass has read its rows; q and the state tile once its round 3
  // and A_last term are done.
  auto prefetch_kva = [&](int cc) {
    const int tb = cc * kC;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int i = tid + kThreads * m;
      const int row = i >> 4, c16 = i & 15;
      const uint32_t dst = (c16 >> 3) * 16384u + umma::sw128_off(row, c16 & 7);
      umma::cp_async16(aK + dst, k + (size_t)b * a.k_st.b + (size_t)(tb + row) * a.k_st.l + c16 * 8);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i = tid + kThreads * m;
      const int row = i >> 3, c8 = i & 7;
      umma::cp_async16(aV + umma::sw128_off(row, c8),
                       v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h + (size_t)(tb + row) * a.v_st.l + c8 * 8);
    }
    // dy into the g tile (g is computed in place) and z into the vd tile (free until P2)
    const __nv_bfloat16* dyb = dy + (size_t)b * a.dy_st.b + (size_t)h * a.dy_st.h + (size_t)tb * a.dy_st.l;
    const __nv_bfloat16* zb = z ? z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)tb * a.z_st.l : nullptr;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i = tid + kThreads * m;
      const int row = i >> 3, c8 = i & 7;
      umma::cp_async16(aG + umma::sw128_off(row, c8), dyb + (size_t)row * a.dy_st.l + c8 * 8);
      if (zb) umma::cp_async16(aVd + umma::sw128_off(row, c8), zb + (size_t)row * a.z_st.l + c8 * 8);
    }
    const int n4 = Nr >> 2;  // 16-byte chunks per angle row
    const uint32_t aAng = umma::smem_u32(sm + kAng);
    for (int i = tid; i < kC * n4; i += kThreads) {
      const int row = i / n4, c4 = i - row * n4;
      umma::cp_async16(aAng + row * 256 + 16 * (c4 ^ (row & 15)),
                       RAW ? a.angles + (size_t)b * a.ang_st.b + (size_t)(tb + row) * a.ang_st.l + 4 * c4
                           : a.phi + (bh * L + tb + row) * Nr + 4 * c4);
    }
    umma::cp_async_commit();
  };
  auto prefetch_qst = [&](int cc) {
    const int tb = cc * kC;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int i = tid + kThreads * m;
      const int row = i >> 4, c16 = i & 15;
      const uint32_t dst = (c16 >> 3) * 16384u + umma::sw128_off(row, c16 & 7);
      umma::cp_async16(aQ + dst, q + (size_t)b * a.q_st.b + (size_t)(tb + row) * a.q_st.l + c16 * 8);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i = tid + kThreads * m;
      umma::cp_async16(aSt + 16u * i, tiles + (bh * (nchunk + 1) + cc) * 16384u + 16u * i);
    }
    umma::cp_async_commit();
  };
  prefetch_kva(nchunk - 1);
  prefetch_qst(nchunk - 1);

#ifdef M3_TC_TIMING
  const int ltid = tid;
  long long tmark_ = clock64();
#endif
  for (int c = nchunk - 1; c >= 0 && ok; --c) {
    const int t0 = c * kC, tg = t0 + t;
    const float alast = ss->alast;
    // ---- P0: per-token scalars, g and e^A g (this chunk's tiles were prefetched) ---------
    const size_t ro = (size_t)b * a.raw_st.b + (size_t)tg * a.raw_st.l + (size_t)h * a.raw_st.h;
    float dt = 0.f, lam = 0.f, ar = 0.f, av = 0.f, dtn = 0.f, lamn = 0.f, gam, scl, adtv;
    if constexpr (RAW) {
      dt = softplusf(a.dt_raw[ro] + dtb);
      lam = sigmoidf_(a.trap_raw[ro]);
      ar = a.a_raw[ro];
      av = fminf(-heavy_tail(ar), -a.a_floor);
      dtn = __shfl_down_sync(0xffffffffu, dt, 1);
      lamn = __shfl_down_sync(0xffffffffu, lam, 1);
      if (lane == 31) {
        dtn = tg + 1 < L ? softplusf(a.dt_raw[ro + a.raw_st.l] + dtb) : 0.f;
        lamn = tg + 1 < L ? sigmoidf_(a.trap_raw[ro + a.raw_st.l]) : 0.f;
      }
      gam = dt * lam;
      scl = gam + dtn * (1.f - lamn);
      adtv = av * dt;
    } else {  // preprocessed boundary: (B, H, L) streams
      adtv = a.adt[bh * L + tg];
      gam = a.gamma[bh * L + tg];
      scl = a.scale[bh * L + tg];
    }
    const float incl = warp_inclusive_scan(adtv * kLog2e);
    if (half == 0 && lane == 31) ss->wtot[warp & 3] = incl;
    if (half == 0) {
      reinterpret_cast<float*>(sm + kScrDt)[t] = dt;
      reinterpret_cast<float*>(sm + kScrScl)[t] = scl;
    }
    umma::cp_async_wait_all();  // this chunk's prefetched tiles (dy / z included)
    __syncthreads();
    float A = incl;
    for (int w = 0; w < (warp & 3); ++w) A += ss->wtot[w];
    const float Alast = ss->wtot[0] + ss->wtot[1] + ss->wtot[2] + ss->wtot[3];
    const float eA = exp2f(A), erev = exp2f(Alast - A);
    if (half == 0) ss->A[t] = A;
    // g = dy silu(z) for this thread's 32 columns; bf16 g and e^A g tiles (rows = token)
    float gv[32];
    {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t so = umma::sw128_off(t, 4 * half + j);
        const uint4 u = *reinterpret_cast<const uint4*>(sm + kG + so);
        const uint32_t d4[4] = {u.x, u.y, u.z, u.w};
        uint32_t z4[4] = {0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u};
        if (z) {
          const uint4 w = *reinterpret_cast<const uint4*>(sm + kVd + so);
          z4[0] = w.x; z4[1] = w.y; z4[2] = w.z; z4[3] = w.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 g2 = bf2f(d4[e]);
          if (z) {
            const float2 z2 = bf2f(z4[e]);
            g2 = mul2(g2, mul2(z2, sigmoid2(z2)));
          }
          gv[8 * j + 2 * e] = g2.x;
          gv[8 * j + 2 * e + 1] = g2.y;
        }
      }
      float ge[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) ge[i] = gv[i] * eA;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        *reinterpret_cast<uint4*>(sm + kG + umma::sw128_off(t, 4 * half + j)) = pack8(gv + 8 * j);
        *reinterpret_cast<uint4*>(sm + kGe + umma::sw128_off(t, 4 * half + j)) = pack8(ge + 8 * j);
      }
    }
    umma::cp_async_wait_all();
    __syncthreads();
    M3_TC_MARK(8);

    // ---- P1: cumulative angles (from the recorded carry) and rotation; phi to scratch ----
    // warp g owns rotary pairs 8g .. 8g+7; lane l the token pairs (2l, 2l+1) + 64 i
    {
      const float* dts = reinterpret_cast<const float*>(sm + kScrDt);
      const float* scls = reinterpret_cast<const float*>(sm + kScrScl);
      float* uws = reinterpret_cast<float*>(sm + kScrUw);
      const int g = warp;
      const bool grot = 8 * g < Nr;
      const float* qbp = ss->bias + 8 * g;
      const float* kbp = ss->bias + kN + 8 * g;
      float off[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) off[r] = (RAW && grot) ? phis[(bh * nchunk + c) * Nr + 8 * g + r] : 0.f;
#pragma unroll 1
      for (int i = 0; i < 2; ++i) {
        const int tb = 64 * i + 2 * lane;
        float ph[2][8];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int r = 0; r < 8; ++r) ph[j][r] = 0.f;
        if (grot) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int row = tb + j;
            const uint8_t* ap = sm + kAng + row * 256;
            const float4 lo = *reinterpret_cast<const float4*>(ap + 16 * ((2 * g) ^ (row & 15)));
            const float4 hi = *reinterpret_cast<const float4*>(ap + 16 * ((2 * g + 1) ^ (row & 15)));
            ph[j][0] = lo.x; ph[j][1] = lo.y; ph[j][2] = lo.z; ph[j][3] = lo.w;
            ph[j][4] = hi.x; ph[j][5] = hi.y; ph[j][6] = hi.z; ph[j][7] = hi.w;
          }
          if constexpr (RAW) {  // raw angles -> cumulative angles (the preprocessed boundary gives phi)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int r = 0; r < 8; ++r) ph[j][r] = tanh_acc(ph[j][r]);
#pragma unroll
          for (int r = 0; r < 8; ++r)
            *reinterpret_cast<float2*>(ths + (8 * g + r) * kC + tb) = f2(ph[0][r], ph[1][r]);
          const float2 w = mul2(*reinterpret_cast<const float2*>(dts + tb), f2s(kPi));
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const float x0 = ph[0][r] * w.x, x1 = ph[1][r] * w.y;
            const float inc = warp_inclusive_scan(x0 + x1);
            ph[1][r] = off[r] + inc;
            ph[0][r] = ph[1][r] - x1;
            off[r] += __shfl_sync(0xffffffffu, inc, 31);
          }
          }
#pragma unroll
          for (int r = 0; r < 8; ++r)
            *reinterpret_cast<float2*>(phs + (8 * g + r) * kC + tb) = f2(ph[0][r], ph[1][r]);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int tt = tb + j;
          float cs[8], sn[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            cs[r] = 1.f;
            sn[r] = 0.f;
            if (grot) sincos_wrapped(wrap_fast(ph[j][r]), &sn[r], &cs[r]);
          }
          const uint32_t soff = umma::sw128_off(tt, g);
          const uint4 uql = *reinterpret_cast<const uint4*>(sm + kQ + soff);
          const uint4 uqh = *reinterpret_cast<const uint4*>(sm + kQ + 16384 + soff);
          const uint4 ukl = *reinterpret_cast<const uint4*>(sm + kK + soff);
          const uint4 ukh = *reinterpret_cast<const uint4*>(sm + kK + 16384 + soff);
          rqs[g * kC + tt] = uql;  // raw rows for the pullback
          rqs[(8 + g) * kC + tt] = uqh;
          rks[g * kC + tt] = ukl;
          rks[(8 + g) * kC + tt] = ukh;
          const uint32_t ql[4] = {uql.x, uql.y, uql.z, uql.w}, qh[4] = {uqh.x, uqh.y, uqh.z, uqh.w};
          const uint32_t kl[4] = {ukl.x, ukl.y, ukl.z, ukl.w}, kh[4] = {ukh.x, ukh.y, ukh.z, ukh.w};
          const float2 sc = f2s(scls[tt]);
          uint32_t pq_lo[4], pq_hi[4], pk_lo[4], pk_hi[4];
          float2 uw2 = f2s(0.f);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 c2 = f2(cs[2 * e], cs[2 * e + 1]), s2 = f2(sn[2 * e], sn[2 * e + 1]);
            const float2 ns2 = f2(-sn[2 * e], -sn[2 * e + 1]);
            const float2 ulo = add2(bf2f(ql[e]), *reinterpret_cast<const float2*>(qbp + 2 * e));
            const float2 uhi = add2(bf2f(qh[e]), *reinterpret_cast<const float2*>(qbp + 64 + 2 * e));
            const float2 wlo = add2(bf2f(kl[e]), *reinterpret_cast<const float2*>(kbp + 2 * e));
            const float2 whi = add2(bf2f(kh[e]), *reinterpret_cast<const float2*>(kbp + 64 + 2 * e));
            uw2 = fma2(ulo, wlo, uw2);
            uw2 = fma2(uhi, whi, uw2);
            pq_lo[e] = f2bf(fma2(uhi, ns2, mul2(ulo, c2)));
            pq_hi[e] = f2bf(fma2(ulo, s2, mul2(uhi, c2)));
            pk_lo[e] = f2bf(mul2(fma2(whi, ns2, mul2(wlo, c2)), sc));
            pk_hi[e] = f2bf(mul2(fma2(wlo, s2, mul2(whi, c2)), sc));
          }
          *reinterpret_cast<uint4*>(sm + kQ + soff) = make_uint4(pq_lo[0], pq_lo[1], pq_lo[2], pq_lo[3]);
          *reinterpret_cast<uint4*>(sm + kQ + 16384 + soff) = make_uint4(pq_hi[0], pq_hi[1], pq_hi[2], pq_hi[3]);
          *reinterpret_cast<uint4*>(sm + kK + soff) = make_uint4(pk_lo[0], pk_lo[1], pk_lo[2], pk_lo[3]);
          *reinterpret_cast<uint4*>(sm + kK + 16384 + soff) = make_uint4(pk_hi[0], pk_hi[1], pk_hi[2], pk_hi[3]);
          uws[g * 128 + tt] = uw2.x + uw2.y;
        }
      }
    }
    M3_TC_MARK(9);
    // ---- P2: dqk_diag = g.v (halves), v exp2(A_last - A) tile -------------------------
    uint32_t vreg[16];
    {
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = *reinterpret_cast<const uint4*>(sm + kV + umma::sw128_off(t, 4 * half + j));
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
        float d[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          vreg[4 * j + e] = w4[e];
          const float v0 = bf16lo(w4[e]), v1 = bf16hi(w4[e]);
          part += gv[8 * j + 2 * e] * v0 + gv[8 * j + 2 * e + 1] * v1;
          d[2 * e] = v0 * erev;
          d[2 * e + 1] = v1 * erev;
        }
        *reinterpret_cast<uint4*>(sm + kVd + umma::sw128_off(t, 4 * half + j)) = pack8(d);
      }
      reinterpret_cast<float*>(sm + kScrQkd)[half * 128 + t] = part;
    }
    umma::fence_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    float uwt = 0.f;
    {
      const float* uws = reinterpret_cast<const float*>(sm + kScrUw);
#pragma unroll
      for (int gg = 0; gg < 8; ++gg) uwt += uws[gg * 128 + t];
    }
    const float dg = uwt * gam + Dh;
    const float qkd = reinterpret_cast<const float*>(sm + kScrQkd)[t] + reinterpret_cast<const float*>(sm + kScrQkd)[128 + t];

    M3_TC_MARK(10);
    // ---- round 1: Wm, dM, Yi ------------------------------------------------------------
    if (tid == 0) {
      constexpr uint32_t i_wm = umma::idesc_bf16(128, 128, false, false);
      constexpr uint32_t i_yi = umma::idesc_bf16(128, 64, false, true);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t km = (ks >> 2) * 16384u + (ks & 3) * 32u, mn = ks * 2048u;
        const uint64_t dq = umma::smem_desc(aQ + km, 16, 1024);
        umma::mma_bf16(tm + 0, dq, umma::smem_desc(aK + km, 16, 1024), i_wm, ks > 0);
        umma::mma_bf16(tm + 256, dq, umma::smem_desc(aSt + mn, 16384, 1024), i_yi, ks > 0);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma::mma_bf16(tm + 128, umma::smem_desc(aG + ks * 32u, 16, 1024), umma::smem_desc(aV + ks * 32u, 16, 1024),
                       i_wm, ks > 0);
      umma::commit(&ss->mbar[0]);
    }
    if (__syncthreads_or(!umma::mbar_wait(&ss->mbar[0], (nchunk - 1 - c) & 1))) {
      if (tid == 0) atomicExch(&g_m3_device_error, 11);
      ok = false;
      break;
    }
    umma::fence_after_sync();

    M3_TC_MARK(11);
    // ---- mask: one decay for Wm and dM, bf16 into their tiles (rows = token) -----------
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      float wv[32], mv[32];
      const int sb = 64 * half + 32 * cb;
      umma::tmem_ld32(tm + lane_base + sb, wv);
      umma::tmem_ld32(tm + lane_base + 128 + sb, mv);
      umma::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float w8[8], m8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int s = sb + 8 * j + e;
          float wd = 0.f, md = 0.f;
          if (s < t) {
            const float dec = ex2(fminf(A - ss->A[s], 0.f));
            wd = wv[8 * j + e] * dec;
            md = mv[8 * j + e] * dec;
          }
          w8[e] = wd;
          m8[e] = md;
        }
        *reinterpret_cast<uint4*>(sm + kWm + 16384 * half + umma::sw128_off(t, 4 * cb + j)) = pack8(w8);
        *reinterpret_cast<uint4*>(sm + kDM + 16384 * half + umma::sw128_off(t, 4 * cb + j)) = pack8(m8);
      }
    }
    umma::fence_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    M3_TC_MARK(12);
    // ---- round 2 ----------------------------------------------------------------------------
    if (tid == 0) {
      constexpr uint32_t i_ya = umma::idesc_bf16(128, 64, false, true);
      constexpr uint32_t i_dva = umma::idesc_bf16(128, 64, true, true);
      constexpr uint32_t i_dq = umma::idesc_bf16(128, 128, false, true);
      constexpr uint32_t i_dqb = umma::idesc_bf16(128, 128, false, false);
      constexpr uint32_t i_dk = umma::idesc_bf16(128, 128, true, true);
      constexpr uint32_t i_dvb = umma::idesc_bf16(128, 64, false, true);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t km = (ks >> 2) * 16384u + (ks & 3) * 32u, mn = ks * 2048u;
        umma::mma_bf16(tm + 0, umma::smem_desc(aWm + km, 16, 1024), umma::smem_desc(aV + mn, 16384, 1024), i_ya, ks > 0);
        umma::mma_bf16(tm + 64, umma::smem_desc(aWm + mn, 16384, 1024), umma::smem_desc(aG + mn, 16384, 1024), i_dva,
                       ks > 0);
        umma::mma_bf16(tm + 128, umma::smem_desc(aDM + km, 16, 1024), umma::smem_desc(aK + mn, 16384, 1024), i_dq,
                       ks > 0);
        umma::mma_bf16(tm + 320, umma::smem_desc(aDM + mn, 16384, 1024), umma::smem_desc(aQ + mn, 16384, 1024), i_dk,
                       ks > 0);
        umma::mma_bf16(tm + 448, umma::smem_desc(aK + km, 16, 1024), umma::smem_desc(aGt + mn, 16384, 1024), i_dvb,
                       ks > 0);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        umma::mma_bf16(tm + 128, umma::smem_desc(aGe + ks * 32u, 16, 1024), umma::smem_desc(aSt + ks * 32u, 16, 1024),
                       i_dqb, true);
        umma::mma_bf16(tm + 320, umma::smem_desc(aVd + ks * 32u, 16, 1024), umma::smem_desc(aGt + ks * 32u, 16, 1024),
                       i_dqb, true);
      }
      umma::commit(&ss->mbar[1]);
    }
    // dy / z rows for the dz epilogue: loads in flight while round 2 runs
    uint4 ud[4], uz[4];
    {
      const __nv_bfloat16* dyr = dy + (size_t)b * a.dy_st.b + (size_t)h * a.dy_st.h + (size_t)tg * a.dy_st.l + 32 * half;
      const __nv_bfloat16* zr = z ? z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)tg * a.z_st.l + 32 * half
                                  : nullptr;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ud[j] = *reinterpret_cast<const uint4*>(dyr + 8 * j);
        uz[j] = zr ? *reinterpret_cast<const uint4*>(zr + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if (__syncthreads_or(!umma::mbar_wait(&ss->mbar[1], (nchunk - 1 - c) & 1))) {
      if (tid == 0) atomicExch(&g_m3_device_error, 12);
      ok = false;
      break;
    }
    umma::fence_after_sync();

    M3_TC_MARK(13);
    // ---- epilogue: ybar -> dz, dv ---------------------------------------------------------
    float gq[32];  // g = dy silu(z) once more (same arithmetic as above) for dv's diagonal term
    {
      float yi[32], ya[32];
      umma::tmem_ld32(tm + lane_base + 256 + 32 * half, yi);
      umma::tmem_ld32(tm + lane_base + 32 * half, ya);
      umma::tmem_wait_ld();
      float* dzs = reinterpret_cast<float*>(sm + kStDz) + t * 64;  // float4 groups XOR-swizzled by row
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t d4[4] = {ud[j].x, ud[j].y, ud[j].z, ud[j].w}, z4[4] = {uz[j].x, uz[j].y, uz[j].z, uz[j].w};
        float o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * j + 2 * e;
          const float2 d2 = bf2f(d4[e]);
          float2 g2 = d2;
          if (z) {
            const float2 z2 = bf2f(z4[e]);
            const float2 sg = sigmoid2(z2);
            g2 = mul2(d2, mul2(z2, sg));
            const float2 ybar = fma2(f2s(dg), bf2f(vreg[4 * j + e]), fma2(f2s(eA), f2(yi[i], yi[i + 1]), f2(ya[i], ya[i + 1])));
            const float2 tz = fma2(z2, f2(-sg.x, -sg.y), add2(z2, f2s(1.f)));  // 1 + z (1 - sg)
            const float2 r = mul2(mul2(d2, ybar), mul2(sg, tz));
            o[2 * e] = r.x;
            o[2 * e + 1] = r.y;
          }
          gq[i] = g2.x;
          gq[i + 1] = g2.y;
        }
        if (z) {
          *reinterpret_cast<float4*>(dzs + 4 * ((8 * half + 2 * j) ^ (t & 7))) = make_float4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<float4*>(dzs + 4 * ((8 * half + 2 * j + 1) ^ (t & 7))) = make_float4(o[4], o[5], o[6], o[7]);
        }
      }
    }
    umma::fence_before_sync();
    __syncthreads();  // Yi has been read: round 3 may overwrite its columns
    umma::fence_after_sync();
    if (tid == 0) {
      constexpr uint32_t i_dg = umma::idesc_bf16(128, 64, true, true);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma::mma_bf16(tm + 256, umma::smem_desc(aQ + ks * 2048u, 16384, 1024),
                       umma::smem_desc(aGe + ks * 2048u, 16384, 1024), i_dg, ks > 0);
      umma::commit(&ss->mbar[2]);
    }
    {
      float da[32], db[32];
      umma::tmem_ld32(tm + lane_base + 64 + 32 * half, da);
      umma::tmem_ld32(tm + lane_base + 448 + 32 * half, db);
      umma::tmem_wait_ld();
      float* dvs = reinterpret_cast<float*>(sm + kStDv) + t * 64;
      const bool last = (tg == L - 1) && a.dfinal_v;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          o[u] = da[i + u] + erev * db[i + u] + dg * gq[i + u];
          if (last) o[u] += a.dfinal_v[bh * kP + 32 * half + i + u];
        }
        *reinterpret_cast<float4*>(dvs + 4 * ((8 * half + i / 4) ^ (t & 7))) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
    __syncthreads();
    {
      // the chunk's dv (and dz) rows are one contiguous 32 KB block each: coalesced stores
      const float* dvs = reinterpret_cast<const float*>(sm + kStDv);
      const float* dzs = reinterpret_cast<const float*>(sm + kStDz);
      const bool gbf = a.grad_dtype == M3_DTYPE_BF16;
      const size_t obv = (size_t)b * a.dv_st.b + (size_t)h * a.dv_st.h + (size_t)t0 * a.dv_st.l;
      const size_t obz = (size_t)b * a.dz_st.b + (size_t)h * a.dz_st.h + (size_t)t0 * a.dz_st.l;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int idx = tid + kThreads * m, row = idx >> 4, g4 = idx & 15;
        const int so = row * 64 + 4 * (g4 ^ (row & 7));
        const size_t ov = obv + (size_t)row * a.dv_st.l + 4 * g4, oz = obz + (size_t)row * a.dz_st.l + 4 * g4;
        const float4 v4 = *reinterpret_cast<const float4*>(dvs + so);
        float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (z) z4 = *reinterpret_cast<const float4*>(dzs + so);
        if (gbf) {  // bf16 gradients: 8-byte stores of 4 rounded values
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.dv) + ov) =
              make_uint2(umma::pack_bf16x2(v4.x, v4.y), umma::pack_bf16x2(v4.z, v4.w));
          if (z)
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.dz) + oz) =
                make_uint2(umma::pack_bf16x2(z4.x, z4.y), umma::pack_bf16x2(z4.z, z4.w));
        } else {
          *reinterpret_cast<float4*>(a.dv + ov) = v4;
          if (z) *reinterpret_cast<float4*>(a.dz + oz) = z4;
        }
      }
    }
    __syncthreads();  // the staging tiles are free for the pullback's rows

    M3_TC_MARK(14);
    // ---- pullback through the rotation (fp32, recomputed q~ / k~), 8 pairs at a time -------
    float dsc = 0.f, dAp = 0.f;
    {
      const float dgm = qkd * gam;
      float* dus = reinterpret_cast<float*>(sm + kDu) + t * 128;
      float* dws = reinterpret_cast<float*>(sm + kDw) + t * 128;
      const bool lastk = (tg == L - 1) && a.dfinal_k;
      float2 dsc2 = f2s(0.f), dAp2 = f2s(0.f);
#pragma unroll 2
      for (int sbk = 0; sbk < 4; ++sbk) {
        const int j0 = 32 * half + 8 * sbk;
        const bool grot = j0 < Nr;  // Nr % 8 == 0: the 8 pairs rotate together or not at all
        float dql[8], dqh[8], dkl[8], dkh[8];
        tmem_ld8(tm + lane_base + 128 + j0, dql);
        tmem_ld8(tm + lane_base + 128 + 64 + j0, dqh);
        tmem_ld8(tm + lane_base + 320 + j0, dkl);
        tmem_ld8(tm + lane_base + 320 + 64 + j0, dkh);
        const uint4 uq0 = rqs[(j0 >> 3) * kC + t], uq1 = rqs[(8 + (j0 >> 3)) * kC + t];
        const uint4 uk0 = rks[(j0 >> 3) * kC + t], uk1 = rks[(8 + (j0 >> 3)) * kC + t];
        const uint32_t ql[4] = {uq0.x, uq0.y, uq0.z, uq0.w}, qh[4] = {uq1.x, uq1.y, uq1.z, uq1.w};
        const uint32_t kl[4] = {uk0.x, uk0.y, uk0.z, uk0.w}, kh[4] = {uk1.x, uk1.y, uk1.z, uk1.w};
        float bq[16], bk[16];  // biases of pairs j0 .. j0+7: [0, 8) low halves, [8, 16) high halves
        {
          const float4* qb4 = reinterpret_cast<const float4*>(ss->bias + j0);
          const float4* kb4 = reinterpret_cast<const float4*>(ss->bias + kN + j0);
          const float4 v[8] = {qb4[0], qb4[1], qb4[16], qb4[17], kb4[0], kb4[1], kb4[16], kb4[17]};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            bq[4 * m] = v[m].x; bq[4 * m + 1] = v[m].y; bq[4 * m + 2] = v[m].z; bq[4 * m + 3] = v[m].w;
            bk[4 * m] = v[4 + m].x; bk[4 * m + 1] = v[4 + m].y; bk[4 * m + 2] = v[4 + m].z; bk[4 * m + 3] = v[4 + m].w;
          }
        }
        float* pp = phs + j0 * kC + t;
        float phv[8];
        if (grot)
#pragma unroll
          for (int r = 0; r < 8; ++r) phv[r] = pp[r * kC];
        umma::tmem_wait_ld();
        float2 dul[4], duh[4], dwl[4], dwh[4], dph[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 2 * e;
          float2 c2 = f2s(1.f), s2 = f2s(0.f);
          if (grot) {
            sincos_wrapped(wrap_fast(phv[r]), &s2.x, &c2.x);
            sincos_wrapped(wrap_fast(phv[r + 1]), &s2.y, &c2.y);
          }
          const float2 ns2 = f2(-s2.x, -s2.y);
          const float2 ulo = add2(bf2f(ql[e]), f2(bq[r], bq[r + 1]));
          const float2 uhi = add2(bf2f(qh[e]), f2(bq[8 + r], bq[8 + r + 1]));
          const float2 wlo = add2(bf2f(kl[e]), f2(bk[r], bk[r + 1]));
          const float2 whi = add2(bf2f(kh[e]), f2(bk[8 + r], bk[8 + r + 1]));
          const float2 qlo = fma2(uhi, ns2, mul2(ulo, c2)), qhi = fma2(ulo, s2, mul2(uhi, c2));
          const float2 klo = fma2(whi, ns2, mul2(wlo, c2)), khi = fma2(wlo, s2, mul2(whi, c2));
          const float2 gql = f2(dql[r], dql[r + 1]), gqh = f2(dqh[r], dqh[r + 1]);
          const float2 gkl = f2(dkl[r], dkl[r + 1]), gkh = f2(dkh[r], dkh[r + 1]);
          float2 dklo = mul2(gkl, f2s(scl)), dkhi = mul2(gkh, f2s(scl));
          if (lastk) {
            const float* fk = a.dfinal_k + bh * kN + j0 + r;
            dklo = add2(dklo, f2(fk[0], fk[1]));
            dkhi = add2(dkhi, f2(fk[64], fk[65]));
          }
          const float2 dg2 = f2s(dgm);
          dul[e] = fma2(dg2, wlo, fma2(gqh, s2, mul2(gql, c2)));
          duh[e] = fma2(dg2, whi, fma2(gql, ns2, mul2(gqh, c2)));
          dwl[e] = fma2(dg2, ulo, fma2(dkhi, s2, mul2(dklo, c2)));
          dwh[e] = fma2(dg2, uhi, fma2(dklo, ns2, mul2(dkhi, c2)));
          const float2 kd = fma2(gkh, khi, mul2(gkl, klo));  // khat-side inner product
          dsc2 = add2(dsc2, kd);
          dAp2 = fma2(f2s(-scl), kd, fma2(qhi, gqh, fma2(qlo, gql, dAp2)));
          dph[e] = grot ? add2(fma2(gqh, qlo, mul2(f2(-gql.x, -gql.y), qhi)), fma2(dkhi, klo, mul2(f2(-dklo.x, -dklo.y), khi)))
                        : f2s(0.f);
        }
        if (grot)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            pp[(2 * e) * kC] = dph[e].x;
            pp[(2 * e + 1) * kC] = dph[e].y;
          }
        // per-head rows for the bias reductions, float4 groups XOR-swizzled by token
        const int sw = t & 7;
        *reinterpret_cast<float4*>(dus + 4 * (((j0 >> 2)) ^ sw)) = make_float4(dul[0].x, dul[0].y, dul[1].x, dul[1].y);
        *reinterpret_cast<float4*>(dus + 4 * (((j0 >> 2) + 1) ^ sw)) = make_float4(dul[2].x, dul[2].y, dul[3].x, dul[3].y);
        *reinterpret_cast<float4*>(dus + 4 * (((64 + j0) >> 2) ^ sw)) = make_float4(duh[0].x, duh[0].y, duh[1].x, duh[1].y);
        *reinterpret_cast<float4*>(dus + 4 * ((((64 + j0) >> 2) + 1) ^ sw)) = make_float4(duh[2].x, duh[2].y, duh[3].x, duh[3].y);
        *reinterpret_cast<float4*>(dws + 4 * (((j0 >> 2)) ^ sw)) = make_float4(dwl[0].x, dwl[0].y, dwl[1].x, dwl[1].y);
        *reinterpret_cast<float4*>(dws + 4 * (((j0 >> 2) + 1) ^ sw)) = make_float4(dwl[2].x, dwl[2].y, dwl[3].x, dwl[3].y);
        *reinterpret_cast<float4*>(dws + 4 * (((64 + j0) >> 2) ^ sw)) = make_float4(dwh[0].x, dwh[0].y, dwh[1].x, dwh[1].y);
        *reinterpret_cast<float4*>(dws + 4 * ((((64 + j0) >> 2) + 1) ^ sw)) = make_float4(dwh[2].x, dwh[2].y, dwh[3].x, dwh[3].y);
      }
      dsc = dsc2.x + dsc2.y;
      dAp = dAp2.x + dAp2.y;
    }
    float* part = reinterpret_cast<float*>(sm + kScrPart);  // [2 halves][2][128]: dscale, dA
    part[(half * 2 + 0) * 128 + t] = dsc;
    part[(half * 2 + 1) * 128 + t] = dAp;
    if (half == 0) reinterpret_cast<float*>(sm + kScrDtb)[t] = dt;
    __syncthreads();

    M3_TC_MARK(15);
    // ---- bias column sums; angle adjoints (suffix over tokens) ------------------------------
    {
      // warps 0-3: du rows (-> dq), warps 4-7: dw rows (-> dk), 32 token rows each; lane l
      // owns columns 4l .. 4l+3.  Row-contiguous head-sum adds (one 512-byte row per warp
      // instruction) and the per-head bias column sums from the same loads.
      const int mat = warp >> 2;
      const float* src = reinterpret_cast<const float*>(sm + (mat ? kDw : kDu));
      float* dst = (mat ? a.dk : a.dq) + ((size_t)b * L + t0) * kN + 4 * lane;
#pragma unroll 4
      for (int rr = 0; rr < 32; ++rr) {
        const int tt = 32 * (warp & 3) + ((rr + 5 * h) & 31);  // heads start on different rows
        const float4 v = *reinterpret_cast<const float4*>(src + tt * 128 + 4 * (lane ^ (tt & 7)));
        bias01 = add2(bias01, f2(v.x, v.y));
        bias23 = add2(bias23, f2(v.z, v.w));
        red_add4(dst + (size_t)tt * kN, v.x, v.y, v.z, v.w);
      }
    }
    if constexpr (!RAW) {
      // preprocessed boundary: dphi is the pullback's per-token angle adjoint; the chunk's
      // (128, Nr) block of dphi is contiguous
      float* dst = a.dphi + (bh * L + t0) * Nr;
      for (int idx = tid; idx < kC * Nr; idx += kThreads) {
        const int tt = idx / Nr, r = idx - tt * Nr;
        dst[idx] = phs[r * kC + tt];
      }
    } else {
      const int g = warp;
      const bool grot = 8 * g < Nr;
      float* dthp = reinterpret_cast<float*>(sm + kScrTh);  // [8][128]
      const float* dts = reinterpret_cast<const float*>(sm + kScrDtb);
#pragma unroll 1
      for (int i = 1; i >= 0; --i) {  // lane l: tokens 2l, 2l+1 of the 64-token block i
        const int tb = 64 * i + 2 * lane;
        float share[2] = {0.f, 0.f};
        if (grot) {
          float dp[2][8], th[2][8];
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const float2 d2 = *reinterpret_cast<const float2*>(phs + (8 * g + r) * kC + tb);
            const float2 t2 = *reinterpret_cast<const float2*>(ths + (8 * g + r) * kC + tb);
            dp[0][r] = d2.x;
            dp[1][r] = d2.y;
            th[0][r] = t2.x;
            th[1][r] = t2.y;
          }
          const float2 wdt = mul2(*reinterpret_cast<const float2*>(dts + tb), f2s(kPi));
          float dan[2][8];
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            // suffix over tokens: this lane's pair plus every later lane of the block
            const float sfx = warp_suffix_scan(dp[0][r] + dp[1][r]);
            const float dth0 = dcarry8[r] + sfx, dth1 = dth0 - dp[0][r];
            dcarry8[r] += __shfl_sync(0xffffffffu, sfx, 0);
            const float th0 = th[0][r], th1 = th[1][r];
            dan[0][r] = dth0 * wdt.x * (1.f - th0 * th0);
            dan[1][r] = dth1 * wdt.y * (1.f - th1 * th1);
            share[0] += dth0 * th0 * kPi;
            share[1] += dth1 * th1 * kPi;
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float* dap = a.dangles + ((size_t)b * L + t0 + tb + j) * Nr + 8 * g;
            red_add4(dap, dan[j][0], dan[j][1], dan[j][2], dan[j][3]);
            red_add4(dap + 4, dan[j][4], dan[j][5], dan[j][6], dan[j][7]);
          }
        }
        *reinterpret_cast<float2*>(dthp + g * 128 + tb) = f2(share[0], share[1]);
      }
    }
    __syncthreads();
    if (c > 0) prefetch_kva(c - 1);  // the k, v and dw / angle tiles are free now

    M3_TC_MARK(16);
    // ---- per-token scalars: dadt (suffix of dA + the A_last term), preprocess adjoint -------
    {
      const float dscl = part[t] + part[256 + t];
      const float dA = part[128 + t] + part[384 + t];
      // suffix sum of dA over the chunk's 128 tokens (warps 0..3 own 32 tokens each)
      const float sfx = warp_suffix_scan(dA);
      if (half == 0 && lane == 0) ss->wtot[warp & 3] = sfx;
      __syncthreads();
      float dadt = sfx + alast;
      for (int w = (warp & 3) + 1; w < 4; ++w) dadt += ss->wtot[w];
      const float dscp = __shfl_up_sync(0xffffffffu, dscl, 1);
      if (!RAW && half == 0) {  // kernel_bwd.py:592-600: the preprocessed boundary's scalar gradients
        if (a.d_skip) dD_acc += qkd;
        a.dadt[bh * L + tg] = dadt;
        a.dgamma[bh * L + tg] = qkd * uwt;
        a.dscale[bh * L + tg] = dscl;
      }
      float dth = 0.f;
      if (RAW) {
        const float* dthp = reinterpret_cast<const float*>(sm + kScrTh);
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) dth += dthp[gg * 128 + t];
      }
      if (RAW && half == 0) {
        float prev = dscp;
        if (lane == 0) prev = t > 0 ? part[t - 1] + part[256 + t - 1] : 0.f;
        const float dgam = qkd * uwt;
        if (a.d_skip) dD_acc += qkd;
        const float ddt = (dgam + dscl) * lam + prev * (1.f - lam) + dadt * av + dth;
        const float dlam = (dgam + dscl) * dt - prev * dt;
        const float sgd = sigmoidf_(a.dt_raw[ro] + dtb);
        const size_t od = ((size_t)b * L + tg) * H + h;
        a.ddt_raw[od] = ddt * sgd;
        ddtb_acc += ddt * sgd;
        const bool open = -heavy_tail(ar) < -a.a_floor;
        const float htp = ar >= 0.f ? 1.f : 1.f / ((1.f - ar) * (1.f - ar));
        a.da_raw[od] = open ? -(dadt * dt) * htp : 0.f;
        a.dtrap_raw[od] = dlam * lam * (1.f - lam);
        if (t == kC - 1 && tg + 1 < L) {
          // scale of this chunk's last token reaches dt / lambda of the next chunk's first
          // token, whose gradients this block wrote one iteration earlier
          const size_t on = ro + a.raw_st.l, odn = od + H;
          const float sgn = sigmoidf_(a.dt_raw[on] + dtb);
          const float e_dt = dscl * (1.f - lamn) * sgn;
          a.ddt_raw[odn] += e_dt;
          ddtb_acc += e_dt;
          a.dtrap_raw[odn] += -dscl * dtn * lamn * (1.f - lamn);
        }
      }
    }

    M3_TC_MARK(17);
    // ---- round 3 result: G <- exp2(A_last) G + dG; A_last term of the previous chunk -------
    if (__syncthreads_or(!umma::mbar_wait(&ss->mbar[2], (nchunk - 1 - c) & 1))) {
      if (tid == 0) atomicExch(&g_m3_device_error, 13);
      ok = false;
      break;
    }
    umma::fence_after_sync();
    {
      float dG[32];
      umma::tmem_ld32(tm + lane_base + 256 + 32 * half, dG);
      umma::tmem_wait_ld();
      const float eAl = exp2f(Alast);
      float partS = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) G[i] = G[i] * eAl + dG[i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        *reinterpret_cast<uint4*>(sm + kGt + umma::sw128_off(t, 4 * half + j)) = pack8(G + 8 * j);
        const uint4 u = *reinterpret_cast<const uint4*>(sm + kSt + umma::sw128_off(t, 4 * half + j));
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) partS += G[8 * j + 2 * e] * bf16lo(w4[e]) + G[8 * j + 2 * e + 1] * bf16hi(w4[e]);
      }
      const float tot = cta_sum(partS, ss);
      if (tid == 0) ss->alast = tot;
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (c > 0) prefetch_qst(c - 1);
    M3_TC_MARK(18);
  }
  umma::cp_async_wait_all();  // nothing of ours still lands in shared memory after an early exit

  if (ok) {
    // ---- seeds (kernel_bwd.py:636-646), angle carry, per-head reductions ------------------
    if (a.seed_ssm) {
      const size_t o0 = (size_t)b * a.raw_st.b + (size_t)h * a.raw_st.h;
      float dt0 = 0.f, lam0 = 0.f, coef;
      if constexpr (RAW) {
        dt0 = softplusf(a.dt_raw[o0] + dtb);
        lam0 = sigmoidf_(a.trap_raw[o0]);
        coef = dt0 * (1.f - lam0);
      } else {
        coef = a.seed_coef[bh];
      }
      const float kp = a.seed_k[bh * kN + t];
      float pk = 0.f, pc = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int p = 32 * half + i;
        a.dseed_ssm[(bh * kP + p) * kN + t] = G[i];
        const float vp = a.seed_v[bh * kP + p];
        pk += G[i] * vp;
        pc += G[i] * vp * kp;
        atomicAdd(a.dseed_v + bh * kP + p, coef * G[i] * kp);
      }
      atomicAdd(a.dseed_k + bh * kN + t, coef * pk);
      const float dcoef = cta_sum(pc, ss);
      if (!RAW && tid == 0) a.dseed_coef[bh] = dcoef;
      if (RAW && tid == 0) {
        const size_t od = (size_t)b * L * H + h;
        const float sg = sigmoidf_(a.dt_raw[o0] + dtb);
        const float e_dt = dcoef * (1.f - lam0) * sg;
        a.ddt_raw[od] += e_dt;
        ddtb_acc += e_dt;
        a.dtrap_raw[od] += -dcoef * dt0 * lam0 * (1.f - lam0);
      }
    }
    if (RAW && a.dseed_phi && lane == 0 && 8 * warp < Nr)
#pragma unroll
      for (int r = 0; r < 8; ++r) a.dseed_phi[bh * Nr + 8 * warp + r] = dcarry8[r];
    {
      float* bb = (warp >= 4 ? a.dk_bias : a.dq_bias) + h * kN + 4 * lane;
      atomicAdd(bb, bias01.x);
      atomicAdd(bb + 1, bias01.y);
      atomicAdd(bb + 2, bias23.x);
      atomicAdd(bb + 3, bias23.y);
    }
    const float dD = cta_sum(dD_acc, ss);
    const float ddb = cta_sum(ddtb_acc, ss);
    if (tid == 0) {
      if (a.d_skip) atomicAdd(a.dd_skip + h, dD);
      if (RAW) atomicAdd(a.ddt_bias + h, ddb);
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tm, 512);
}

}  // namespace tcb
}  // namespace m3
