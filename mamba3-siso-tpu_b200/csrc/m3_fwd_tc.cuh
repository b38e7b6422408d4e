// Tensor-core (tcgen05 / TMEM) chunked forward for the production shape:
// bf16 I/O and bf16 matmul operands, N = 128, P = 64, 128-token chunks.
//
// One CTA per SM holds two independent "slots" of 256 threads; each slot walks one
// (b, h) sequence chunk by chunk with its own 112 KB of shared memory and 256 TMEM
// columns, so while one slot waits on the tensor core the other runs its CUDA-core
// phases.  Per 128-token chunk (A_t = prefix sum of adt log2 e inside the chunk):
//
//   CUDA cores : per-token dt / A / lambda / gamma / scale (fused preprocess), the
//                cumulative rotary angles, rotation of q and k (bf16 q~, khat = k~ scale
//                into SWIZZLE_128B K-major tiles), v and v exp2(A_last - A) tiles
//   tcgen05    : S = q~ khat^T            (128 x 128, K = N)    -> TMEM [0, 128)
//                Yi = q~ St^T             (128 x 64,  K = N)    -> TMEM [128, 192)
//                dSt = khat^T vd          (128 x 64,  K = 128)  -> TMEM [192, 256)
//   CUDA cores : St <- exp2(A_last) St + dSt (fp32, registers), bf16 copy for the next
//                chunk's readout; decay mask of S -> bf16 into the q~ tile
//   tcgen05    : Ya = mask(S) v           (128 x 64,  K = 128)  -> TMEM [0, 64)
//   CUDA cores : y = exp2(A) Yi + Ya + (D + gamma u.w) v, times silu(z), store.
//
// This is kernel_fwd.py:55-201 of the reference (the same bf16 rounding points:
// kernel_fwd.py:139-187) with reference.py:104-199's preprocessing fused in.  Every
// wait on the tensor core is bounded; a time-out records an error in g_m3_device_error
// and the slot winds down instead of spinning.
#pragma once

#include "m3_chunk_common.cuh"
#include "m3_umma.cuh"

namespace m3 {

__device__ int g_m3_device_error;  // non-zero after a bounded wait gave up

#ifdef M3_TC_TIMING
// Per-phase cycle totals of slot-thread 0 of every slot (diagnostic builds only).
__device__ unsigned long long g_m3_tc_timing[24];
#define M3_TC_MARK(i)                                                   \
  do {                                                                  \
    if (ltid == 0) {                                                    \
      const long long now_ = clock64();                                 \
      atomicAdd(&g_m3_tc_timing[i], (unsigned long long)(now_ - tmark_)); \
      tmark_ = now_;                                                    \
    }                                                                   \
  } while (0)
#else
#define M3_TC_MARK(i) \
  do {                \
  } while (0)
#endif

namespace tc {

constexpr int kN = 128, kP = 64, kC = 128;
constexpr int kSlotThreads = 256;
constexpr int kThreads = 2 * kSlotThreads;
constexpr uint32_t kQ = 0, kK = 32768, kV = 65536, kVd = 81920, kSt = 98304, kSlotBytes = 114688;
// scratch laid over the vd tile while it is not live
constexpr uint32_t kScrDt = 0, kScrScl = 512, kScrUw = 1024, kScrA = 0;  // uw: [8][128] floats
constexpr uint32_t kScrBias = 5120;  // the head's q_bias, k_bias [2][128] (loaded with the khat prefetch)

struct SlotSmall {
  uint64_t mbar[2];
  float wtot[4];
};
struct CtaSmall {
  SlotSmall slot[2];
  uint32_t tmem;
};
constexpr size_t kSmemBytes = 2 * (size_t)kSlotBytes + sizeof(CtaSmall) + 1024;  // + alignment slack

__device__ __forceinline__ void slot_sync(int slot) {
  asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(kSlotThreads) : "memory");
}

// Barrier over the slot's threads that also ORs `pred` across them, so a decision taken
// after a bounded wait is the same in every thread of the slot.
__device__ __forceinline__ bool slot_any(int slot, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %2, 0;\n\t"
      "bar.red.or.pred p, %1, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"(slot + 1), "r"((uint32_t)pred), "r"(kSlotThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// 16 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  u.x = umma::pack_bf16x2(f[0], f[1]);
  u.y = umma::pack_bf16x2(f[2], f[3]);
  u.z = umma::pack_bf16x2(f[4], f[5]);
  u.w = umma::pack_bf16x2(f[6], f[7]);
  return u;
}

// Outputs of the states-only mode used by the backward's recompute sweep: the bf16 state
// tile image (the layout the backward's tensor-core operands use) at every chunk start
// plus the final state, and the rotary-angle carry at every chunk start.  A full forward
// given them writes the same (so a backward on the same inputs can skip its sweep).
struct TcStates {
  uint8_t* tiles;  // (B*H, nchunk + 1, 16 KB)
  float* phis;     // (B*H, nchunk, Nr)
};

template <bool RAW, bool STATES>
__global__ void __launch_bounds__(kThreads, 1) fwd_tc_kernel(const M3FwdArgs a, const TcStates so) {
  extern __shared__ uint8_t smraw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  CtaSmall* cs = (CtaSmall*)(base + 2 * kSlotBytes);
  const int slot = threadIdx.x / kSlotThreads;
  const int ltid = threadIdx.x % kSlotThreads;
  const int lwarp = ltid >> 5, lane = ltid & 31;
  uint8_t* sm = base + slot * kSlotBytes;
  SlotSmall* ss = &cs->slot[slot];
  const int H = a.dims.nheads, L = a.dims.seqlen, Nr = a.dims.n_angles;
  const int nseq = a.dims.batch * H;
  const int seq = blockIdx.x * 2 + slot;
  const bool active = seq < nseq;

  if (threadIdx.x < 32) umma::tmem_alloc(&cs->tmem, 512);
  if (ltid == 0) {
    umma::mbar_init(&ss->mbar[0], 1);
    umma::mbar_init(&ss->mbar[1], 1);
    umma::fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = cs->tmem + (uint32_t)slot * 256u;

  if (active) {
    const int b = seq / H, h = seq % H;
    const size_t bh = (size_t)seq;
    const int t = ltid & 127, half = ltid >> 7;    // token row / state row, column half
    const uint32_t lane_base = (uint32_t)(32 * (lwarp & 3)) << 16;
    const __nv_bfloat16* q = (const __nv_bfloat16*)a.q;
    const __nv_bfloat16* k = (const __nv_bfloat16*)a.k;
    const __nv_bfloat16* v = (const __nv_bfloat16*)a.v;
    const __nv_bfloat16* z = (const __nv_bfloat16*)a.z;
    __nv_bfloat16* y = (__nv_bfloat16*)a.y;
    const float Dh = a.d_skip ? a.d_skip[h] : 0.f;
    const int nchunk = L / kC;
    const int chunk_sub = a.dims.chunk / kC;
    // 32-byte rotary-group pieces of the angle (or phi) rows can be read with one load
    const bool ang32 = RAW ? ((uintptr_t)a.angles % 32 == 0 && a.ang_st.l % 8 == 0 && a.ang_st.b % 8 == 0)
                           : ((uintptr_t)a.phi % 32 == 0 && Nr % 8 == 0);
    const uint32_t sQ = umma::smem_u32(sm + kQ), sK = umma::smem_u32(sm + kK), sV = umma::smem_u32(sm + kV);
    const uint32_t sVd = umma::smem_u32(sm + kVd), sSt = umma::smem_u32(sm + kSt);
    bool ok = true;

    // ---- initial state: registers hold St[n = t][p = 32 half + i] (fp32) ------------
    // The fp32 state lives in TMEM columns [192, 256) of the slot (lane n = t, columns
    // 32 half ..): the state-update MMA accumulates onto it after the threads have scaled
    // it by exp2(A_last) in place.  A bf16 copy in the St tile feeds the readout MMA.
    float carry8[8];
    {
      float st[32];
      float coef = 0.f;
      if (a.seed_ssm) {
        if (RAW) {
          const size_t o = (size_t)b * a.raw_st.b + (size_t)h * a.raw_st.h;
          coef = softplusf(a.dt_raw[o] + a.dt_bias[h]) * (1.f - sigmoidf_(a.trap_raw[o]));
        } else {
          coef = a.seed_coef[bh];
        }
      }
      const float kprev = a.seed_ssm ? a.seed_k[bh * kN + t] : 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int p = 32 * half + i;
        st[i] = a.seed_ssm ? a.seed_ssm[(bh * kP + p) * kN + t] + coef * a.seed_v[bh * kP + p] * kprev : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(sm + kSt + umma::sw128_off(t, 4 * half + j)) = pack8(st + 8 * j);
      umma::tmem_st32(tm + lane_base + 192 + 32 * half, st);
      umma::tmem_wait_st();
#pragma unroll
      for (int r = 0; r < 8; ++r)  // angle carry of this warp's rotary group (raw boundary)
        carry8[r] = (RAW && a.seed_phi && 8 * lwarp + r < Nr) ? a.seed_phi[bh * Nr + 8 * lwarp + r] : 0.f;
    }
    umma::fence_before_sync();
    slot_sync(slot);

    // Raw q / k rows of chunk `cc` straight into the q~ / khat tiles (K-major, swizzled)
    // and its v rows into the v tile (MN-major); rotated / scaled in place afterwards.
    auto prefetch_qv = [&](int cc) {
      const int tb = cc * kC;
#pragma unroll
      for (int m = 0; m < (STATES ? 0 : 8); ++m) {
        const int i = ltid + kSlotThreads * m;  // 0 .. 2047
        const int row = i >> 4, c16 = i & 15;
        const uint32_t dst = (c16 >> 3) * 16384u + umma::sw128_off(row, c16 & 7);
        umma::cp_async16(sQ + dst, q + (size_t)b * a.q_st.b + (size_t)(tb + row) * a.q_st.l + c16 * 8);
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = ltid + kSlotThreads * m;  // 0 .. 1023
        const int row = i >> 3, c8 = i & 7;
        umma::cp_async16(sV + umma::sw128_off(row, c8),
                         v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h + (size_t)(tb + row) * a.v_st.l + c8 * 8);
      }
      umma::cp_async_commit();
    };
    auto prefetch_k = [&](int cc) {
      const int tb = cc * kC;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int i = ltid + kSlotThreads * m;
        const int row = i >> 4, c16 = i & 15;
        const uint32_t dst = (c16 >> 3) * 16384u + umma::sw128_off(row, c16 & 7);
        umma::cp_async16(sK + dst, k + (size_t)b * a.k_st.b + (size_t)(tb + row) * a.k_st.l + c16 * 8);
      }
      if (ltid < 64)  // biases into the vd tile's scratch (its y staging has been stored by now)
        umma::cp_async16(sVd + kScrBias + 16 * ltid, (ltid < 32 ? a.q_bias + h * kN : a.k_bias + h * kN - 128) + 4 * ltid);
      umma::cp_async_commit();
    };
    prefetch_qv(0);
    prefetch_k(0);
    // raw per-token scalars of chunk `cc` for this thread's token row
    const float dtb = RAW ? a.dt_bias[h] : 0.f;
    float rs[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    auto load_scalars = [&](int cc) {
      const int tt = cc * kC + t;
      if (RAW) {
        const size_t o = (size_t)b * a.raw_st.b + (size_t)tt * a.raw_st.l + (size_t)h * a.raw_st.h;
        rs[0] = a.dt_raw[o];
        rs[1] = a.a_raw[o];
        rs[2] = a.trap_raw[o];
        if (lane == 31 && tt + 1 < L) {
          rs[3] = a.dt_raw[o + a.raw_st.l];
          rs[4] = a.trap_raw[o + a.raw_st.l];
        }
      } else {
        const size_t o = bh * L + tt;
        rs[0] = a.adt[o];
        rs[1] = a.gamma[o];
        rs[2] = a.scale[o];
      }
    };
    load_scalars(0);

#ifdef M3_TC_TIMING
    long long tmark_ = clock64();
#endif
    auto dump_state_tile = [&](int cc) {
      uint4* dst = reinterpret_cast<uint4*>(so.tiles + (bh * (nchunk + 1) + cc) * 16384u);
      const uint4* src = reinterpret_cast<const uint4*>(sm + kSt);
#pragma unroll
      for (int m = 0; m < 4; ++m) dst[ltid + kSlotThreads * m] = src[ltid + kSlotThreads * m];
    };
    for (int c = 0; c < nchunk && ok; ++c) {
      const int t0 = c * kC;
      const int tg = t0 + t;  // this thread's token (row roles)
      if (so.tiles) {  // the backward's sweep, or a forward saving the states for the backward
        dump_state_tile(c);
        if (RAW && lane == 0 && 8 * lwarp < Nr)
#pragma unroll
          for (int r = 0; r < 8; ++r) so.phis[(bh * nchunk + c) * Nr + 8 * lwarp + r] = carry8[r];
      }
      // ---- phase 1: per-token scalars (raw values were loaded during the last chunk) ---
      float dt = 0.f, adt, gam, scl;
      if (RAW) {
        dt = softplusf(rs[0] + dtb);
        const float lam = sigmoidf_(rs[2]);
        adt = fminf(-heavy_tail(rs[1]), -a.a_floor) * dt;
        float dtn = __shfl_down_sync(0xffffffffu, dt, 1), lamn = __shfl_down_sync(0xffffffffu, lam, 1);
        if (lane == 31) {  // the successor lives in the next warp or the next chunk
          dtn = tg + 1 < L ? softplusf(rs[3] + dtb) : 0.f;
          lamn = tg + 1 < L ? sigmoidf_(rs[4]) : 0.f;
        }
        gam = dt * lam;
        scl = gam + dtn * (1.f - lamn);
      } else {
        adt = rs[0];
        gam = rs[1];
        scl = rs[2];
      }
      const float incl = warp_inclusive_scan(adt * kLog2e);
      if (half == 0 && lane == 31) ss->wtot[lwarp & 3] = incl;
      if (half == 0) {
        if (RAW) reinterpret_cast<float*>(sm + kVd + kScrDt)[t] = dt;
        reinterpret_cast<float*>(sm + kVd + kScrScl)[t] = scl;
      }
      umma::cp_async_wait_all();  // this chunk's q / k / v rows have landed
      slot_sync(slot);
      float A = incl;
      for (int w = 0; w < (lwarp & 3); ++w) A += ss->wtot[w];
      const float Alast = ss->wtot[0] + ss->wtot[1] + ss->wtot[2] + ss->wtot[3];
      M3_TC_MARK(0);

      // ---- phase 2: cumulative angles and rotation ---------------------------------------
      // Warp g owns rotary pairs (8g .. 8g+7, 64+8g .. 64+8g+7): one 16-byte swizzle chunk
      // of each q / k half-row.  Lane l owns the token pairs (2l, 2l+1) + 64 i; the prefix
      // over tokens is one warp scan of the pair sums per angle and 64-token block, and the
      // carry across chunks stays in registers (the same value in every lane of the warp).
      {
        const float* dts = reinterpret_cast<const float*>(sm + kVd + kScrDt);
        const float* scls = reinterpret_cast<const float*>(sm + kVd + kScrScl);
        float* uws = reinterpret_cast<float*>(sm + kVd + kScrUw);  // [8 groups][128 tokens]
        const int g = lwarp;
        const bool grot = 8 * g < Nr;  // Nr % 8 == 0: a group rotates entirely or not at all
        const float* qbp = reinterpret_cast<const float*>(sm + kVd + kScrBias) + 8 * g;
        const float* kbp = qbp + kN;
        float off[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) off[r] = carry8[r];
#pragma unroll 1
        for (int i = 0; i < 2; ++i) {
          const int tb = 64 * i + 2 * lane;
          float ph[2][8];
          if (grot) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int tgl = t0 + tb + j;
              const float* pp = RAW ? a.angles + (size_t)b * a.ang_st.b + (size_t)tgl * a.ang_st.l + 8 * g
                                    : a.phi + (bh * L + tgl) * Nr + 8 * g;
              if (ang32) {
                ldg8(pp, ph[j]);
              } else {
                const float4 lo = *reinterpret_cast<const float4*>(pp);
                const float4 hi = *reinterpret_cast<const float4*>(pp + 4);
                ph[j][0] = lo.x; ph[j][1] = lo.y; ph[j][2] = lo.z; ph[j][3] = lo.w;
                ph[j][4] = hi.x; ph[j][5] = hi.y; ph[j][6] = hi.z; ph[j][7] = hi.w;
              }
            }
            if (RAW) {
              const float2 w = mul2(*reinterpret_cast<const float2*>(dts + tb), f2s(kPi));
#pragma unroll
              for (int r = 0; r < 8; ++r) {
                const float x0 = tanh_acc(ph[0][r]) * w.x, x1 = tanh_acc(ph[1][r]) * w.y;
                const float incl = warp_inclusive_scan(x0 + x1);
                ph[1][r] = off[r] + incl;
                ph[0][r] = ph[1][r] - x1;
                off[r] += __shfl_sync(0xffffffffu, incl, 31);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int tt = tb + j, tgl = t0 + tt;
            float cs[8], sn[8];
  #pragma unroll
            for (int r = 0; r < 8; ++r) {
              cs[r] = 1.f;
              sn[r] = 0.f;
              if (grot) sincos_wrapped(wrap_fast(ph[j][r]), &sn[r], &cs[r]);
            }
            const uint32_t soff = umma::sw128_off(tt, g);
            uint4 uql = make_uint4(0u, 0u, 0u, 0u), uqh = uql;
            if constexpr (!STATES) {  // the states-only sweep needs khat alone
              uql = *reinterpret_cast<const uint4*>(sm + kQ + soff);
              uqh = *reinterpret_cast<const uint4*>(sm + kQ + 16384 + soff);
            }
            const uint4 ukl = *reinterpret_cast<const uint4*>(sm + kK + soff);
            const uint4 ukh = *reinterpret_cast<const uint4*>(sm + kK + 16384 + soff);
            const uint32_t ql[4] = {uql.x, uql.y, uql.z, uql.w}, qh[4] = {uqh.x, uqh.y, uqh.z, uqh.w};
            const uint32_t kl[4] = {ukl.x, ukl.y, ukl.z, ukl.w}, kh[4] = {ukh.x, ukh.y, ukh.z, ukh.w};
            const float sc = scls[tt];
            uint32_t pq_lo[4], pq_hi[4], pk_lo[4], pk_hi[4];
            float2 uw2 = f2s(0.f);
  #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 c2 = f2(cs[2 * e], cs[2 * e + 1]), s2 = f2(sn[2 * e], sn[2 * e + 1]);
              const float2 ns2 = f2(-sn[2 * e], -sn[2 * e + 1]);
              const float2 wlo = add2(bf2f(kl[e]), *reinterpret_cast<const float2*>(kbp + 2 * e));
              const float2 whi = add2(bf2f(kh[e]), *reinterpret_cast<const float2*>(kbp + 64 + 2 * e));
              if constexpr (!STATES) {
                const float2 ulo = add2(bf2f(ql[e]), *reinterpret_cast<const float2*>(qbp + 2 * e));
                const float2 uhi = add2(bf2f(qh[e]), *reinterpret_cast<const float2*>(qbp + 64 + 2 * e));
                uw2 = fma2(ulo, wlo, uw2);
                uw2 = fma2(uhi, whi, uw2);
                pq_lo[e] = f2bf(fma2(uhi, ns2, mul2(ulo, c2)));
                pq_hi[e] = f2bf(fma2(ulo, s2, mul2(uhi, c2)));
              }
              const float2 klo = fma2(whi, ns2, mul2(wlo, c2));
              const float2 khi = fma2(wlo, s2, mul2(whi, c2));
              if (tgl == L - 1 && a.final_k) {  // final k is rotated but unscaled (kernel_fwd.py:192-201)
                float* fk = a.final_k + bh * kN + 8 * g + 2 * e;
                fk[0] = klo.x;
                fk[1] = klo.y;
                fk[64] = khi.x;
                fk[65] = khi.y;
              }
              pk_lo[e] = f2bf(mul2(klo, f2s(sc)));
              pk_hi[e] = f2bf(mul2(khi, f2s(sc)));
            }
            if constexpr (!STATES) {
              *reinterpret_cast<uint4*>(sm + kQ + soff) = make_uint4(pq_lo[0], pq_lo[1], pq_lo[2], pq_lo[3]);
              *reinterpret_cast<uint4*>(sm + kQ + 16384 + soff) = make_uint4(pq_hi[0], pq_hi[1], pq_hi[2], pq_hi[3]);
              uws[g * 128 + tt] = uw2.x + uw2.y;
            }
            *reinterpret_cast<uint4*>(sm + kK + soff) = make_uint4(pk_lo[0], pk_lo[1], pk_lo[2], pk_lo[3]);
            *reinterpret_cast<uint4*>(sm + kK + 16384 + soff) = make_uint4(pk_hi[0], pk_hi[1], pk_hi[2], pk_hi[3]);
          }
        }
        if (RAW)
#pragma unroll
          for (int r = 0; r < 8; ++r) carry8[r] = wrap_fast(off[r]);
      }
      M3_TC_MARK(1);
      umma::fence_async_smem();  // the q~ / khat tiles, for the MMAs issued below
      umma::fence_before_sync();
      slot_sync(slot);
      float dg = 0.f;
      if constexpr (!STATES) {
        const float* uws = reinterpret_cast<const float*>(sm + kVd + kScrUw);
        float uw = 0.f;
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) uw += uws[gg * 128 + t];
        dg = uw * gam + Dh;
      }
      slot_sync(slot);

      // S = q~ khat^T and Yi = q~ S^T need nothing of phase 3: they run while it does
      if constexpr (!STATES) {
        umma::fence_after_sync();
        if (ltid == 0) {
          constexpr uint32_t id_s = umma::idesc_bf16(128, 128, false, false);
          constexpr uint32_t id_yi = umma::idesc_bf16(128, 64, false, true);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t kmaj = (ks >> 2) * 16384u + (ks & 3) * 32u;
            const uint64_t dq = umma::smem_desc(sQ + kmaj, 16, 1024);
            umma::mma_bf16(tm + 0, dq, umma::smem_desc(sK + kmaj, 16, 1024), id_s, ks > 0);
            umma::mma_bf16(tm + 128, dq, umma::smem_desc(sSt + ks * 2048u, 16384, 1024), id_yi, ks > 0);
          }
        }
      }
      M3_TC_MARK(2);
      // ---- phase 3: v and v exp2(A_last - A) tiles (MN-major: row = token) -------------
      uint32_t vreg[16];  // this thread's 32 v values (bf16 pairs), kept for the diagonal term
      {
        const float e = exp2f(Alast - A);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 u = *reinterpret_cast<const uint4*>(sm + kV + umma::sw128_off(t, 4 * half + j));
          vreg[4 * j + 0] = u.x;
          vreg[4 * j + 1] = u.y;
          vreg[4 * j + 2] = u.z;
          vreg[4 * j + 3] = u.w;

          const float2 e2 = f2s(e);
          const uint4 d = make_uint4(f2bf(mul2(bf2f(u.x), e2)), f2bf(mul2(bf2f(u.y), e2)), f2bf(mul2(bf2f(u.z), e2)),
                                     f2bf(mul2(bf2f(u.w), e2)));
          *reinterpret_cast<uint4*>(sm + kVd + umma::sw128_off(t, 4 * half + j)) = d;
        }
      }
      // scale the TMEM state by exp2(A_last) so the update MMA can accumulate onto it; the
      // chunk-start state residual is this state before scaling
      {
        float sv[32];
        umma::tmem_ld32(tm + lane_base + 192 + 32 * half, sv);
        umma::tmem_wait_ld();
        if (a.chunk_states && c % chunk_sub == 0) {
          const int nc = L / a.dims.chunk, ci = c / chunk_sub;
          const size_t sb = ((bh * nc + ci) * kP) * kN;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const size_t o = sb + (size_t)(32 * half + i) * kN + t;
            if (a.chunk_states_dtype == M3_DTYPE_BF16) ((__nv_bfloat16*)a.chunk_states)[o] = __float2bfloat16_rn(sv[i]);
            else ((float*)a.chunk_states)[o] = sv[i];
          }
        }
        const float2 eAl = f2s(exp2f(Alast));
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 r = mul2(f2(sv[i], sv[i + 1]), eAl);
          sv[i] = r.x;
          sv[i + 1] = r.y;
        }
        umma::tmem_st32(tm + lane_base + 192 + 32 * half, sv);
        umma::tmem_wait_st();
      }
      umma::fence_async_smem();
      umma::fence_before_sync();
      slot_sync(slot);
      umma::fence_after_sync();

      M3_TC_MARK(3);
      // ---- phase 4: the state update on the tensor core (S and Yi are already running) -----
      if (ltid == 0) {
        constexpr uint32_t id_ds = umma::idesc_bf16(128, 64, true, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t mn = ks * 2048u;
          umma::mma_bf16(tm + 192, umma::smem_desc(sK + mn, 16384, 1024), umma::smem_desc(sVd + mn, 16384, 1024),
                         id_ds, true);
        }
        umma::commit(&ss->mbar[0]);  // tracks S and Yi too (issued earlier by this thread)
      }
      if (slot_any(slot, !umma::mbar_wait(&ss->mbar[0], c & 1))) {
        if (ltid == 0) atomicExch(&g_m3_device_error, 1);
        ok = false;
        break;
      }
      umma::fence_after_sync();

      // the khat tile is free until the next chunk: stage the chunk's z rows there (rows of
      // 128 bytes, four per warp instruction)
      if (!STATES && z) {
        const __nv_bfloat16* zb = z + (size_t)b * a.z_st.b + (size_t)h * a.z_st.h + (size_t)t0 * a.z_st.l;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int i = ltid + kSlotThreads * m, row = i >> 3, c8 = i & 7;
          umma::cp_async16(sK + umma::sw128_off(row, c8), zb + (size_t)row * a.z_st.l + 8 * c8);
        }
      }
      umma::cp_async_commit();
      M3_TC_MARK(4);
      // ---- phase 5a: the updated state -> bf16 St tile for the next chunk's readout --------
      {
        float sv[32];
        umma::tmem_ld32(tm + lane_base + 192 + 32 * half, sv);
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(sm + kSt + umma::sw128_off(t, 4 * half + j)) = pack8(sv + 8 * j);
        if (half == 0) reinterpret_cast<float*>(sm + kVd + kScrA)[t] = A;
      }
      slot_sync(slot);
      if constexpr (STATES) {  // nothing else of this chunk is needed: fetch the next one
        if (c + 1 < nchunk) {
          prefetch_qv(c + 1);
          prefetch_k(c + 1);
          load_scalars(c + 1);
        }
        continue;
      }
      // ---- phase 5b: decay mask of S -> bf16 into the q~ tile -----------------------------
      {
        const float* As = reinterpret_cast<const float*>(sm + kVd + kScrA);
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
          float sv[32];
          const int sb = 64 * half + 32 * cb;
          const bool any = sb < t;
          umma::tmem_ld32(tm + lane_base + sb, sv);
          umma::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t m[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int s = sb + 8 * j + 2 * e;
              const float2 as = *reinterpret_cast<const float2*>(As + s);
              const float2 d = add2(f2s(A), f2(-as.x, -as.y));
              float2 val = mul2(f2(sv[8 * j + 2 * e], sv[8 * j + 2 * e + 1]),
                                f2(ex2(fminf(d.x, 0.f)), ex2(fminf(d.y, 0.f))));
              if (!(any && s < t)) val.x = 0.f;
              if (!(any && s + 1 < t)) val.y = 0.f;
              m[e] = f2bf(val);
            }
            *reinterpret_cast<uint4*>(sm + kQ + 16384 * half + umma::sw128_off(t, 4 * cb + j)) =
                make_uint4(m[0], m[1], m[2], m[3]);
          }
        }
      }
      umma::fence_async_smem();
      umma::fence_before_sync();
      slot_sync(slot);
      umma::fence_after_sync();
      if (ltid == 0) {
        constexpr uint32_t id_ya = umma::idesc_bf16(128, 64, false, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t kmaj = (ks >> 2) * 16384u + (ks & 3) * 32u;
          umma::mma_bf16(tm + 0, umma::smem_desc(sQ + kmaj, 16, 1024), umma::smem_desc(sV + ks * 2048u, 16384, 1024),
                         id_ya, ks > 0);
        }
        umma::commit(&ss->mbar[1]);
      }
      if (slot_any(slot, !umma::mbar_wait(&ss->mbar[1], c & 1))) {
        if (ltid == 0) atomicExch(&g_m3_device_error, 2);
        ok = false;
        break;
      }
      umma::fence_after_sync();
      if (c + 1 < nchunk) {  // the q~ and v tiles are free again
        prefetch_qv(c + 1);
        load_scalars(c + 1);
      } else {
        umma::cp_async_commit();  // an empty group keeps the wait_group count below exact
      }
      M3_TC_MARK(5);

      // ---- phase 6: output -----------------------------------------------------------------
      {
        const float2 eA = f2s(exp2f(A)), dg2 = f2s(dg);
        if (z) {  // the z group (committed before q~ / v) of every thread of the slot
          asm volatile("cp.async.wait_group %0;" ::"n"(1) : "memory");
          slot_sync(slot);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {  // 16 columns at a time
          float yi[16], ya[16];
          tmem_ld16(tm + lane_base + 128 + 32 * half + 16 * hh, yi);
          tmem_ld16(tm + lane_base + 32 * half + 16 * hh, ya);
          umma::tmem_wait_ld();
          float2 o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            o[i] = fma2(dg2, bf2f(vreg[8 * hh + i]), fma2(eA, f2(yi[2 * i], yi[2 * i + 1]), f2(ya[2 * i], ya[2 * i + 1])));
          if (a.ybar) {
            float* yb = a.ybar + (bh * L + tg) * kP + 32 * half + 16 * hh;
#pragma unroll
            for (int i = 0; i < 8; i += 2) *reinterpret_cast<float4*>(yb + 2 * i) = make_float4(o[i].x, o[i].y, o[i + 1].x, o[i + 1].y);
          }
          uint32_t packed[8];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            uint4 u = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
            if (z) u = *reinterpret_cast<const uint4*>(sm + kK + umma::sw128_off(t, 4 * half + 2 * hh + j));
            const uint32_t zz[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 r = o[4 * j + e];
              if (z) r = mul2(r, silu2(bf2f(zz[e])));
              packed[4 * j + e] = f2bf(r);
            }
          }
          // y row pieces into the (free) vd tile; stored below as whole rows
          *reinterpret_cast<uint4*>(sm + kVd + umma::sw128_off(t, 4 * half + 2 * hh)) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
          *reinterpret_cast<uint4*>(sm + kVd + umma::sw128_off(t, 4 * half + 2 * hh + 1)) =
              make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
      umma::cp_async_wait_all();  // z reads done and nothing of ours still lands in the khat tile
      umma::fence_before_sync();
      slot_sync(slot);
      umma::fence_after_sync();
      {
        __nv_bfloat16* yb = y + (size_t)b * a.y_st.b + (size_t)h * a.y_st.h + (size_t)t0 * a.y_st.l;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int i = ltid + kSlotThreads * m, row = i >> 3, c8 = i & 7;
          *reinterpret_cast<uint4*>(yb + (size_t)row * a.y_st.l + 8 * c8) =
              *reinterpret_cast<const uint4*>(sm + kVd + umma::sw128_off(row, c8));
        }
      }
      if (c + 1 < nchunk) prefetch_k(c + 1);
      umma::fence_before_sync();
      slot_sync(slot);
      umma::fence_after_sync();
      M3_TC_MARK(6);
    }

    if (so.tiles) {
      slot_sync(slot);
      dump_state_tile(nchunk);
    }
    // ---- final state (kernel_fwd.py:189-201) ---------------------------------------------
    if (a.final_ssm) {
      float sv[32];
      umma::fence_after_sync();
      umma::tmem_ld32(tm + lane_base + 192 + 32 * half, sv);
      umma::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) a.final_ssm[(bh * kP + 32 * half + i) * kN + t] = sv[i];
    }
    if (a.final_v && ltid < kP) {
      const __nv_bfloat16* vr = v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h + (size_t)(L - 1) * a.v_st.l;
      a.final_v[bh * kP + ltid] = __bfloat162float(vr[ltid]);
    }
    if (a.final_phi) {
      if (RAW) {
        if (lane == 0 && 8 * lwarp < Nr)
#pragma unroll
          for (int r = 0; r < 8; ++r) a.final_phi[bh * Nr + 8 * lwarp + r] = carry8[r];
      } else if (ltid < Nr) {
        a.final_phi[bh * Nr + ltid] = a.phi[(bh * L + L - 1) * Nr + ltid];
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) umma::tmem_dealloc(cs->tmem, 512);
}

}  // namespace tc
}  // namespace m3
