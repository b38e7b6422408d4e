// Warp-specialised, TMA-fed tcgen05 forward for the production shape (raw boundary,
// bf16 I/O and operands, N = 128, P = 64, 128-token chunks, n_angles % 8 == 0).
//
// One persistent CTA per SM walks (b, h) sequences; inside a sequence the chunks flow
// through a two-stage pipeline whose roles run concurrently:
//
//   warp 0      TMA producer: q, k rows (two 64-column SWIZZLE_128B boxes each) and the
//               v rows of chunk c into stage c & 1, completion on an mbarrier.
//   warp 1      tcgen05 issuer (one thread):  S = q~ khat^T, Yi = q~ St^T, the state
//               update St += khat^T vd, then Ya = P v for the previous chunk.
//   warp 2      per-token scalars one chunk ahead: softplus / sigmoid / heavy-tail,
//               gamma, the trapezoid scale (with the successor token), the log2 decay
//               prefix A.
//   warp 3      y out and z in: TMA store of each chunk's y tile, TMA load of the next z.
//   warps 4-11  rotary (256 threads): cumulative angles of the chunk (lane = 4 tokens x
//               one 8-angle group; serial + lane + cross-warp scans), sin / cos on the
//               SFU, rotation of q and k in place into the q~ / khat operand tiles, and
//               the v exp2(A_last - A) tile of the state update.  Needs nothing of the
//               state, so it runs a chunk ahead of the tensor core.
//   warps 12-15 state and output (thread = TMEM lane): the state pass (bf16 state tile for
//               the next readout, scaling by the next chunk's exp2(A_last), final state),
//               the decay mask S -> P (bf16, into TMEM over the S columns just read), the
//               accumulator seed exp2(A) Yi + (D + gamma u.w) v, the gated output.  In the
//               states-only mode, which has no output, they instead rotate half of each
//               chunk's k rows two chunks ahead (the rotary warps pass the angles through
//               the unused q tile), so the rotary warps, the critical role, do half the
//               rotation.
//
// TMEM (512 columns): S[2] 0..255, Yi[2] 256..383, the fp32 state 384..447 (lane n,
// column p), the output accumulator 448..511; the bf16 mask P of a chunk is written over
// the first 64 columns of its S buffer once they are read (the A operand of Ya).  Shared
// memory: two 96 KB stages {q~ 32K, khat 32K, v 16K, vd 16K}, the bf16 state tile 16K; the
// vd tile of a stage later holds that chunk's z and then its y.  The q / k rows of a stage
// are refilled as soon as the chunk's first MMAs are done, its v rows after Ya.
//
// The math is kernel_fwd.py:55-201 of the reference with reference.py:104-199's
// preprocessing fused in; the bf16 rounding points are the reference kernel's
// (q~, khat, v, the state at the readout, the masked scores, the decayed v).  Two
// differences, both inside the bf16 bound: u.w of the skip term is read off the S
// diagonal (S_ii = scale_i u_i.w_i up to the operand rounding), and the gate's sigmoid
// uses the SFU tanh.  Every wait is bounded (about 2 s of SM clock); a time-out records
// an error code in g_m3_device_error, raises a CTA-wide abort flag and every role winds
// down, waits for its own copies and frees TMEM.
#pragma once

#include <cuda.h>

#include "m3_chunk_common.cuh"
#include "m3_umma.cuh"

namespace m3 {
namespace ws {

constexpr int kN = 128, kP = 64, kC = 128;
constexpr int kThreads = 512;
constexpr uint32_t kStageBytes = 98304;
constexpr uint32_t kOQ = 0, kOK = 32768, kOV = 65536, kOVD = 81920;
constexpr uint32_t kOST = 2 * kStageBytes;     // bf16 state tile (B operand of Yi)
constexpr uint32_t kOSmall = kOST + 16384;
constexpr uint32_t kTS = 0, kTYi = 256, kTSt = 384, kTAcc = 448;
constexpr long long kWaitLimit = 4000000000LL;  // SM cycles
constexpr uint32_t kSuspendNs = 1u << 20;        // try_wait may park the warp this long

struct Small {
  // per-token scalars of three chunks in flight (chunk g in slot g % 3); cf = the decay
  // from a token to the end of its 32-token block, exp2(A_{block end} - A)
  float dt[3][kC], scl[3][kC], A[3][kC], gam[3][kC], cf[3][kC];
  float part[2][8][64];  // per rot warp: angle sums of its 16 tokens
  float cbuf[2][64];     // angle carry into the next chunk (written by the last rot warp)
  // this sequence's biases for rotary pair e (0..3) of group g: [.][e][0][g] = q (lo, lo+1,
  // hi, hi+1), [.][e][1][g] = the same for k; two copies by sequence parity.  A quarter-warp
  // (eight groups) reads 128 contiguous bytes.
  float bias[2][4][2][8][4];
  uint64_t full_qk[2], full_v[2], rot_done[2], mma1[2], mma2[2], p_ready[2], yfree[2], zfull[2], ystaged[2];
  uint64_t ang_ready[2];  // states-only mode: angles of the tokens the state warps rotate
  uint64_t scal_ready[3], scal_free[3];
  uint64_t state_ready, drain;
  uint32_t tmem;
  int abort_flag;
#ifdef M3_WS_TIMING
  unsigned int tacc[128], tcnt[128];  // per-CTA cycle sums and counts by code
#endif
};
constexpr size_t kSmemBytes = kOSmall + sizeof(Small) + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "more shared memory than a B200 CTA can have");

// Arguments beyond M3FwdArgs.
struct Extra {
  const float* T;  // tanh(angles) / 2 (turns), (B, L, Nr) contiguous; NULL = computed here
  uint8_t* tiles;  // backward workspace: chunk-start bf16 state tiles (NULL = not saved)
  float* phis;     //                     chunk-start angle carries
  int nunits;
};

// ---- small PTX helpers ----------------------------------------------------------------
__device__ __forceinline__ void arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_u32(mbar)) : "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(umma::smem_u32(mbar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load3(void* dst, const CUtensorMap* tm, int x, int y, int z, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(umma::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(umma::smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void tma_load4(void* dst, const CUtensorMap* tm, int x, int y, int z, int w,
                                          uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(umma::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(umma::smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void tma_store4(const CUtensorMap* tm, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(umma::smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Barrier over the 256 rotary threads that ORs `pred` across them.
__device__ __forceinline__ bool rot_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, 256, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

#ifdef M3_WS_TIMING
// Diagnostic builds only: cycles spent in each wait site / phase (index = code) and counts.
__device__ unsigned long long g_ws_wait[2][128];
#define WS_MARK(code)                                                         \
  do {                                                                        \
    if ((threadIdx.x & 31) == 0) {                                            \
      const long long now_ = clock64();                                       \
      atomicAdd(&sm->tacc[code], (unsigned int)(now_ - tmark_));              \
      atomicAdd(&sm->tcnt[code], 1u);                                         \
      tmark_ = now_;                                                          \
    }                                                                         \
  } while (0)
#define WS_MARK_INIT long long tmark_ = clock64()
#else
#define WS_MARK(code) \
  do {                \
  } while (0)
#define WS_MARK_INIT
#endif

// Bounded wait on phase `parity` of `mbar`; false on time-out or when another role
// already gave up (the CTA-wide abort flag).
__device__ __forceinline__ bool wait(Small* sm, uint64_t* mbar, uint32_t parity, int code) {
  const uint32_t a = umma::smem_u32(mbar);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(kSuspendNs)
        : "memory");
#ifdef M3_WS_TIMING
    if (done && (threadIdx.x & 31) == 0) {
      atomicAdd(&sm->tacc[code], (unsigned int)(clock64() - t0));
      atomicAdd(&sm->tcnt[code], 1u);
    }
#endif
    if (done) return true;
    if (*(volatile int*)&sm->abort_flag) return false;
    if (clock64() - t0 > kWaitLimit) {
      *(volatile int*)&sm->abort_flag = 1;
      atomicExch(&g_m3_device_error, code);
      return false;
    }
  }
}
// The same for every lane of a warp, with one answer for the whole warp.
__device__ __forceinline__ bool wait_warp(Small* sm, uint64_t* mbar, uint32_t parity, int code) {
  return __all_sync(0xffffffffu, wait(sm, mbar, parity, code));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) { umma::tmem_ld32(taddr, v); }

// D[tmem] (+)= A[tmem] * B[smem] (kind::f16; A is M = 128 lanes x K packed two bf16 per
// 32-bit column).  Issued by one thread.
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
}

// 8 consecutive fp32 TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = __uint_as_float(r[q]);
}
// 4 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// x - round_to_nearest(x) for |x| < 2^22, on the FMA pipe (round-to-nearest of the sum
// with 1.5 * 2^23 leaves the integer part).
__device__ __forceinline__ float frac_centered(float x) {
  const float r = (x + 12582912.f) - 12582912.f;
  return x - r;
}

__device__ __forceinline__ uint4 tc_pack8(const float* f) {
  return make_uint4(umma::pack_bf16x2(f[0], f[1]), umma::pack_bf16x2(f[2], f[3]), umma::pack_bf16x2(f[4], f[5]),
                    umma::pack_bf16x2(f[6], f[7]));
}

// Eight consecutive floats: one 256-bit load when the address is 32-byte aligned.
__device__ __forceinline__ void ld8(const float* p, bool al32, float (&v)[8]) {
  if (al32) {
    ldg8(p, v);
  } else {
    const float4 lo = *reinterpret_cast<const float4*>(p), hi = *reinterpret_cast<const float4*>(p + 4);
    v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
    v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
  }
}

__device__ __forceinline__ float sin_approx(float x) {
  float y;
  asm("sin.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float cos_approx(float x) {
  float y;
  asm("cos.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// tanh(angles) / 2, the head-shared rotary rate in turns (pi radians = half a turn), into a
// (B, L, Nr) buffer: computed once per (b, t, r) instead of once per head inside the scan.
__global__ void angle_rate_kernel(const float* __restrict__ angles, M3Strides st, int B, int L, int Nr,
                                  float* __restrict__ T) {
  const int q = Nr / 4;
  const size_t n = (size_t)B * L * q;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int r4 = (int)(i % q);
    const size_t bl = i / q;
    const int t = (int)(bl % L), b = (int)(bl / L);
    const float4 x = *reinterpret_cast<const float4*>(angles + (size_t)b * st.b + (size_t)t * st.l + 4 * r4);
    float4 y;
    y.x = tanh_acc(x.x) * 0.5f;
    y.y = tanh_acc(x.y) * 0.5f;
    y.z = tanh_acc(x.z) * 0.5f;
    y.w = tanh_acc(x.w) * 0.5f;
    *reinterpret_cast<float4*>(T + bl * Nr + 4 * r4) = y;
  }
}

// ST: states only -- no y; the k rotation, the state update and the state pass alone (the
// backward's chunk-start states, or pass 1 of a split over the sequence length).
template <bool PRE_T, bool ST>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_ws_kernel(const __grid_constant__ M3FwdArgs a, const __grid_constant__ CUtensorMap tq,
                  const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                  const __grid_constant__ CUtensorMap tz, const __grid_constant__ CUtensorMap ty, const Extra ex) {
  extern __shared__ uint8_t smraw[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  Small* sm = (Small*)(base + kOSmall);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.dims.nheads, L = a.dims.seqlen, Nr = a.dims.n_angles;
  const int nchunk = L / kC;
  const bool saving = ex.tiles != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 3; ++s) {
      umma::mbar_init(&sm->scal_ready[s], 1);
      umma::mbar_init(&sm->scal_free[s], 12);
    }
    for (int s = 0; s < 2; ++s) {
      umma::mbar_init(&sm->full_qk[s], 1);
      umma::mbar_init(&sm->full_v[s], 1);
      umma::mbar_init(&sm->rot_done[s], ST ? 12 : 8);  // states-only: the state warps rotate too
      umma::mbar_init(&sm->ang_ready[s], 8);
      umma::mbar_init(&sm->mma1[s], 1);
      umma::mbar_init(&sm->mma2[s], 1);
      umma::mbar_init(&sm->p_ready[s], 4);
      umma::mbar_init(&sm->yfree[s], 1);
      umma::mbar_init(&sm->zfull[s], 1);
      umma::mbar_init(&sm->ystaged[s], 4);
    }
    umma::mbar_init(&sm->state_ready, 4);
    umma::mbar_init(&sm->drain, 1);
    sm->abort_flag = 0;
    umma::fence_mbar_init();
  }
#ifdef M3_WS_TIMING
  if (threadIdx.x < 128) sm->tacc[threadIdx.x] = sm->tcnt[threadIdx.x] = 0u;
#endif
  if (warp == 1) umma::tmem_alloc(&sm->tmem, 512);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = sm->tmem;
  if (warp < 4) {
  if (warp == 0) {
    // ================================ TMA producer =================================
    if (lane == 0) {
      uint32_t G = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
        const int b = u / H, h = u % H;
        for (int c = 0; c < nchunk; ++c, ++G) {
          const int s = G & 1;
          uint8_t* st = base + s * kStageBytes;
          const int t0 = c * kC;
          // q / k: free once chunk G-2's S, Yi and state update have read them
          if (G >= 2 && !(ok = wait(sm, &sm->mma1[s], ((G - 2) >> 1) & 1, 21))) break;
          expect_tx(&sm->full_qk[s], ST ? 32768 : 2 * 32768);
          if (!ST) {
            tma_load3(st + kOQ, &tq, 0, t0, b, &sm->full_qk[s]);
            tma_load3(st + kOQ + 16384, &tq, 64, t0, b, &sm->full_qk[s]);
          }
          tma_load3(st + kOK, &tk, 0, t0, b, &sm->full_qk[s]);
          tma_load3(st + kOK + 16384, &tk, 64, t0, b, &sm->full_qk[s]);
          // v: free once chunk G-2's Ya has read it
          if (!ST && G >= 2 && !(ok = wait(sm, &sm->mma2[s], ((G - 2) >> 1) & 1, 22))) break;
          expect_tx(&sm->full_v[s], 16384);
          tma_load4(st + kOV, &tv, 0, t0, h, b, &sm->full_v[s]);
        }
      }
      if (!ok) {  // loads in flight land before the CTA exits
        for (uint32_t g = (G >= 2 ? G - 2 : 0); g <= G; ++g) {
          for (int w = 0; w < 2; ++w) {
            uint32_t done = 0;
            const long long t0 = clock64();
            uint64_t* mb = w ? &sm->full_v[g & 1] : &sm->full_qk[g & 1];
            while (!done && clock64() - t0 < kWaitLimit / 8) {
              asm volatile(
                  "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                  "selp.u32 %0, 1, 0, p;\n\t}\n"
                  : "=r"(done)
                  : "r"(umma::smem_u32(mb)), "r"((g >> 1) & 1)
                  : "memory");
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ================================ tcgen05 issuer ================================
    if (lane == 0) {
      constexpr uint32_t id_s = umma::idesc_bf16(128, 128, false, false);
      constexpr uint32_t id_yi = umma::idesc_bf16(128, 64, false, true);
      constexpr uint32_t id_ds = umma::idesc_bf16(128, 64, true, true);
      const uint32_t sST = umma::smem_u32(base + kOST);
      auto issue_ya = [&](uint32_t Gp) -> bool {
        const int sp = Gp & 1;
        if (!wait(sm, &sm->p_ready[sp], (Gp >> 1) & 1, 31)) return false;
        umma::fence_after_sync();
        const uint32_t sV = umma::smem_u32(base + sp * kStageBytes + kOV);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)  // A = P from TMEM: 16 bf16 of K per step = 8 columns
          mma_bf16_tmem_a(tm + kTAcc, tm + kTS + 128 * sp + 8 * ks, umma::smem_desc(sV + ks * 2048u, 16384, 1024),
                          id_yi, true);
        umma::commit(&sm->mma2[sp]);
        return true;
      };
      uint32_t G = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
        for (int c = 0; c < nchunk; ++c, ++G) {
          const int s = G & 1;
          const uint32_t sQ = umma::smem_u32(base + s * kStageBytes + kOQ);
          const uint32_t sK = umma::smem_u32(base + s * kStageBytes + kOK);
          const uint32_t sVd = umma::smem_u32(base + s * kStageBytes + kOVD);
          if (!(ok = wait(sm, &sm->rot_done[s], (G >> 1) & 1, 32))) break;
          umma::fence_after_sync();
#pragma unroll
          for (int ks = 0; ks < (ST ? 0 : 8); ++ks) {
            const uint32_t kmaj = (ks >> 2) * 16384u + (ks & 3) * 32u;
            umma::mma_bf16(tm + kTS + 128 * s, umma::smem_desc(sQ + kmaj, 16, 1024),
                           umma::smem_desc(sK + kmaj, 16, 1024), id_s, ks > 0);
          }
          if (!(ok = wait(sm, &sm->state_ready, G & 1, 33))) break;
          umma::fence_after_sync();
#pragma unroll
          for (int ks = 0; ks < (ST ? 0 : 8); ++ks) {
            const uint32_t kmaj = (ks >> 2) * 16384u + (ks & 3) * 32u;
            umma::mma_bf16(tm + kTYi + 64 * s, umma::smem_desc(sQ + kmaj, 16, 1024),
                           umma::smem_desc(sST + ks * 2048u, 16384, 1024), id_yi, ks > 0);
          }
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t mn = ks * 2048u;
            umma::mma_bf16(tm + kTSt, umma::smem_desc(sK + mn, 16384, 1024), umma::smem_desc(sVd + mn, 16384, 1024),
                           id_ds, true);
          }
          umma::commit(&sm->mma1[s]);
          if (!ST && c > 0 && !(ok = issue_ya(G - 1))) break;
        }
        if (!ST && ok && !(ok = issue_ya(G - 1))) break;
      }
      // every MMA issued has completed before TMEM is freed
      umma::commit(&sm->drain);
      uint32_t done = 0;
      const long long t0 = clock64();
      while (!done && clock64() - t0 < kWaitLimit / 4) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(umma::smem_u32(&sm->drain))
            : "memory");
      }
    }
  } else if (warp == 2) {
    // ================================ per-token scalars =============================
    uint32_t G = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
      const int b = u / H, h = u % H;
      const float dtb = a.dt_bias[h];
      float rdt[4], ra[4], rtr[4], sdt = 0.f, str = 0.f;
      auto load_raw = [&](int c) {
        const int t = c * kC + 4 * lane;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const size_t o = (size_t)b * a.raw_st.b + (size_t)(t + j) * a.raw_st.l + (size_t)h * a.raw_st.h;
          rdt[j] = a.dt_raw[o];
          ra[j] = a.a_raw[o];
          rtr[j] = a.trap_raw[o];
        }
        if (lane == 31 && c * kC + kC < L) {
          const size_t o = (size_t)b * a.raw_st.b + (size_t)(c * kC + kC) * a.raw_st.l + (size_t)h * a.raw_st.h;
          sdt = a.dt_raw[o];
          str = a.trap_raw[o];
        }
      };
      load_raw(0);
      for (int c = 0; c < nchunk; ++c, ++G) {
        float dt[4], lam[4], adt[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          dt[j] = softplusf(rdt[j] + dtb);
          lam[j] = sigmoidf_(rtr[j]);
          adt[j] = fminf(-heavy_tail(ra[j]), -a.a_floor) * dt[j];
        }
        float dtn = __shfl_down_sync(0xffffffffu, dt[0], 1), lamn = __shfl_down_sync(0xffffffffu, lam[0], 1);
        if (lane == 31) {
          const bool more = c * kC + kC < L;
          dtn = more ? softplusf(sdt + dtb) : 0.f;
          lamn = more ? sigmoidf_(str) : 0.f;
        }
        float gam[4], scl[4], A[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gam[j] = dt[j] * lam[j];
          const float dn = j < 3 ? dt[j + 1] : dtn, ln = j < 3 ? lam[j + 1] : lamn;
          scl[j] = gam[j] + dn * (1.f - ln);
        }
        float run = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          run += adt[j] * kLog2e;
          A[j] = run;
        }
        const float incl = warp_inclusive_scan(run);
        const float off = incl - run;
#pragma unroll
        for (int j = 0; j < 4; ++j) A[j] += off;
        if (c + 1 < nchunk) load_raw(c + 1);  // next chunk's raw values in flight
        const float Ae = __shfl_sync(0xffffffffu, A[3], lane | 7);  // end of this 32-token block
        const int s3 = G % 3;
        if (G >= 3 && !(ok = wait_warp(sm, &sm->scal_free[s3], (G / 3 - 1) & 1, 41))) break;
        *reinterpret_cast<float4*>(&sm->dt[s3][4 * lane]) = make_float4(dt[0], dt[1], dt[2], dt[3]);
        *reinterpret_cast<float4*>(&sm->scl[s3][4 * lane]) = make_float4(scl[0], scl[1], scl[2], scl[3]);
        *reinterpret_cast<float4*>(&sm->A[s3][4 * lane]) = make_float4(A[0], A[1], A[2], A[3]);
        *reinterpret_cast<float4*>(&sm->gam[s3][4 * lane]) = make_float4(gam[0], gam[1], gam[2], gam[3]);
        *reinterpret_cast<float4*>(&sm->cf[s3][4 * lane]) =
            make_float4(ex2(Ae - A[0]), ex2(Ae - A[1]), ex2(Ae - A[2]), ex2(Ae - A[3]));
        __syncwarp();
        if (lane == 0) arrive(&sm->scal_ready[s3]);
      }
    }
  } else if (warp == 3 && !ST) {
    // ================================ y out, z in ===================================
    if (lane == 0) {
      uint32_t G = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
        const int b = u / H, h = u % H;
        for (int c = 0; c < nchunk; ++c, ++G) {
          const int s = G & 1;
          uint8_t* vd = base + s * kStageBytes + kOVD;
          if (a.z) {  // the vd tile is free once the state update has read it
            if (!(ok = wait(sm, &sm->mma1[s], (G >> 1) & 1, 51))) break;
            expect_tx(&sm->zfull[s], 16384);
            tma_load4(vd, &tz, 0, c * kC, h, b, &sm->zfull[s]);
          }
          if (!(ok = wait(sm, &sm->ystaged[s], (G >> 1) & 1, 52))) break;
          tma_store4(&ty, vd, 0, c * kC, h, b);
          bulk_commit();
          bulk_wait_read();
          arrive(&sm->yfree[s]);
        }
      }
      bulk_wait_all();
    }
  }
  } else {
  if (warp < 12) {
    // ================================ rotary =========================================
    const int r = warp - 4, p = lane >> 3, g = lane & 7;
    const int tl = 16 * r + 4 * p;  // first of this thread's four tokens in the chunk
    const bool grot = 8 * g < Nr;
    const bool ang32 = (uintptr_t)a.angles % 32 == 0 && a.ang_st.l % 8 == 0 && a.ang_st.b % 8 == 0;
    uint32_t G = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
      const int b = u / H, h = u % H;
      const size_t bh = (size_t)u;
      if (r == 0 && p == 0) {  // this head's biases of group g into shared memory
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float* qb = a.q_bias + h * kN + 8 * g + 2 * e;
          const float* kb = a.k_bias + h * kN + 8 * g + 2 * e;
          *reinterpret_cast<float4*>(sm->bias[u & 1][e][0][g]) = make_float4(qb[0], qb[1], qb[64], qb[65]);
          *reinterpret_cast<float4*>(sm->bias[u & 1][e][1][g]) = make_float4(kb[0], kb[1], kb[64], kb[65]);
        }
      }
      float carry[8];  // angles are carried in turns
#pragma unroll
      for (int e = 0; e < 8; ++e)
        carry[e] = (grot && a.seed_phi) ? a.seed_phi[bh * Nr + 8 * g + e] * 0.15915494309189535f : 0.f;
      // rotary rates tanh(angles) / 2 of this thread's 4 tokens x 8 angles of chunk `cc`
      float th[4][8];
      auto load_rates = [&](int cc) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (grot) {
            if constexpr (PRE_T) {
              ldg8(ex.T + ((size_t)b * L + cc * kC + tl + j) * Nr + 8 * g, th[j]);
            } else {
              const float* pa = a.angles + (size_t)b * a.ang_st.b + (size_t)(cc * kC + tl + j) * a.ang_st.l + 8 * g;
              ld8(pa, ang32, th[j]);
#pragma unroll
              for (int e = 0; e < 8; ++e) th[j][e] = tanh_acc(th[j][e]) * 0.5f;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) th[j][e] = 0.f;
          }
        }
      };
      bool yok = true;
      for (int c = 0; c < nchunk; ++c, ++G) {
        const int s = G & 1;
        const int t0 = c * kC;
        uint8_t* st = base + s * kStageBytes;
        WS_MARK_INIT;
        load_rates(c);
        const int s3 = G % 3;
        bool wok = yok && wait_warp(sm, &sm->scal_ready[s3], (G / 3) & 1, 61);
        WS_MARK(81);
        const float4 dt4 = *reinterpret_cast<const float4*>(&sm->dt[s3][tl]);
        const float dtj[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
        // ---- angle increments (rates loaded one chunk ahead), serial prefix ----------
        float x[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) x[j][e] = th[j][e] * dtj[j];
#pragma unroll
        for (int j = 1; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) x[j][e] += x[j - 1][e];
        // ---- across the 4 token quads of the warp (lanes g, g+8, g+16, g+24) ---------
        float excl[8], tot[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float tt = x[3][e];
          float y = __shfl_up_sync(0xffffffffu, tt, 8);
          if (p >= 1) tt += y;
          y = __shfl_up_sync(0xffffffffu, tt, 16);
          if (p >= 2) tt += y;
          tot[e] = tt;  // inclusive over quads 0 .. p (the warp's total at p == 3)
          excl[e] = __shfl_up_sync(0xffffffffu, tt, 8);
          if (p == 0) excl[e] = 0.f;
        }
        if (p == 3) {
          *reinterpret_cast<float4*>(&sm->part[s][r][8 * g]) = make_float4(tot[0], tot[1], tot[2], tot[3]);
          *reinterpret_cast<float4*>(&sm->part[s][r][8 * g + 4]) = make_float4(tot[4], tot[5], tot[6], tot[7]);
        }
        WS_MARK(82);
        if (rot_any(!wok)) {
          ok = false;
          break;
        }
        WS_MARK(83);
        // ---- carry into this warp's first token --------------------------------------
        float bse[8];
        if (c > 0) {
          const float4 c0 = *reinterpret_cast<const float4*>(&sm->cbuf[s ^ 1][8 * g]);
          const float4 c1 = *reinterpret_cast<const float4*>(&sm->cbuf[s ^ 1][8 * g + 4]);
          bse[0] = c0.x; bse[1] = c0.y; bse[2] = c0.z; bse[3] = c0.w;
          bse[4] = c1.x; bse[5] = c1.y; bse[6] = c1.z; bse[7] = c1.w;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) bse[e] = carry[e];
        }
        if (saving && r == 0 && p == 0 && grot) {  // radians in [0, 2 pi), as the backward reads them
          float* dst = ex.phis + (bh * nchunk + c) * Nr + 8 * g;
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = (bse[e] - floorf(bse[e])) * kTwoPi;
        }
        for (int rr = 0; rr < r; ++rr) {
          const float4 p0 = *reinterpret_cast<const float4*>(&sm->part[s][rr][8 * g]);
          const float4 p1 = *reinterpret_cast<const float4*>(&sm->part[s][rr][8 * g + 4]);
          bse[0] += p0.x; bse[1] += p0.y; bse[2] += p0.z; bse[3] += p0.w;
          bse[4] += p1.x; bse[5] += p1.y; bse[6] += p1.z; bse[7] += p1.w;
        }
        if (r == 7 && p == 0) {
          const float4 p0 = *reinterpret_cast<const float4*>(&sm->part[s][7][8 * g]);
          const float4 p1 = *reinterpret_cast<const float4*>(&sm->part[s][7][8 * g + 4]);
          const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
          float nx[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float t = bse[e] + pv[e];
            nx[e] = t - floorf(t);  // turns in [0, 1)
          }
          *reinterpret_cast<float4*>(&sm->cbuf[s][8 * g]) = make_float4(nx[0], nx[1], nx[2], nx[3]);
          *reinterpret_cast<float4*>(&sm->cbuf[s][8 * g + 4]) = make_float4(nx[4], nx[5], nx[6], nx[7]);
          if (c == nchunk - 1 && a.final_phi && grot)
#pragma unroll
            for (int e = 0; e < 8; ++e) a.final_phi[bh * Nr + 8 * g + e] = nx[e] * kTwoPi;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) bse[e] += excl[e];
        // absolute angles (turns) of the four tokens; the token loop below is rolled to keep
        // the code small, so it always works on ph[0] and shifts the array by one
        float ph[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) ph[j][e] = bse[e] + x[j][e];
        WS_MARK(84);
        wok = wait_warp(sm, &sm->full_qk[s], (G >> 1) & 1, 62);
        yok = yok && wok;
        WS_MARK(85);
        // ---- rotation of the four tokens --------------------------------------------
        const float4 sc4 = *reinterpret_cast<const float4*>(&sm->scl[s3][tl]);
        const float sclj[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
        uint8_t* sQ = st + kOQ;
        uint8_t* sK = st + kOK;
        float sclr = sclj[0];
        // states-only mode: the state warps, idle but for the state pass, rotate the last two
        // tokens of every quad; their absolute angles (turns) go through the q tile, which
        // this mode does not load
        constexpr int kRotTok = ST ? 2 : 4;
#pragma unroll 1
        for (int j = 0; j < kRotTok; ++j) {
          const int t = tl + j;
          // sin / cos of the angle reduced to [-pi, pi] (the SFU's accurate range)
          float cs[8], sn[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (grot) {
              const float xs = frac_centered(ph[0][e]) * kTwoPi;
#ifdef M3_ABL_NO_SFU  // diagnostic ablation: timing only, wrong values
              cs[e] = 1.f - 0.5f * xs * xs;
              sn[e] = xs;
#else
              cs[e] = cos_approx(xs);
              sn[e] = sin_approx(xs);
#endif
            } else {
              cs[e] = 1.f;
              sn[e] = 0.f;
            }
          }
          const uint32_t soff = umma::sw128_off(t, g);
          const uint4 uql = *reinterpret_cast<const uint4*>(sQ + soff);
          const uint4 uqh = *reinterpret_cast<const uint4*>(sQ + 16384 + soff);
          const uint4 ukl = *reinterpret_cast<const uint4*>(sK + soff);
          const uint4 ukh = *reinterpret_cast<const uint4*>(sK + 16384 + soff);
          const uint32_t ql[4] = {uql.x, uql.y, uql.z, uql.w}, qh[4] = {uqh.x, uqh.y, uqh.z, uqh.w};
          const uint32_t kl[4] = {ukl.x, ukl.y, ukl.z, ukl.w}, kh[4] = {ukh.x, ukh.y, ukh.z, ukh.w};
          const float2 sc2 = f2s(sclr);

          const bool fin = a.final_k && c == nchunk - 1 && t == kC - 1;
          uint32_t oq_lo[4], oq_hi[4], ok_lo[4], ok_hi[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 c2 = f2(cs[2 * e], cs[2 * e + 1]), s2 = f2(sn[2 * e], sn[2 * e + 1]);
            const float4 bq = *reinterpret_cast<const float4*>(sm->bias[u & 1][e][0][g]);
            const float4 bk = *reinterpret_cast<const float4*>(sm->bias[u & 1][e][1][g]);
            const float2 ulo = add2(bf2f(ql[e]), f2(bq.x, bq.y));
            const float2 uhi = add2(bf2f(qh[e]), f2(bq.z, bq.w));
            const float2 wlo = add2(bf2f(kl[e]), f2(bk.x, bk.y));
            const float2 whi = add2(bf2f(kh[e]), f2(bk.z, bk.w));
            // lo' = lo cos - hi sin;  hi' = lo sin + hi cos
#ifdef M3_ABL_NO_ROT  // diagnostic ablation: timing only, wrong values
            const float2 qlo = add2(ulo, c2), qhi = add2(uhi, s2), klo = add2(wlo, c2), khi = add2(whi, s2);
#else
            const float2 ns2 = f2(-s2.x, -s2.y);
            const float2 qlo = fma2(uhi, ns2, mul2(ulo, c2));
            const float2 qhi = fma2(ulo, s2, mul2(uhi, c2));
            const float2 klo = fma2(whi, ns2, mul2(wlo, c2));
            const float2 khi = fma2(wlo, s2, mul2(whi, c2));
#endif
            if (fin) {  // the final k is rotated but unscaled (kernel_fwd.py:192-201)
              float* fk = a.final_k + bh * kN + 8 * g + 2 * e;
              fk[0] = klo.x;
              fk[1] = klo.y;
              fk[64] = khi.x;
              fk[65] = khi.y;
            }
            oq_lo[e] = f2bf(qlo);
            oq_hi[e] = f2bf(qhi);
            ok_lo[e] = f2bf(mul2(klo, sc2));
            ok_hi[e] = f2bf(mul2(khi, sc2));
          }
          if (!ST) {
            *reinterpret_cast<uint4*>(sQ + soff) = make_uint4(oq_lo[0], oq_lo[1], oq_lo[2], oq_lo[3]);
            *reinterpret_cast<uint4*>(sQ + 16384 + soff) = make_uint4(oq_hi[0], oq_hi[1], oq_hi[2], oq_hi[3]);
          }
          *reinterpret_cast<uint4*>(sK + soff) = make_uint4(ok_lo[0], ok_lo[1], ok_lo[2], ok_lo[3]);
          *reinterpret_cast<uint4*>(sK + 16384 + soff) = make_uint4(ok_hi[0], ok_hi[1], ok_hi[2], ok_hi[3]);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            ph[0][e] = ph[1][e];
            ph[1][e] = ph[2][e];
            ph[2][e] = ph[3][e];
          }
          sclr = j == 0 ? sclj[1] : j == 1 ? sclj[2] : sclj[3];
        }
        if constexpr (ST) {  // ph[0], ph[1] now hold tokens tl + 2, tl + 3
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float* dst = reinterpret_cast<float*>(sQ + (tl + 2 + j) * 256 + 32 * g);
            *reinterpret_cast<float4*>(dst) = make_float4(ph[j][0], ph[j][1], ph[j][2], ph[j][3]);
            *reinterpret_cast<float4*>(dst + 4) = make_float4(ph[j][4], ph[j][5], ph[j][6], ph[j][7]);
          }
          __syncwarp();
          if (lane == 0) arrive(&sm->ang_ready[s]);
        }
        WS_MARK(86);
        // ---- vd = v exp2(A_last - A) for this warp's 16 rows --------------------------
        if (!ST && G >= 2) yok = yok && wait_warp(sm, &sm->yfree[s], ((G - 2) >> 1) & 1, 63);
        yok = yok && wait_warp(sm, &sm->full_v[s], (G >> 1) & 1, 64);
        WS_MARK(87);
        {
          const float Alast = sm->A[s3][kC - 1];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const int idx = lane + 32 * m, row = 16 * r + (idx >> 3), c8 = idx & 7;
            const float2 e2 = f2s(ex2(Alast - sm->A[s3][row]));
            const uint32_t off = umma::sw128_off(row, c8);
            const uint4 u4 = *reinterpret_cast<const uint4*>(st + kOV + off);
            *reinterpret_cast<uint4*>(st + kOVD + off) =
                make_uint4(f2bf(mul2(bf2f(u4.x), e2)), f2bf(mul2(bf2f(u4.y), e2)), f2bf(mul2(bf2f(u4.z), e2)),
                           f2bf(mul2(bf2f(u4.w), e2)));
          }
        }
        umma::fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          arrive(&sm->rot_done[s]);
          arrive(&sm->scal_free[s3]);
        }
        WS_MARK(88);
      }
      if (!ok) break;
    }
  } else {
    // ================================ state and output ===============================
    const int qd = warp & 3;
    const int i = 32 * qd + lane;  // TMEM lane: token row (S, Yi, acc) or state row n
    const uint32_t lrow = (uint32_t)(32 * qd) << 16;
    uint32_t G = 0;
    bool ok = true;
    // states-only mode: rotate tokens 4m + 2, 4m + 3 of chunk cr (pipeline index Gr) into the
    // khat tile, from the angles the rotary warps left in the q tile; then count towards
    // rot_done.  Item = (one of those 64 tokens, an 8-angle group); four per thread.
    auto st_rotate = [&](uint32_t Gr, int cr, int u_, size_t bh_) -> bool {
      const int sr = Gr & 1, s3r = Gr % 3;
      uint8_t* str = base + sr * kStageBytes;
      if (!wait_warp(sm, &sm->ang_ready[sr], (Gr >> 1) & 1, 76)) return false;
      if (!wait_warp(sm, &sm->full_qk[sr], (Gr >> 1) & 1, 77)) return false;
      uint8_t* sK = str + kOK;
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        const int idx = i + 128 * m, tok = idx >> 3, g = idx & 7;
        const int t = 4 * (tok >> 1) + 2 + (tok & 1);
        const bool grot = 8 * g < Nr;
        const float* ap = reinterpret_cast<const float*>(str + kOQ + t * 256 + 32 * g);
        const float4 a0 = *reinterpret_cast<const float4*>(ap), a1 = *reinterpret_cast<const float4*>(ap + 4);
        const float ang[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float cs[8], sn[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (grot) {
            const float xs = frac_centered(ang[e]) * kTwoPi;
            cs[e] = cos_approx(xs);
            sn[e] = sin_approx(xs);
          } else {
            cs[e] = 1.f;
            sn[e] = 0.f;
          }
        }
        const uint32_t soff = umma::sw128_off(t, g);
        const uint4 ukl = *reinterpret_cast<const uint4*>(sK + soff);
        const uint4 ukh = *reinterpret_cast<const uint4*>(sK + 16384 + soff);
        const uint32_t kl[4] = {ukl.x, ukl.y, ukl.z, ukl.w}, kh[4] = {ukh.x, ukh.y, ukh.z, ukh.w};
        const float2 sc2 = f2s(sm->scl[s3r][t]);
        const bool fin = a.final_k && cr == nchunk - 1 && t == kC - 1;
        uint32_t ok_lo[4], ok_hi[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 c2 = f2(cs[2 * e], cs[2 * e + 1]), s2 = f2(sn[2 * e], sn[2 * e + 1]);
          const float4 bk = *reinterpret_cast<const float4*>(sm->bias[u_ & 1][e][1][g]);
          const float2 wlo = add2(bf2f(kl[e]), f2(bk.x, bk.y));
          const float2 whi = add2(bf2f(kh[e]), f2(bk.z, bk.w));
          const float2 ns2 = f2(-s2.x, -s2.y);
          const float2 klo = fma2(whi, ns2, mul2(wlo, c2));
          const float2 khi = fma2(wlo, s2, mul2(whi, c2));
          if (fin) {  // the final k is rotated but unscaled
            float* fk = a.final_k + bh_ * kN + 8 * g + 2 * e;
            fk[0] = klo.x;
            fk[1] = klo.y;
            fk[64] = khi.x;
            fk[65] = khi.y;
          }
          ok_lo[e] = f2bf(mul2(klo, sc2));
          ok_hi[e] = f2bf(mul2(khi, sc2));
        }
        *reinterpret_cast<uint4*>(sK + soff) = make_uint4(ok_lo[0], ok_lo[1], ok_lo[2], ok_lo[3]);
        *reinterpret_cast<uint4*>(sK + 16384 + soff) = make_uint4(ok_hi[0], ok_hi[1], ok_hi[2], ok_hi[3]);
      }
      umma::fence_async_smem();
      __syncwarp();
      if (lane == 0) arrive(&sm->rot_done[sr]);
      return true;
    };
    for (int u = blockIdx.x; u < ex.nunits && ok; u += gridDim.x) {
      const int b = u / H, h = u % H;
      const size_t bh = (size_t)u;
      const float Dh = a.d_skip ? a.d_skip[h] : 0.f;
      const uint32_t G0 = G;
      uint8_t* sST = base + kOST;
      // ---- initial state: seed (+ the trapezoid seed term), scaled for chunk 0 --------
      {
        if (!(ok = wait_warp(sm, &sm->scal_ready[G0 % 3], (G0 / 3) & 1, 71))) break;
        float stv[32];
        float coef = 0.f, kprev = 0.f;
        if (a.seed_ssm) {
          const size_t o = (size_t)b * a.raw_st.b + (size_t)h * a.raw_st.h;
          coef = softplusf(a.dt_raw[o] + a.dt_bias[h]) * (1.f - sigmoidf_(a.trap_raw[o]));
          kprev = a.seed_k[bh * kN + i];
        }
        const float eA = exp2f(sm->A[G0 % 3][kC - 1]);
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            const int pp = 32 * hh + q;
            stv[q] = a.seed_ssm ? a.seed_ssm[(bh * kP + pp) * kN + i] + coef * a.seed_v[bh * kP + pp] * kprev : 0.f;
          }
          uint4 rowv[4];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            rowv[cc] = tc_pack8(stv + 8 * cc);
            *reinterpret_cast<uint4*>(sST + umma::sw128_off(i, 4 * hh + cc)) = rowv[cc];
          }
          if (saving) {
            uint8_t* dst = ex.tiles + (bh * (nchunk + 1)) * 16384u;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) *reinterpret_cast<uint4*>(dst + umma::sw128_off(i, 4 * hh + cc)) = rowv[cc];
          }
#pragma unroll
          for (int q = 0; q < 32; ++q) stv[q] *= eA;
          umma::tmem_st32(tm + lrow + kTSt + 32 * hh, stv);
        }
        umma::tmem_wait_st();
        umma::fence_async_smem();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) arrive(&sm->state_ready);
      }
      auto epilogue = [&](uint32_t Ge, int ce) -> bool {
        const int se = Ge & 1;
        uint8_t* vd = base + se * kStageBytes + kOVD;
        if (!wait_warp(sm, &sm->mma2[se], (Ge >> 1) & 1, 72)) return false;
        umma::fence_after_sync();
        if (a.z && !wait_warp(sm, &sm->zfull[se], (Ge >> 1) & 1, 73)) return false;
#pragma unroll 1
        for (int c2 = 0; c2 < 4; ++c2) {  // 16 output columns at a time: two TMEM loads per wait
          float acc[2][8];
          tmem_ld8(tm + lrow + kTAcc + 16 * c2, acc[0]);
          tmem_ld8(tm + lrow + kTAcc + 16 * c2 + 8, acc[1]);
          uint32_t zw[2][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
          if (a.z) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint4 zz = *reinterpret_cast<const uint4*>(vd + umma::sw128_off(i, 2 * c2 + hh));
              zw[hh][0] = zz.x; zw[hh][1] = zz.y; zw[hh][2] = zz.z; zw[hh][3] = zz.w;
            }
          }
          umma::tmem_wait_ld();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 o = f2(acc[hh][2 * e], acc[hh][2 * e + 1]);
              if (a.z) {
                const float2 zf = bf2f(zw[hh][e]);
                // silu(z) = z sigmoid(z) = z (0.5 + 0.5 tanh(z / 2))
                const float2 th = f2(tanh_approx(0.5f * zf.x), tanh_approx(0.5f * zf.y));
                o = mul2(o, mul2(zf, fma2(th, f2s(0.5f), f2s(0.5f))));
              }
              w[e] = f2bf(o);
            }
            *reinterpret_cast<uint4*>(vd + umma::sw128_off(i, 2 * c2 + hh)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        umma::fence_async_smem();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) arrive(&sm->ystaged[se]);
        if (ce == nchunk - 1 && a.final_v && i < kP) {
          const __nv_bfloat16* vr = (const __nv_bfloat16*)a.v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h +
                                    (size_t)(L - 1) * a.v_st.l;
          a.final_v[bh * kP + i] = __bfloat162float(vr[i]);
        }
        return true;
      };
      if constexpr (ST) {  // two chunks ahead of the state update they feed
        if (!(ok = st_rotate(G, 0, u, bh))) break;
        if (nchunk > 1 && !(ok = st_rotate(G + 1, 1, u, bh))) break;
      }
      for (int c = 0; c < nchunk; ++c, ++G) {
        const int s = G & 1;
        const bool last = c == nchunk - 1;
        WS_MARK_INIT;
        if (!(ok = wait_warp(sm, &sm->mma1[s], (G >> 1) & 1, 74))) break;
        umma::fence_after_sync();
        WS_MARK(91);
        // ---- state pass: bf16 tile for the next readout, scale for the next chunk ------
        {
          float eAn = 1.f;
          if (!last) {
            if (!(ok = wait_warp(sm, &sm->scal_ready[(G + 1) % 3], ((G + 1) / 3) & 1, 75))) break;
            eAn = exp2f(sm->A[(G + 1) % 3][kC - 1]);
          }
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            float stv[32];
            tmem_ld32(tm + lrow + kTSt + 32 * hh, stv);
            umma::tmem_wait_ld();
            // the bf16 tile is the B operand of the next chunk's Yi (none in states-only mode)
            // and what the backward reads when the states are saved
            if ((!ST && !last) || saving) {
              uint4 rowv[4];
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
                rowv[cc] = tc_pack8(stv + 8 * cc);
                if (!ST && !last) *reinterpret_cast<uint4*>(sST + umma::sw128_off(i, 4 * hh + cc)) = rowv[cc];
              }
              if (saving) {
                uint8_t* dst = ex.tiles + (bh * (nchunk + 1) + c + 1) * 16384u;
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                  *reinterpret_cast<uint4*>(dst + umma::sw128_off(i, 4 * hh + cc)) = rowv[cc];
              }
            }
            if (last) {
              if (a.final_ssm)
#pragma unroll
                for (int q = 0; q < 32; ++q) a.final_ssm[(bh * kP + 32 * hh + q) * kN + i] = stv[q];
            } else {
#pragma unroll
              for (int q = 0; q < 32; q += 2) {
                const float2 v2 = mul2(f2(stv[q], stv[q + 1]), f2s(eAn));
                stv[q] = v2.x;
                stv[q + 1] = v2.y;
              }
              umma::tmem_st32(tm + lrow + kTSt + 32 * hh, stv);
            }
          }
          if (!last) {
            umma::tmem_wait_st();
            umma::fence_async_smem();
            umma::fence_before_sync();
            __syncwarp();
            if (lane == 0) arrive(&sm->state_ready);
          }
        }
        WS_MARK(92);
        if constexpr (ST) {  // no output: the state pass is all; release this chunk's scalars
          __syncwarp();
          if (lane == 0) arrive(&sm->scal_free[G % 3]);
          if (last && a.final_v && i < kP) {
            const __nv_bfloat16* vr = (const __nv_bfloat16*)a.v + (size_t)b * a.v_st.b + (size_t)h * a.v_st.h +
                                      (size_t)(L - 1) * a.v_st.l;
            a.final_v[bh * kP + i] = __bfloat162float(vr[i]);
          }
          if (c + 2 < nchunk && !(ok = st_rotate(G + 2, c + 2, u, bh))) break;
          continue;
        }
        // ---- output of the previous chunk ------------------------------------------------
        if (c > 0 && !(ok = epilogue(G - 1, c - 1))) break;
        WS_MARK(93);
        // ---- decay mask S -> P (bf16, into TMEM over S's first 64 columns), acc seed ----
        {
          const int s3 = G % 3;
          const float* As = sm->A[s3];
          const float* Cf = sm->cf[s3];
          const float Ai = As[i];
          const uint32_t tS = tm + lrow + kTS + 128 * s;
          float sii = 0.f;
#pragma unroll 1
          for (int J = 0; J < 4; ++J) {
            // off-diagonal blocks: exp2(A_i - A_j) = exp2(A_i - A_end(J)) exp2(A_end(J) - A_j),
            // both factors <= 1; the diagonal block takes exp2(A_i - A_j) directly
            const float rf = J < qd ? ex2(Ai - As[32 * J + 31]) : 1.f;
            const float* fac = (J < qd ? Cf : As) + 32 * J;
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {  // 8 columns of S -> 4 packed columns of P
              uint32_t w[4] = {0u, 0u, 0u, 0u};
              if (J <= qd) {
                float sv[8];
                tmem_ld8(tS + 32 * J + 8 * cc, sv);
                const float4 a0 = *reinterpret_cast<const float4*>(fac + 8 * cc);
                const float4 a1 = *reinterpret_cast<const float4*>(fac + 8 * cc + 4);
                const float aj[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                umma::tmem_wait_ld();
                if (J < qd) {
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    w[e] = f2bf(mul2(mul2(f2(sv[2 * e], sv[2 * e + 1]), f2(aj[2 * e], aj[2 * e + 1])), f2s(rf)));
                } else {
                  const int j0 = 32 * J + 8 * cc;
#pragma unroll
                  for (int e = 0; e < 8; ++e) {
                    if (j0 + e == i) sii = sv[e];
                    sv[e] = j0 + e < i ? sv[e] * ex2(Ai - aj[e]) : 0.f;
                  }
#pragma unroll
                  for (int e = 0; e < 4; ++e) w[e] = f2bf(f2(sv[2 * e], sv[2 * e + 1]));
                }
              }
              // P columns 16J + 4cc .. +3 lie over S columns this thread has already read
              tmem_st4(tS + 16 * J + 4 * cc, w);
            }
          }
          const float scl = sm->scl[s3][i], gam = sm->gam[s3][i];
          const float dg = Dh + (scl > 0.f ? gam * sii * rcp_approx(scl) : 0.f);
          const float eA = ex2(Ai);
          const uint8_t* sV = base + s * kStageBytes + kOV;
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            float yi[32];
            tmem_ld32(tm + lrow + kTYi + 64 * s + 32 * hh, yi);
            umma::tmem_wait_ld();
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const uint4 vv = *reinterpret_cast<const uint4*>(sV + umma::sw128_off(i, 4 * hh + cc));
              const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 o = fma2(f2s(dg), bf2f(vw[e]), mul2(f2s(eA), f2(yi[8 * cc + 2 * e], yi[8 * cc + 2 * e + 1])));
                yi[8 * cc + 2 * e] = o.x;
                yi[8 * cc + 2 * e + 1] = o.y;
              }
            }
            umma::tmem_st32(tm + lrow + kTAcc + 32 * hh, yi);
          }
          umma::tmem_wait_st();
          umma::fence_async_smem();
          umma::fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            arrive(&sm->p_ready[s]);
            arrive(&sm->scal_free[s3]);
          }
        }
        WS_MARK(94);
      }
      if (!ok) break;
      if (!ST && !(ok = epilogue(G - 1, nchunk - 1))) break;
    }
  }
  }

  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) umma::tmem_dealloc(tm, 512);
#ifdef M3_WS_TIMING
  if (threadIdx.x < 128 && sm->tcnt[threadIdx.x]) {
    atomicAdd(&g_ws_wait[0][threadIdx.x], (unsigned long long)sm->tacc[threadIdx.x]);
    atomicAdd(&g_ws_wait[1][threadIdx.x], (unsigned long long)sm->tcnt[threadIdx.x]);
  }
#endif
}

}  // namespace ws
}  // namespace m3
