// Skinny tcgen05 GEMM for the decode step's projections at batch > 8: out (M, N) bf16 =
// [residual +] a (M, K) bf16 @ w, M <= 256, fp32 accumulation in TMEM, one bf16 rounding.
// Replaces the matmul / addmm calls of model.lm_decode_step (reference model.py:244-296:
// in_proj, out_proj + residual, fc1, fc2 + residual, the tied head) at B = 256, where a
// library GEMM leaves most SMs idle (K = 4096, N = 2048 is 32 tiles of 128 x 128).
//
// One CTA per 128-column tile of w and all M rows (two M = 128 MMAs into 256 TMEM
// columns), so every weight byte crosses HBM once.  When there are too few column tiles to
// fill the SMs, K is split over a thread-block cluster of CS CTAs (1, 2 or 4): each CTA
// stages its fp32 partial tile in shared memory, and after a cluster barrier CTA r sums rows
// [r 256 / CS, (r + 1) 256 / CS) over the CS partials in rank order through distributed
// shared memory (the same fixed order every call, so the result is deterministic), adds the
// residual and writes bf16.
//
// Warps: 0 TMA producer (4-stage ring of a 256 x 64 tile of a and a 64 x 128 tile of w,
// SWIZZLE_128B, mbarrier expect-tx), 1 tcgen05 issuer, 2-9 epilogue (two warpgroups, one
// per 128-row half; thread = TMEM lane).  w is (K, N) with N contiguous (MN-major B
// operand) or, for the tied head, (N, K) with K contiguous (K-major).  Every wait is bounded;
// on time-out the CTA records an error code, skips its remaining work, still takes part in
// both cluster barriers (so no peer waits forever), waits for its own loads and frees TMEM.
#include <cuda.h>

#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_umma.cuh"

namespace m3 {
namespace gm {

__device__ int g_gemm_error;  // non-zero after a bounded wait gave up (read by m3_device_error)

#ifdef M3_GEMM_TIMING
// Diagnostic builds only: %globaltimer stamps per CTA (entry, setup, accumulator ready,
// staged, reduced, exit).
__device__ unsigned long long g_gemm_t[1024][6];
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define GM_STAMP(i)                                                                          \
  do {                                                                                       \
    const int b_ = blockIdx.x * gridDim.y + blockIdx.y;                                      \
    if (b_ < 1024) g_gemm_t[b_][i] = gtime();                                                \
  } while (0)
#else
#define GM_STAMP(i) \
  do {              \
  } while (0)
#endif

constexpr int kBN = 128, kBK = 64, kStages = 4, kThreads = 320;
constexpr uint32_t kABytes = 256u * kBK * 2u;  // 32 KB: 256 rows x 128 B
constexpr uint32_t kBBytes = (uint32_t)kBK * kBN * 2u;  // 16 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kRow = 132;  // fp32 staging row stride (floats): conflict-free row writes
constexpr uint32_t kStagingBytes = 256u * kRow * 4u;
static_assert(kStagingBytes <= kStages * kStageBytes, "staging must fit in the stage ring");
constexpr long long kWaitLimit = 2000000000LL;

struct Small {
  uint64_t full[kStages], empty[kStages], acc_full;
  uint32_t tmem;
  int abort_flag;
};
constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + sizeof(Small);

__device__ __forceinline__ void tma_load2(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          umma::smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(umma::smem_u32(mbar))
      : "memory");
}

__device__ __forceinline__ void expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(umma::smem_u32(mbar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool wait_bar(Small* sm, uint64_t* mbar, uint32_t parity, int code) {
  const uint32_t a = umma::smem_u32(mbar);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(1u << 16)
        : "memory");
    if (done) return true;
    if (*(volatile int*)&sm->abort_flag) return false;
    if (clock64() - t0 > kWaitLimit) {
      *(volatile int*)&sm->abort_flag = 1;
      atomicExch(&g_gemm_error, code);
      return false;
    }
  }
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ float4 ld_peer4(uint32_t local_saddr, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local_saddr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(ra));
  return v;
}

struct Params {
  int m, n, k, kc;  // kc: this CTA's share of K
  int w_kmajor;
  const __nv_bfloat16* residual;
  int64_t ldr;
  __nv_bfloat16* out;
  int64_t ldo;
};

// Rows [rank 256 / CS, (rank + 1) 256 / CS) of the tile: the CS partials summed in rank
// order, the residual added, one bf16 rounding.  Thread t takes 4-column groups
// t, t + 256, ...; 8 / CS of them per round, so 8 partial loads are in flight at a time.
template <int CS>
__device__ __forceinline__ void reduce_rows(const Params& p, uint32_t sbase, uint32_t rank, int n0, int t) {
  constexpr int kPer = 256 / CS, kJ = kPer * (kBN / 4) / 256, kU = 8 / CS;
  const int r0 = (int)rank * kPer;
#pragma unroll 1
  for (int j0 = 0; j0 < kJ; j0 += kU) {
    float4 v[kU][CS];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int idx = t + 256 * (j0 + u), rr = r0 + idx / (kBN / 4), c4 = idx % (kBN / 4);
      const uint32_t off = sbase + (uint32_t)(rr * kRow + 4 * c4) * 4u;
#pragma unroll
      for (int pr = 0; pr < CS; ++pr) v[u][pr] = ld_peer4(off, (uint32_t)pr);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int idx = t + 256 * (j0 + u), rr = r0 + idx / (kBN / 4), c4 = idx % (kBN / 4), col = n0 + 4 * c4;
      if (rr >= p.m || col >= p.n) continue;
      float4 acc = v[u][0];
#pragma unroll
      for (int pr = 1; pr < CS; ++pr) {
        acc.x += v[u][pr].x;
        acc.y += v[u][pr].y;
        acc.z += v[u][pr].z;
        acc.w += v[u][pr].w;
      }
      if (p.residual) {
        const uint2 r2 = *reinterpret_cast<const uint2*>(p.residual + (size_t)rr * p.ldr + col);
        acc.x += __uint_as_float(r2.x << 16);
        acc.y += __uint_as_float(r2.x & 0xffff0000u);
        acc.z += __uint_as_float(r2.y << 16);
        acc.w += __uint_as_float(r2.y & 0xffff0000u);
      }
      *reinterpret_cast<uint2*>(p.out + (size_t)rr * p.ldo + col) =
          make_uint2(umma::pack_bf16x2(acc.x, acc.y), umma::pack_bf16x2(acc.z, acc.w));
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, const Params p) {
  extern __shared__ uint8_t smraw[];
  if (threadIdx.x == 0) GM_STAMP(0);
  uint8_t* base = (uint8_t*)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
  Small* sm = (Small*)(base + kStages * kStageBytes);
  float* stg = reinterpret_cast<float*>(base);  // staging, over the stage ring once the MMAs are done
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int CS = gridDim.y;
  const uint32_t rank = cluster_rank();
  const int k0 = (int)blockIdx.y * p.kc;
  const int nk = p.kc / kBK;
  const bool two = p.m > 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      umma::mbar_init(&sm->full[s], 1);
      umma::mbar_init(&sm->empty[s], 1);
    }
    umma::mbar_init(&sm->acc_full, 1);
    sm->abort_flag = 0;
    umma::fence_mbar_init();
  }
  if (warp == 1) umma::tmem_alloc(&sm->tmem, 256);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tm = sm->tmem;
  if (threadIdx.x == 0) GM_STAMP(1);

  if (warp == 0) {
    // ================================ TMA producer ================================
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        if (it >= kStages && !wait_bar(sm, &sm->empty[s], ((it / kStages) - 1) & 1, 81)) break;
        uint8_t* sa = base + s * kStageBytes;
        uint8_t* sb = sa + kABytes;
        const int kk = k0 + it * kBK;
        expect_tx(&sm->full[s], kStageBytes);
        tma_load2(sa, &ta, kk, 0, &sm->full[s]);
        if (p.w_kmajor) {
          tma_load2(sb, &tw, kk, n0, &sm->full[s]);
        } else {
          tma_load2(sb, &tw, n0, kk, &sm->full[s]);
          tma_load2(sb + kBBytes / 2, &tw, n0 + 64, kk, &sm->full[s]);
        }
        ++issued;
      }
      // loads still in flight land before the CTA moves on
      for (int it = issued - kStages < 0 ? 0 : issued - kStages; it < issued; ++it) {
        const int s = it % kStages;
        const long long t0 = clock64();
        uint32_t done = 0;
        while (!done && clock64() - t0 < kWaitLimit / 8) {
          asm volatile(
              "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
              "selp.u32 %0, 1, 0, q;\n\t}\n"
              : "=r"(done)
              : "r"(umma::smem_u32(&sm->full[s])), "r"((uint32_t)(it / kStages) & 1)
              : "memory");
        }
      }
    }
  } else if (warp == 1) {
    // ================================ tcgen05 issuer ================================
    if (lane == 0) {
      const uint32_t idesc = umma::idesc_bf16(128, kBN, false, !p.w_kmajor);
      bool ok = true;
      for (int it = 0; it < nk && ok; ++it) {
        const int s = it % kStages;
        if (!(ok = wait_bar(sm, &sm->full[s], (it / kStages) & 1, 82))) break;
        umma::fence_after_sync();
        const uint32_t sa = umma::smem_u32(base + s * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t db = p.w_kmajor ? umma::smem_desc(sb + ks * 32u, 16, 1024)
                                         : umma::smem_desc(sb + ks * 2048u, kBBytes / 2, 1024);
          const bool acc = it > 0 || ks > 0;
          umma::mma_bf16(tm, umma::smem_desc(sa + ks * 32u, 16, 1024), db, idesc, acc);
          if (two) umma::mma_bf16(tm + 128, umma::smem_desc(sa + 16384u + ks * 32u, 16, 1024), db, idesc, acc);
        }
        umma::commit(&sm->empty[s]);
      }
      umma::commit(&sm->acc_full);  // also the drain: every MMA issued has completed
      if (!ok) {
        // make sure the issued MMAs are done before TMEM is freed
        const long long t0 = clock64();
        uint32_t done = 0;
        while (!done && clock64() - t0 < kWaitLimit / 8) {
          asm volatile(
              "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.shared::cta.b64 q, [%1], 0;\n\t"
              "selp.u32 %0, 1, 0, q;\n\t}\n"
              : "=r"(done)
              : "r"(umma::smem_u32(&sm->acc_full))
              : "memory");
        }
      }
    }
  } else {
    // ============================ accumulator -> staging ============================
    const int ew = warp - 2, q = warp & 3, mh = ew >> 2;
    const int row = mh * 128 + q * 32 + lane;
    const bool ok = wait_bar(sm, &sm->acc_full, 0, 83);
    umma::fence_after_sync();
    if (threadIdx.x == 64) GM_STAMP(2);
    if (ok && (mh == 0 || two)) {
#pragma unroll 1
      for (int c = 0; c < kBN; c += 32) {
        float v[32];
        umma::tmem_ld32(tm + ((uint32_t)(q * 32) << 16) + mh * 128 + c, v);
        umma::tmem_wait_ld();
        float* dst = stg + row * kRow + c;
#pragma unroll
        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
    }
  }
  umma::fence_before_sync();
  __syncwarp();
  cluster_sync_all();  // every CTA's partial is staged
  if (threadIdx.x == 64) GM_STAMP(3);

  if (warp >= 2 && !*(volatile int*)&sm->abort_flag) {
    const int t = threadIdx.x - 64;  // 0..255
    const uint32_t sbase = umma::smem_u32(stg);
    switch (CS) {
      case 1: reduce_rows<1>(p, sbase, rank, n0, t); break;
      case 2: reduce_rows<2>(p, sbase, rank, n0, t); break;
      default: reduce_rows<4>(p, sbase, rank, n0, t); break;
    }
  }
  if (threadIdx.x == 64) GM_STAMP(4);
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while a peer may still read its staging
  umma::fence_after_sync();
  if (warp == 1) umma::tmem_dealloc(tm, 256);
  if (threadIdx.x == 64) GM_STAMP(5);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)q;
  }
  return fn;
}

// 2-D bf16 map: `inner` contiguous elements per row, `outer` rows `ld` elements apart;
// boxes of 64 x box_outer, SWIZZLE_128B, zero fill outside the tensor.
static bool map2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, int64_t ld, uint32_t box_outer) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  const cuuint64_t gd[2] = {inner, outer};
  const cuuint64_t gs[1] = {(cuuint64_t)ld * 2u};
  const cuuint32_t box[2] = {64u, box_outer};
  const cuuint32_t es[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), gd, gs, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count() {
  int dev = 0, c = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
  return c;
}

}  // namespace gm

#ifdef M3_GEMM_TIMING
extern "C" int m3_debug_gemm_timing(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, gm::g_gemm_t, sizeof(unsigned long long) * 1024 * 6) == cudaSuccess ? 0 : -1;
}
#endif

int read_gemm_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gm::g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(gm::g_gemm_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace m3

using namespace m3;

extern "C" int m3_gemm_bf16(const M3GemmArgs* args, void* stream) {
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  const M3GemmArgs& a = *args;
  if (a.m <= 0 || a.m > 256 || a.n <= 0 || a.k <= 0)
    return set_error(M3_ERR_SHAPE, "m3_gemm_bf16: need 0 < m <= 256, n > 0, k > 0");
  if (a.k % gm::kBK || a.n % 8)
    return set_error(M3_ERR_UNSUPPORTED, "m3_gemm_bf16: k must be a multiple of 64 and n of 8");
  if (!a.a || !a.w || !a.out) return set_error(M3_ERR_ARG, "m3_gemm_bf16: NULL pointer");
  const int64_t lda = a.lda ? a.lda : a.k, ldo = a.ldo ? a.ldo : a.n, ldr = a.ldr ? a.ldr : a.n;
  const int64_t ldw = a.ldw ? a.ldw : (a.w_kmajor ? a.k : a.n);
  auto al16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
  if (!al16(a.a) || !al16(a.w) || lda % 8 || ldw % 8 || ((uintptr_t)a.out & 7u) || ldo % 4 ||
      (a.residual && (((uintptr_t)a.residual & 7u) || ldr % 4)))
    return set_error(M3_ERR_UNSUPPORTED, "m3_gemm_bf16: operands need 16-byte rows (a, w) and 8-byte rows (out, residual)");
  const int ntiles = (a.n + gm::kBN - 1) / gm::kBN;
  // K split over a cluster until the tiles fill most SMs (each CTA keeps >= 4 k-steps)
  const int nsm = gm::sm_count();
  // (at most 4: clusters of 8 CTAs of this size do not all fit on the GPU at once)
  int cs = 1;
  if (a.ksplit) {
    if (a.ksplit != 1 && a.ksplit != 2 && a.ksplit != 4) return set_error(M3_ERR_ARG, "m3_gemm_bf16: ksplit must be 0, 1, 2 or 4");
    if (a.k % (gm::kBK * a.ksplit)) return set_error(M3_ERR_SHAPE, "m3_gemm_bf16: k must split into multiples of 64");
    cs = a.ksplit;
  } else {
    while (cs < 4 && ntiles * cs * 2 <= nsm + nsm / 4 && a.k % (gm::kBK * cs * 2) == 0 && a.k / (cs * 2) >= 4 * gm::kBK)
      cs *= 2;
  }
  CUtensorMap ta, tw;
  if (!gm::map2d(&ta, a.a, (uint64_t)a.k, (uint64_t)a.m, lda, 256u) ||
      !(a.w_kmajor ? gm::map2d(&tw, a.w, (uint64_t)a.k, (uint64_t)a.n, ldw, (uint32_t)gm::kBN)
                   : gm::map2d(&tw, a.w, (uint64_t)a.n, (uint64_t)a.k, ldw, (uint32_t)gm::kBK)))
    return set_error(M3_ERR_LAUNCH, "m3_gemm_bf16: cuTensorMapEncodeTiled failed");
  gm::Params p;
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.kc = a.k / cs;
  p.w_kmajor = a.w_kmajor ? 1 : 0;
  p.residual = (const __nv_bfloat16*)a.residual;
  p.ldr = ldr;
  p.out = (__nv_bfloat16*)a.out;
  p.ldo = ldo;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr[dev]) {
    if (cudaFuncSetAttribute(gm::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gm::kSmemBytes) !=
        cudaSuccess)
      return check_launch("m3_gemm_bf16: cudaFuncSetAttribute");
    if (dev < 64) attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ntiles, cs, 1);
  cfg.blockDim = dim3(gm::kThreads, 1, 1);
  cfg.dynamicSmemBytes = gm::kSmemBytes;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 1;
  at[0].val.clusterDim.y = cs;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gm::gemm_kernel, ta, tw, p);
  if (e != cudaSuccess) return set_error(M3_ERR_LAUNCH, cudaGetErrorString(e));
  return check_launch("m3_gemm_bf16");
}
