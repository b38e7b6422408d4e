// Small-batch projections of the decode step (model.py:244-296 at batch <= 8): out = f(x) @ W
// (+ residual), W a bf16 (K, N) row-major weight.  At M <= 8 rows the product is a stream of W
// through the SMs, so the kernel is built to read W at HBM speed and to absorb the elementwise
// work around each projection of lm_decode_step:
//   x_mode 0: f(x) = x
//   x_mode 1: f(x) = RMSNorm(x) * norm_w (layer.py:190-198; fp32 math, rounded to bf16 as the
//             layer's norm output is) -- the block norm before in_proj, the MLP norm before fc1
//   x_mode 2: f(x) = value * silu(gate), value / gate the two K-halves of a 2K-wide x row, each
//             product rounded to bf16 like the two torch ops it replaces (model.py:125-137)
//   residual: out = bf16(residual + acc), the rounding of torch.addmm.
// Grid: 256-column blocks x KSPLIT slices of K.  A CTA's 8 warps take every 8th row of its
// slice; lane l owns 8 consecutive columns (one 16-byte load of W per row), so a warp reads
// whole 512-byte row segments.  Partials go to a workspace; the last CTA of a column block (a
// ticket counter, no waiting) sums the slices in a fixed order, so results are deterministic,
// applies the residual, writes bf16 and resets its ticket for the next call.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "m3_internal.h"

namespace m3 {
int gemv_ksplit(int m, int k, int n);
int gemv_slice_rows(int k, int ks);
namespace {

constexpr int kGvThreads = 256, kGvWarps = 8, kGvCols = 256;

__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16(x)); }
__device__ __forceinline__ float bfv(const __nv_bfloat16* p) { return __bfloat162float(*p); }

constexpr int kGvR = 8;  // rows per warp per batch (16-byte loads in flight per lane)

template <int M>
__global__ void __launch_bounds__(kGvThreads) gemv_kernel(M3GemvArgs a, int slice_rows) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cb = blockIdx.x, ks = blockIdx.y, nks = gridDim.y;
  const int K = a.k, N = a.n;
  const int k0 = ks * slice_rows, k1 = min(K, k0 + slice_rows);
  const int nb = slice_rows / (kGvR * kGvWarps);  // batches per warp
  extern __shared__ float xs[];  // [slice_rows][M]: f(x) of this slice; later the warps' partials
  __shared__ float s_rstd[8];
  __shared__ float s_red[kGvWarps][8];
  __shared__ int s_last;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x);

  // this warp's rows of batch b: k0 + (b * kGvR + j) * 8 + warp, j < kGvR
  const int col = cb * kGvCols + lane * 8;
  const bool colok = col < N;
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(a.w) + col;
  auto load_batch = [&](int b, uint4 (&w)[kGvR]) {
#pragma unroll
    for (int j = 0; j < kGvR; ++j) {
      const int k = k0 + (b * kGvR + j) * kGvWarps + warp;
      w[j] = (colok && k < k1) ? __ldg(reinterpret_cast<const uint4*>(wp + (size_t)k * a.w_ld))
                               : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  float acc[M][8];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[m][c] = 0.f;
  auto fma_batch = [&](int b, const uint4 (&w)[kGvR]) {
#pragma unroll
    for (int j = 0; j < kGvR; ++j) {
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&w[j]);
      float wv[8];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 f = __bfloat1622float2(h2[c]);
        wv[2 * c] = f.x;
        wv[2 * c + 1] = f.y;
      }
      const float* xr = xs + ((b * kGvR + j) * kGvWarps + warp) * M;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float xv = xr[m];
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[m][c] = fmaf(xv, wv[c], acc[m][c]);
      }
    }
  };
  uint4 wa[kGvR], wb[kGvR];
  load_batch(0, wa);  // in flight while f(x) is formed

  // f(x) of the slice (row norms over the whole K first: every CTA recomputes them from L2)
  if (a.x_mode == 1) {
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = 0.f;
    for (int k = tid; k < K; k += kGvThreads)
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (m < a.m) {
          const float v = bfv(x + (size_t)m * a.x_ld + k);
          ss[m] += v * v;
        }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = ss[m];
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) s_red[warp][m] = v;
    }
    __syncthreads();
    if (tid < M) {
      float v = 0.f;
      for (int w = 0; w < kGvWarps; ++w) v += s_red[w][tid];
      s_rstd[tid] = rsqrtf(v / K + a.eps);
    }
    __syncthreads();
  }
  for (int i = tid; i < slice_rows * M; i += kGvThreads) {  // rows past K read as 0 (their W is 0 too)
    const int kk = i / M, m = i - kk * M, k = k0 + kk;
    float v = 0.f;
    if (m < a.m && k < k1) {
      const __nv_bfloat16* row = x + (size_t)m * a.x_ld;
      if (a.x_mode == 2) {
        const float val = bfv(row + k), g = bfv(row + K + k);
        const float sg = rbf(g / (1.f + expf(-g)));
        v = rbf(val * sg);
      } else if (a.x_mode == 1) {
        v = rbf(bfv(row + k) * s_rstd[m] * a.norm_w[k]);
      } else {
        v = bfv(row + k);
      }
    }
    xs[kk * M + m] = v;
  }
  __syncthreads();

  // the products, the next batch's loads issued before this batch's arithmetic
  for (int b = 0; b < nb; b += 2) {
    if (b + 1 < nb) load_batch(b + 1, wb);
    fma_batch(b, wa);
    if (b + 2 < nb) load_batch(b + 2, wa);
    if (b + 1 < nb) fma_batch(b + 1, wb);
  }
  // reduce the 8 warps through shared memory (the f(x) buffer is free once all warps are done)
  __syncthreads();
  float(*s_part)[M][kGvCols] = reinterpret_cast<float(*)[M][kGvCols]>(xs);
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int c = 0; c < 8; ++c) s_part[warp][m][lane * 8 + c] = acc[m][c];
  __syncthreads();
  float* part = a.scratch + ((size_t)ks * M) * N;  // this slice's (M, N) partial
  for (int i = tid; i < M * kGvCols; i += kGvThreads) {
    const int m = i / kGvCols, c = i - m * kGvCols, n = cb * kGvCols + c;
    if (n < N) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kGvWarps; ++w) v += s_part[w][m][c];
      part[(size_t)m * N + n] = v;
    }
  }
  // the last slice to finish this column block reduces all slices in order
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(a.tickets + cb, 1) == nks - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const __nv_bfloat16* res = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  for (int i = tid; i < M * kGvCols; i += kGvThreads) {
    const int m = i / kGvCols, c = i - m * kGvCols, n = cb * kGvCols + c;
    if (n < N && m < a.m) {
      float v = 0.f;
      for (int s = 0; s < nks; ++s) v += __ldcg(a.scratch + ((size_t)s * M + m) * N + n);
      if (res) v += bfv(res + (size_t)m * a.r_ld + n);
      out[(size_t)m * a.out_ld + n] = __float2bfloat16(v);
    }
  }
  if (tid == 0) a.tickets[cb] = 0;
}

template <int M>
int run_gemv(const M3GemvArgs& a, cudaStream_t s) {
  const int cbs = (a.n + kGvCols - 1) / kGvCols;
  const int ks = gemv_ksplit(a.m, a.k, a.n);
  const int slice = gemv_slice_rows(a.k, ks);
  const size_t part = (size_t)kGvWarps * M * kGvCols, fx = (size_t)slice * M;
  const size_t smem = (part > fx ? part : fx) * sizeof(float);
  if (smem > 200 * 1024) return set_error(M3_ERR_SHAPE, "m3_gemv_bf16: K too long for one slice");
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(gemv_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return check_launch("m3_gemv_bf16: cudaFuncSetAttribute");
    attr[dev] = true;
  }
  gemv_kernel<M><<<dim3(cbs, ks), kGvThreads, smem, s>>>(a, slice);
  return check_launch("m3_gemv_bf16");
}

}  // namespace

// K slices: about two CTAs per SM over the column blocks, each slice a multiple of one batch
// (kGvR rows for each of the 8 warps)
int gemv_ksplit(int m, int k, int n) {
  (void)m;
  const int cbs = (n + kGvCols - 1) / kGvCols;
  const int target = (296 + cbs - 1) / cbs;
  const int rows = gemv_slice_rows(k, target);
  return (k + rows - 1) / rows;
}

int gemv_slice_rows(int k, int ks) {
  const int unit = kGvR * kGvWarps;
  int rows = (k + ks - 1) / ks;
  return (rows + unit - 1) / unit * unit;
}

int launch_gemv(const M3GemvArgs& a, cudaStream_t s) {
  if (a.m <= 1) return run_gemv<1>(a, s);
  if (a.m <= 2) return run_gemv<2>(a, s);
  if (a.m <= 4) return run_gemv<4>(a, s);
  return run_gemv<8>(a, s);
}

}  // namespace m3
