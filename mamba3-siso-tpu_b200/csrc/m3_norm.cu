// Fused RMS normalisation of rows (layer.py:190-198, model.py's block / final norms):
//   y = x * rsqrt(mean(x^2) + eps) * w      in fp32, stored in x's dtype.
// One warp (or four, for rows of 1024+) per row: a pass for the sum of squares (16-byte vectors when the row allows),
// a warp reduction, and a pass that scales (the row is back from L1 / L2).  Replaces the
// seven elementwise / reduction launches of the unfused form in the decode and inference
// paths.
#include "m3_common.cuh"
#include "m3_internal.h"

namespace m3 {

constexpr int kNormThreads = 256;

// TPR threads per row (32: one warp; 128: four warps joined through shared memory, for
// long rows, so that a few hundred rows still fill the GPU).
template <typename T, typename W, bool VEC, int TPR>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const T* __restrict__ x, int64_t xs,
                                                                const W* __restrict__ w, T* __restrict__ y, int64_t ys,
                                                                int64_t rows, int dim, float eps,
                                                                float* __restrict__ rstd_out) {
  constexpr int RPC = kNormThreads / TPR;  // rows per CTA
  __shared__ float part[kNormThreads / 32];
  const int sub = threadIdx.x % TPR;      // this thread's index within its row
  const int64_t row = (int64_t)blockIdx.x * RPC + threadIdx.x / TPR;
  const bool live = row < rows;
  const T* xr = x + row * xs;
  T* yr = y + row * ys;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  float ss = 0.f;
  if (live) {
    if (VEC) {
      for (int i = sub * V; i < dim; i += TPR * V) {
        const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float f = ld(e + j);
          ss = fmaf(f, f, ss);
        }
      }
    } else {
      for (int i = sub; i < dim; i += TPR) {
        const float f = ld(xr + i);
        ss = fmaf(f, f, ss);
      }
    }
  }
  ss = warp_sum(ss);
  if (TPR > 32) {
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    const int w0 = (threadIdx.x / TPR) * (TPR / 32);
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < TPR / 32; ++k) ss += part[w0 + k];
  }
  if (!live) return;
  const float r = rsqrtf(ss / (float)dim + eps);
  if (rstd_out && sub == 0) rstd_out[row] = r;
  if (VEC) {
    for (int i = sub * V; i < dim; i += TPR * V) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
      const T* e = reinterpret_cast<const T*>(&u);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < V; ++j) stg<T>(oe + j, ld(e + j) * r * ld(w + i + j));
      *reinterpret_cast<uint4*>(yr + i) = o;
    }
  } else {
    for (int i = sub; i < dim; i += TPR) stg<T>(yr + i, ld(xr + i) * r * ld(w + i));
  }
}

template <typename T, typename W, int TPR>
static int run_norm_t(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int dim, float eps,
                      float* rstd, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T), RPC = kNormThreads / TPR;
  const bool vec = dim % V == 0 && xs % V == 0 && ys % V == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 16) == 0;
  const int64_t grid = (rows + RPC - 1) / RPC;
  if (vec)
    rms_norm_kernel<T, W, true, TPR><<<(unsigned)grid, kNormThreads, 0, s>>>((const T*)x, xs, (const W*)w, (T*)y, ys,
                                                                             rows, dim, eps, rstd);
  else
    rms_norm_kernel<T, W, false, TPR><<<(unsigned)grid, kNormThreads, 0, s>>>((const T*)x, xs, (const W*)w, (T*)y, ys,
                                                                              rows, dim, eps, rstd);
  return check_launch("m3_rms_norm");
}

template <typename T, typename W>
static int run_norm(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int dim, float eps,
                    float* rstd, cudaStream_t s) {
  return dim >= 1024 ? run_norm_t<T, W, 128>(x, xs, w, y, ys, rows, dim, eps, rstd, s)
                     : run_norm_t<T, W, 32>(x, xs, w, y, ys, rows, dim, eps, rstd, s);
}

int launch_rms_norm(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int dim, float eps,
                    int x_dtype, int w_dtype, float* rstd, cudaStream_t s) {
  const bool xb = x_dtype == M3_DTYPE_BF16, wb = w_dtype == M3_DTYPE_BF16;
  if (xb) return wb ? run_norm<__nv_bfloat16, __nv_bfloat16>(x, xs, w, y, ys, rows, dim, eps, rstd, s)
                    : run_norm<__nv_bfloat16, float>(x, xs, w, y, ys, rows, dim, eps, rstd, s);
  return wb ? run_norm<float, __nv_bfloat16>(x, xs, w, y, ys, rows, dim, eps, rstd, s)
            : run_norm<float, float>(x, xs, w, y, ys, rows, dim, eps, rstd, s);
}

// Backward of y = x r w, r = rsqrt(mean(x^2) + eps), per row with g = dy o w:
//   dx = r g - x (r^3 / dim) sum(g o x)         dw = sum over rows of dy o x r
// One warp per row, rows strided over a persistent grid; each lane keeps its COLS columns'
// dw partial sums in registers (dim <= 32 COLS) and adds them to dw once per CTA.
template <typename T, typename W, int COLS>
__global__ void __launch_bounds__(kNormThreads) rms_norm_bwd_kernel(const T* __restrict__ x, int64_t xs,
                                                                    const W* __restrict__ w, const float* __restrict__ rstd,
                                                                    const T* __restrict__ dy, int64_t dys,
                                                                    T* __restrict__ dx, int64_t dxs,
                                                                    float* __restrict__ dw, int64_t rows, int dim) {
  __shared__ float dws[COLS * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < dim; i += kNormThreads) dws[i] = 0.f;
  __syncthreads();
  float acc[COLS];
#pragma unroll
  for (int j = 0; j < COLS; ++j) acc[j] = 0.f;
  for (int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + warp; row < rows;
       row += (int64_t)gridDim.x * (kNormThreads / 32)) {
    const T* xr = x + row * xs;
    const T* gr = dy + row * dys;
    const float r = rstd[row];
    float sgx = 0.f;
#pragma unroll
    for (int j = 0; j < COLS; ++j) {
      const int i = lane + 32 * j;
      if (i < dim) sgx = fmaf(ld(gr + i) * ld(w + i), ld(xr + i), sgx);
    }
    sgx = warp_sum(sgx);
    const float c = r * r * r * sgx / (float)dim;
#pragma unroll
    for (int j = 0; j < COLS; ++j) {
      const int i = lane + 32 * j;
      if (i < dim) {
        const float xv = ld(xr + i), gv = ld(gr + i);
        stg<T>(dx + row * dxs + i, r * gv * ld(w + i) - xv * c);
        acc[j] = fmaf(gv, xv * r, acc[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < COLS; ++j) {
    const int i = lane + 32 * j;
    if (i < dim) atomicAdd(&dws[i], acc[j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += kNormThreads) atomicAdd(dw + i, dws[i]);
}

template <typename T, typename W>
static int run_norm_bwd(const void* x, int64_t xs, const void* w, const float* rstd, const void* dy, int64_t dys,
                        void* dx, int64_t dxs, float* dw, int64_t rows, int dim, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (rows + kNormThreads / 32 - 1) / (kNormThreads / 32);
  const int grid = (int)(need < 4 * sms ? need : 4 * sms);
  const int g = grid > 0 ? grid : 1;
  if (dim <= 128)
    rms_norm_bwd_kernel<T, W, 4><<<g, kNormThreads, 0, s>>>((const T*)x, xs, (const W*)w, rstd, (const T*)dy, dys,
                                                            (T*)dx, dxs, dw, rows, dim);
  else if (dim <= 512)
    rms_norm_bwd_kernel<T, W, 16><<<g, kNormThreads, 0, s>>>((const T*)x, xs, (const W*)w, rstd, (const T*)dy, dys,
                                                             (T*)dx, dxs, dw, rows, dim);
  else
    rms_norm_bwd_kernel<T, W, 64><<<g, kNormThreads, 0, s>>>((const T*)x, xs, (const W*)w, rstd, (const T*)dy, dys,
                                                             (T*)dx, dxs, dw, rows, dim);
  return check_launch("m3_rms_norm_bwd");
}

int launch_rms_norm_bwd(const void* x, int64_t xs, const void* w, const float* rstd, const void* dy, int64_t dys,
                        void* dx, int64_t dxs, float* dw, int64_t rows, int dim, int x_dtype, int w_dtype,
                        cudaStream_t s) {
  const bool xb = x_dtype == M3_DTYPE_BF16, wb = w_dtype == M3_DTYPE_BF16;
  if (xb) return wb ? run_norm_bwd<__nv_bfloat16, __nv_bfloat16>(x, xs, w, rstd, dy, dys, dx, dxs, dw, rows, dim, s)
                    : run_norm_bwd<__nv_bfloat16, float>(x, xs, w, rstd, dy, dys, dx, dxs, dw, rows, dim, s);
  return wb ? run_norm_bwd<float, __nv_bfloat16>(x, xs, w, rstd, dy, dys, dx, dxs, dw, rows, dim, s)
            : run_norm_bwd<float, float>(x, xs, w, rstd, dy, dys, dx, dxs, dw, rows, dim, s);
}

// ---- gated activation of the MLP (model.py:125-137): out = value * silu(gate) ----------
// value / gate are the two k-wide halves of each x row; silu(gate) and the product are each
// rounded to the I/O dtype, as the two torch ops this replaces round them.  8 elements per
// thread with 16-byte loads when the rows allow it.
template <typename T>
__device__ __forceinline__ float rnd_t(float v) {
  return static_cast<float>(static_cast<T>(v));
}

template <typename T>
__global__ void gated_act_kernel(const T* __restrict__ x, int64_t xs, T* __restrict__ out, int64_t os, int64_t rows,
                                 int k) {
  const int64_t per_row = k / 8;
  const int64_t total = rows * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    const T* row = x + r * xs;
    T vv[8], gg[8], oo[8];
    *reinterpret_cast<uint4*>(vv) = *reinterpret_cast<const uint4*>(row + c);
    *reinterpret_cast<uint4*>(gg) = *reinterpret_cast<const uint4*>(row + k + c);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float g = static_cast<float>(gg[j]);
      const float sg = rnd_t<T>(g / (1.f + expf(-g)));
      oo[j] = static_cast<T>(static_cast<float>(vv[j]) * sg);
    }
    *reinterpret_cast<uint4*>(out + r * os + c) = *reinterpret_cast<const uint4*>(oo);
  }
}

int launch_gated_act(const void* x, int64_t xs, void* out, int64_t os, int64_t rows, int k, cudaStream_t s) {
  const int64_t total = rows * (k / 8);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  gated_act_kernel<__nv_bfloat16><<<grid > 0 ? grid : 1, 256, 0, s>>>((const __nv_bfloat16*)x, xs, (__nv_bfloat16*)out,
                                                                      os, rows, k);
  return check_launch("m3_gated_act");
}

}  // namespace m3
