// The two small kernels of the forward's split over the sequence length (a batch of few
// (b, h) sequences cut into G segments that run side by side on the tensor-core forward).
//
//   m3_siso_split_prep:  per (b, segment, 64-token tile), from the raw streams, for every
//                        head: the tile's sums of tanh(angle) dt per angle and of adt
//                        (natural log), and the seed coefficient dt (1 - lam) of each
//                        segment's first token (reference.py:104-199 summed per tile).
//                        tanh(angle) and dt are formed once per token in shared memory and
//                        contracted over the tile's tokens for all (head, angle) pairs.
//   m3_siso_split_carry: per (b, h), serially over the segments.  Angles-only launch
//                        (s_loc NULL, before the states-only pass): the tile sums reduced in
//                        a fixed order into the segment's angle increment and decay a_seg,
//                        and the entering angle phi_in(j) = wrap(phi0 + pi sum_{i<j} inc_i).
//                        Full launch: the entering state S_in(j), with S_in(0) the caller's
//                        state and S_in(j+1) = e^{A_j} (S_in(j) + c_j v_{j-1} k_{j-1}^T) + S_j,
//                        where S_j, k_j, v_j are the states-only pass's results of segment j
//                        from a zero state at its true entering angle (the segment chaining
//                        of siso.py:154-216 is linear in the entering state).
// Tile sums are fp32 over 64 tokens; everything across tiles and segments is fp64.
#include "m3_common.cuh"
#include "m3_internal.h"

namespace m3 {
namespace {

constexpr int kSplitTile = M3_SPLIT_TILE;
constexpr int kMaxSegments = 64;
constexpr int kCarrySlices = 8;     // blocks per (b, h) for the state rebuild
constexpr int kPrepThreads = 256;

// One block per (b, segment, tile).  Dynamic shared memory: tanh(angle) (kSplitTile, Nr),
// dt and adt (kSplitTile, H) each.
__global__ void __launch_bounds__(kPrepThreads) split_prep_kernel(M3SplitPrepArgs a) {
  extern __shared__ float sm[];
  const int H = a.nheads, Nr = a.n_angles, G = a.segments;
  const int S = a.seqlen / (G * kSplitTile);
  const int s = blockIdx.x % S, bg = blockIdx.x / S, g = bg % G, b = bg / G;
  const int t0 = (g * S + s) * kSplitTile;
  float* th = sm;                       // [t][r]
  float* dt = th + kSplitTile * Nr;     // [t][h]
  float* adt = dt + kSplitTile * H;     // [t][h]
  // loads in batches of 8 per thread, all issued before the arithmetic
  constexpr int kB = 8;
  for (int i0 = threadIdx.x; i0 < kSplitTile * Nr; i0 += kB * blockDim.x) {
    float x[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int i = i0 + u * blockDim.x, t = i / Nr, r = i % Nr;
      x[u] = i < kSplitTile * Nr ? __ldg(a.angles + (size_t)b * a.ang_st.b + (size_t)(t0 + t) * a.ang_st.l + r) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kB; ++u)
      if (i0 + u * blockDim.x < kSplitTile * Nr) th[i0 + u * blockDim.x] = tanhf(x[u]);
  }
  for (int i0 = threadIdx.x; i0 < kSplitTile * H; i0 += kB * blockDim.x) {
    float dr[kB], ar[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int i = i0 + u * blockDim.x, t = i / H, h = i % H;
      const size_t o = (size_t)b * a.raw_st.b + (size_t)(t0 + t) * a.raw_st.l + (size_t)h * a.raw_st.h;
      const bool in = i < kSplitTile * H;
      dr[u] = in ? __ldg(a.dt_raw + o) + __ldg(a.dt_bias + h) : 0.f;
      ar[u] = in ? __ldg(a.a_raw + o) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int i = i0 + u * blockDim.x, t = i / H, h = i % H;
      if (i >= kSplitTile * H) continue;
      const float d = softplusf(dr[u]);
      dt[i] = d;
      adt[i] = fminf(-heavy_tail(ar[u]), -a.a_floor) * d;
      if (s == 0 && t == 0) {
        const size_t o = (size_t)b * a.raw_st.b + (size_t)t0 * a.raw_st.l + (size_t)h * a.raw_st.h;
        a.coef[((size_t)b * G + g) * H + h] = d * (1.f - sigmoidf_(__ldg(a.trap_raw + o)));
      }
    }
  }
  __syncthreads();
  float* out = a.partial + (((size_t)b * G + g) * S + s) * H * (Nr + 1);
  if (Nr % 4 == 0) {
    // thread = (head, 4 consecutive angles): one 128-bit read of tanh per 4 FMAs
    const int nq = Nr / 4;
    for (int o = threadIdx.x; o < H * nq; o += blockDim.x) {
      const int h = o / nq, r4 = 4 * (o % nq);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int t = 0; t < kSplitTile; ++t) {
        const float4 x = *reinterpret_cast<const float4*>(th + t * Nr + r4);
        const float d = dt[t * H + h];
        acc.x = fmaf(x.x, d, acc.x);
        acc.y = fmaf(x.y, d, acc.y);
        acc.z = fmaf(x.z, d, acc.z);
        acc.w = fmaf(x.w, d, acc.w);
      }
      float* dst = out + h * (Nr + 1) + r4;
      dst[0] = acc.x;
      dst[1] = acc.y;
      dst[2] = acc.z;
      dst[3] = acc.w;
    }
  } else {
    for (int o = threadIdx.x; o < H * Nr; o += blockDim.x) {
      const int h = o / Nr, r = o % Nr;
      float acc = 0.f;
#pragma unroll 8
      for (int t = 0; t < kSplitTile; ++t) acc = fmaf(th[t * Nr + r], dt[t * H + h], acc);
      out[h * (Nr + 1) + r] = acc;
    }
  }
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.f;
#pragma unroll 8
    for (int t = 0; t < kSplitTile; ++t) acc += adt[t * H + h];
    out[h * (Nr + 1) + Nr] = acc;
  }
}

// Angles-only launch: grid (B * H).  Full launch: grid (B * H, kCarrySlices), slice 0 also
// writes the entering k / v; every slice rebuilds its share of the (P, N) entering states.
__global__ void split_carry_kernel(M3SplitCarryArgs a) {
  const int bh = blockIdx.x, b = bh / a.nheads, h = bh % a.nheads;
  const int G = a.segments, N = a.state_dim, P = a.headdim, Nr = a.n_angles, H = a.nheads;
  if (blockIdx.y == 0) {
    if (!a.s_loc) {
      // tile sums -> segment sums (one thread per (segment, angle or decay), fixed order),
      // then the entering angles serially over the segments
      __shared__ double seg[kMaxSegments * 65];
      const int S = a.tiles, R = Nr + 1;
      for (int e = threadIdx.x; e < G * R; e += blockDim.x) {
        const int j = e / R, r = e % R;
        const float* pp = a.partial + ((size_t)b * G + j) * S * H * R + (size_t)h * R + r;
        double sum = 0.0;
        constexpr int kB = 8;
        for (int t0 = 0; t0 < S; t0 += kB) {
          float x[kB];
#pragma unroll
          for (int u = 0; u < kB; ++u) x[u] = t0 + u < S ? __ldg(pp + (size_t)(t0 + u) * H * R) : 0.f;
#pragma unroll
          for (int u = 0; u < kB; ++u) sum += (double)x[u];
        }
        seg[e] = sum;
        if (r == Nr) a.a_seg[((size_t)b * G + j) * H + h] = (float)sum;
      }
      __syncthreads();
      for (int r = threadIdx.x; r < Nr; r += blockDim.x) {
        double phi = a.seed_phi ? a.seed_phi[(size_t)bh * Nr + r] : 0.0;
        for (int j = 0; j < G; ++j) {
          const double wr = phi - 6.283185307179586 * floor(phi / 6.283185307179586);
          a.phi_in[(((size_t)b * G + j) * H + h) * Nr + r] = (float)wr;
          phi = wr + 3.14159265358979323846 * seg[j * R + r];
        }
      }
      return;  // angles only (before the states-only pass)
    }
    // entering k / v: the caller's for segment 0, segment j-1's last ones after that
    {
      for (int e = threadIdx.x; e < G * (N + P); e += blockDim.x) {
        const int j = e / (N + P), c = e % (N + P);
        const size_t o = ((size_t)b * G + j) * H + h, op = ((size_t)b * G + j - 1) * H + h;
        if (c < N)
          a.c_k[o * N + c] = j == 0 ? (a.seed_k ? a.seed_k[(size_t)bh * N + c] : 0.f) : a.k_last[op * N + c];
        else
          a.c_v[o * P + c - N] =
              j == 0 ? (a.seed_v ? a.seed_v[(size_t)bh * P + c - N] : 0.f) : a.v_last[op * P + c - N];
      }
    }
  }
  if (!a.s_loc) return;
  // entering states, one (p, n) element per thread step
  __shared__ double ea[kMaxSegments];
  __shared__ float cf[kMaxSegments];
  for (int j = threadIdx.x; j < G; j += blockDim.x) {
    const size_t o = ((size_t)b * G + j) * H + h;
    ea[j] = exp((double)a.a_seg[o]);
    cf[j] = a.coef[o];
  }
  __syncthreads();
  const int per = (P * N + gridDim.y - 1) / gridDim.y, e0 = blockIdx.y * per, e1 = min(P * N, e0 + per);
  for (int e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
    const int p = e / N, n = e % N;
    double s = a.seed_ssm ? a.seed_ssm[(size_t)bh * P * N + e] : 0.0;
    for (int j = 0; j < G; ++j) {
      const size_t o = ((size_t)b * G + j) * H + h;
      a.c_ssm[o * P * N + e] = (float)s;
      double kp, vp;
      if (j == 0) {
        kp = a.seed_k ? a.seed_k[(size_t)bh * N + n] : 0.0;
        vp = a.seed_v ? a.seed_v[(size_t)bh * P + p] : 0.0;
      } else {
        const size_t op = ((size_t)b * G + j - 1) * H + h;
        kp = a.k_last[op * N + n];
        vp = a.v_last[op * P + p];
      }
      s = ea[j] * (s + (double)cf[j] * vp * kp) + (double)a.s_loc[o * P * N + e];
    }
  }
}

}  // namespace
}  // namespace m3

using namespace m3;

extern "C" int m3_siso_split_prep(const M3SplitPrepArgs* args, void* stream) {
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  const M3SplitPrepArgs& a = *args;
  if (a.batch <= 0 || a.seqlen <= 0 || a.nheads <= 0 || a.n_angles <= 0 || a.segments <= 0 ||
      a.seqlen % (a.segments * kSplitTile))
    return set_error(M3_ERR_SHAPE, "m3_siso_split_prep: bad dims (seqlen must be a multiple of 64 * segments)");
  if (!a.dt_raw || !a.a_raw || !a.trap_raw || !a.angles || !a.dt_bias || !a.partial || !a.coef)
    return set_error(M3_ERR_ARG, "m3_siso_split_prep: NULL pointer");
  const size_t smem = (size_t)kSplitTile * (a.n_angles + 2 * a.nheads) * sizeof(float);
  if (smem > 200 * 1024) return set_error(M3_ERR_SHAPE, "m3_siso_split_prep: too many heads / angles");
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(split_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int blocks = a.batch * (a.seqlen / kSplitTile);
  split_prep_kernel<<<blocks, kPrepThreads, smem, (cudaStream_t)stream>>>(a);
  return check_launch("m3_siso_split_prep");
}

extern "C" int m3_siso_split_carry(const M3SplitCarryArgs* args, void* stream) {
  if (!args) return set_error(M3_ERR_ARG, "args is NULL");
  const M3SplitCarryArgs& a = *args;
  if (a.batch <= 0 || a.nheads <= 0 || a.segments <= 0 || a.segments > kMaxSegments || a.tiles <= 0 ||
      a.state_dim <= 0 || a.headdim <= 0 || a.n_angles <= 0 || a.n_angles > 64)
    return set_error(M3_ERR_SHAPE, "m3_siso_split_carry: bad dims");
  if (!a.a_seg || (!a.s_loc && (!a.partial || !a.phi_in)) ||
      (a.s_loc && (!a.coef || !a.k_last || !a.v_last || !a.c_ssm || !a.c_k || !a.c_v)))
    return set_error(M3_ERR_ARG, "m3_siso_split_carry: NULL pointer");
  split_carry_kernel<<<dim3(a.batch * a.nheads, a.s_loc ? kCarrySlices : 1), 256, 0, (cudaStream_t)stream>>>(a);
  return check_launch("m3_siso_split_carry");
}
