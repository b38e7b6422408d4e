// Single-token decode step (mamba3_pallas/kernel_decode.py:56-233, reference.py:442-490):
//
//   phi' = wrap(phi + tanh(angles) pi dt)                 per head (dt is per head)
//   q~, k~ = R(phi') (q + q_bias), R(phi') (k + k_bias)
//   S'   = alpha S + beta v_prev k_prev^T + gamma v k~^T,  alpha = exp(adt),
//          beta = alpha dt (1 - lam), gamma = dt lam
//   y    = (S' q~ + D v) * silu(z)
//
// A bandwidth-bound read-modify-write of the (P, N) fp32 state, which is touched once.
// A persistent grid (a few CTAs per SM) walks the (b, h) items; each CTA streams the
// states through two shared-memory buffers with bulk copies (cp.async.bulk, completion on
// an mbarrier, no register staging): while item i is updated in one buffer, item i + grid
// is already on its way into the other, and item i goes back to HBM with a bulk store.
// Per item a preamble computes the rotated q~ / k~ columns and the per-row coefficients
// beta v_prev, gamma v, D v and silu(z) into shared memory (its global loads overlap the
// state copy).  The update runs over consecutive float4 of the state (whole rows per
// warp instruction at N = 128) with packed fp32x2 arithmetic; the readout S' q~ is a
// shuffle reduction over the lanes of a row.  The state, k, v and phi buffers are updated
// in place.  Every wait is bounded: on time-out the kernel records an error and returns.
#pragma once

#include "m3_common.cuh"
#include "m3_umma.cuh"

namespace m3 {

template <typename T> __device__ __forceinline__ float rnd_io(float x);
template <> __device__ __forceinline__ float rnd_io<float>(float x) { return x; }
template <> __device__ __forceinline__ float rnd_io<__nv_bfloat16>(float x) {
  return __bfloat162float(__float2bfloat16(x));
}

constexpr int kDecThreads = 256;
constexpr int kDecCtasPerSm = 3;

__device__ int g_m3_dec_error;  // non-zero after a bounded wait of the decode kernel gave up

namespace bulk {
__device__ __forceinline__ void expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(umma::smem_u32(mbar)), "r"(bytes)
               : "memory");
}
// global -> shared of this CTA, completion counted on `mbar`
__device__ __forceinline__ void load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   umma::smem_u32(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(umma::smem_u32(mbar))
               : "memory");
}
// shared -> global, tracked by this thread's bulk groups
__device__ __forceinline__ void store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(umma::smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void wait_reads() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
}  // namespace bulk

template <int N, int P>
struct DecSmem {
  static constexpr uint32_t kStateBytes = P * N * 4;
  static constexpr size_t kBytes = 2 * (size_t)kStateBytes;  // the two state buffers (dynamic)
};

// FUSED: the lm_decode_step variant (in-kernel B / C norms, bf16 scalar streams); the plain
// variant compiles both out, so the standalone decode keeps its shorter preamble.
template <int N, int P, typename T, bool MMB, bool FUSED>
__global__ void __launch_bounds__(kDecThreads, kDecCtasPerSm) decode_kernel(const M3DecodeArgs a) {
  static_assert(N <= 128 && P <= 128 && N % 4 == 0 && (P * N / 4) % 32 == 0, "decode tiling");
  constexpr int LPR = N / 4;              // lanes (float4 columns) per state row
  constexpr int NF4 = P * N / 4;          // float4 of one (b, h) state
  constexpr int EPT = (NF4 + kDecThreads - 1) / kDecThreads;
  constexpr int H2 = N / 2;
  constexpr uint32_t kBytes = DecSmem<N, P>::kStateBytes;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ uint64_t mbar[2];
  __shared__ __align__(16) float s_q[N], s_k[N], s_kp[N];  // q~ (readout-rounded), k~, previous k~
  __shared__ float s_bv[P], s_gv[P], s_dv[P], s_gate[P];  // beta v_prev, gamma v, D v, silu(z)
  __shared__ float s_ph[64];
  __shared__ float s_ssq[2][4];  // per-warp sums of q^2, k^2 for the fused norms
  const int tid = threadIdx.x;
  const int H = a.nheads, Nr = a.n_angles;
  const int total = a.batch * H;
  auto buf = [&](int sel) { return reinterpret_cast<float4*>(dsm + (size_t)sel * kBytes); };

  if (tid == 0) {
    umma::mbar_init(&mbar[0], 1);
    umma::mbar_init(&mbar[1], 1);
    umma::fence_mbar_init();
  }
  __syncthreads();
  int it = blockIdx.x;
  if (tid == 0 && it < total) {
    bulk::expect_tx(&mbar[0], kBytes);
    bulk::load(buf(0), a.ssm + (size_t)it * P * N, kBytes, &mbar[0]);
  }

  // Global inputs of one item's preamble, loaded one item ahead (in registers) so that their
  // latency overlaps the previous item's update.
  struct In {
    float dtr, ar, trr;       // raw dt / A / trap (or adt / dt / lam)
    float u, w, um, wm, kpv;  // column threads: q, k, their pair partners, k_prev
    float bq, bk, bqm, bkm;   // the biases of those columns (added after the fused norm)
    float ph, an;             // angle threads: phi, raw angle
    float vc, vp, zz;         // row threads: v, v_prev, z
  };
  const int n = tid, j = n < H2 ? n : n - H2;
  const int mm = n < H2 ? n + H2 : n - H2;  // the pair partner
  const bool sbf = FUSED && a.scalar_dtype == M3_DTYPE_BF16;
  auto lds = [&](const float* p, size_t i) {  // a scalar-stream element in scalar_dtype
    return sbf ? ld(reinterpret_cast<const __nv_bfloat16*>(p) + i) : p[i];
  };
  const bool fnorm = FUSED && a.q_norm_w != nullptr;
  auto load_in = [&](int item, In& x) {
    const int b = item / H, h = item % H;
    const size_t bh = (size_t)item;
    if (a.raw) {
      const size_t o = (size_t)b * a.raw_stride_b + h;
      x.dtr = lds(a.dt_raw, o) + a.dt_bias[h];
      x.ar = lds(a.a_raw, o);
      x.trr = lds(a.trap_raw, o);
    } else {
      x.dtr = lds(a.adt, bh);
      x.ar = lds(a.dt, bh);
      x.trr = lds(a.lam, bh);
    }
    if (tid < N) {
      const T* q = (const T*)a.q + (size_t)b * a.qk_stride_b;
      const T* k = (const T*)a.k + (size_t)b * a.qk_stride_b;
      x.u = ld(q + n);
      x.w = ld(k + n);
      x.bq = a.q_bias[h * N + n];
      x.bk = a.k_bias[h * N + n];
      if (j < Nr) {
        x.um = ld(q + mm);
        x.wm = ld(k + mm);
        x.bqm = a.q_bias[h * N + mm];
        x.bkm = a.k_bias[h * N + mm];
      }
      x.kpv = a.state_k[bh * N + n];
    }
    if (tid < Nr) {
      x.ph = a.phi[bh * Nr + tid];
      x.an = lds(a.angles, (size_t)b * a.ang_stride_b + tid);
    }
    if (tid >= 128 && tid < 128 + P) {
      const int p = tid - 128;
      x.vc = ld((const T*)a.v + (size_t)b * a.vz_stride_b + (size_t)h * P + p);
      x.vp = a.state_v[bh * P + p];
      x.zz = a.z ? ld((const T*)a.z + (size_t)b * a.vz_stride_b + (size_t)h * P + p) : 0.f;
    }
  };
  In cur{};
  if (it < total) load_in(it, cur);

  for (int kk = 0; it < total; it += gridDim.x, ++kk) {
    const int sel = kk & 1;
    const int nxt = it + gridDim.x;
    if (tid == 0 && nxt < total) {
      bulk::wait_reads();  // the store that last read the other buffer has read it
      bulk::expect_tx(&mbar[sel ^ 1], kBytes);
      bulk::load(buf(sel ^ 1), a.ssm + (size_t)nxt * P * N, kBytes, &mbar[sel ^ 1]);
    }
    In nx{};
    if (nxt < total) load_in(nxt, nx);
    const int h = it % H;
    const size_t bh = (size_t)it;

    // ---- scalars (raw == 1 fuses model.py:274-277) -----------------------------------
    float adt, dt, lam;
    if (a.raw) {
      dt = softplusf(cur.dtr);
      adt = fminf(-heavy_tail(cur.ar), -a.a_floor) * dt;
      lam = sigmoidf_(cur.trr);
    } else {
      adt = cur.dtr;
      dt = cur.ar;
      lam = cur.trr;
    }
    const float alpha = expf(adt);
    const float beta = alpha * dt * (1.f - lam);
    const float gamma = dt * lam;

    // ---- preamble: advanced angles, per-row coefficients --------------------------------------
    if (fnorm && tid < 128) {  // per-warp sums of squares of the raw q / k row
      float sq = tid < N ? cur.u * cur.u : 0.f, sk = tid < N ? cur.w * cur.w : 0.f;
      for (int o = 16; o; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      if ((tid & 31) == 0) {
        s_ssq[0][tid >> 5] = sq;
        s_ssq[1][tid >> 5] = sk;
      }
    }
    if (tid < Nr) s_ph[tid] = wrap_fast(cur.ph + tanh_acc(cur.an) * kPi * dt);
    if (tid >= 128 && tid < 128 + P) {
      const int p = tid - 128;
      s_bv[p] = beta * cur.vp;
      s_gv[p] = gamma * cur.vc;
      s_dv[p] = a.d_skip ? a.d_skip[h] * cur.vc : 0.f;
      s_gate[p] = a.z ? cur.zz * sigmoidf_(cur.zz) : 1.f;
      a.state_v[bh * P + p] = cur.vc;
    }
    __syncthreads();
    // rotary columns: x cos + rot_half(x) sin, rot_half = [-hi, lo]  (layout.py:375-398)
    if (tid < N) {
      float u = cur.u, w = cur.w, um = cur.um, wm = cur.wm;
      if (fnorm) {  // layer.py:190-198 on the C / B columns, rounded to the I/O dtype like the layer's norm
        const float rq = rsqrtf((s_ssq[0][0] + s_ssq[0][1] + s_ssq[0][2] + s_ssq[0][3]) / N + a.norm_eps);
        const float rk = rsqrtf((s_ssq[1][0] + s_ssq[1][1] + s_ssq[1][2] + s_ssq[1][3]) / N + a.norm_eps);
        u = rnd_io<T>(u * rq * a.q_norm_w[n]);
        w = rnd_io<T>(w * rk * a.k_norm_w[n]);
        if (j < Nr) {
          um = rnd_io<T>(um * rq * a.q_norm_w[mm]);
          wm = rnd_io<T>(wm * rk * a.k_norm_w[mm]);
        }
      }
      u += cur.bq;
      w += cur.bk;
      if (j < Nr) {
        um += cur.bqm;
        wm += cur.bkm;
      }
      float qv = u, kv = w;
      if (j < Nr) {
        float sn, cs;
        sincos_wrapped(s_ph[j], &sn, &cs);
        const float sgn = n < H2 ? -1.f : 1.f;
        qv = u * cs + sgn * um * sn;
        kv = w * cs + sgn * wm * sn;
      }
      s_q[n] = mmr<MMB>(qv);
      s_k[n] = kv;
      s_kp[n] = cur.kpv;
      a.state_k[bh * N + n] = kv;
    }
    if (tid < Nr) a.phi[bh * Nr + tid] = s_ph[tid];  // nobody reads the old phi any more

    // ---- this item's state has landed ------------------------------------------------------
    if (__syncthreads_or(!umma::mbar_wait(&mbar[sel], (kk >> 1) & 1))) {
      if (tid == 0) atomicExch(&g_m3_dec_error, 21);
      break;
    }

    // ---- S' = alpha S + (beta v_prev) k_prev^T + (gamma v) k~^T; y = (S' q~ + D v) silu(z) -----
    float4* st = buf(sel);
    const int c4 = tid % LPR;
    const float4 q4 = *reinterpret_cast<const float4*>(s_q + 4 * c4);
    const float4 k4 = *reinterpret_cast<const float4*>(s_k + 4 * c4);
    const float4 kp4 = *reinterpret_cast<const float4*>(s_kp + 4 * c4);
    const float2 al2 = f2s(alpha);
    T* yrow = (T*)a.y + bh * P;
#pragma unroll
    for (int m = 0; m < EPT; ++m) {
      const int i = tid + kDecThreads * m;
      if (NF4 % kDecThreads != 0 && i >= NF4) break;  // NF4 % 32 == 0: whole warps stop together
      const int p = i / LPR;
      const float4 S = st[i];
      const float2 bv = f2s(s_bv[p]), gv = f2s(s_gv[p]);
      const float2 s01 = fma2(al2, f2(S.x, S.y), fma2(bv, f2(kp4.x, kp4.y), mul2(gv, f2(k4.x, k4.y))));
      const float2 s23 = fma2(al2, f2(S.z, S.w), fma2(bv, f2(kp4.z, kp4.w), mul2(gv, f2(k4.z, k4.w))));
      st[i] = make_float4(s01.x, s01.y, s23.x, s23.y);
      float2 r01 = s01, r23 = s23;
      if (MMB) {  // bf16 readout operands (kernel_decode.py, BF16 policy)
        r01 = bf2f(f2bf(s01));
        r23 = bf2f(f2bf(s23));
      }
      const float2 pr = fma2(r23, f2(q4.z, q4.w), mul2(r01, f2(q4.x, q4.y)));
      float part = pr.x + pr.y;
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (c4 == 0) stg<T>(yrow + p, (part + s_dv[p]) * s_gate[p]);
    }
    umma::fence_async_smem();  // this thread's state writes, for the bulk store
    __syncthreads();
    if (tid == 0) bulk::store(a.ssm + (size_t)it * P * N, st, kBytes);
    cur = nx;
  }
  if (tid == 0) bulk::wait_all();  // the stores have finished before the CTA's shared memory goes away
}

}  // namespace m3
