// Per-sub-chunk scalar preparation shared by the forward and backward kernels.
#pragma once

#include "m3_common.cuh"

namespace m3 {

// Fill, for tokens t0 .. t0+CS-1 of sequence (b, h):
//   adts[i] = adt, gam[i] = gamma, scl[i] = scale, A[i] = inclusive prefix of adt log2 e
//   dtv[0..CS], lamv[0..CS] (raw boundary only; index CS is the successor token, zero at
//   the sequence end -- reference.py:104-131), av[i] = A_h,t (raw only).
// Must be called by all threads of the block; ends with a __syncthreads.
template <int CS, int NT, class Args>
__device__ __forceinline__ void prep_scalars(const Args& a, int b, int h, int t0, float* adts, float* gam,
                                             float* scl, float* A, float* dtv, float* lamv, float* av) {
  static_assert(CS == 32 || CS == 64, "sub-chunk");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.dims.nheads, L = a.dims.seqlen;
  if (a.raw) {
    for (int i = tid; i <= CS; i += NT) {
      const int t = t0 + i;
      float dt = 0.f, lam = 0.f;
      if (t < L) {
        const size_t o = (size_t)b * a.raw_st.b + (size_t)t * a.raw_st.l + (size_t)h * a.raw_st.h;
        dt = softplusf(a.dt_raw[o] + a.dt_bias[h]);
        lam = sigmoidf_(a.trap_raw[o]);
        if (i < CS) {
          const float aa = fminf(-heavy_tail(a.a_raw[o]), -a.a_floor);
          av[i] = aa;
          adts[i] = aa * dt;
        }
      }
      dtv[i] = dt;
      lamv[i] = lam;
    }
    __syncthreads();
    for (int i = tid; i < CS; i += NT) {
      gam[i] = dtv[i] * lamv[i];
      scl[i] = gam[i] + dtv[i + 1] * (1.f - lamv[i + 1]);
    }
  } else {
    const size_t bh = (size_t)b * H + h;
    for (int i = tid; i < CS; i += NT) {
      const size_t o = bh * L + t0 + i;
      adts[i] = a.adt[o];
      gam[i] = a.gamma[o];
      scl[i] = a.scale[o];
    }
  }
  __syncthreads();
  if (warp == 0) {
    if (CS == 64) {
      const float x0 = adts[2 * lane] * kLog2e, x1 = adts[2 * lane + 1] * kLog2e;
      const float incl = warp_inclusive_scan(x0 + x1);
      A[2 * lane] = incl - x1;
      A[2 * lane + 1] = incl;
    } else {
      A[lane] = warp_inclusive_scan(adts[lane] * kLog2e);
    }
  }
  __syncthreads();
}

// Cumulative rotary angles of tokens t0 .. t0+CS-1 (reference.py:134-157) from the
// head-shared raw angles and this head's dt: phis[i*ld + r] = wrap(carry[r] + sum theta).
// Advances carry[r] past the sub-chunk.  `part` needs NT floats.  All threads call it;
// it ends with a __syncthreads.
template <int CS, int NT, class Args>
__device__ __forceinline__ void phi_scan(const Args& a, int b, int t0, const float* dtv, float* phis, int ld,
                                         float* carry, float* part) {
  const int tid = threadIdx.x, Nr = a.dims.n_angles;
  const int G = NT / Nr;
  const int tpg = (CS + G - 1) / G;
  const int r = tid % Nr, g = tid / Nr;
  const size_t abase = (size_t)b * a.ang_st.b;
  if (g < G) {
    float run = 0.f;
    const int i1 = min(CS, (g + 1) * tpg);
    for (int i = g * tpg; i < i1; ++i) {
      run += tanhf(a.angles[abase + (size_t)(t0 + i) * a.ang_st.l + r]) * kPi * dtv[i];
      phis[i * ld + r] = run;
    }
    part[g * Nr + r] = run;
  }
  __syncthreads();
  if (g < G) {
    float off = carry[r];
    for (int g2 = 0; g2 < g; ++g2) off += part[g2 * Nr + r];
    const int i1 = min(CS, (g + 1) * tpg);
    for (int i = g * tpg; i < i1; ++i) phis[i * ld + r] = wrap2pi(phis[i * ld + r] + off);
  }
  __syncthreads();
  if (g == 0) {
    float tot = carry[r];
    for (int g2 = 0; g2 < G; ++g2) tot += part[g2 * Nr + r];
    carry[r] = wrap2pi(tot);
  }
  __syncthreads();
}

}  // namespace m3
