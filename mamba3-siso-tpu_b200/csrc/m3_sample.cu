// Token sampling for generation (mamba3_pallas/train.py:454-500, _pick_token): repetition
// penalty on the recent window, temperature, nucleus (top-p) filter, categorical draw --
// one 8-CTA cluster per row (partials combined through distributed shared memory), no sort.  Plus the window bookkeeping of train.py:559-579 on the
// device, so that a generation loop can run as a replayed CUDA graph with no host round
// trip per token.
//
// Nucleus rule of the reference: sort descending (argsort reversed, so among equal values
// the higher index comes first), keep entry i iff the probability mass strictly before it
// in that order is < top_p.  Here the probabilities are fixed point: q_i = round(2^32 *
// exp(x_i - max x)), so every sum is an exact integer (order-independent, deterministic),
// and the cut is found by a radix select over the order-preserving 32-bit key of x:
// four 8-bit rounds of a mass histogram locate the key K* of the group at which the mass
// from the top crosses top_p * sum(q).  Entries with key > K* are kept; of the group with
// key K*, the n_keep highest indices (n_keep = ceil((T - mass above) / q_K*)).
// The draw: u = floor(U * kept mass) with U uniform in [0, 1) from SplitMix64 (Steele,
// Lea & Flood 2014) of (seed, row, step counter); the token is the first index, in index
// order, whose running kept mass exceeds u.
#include <cuda_bf16.h>
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "m3_internal.h"

namespace m3 {
namespace {

constexpr int kCluster = 8;                 // CTAs per row (portable cluster size)
constexpr int kThreads = 512, kWarps = kThreads / 32;
constexpr size_t kMaxEntBytes = 180 * 1024;  // dynamic shared memory for one CTA's entries
constexpr double kQScale = 4294967296.0;  // 2^32: sum over a row stays below 2^53

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// order-preserving map float -> uint32 (larger float, larger key)
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float kfloat(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
// fixed-point mass of x against the row max, saturated to 32 bits (NaN from an all -inf
// row -> 0).  Every later pass reads the stored value, so the passes agree exactly.
__device__ __forceinline__ uint32_t qmass(float x, float mx) {
  const float e = expf(x - mx);
  if (!(e > 0.f)) return 0u;
  const double v = rint((double)e * kQScale);
  return v >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)v;
}

// Add q to `bin` of this warp's private histogram, kept as two 32-bit halves (low and high
// 16 bits of each q; below 2^32 per counter while a warp's range is < 65,536 entries, i.e.
// vocab < 8,388,608) so that the
// shared-memory atomics are native 32-bit adds -- a row's keys share their top bits, and
// many lanes of a warp hit the same bin.
__device__ __forceinline__ void hist_add(uint32_t (*hist)[256], uint32_t bin, uint32_t q, bool active) {
  if (active) {
    atomicAdd(&hist[0][bin], q & 0xFFFFu);
    atomicAdd(&hist[1][bin], q >> 16);
  }
}

struct Smem {
  uint32_t whist[kWarps][2][256];         // per-warp private histograms (low, high halves)
  unsigned long long chist[2][256];       // this CTA's histogram (double-buffered by round)
  unsigned long long ghist[256];          // the row's histogram (sum over the cluster)
  unsigned long long wsum[kWarps];
  unsigned long long cval[4];             // this CTA's partials read by the cluster: Zq, kept mass
  float wmax[kWarps];
  float cmax;
  int wcnt[kWarps];
  int ccnt;
  unsigned long long zq, above, nkeep, zk;
  uint32_t prefix, kstar;
  int all_kept, skip;
};

template <typename T>
__device__ __forceinline__ float load_logit(const T* p);
template <>
__device__ __forceinline__ float load_logit<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    sample_kernel(M3SampleArgs a, bool ent_in_smem) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ Smem s;
  const int crank = (int)cluster.block_rank();
  const int row = blockIdx.x / kCluster, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.vocab;
  const bool skip = a.done ? a.done[row] != 0 : false;  // uniform over the cluster
  if (skip) return;
  // read before the first cluster barrier: the CTA that draws the token advances it
  const int64_t step = a.counter ? a.counter[row] : 0;
  // contiguous index ranges: CTA crank, then warp, in multiples of 32
  const int per_cta = ((V + kCluster * 32 - 1) / (kCluster * 32)) * 32;
  const int per_w = ((per_cta + kWarps * 32 - 1) / (kWarps * 32)) * 32;
  const int c0 = crank * per_cta, c1 = min(V, c0 + per_cta);
  const int w0 = c0 + warp * per_w, w1 = min(c1, w0 + per_w);
  const T* lg = reinterpret_cast<const T*>(a.logits) + (size_t)row * a.logits_ld;
  // (key, q) per entry: this CTA's range in shared memory when it fits, else the workspace
  extern __shared__ uint2 ent[];
  uint2* kq = ent_in_smem ? ent : reinterpret_cast<uint2*>(a.scratch) + (size_t)row * V + c0;
  const int32_t* seen = a.seen_count ? a.seen_count + (size_t)row * V : nullptr;
  const unsigned le_mask = (2u << lane) - 1u;
  uint32_t (*wh)[256] = s.whist[warp];

  auto cluster_sum = [&](const unsigned long long* local) {  // sum of `local` over the cluster's CTAs
    unsigned long long v = 0ull;
    for (int r = 0; r < kCluster; ++r) v += *cluster.map_shared_rank(local, r);
    return v;
  };

  // pass 1: penalised, tempered logits; row max
  float mx = -INFINITY;
#pragma unroll 8
  for (int i = w0 + lane; i < w1; i += 32) {
    float l = load_logit(lg + i);
    if (seen && seen[i] > 0) l = l > 0.f ? l / a.rep_penalty : l * a.rep_penalty;
    l = l / a.temperature;
    kq[i - c0].x = __float_as_uint(l);
    mx = fmaxf(mx, l);
  }
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) s.wmax[warp] = mx;
  for (int j = lane; j < 256; j += 32) wh[0][j] = wh[1][j] = 0u;
  __syncthreads();
  if (tid == 0) {
    float m = s.wmax[0];
    for (int w = 1; w < kWarps; ++w) m = fmaxf(m, s.wmax[w]);
    s.cmax = m;
  }
  cluster.sync();
  mx = -INFINITY;
  for (int r = 0; r < kCluster; ++r) mx = fmaxf(mx, *cluster.map_shared_rank(&s.cmax, r));

  // pass 2: keys and fixed-point masses, total mass, first radix round's histogram
  unsigned long long zq = 0ull;
  for (int base = w0; base < w1; base += 32) {
    const int i = base + lane;
    uint32_t k = 0u, q = 0u;
    if (i < w1) {
      const float x = __uint_as_float(kq[i - c0].x);
      k = fkey(x);
      q = qmass(x, mx);
      kq[i - c0] = make_uint2(k, q);
    }
    zq += q;
    hist_add(wh, k >> 24, q, q != 0u);
  }
  for (int o = 16; o; o >>= 1) zq += __shfl_xor_sync(0xffffffffu, zq, o);
  if (lane == 0) s.wsum[warp] = zq;
  __syncthreads();
  if (tid == 0) {
    unsigned long long z = 0ull;
    for (int w = 0; w < kWarps; ++w) z += s.wsum[w];
    s.cval[0] = z;
    s.prefix = 0u;
    s.above = 0ull;
    s.all_kept = 0;
  }

  double thr = 0.0;
  for (int r = 0; r < 4; ++r) {
    const int shift = 24 - 8 * r, buf = r & 1;
    if (r > 0) {
      const uint32_t pre = s.prefix;
      for (int base = w0; base < w1; base += 32) {
        const int i = base + lane;
        const uint2 e = i < w1 ? kq[i - c0] : make_uint2(0u, 0u);
        const bool in = i < w1 && e.y != 0u && (e.x >> (shift + 8)) == pre;
        hist_add(wh, (e.x >> shift) & 255u, e.y, in);
      }
    }
    __syncthreads();
    if (tid < 256) {  // this CTA's histogram; private ones cleared for the next round
      unsigned long long v = 0ull;
      for (int w = 0; w < kWarps; ++w) {
        v += (unsigned long long)s.whist[w][0][tid] + ((unsigned long long)s.whist[w][1][tid] << 16);
        s.whist[w][0][tid] = s.whist[w][1][tid] = 0u;
      }
      s.chist[buf][tid] = v;
    }
    cluster.sync();
    if (tid < 256) s.ghist[tid] = cluster_sum(&s.chist[buf][tid]);
    if (r == 0 && tid == 0) s.zq = cluster_sum(&s.cval[0]);
    __syncthreads();
    // top_p <= 0 keeps the top-1 alone (mass strictly before it is 0 < 0.5 fixed-point units)
    thr = fmax((double)a.top_p * (double)s.zq, 0.5);
    if (warp == 0) {  // lane l owns bins 255-8l .. 248-8l (descending); find where thr is crossed
      unsigned long long loc = 0ull;
#pragma unroll
      for (int j = 0; j < 8; ++j) loc += s.ghist[255 - 8 * lane - j];
      unsigned long long incl = loc;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned long long above = s.above;
      const bool cross = (double)(above + incl) >= thr && (double)(above + incl - loc) < thr;
      const unsigned m = __ballot_sync(0xffffffffu, cross);
      if (m == 0u) {
        if (lane == 0 && r == 0) s.all_kept = 1;  // total mass below thr (top_p >= 1)
      } else if (lane == __ffs(m) - 1) {
        unsigned long long acc = above + incl - loc;
        for (int j = 0; j < 8; ++j) {
          const int bin = 255 - 8 * lane - j;
          const unsigned long long h = s.ghist[bin];
          if ((double)(acc + h) >= thr) {
            s.prefix = (s.prefix << 8) | (uint32_t)bin;
            s.above = acc;
            break;
          }
          acc += h;
        }
      }
    }
    __syncthreads();
    if (s.all_kept) break;
  }
  const bool all_kept = s.all_kept != 0;
  if (tid == 0 && !all_kept) {
    const uint32_t ks = s.prefix;
    s.kstar = ks;
    const unsigned long long pk = qmass(kfloat(ks), mx);
    // smallest n with above + n * pk >= thr; at least 1 (the group's first entry crosses)
    unsigned long long n = (unsigned long long)ceil((thr - (double)s.above) / (double)pk);
    if (n < 1ull) n = 1ull;
    while (n > 1ull && (double)(s.above + (n - 1ull) * pk) >= thr) --n;
    while ((double)(s.above + n * pk) < thr) ++n;
    s.nkeep = n;
  }
  __syncthreads();
  const uint32_t kstar = all_kept ? 0u : s.kstar;
  const unsigned long long nkeep = all_kept ? 0ull : s.nkeep;

  // K* entries per warp range, and per CTA (for the ranks counted from the top index)
  int cnt = 0;
  if (!all_kept)
    for (int i = w0 + lane; i < w1; i += 32) cnt += kq[i - c0].x == kstar;
  for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) s.wcnt[warp] = cnt;
  __syncthreads();
  if (tid == 0) {
    int c = 0;
    for (int w = 0; w < kWarps; ++w) c += s.wcnt[w];
    s.ccnt = c;
  }
  cluster.sync();
  long long higher = 0;  // K* entries at indices above this warp's range
  for (int r = crank + 1; r < kCluster; ++r) higher += *cluster.map_shared_rank(&s.ccnt, r);
  for (int w = warp + 1; w < kWarps; ++w) higher += s.wcnt[w];
  const int wtot = s.wcnt[warp];

  auto kept_q = [&](int i, int& below) -> uint32_t {
    const uint2 e = i < w1 ? kq[i - c0] : make_uint2(0u, 0u);
    const bool isk = !all_kept && i < w1 && e.x == kstar;
    const unsigned bm = __ballot_sync(0xffffffffu, isk);
    const long long rank = higher + (wtot - (below + __popc(bm & le_mask)));  // K* entries at > i
    const bool keep = i < w1 && (all_kept || e.x > kstar || (isk && rank < (long long)nkeep));
    below += __popc(bm);
    return keep ? e.y : 0u;
  };
  unsigned long long wk = 0ull;
  {
    int below = 0;
    for (int base = w0; base < w1; base += 32) wk += kept_q(base + lane, below);
  }
  for (int o = 16; o; o >>= 1) wk += __shfl_xor_sync(0xffffffffu, wk, o);
  if (lane == 0) s.wsum[warp] = wk;
  __syncthreads();
  if (tid == 0) {
    unsigned long long z = 0ull;
    for (int w = 0; w < kWarps; ++w) z += s.wsum[w];
    s.cval[1] = z;
  }
  cluster.sync();
  unsigned long long zk = 0ull, pre = 0ull;  // kept mass of the row; of the CTAs before this one
  for (int r = 0; r < kCluster; ++r) {
    const unsigned long long v = *cluster.map_shared_rank(&s.cval[1], r);
    zk += v;
    if (r < crank) pre += v;
  }
  for (int w = 0; w < warp; ++w) pre += s.wsum[w];

  if (a.probs_out) {  // the filtered distribution (kept mass / total kept mass)
    float* po = a.probs_out + (size_t)row * a.probs_ld;
    int below = 0;
    for (int base = w0; base < w1; base += 32) {
      const uint32_t q = kept_q(base + lane, below);
      if (base + lane < w1) po[base + lane] = (float)((double)q / (double)zk);
    }
  }

  // the draw: the warp whose range holds u walks it
  const uint64_t r64 = splitmix64(a.seed ^ splitmix64(((uint64_t)row << 40) ^ (uint64_t)step));
  const double U = (double)(r64 >> 11) * (1.0 / 9007199254740992.0);
  unsigned long long u = (unsigned long long)(U * (double)zk);
  if (u >= zk && zk > 0ull) u = zk - 1ull;
  int64_t tok = -1;
  if (zk > 0ull && u >= pre && u < pre + s.wsum[warp]) {
    int below = 0;
    unsigned long long run = pre;
    for (int base = w0; base < w1; base += 32) {
      const unsigned long long q = kept_q(base + lane, below);
      unsigned long long incl = q;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, q > 0ull && run + incl > u);
      if (hit) {
        tok = base + __ffs(hit) - 1;
        break;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  } else if (zk == 0ull && crank == 0 && warp == 0) {
    tok = 0;  // no finite logit in the row
  }

  // bookkeeping (train.py:559-579), by the one lane that found the token: output, history,
  // stop, window ring and seen counts, draw counter
  if (tok >= 0 && lane == 0) {
    a.out_token[row] = tok;
    if (a.history && step < a.history_cap) a.history[(size_t)row * a.history_cap + step] = tok;
    bool stop = false;
    for (int j = 0; j < a.n_stop; ++j) stop |= a.stop_ids[j] == tok;
    if (stop && a.done) a.done[row] = 1;
    if (!stop && a.window && a.rep_window > 0) {
      int32_t* ring = a.window + (size_t)row * a.rep_window;
      int32_t* st = a.window_state + 2 * row;  // [length, head]
      int32_t* cntp = a.seen_count + (size_t)row * V;
      int len = st[0], head = st[1];
      if (len < a.rep_window) {
        ring[(head + len) % a.rep_window] = (int32_t)tok;
        ++len;
      } else {
        const int32_t dropped = ring[head];
        ring[head] = (int32_t)tok;
        head = (head + 1) % a.rep_window;
        cntp[dropped] -= 1;
      }
      cntp[tok] += 1;
      st[0] = len;
      st[1] = head;
    }
    if (a.counter) a.counter[row] = step + 1;
  }
  cluster.sync();  // no CTA leaves while others may still read its shared memory
}

}  // namespace

int launch_sample(const M3SampleArgs& a, cudaStream_t s) {
  // a CTA's entries stay in shared memory when its range fits beside the static arrays
  const int per_cta = ((a.vocab + kCluster * 32 - 1) / (kCluster * 32)) * 32;
  const size_t dyn = (size_t)per_cta * sizeof(uint2);
  const bool in_smem = dyn <= kMaxEntBytes;
  auto* kern = a.logits_dtype == M3_DTYPE_BF16 ? sample_kernel<__nv_bfloat16> : sample_kernel<float>;
  static bool attr_done[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int ti = a.logits_dtype == M3_DTYPE_BF16 ? 1 : 0;
  if (dev < 64 && !attr_done[ti][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxEntBytes) != cudaSuccess)
      return check_launch("m3_sample_tokens: cudaFuncSetAttribute");
    attr_done[ti][dev] = true;
  }
  kern<<<a.batch * kCluster, kThreads, in_smem ? dyn : 0, s>>>(a, in_smem);
  return check_launch("m3_sample_tokens");
}

}  // namespace m3
