/*
 * m3_siso.h -- C ABI of the B200 Mamba-3 SISO scan library (libm3siso.so).
 *
 * Plain pointers and sizes only: no CUDA or torch types cross this boundary.  Every
 * tensor pointer is a DEVICE pointer; `stream` is a cudaStream_t passed as void*
 * (NULL = legacy default stream).  Calls are stream-ordered and never synchronise the
 * host.  Each entry point returns M3_OK (0) or a negative M3_ERR_* code, and on error
 * m3_last_error() returns a thread-local message -- the counterpart of the reference's
 * Python ValueErrors (mamba3_pallas/kernel_fwd.py:249-277, layout.py:232-235,
 * layout.py:500-506, reference.py:354-355).
 *
 * Layouts follow the reference kernel boundary (mamba3_pallas/kernel_fwd.py:226-248):
 *   q, k          (B, L, N)      head-shared post-RMSNorm C and B, half-split rotary layout
 *   v, z, y, dy   (B, H, L, P)
 *   adt/gamma/scale (B, H, L) f32;  phi (B, H, L, Nr) f32          [preprocessed boundary]
 *   dt_raw/a_raw/trap_raw (B, L, H) f32; angles (B, L, Nr) f32    [raw boundary]
 *   q_bias, k_bias (H, N) f32;  d_skip, dt_bias (H) f32
 *   state: ssm (B, H, P, N) f32, k (B, H, N) f32 rotated-unscaled, v (B, H, P) f32,
 *          phi (B, H, Nr) f32                  (reference.py:46-63, SISOState)
 * Strides are in ELEMENTS; the innermost axis (N, P or Nr) must be contiguous.  A zero
 * stride selects the contiguous default, so a zero-initialised struct describes dense
 * tensors.
 */
#ifndef M3_SISO_H
#define M3_SISO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  M3_OK = 0,
  M3_ERR_ARG = -1,          /* NULL pointer where one is required, bad flag value      */
  M3_ERR_SHAPE = -2,        /* inconsistent or non-positive dims, L % chunk != 0       */
  M3_ERR_UNSUPPORTED = -3,  /* (N, P, Nr, chunk, dtype) combination not compiled       */
  M3_ERR_WORKSPACE = -4,    /* workspace missing or too small                          */
  M3_ERR_LAUNCH = -5,       /* CUDA launch / attribute error                           */
};

enum { M3_DTYPE_F32 = 0, M3_DTYPE_BF16 = 1 };

/* Matmul-operand policy (mamba3_pallas/layout.py:243-291, DtypePolicy):
 * F32  -- every contraction in true fp32;
 * BF16 -- operands rounded to bf16 where the reference kernel rounds them, fp32
 *         accumulation, fp32 state. */
enum { M3_POLICY_F32 = 0, M3_POLICY_BF16 = 1 };

typedef struct M3Dims {
  int32_t batch, seqlen, nheads, state_dim, headdim, n_angles, chunk;
} M3Dims;

/* Strides (elements) of a rank-3/4 tensor's outer axes.  For (B, L, N)-shaped tensors
 * `h` is ignored; for (B, L, H) raw streams the innermost H stride is `h`. */
typedef struct M3Strides {
  int64_t b, h, l;
} M3Strides;

/* ---------------------------------------------------------------------------------
 * Forward chunked scan.
 * Replaces kernel_fwd.siso_forward (mamba3_pallas/kernel_fwd.py:204-388) when
 * raw == 0, and siso.siso_segment's preprocess + primal (mamba3_pallas/siso.py:154-216,
 * reference.py:160-199) when raw == 1 (softplus / heavy-tail / sigmoid / trapezoid
 * shift / cumulative angles fused into the kernel).
 * ------------------------------------------------------------------------------- */
typedef struct M3FwdArgs {
  M3Dims dims;
  int32_t io_dtype;   /* dtype of q, k, v, z, y (M3_DTYPE_*) */
  int32_t policy;     /* M3_POLICY_* */
  int32_t raw;        /* 0: preprocessed boundary, 1: raw boundary */
  float a_floor;      /* raw boundary: A <= -a_floor */

  const void *q, *k;  M3Strides q_st, k_st;
  const void *v;      M3Strides v_st;
  const void *z;      M3Strides z_st;   /* gate, NULL = ungated */

  const float *adt, *gamma, *scale;     /* raw == 0 */
  const float *phi;

  const float *dt_raw, *a_raw, *trap_raw; M3Strides raw_st;  /* raw == 1 */
  const float *angles;                    M3Strides ang_st;
  const float *dt_bias;

  const float *q_bias, *k_bias;
  const float *d_skip;                  /* NULL = no skip */

  /* Carried state: all of ssm/k/v (and coef for raw == 0) or none. */
  const float *seed_ssm, *seed_k, *seed_v;
  const float *seed_coef;               /* raw == 0: dt_0 (1 - lam_0), (B, H) */
  const float *seed_phi;                /* raw == 1: phi_init (B, H, Nr), may be NULL */

  void *y;            M3Strides y_st;   /* NULL: final state only (tensor-core shapes only) */
  float *final_ssm, *final_k, *final_v;
  float *final_phi;                     /* raw == 1: phi at the last position; may be NULL */

  float *ybar;                          /* optional (B, H, L, P) f32 pre-gate output   */
  void *chunk_states;                   /* optional (B, H, L/chunk, P, N) chunk-start states */
  int32_t chunk_states_dtype;           /* M3_DTYPE_* of chunk_states */

  int32_t kernel;                       /* M3_KERNEL_*: 0 = pick automatically */

  /* Optional: the workspace of a later m3_siso_bwd on the same inputs and seeds.  When the
   * forward runs on tensor cores (m3_siso_fwd_saves_states() == 1) it also writes there the
   * chunk-start states the backward would otherwise recompute; that backward then sets
   * states_ready.  bwd_states_bytes >= m3_siso_bwd_workspace_size(&dims). */
  void *bwd_states;
  size_t bwd_states_bytes;

  /* Optional scratch of m3_siso_fwd_workspace_size(&dims) bytes, 256-byte aligned: the
   * raw-boundary tensor-core forward stores the head-shared rotary rates tanh(angles) pi
   * there once instead of computing them once per head.  NULL is allowed (slower). */
  void *fwd_workspace;
  size_t fwd_workspace_bytes;
  /* 1: fwd_workspace already holds the rates of these angles (an earlier call on the same
   * angles and dims filled it, e.g. the states-only pass before the full one), so they are
   * not computed again.  0: computed by this call. */
  int32_t fwd_workspace_ready;
} M3FwdArgs;

/* Kernel selection for m3_siso_fwd / m3_siso_bwd.  AUTO uses the tcgen05 tensor-core kernel where it
 * applies (bf16 I/O, bf16 policy, N = 128, P = 64, chunk % 128 == 0, n_angles a
 * multiple of 8 and <= 64, 16-byte aligned rows; for the backward also the raw boundary)
 * and the generic CUDA-core kernel otherwise. */
enum { M3_KERNEL_AUTO = 0, M3_KERNEL_GENERIC = 1, M3_KERNEL_TENSORCORE = 2, M3_KERNEL_TENSORCORE_V1 = 3 };
/* M3_KERNEL_TENSORCORE runs the warp-specialised TMA-fed forward where it applies (raw
 * boundary, y requested, no residual outputs) and the two-sequence tensor-core kernel
 * otherwise; M3_KERNEL_TENSORCORE_V1 always runs the latter (kept for comparison). */

int m3_siso_fwd(const M3FwdArgs *args, void *stream);
/* Bytes of M3FwdArgs.fwd_workspace for these dims (B * L * n_angles floats, rounded up). */
size_t m3_siso_fwd_workspace_size(const M3Dims *dims);
/* 1 if m3_siso_fwd(args) takes the tensor-core path and so fills bwd_states, else 0. */
int m3_siso_fwd_saves_states(const M3FwdArgs *args);

/* ---------------------------------------------------------------------------------
 * Backward.  Replaces kernel_bwd.siso_backward (mamba3_pallas/kernel_bwd.py:534-669;
 * kernel 103-355, epilogue 592-651) for raw == 0, and additionally the autodiff of
 * reference.preprocess for raw == 1.  Chunk states are recomputed, not read from the
 * forward: `workspace` (m3_siso_bwd_workspace_size bytes, 256-byte aligned) holds them.
 * All gradient outputs are f32 and are overwritten (not accumulated into).
 * ------------------------------------------------------------------------------- */
typedef struct M3BwdArgs {
  M3Dims dims;
  int32_t io_dtype, policy, raw;
  float a_floor;

  const void *q, *k;  M3Strides q_st, k_st;
  const void *v;      M3Strides v_st;
  const void *z;      M3Strides z_st;
  const float *adt, *gamma, *scale, *phi;
  const float *dt_raw, *a_raw, *trap_raw; M3Strides raw_st;
  const float *angles;                    M3Strides ang_st;
  const float *dt_bias;
  const float *q_bias, *k_bias, *d_skip;
  const float *seed_ssm, *seed_k, *seed_v, *seed_coef, *seed_phi;

  const void *dy;     M3Strides dy_st;    /* cotangent of the gated output y */
  const float *dfinal_ssm, *dfinal_k, *dfinal_v, *dfinal_phi;  /* each may be NULL */

  float *dq, *dk;                         /* (B, L, N), summed over heads */
  float *dv;                              /* (B, H, L, P) */
  float *dz;                              /* (B, H, L, P); required iff z != NULL */
  float *dadt, *dgamma, *dscale, *dphi;   /* raw == 0 */
  float *ddt_raw, *da_raw, *dtrap_raw;    /* raw == 1, (B, L, H) dense */
  float *dangles;                         /* raw == 1, (B, L, Nr) dense */
  float *ddt_bias;                        /* raw == 1, (H) */
  float *dq_bias, *dk_bias;               /* (H, N) */
  float *dd_skip;                         /* (H); required iff d_skip != NULL */
  float *dseed_ssm, *dseed_k, *dseed_v;   /* required iff a seed is given */
  float *dseed_coef;                      /* raw == 0 with a seed */
  float *dseed_phi;                       /* raw == 1 with seed_phi */

  void *workspace;
  size_t workspace_bytes;

  int32_t kernel;                         /* M3_KERNEL_*: 0 = pick automatically */
  int32_t grad_dtype;                     /* M3_DTYPE_* of dv and dz (0 = f32; bf16 halves the
                                             bytes when the primal v / z are bf16) */
  int32_t states_ready;                   /* 1: `workspace` was passed as bwd_states to an
                                             m3_siso_fwd on these inputs that saved them: the
                                             tensor-core backward skips its recompute sweep */
  M3Strides dv_st, dz_st;                 /* element strides of dv / dz over (B, H, L), P
                                             contiguous (0 = dense (B, H, L, P)); e.g. a
                                             (B, L, H, P) buffer seen as (B, H, L, P) */
} M3BwdArgs;

size_t m3_siso_bwd_workspace_size(const M3Dims *dims);
int m3_siso_bwd(const M3BwdArgs *args, void *stream);

/* The same backward for callers that cannot allocate device memory -- a custom call or
 * plugin that is handed only its inputs and outputs by an allocator it does not own, or
 * a server that forbids device allocation after start-up.  No counterpart in the
 * reference (its backward's scratch is XLA-managed VMEM/HBM).  Arguments as for
 * m3_siso_bwd, except that `workspace` / `workspace_bytes` are ignored: the scratch is a
 * fixed array inside the library (m3_siso_bwd_noalloc_scratch_bytes() = 64 MiB per
 * device, resident until exit).  Problems whose m3_siso_bwd_workspace_size() exceeds it
 * fail with M3_ERR_WORKSPACE.  Nothing is allocated.  All calls on a device share the
 * array, so calls that overlap on the GPU race and must be serialised by the caller.
 * The first call on each device (and the first after its primary context was re-created,
 * e.g. by cudaDeviceReset) resolves the array's address; make it before any stream
 * capture.  `stream` must belong to the current device (else M3_ERR_ARG). */
int m3_siso_bwd_noalloc(const M3BwdArgs *args, void *stream);
size_t m3_siso_bwd_noalloc_scratch_bytes(void);

/* ---------------------------------------------------------------------------------
 * The forward split over the sequence length (kernel_fwd._forward_raw_split): when a batch
 * has too few (b, h) sequences to fill the GPU, each is cut into `segments` pieces scanned
 * side by side.  No counterpart kernel in the reference; the result is its segment chaining
 * (mamba3_pallas/siso.py:154-216) applied piece after piece.
 *   prep:  per (b, segment, 64-token tile): partial (B, G, S, H, Nr + 1), S = seqlen /
 *          (64 G), = the tile's sums of tanh(angles) dt per angle, then of adt; coef (B, G, H)
 *          = dt (1 - lam) of each segment's first token.  seqlen % (64 G) == 0.
 *   carry: per (b, h).  With s_loc == NULL (before the states-only pass): partial reduced
 *          into a_seg (B, G, H) = sum adt per segment and the entering angles phi_in
 *          (B*G, H, Nr).  With s_loc, from a states-only pass of every segment from a zero
 *          state at its true angle (s_loc (B*G, H, P, N), k_last (B*G, H, N), v_last
 *          (B*G, H, P)): the entering c_ssm, c_k, c_v of every segment for the full pass.
 * ------------------------------------------------------------------------------- */
#define M3_SPLIT_TILE 64

typedef struct M3SplitPrepArgs {
  int32_t batch, seqlen, nheads, n_angles, segments;
  float a_floor;
  const float *dt_raw, *a_raw, *trap_raw; M3Strides raw_st;   /* (B, L, H), strides as M3FwdArgs */
  const float *angles;                    M3Strides ang_st;   /* (B, L, Nr) */
  const float *dt_bias;
  float *partial, *coef;
} M3SplitPrepArgs;

typedef struct M3SplitCarryArgs {
  int32_t batch, nheads, segments, tiles, state_dim, headdim, n_angles;
  const float *partial;
  float *a_seg;                                               /* written by the angles-only launch */
  const float *coef;
  const float *s_loc, *k_last, *v_last;
  const float *seed_ssm, *seed_k, *seed_v, *seed_phi;         /* (B, H, ...), each may be NULL */
  float *phi_in, *c_ssm, *c_k, *c_v;
} M3SplitCarryArgs;

int m3_siso_split_prep(const M3SplitPrepArgs *args, void *stream);
int m3_siso_split_carry(const M3SplitCarryArgs *args, void *stream);

/* ---------------------------------------------------------------------------------
 * Single-token decode step.  Replaces kernel_decode.decode_step / siso_decode /
 * siso_decode_folded (mamba3_pallas/kernel_decode.py:252-471).  The state buffers are
 * updated IN PLACE (the reference donates them: kernel_decode.py:350-352, 454).
 * raw == 1 also fuses lm_decode_step's length-1 preprocess (model.py:274-277).
 * ------------------------------------------------------------------------------- */
typedef struct M3DecodeArgs {
  int32_t batch, nheads, state_dim, headdim, n_angles;
  int32_t io_dtype, policy, raw;
  float a_floor;
  const void *q, *k;          /* (B, N) */
  int64_t qk_stride_b;        /* 0 = N */
  const void *v, *z;          /* (B, H, P), z may be NULL */
  int64_t vz_stride_b;        /* 0 = H * P (head stride is P) */
  const float *adt, *dt, *lam;            /* raw == 0: (B, H) */
  const float *dt_raw, *a_raw, *trap_raw; /* raw == 1: (B, H) */
  int64_t raw_stride_b;                   /* 0 = H */
  const float *dt_bias;                   /* raw == 1 */
  const float *angles;        /* (B, Nr) raw pre-tanh rates */
  int64_t ang_stride_b;       /* 0 = Nr */
  const float *q_bias, *k_bias, *d_skip;
  float *ssm, *state_k, *state_v, *phi;   /* in/out */
  void *y;                    /* (B, H, P) io_dtype */
  /* Fusions for lm_decode_step (a zeroed tail keeps the plain behaviour): */
  int32_t scalar_dtype;       /* M3_DTYPE_* of dt_raw / a_raw / trap_raw (or adt / dt / lam) and
                                 angles: the in_proj columns can be read as they are */
  const float *q_norm_w, *k_norm_w;  /* (N) gains: q and k are the raw C / B columns and are
                                 RMS-normalised in the kernel (layer.py:190-198: fp32 math,
                                 rounded to io_dtype) before the biases; NULL = already normed */
  float norm_eps;
} M3DecodeArgs;

int m3_siso_decode(const M3DecodeArgs *args, void *stream);

/* Device-side error word: non-zero if a kernel gave up on a bounded wait for the tensor
 * core or for a bulk copy (the kernel then winds down instead of spinning).  Synchronises
 * the device.  `reset` != 0 clears it. */
int m3_device_error(int reset);

/* Host plumbing for callers that stream host buffers through the scan in pieces (no
 * counterpart in the reference, whose inputs are device arrays): `height` rows of `width`
 * bytes, row pitches `dpitch` / `spitch`, between any host (pinned) and device pointers,
 * asynchronous on `stream`.  One strided copy moves an L-segment of every batch row. */
int m3_copy2d_async(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t height,
                    void *stream);

/* RMS normalisation of `rows` rows of `dim` elements (layer.py:190-198):
 * y = x * rsqrt(mean(x^2) + eps) * weight, computed in fp32 and stored in x's dtype.  Row
 * strides in elements; x / y dtype and weight dtype are M3_DTYPE_*.  The decode and
 * inference paths' block, B / C and final norms. */
int m3_rms_norm(const void *x, int64_t x_row_stride, const void *weight, void *y, int64_t y_row_stride, int64_t rows,
                int32_t dim, float eps, int32_t x_dtype, int32_t w_dtype, float *rstd, void *stream);
/* `rstd` (optional, `rows` floats) receives rsqrt(mean(x^2) + eps) per row for the backward:
 * dx = r (dy o w) - x r^3 / dim sum(dy o w o x) (x's dtype, row stride dx_row_stride) and
 * dweight += sum over rows of dy o x r (fp32, `dim` floats, accumulated: zero it first).
 * dim <= 2048. */
int m3_rms_norm_bwd(const void *x, int64_t x_row_stride, const void *weight, const float *rstd, const void *dy,
                    int64_t dy_row_stride, void *dx, int64_t dx_row_stride, float *dweight, int64_t rows, int32_t dim,
                    int32_t x_dtype, int32_t w_dtype, void *stream);

/* ---------------------------------------------------------------------------------
 * Small-batch projection of the decode step (model.py:244-296 at batch <= 8):
 *   out (m, n) = f(x) @ w (+ residual),  w bf16 (k, n) row-major, x / residual / out bf16,
 * with f chosen by x_mode: 0 identity; 1 RMS norm of each x row times norm_w (layer.py:190-198,
 * fp32 math rounded to bf16); 2 value * silu(gate) with value / gate the two k-halves of a
 * 2k-wide x row (model.py:125-137).  residual (optional) is added before the one rounding
 * (torch.addmm's).  Workspace: scratch of m3_gemv_scratch_floats(m, k, n) floats and
 * tickets of (n + 255) / 256 ints that must be zero before the first call (each call leaves
 * them zero).  Deterministic.  m <= 8; every leading dimension and n multiples of 8.
 * ------------------------------------------------------------------------------- */
typedef struct M3GemvArgs {
  int32_t m, k, n, x_mode;
  const void *x;       int64_t x_ld;
  const float *norm_w; float eps;
  const void *w;       int64_t w_ld;
  const void *residual; int64_t r_ld;
  void *out;           int64_t out_ld;
  float *scratch;
  int32_t *tickets;
} M3GemvArgs;

int m3_gemv_bf16(const M3GemvArgs *args, void *stream);

/* ---------------------------------------------------------------------------------
 * Skinny GEMM for the decode step's projections at batch > 8 (the matmul / addmm calls of
 * model.lm_decode_step, mamba3_pallas/model.py:244-296): out (m, n) bf16 =
 * [residual +] a (m, k) bf16 @ w, m <= 256, fp32 accumulation, one bf16 rounding.
 * w_kmajor == 0: w is (k, n), row stride ldw (>= n); w_kmajor == 1: w is (n, k) with k
 * contiguous (the tied head, embed^T).  k % 64 == 0, n % 8 == 0; a and w 16-byte aligned
 * with 16-byte row strides, out / residual 8-byte aligned.  Strides in elements, 0 = dense.
 * residual may equal out (in-place residual add).  Deterministic: K splits are summed in a
 * fixed order.
 * ------------------------------------------------------------------------------- */
typedef struct M3GemmArgs {
  int32_t m, n, k, w_kmajor;
  int32_t ksplit;       /* CTAs sharing K in a cluster: 0 = chosen here, else 1, 2 or 4 */
  int32_t reserved;
  const void *a;        int64_t lda;
  const void *w;        int64_t ldw;
  const void *residual; int64_t ldr;   /* NULL = none */
  void *out;            int64_t ldo;
} M3GemmArgs;

int m3_gemm_bf16(const M3GemmArgs *args, void *stream);
size_t m3_gemv_scratch_floats(int32_t m, int32_t k, int32_t n);

/* ---------------------------------------------------------------------------------
 * Token sampling for generation (mamba3_pallas/train.py:454-500 `_pick_token`, and the
 * window bookkeeping of train.py:559-579): per row, logits -> repetition penalty on the
 * ids whose `seen_count` is > 0 (l / rep_penalty if l > 0 else l * rep_penalty), divide by
 * temperature, keep the nucleus (descending order, ties by higher index first; an entry
 * stays iff the mass strictly before it is < top_p), draw one id.  The draw is a
 * function of (seed, row, counter[row]) only, so a replayed CUDA graph advances by the
 * device-side counter.  After the draw: out_token[row] = id; history[row][counter] = id
 * (if history and counter < history_cap); a stop id sets done[row] (rows with done set
 * are skipped); otherwise the id enters the window ring (length rep_window, state
 * [length, head] in window_state) and seen_count follows it.  counter[row] += 1.
 * ------------------------------------------------------------------------------- */
typedef struct M3SampleArgs {
  int32_t batch, vocab;
  int32_t logits_dtype;        /* M3_DTYPE_F32 or M3_DTYPE_BF16 */
  int64_t logits_ld;           /* elements between rows (>= vocab) */
  const void *logits;          /* (batch, logits_ld) */
  float temperature, top_p, rep_penalty;
  uint64_t seed;
  int64_t *counter;            /* (batch,) draws so far; NULL = always 0 */
  int32_t *seen_count;         /* (batch, vocab) window occurrence counts; NULL = no penalty */
  int32_t *window;             /* (batch, rep_window) ring; NULL = no window update */
  int32_t *window_state;       /* (batch, 2) [length, head] */
  int32_t rep_window;
  const int64_t *stop_ids;     /* n_stop ids (device) */
  int32_t n_stop;
  int32_t *done;               /* (batch,) or NULL */
  int64_t *out_token;          /* (batch,) */
  int64_t *history;            /* (batch, history_cap) or NULL */
  int64_t history_cap;
  void *scratch;               /* (batch, vocab) x 8 bytes of workspace; only read when
                                  vocab > 184320 (else a row lives in shared memory), may
                                  be NULL below that */
  float *probs_out;            /* optional (batch, probs_ld): the filtered distribution */
  int64_t probs_ld;
} M3SampleArgs;

int m3_sample_tokens(const M3SampleArgs *args, void *stream);

/* The gated MLP activation of model.py:125-137 at inference: out (rows, k) = value * silu(gate),
 * value / gate the two k-wide halves of each x row (bf16; silu(gate) and the product each
 * rounded to bf16 like the two torch ops it replaces).  k and the row strides multiples of 8,
 * 16-byte aligned rows. */
int m3_gated_act_bf16(const void *x, int64_t x_row_stride, void *out, int64_t out_row_stride, int64_t rows,
                      int32_t k, void *stream);

/* Last error message of this thread ("" if none). */
const char *m3_last_error(void);

/* Library version, for the bindings' load check. */
int m3_version(void);

#ifdef __cplusplus
}
#endif

#endif /* M3_SISO_H */
