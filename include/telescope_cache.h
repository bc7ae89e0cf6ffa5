/*
 * telescope_cache.h -- C ABI of the B200 (sm_100a) telescoping-attention
 * library (libtelescope_b200.so).
 *
 * Every entry point takes plain pointers, sizes and a cudaStream_t (passed as
 * void*), and returns an int status (TC_OK on success).  Device tensors are
 * dense row-major ("BSHD") buffers:
 *
 *   q          [B, N, Hq, Dk]        out   [B, N, Hq, Dv]     lse [B, N, Hq] f32
 *   packed k   [B, total, Hkv, Dk]   packed v [B, total, Hkv, Dv]
 *   packed w   [B, total, Hkv]       (total = sum of level lengths N >> l)
 *
 * GQA maps query head hq to KV head hq / (Hq / Hkv).  The schedule (fmap,
 * cache_size, N) is described by tc_schedule, built by tc_schedule_init.
 *
 * Each function names the reference interface it replaces (paths inside the
 * Knarf04/telescope_cache project).
 */
#ifndef TELESCOPE_CACHE_H
#define TELESCOPE_CACHE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TC_MAX_LEVELS 16

/* status codes */
#define TC_OK 0
#define TC_ERR_ARG 1          /* invalid argument (shape, schedule, pointer) */
#define TC_ERR_UNSUPPORTED 2  /* valid, but not supported by this build     */
#define TC_ERR_CUDA 3         /* a CUDA runtime call or launch failed        */
#define TC_ERR_SCHEDULE 4     /* fmap not dyadically aligned / not 1..L     */

/* element types */
#define TC_F32 0
#define TC_BF16 1
#define TC_F16 2

/* positional modes (reference.py:675-768) */
#define TC_POS_NONE 0
#define TC_POS_ROPE 1
#define TC_POS_RELATIVE 2

/* device status word bits, OR-ed by kernels into a caller-owned int32 */
#define TC_DEV_WAIT_TIMEOUT 1  /* a bounded mbarrier wait gave up           */
#define TC_DEV_BAD_INDEX 2     /* a bounds check rejected an index          */

typedef struct tc_schedule {
  int32_t num_levels;                  /* L + 1                              */
  int32_t cache_size;
  int32_t seq_len;                     /* N                                  */
  int32_t coarsest_span;               /* range_spec.coarsest_lifetime_span  */
  int32_t act[TC_MAX_LEVELS];          /* activation times a[0..L]           */
  int32_t level_len[TC_MAX_LEVELS];    /* N >> l                             */
  int64_t offsets[TC_MAX_LEVELS + 1];  /* packed level offsets               */
} tc_schedule;

/* ------------------------------------------------------------------------ */
/* library                                                                   */
/* ------------------------------------------------------------------------ */

/* Library version, for the Python loader's sanity check. */
int tc_version(void);

/* Number of CUDA kernels this library has launched since it was loaded. */
int64_t tc_launch_count(void);

/* ------------------------------------------------------------------------ */
/* schedule (host side; pure integer)                                        */
/* ------------------------------------------------------------------------ */

/* fmap values fmap[1..L] (fmap_vals[i] = fmap[i+1]) -> activation times,
 * level lengths, packed offsets and the coarsest lifetime span.
 * Replaces RangeSpec.from_fmap + activation_times_from_fmap +
 * coarsest_lifetime_span (telescoping_attn/range_spec.py:26-126, :287-317).
 * Returns TC_ERR_SCHEDULE on keys/alignment errors, TC_ERR_ARG on sizes. */
int tc_schedule_init(const int32_t* fmap_vals, int32_t num_summary_levels,
                     int32_t cache_size, int32_t seq_len, tc_schedule* out);

/* Same, from explicit activation times (RangeSpec(activation_times, ...),
 * range_spec.py:57-76). */
int tc_schedule_from_times(const int32_t* act, int32_t num_levels, int32_t cache_size,
                           int32_t seq_len, tc_schedule* out);

/* Visible-set statistics over every query q in [0, N):
 * out[0] = min_q |A(q)|, out[1] = max_q |A(q)|, out[2] = sum_q |A(q)|.
 * Lets the host raise the reference's RuntimeError for an empty row
 * (reference.py:1060-1064) and ValueError for a relative table that is too
 * small (reference.py:441-452) before any launch. */
int tc_schedule_stats(const tc_schedule* s, int64_t* out3);

/* Per-level decode ring capacities (reference.py:1739-1772). caps_out has
 * num_levels entries. Returns TC_ERR_ARG if the fine levels exceed the cache. */
int tc_decode_caps(const int32_t* act, int32_t num_levels, int32_t cache_size,
                   int32_t* caps_out);

/* Per-query level bounds [lo, hi) (EMPTY = 0,0) from the branch-free closed
 * forms, evaluated on the HOST: out[(i * num_levels + l) * 2 + {0,1}].
 * range_spec.level_row_bounds / range_bounds (range_spec.py:142-171, :324-336). */
int tc_range_bounds_host(const tc_schedule* s, const int32_t* qs, int32_t n, int32_t* out);

/* Hulls on the HOST: kind 0 = fwd_bounds over query blocks [lo[i], hi[i]),
 * kind 1 = bwd_bounds over node tiles [lo[i], hi[i]) at `level`.
 * out[i*2 + {0,1}] (range_spec.py:187-202, :256-281, :360-402). */
int tc_hulls_host(const tc_schedule* s, int32_t kind, int32_t level, const int32_t* lo,
                  const int32_t* hi, int32_t n, int32_t* out);

/* ------------------------------------------------------------------------ */
/* device debug                                                              */
/* ------------------------------------------------------------------------ */

/* The same per-query bounds, computed by a CUDA kernel (the closed forms the
 * attention kernels use).  qs/out are DEVICE pointers, layout as above. */
int tc_range_bounds_device(const tc_schedule* s, const int32_t* qs, int32_t n, int32_t* out,
                           void* stream);

/* ------------------------------------------------------------------------ */
/* Phase 1: dyadic summary tree                                              */
/* ------------------------------------------------------------------------ */

typedef struct tc_tree_args {
  int32_t B, N, Hq, Hkv, Dk, Dv;
  int32_t num_summary_levels;  /* L (tree has L + 1 levels)                 */
  int32_t dtype;               /* q/k/v/packed element type                 */
  int32_t w_dtype;             /* packed w element type                     */
  const void* q;               /* [B, N, Hq, Dk]  (qk weight mode)          */
  const void* k;               /* [B, N, Hkv, Dk] pre-conv keys             */
  const void* v;               /* [B, N, Hkv, Dv]                           */
  const void* w0;              /* [B, N, Hkv] precomputed level-0 weights
                                  (linear mode), or NULL for qk mode        */
  const void* k_conv_w;        /* [Hkv*Dk, K] or NULL                       */
  const void* v_conv_w;        /* [Hkv*Dv, K] or NULL                       */
  int32_t conv_dtype;          /* element type of the conv weights          */
  int32_t conv_k;              /* conv width K (0 = no conv)                */
  void* k_packed;              /* [B, total, Hkv, Dk] out                   */
  void* v_packed;              /* [B, total, Hkv, Dv] out                   */
  void* w_packed;              /* [B, total, Hkv]     out                   */
  int64_t total;               /* sum_l (N >> l)                            */
} tc_tree_args;

/* Fused short conv + merge weights + all-level softmax pair merges + packing
 * into the level-major buffer.  Replaces short_conv, compute_summary_weights,
 * build_dyadic_summaries and pack_levels (reference.py:117-211, :465-640). */
int tc_build_tree(const tc_tree_args* a, void* stream);

/* Phase-1 VJP: the backward of build_dyadic_summaries (reference.py:465-584,
 * which the reference takes through torch autograd), from the upstream
 * gradients of the packed levels to the gradients of the level-0 (post-conv)
 * keys, values and merge weights, and of q.
 *
 * From the coarsest level down every parent's gradient goes to its two
 * children (alpha = softmax(w0, w1), parent = sum alpha child, w_parent =
 * logsumexp(w0, w1)).  In qk weight mode (q non-NULL, detach 0) the level-0
 * weight gradient then goes through w = logsumexp_e(q_e . k / sqrt(Dk)):
 * dq is written and its k part is in dk0.  With q NULL (linear weights) or
 * detach 1 dq is not touched; dw0, when non-NULL, receives the level-0
 * weight gradient (for the caller's x @ w_proj^T GEMMs).
 *
 * Upstream gradients have the element type of what they are the gradient
 * of (gk / gv: dtype, gw: w_dtype); a NULL one counts as zeros.  dq has
 * dtype; dk0 / dv0 have d0_dtype (dtype, or TC_F32 for a following conv
 * VJP).  Levels above the 64-leaf tiles (L > 6) need device scratch of
 * tc_tree_bwd_scratch_bytes(a) bytes (0 otherwise). */
typedef struct tc_tree_bwd_args {
  int32_t B, N, Hq, Hkv, Dk, Dv;
  int32_t num_summary_levels;  /* L (tree has L + 1 levels)                 */
  int32_t dtype;               /* q, packed k / v, gk / gv element type     */
  int32_t w_dtype;             /* packed w and gw element type              */
  int32_t detach;              /* detach_weights: no gradient through w     */
  const void* q;               /* [B, N, Hq, Dk] (qk mode) or NULL          */
  const void* k_packed;        /* [B, total, Hkv, Dk] forward levels        */
  const void* v_packed;        /* [B, total, Hkv, Dv]                       */
  const void* w_packed;        /* [B, total, Hkv]                           */
  const void* gk_packed;       /* [B, total, Hkv, Dk] upstream, or NULL     */
  const void* gv_packed;       /* [B, total, Hkv, Dv] upstream, or NULL     */
  const void* gw_packed;       /* [B, total, Hkv] upstream, or NULL         */
  void* dq;                    /* [B, N, Hq, Dk] out (qk mode)              */
  int32_t dq_dtype;            /* must equal dtype                          */
  int32_t d0_dtype;            /* dtype or TC_F32                           */
  void* dk0;                   /* [B, N, Hkv, Dk] out                       */
  void* dv0;                   /* [B, N, Hkv, Dv] out                       */
  float* dw0;                  /* [B, N, Hkv] out, or NULL                  */
  void* scratch;               /* device scratch                            */
  int64_t scratch_bytes;
  int64_t total;               /* sum_l (N >> l)                            */
} tc_tree_bwd_args;
int64_t tc_tree_bwd_scratch_bytes(const tc_tree_bwd_args* a);  /* -1 on bad arguments */
int tc_build_tree_bwd(const tc_tree_bwd_args* a, void* stream);

/* VJP of short_conv (reference.py:167-211) for one tensor x [B, N, C] with
 * conv weight w [C, K]: dx[t] = dy[t] + sum_j w[c, j] dy[t + K - 1 - j] and
 * dw[c, j] = sum_{b, t} dy[t, c] x[t - K + 1 + j, c].  dy is fp32; dx is
 * written in dtype, dw in fp32.  The dw reduction runs in a fixed order
 * (per-chunk partials, then their sum): partial_floats must be at least
 * B * ceil(N / 256) * C * K. */
int tc_short_conv_bwd(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                      int32_t w_dtype, const void* w, const float* dy, void* dx, float* dw, float* partials,
                      int64_t partial_floats, void* stream);

/* tc_short_conv_bwd with segment resets: seq_idx [B, N] int32 (NULL = one
 * sequence per batch row) pairs a tap between rows s and t only when
 * seq_idx[b, s] == seq_idx[b, t].  The VJP of tc_short_conv_seg.  No
 * reference counterpart: the reference's short_conv leaves resets across
 * packed examples as a TODO (reference.py:186-189). */
int tc_short_conv_seg_bwd(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                          int32_t w_dtype, const void* w, const int32_t* seq_idx, const float* dy, void* dx,
                          float* dw, float* partials, int64_t partial_floats, void* stream);

/* Projection epilogues of tc_linear */
#define TC_LIN_STORE 0  /* out = A B^T                                  */
#define TC_LIN_GATE 1   /* out = SiLU(A B^T) * aux (aux: out's type)    */

/* out[m, n] = sum_k A[m, k] B[n, k] (x @ W^T) for row-major A [M, K] (row
 * stride lda), B [N, K] (ldb) and out [M, N] (ldo), fp32 accumulation; with
 * TC_LIN_GATE, out = SiLU(A B^T) * aux for aux [M, N] (ld_aux, out's type).
 * Replaces the x.matmul(W.t()) of compute_linear_weights (reference.py:148-164),
 * compute_relative_states (reference.py:374-395), apply_output_gate
 * (reference.py:1187-1219, gate and product fused) and the relative-bias
 * logits states @ proj (reference.py:764-767).  bf16/f16 operands of one type
 * (lda, ldb multiples of 8, 16-byte aligned) run on the tensor cores with an
 * output of that type or f32; other types run a SIMT kernel.  With few
 * row blocks and a long K (a decode-time projection) the tensor-core path
 * splits K and needs caller-owned, 16-byte aligned fp32 scratch of
 * tc_linear_scratch_floats(M, N, K, out_dtype) floats (0: none); with less
 * it runs unsplit.  dev_status (optional) receives TC_DEV_WAIT_TIMEOUT if a
 * bounded wait gave up. */
int64_t tc_linear_scratch_floats(int64_t M, int32_t N, int32_t K, int32_t out_dtype);
int tc_linear(int64_t M, int32_t N, int32_t K, int32_t a_dtype, const void* a, int64_t lda,
              int32_t b_dtype, const void* b, int64_t ldb, int32_t out_dtype, void* out, int64_t ldo,
              int32_t epilogue, const void* aux, int64_t ld_aux, float* scratch, int64_t scratch_floats,
              int32_t* dev_status, void* stream);

/* out[n1, n2] = sum_m A[m, n1] B[m, n2] for row-major A [M, N1] and B [M, N2]
 * (the weight gradient dW = dy^T x of a projection, autograd of
 * x @ W^T in reference.py:148-164 and :1187-1219), fp32 accumulation,
 * deterministic (row chunks reduced in order).  bf16/f16 operands of one
 * type run on the tensor cores (B read in place, A transposed into the
 * scratch), others on a SIMT kernel.  scratch: caller-owned, 16-byte
 * aligned, tc_linear_wgrad_scratch_floats(M, N1, N2) floats (0: none).
 * dev_status (optional) as for tc_linear. */
int64_t tc_linear_wgrad_scratch_floats(int64_t M, int32_t N1, int32_t N2);
int tc_linear_wgrad(int64_t M, int32_t N1, int32_t N2, int32_t a_dtype, const void* a, int64_t lda,
                    int32_t b_dtype, const void* b, int64_t ldb, int32_t out_dtype, void* out, int64_t ldo,
                    float* scratch, int64_t scratch_floats, int32_t* dev_status, void* stream);

/* w[b, t, h] = x[b, t, :] . w_proj[h, :] (compute_linear_weights,
 * reference.py:148-164).  x [rows, E], w_proj [H, E], out [rows, H]. */
int tc_linear_weights(int64_t rows, int32_t E, int32_t H, int32_t x_dtype, const void* x,
                      int32_t p_dtype, const void* w_proj, int32_t out_dtype, void* out,
                      void* stream);

/* w[b, t, hkv] = logsumexp_e(q[b, t, hkv*E + e] . k[b, t, hkv] / sqrt(Dk)),
 * q [B, N, Hq, Dk], k [B, N, Hkv, Dk], out [B, N, Hkv] (compute_summary_weights,
 * reference.py:117-145). */
int tc_qk_weights(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t Dk, int32_t dtype,
                  const void* q, const void* k, int32_t out_dtype, void* out, void* stream);

/* VJP of tc_qk_weights (the autograd of compute_summary_weights,
 * reference.py:117-145) for an upstream gradient dw [B, N, Hkv] of type
 * g_dtype: with p_e = softmax over the group of q_e . k / sqrt(Dk),
 * dq_e = dw p_e k / sqrt(Dk), dk = sum_e dw p_e q_e / sqrt(Dk); fp32 math,
 * dq / dk written in dtype.  Dk <= 256. */
int tc_qk_weights_bwd(int32_t B, int32_t N, int32_t Hq, int32_t Hkv, int32_t Dk, int32_t dtype,
                      const void* q, const void* k, int32_t g_dtype, const void* dw, void* dq, void* dk,
                      void* stream);

/* Causal depthwise short conv with fp32 taps and fp32 residual, one cast:
 * y[b, t, c] = x[b, t, c] + sum_j w[c, j] x[b, t - K + 1 + j, c]
 * (short_conv, reference.py:167-211).  x, y [B, N, C]; w [C, K]. */
int tc_short_conv(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                  int32_t w_dtype, const void* w, void* y, void* stream);

/* tc_short_conv with segment resets for packed examples: seq_idx [B, N]
 * int32 (NULL = one sequence per batch row); the tap at row s reaches row t
 * only when seq_idx[b, s] == seq_idx[b, t].  No reference counterpart: the
 * reference's short_conv leaves these resets as a TODO (reference.py:186-189). */
int tc_short_conv_seg(int32_t B, int32_t N, int32_t C, int32_t dtype, const void* x, int32_t K,
                      int32_t w_dtype, const void* w, const int32_t* seq_idx, void* y, void* stream);

/* ------------------------------------------------------------------------ */
/* positional helpers                                                        */
/* ------------------------------------------------------------------------ */

/* Rotate-half RoPE of the rows of x [B, S, H, D] into y (same dtype), in
 * fp32, rounded once to the element type (apply_rope, reference.py:267-302).
 * pos_kind 0: position of row s is s (query rows);
 * pos_kind 1: rows are a packed level-major buffer of schedule `sched`,
 *             position of (level l, node j) is (j + 1) 2^l - 1
 *             (summary_token_position, reference.py:219-237).
 * pos_kind 2: positions[B * S * H] (int32, device) give every row's position.
 * inverse != 0 rotates by -theta. */
int tc_rope_apply(int32_t B, int64_t S, int32_t H, int32_t D, int32_t dtype, const void* x,
                  void* y, const float* cos_t, const float* sin_t, int32_t n_pos,
                  int32_t pos_kind, const tc_schedule* sched, const int32_t* positions,
                  int32_t inverse, void* stream);

/* ------------------------------------------------------------------------ */
/* Phase 2 attention                                                         */
/* ------------------------------------------------------------------------ */

typedef struct tc_attn_args {
  int32_t B, N, Hq, Hkv, Dk, Dv;
  int32_t dtype;            /* q, packed k/v, out, dq, dk, dv element type    */
  int32_t has_softcap;
  float softcap;
  int32_t position_mode;    /* TC_POS_*                                      */
  const void* q;            /* [B, N, Hq, Dk]   (already rotated for rope)   */
  const void* k;            /* [B, total, Hkv, Dk] (already rotated)         */
  const void* v;            /* [B, total, Hkv, Dv]                           */
  const void* rel_states;   /* [B, N, Hq, d_rel] (relative)                  */
  const void* rel_proj;     /* [d_rel, rel_bins]                             */
  int32_t rel_dtype;        /* element type of rel_states and rel_proj       */
  int32_t d_rel, rel_bins;
  const float* rope_cos;    /* [n_pos, Dk/2] backward only: the kernels      */
  const float* rope_sin;    /* rotate dq/dk back by R(-p) in fp32 (rope)     */
  int32_t rope_npos;
  void* out;                /* [B, N, Hq, Dv]                                */
  float* lse;               /* [B, N, Hq]                                    */
  /* backward only */
  const void* o;            /* forward out [B, N, Hq, Dv]                    */
  const void* dout;         /* [B, N, Hq, Dv]                                */
  const float* dlse;        /* [B, N, Hq] or NULL                            */
  float* delta;             /* scratch [B, N, Hq] f32                        */
  void* dq;                 /* [B, N, Hq, Dk]                                */
  void* dk;                 /* [B, total, Hkv, Dk]                           */
  void* dv;                 /* [B, total, Hkv, Dv]                           */
  float* drel;              /* [B, N, Hq, rel_bins] f32 or NULL.  With
                               rel_logits the kernels write every element;
                               without, only visible bins are written and
                               the caller zero-fills                         */
  int32_t* dev_status;      /* device status word (TC_DEV_*), or NULL        */
  int32_t impl;             /* 0 auto, 1 SIMT (any shape, any dtype),
                               2 tensor core (bf16/f16, Dk = Dv = 128)       */
  /* Relative mode on the tensor-core path: the bias logits
   * rel_logits[row, pad + d] = relative_states[row] . relative_proj[:, d]
   * (row = (b * N + q) * Hq + hq, d = bin distance) in the element type,
   * with `pad` (>= 136) zero columns on each side of the bins a query can
   * reach; row stride rel_logits_stride elements (a multiple of 8).  NULL: the
   * relative mode runs on the SIMT kernels, which form the bias from
   * rel_states / rel_proj directly. */
  const void* rel_logits;
  int64_t rel_logits_stride;
  int32_t rel_logits_pad;
  int32_t tile_n;           /* forward KV tile width: 0 auto, 64 or 128      */
} tc_attn_args;

/* Phase-2 forward: (out, lse) over the packed level-major K/V
 * (multilevel_attention_forward, reference.py:771-1071). */
int tc_attn_fwd(const tc_attn_args* a, const tc_schedule* s, void* stream);

/* Phase-2 backward: dq, dk_packed, dv_packed and (relative) drel_logits, with
 * the sink dlse seed folded into Delta (multilevel_attention_backward,
 * reference.py:1249-1672).  For rope, q and k are passed already rotated
 * and dq/dk are rotated back by R(-p) in fp32 before the single cast. */
int tc_attn_bwd(const tc_attn_args* a, const tc_schedule* s, void* stream);

/* Status of tc_attn_bwd_noalloc when B * N * Hq exceeds its fixed scratch. */
#define TC_ERR_SCRATCH_LIMIT 5

/* tc_attn_bwd for callers that cannot allocate device memory (a framework or
 * serving engine whose own pool has reserved the GPU, a host runtime that only
 * hands out buffers it owns).  No counterpart in the reference: it exists only
 * for this C ABI.  Same arguments as tc_attn_bwd except that a->delta is
 * ignored: the Delta scratch lives in a fixed 2^22-float (16 MiB) device array
 * inside the library, held by every GPU that loads it, so B * N * Hq must be
 * <= 4194304 (else TC_ERR_SCRATCH_LIMIT).  Nothing is allocated.  Every call
 * looks up the array's address on the current device; the first call on a
 * device also loads the library there (make it before any stream capture).
 * Calls that overlap on the GPU share the array and race. */
int tc_attn_bwd_noalloc(const tc_attn_args* a, const tc_schedule* s, void* stream);

/* Failure-detection self-test (no reference counterpart): one kernel waits on
 * a pipeline barrier that nothing completes, through the bounded wait every
 * tensor-core kernel uses; the wait gives up (well under a second), ORs
 * TC_DEV_WAIT_TIMEOUT into *dev_status and the kernel returns normally. */
int tc_selftest_wait_timeout(int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* post-ops                                                                  */
/* ------------------------------------------------------------------------ */

/* out_sink = out * (sigmoid(lse - sinks[h]) rounded to out's type)
 * (apply_attention_sink, reference.py:1082-1122).  rows = B*N. */
int tc_sink_fwd(int64_t rows, int32_t Hq, int32_t Dv, int32_t dtype, const void* out,
                const float* lse, int32_t sink_dtype, const void* sinks, void* y,
                void* stream);

/* (dout_pre, dlse, dsinks) (attention_sink_backward, reference.py:1125-1184).
 * dsinks_f32 is [Hq] f32 and is overwritten. */
int tc_sink_bwd(int64_t rows, int32_t Hq, int32_t Dv, int32_t dtype, const void* out,
                const float* lse, int32_t sink_dtype, const void* sinks, const void* dout,
                void* dout_pre, float* dlse, float* dsinks_f32, void* stream);

/* y = SiLU(g) * out, g = x @ W_g^T precomputed (apply_output_gate,
 * reference.py:1187-1219).  n = number of elements. */
int tc_gate_apply(int64_t n, int32_t dtype, const void* out, int32_t g_dtype, const void* g,
                  int32_t y_dtype, void* y, void* stream);

/* ------------------------------------------------------------------------ */
/* incremental decode                                                        */
/* ------------------------------------------------------------------------ */

/* decode step modes */
#define TC_DECODE_FULL 0     /* advance the state, then attend (decode_step)  */
#define TC_DECODE_ADVANCE 1  /* advance only (advance_decode_state)           */
#define TC_DECODE_ROTATE 3   /* rebuild ring_k_rot: every node visible to query t,
                                rotated at its summary position (rope)      */
#define TC_DECODE_ATTEND 2   /* attend only, state untouched
                                (multilevel_attention_decode)                 */

typedef struct tc_decode_args {
  int32_t mode;              /* TC_DECODE_*                                  */
  int32_t B, Hq, Hkv, Dk, Dv;
  int32_t dtype;             /* ring / token element type                   */
  int32_t w_dtype;           /* ring w element type                         */
  int32_t t;                 /* token consumed (FULL/ADVANCE) or attended (ATTEND) */
  int32_t num_levels, cache_size;
  int32_t act[TC_MAX_LEVELS];
  int32_t caps[TC_MAX_LEVELS];
  int32_t ring_off[TC_MAX_LEVELS + 1];
  void* ring_k;              /* [B, sum(caps), Hkv, Dk]   (in place)        */
  void* ring_v;              /* [B, sum(caps), Hkv, Dv]                     */
  void* ring_w;              /* [B, sum(caps), Hkv]                         */
  void* conv_k;              /* [B, K-1, Hkv*Dk] or NULL  (in place)        */
  void* conv_v;              /* [B, K-1, Hkv*Dv] or NULL                    */
  const void* k_conv_w;      /* [Hkv*Dk, K] or NULL                         */
  const void* v_conv_w;      /* [Hkv*Dv, K] or NULL                         */
  int32_t conv_dtype, conv_k_width;
  const void* q_t;           /* [B, Hq, Dk]                                 */
  const void* k_t;           /* [B, Hkv, Dk] raw (pre-conv)                 */
  const void* v_t;           /* [B, Hkv, Dv]                                */
  const void* w_t;           /* [B, Hkv] precomputed linear weights or NULL */
  int32_t has_softcap;
  float softcap;
  int32_t position_mode;
  const float* rope_cos;     /* [n_pos, Dk/2] */
  const float* rope_sin;
  const void* rel_states;    /* [B, Hq, d_rel] */
  const void* rel_proj;      /* [d_rel, rel_bins] */
  int32_t rel_dtype, d_rel, rel_bins;
  const void* sinks;         /* [Hq] or NULL */
  int32_t sink_dtype;
  const void* gate_pre;      /* [B, Hq*Dv] = x_t @ W_g^T, or NULL */
  int32_t gate_dtype;
  void* out;                 /* [B, Hq, Dv] post-sink/gate, element type = dtype */
  float* lse;                /* [B, Hq] pre-sink                           */
  void* k_new;               /* [B, Hkv, Dk] post-conv key as stored, or NULL */
  void* v_new;               /* [B, Hkv, Dv] */
  /* Optional fp32 scratch for splitting each (batch, KV head)'s visible
   * entries over several CTAs (Dk = Dv = 128, 16-bit rings): at least
   * B * Hkv * 8 * (Hq / Hkv) * 130 floats.  NULL (or smaller) runs the step
   * unsplit in one launch. */
  float* workspace;
  int64_t workspace_floats;
  /* rope: [B, sum(caps), Hkv, Dk] copies of the ring keys rotated at their
   * summary positions, or NULL.  Given, FULL / ADVANCE also write the rotated
   * copies of the rows they create and the attention reads them instead of
   * rotating every visible key; ROTATE rebuilds it from ring_k. */
  void* ring_k_rot;
} tc_decode_args;

/* One fused decode step for token t: short_conv_step, merge weight, the
 * single ruler-tick merge into the per-level ring, the level-0 write, the
 * multilevel attention read of query t, sink and gate
 * (decode_step = advance_decode_state + multilevel_attention_decode +
 *  apply_attention_sink + apply_output_gate, reference.py:1948-2317). */
int tc_decode_step(const tc_decode_args* a, void* stream);

typedef struct tc_decode_init_args {
  int32_t B, Hkv, Dk, Dv;
  int32_t dtype;                          /* level / ring k and v element type  */
  int32_t w_dtype;                        /* level / ring w element type        */
  int32_t num_levels;
  int32_t caps[TC_MAX_LEVELS];
  int32_t ring_off[TC_MAX_LEVELS + 1];
  int32_t lo[TC_MAX_LEVELS];              /* live range [lo, hi) of query N-1   */
  int32_t hi[TC_MAX_LEVELS];              /* per level (hi - lo <= caps[l])     */
  const void* k_lv[TC_MAX_LEVELS];        /* level l keys [B, >= hi, Hkv, Dk]   */
  const void* v_lv[TC_MAX_LEVELS];        /* level l values [B, >= hi, Hkv, Dv] */
  const void* w_lv[TC_MAX_LEVELS];        /* level l weights [B, >= hi, Hkv]    */
  /* batch and token strides of each level tensor, in elements; the
   * (Hkv, D) block of a token (the Hkv weights for w) is dense. */
  int64_t k_stride_b[TC_MAX_LEVELS], k_stride_n[TC_MAX_LEVELS];
  int64_t v_stride_b[TC_MAX_LEVELS], v_stride_n[TC_MAX_LEVELS];
  int64_t w_stride_b[TC_MAX_LEVELS], w_stride_n[TC_MAX_LEVELS];
  void* ring_k;                           /* [B, sum(caps), Hkv, Dk] written whole */
  void* ring_v;                           /* [B, sum(caps), Hkv, Dv]            */
  void* ring_w;                           /* [B, sum(caps), Hkv]                */
} tc_decode_init_args;

/* Prefill hand-off on the device: every ring slot of every level receives
 * the node of that level live at query N-1 that maps to it
 * (slot = ring_off[l] + j % caps[l]), or zeros when none does, in one launch
 * (the ring placement of init_decode_state, reference.py:1848-1930; the conv
 * history rows stay with the caller). */
int tc_decode_init(const tc_decode_init_args* a, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TELESCOPE_CACHE_H */
