/*
 * pbk.h -- C ABI of the B200 (sm_100a) kernels for PseudoBrain's hot path.
 *
 * Everything here is plain C: device pointers, sizes, element strides, a dtype
 * code per tensor and a cudaStream_t passed as void*. The library allocates no
 * device memory: the caller owns every tensor, outputs and workspaces included
 * (workspace sizes come from the *_workspace_size queries). Calls are
 * stream-ordered, never synchronise the host, keep no pointer past the call and
 * are re-entrant on different streams.
 *
 * Every entry point returns a pbk status (0 = PBK_OK, negative = error);
 * pbk_status_string() names it. Arguments are validated on the host before any
 * launch: a call that returns an error launched nothing.
 *
 * Layouts follow the reference (defnotean/pseudobrain):
 *   q, k  [B, T, Hk, dk]    v, o  [B, T, Hv, dv]    g, beta  [B, T, Hv]
 *   state [slots, Hv, dk, dv] fp32 (PBK_STATE_KV, the PyTorch core's [B,H,K,V])
 *         or [slots, Hv, dv, dk] (PBK_STATE_VK, vLLM's state pool layout)
 * Value head j reads key head j / (Hv / Hk), the repeat_interleave GQA map of
 * pseudobrain/gated_deltanet.py:422-424; the kernels never materialise it.
 */
#ifndef PBK_H_
#define PBK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PBK_ABI_VERSION 1

#if defined(__GNUC__)
#define PBK_API __attribute__((visibility("default")))
#else
#define PBK_API
#endif

/* status codes */
#define PBK_OK 0
#define PBK_ERR_INVALID (-1)   /* null pointer or out-of-range argument */
#define PBK_ERR_SHAPE (-2)     /* shape this build does not support */
#define PBK_ERR_DTYPE (-3)     /* unsupported dtype code */
#define PBK_ERR_ALIGN (-4)     /* pointer or stride not aligned for vector access */
#define PBK_ERR_DEVICE (-5)    /* current device is not sm_100 */
#define PBK_ERR_LAUNCH (-6)    /* the CUDA launch failed */
#define PBK_ERR_TIMEOUT (-7)   /* a bounded device-side wait gave up */
#define PBK_ERR_WORKSPACE (-8) /* workspace missing or too small */
#define PBK_ERR_TOO_LARGE (-9) /* problem exceeds the fixed scratch of pbk_quest_select_noalloc */

/* dtype codes */
#define PBK_F32 0
#define PBK_BF16 1

/* state layouts */
#define PBK_STATE_KV 0 /* [.., dk, dv]: pseudobrain/gated_deltanet.py:72-75 */
#define PBK_STATE_VK 1 /* [.., dv, dk]: vLLM mamba state pool */

/* A strided view of a [B, T, H, D] (or [B, T, H]) tensor whose last dimension is
 * contiguous. Strides are in elements. */
typedef struct pbk_view {
  const void* data;
  int64_t stride_b, stride_t, stride_h;
  int32_t dtype;
  int32_t pad_;
} pbk_view;

/* One gated delta rule problem (prefill or decode).
 * h0 is the initial state [slots, Hv, ...] (NULL = zeros, prefill only); state
 * receives the final state. For decode, state is updated in place (h0 must be
 * NULL or equal to state). state_indices[b] picks the slot of sequence b
 * (NULL = slot b); a negative index skips that sequence (vLLM's padding slot). */
typedef struct pbk_gdn_desc {
  int32_t batch, seqlen, hk, hv, dk, dv;
  pbk_view q, k, v, g, beta;
  pbk_view o;                 /* output; data is written */
  const float* h0;
  float* state;
  int64_t state_slot_stride;  /* elements between slots; Hv*dk*dv when dense */
  int32_t state_layout;       /* PBK_STATE_KV or PBK_STATE_VK */
  int32_t pad_;
  const int32_t* state_indices;
  float scale;                /* the query scale, dk**-0.5 in the reference */
  int32_t pad2_;
} pbk_gdn_desc;

/* Layer pieces around the recurrence (vLLM's adapter path: causal_conv1d, fused gating,
 * q/k L2 norm in the producer, gated RMSNorm on the output). Channel views use stride_h as
 * the channel stride; [B, T, H, 128] views have a contiguous last dim. */
typedef struct pbk_conv_desc {
  int32_t batch, seqlen, hk, hv;
  int32_t width;    /* convolution taps, 1..8 (4 in Qwen3-Next); ignored when weight is NULL */
  int32_t l2mode;   /* q/k normalisation: 0 none, 1 'max' (x / max(|x|, eps)), 2 'hf' (x rsqrt(|x|^2 + eps)) */
  float eps;        /* the normalisation eps (1e-6 in the reference) */
  int32_t pad_;
  pbk_view x;        /* [B, T, (2 hk + hv) 128] inputs q | k | v channels */
  pbk_view tail;     /* [B, width - 1, channels] the inputs before x; data NULL: zeros */
  pbk_view new_tail; /* [B, width - 1, channels] written with the last width - 1 inputs; NULL: skipped */
  const float* weight; /* [channels, width] fp32 contiguous (weight[:, width-1] multiplies x_t); NULL: SiLU only */
  pbk_view q, k, v;  /* [B, T, hk | hk | hv, 128] outputs */
} pbk_conv_desc;

typedef struct pbk_gating_desc {
  int32_t batch, seqlen, hv, pad_;
  pbk_view decay;      /* [B, T, 2 hv]: a | b */
  const float* a_log;  /* [hv] */
  const float* dt_bias; /* [hv] */
  pbk_view g, beta;    /* [B, T, hv] outputs */
} pbk_gating_desc;

typedef struct pbk_out_norm_desc {
  int32_t batch, seqlen, hv, weight_dtype;
  float eps;          /* 1e-5 in the reference */
  int32_t pad_;
  pbk_view o, gate, out; /* [B, T, hv, 128] each */
  const void* weight;    /* [128] */
} pbk_out_norm_desc;

PBK_API int pbk_abi_version(void);
PBK_API const char* pbk_status_string(int status);
/* The CUDA error message behind the calling thread's last PBK_ERR_LAUNCH ("no error"
 * when there was none). */
PBK_API const char* pbk_last_launch_error(void);
/* PBK_OK when `device` is an sm_100 (B200-class) GPU. */
PBK_API int pbk_device_check(int device);
/* Reads (and with clear != 0 resets) the current device's error word, which the
 * tensor-core kernels set to a nonzero code when a bounded device-side wait gives up
 * (the PBK_ERR_TIMEOUT condition; the code names the wait). Synchronises with the
 * device: a diagnostic, not for hot paths. The word's device address is looked up once
 * per device and kept: a device reset (cudaDeviceReset) while libpbk is loaded is not
 * supported. */
PBK_API int pbk_device_error(int* code, int clear);

/* Gated delta rule over few tokens per sequence with the state held in registers:
 * the recurrence of delta_rule_sequential, pseudobrain/gated_deltanet.py:93-107,
 * and the decode step vLLM runs as fused_recurrent_gated_delta_rule
 * (vllm/model_executor/layers/fla/ops/fused_recurrent.py). One read and one write
 * of each fp32 state for any seqlen. Requires dk == dv == 128; q/k/v bf16 or fp32;
 * g/beta bf16 or fp32; o bf16 or fp32. */
PBK_API int pbk_gdn_decode(const pbk_gdn_desc* desc, void* stream);

/* What vLLM's decode ops add around pbk_gdn_decode's recurrence, for pbk_gdn_decode_ext:
 * vllm/model_executor/layers/fla/ops/fused_recurrent.py:256-336
 * (fused_recurrent_gated_delta_rule_packed_decode), :20-170 (fused_recurrent_gated_delta_rule)
 * and fused_sigmoid_gating.py:24-180 (fused_sigmoid_gating_delta_rule_update). */
typedef struct pbk_decode_ext {
  int32_t gating;            /* 1: g = -exp(A_log) softplus(a + dt_bias) and beta = sigmoid(b) per token and
                                value head (desc->g and desc->beta are not read); 0: desc->g, desc->beta */
  int32_t beta_round;        /* 1: sigmoid(b) is rounded to b's dtype before use (the packed decode) */
  float softplus_beta;       /* softplus(x) = log(1 + exp(sb x)) / sb while sb x <= threshold, else x */
  float softplus_threshold;  /* (vLLM: sb = 1, threshold = 20) */
  pbk_view a, b;             /* [B, T, Hv] raw gate inputs (gating = 1) */
  const void* a_log;         /* [Hv] */
  const void* dt_bias;       /* [Hv] */
  int32_t a_log_dtype, dt_bias_dtype;
  int32_t l2norm;            /* q and k per head before the query scale: 0 none, 1 x / sqrt(sum x^2 + eps),
                                2 x rsqrt(sum x^2 + eps) (fp32) */
  float eps;                 /* 1e-6 in vLLM */
  int32_t null_slot;         /* 1: a state index <= 0 is vLLM's null block (the sequence is skipped);
                                0: only a negative index skips (pbk_gdn_decode's rule) */
  int32_t zero_skipped;      /* 1: a skipped sequence's outputs are written as zeros (the packed decode) */
  const int32_t* cu_seqlens; /* [batch + 1] row offsets of each sequence in [1, rows, H, D] tensors, or NULL:
                                dense [batch, seqlen, ...] */
  int64_t index_stride;      /* > 0: state_indices is [batch, index_stride] (speculative decoding): the initial
                                state is column num_accepted[n] - 1 (0 without num_accepted) of row n, and the
                                state after token t is written to column t (null columns skipped); 0: one
                                slot per sequence, read and written */
  const int32_t* num_accepted; /* [batch] accepted tokens per sequence, or NULL */
} pbk_decode_ext;

/* pbk_gdn_decode with vLLM's decode-op semantics (pbk_decode_ext): the same kernel, reading
 * and writing each state once per token span (and once more per token under speculative
 * decoding). desc->seqlen is the dense token count (ignored with cu_seqlens); the state pool
 * is updated in place (desc->h0 NULL or equal to desc->state). */
PBK_API int pbk_gdn_decode_ext(const pbk_gdn_desc* desc, const pbk_decode_ext* ext, void* stream);

/* Chunked gated delta rule (prefill): the chunkwise WY algorithm of
 * delta_rule_chunked, pseudobrain/gated_deltanet.py:110-165 (chunk 64), reading h0
 * (NULL = zeros) and writing the final state into `state` (h0 == state is allowed:
 * in place) and every token's output into o. Sequence ends that are not a multiple
 * of 64 are padded with identity steps as the reference does. Requires
 * dk == dv == 128. With bf16 q/k/v, o.data may be NULL: only the final state is
 * computed (the segment runs of pbk_gdn_segment_scan). */
PBK_API int pbk_gdn_prefill(const pbk_gdn_desc* desc, void* stream);

/* pbk_gdn_prefill with the chunk solve split out: on the tensor-core path (bf16 q/k/v) a
 * first kernel solves every chunk of every (sequence, value head) at once -- the
 * state-independent T = (I + A)^-1 of gated_deltanet.py:131-140, its products with
 * diag(beta) and diag(beta gamma) and the chunk's decay scalars, 17,936 bytes per chunk --
 * into `workspace`, and the recurrence kernel copies them in instead of solving in line. Same results as pbk_gdn_prefill (the
 * same arithmetic). workspace: at least pbk_gdn_prefill_workspace(desc) bytes, 16-byte
 * aligned, private to the call until it completes on `stream`. Off the tensor-core path
 * (fp32 inputs) the workspace is unused and may be NULL. */
PBK_API size_t pbk_gdn_prefill_workspace(const pbk_gdn_desc* desc);
PBK_API int pbk_gdn_prefill_ws(const pbk_gdn_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* pbk_gdn_prefill_ws that also writes the chunk quantities the reference's fla custom op
 * returns beside (o, final state) -- pseudobrain::gated_delta_chunk, gated_deltanet.py:200-216,
 * whose backward consumes them: gc [B, T, Hv] fp32, the cumulative sum of g within each
 * 64-token chunk (fla's chunk-local cumsum), and a [B, T, Hv, 64] (bf16 or fp32, last dim
 * contiguous, 16-byte aligned rows), row t of its chunk's T = (I + A)^-1 with
 * A_ti = beta_t (k_t . k_i) exp(gc_t - gc_i) for i < t (fla's solve_tril output, the
 * reference's `solve`, gated_deltanet.py:145-150); entries past the chunk's last valid step
 * are zero. o.data must be set. Same workspace as pbk_gdn_prefill_ws. */
PBK_API int pbk_gdn_prefill_aux(const pbk_gdn_desc* desc, const pbk_view* gc, const pbk_view* a, void* workspace,
                                size_t workspace_bytes, void* stream);

/* The two halves of pbk_gdn_prefill_ws, tensor-core path only (PBK_ERR_INVALID otherwise):
 * pbk_gdn_chunk_solve writes the workspace from k, g and beta; pbk_gdn_prefill_solved runs
 * the recurrence from a workspace holding the solve of the same chunks. Slot (b, chunk, h)
 * sits at ((b * nchunks + chunk) * hv + h) * 17,936 bytes, so the solve of one long sequence
 * also serves runs over segments of it (whole chunks, viewed as a batch of segments; a
 * later segment starts at its first chunk's slot): the sequence-split prefill solves once
 * and runs the recurrence three times. */
/* Packed varlen prefill (vLLM's chunked-prefill batch; tensor-core path, bf16 q/k/v): desc
 * describes [1, T, H, 128] tensors (batch 1, seqlen = T total rows). Sequence s is rows
 * cu_seqlens[s] .. cu_seqlens[s+1] of them (cu_seqlens: num_seqs + 1 ascending int32 on the
 * device, 16-byte aligned), starts from h0 slot state_indices[s] (or s when state_indices is
 * NULL; a negative index skips the sequence) and ends in that slot of `state`; its outputs go
 * to its rows of o. Each sequence is the reference's delta_rule_chunked on its own
 * (gated_deltanet.py:110-165, chunks counted from the sequence's first row). Workspace:
 * pbk_gdn_prefill_varlen_workspace(desc, num_seqs) bytes, 16-byte aligned, private to the
 * call until it completes on `stream`. */
PBK_API size_t pbk_gdn_prefill_varlen_workspace(const pbk_gdn_desc* desc, int32_t num_seqs);
PBK_API int pbk_gdn_prefill_varlen(const pbk_gdn_desc* desc, const int32_t* cu_seqlens, int32_t num_seqs,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* Causal depthwise convolution + SiLU over the q | k | v channels with a carried tail
 * (short_convolution, gated_deltanet.py:314-338), q and k L2-normalised per 128-channel head
 * (l2_normalize, :59-70); fp32 arithmetic, outputs in their views' dtypes. new_tail must not
 * overlap tail. */
PBK_API int pbk_gdn_conv_norm(const pbk_conv_desc* desc, void* stream);
/* Row-wise L2 normalisation of x [B, T, H, 128] into out (same shape; bf16 or fp32 each,
 * last dim contiguous): mode 1 x / max(|x|, eps) (F.normalize, gated_deltanet.py:59-70),
 * mode 2 x rsqrt(|x|^2 + eps) (the in-kernel q/k norm of vLLM's GDN ops), fp32 arithmetic. */
PBK_API int pbk_l2norm(pbk_view x, pbk_view out, int32_t batch, int32_t seqlen, int32_t heads, int32_t mode,
                       float eps, void* stream);
/* g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (gated_deltanet.py:427-429). */
PBK_API int pbk_gdn_gating(const pbk_gating_desc* desc, void* stream);

/* The decode step of GatedDeltaNetLayer.forward (pseudobrain/gated_deltanet.py:411-440, the
 * few-token case select_kernel sends to delta_rule_sequential, :291-294) from the input
 * projection's output to the gated, normed per-step output, for pbk_gdn_decode_layer. */
typedef struct pbk_gdn_layer_desc {
  int32_t batch, seqlen, hk, hv; /* dense [B, T, ..]; dk == dv == 128 */
  int32_t width;       /* conv taps 1..8 (conv_weight[:, width-1] multiplies the current input) */
  int32_t l2mode;      /* q/k normalisation: 0 none, 1 'max' (x / max(|x|, eps)), 2 'hf' (x rsqrt(|x|^2 + eps)) */
  float l2_eps;        /* 1e-6 in the reference */
  float norm_eps;      /* the output RMSNorm eps, 1e-5 in the reference */
  float scale;         /* the query scale, dk ** -0.5 */
  int32_t state_layout; /* PBK_STATE_KV or PBK_STATE_VK */
  pbk_view qkv;        /* [B, T, (2 hk + hv) 128] the projection's q | k | v channels before the
                          convolution (stride_h = channel stride) */
  pbk_view tail;       /* [B, width - 1, channels] the conv inputs before qkv; data NULL: zeros */
  pbk_view new_tail;   /* [B, width - 1, channels] receives the last width - 1 inputs; may be `tail`
                          itself (in place: the value heads of a key head then run as one thread-block
                          cluster, so hv / hk must be at most 8); NULL: not written */
  const float* conv_weight; /* [channels, width] fp32 contiguous; NULL: SiLU only, no tail */
  pbk_view decay;      /* [B, T, 2 hv]: a | b, the raw decay and beta gate inputs */
  const float* a_log;  /* [hv] fp32 */
  const float* dt_bias; /* [hv] fp32 */
  pbk_view gate;       /* [B, T, hv 128] the output gate z (stride_h = channel stride) */
  const void* o_norm;  /* [128] the output RMSNorm weight */
  int32_t o_norm_dtype;
  int32_t pad_;
  pbk_view out;        /* [B, T, hv, 128] the gated, normed output (bf16 or fp32) */
  float* state;        /* [slots, hv, 128, 128] fp32, updated in place */
  int64_t state_slot_stride; /* elements between slots */
  const int32_t* state_indices; /* slot of sequence b (NULL: b); a negative index skips the sequence */
} pbk_gdn_layer_desc;

/* One kernel for the layer's decode step: short_convolution with the carried tail and SiLU
 * (:314-338), the q/k L2 norm (:59-70), the gating (:427-429), the recurrence
 * (delta_rule_sequential, :93-107) on the register-resident state, and the output
 * o rsqrt(mean(o^2) + eps) o_norm SiLU(z) (:439-440) -- fp32 throughout, so q, k, v, g and
 * beta never reach memory (pbk_gdn_conv_norm + pbk_gdn_gating + pbk_gdn_decode +
 * pbk_gdn_out_norm in one launch). Meant for the few tokens per sequence of a decode step;
 * any seqlen is accepted. */
PBK_API int pbk_gdn_decode_layer(const pbk_gdn_layer_desc* desc, void* stream);

/* GatedDeltaNetLayer.forward over a prefill (gated_deltanet.py:411-440, the chunked
 * recurrence of :110-165) from the input projection's output to the gated, normed output, in
 * three launches: (1) the chunk solve with the producer stages fused in -- each CTA convolves
 * its chunk's q | k | v channels (short_convolution with the carried tail and SiLU), L2-
 * normalises q and k and computes g and beta from the raw gate inputs, so the standalone conv
 * and gating passes never run -- writing q, k, v (bf16) and its chunk records into the
 * workspace; (2) the tensor-core recurrence from them (desc->state is read as h0 and receives
 * the final state, slot state_indices[b] or b); (3) the output RMSNorm and SiLU gate. Needs
 * bf16 qkv with contiguous channels (stride_h 1, row strides multiples of 8 elements, 16-byte
 * aligned: its rows arrive by TMA) and gate channels contiguous; new_tail must not be tail. Workspace:
 * pbk_gdn_prefill_layer_workspace(desc) bytes, 16-byte aligned, private to the call until it
 * completes on `stream`. */
PBK_API size_t pbk_gdn_prefill_layer_workspace(const pbk_gdn_layer_desc* desc);
PBK_API int pbk_gdn_prefill_layer(const pbk_gdn_layer_desc* desc, void* workspace, size_t workspace_bytes,
                                  void* stream);
/* out = o rsqrt(mean(o^2) + eps) weight SiLU(gate) per 128-wide head row
 * (gated_deltanet.py:439-440). */
PBK_API int pbk_gdn_out_norm(const pbk_out_norm_desc* desc, void* stream);

PBK_API int pbk_gdn_chunk_solve(const pbk_gdn_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
PBK_API int pbk_gdn_prefill_solved(const pbk_gdn_desc* desc, const void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Segment scan for a prefill split along T into nseg segments of whole 64-token chunks
 * (parallelism inside one long sequence; the reference runs a sequence's chunks in
 * order, gated_deltanet.py:157-163). A segment's recurrence is affine in its initial
 * state, S_out = A S_in + b: b is its final state from zeros and m = A + b its final
 * state from the identity (two pbk_gdn_prefill runs of all segments at once, o = NULL).
 * With b, m [batch, nseg - 1, hv, 128, 128] and h0 [batch, hv, 128, 128] (NULL =
 * zeros), writes starts [batch, nseg, hv, 128, 128]:
 *   starts[0] = h0,  starts[p + 1] = (m[p] - b[p]) starts[p] + b[p]   (fp32, exact);
 * a third run from `starts` then gives every token's output and the final state.
 * [K,V] state layout, dense, 16-byte aligned. */
PBK_API int pbk_gdn_segment_scan(const float* b, const float* m, const float* h0, float* starts, int32_t batch,
                                 int32_t nseg, int32_t hv, void* stream);

/* ------------------------------------------------------------------------
 * Quest page-bounded exact memory (pseudobrain/exact_memory.py, flat mode).
 *
 * One archive of evicted keys/values [kv, n_arch, d] (bf16) with per-page key
 * bounds [kv, n_arch / page, d] (bf16, elementwise max and min of each complete
 * page), and nq independent query groups q [nq, t, h, d] (bf16): the t rows of a
 * group share one page selection per key head, as the t queries of one call of
 * the reference's retrieve() do (exact_memory.py:88-152). Query head j reads key
 * head j / (h / kv).
 * ------------------------------------------------------------------------ */
typedef struct pbk_quest_desc {
  int32_t nq, t, h, kv, d;  /* d must be 128 */
  int32_t page;             /* tokens per page */
  int32_t n_arch;           /* archived tokens; complete pages n_arch / page are scored, the rest is the tail */
  int32_t budget;           /* pages kept per (group, key head): k = min(budget, n_arch / page) */
  int32_t n_win;            /* window keys */
  int32_t window, sinks;    /* window key visible to a query at qpos: kpos <= qpos and
                               (qpos - kpos < window or kpos < sinks) (transplant.py:621-622) */
  float scale;              /* softmax scale, d**-0.5 for SDPA's default */
  const void* q;
  int64_t q_stride_n, q_stride_t, q_stride_h;
  const int32_t* qpos;      /* [nq, t] query positions */
  const void* kmax;
  const void* kmin;
  int64_t bnd_stride_kv, bnd_stride_p;
  const void* keys;
  const void* values;
  int64_t arc_stride_kv, arc_stride_n;
  const void* win_keys;
  const void* win_values;
  int64_t win_stride_kv, win_stride_n;
  const int32_t* kpos;      /* [n_win] positions of the window keys */
  int32_t* pages;           /* [nq, kv, k] selected pages, ascending (written by select, read by attend) */
  float* scores;            /* optional [nq, kv, n_arch / page] fp32 page scores (NULL: workspace) */
  void* out;                /* [nq, t, h, d] attention output */
  int64_t out_stride_n, out_stride_t, out_stride_h;
  int32_t out_dtype;
  int32_t pad_;
} pbk_quest_desc;

/* Per-token block scores and exact rescoring of the serving path's per-token selector
 * (pb27_vllm/memory.py:1009-1294). Query token t of q [T, H, D] (bf16, element strides) and
 * key head h score candidate j of n_pool: block b = cand[h * cand_stride_kv + j] (or j when
 * cand is NULL). out [KV, T, n_pool] fp32 at element strides out_stride_kv, out_stride_t. */
typedef struct pbk_token_desc {
  int32_t t, h, kv, d;          /* query tokens, query heads, key heads; d must be 128; h / kv <= 32 */
  int32_t n_pool;               /* candidates per key head */
  int32_t full;                 /* scores: blocks [0, full) carry bounds; others score -inf */
  int32_t hole_lo, hole_hi;     /* scores: blocks in [hole_lo, hole_hi) score -inf (none if hole_hi <= hole_lo) */
  int32_t rope_mask;            /* scores: nonzero zeroes the query dims below d / 4 (memory.py:1043-1045) */
  int32_t block;                /* rescoring: tokens per block */
  const void* q;
  int64_t q_stride_t, q_stride_h;
  const void* kmax;             /* scores: [KV, >= full, D] bf16 block bounds */
  const void* kmin;
  int64_t bnd_stride_kv, bnd_stride_p;
  const void* keys;             /* rescoring: [KV, rows, D] bf16, block b = rows b * block .. + block - 1 */
  int64_t key_stride_kv, key_stride_n;
  const int32_t* cand;
  int64_t cand_stride_kv;
  float* out;
  int64_t out_stride_kv, out_stride_t;
} pbk_token_desc;

/* out[h][t][j] = max over the query heads of key head h (token t) of
 * sum_d q_d * (q_d > 0 ? kmax : kmin)[b][d], summed over d = 0 .. 127 in order, or -inf for
 * a block outside [0, full) or inside the hole (memory.py:1079-1098). */
PBK_API int pbk_quest_token_scores(const pbk_token_desc* desc, void* stream);
/* out[h][t][j] = max over the query heads of key head h (token t) and the block's tokens of
 * q . k in fp32 (the exact rescoring, memory.py:1192-1202). */
PBK_API int pbk_quest_token_rerank(const pbk_token_desc* desc, void* stream);
/* ranks[r][i] = position of x[r][i] in row r sorted descending, ties in index order
 * (_ranks, memory.py:881-885), for `rows` rows of n <= 16384 fp32 values. */
PBK_API int pbk_quest_row_ranks(const float* x, int64_t x_stride, int32_t rows, int32_t n, int32_t* ranks,
                                int64_t ranks_stride, void* stream);

/* Bytes of caller-provided device workspace pbk_quest_select / pbk_quest_attend need
 * for `desc` (0 when none; 256-byte aligned pointers). */
PBK_API size_t pbk_quest_select_workspace(const pbk_quest_desc* desc);
PBK_API size_t pbk_quest_attend_workspace(const pbk_quest_desc* desc);

/* Page scores and top-k selection (exact_memory.py:94-98,124-125,135,144): for every
 * group and key head, score page p as the maximum over the group's t * h/kv query rows
 * of sum_d max(q_d kmax_pd, q_d kmin_pd) in fp32, keep the k highest (ties to the
 * lowest page index) and write them to desc->pages in ascending order.
 * The selection is bit-exact with respect to one fixed order: each row's fp32 sum runs
 * over d = 0 .. 127 in order (products of two bf16 values are exact in fp32). Up to 64
 * query rows per key head the scores come from the tensor cores, whose sums differ from
 * that order by at most 2^-14 ||q_r||_1 max|bound|; the top-k re-scores every page within
 * twice that of its threshold in the fixed order, so the pages equal the fixed order's
 * selection. desc->scores (when given) receives the tensor-core scores. */
PBK_API int pbk_quest_select(const pbk_quest_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
/* pbk_quest_select in parts (bit mask): 1 the page scores and segment maxima into the
 * workspace, 2 the top-k selection from them (3: both). A caller overlaps other work with
 * the top-k by launching the parts apart, in order, with the same workspace. */
PBK_API int pbk_quest_select_parts(const pbk_quest_desc* desc, int32_t parts, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* Largest number of page scores (nq * kv * (n_arch / page)) pbk_quest_select_noalloc
 * can hold: 4,194,304 fp32 = 16 MiB, enough for 8 query groups x 8 key heads over a
 * 1M-token archive in 16-token pages. Its array also holds the per-32-page and per-128-
 * page maxima (17.0 MiB in all). */
#define PBK_QUEST_NOALLOC_MAX_SCORES 4194304

/* pbk_quest_select for callers that cannot allocate device memory. This entry point has
 * no counterpart in the reference. Some hosts own all device memory themselves (a serving
 * engine that has reserved the free HBM for its KV cache, or a foreign-language caller
 * with no handle on the framework's allocator): for them a workspace allocation fails or
 * stalls the device. This variant takes no workspace: the page scores and their per-32-
 * page maxima and the per-tile bound magnitudes go to a fixed 17.0 MiB array that libpbk
 * places in device memory (every GPU that loads the library holds it until the process
 * exits); when desc->scores is given, the scores go there instead. It calls no allocator.
 * Problems with more than PBK_QUEST_NOALLOC_MAX_SCORES scores, or whose maxima alone
 * exceed the array, return PBK_ERR_TOO_LARGE and launch nothing; every problem of at most
 * PBK_QUEST_NOALLOC_MAX_SCORES scores over at least 128 pages per row fits. The first call
 * on a device looks up the array's device address (once per device, with that device
 * current) and keeps it for the life of the process; make that first call before any
 * stream capture, and do not reset the device (cudaDeviceReset) while libpbk is loaded:
 * the kept address would then be stale. All calls share the one array: calls that overlap
 * on the GPU (two streams at once) race on it, so serialise them. Nothing in the array
 * needs to start at zero: each call overwrites every value it reads. Results equal
 * pbk_quest_select's. */
PBK_API int pbk_quest_select_noalloc(const pbk_quest_desc* desc, void* stream);

/* Exact softmax attention of every query row over [selected pages ; partial tail ;
 * window keys] with the window mask (pseudobrain/transplant.py:619-628), as a
 * split-key pass plus a log-sum-exp combine. Gathers the pages itself. */
PBK_API int pbk_quest_attend(const pbk_quest_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* pbk_quest_attend with n_sink always-visible keys placed before the selected pages:
 * rows 0 .. n_sink-1 of sink_keys / sink_values (bf16, element strides sink_stride_kv per
 * key head and sink_stride_n per row). This is the key set of the serving path's
 * piece_attention (pb27_vllm/memory.py:1311-1490): the sink positions, the retrieved
 * blocks, the partial block before the window and the masked window. Workspace bytes from
 * pbk_quest_attend_sinks_workspace(desc, n_sink). */
PBK_API size_t pbk_quest_attend_sinks_workspace(const pbk_quest_desc* desc, int32_t n_sink);
PBK_API int pbk_quest_attend_sinks(const pbk_quest_desc* desc, const void* sink_keys, const void* sink_values,
                                   int32_t n_sink, int64_t sink_stride_kv, int64_t sink_stride_n, void* workspace,
                                   size_t workspace_bytes, void* stream);
/* pbk_quest_attend_sinks in parts (bit mask): 1 the partials of the retrieved keys (sinks,
 * pages, tail), 2 the partials of the window keys, 4 their combination into out (7: all).
 * The window part does not read desc.pages, so it may run while the selection's top-k is
 * still computing them; the combine runs after both, with the same workspace. */
PBK_API int pbk_quest_attend_parts(const pbk_quest_desc* desc, const void* sink_keys, const void* sink_values,
                                   int32_t n_sink, int64_t sink_stride_kv, int64_t sink_stride_n, int32_t parts,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* Exact rerank (pb27_vllm/memory.py:854-872): for c candidate pages per (group, key head),
 * cand [nq, kv, c] int32 ascending, the exact score max over the head's query rows
 * and the page's tokens of q.k (fp32 on bf16 keys); the best
 * k = min(desc->budget, c) candidates, ties to the lowest page, go to desc->pages
 * [nq, kv, k] ascending. Uses desc->q, keys (arc strides), page; workspace bytes from
 * pbk_quest_rerank_workspace(desc, c). */
PBK_API size_t pbk_quest_rerank_workspace(const pbk_quest_desc* desc, int32_t c);
PBK_API int pbk_quest_rerank(const pbk_quest_desc* desc, const int32_t* cand, int32_t c, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Copy `sel` pages per (group, key head) listed in desc->pages ([nq, kv, sel], any
 * order, repeats allowed) and then the partial tail into out_keys / out_values
 * [nq, kv, sel * page + tail, d] (bf16, contiguous): what retrieve() returns
 * (exact_memory.py:145-151). */
PBK_API int pbk_quest_gather(const pbk_quest_desc* desc, int32_t sel, void* out_keys, void* out_values, void* stream);

/* Page bounds (exact_memory.py:43-50): kmax/kmin [kv, p, d] for pages
 * first_page .. ceil(n / page) - 1 of keys [kv, n, d] (bf16); a trailing partial page
 * takes the bounds of the keys it holds. Recomputing from the first incomplete page is
 * archive_append's refresh (exact_memory.py:66-85). */
PBK_API int pbk_quest_bounds(const void* keys, int32_t kv, int32_t n, int32_t d, int32_t page,
                             int64_t key_stride_kv, int64_t key_stride_n, void* kmax, void* kmin,
                             int64_t bnd_stride_kv, int64_t bnd_stride_p, int32_t first_page, void* stream);

/* Super-block bounds (exact_memory.py:53-63 _superbounds; pb27_vllm/memory.py:280-306
 * _update_superbounds): for super-blocks s in [first_sb, min(end_sb, ceil(n_blk / sblk))),
 * smax[h][s] = elementwise max of kmax[h][b] and smin[h][s] = min of kmin[h][b] over the
 * blocks b in [s * sblk, min(n_blk, (s + 1) * sblk)). Page bounds [kv, >= n_blk, d] and
 * super-block bounds [kv, *, d] are bf16 with element strides. */
PBK_API int pbk_quest_superbounds(const void* kmax, const void* kmin, int32_t kv, int32_t n_blk, int32_t d,
                                  int32_t sblk, int64_t bnd_stride_kv, int64_t bnd_stride_p, void* smax, void* smin,
                                  int64_t sb_stride_kv, int64_t sb_stride_p, int32_t first_sb, int32_t end_sb,
                                  void* stream);

/* RoPE repositioning of archived keys fused with their gather (pb27_vllm/memory.py:574-677:
 * _reposition_rope_sinks, _reposition_rope_blocks). For key head h, output row r < n_blk *
 * block is row s = r % block of block j = r / block, read from archive row origin +
 * blocks[h][j] * block + s (blocks NULL: block j itself); rows n_blk * block .. + tail_n are
 * archive rows tail0 .. tail0 + tail_n, copied as they are. Block j's keys turn by the angle
 * delta_j * inv_freq[i] in the pairs (i, i + d/8), i < d/8 (the first d/4 dims; the rest are
 * copied), in fp32 with the products and the difference rounded apart, then to bf16:
 *   mode 0: delta 0 (a plain gather);
 *   mode 1 (contiguous runs, the attention's retrieved blocks, :644-664): blocks placed in
 *     [ref_pos - max(arc_span, n_blk block), ref_pos) one block apart plus a share of the
 *     slack proportional to the historical gaps before them (blocks ascending);
 *   mode 2 (proportional, the rerank's candidates, :640-643): delta_j =
 *     round(max(ref_pos - pos_j, 0) * scale), pos_j = origin + blocks[h][j] * block;
 *   mode 3: delta_j = const_delta for every block (the sink keys, :585-596).
 * Values are gathered the same way, never rotated. Archive rows outside [0, n_rows) read as
 * zeros. Outputs out_keys / out_values (NULL: keys only) are bf16 [kv, n_blk * block +
 * tail_n, d], contiguous; delta (fp32 [kv, n_blk], required for modes 1 and 2, written) holds
 * each block's shift. */
typedef struct pbk_rope_gather_desc {
  int32_t kv, d, block, n_blk;   /* d must be 128 */
  int32_t origin, n_rows;        /* archive position of block 0; archive rows */
  int32_t ref_pos, arc_span;
  int32_t mode, tail0, tail_n;
  float scale;                   /* mode 2 */
  float const_delta;             /* mode 3 */
  int32_t pad_;
  const int32_t* blocks;         /* [kv, n_blk] block indices, or NULL */
  const float* inv_freq;         /* [d / 8] rotary inverse frequencies */
  const void* keys;
  const void* values;            /* may be NULL (keys only) */
  int64_t stride_kv, stride_n;   /* archive element strides (keys and values alike) */
  void* out_keys;
  void* out_values;
  float* delta;
} pbk_rope_gather_desc;

PBK_API int pbk_quest_rope_gather(const pbk_rope_gather_desc* desc, void* stream);

/* The serving archive's KV write fused with its block summaries (pb27_vllm/memory.py:310-395
 * Archive.write, :399-430 _refresh_range). New rows [n, kv, d] (token-major, as the KV cache
 * hands them over) go to archive rows p0 .. p0 + n - 1 (pos NULL) or pos[i] (int32, any
 * order). For every block b in [blk_lo, blk_hi] (rows origin + b * block ..) over the rows
 * written so far, end = max(size, p0 + n) (contiguous) or size: kmax / kmin = elementwise
 * max / min of the keys, kmean / vmean (optional) = mean of the keys / values with a partial
 * block padded by its last row (as the reference pads it); new rows are read once, from the
 * input, and written as they are summarised. A contiguous write passes the blocks it touches
 * (the reference's fast path plus its refresh of the partial ends); a write with pos passes
 * none (blk_hi < blk_lo) and refreshes its blocks later with n = 0. All bf16. */
typedef struct pbk_archive_write_desc {
  int32_t kv, d, block, origin;  /* d must be 128 */
  int32_t cap, size;             /* archive rows; rows written before this call */
  int32_t p0, n;
  int32_t blk_lo, blk_hi;
  const int32_t* pos;            /* [n] rows, or NULL: contiguous from p0 */
  const void* k;
  const void* v;
  int64_t in_stride_n, in_stride_kv;
  void* keys;
  void* values;
  int64_t arc_stride_kv, arc_stride_n;
  void* kmax;
  void* kmin;
  void* kmean;                   /* may be NULL */
  void* vmean;                   /* may be NULL */
  int64_t bnd_stride_kv, bnd_stride_p;
} pbk_archive_write_desc;

PBK_API int pbk_quest_archive_write(const pbk_archive_write_desc* desc, void* stream);

/* Super-block means (memory.py:296-306): smean[h][s] = mean of bmean[h][b] over the blocks b
 * in [s * sblk, min(n_blk, (s + 1) * sblk)), for s in [first_sb, min(end_sb, ceil(n_blk /
 * sblk))); bf16, fp32 sums. Same arguments as pbk_quest_superbounds with one input and one
 * output. */
PBK_API int pbk_quest_supermeans(const void* bmean, int32_t kv, int32_t n_blk, int32_t d, int32_t sblk,
                                 int64_t bnd_stride_kv, int64_t bnd_stride_p, void* smean, int64_t sb_stride_kv,
                                 int64_t sb_stride_p, int32_t first_sb, int32_t end_sb, void* stream);

/* Options of pbk_quest_select_levels. */
typedef struct pbk_quest_levels {
  const void* smax;         /* bf16 super-block bounds [kv, >= ceil(full / sblk), d]; NULL: one level */
  const void* smin;
  int64_t sb_stride_kv, sb_stride_p;
  int32_t sblk;             /* pages per super-block (>= 2 with smax) */
  int32_t m_sb;             /* super-blocks kept, 1 .. ceil(full / sblk); the reference takes
                               min(max(16, ceil(2 k / sblk)), ceil(full / sblk)) */
  int32_t hole_lo, hole_hi; /* pages [hole_lo, hole_hi) score -inf (hole_hi <= hole_lo: no hole) */
  int32_t pad_;
} pbk_quest_levels;

/* Page selection with the reference's other scoring modes, full = n_arch / page pages:
 * - two levels (lv->smax given; exact_memory.py:107-122, pb27_vllm/memory.py:802-836): the
 *   m_sb super-blocks of highest bound score (the page score formula on smax/smin over
 *   super-blocks 0 .. ceil(full / sblk) - 1, ties to the lowest), then the bound scores of
 *   their pages s * sblk + j, those at or past `full` or inside the hole scoring -inf, and
 *   the best k = min(budget, full, m_sb * sblk) of those candidates;
 * - one level with a hole (lv->smax NULL; memory.py:848-853): pbk_quest_select's scores with
 *   the hole's pages at -inf, best k = min(budget, full).
 * Ties go to the lowest candidate (page) index; the k pages go to desc->pages [nq, kv, k] in
 * ascending order. A caller whose hole leaves fewer than budget valid pages passes the
 * smaller budget, as the reference does (memory.py:788). desc->scores is not used. Workspace
 * bytes from pbk_quest_select_levels_workspace(desc, lv). */
PBK_API size_t pbk_quest_select_levels_workspace(const pbk_quest_desc* desc, const pbk_quest_levels* lv);
PBK_API int pbk_quest_select_levels(const pbk_quest_desc* desc, const pbk_quest_levels* lv, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Causal sliding-window attention with sinks (the hybrid model's attention branch,
 * pseudobrain/transplant.py:417-436 causal_attention and its exact chunked form
 * :346-362). Query t of head j sees key s of key head j / (h / kv) when
 *   s <= t  and  (window <= 0  or  t - s < window  or  s < sinks),
 * with softmax(scale * q.k) over the visible keys (scale = d**-0.5 for SDPA's
 * default). window <= 0 is full causal attention.
 * q, o [B, T, h, d] and k, v [B, T, kv, d] as strided views (the reference's
 * [B, H, T, d] is the same tensor with other strides); q/k/v bf16, o bf16 or fp32.
 * Requires d == 128, h a multiple of kv, 16-byte aligned pointers and strides.
 * ------------------------------------------------------------------------ */
typedef struct pbk_swa_desc {
  int32_t batch, seqlen, h, kv, d;
  int32_t window;  /* keys per query including itself; <= 0: unbounded */
  int32_t sinks;   /* leading positions every query sees */
  float scale;
  pbk_view q, k, v;
  pbk_view o;      /* output; data is written */
} pbk_swa_desc;

PBK_API int pbk_swa_prefill(const pbk_swa_desc* desc, void* stream);

/* Copy-engine exchange between the GPUs of one node (the head-sharded hybrid layer's
 * all-gather: pseudobrain/transplant.py WindowedHybridLayer's branch outputs gathered to the
 * hidden layout). The copies run on the copy engines over NVLink and use no SMs, so they
 * overlap kernels that occupy every SM; NCCL's all-gather kernels need SMs and wait for them.
 * pbk_ipc_handle exports the allocation holding `ptr` (PBK_IPC_HANDLE_BYTES bytes into
 * `handle`, ptr's byte offset in it into *offset); another process on the node maps it with
 * pbk_ipc_open (peer access enabled on first use) and unmaps it with pbk_ipc_close;
 * pbk_copy_async copies `bytes` between any two device addresses (mapped peer memory
 * included), stream-ordered. */
#define PBK_IPC_HANDLE_BYTES 64
PBK_API int pbk_ipc_handle(const void* ptr, void* handle, int64_t* offset);
PBK_API int pbk_ipc_open(const void* handle, void** base);
PBK_API int pbk_ipc_close(void* base);
PBK_API int pbk_copy_async(void* dst, const void* src, size_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PBK_H_ */
