// Gated delta rule over a few tokens per sequence (decode), state resident in registers.
//
// Recurrence (pseudobrain/gated_deltanet.py:93-107), per value head and token t:
//   S <- exp(g_t) S;  u = (v_t - S^T k_t) beta_t;  S <- S + k_t u^T;  o_t = S^T (scale q_t)
// With S_dec = exp(g_t) S:  o_t = S_dec^T q_s + (k_t . q_s) u,  so one pass over S
// yields both reductions (S_dec^T k and S_dec^T q) and the update is a rank-1 FMA.
//
// One CTA of 256 threads owns one (sequence, value head) state of 128x128 fp32
// (64 KB): every thread keeps 16 float4 of it in registers for all tokens, so the
// state is read once and written once from/to HBM whatever the token count.
//   PBK_STATE_KV ([dk, dv], rows = key dim): warp w holds rows w, w+8, ..., lane l
//     columns 4l..4l+3; the column sums over rows meet in shared memory.
//   PBK_STATE_VK ([dv, dk], rows = value dim): the same register map over the
//     transposed tile; each row's dot products are warp-shuffle reductions and
//     need no shared memory.
// The HBM roofline bound is (read + write of the fp32 state) / bandwidth.
//
// The extended form (kExt, pbk_gdn_decode_ext) adds what vLLM's decode ops do around the
// same recurrence (vllm/model_executor/layers/fla/ops/fused_recurrent.py:256-336 packed
// decode, :20-170 fused recurrent; fused_sigmoid_gating.py:24-180): the gating
// g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) computed from the raw gate
// inputs, the per-head L2 norm of q and k, packed sequences of any length (cu_seqlens),
// vLLM's null slot (index <= 0), and speculative decoding (2-D state indices: the initial
// state from column num_accepted - 1, the state after token t into column t).
#include "common.cuh"

namespace pbk {

// Device-side copy of pbk_decode_ext (plus nothing): passed by value to the kernel.
struct DecodeExt {
  int gating, beta_round, l2norm, null_slot, zero_skipped;
  float softplus_beta, softplus_threshold, eps;
  pbk_view a, b;
  const void* a_log;
  const void* dt_bias;
  int a_log_dtype, dt_bias_dtype;
  const int32_t* cu_seqlens;
  int64_t index_stride;
  const int32_t* num_accepted;
};

namespace {

constexpr int kDim = 128;        // dk == dv
constexpr int kThreads = 256;    // 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kRows = kDim / kWarps;  // 16 state rows per thread, 4 columns each

__device__ __forceinline__ float round_to(float x, int dtype) {
  return dtype == PBK_BF16 ? __bfloat162float(__float2bfloat16_rn(x)) : x;
}

template <typename TIn, typename TOut, int LAYOUT, bool kExt>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const pbk_gdn_desc d, const DecodeExt x) {
  const int n = blockIdx.x / d.hv;  // sequence
  const int h = blockIdx.x - n * d.hv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // this sequence's rows: dense [B, T, ..] (batch n, rows 0 .. seqlen) or packed (batch 0)
  int64_t bsel = n, row0 = 0;
  int ntok = d.seqlen;
  if (kExt && x.cu_seqlens != nullptr) {
    bsel = 0;
    row0 = x.cu_seqlens[n];
    ntok = x.cu_seqlens[n + 1] - x.cu_seqlens[n];
  }
  const int hk = h / (d.hv / d.hk);
  TOut* ob = reinterpret_cast<TOut*>(const_cast<void*>(d.o.data)) + bsel * d.o.stride_b + row0 * d.o.stride_t +
             h * d.o.stride_h;
  // the state slot read (and, without per-token columns, written)
  int64_t slot = n;
  const bool per_token = kExt && x.index_stride > 0;
  if (d.state_indices != nullptr) {
    if (per_token) {
      const int col = x.num_accepted != nullptr ? x.num_accepted[n] - 1 : 0;
      slot = d.state_indices[(int64_t)n * x.index_stride + col];
    } else {
      slot = d.state_indices[n];
    }
    const bool skip = (kExt && x.null_slot) ? slot <= 0 : slot < 0;
    if (skip) {  // padding / null slot (uniform for the CTA): nothing to read or write
      if (kExt && x.zero_skipped)
        for (int i = tid; i < ntok * kDim; i += kThreads)
          ob[(int64_t)(i / kDim) * d.o.stride_t + (i % kDim)] = from_f32<TOut>(0.f);
      return;
    }
  }
  if (kExt && ntok <= 0) return;
  const int64_t tile = slot * d.state_slot_stride + (int64_t)h * kDim * kDim;
  float* S = d.state + tile;
  const float* S0 = (d.h0 != nullptr ? d.h0 + tile : S);

  __shared__ float sh_k[kDim], sh_q[kDim], sh_v[kDim], sh_u[kDim];
  __shared__ __align__(16) float red[2][kWarps][kDim];
  __shared__ float sh_kq;
  __shared__ float sh_norm[2][4];

  float4 s[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) s[i] = ld_f4_stream(S0 + (int64_t)(warp + kWarps * i) * kDim + 4 * lane);

  const TIn* qb = reinterpret_cast<const TIn*>(d.q.data) + bsel * d.q.stride_b + row0 * d.q.stride_t + hk * d.q.stride_h;
  const TIn* kb = reinterpret_cast<const TIn*>(d.k.data) + bsel * d.k.stride_b + row0 * d.k.stride_t + hk * d.k.stride_h;
  const TIn* vb = reinterpret_cast<const TIn*>(d.v.data) + bsel * d.v.stride_b + row0 * d.v.stride_t + h * d.v.stride_h;

  for (int t = 0; t < ntok; ++t) {
    float gam, bet;
    if (kExt && x.gating) {
      // vLLM's gating: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
      const int64_t at = bsel * x.a.stride_b + (row0 + t) * x.a.stride_t + h * x.a.stride_h;
      const int64_t bt = bsel * x.b.stride_b + (row0 + t) * x.b.stride_t + h * x.b.stride_h;
      const float xa = load_any(x.a.data, at, x.a.dtype) + load_any(x.dt_bias, h, x.dt_bias_dtype);
      const float sb = x.softplus_beta;
      const float sp = sb * xa <= x.softplus_threshold ? logf(1.f + expf(sb * xa)) / sb : xa;
      const float g = -expf(load_any(x.a_log, h, x.a_log_dtype)) * sp;
      gam = expf(g);
      const float sig = 1.f / (1.f + expf(-load_any(x.b.data, bt, x.b.dtype)));
      bet = x.beta_round ? round_to(sig, x.b.dtype) : sig;
    } else {
      gam = expf(load_any(d.g.data, bsel * d.g.stride_b + (row0 + t) * d.g.stride_t + h * d.g.stride_h, d.g.dtype));
      bet = load_any(d.beta.data, bsel * d.beta.stride_b + (row0 + t) * d.beta.stride_t + h * d.beta.stride_h,
                     d.beta.dtype);
    }
    if (tid < kDim) {
      sh_k[tid] = to_f32(kb[t * d.k.stride_t + tid]);
      sh_v[tid] = to_f32(vb[t * d.v.stride_t + tid]);
    } else {
      const float qv = to_f32(qb[t * d.q.stride_t + tid - kDim]);
      sh_q[tid - kDim] = (kExt && x.l2norm) ? qv : qv * d.scale;
    }
    if (kExt && x.l2norm) {
      // per-head L2 norm of k (warps 0-3) and q (warps 4-7) in fp32, then q's scale
      const float own = tid < kDim ? sh_k[tid] : sh_q[tid - kDim];
      const float ss = warp_sum(own * own);
      if (lane == 0) sh_norm[warp >> 2][warp & 3] = ss;
      __syncthreads();
      const int which = tid < kDim ? 0 : 1;
      const float tot = sh_norm[which][0] + sh_norm[which][1] + sh_norm[which][2] + sh_norm[which][3] + x.eps;
      const float nv = x.l2norm == 1 ? own / sqrtf(tot) : own * rsqrtf(tot);
      if (tid < kDim) sh_k[tid] = nv;
      else sh_q[tid - kDim] = nv * d.scale;
    }
    __syncthreads();
    TOut* ot = ob + t * d.o.stride_t;
    if constexpr (LAYOUT == PBK_STATE_KV) {
      float4 ak = make_float4(0.f, 0.f, 0.f, 0.f), aq = ak;
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = warp + kWarps * i;
        const float kr = sh_k[r], qr = sh_q[r];
        s[i].x *= gam; s[i].y *= gam; s[i].z *= gam; s[i].w *= gam;
        ak.x = fmaf(s[i].x, kr, ak.x); ak.y = fmaf(s[i].y, kr, ak.y);
        ak.z = fmaf(s[i].z, kr, ak.z); ak.w = fmaf(s[i].w, kr, ak.w);
        aq.x = fmaf(s[i].x, qr, aq.x); aq.y = fmaf(s[i].y, qr, aq.y);
        aq.z = fmaf(s[i].z, qr, aq.z); aq.w = fmaf(s[i].w, qr, aq.w);
      }
      *reinterpret_cast<float4*>(&red[0][warp][4 * lane]) = ak;
      *reinterpret_cast<float4*>(&red[1][warp][4 * lane]) = aq;
      if (warp == 0) {
        float p = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) p = fmaf(sh_k[4 * lane + j], sh_q[4 * lane + j], p);
        p = warp_sum(p);
        if (lane == 0) sh_kq = p;
      }
      __syncthreads();
      if (tid < kDim) {
        float kv = 0.f, qv = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          kv += red[0][w][tid];
          qv += red[1][w][tid];
        }
        const float u = (sh_v[tid] - kv) * bet;
        sh_u[tid] = u;
        ot[tid] = from_f32<TOut>(fmaf(sh_kq, u, qv));
      }
      __syncthreads();
      const float4 u4 = *reinterpret_cast<const float4*>(&sh_u[4 * lane]);
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const float kr = sh_k[warp + kWarps * i];
        s[i].x = fmaf(kr, u4.x, s[i].x); s[i].y = fmaf(kr, u4.y, s[i].y);
        s[i].z = fmaf(kr, u4.z, s[i].z); s[i].w = fmaf(kr, u4.w, s[i].w);
      }
    } else {
      const float4 k4 = *reinterpret_cast<const float4*>(&sh_k[4 * lane]);
      const float4 q4 = *reinterpret_cast<const float4*>(&sh_q[4 * lane]);
      const float kq = warp_sum(k4.x * q4.x + k4.y * q4.y + k4.z * q4.z + k4.w * q4.w);
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int c = warp + kWarps * i;  // value column of this register row
        s[i].x *= gam; s[i].y *= gam; s[i].z *= gam; s[i].w *= gam;
        const float pk = warp_sum(s[i].x * k4.x + s[i].y * k4.y + s[i].z * k4.z + s[i].w * k4.w);
        const float pq = warp_sum(s[i].x * q4.x + s[i].y * q4.y + s[i].z * q4.z + s[i].w * q4.w);
        const float u = (sh_v[c] - pk) * bet;
        s[i].x = fmaf(k4.x, u, s[i].x); s[i].y = fmaf(k4.y, u, s[i].y);
        s[i].z = fmaf(k4.z, u, s[i].z); s[i].w = fmaf(k4.w, u, s[i].w);
        if (lane == 0) ot[c] = from_f32<TOut>(fmaf(kq, u, pq));
      }
    }
    if (per_token) {  // speculative decoding: the state after token t into column t (if not null)
      const int64_t st = d.state_indices[(int64_t)n * x.index_stride + t];
      if (x.null_slot ? st > 0 : st >= 0) {
        float* Sd = d.state + st * d.state_slot_stride + (int64_t)h * kDim * kDim;
#pragma unroll
        for (int i = 0; i < kRows; ++i) st_f4_stream(Sd + (int64_t)(warp + kWarps * i) * kDim + 4 * lane, s[i]);
      }
    }
    __syncthreads();  // the next token restages shared memory
  }
  if (!per_token) {
#pragma unroll
    for (int i = 0; i < kRows; ++i) st_f4_stream(S + (int64_t)(warp + kWarps * i) * kDim + 4 * lane, s[i]);
  }
}

template <typename TIn, typename TOut, bool kExt>
cudaError_t launch_layout(const pbk_gdn_desc& d, const DecodeExt& x, cudaStream_t st) {
  const dim3 grid((unsigned)((int64_t)d.batch * d.hv));
  if (d.state_layout == PBK_STATE_KV)
    gdn_decode_kernel<TIn, TOut, PBK_STATE_KV, kExt><<<grid, kThreads, 0, st>>>(d, x);
  else
    gdn_decode_kernel<TIn, TOut, PBK_STATE_VK, kExt><<<grid, kThreads, 0, st>>>(d, x);
  return cudaGetLastError();
}

template <bool kExt>
cudaError_t launch_any(const pbk_gdn_desc& d, const DecodeExt& x, cudaStream_t st) {
  const bool in_bf16 = d.q.dtype == PBK_BF16, out_bf16 = d.o.dtype == PBK_BF16;
  if (in_bf16 && out_bf16) return launch_layout<__nv_bfloat16, __nv_bfloat16, kExt>(d, x, st);
  if (in_bf16) return launch_layout<__nv_bfloat16, float, kExt>(d, x, st);
  if (out_bf16) return launch_layout<float, __nv_bfloat16, kExt>(d, x, st);
  return launch_layout<float, float, kExt>(d, x, st);
}

}  // namespace

cudaError_t launch_gdn_decode(const pbk_gdn_desc& d, cudaStream_t st) { return launch_any<false>(d, DecodeExt{}, st); }

cudaError_t launch_gdn_decode_ext(const pbk_gdn_desc& d, const pbk_decode_ext& e, cudaStream_t st) {
  DecodeExt x;
  x.gating = e.gating;
  x.beta_round = e.beta_round;
  x.l2norm = e.l2norm;
  x.null_slot = e.null_slot;
  x.zero_skipped = e.zero_skipped;
  x.softplus_beta = e.softplus_beta;
  x.softplus_threshold = e.softplus_threshold;
  x.eps = e.eps;
  x.a = e.a;
  x.b = e.b;
  x.a_log = e.a_log;
  x.dt_bias = e.dt_bias;
  x.a_log_dtype = e.a_log_dtype;
  x.dt_bias_dtype = e.dt_bias_dtype;
  x.cu_seqlens = e.cu_seqlens;
  x.index_stride = e.index_stride;
  x.num_accepted = e.num_accepted;
  return launch_any<true>(d, x, st);
}

}  // namespace pbk
