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
#include "common.cuh"

namespace pbk {
namespace {

constexpr int kDim = 128;        // dk == dv
constexpr int kThreads = 256;    // 8 warps
constexpr int kWarps = kThreads / 32;
constexpr int kRows = kDim / kWarps;  // 16 state rows per thread, 4 columns each

template <typename TIn, typename TOut, int LAYOUT>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_kernel(const pbk_gdn_desc d) {
  const int b = blockIdx.x / d.hv;
  const int h = blockIdx.x - b * d.hv;
  int64_t slot = b;
  if (d.state_indices != nullptr) {
    slot = d.state_indices[b];
    if (slot < 0) return;  // padding slot: nothing to read or write
  }
  const int hk = h / (d.hv / d.hk);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tile = slot * d.state_slot_stride + (int64_t)h * kDim * kDim;
  float* S = d.state + tile;
  const float* S0 = (d.h0 != nullptr ? d.h0 + tile : S);

  __shared__ float sh_k[kDim], sh_q[kDim], sh_v[kDim], sh_u[kDim];
  __shared__ __align__(16) float red[2][kWarps][kDim];
  __shared__ float sh_kq;

  float4 s[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) s[i] = ld_f4_stream(S0 + (int64_t)(warp + kWarps * i) * kDim + 4 * lane);

  const TIn* qb = reinterpret_cast<const TIn*>(d.q.data) + b * d.q.stride_b + hk * d.q.stride_h;
  const TIn* kb = reinterpret_cast<const TIn*>(d.k.data) + b * d.k.stride_b + hk * d.k.stride_h;
  const TIn* vb = reinterpret_cast<const TIn*>(d.v.data) + b * d.v.stride_b + h * d.v.stride_h;
  TOut* ob = reinterpret_cast<TOut*>(const_cast<void*>(d.o.data)) + b * d.o.stride_b + h * d.o.stride_h;

  for (int t = 0; t < d.seqlen; ++t) {
    if (tid < kDim) {
      sh_k[tid] = to_f32(kb[t * d.k.stride_t + tid]);
      sh_v[tid] = to_f32(vb[t * d.v.stride_t + tid]);
    } else {
      sh_q[tid - kDim] = to_f32(qb[t * d.q.stride_t + tid - kDim]) * d.scale;
    }
    const float gam = expf(load_any(d.g.data, b * d.g.stride_b + t * d.g.stride_t + h * d.g.stride_h, d.g.dtype));
    const float bet = load_any(d.beta.data, b * d.beta.stride_b + t * d.beta.stride_t + h * d.beta.stride_h,
                               d.beta.dtype);
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
    __syncthreads();  // the next token restages shared memory
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) st_f4_stream(S + (int64_t)(warp + kWarps * i) * kDim + 4 * lane, s[i]);
}

template <typename TIn, typename TOut>
cudaError_t launch_layout(const pbk_gdn_desc& d, cudaStream_t st) {
  const dim3 grid((unsigned)((int64_t)d.batch * d.hv));
  if (d.state_layout == PBK_STATE_KV)
    gdn_decode_kernel<TIn, TOut, PBK_STATE_KV><<<grid, kThreads, 0, st>>>(d);
  else
    gdn_decode_kernel<TIn, TOut, PBK_STATE_VK><<<grid, kThreads, 0, st>>>(d);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gdn_decode(const pbk_gdn_desc& d, cudaStream_t st) {
  const bool in_bf16 = d.q.dtype == PBK_BF16, out_bf16 = d.o.dtype == PBK_BF16;
  if (in_bf16 && out_bf16) return launch_layout<__nv_bfloat16, __nv_bfloat16>(d, st);
  if (in_bf16) return launch_layout<__nv_bfloat16, float>(d, st);
  if (out_bf16) return launch_layout<float, __nv_bfloat16>(d, st);
  return launch_layout<float, float>(d, st);
}

}  // namespace pbk
