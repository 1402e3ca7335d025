// The Gated DeltaNet layer's elementwise stages around the recurrence, as vLLM's adapter
// runs them (causal_conv1d, fused gating, in-kernel q/k L2 norm, gated RMSNorm):
//   conv + norm: y = SiLU(causal depthwise conv of x over time, carried tail) per channel
//     (short_convolution, pseudobrain/gated_deltanet.py:314-338), split into q | k | v heads
//     of 128 channels, q and k L2-normalised per head (l2_normalize, :59-70, 'max' or 'hf'),
//     and the new tail (the last width-1 inputs);
//   gating: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (:427-429);
//   output norm: o * rsqrt(mean(o^2) + eps) * weight * SiLU(gate) (:439-440).
// All arithmetic in fp32. Memory-bound: each reads and writes its tensors once.
#include <algorithm>

#include "common.cuh"

namespace pbk {
namespace {

constexpr int kHd = 128;    // channels per head
constexpr int kTile = 32;   // tokens per CTA of the conv + norm kernel
constexpr int kMaxWidth = 8;

__device__ __forceinline__ float silu(float y) { return y / (1.f + expf(-y)); }
// Store into an output view (pbk_view carries its pointer as const void*).
__device__ __forceinline__ void store_any(const void* p, int64_t i, int dtype, float x) {
  if (dtype == PBK_BF16) const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(p))[i] = __float2bfloat16_rn(x);
  else const_cast<float*>(reinterpret_cast<const float*>(p))[i] = x;
}

// Row r of a [B, T, H] row space into (b, t, h): 32-bit division below 2^31 rows (64-bit
// division costs far more than a row's work).
__device__ __forceinline__ void split_row(int64_t r, int heads, int seqlen, int& b, int& t, int& h) {
  if (r < 0x7fffffffLL) {
    const uint32_t bt = (uint32_t)r / (uint32_t)heads;
    h = (int)((uint32_t)r - bt * (uint32_t)heads);
    t = (int)(bt % (uint32_t)seqlen);
    b = (int)(bt / (uint32_t)seqlen);
  } else {
    h = (int)(r % heads);
    t = (int)((r / heads) % seqlen);
    b = (int)(r / ((int64_t)heads * seqlen));
  }
}

// CTA = (token tile, head of the q | k | v channel layout, sequence); thread = channel.
__global__ void __launch_bounds__(kHd) gdn_conv_norm_kernel(const pbk_conv_desc d) {
  __shared__ float ys[kTile][kHd + 1];
  const int tile = blockIdx.x, hd = blockIdx.y, b = blockIdx.z, c = threadIdx.x;
  const int ch = hd * kHd + c, K = d.weight != nullptr ? d.width : 1, t0 = tile * kTile;
  const int nt = min(kTile, d.seqlen - t0);
  auto x_at = [&](int t) -> float {  // input of step t; t < 0 reads the carried tail
    if (t >= 0) return load_any(d.x.data, b * d.x.stride_b + (int64_t)t * d.x.stride_t + ch * d.x.stride_h, d.x.dtype);
    const int j = K - 1 + t;  // tail row
    if (j < 0 || d.tail.data == nullptr) return 0.f;
    return load_any(d.tail.data, b * d.tail.stride_b + (int64_t)j * d.tail.stride_t + ch * d.tail.stride_h, d.tail.dtype);
  };
  // right-aligned taps: win[i] = x_{t - (kMaxWidth - 1 - i)} for the step t being computed,
  // w[i] its weight (weight[ch][K - kMaxWidth + i]; zero left of the K taps)
  float w[kMaxWidth], win[kMaxWidth];
#pragma unroll
  for (int i = 0; i < kMaxWidth; ++i) {
    const int j = i - (kMaxWidth - K);
    w[i] = (d.weight != nullptr && j >= 0) ? d.weight[(int64_t)ch * K + j] : 0.f;
    win[i] = (i < kMaxWidth - 1 && j >= 0) ? x_at(t0 - (kMaxWidth - 1 - i)) : 0.f;
  }
  for (int i = 0; i < nt; ++i) {
    win[kMaxWidth - 1] = x_at(t0 + i);
    float y = 0.f;
#pragma unroll
    for (int u = 0; u < kMaxWidth; ++u) y = fmaf(w[u], win[u], y);
    ys[i][c] = silu(d.weight != nullptr ? y : win[kMaxWidth - 1]);
#pragma unroll
    for (int u = 0; u < kMaxWidth - 1; ++u) win[u] = win[u + 1];
  }
  // the new tail: inputs T-K+1 .. T-1, written by the tile holding step T-1
  if (d.new_tail.data != nullptr && t0 + nt == d.seqlen) {
    for (int j = 0; j < K - 1; ++j)
      store_any(d.new_tail.data, b * d.new_tail.stride_b + (int64_t)j * d.new_tail.stride_t + ch * d.new_tail.stride_h,
                d.new_tail.dtype, x_at(d.seqlen - K + 1 + j));
  }
  __syncthreads();
  // rows: q heads 0 .. hk-1, k heads hk .. 2hk-1 (normalised), v heads after them
  const bool is_q = hd < d.hk, is_k = !is_q && hd < 2 * d.hk;
  const pbk_view& out = is_q ? d.q : (is_k ? d.k : d.v);
  const int oh = is_q ? hd : (is_k ? hd - d.hk : hd - 2 * d.hk);
  const int warp = c >> 5, lane = c & 31;
  for (int i = warp; i < nt; i += kHd / 32) {
    float v[4], ss = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = ys[i][lane + 32 * u];
      ss = fmaf(v[u], v[u], ss);
    }
    float scale = 1.f;
    if ((is_q || is_k) && d.l2mode != 0) {
      ss = warp_sum(ss);
      // 'max': x / max(||x||, eps) (F.normalize); 'hf': x * rsqrt(sum x^2 + eps)
      scale = d.l2mode == 1 ? 1.f / fmaxf(sqrtf(ss), d.eps) : rsqrtf(ss + d.eps);
    }
    const int64_t base = b * out.stride_b + (int64_t)(t0 + i) * out.stride_t + (int64_t)oh * out.stride_h;
#pragma unroll
    for (int u = 0; u < 4; ++u) store_any(out.data, base + lane + 32 * u, out.dtype, v[u] * scale);
  }
}

// The same for bf16 inputs and outputs with a contiguous channel dim (the common case): the
// tile's input rows (and the width - 1 before it) are staged in shared memory with 16-byte
// loads, all in flight at once; each thread then convolves one channel from shared memory;
// the normalised rows leave as 8-byte stores (lane = 4 channels).
// SiLU for bf16 outputs: y sigmoid(y) = h (1 + tanh h), h = y / 2, with the hardware tanh
// approximation (one special-function instruction; relative error about 2^-11, below the
// bf16 rounding of the result).
__device__ __forceinline__ float tanh_hw(float x) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float silu_fast(float y) {
  const float h = 0.5f * y;
  return fmaf(h, tanh_hw(h), h);
}

// Two threads per channel, each convolving half of the tile's tokens.
constexpr int kVecThreads = 2 * kHd;
template <int K>
__global__ void __launch_bounds__(kVecThreads) gdn_conv_norm_vec_kernel(const pbk_conv_desc d) {
  __shared__ __align__(16) __nv_bfloat16 xs[kTile + kMaxWidth - 1][kHd];
  __shared__ __align__(16) float ys[kTile][kHd + 4];
  // head fastest in the grid: CTAs running together read neighbouring 256-byte slices of the
  // same input rows (and write neighbouring heads of the same output rows)
  const int hd = blockIdx.x, tile = blockIdx.y, b = blockIdx.z, c = threadIdx.x & (kHd - 1);
  const int half = threadIdx.x / kHd;
  constexpr int H = K - 1;
  const int t0 = tile * kTile;
  const int nt = min(kTile, d.seqlen - t0);
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(d.x.data);
  const __nv_bfloat16* tb = reinterpret_cast<const __nv_bfloat16*>(d.tail.data);
  // stage rows r = 0 .. H + nt - 1 (token t0 - H + r); 16 vectors of 8 channels per row
  for (int e = threadIdx.x; e < (H + nt) * 16; e += kVecThreads) {
    const int r = e >> 4, vq = e & 15, t = t0 - H + r;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    const int64_t ch = (int64_t)hd * kHd + 8 * vq;
    if (t >= 0) {
      val = *reinterpret_cast<const uint4*>(xb + b * d.x.stride_b + (int64_t)t * d.x.stride_t + ch);
    } else if (tb != nullptr) {  // the carried tail: row H + t of [B, K - 1, C]
      val = *reinterpret_cast<const uint4*>(tb + b * d.tail.stride_b + (int64_t)(H + t) * d.tail.stride_t + ch);
    }
    *reinterpret_cast<uint4*>(&xs[r][8 * vq]) = val;
  }
  float w[K], win[K];  // taps and the sliding window x_{t-K+1} .. x_t of this channel
#pragma unroll
  for (int j = 0; j < K; ++j) w[j] = d.weight != nullptr ? d.weight[((int64_t)hd * kHd + c) * K + j] : 0.f;
  __syncthreads();
  const int i0 = half * (kTile / 2), i1 = min(i0 + kTile / 2, nt);
#pragma unroll
  for (int j = 0; j < H; ++j) win[j] = __bfloat162float(xs[i0 + j][c]);
#pragma unroll 4
  for (int i = i0; i < i1; ++i) {
    win[H] = __bfloat162float(xs[i + H][c]);
    float y = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) y = fmaf(w[j], win[j], y);
    ys[i][c] = silu_fast(d.weight != nullptr ? y : win[H]);
#pragma unroll
    for (int j = 0; j < H; ++j) win[j] = win[j + 1];
  }
  if (half == 0 && d.new_tail.data != nullptr && t0 + nt == d.seqlen) {
    for (int j = 0; j < H; ++j)  // the last K - 1 inputs: staged rows nt .. nt + H - 1
      store_any(d.new_tail.data, b * d.new_tail.stride_b + (int64_t)j * d.new_tail.stride_t +
                                     ((int64_t)hd * kHd + c) * d.new_tail.stride_h,
                d.new_tail.dtype, __bfloat162float(xs[nt + j][c]));
  }
  __syncthreads();
  const bool is_q = hd < d.hk, is_k = !is_q && hd < 2 * d.hk;
  const pbk_view& out = is_q ? d.q : (is_k ? d.k : d.v);
  const int oh = is_q ? hd : (is_k ? hd - d.hk : hd - 2 * d.hk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < nt; i += kVecThreads / 32) {
    const float4 v = *reinterpret_cast<const float4*>(&ys[i][4 * lane]);
    float scale = 1.f;
    if ((is_q || is_k) && d.l2mode != 0) {
      const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
      scale = d.l2mode == 1 ? 1.f / fmaxf(sqrtf(ss), d.eps) : rsqrtf(ss + d.eps);
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x * scale, v.y * scale);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(v.z * scale, v.w * scale);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    __nv_bfloat16* ob = const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(out.data));
    *reinterpret_cast<uint2*>(ob + b * out.stride_b + (int64_t)(t0 + i) * out.stride_t + (int64_t)oh * out.stride_h +
                              4 * lane) = pk;
  }
}

// One thread per (sequence, token, head); 32-bit index arithmetic (the launcher checks that
// the element count fits), as 64-bit divisions would cost more than the element's work.
__global__ void gdn_gating_kernel(const pbk_gating_desc d) {
  const uint32_t n = (uint32_t)d.batch * d.seqlen * d.hv;
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    const uint32_t row = e / (uint32_t)d.hv;
    const int h = (int)(e - row * (uint32_t)d.hv), t = (int)(row % (uint32_t)d.seqlen), b = (int)(row / (uint32_t)d.seqlen);
    const int64_t ab = b * d.decay.stride_b + (int64_t)t * d.decay.stride_t;
    const float a = load_any(d.decay.data, ab + (int64_t)h * d.decay.stride_h, d.decay.dtype);
    const float bb = load_any(d.decay.data, ab + (int64_t)(d.hv + h) * d.decay.stride_h, d.decay.dtype);
    const float x = a + d.dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, threshold 20 as F.softplus
    const float gv = -expf(d.a_log[h]) * sp;
    const float be = 1.f / (1.f + expf(-bb));
    store_any(d.g.data, b * d.g.stride_b + (int64_t)t * d.g.stride_t + (int64_t)h * d.g.stride_h, d.g.dtype, gv);
    store_any(d.beta.data, b * d.beta.stride_b + (int64_t)t * d.beta.stride_t + (int64_t)h * d.beta.stride_h,
              d.beta.dtype, be);
  }
}

// One warp per (sequence, token, value head) row of 128.
__global__ void __launch_bounds__(256) gdn_out_norm_kernel(const pbk_out_norm_desc d) {
  const int64_t rows = (int64_t)d.batch * d.seqlen * d.hv;
  const int64_t r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  int b, t, h;
  split_row(r, d.hv, d.seqlen, b, t, h);
  const int64_t ob = b * d.o.stride_b + (int64_t)t * d.o.stride_t + (int64_t)h * d.o.stride_h;
  const int64_t gb = b * d.gate.stride_b + (int64_t)t * d.gate.stride_t + (int64_t)h * d.gate.stride_h;
  const int64_t yb = b * d.out.stride_b + (int64_t)t * d.out.stride_t + (int64_t)h * d.out.stride_h;
  float v[4], ss = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    v[u] = load_any(d.o.data, ob + lane + 32 * u, d.o.dtype);
    ss = fmaf(v[u], v[u], ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / kHd + d.eps);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = lane + 32 * u;
    const float gt = load_any(d.gate.data, gb + i, d.gate.dtype);
    const float wt = load_any(d.weight, i, d.weight_dtype);
    store_any(d.out.data, yb + i, d.out.dtype, v[u] * inv * wt * silu(gt));
  }
}

}  // namespace

namespace {
bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
// bf16 in and out, contiguous channels, 16-byte rows in (8-byte out): the staged kernel.
bool conv_vec_ok(const pbk_conv_desc& d) {
  const pbk_view& x = d.x;
  if (x.dtype != PBK_BF16 || x.stride_h != 1 || !aligned(x.data, 16) || x.stride_b % 8 || x.stride_t % 8) return false;
  if (d.tail.data != nullptr && (d.tail.dtype != PBK_BF16 || d.tail.stride_h != 1 || !aligned(d.tail.data, 16) ||
                                 d.tail.stride_b % 8 || d.tail.stride_t % 8))
    return false;
  const pbk_view* outs[3] = {&d.q, &d.k, &d.v};
  for (const pbk_view* o : outs)
    if (o->dtype != PBK_BF16 || !aligned(o->data, 8) || o->stride_b % 4 || o->stride_t % 4 || o->stride_h % 4)
      return false;
  return true;
}
// The output norm with lane = 4 consecutive dims (16-byte fp32 / 8-byte bf16 accesses) for
// contiguous rows, gate bf16, weight fp32; SiLU as silu_fast when the output is bf16.
template <typename TO, typename TG>
__global__ void __launch_bounds__(256) gdn_out_norm_vec_kernel(const pbk_out_norm_desc d) {
  // 32-bit row arithmetic (the launcher takes this kernel only below 2^31 rows)
  const uint32_t rows = (uint32_t)d.batch * d.seqlen * d.hv;
  const uint32_t r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint32_t bt = r / (uint32_t)d.hv;
  const int h = (int)(r - bt * (uint32_t)d.hv), t = (int)(bt % (uint32_t)d.seqlen), b = (int)(bt / (uint32_t)d.seqlen);
  const int64_t ob = b * d.o.stride_b + (int64_t)t * d.o.stride_t + (int64_t)h * d.o.stride_h + 4 * lane;
  const int64_t gb = b * d.gate.stride_b + (int64_t)t * d.gate.stride_t + (int64_t)h * d.gate.stride_h + 4 * lane;
  const int64_t yb = b * d.out.stride_b + (int64_t)t * d.out.stride_t + (int64_t)h * d.out.stride_h + 4 * lane;
  float v[4], g[4];
  if constexpr (sizeof(TO) == 4) {
    const float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(d.o.data) + ob);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
  } else {
    const uint2 x = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(d.o.data) + ob);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
    v[0] = a.x, v[1] = a.y, v[2] = c.x, v[3] = c.y;
  }
  {
    const uint2 x = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(d.gate.data) + gb);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
    const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
    g[0] = a.x, g[1] = a.y, g[2] = c.x, g[3] = c.y;
  }
  const float4 wt = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(d.weight) + 4 * lane);
  const float ww[4] = {wt.x, wt.y, wt.z, wt.w};
  const float inv = rsqrtf(warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]) / kHd + d.eps);
  float y[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) y[u] = v[u] * inv * ww[u] * (sizeof(TG) == 2 ? silu_fast(g[u]) : silu(g[u]));
  if constexpr (sizeof(TG) == 4) {
    float* op = const_cast<float*>(reinterpret_cast<const float*>(d.out.data)) + yb;  // 16-byte aligned
    *reinterpret_cast<float4*>(op) = make_float4(y[0], y[1], y[2], y[3]);
  } else {
    const __nv_bfloat162 lo = __floats2bfloat162_rn(y[0], y[1]), hi = __floats2bfloat162_rn(y[2], y[3]);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    __nv_bfloat16* op = const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(d.out.data)) + yb;
    *reinterpret_cast<uint2*>(op) = pk;  // 8-byte aligned
  }
}

// Row L2 norm: one warp per (sequence, token, head) row of 128, lane = 4 dims.
__global__ void __launch_bounds__(256) gdn_l2norm_kernel(const pbk_view x, const pbk_view out, int batch, int seqlen,
                                                         int heads, int mode, float eps) {
  const int64_t rows = (int64_t)batch * seqlen * heads;
  const int64_t r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  int b, t, h;
  split_row(r, heads, seqlen, b, t, h);
  const int64_t xb = b * x.stride_b + (int64_t)t * x.stride_t + (int64_t)h * x.stride_h;
  const int64_t yb = b * out.stride_b + (int64_t)t * out.stride_t + (int64_t)h * out.stride_h;
  float v[4], ss = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    v[u] = load_any(x.data, xb + lane + 32 * u, x.dtype);
    ss = fmaf(v[u], v[u], ss);
  }
  ss = warp_sum(ss);
  const float scale = mode == 1 ? 1.f / fmaxf(sqrtf(ss), eps) : rsqrtf(ss + eps);
#pragma unroll
  for (int u = 0; u < 4; ++u) store_any(out.data, yb + lane + 32 * u, out.dtype, v[u] * scale);
}

}  // namespace

cudaError_t launch_gdn_l2norm(const pbk_view& x, const pbk_view& out, int batch, int seqlen, int heads, int mode,
                              float eps, cudaStream_t st) {
  const int64_t rows = (int64_t)batch * seqlen * heads;
  if (rows == 0) return cudaSuccess;
  gdn_l2norm_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(x, out, batch, seqlen, heads, mode, eps);
  return cudaGetLastError();
}

cudaError_t launch_gdn_conv_norm(const pbk_conv_desc& d, cudaStream_t st) {
  const dim3 grid((unsigned)((d.seqlen + kTile - 1) / kTile), (unsigned)(2 * d.hk + d.hv), (unsigned)d.batch);
  const dim3 vgrid((unsigned)(2 * d.hk + d.hv), grid.x, (unsigned)d.batch);
  if (conv_vec_ok(d) && grid.x <= 65535u) {
    switch (d.weight != nullptr ? d.width : 1) {
      case 1: gdn_conv_norm_vec_kernel<1><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 2: gdn_conv_norm_vec_kernel<2><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 3: gdn_conv_norm_vec_kernel<3><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 4: gdn_conv_norm_vec_kernel<4><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 5: gdn_conv_norm_vec_kernel<5><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 6: gdn_conv_norm_vec_kernel<6><<<vgrid, kVecThreads, 0, st>>>(d); break;
      case 7: gdn_conv_norm_vec_kernel<7><<<vgrid, kVecThreads, 0, st>>>(d); break;
      default: gdn_conv_norm_vec_kernel<8><<<vgrid, kVecThreads, 0, st>>>(d); break;
    }
  } else {
    gdn_conv_norm_kernel<<<grid, kHd, 0, st>>>(d);
  }
  return cudaGetLastError();
}

cudaError_t launch_gdn_gating(const pbk_gating_desc& d, cudaStream_t st) {
  const int64_t n = (int64_t)d.batch * d.seqlen * d.hv;
  if (n > 0x7fffffffLL) return cudaErrorInvalidValue;  // 32-bit element indices
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  gdn_gating_kernel<<<blocks, 256, 0, st>>>(d);
  return cudaGetLastError();
}

cudaError_t launch_gdn_out_norm(const pbk_out_norm_desc& d, cudaStream_t st) {
  const int64_t rows = (int64_t)d.batch * d.seqlen * d.hv;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  auto rows_ok = [](const pbk_view& x, int64_t elems) {  // 16-byte (fp32) or 8-byte (bf16) lanes
    return aligned(x.data, 4 * elems) && x.stride_b % 4 == 0 && x.stride_t % 4 == 0 && x.stride_h % 4 == 0;
  };
  const bool o32 = d.o.dtype == PBK_F32, out32 = d.out.dtype == PBK_F32;
  const bool vec = rows < 0x7fffffffLL && (o32 || d.o.dtype == PBK_BF16) && d.gate.dtype == PBK_BF16 &&
                   d.weight_dtype == PBK_F32 &&
                   aligned(d.weight, 16) && rows_ok(d.o, o32 ? 4 : 2) && rows_ok(d.gate, 2) &&
                   rows_ok(d.out, out32 ? 4 : 2);
  if (!vec) gdn_out_norm_kernel<<<grid, 256, 0, st>>>(d);
  else if (o32 && out32) gdn_out_norm_vec_kernel<float, float><<<grid, 256, 0, st>>>(d);
  else if (o32) gdn_out_norm_vec_kernel<float, __nv_bfloat16><<<grid, 256, 0, st>>>(d);
  else if (out32) gdn_out_norm_vec_kernel<__nv_bfloat16, float><<<grid, 256, 0, st>>>(d);
  else gdn_out_norm_vec_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, st>>>(d);
  return cudaGetLastError();
}

bool gdn_conv_width_ok(int width) { return width >= 1 && width <= kMaxWidth; }

}  // namespace pbk
