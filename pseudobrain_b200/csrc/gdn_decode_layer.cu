// The decode step of the Gated DeltaNet layer in one kernel: from the input projection's
// output to the gated, normed per-step output (GatedDeltaNetLayer.forward,
// pseudobrain/gated_deltanet.py:411-440, for the few tokens that select_kernel sends to the
// sequential recurrence, :291-294):
//   short_convolution (:314-338): causal depthwise conv over time with the carried tail, SiLU;
//   l2_normalize of q and k per head (:59-70, 'max' or 'hf');
//   g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b) (:427-429);
//   the recurrence of delta_rule_sequential (:93-107), the state updated in place;
//   o * rsqrt(mean(o^2) + eps) * o_norm * SiLU(gate) (:439-440).
// Everything stays in fp32 between the stages (the reference's compute dtype); nothing but the
// output, the state and the new conv tail is written.
//
// One CTA of 256 threads per (sequence, value head), the state in registers as in
// gdn_decode.cu (16 float4 per thread; the [K,V] layout reduces through shared memory, the
// [V,K] layout with warp shuffles). Conv channels of the CTA: its key head's q and k (128
// each) and its value head's v (128); thread c < 128 convolves k and v channel c, thread
// 128 + c q channel c, each with its last width - 1 inputs in registers.
//
// The new tail may overwrite the old one in place. Value heads sharing a key head share that
// key head's q and k tail channels, so those CTAs form one thread-block cluster (Hv / Hk CTAs,
// at most 8): every CTA reads its tail rows, runs the step, then arrives on and waits at the
// cluster barrier before any tail write; the cluster's first CTA writes the q/k channels,
// every CTA its own v channels. A token's loads (the projection row, the gate inputs, the
// output gate) are issued one token ahead, token 0's beside the state loads; bf16 tails and
// rows move through shared memory in 16-byte vectors.
#include "common.cuh"

namespace pbk {

// Device-side copy of pbk_gdn_layer_desc (passed by value).
struct DecodeLayerArgs {
  int batch, seqlen, hk, hv, width, l2mode;
  float l2_eps, norm_eps, scale;
  pbk_view qkv, tail, new_tail, decay, gate, out;
  const float* conv_weight;
  const float* a_log;
  const float* dt_bias;
  const void* o_norm;
  int o_norm_dtype;
  float* state;
  int64_t state_slot_stride;
  const int32_t* state_indices;
  int cluster_sync;  // 1: the tail is rewritten in place by a cluster of Hv / Hk CTAs
  int vec_tail;      // 1: tail and new tail are bf16 rows of contiguous channels, 16-byte aligned
  int vec_x;         // 1: the projection rows are bf16, contiguous channels, 16-byte aligned
};

namespace {

constexpr int kDim = 128;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = kDim / kWarps;

__device__ __forceinline__ float silu_exact(float y) { return y / (1.f + expf(-y)); }

__device__ __forceinline__ void store_any(const void* p, int64_t i, int dtype, float x) {
  if (dtype == PBK_BF16) const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(p))[i] = __float2bfloat16_rn(x);
  else const_cast<float*>(reinterpret_cast<const float*>(p))[i] = x;
}

// Relaxed arrive: the only ordering the tail needs is the old tail's reads before the cluster
// leader's writes, and those reads have long returned (their values feed the state stores
// issued before the arrive). A release arrive would also wait for those 64 KB of stores.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// KMAX: the compiled tap count (4 or 8); the layer's `width` taps are right-aligned in it
// (taps left of them have weight zero).
template <int LAYOUT, int KMAX>
__global__ void __launch_bounds__(kThreads, 2) gdn_decode_layer_kernel(const DecodeLayerArgs a) {
  constexpr int H = KMAX - 1;  // history slots per channel
  const int n = blockIdx.x / a.hv;
  const int h = blockIdx.x - n * a.hv;
  const int ratio = a.hv / a.hk, hkh = h / ratio;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool low = tid < kDim;  // k + v channel c (else q channel c)
  const int c = tid & (kDim - 1);

  int64_t slot = n;
  if (a.state_indices != nullptr) {
    slot = a.state_indices[n];
    if (slot < 0) return;  // padding slot (uniform over the cluster: one sequence)
  }
  float* S = a.state + slot * a.state_slot_stride + (int64_t)h * kDim * kDim;

  __shared__ float sh_k[kDim], sh_q[kDim], sh_v[kDim], sh_u[kDim], sh_o[kDim];
  __shared__ __align__(16) float red[2][kWarps][kDim];
  __shared__ float sh_kq;
  __shared__ float sh_norm[2][4];
  __shared__ float sh_osq[4];

  // the CTA's conv channels: segment 0 its key head's q, 1 its k, 2 its value head's v
  __shared__ __align__(16) __nv_bfloat16 sh_tail[KMAX - 1][3 * kDim];
  __shared__ __align__(16) __nv_bfloat16 sh_x[3 * kDim];
  auto seg_ch = [&](int seg) { return seg == 0 ? hkh * kDim : (seg == 1 ? (a.hk + hkh) * kDim : (2 * a.hk + h) * kDim); };

  // conv channels: A = k (low) or q (high), B = v (low only)
  const int ch_a = low ? (a.hk + hkh) * kDim + c : hkh * kDim + c;
  const int ch_b = (2 * a.hk + h) * kDim + c;
  const bool conv = a.conv_weight != nullptr;
  const int K = conv ? a.width : 1;
  float wa[KMAX], wb[KMAX], ha[H], hb[H];
#pragma unroll
  for (int i = 0; i < KMAX; ++i) {
    const int j = i - (KMAX - K);  // weight column of tap i
    wa[i] = (conv && j >= 0) ? a.conv_weight[(int64_t)ch_a * K + j] : 0.f;
    wb[i] = (conv && low && j >= 0) ? a.conv_weight[(int64_t)ch_b * K + j] : 0.f;
  }
  // history slot i holds the input (H - i) steps back; tail row r = i - (KMAX - K) (zero
  // where the tail has no row or is absent). The vector path stages the CTA's tail slice in
  // shared memory with 16-byte loads (scattered 2-byte loads of it cost far more than its bytes).
  const bool tail_in = conv && K > 1 && a.tail.data != nullptr;
  if (tail_in && a.vec_tail) {
    const __nv_bfloat16* tb = reinterpret_cast<const __nv_bfloat16*>(a.tail.data);
    for (int e = tid; e < (K - 1) * 48; e += kThreads) {
      const int r = e / 48, rem = e - r * 48, seg = rem >> 4, ck = rem & 15;
      const uint4 v = *reinterpret_cast<const uint4*>(tb + (int64_t)n * a.tail.stride_b + (int64_t)r * a.tail.stride_t +
                                                      seg_ch(seg) + 8 * ck);
      *reinterpret_cast<uint4*>(&sh_tail[r + (KMAX - K)][seg * kDim + 8 * ck]) = v;
    }
  }
  // the state: 16 float4 per thread, in flight from here until the recurrence
  float4 s[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i) s[i] = ld_f4_stream(S + (int64_t)(warp + kWarps * i) * kDim + 4 * lane);
  if (tail_in && a.vec_tail) __syncthreads();
#pragma unroll
  for (int i = 0; i < H; ++i) {
    const int r = i - (KMAX - K);
    ha[i] = hb[i] = 0.f;
    if (tail_in && r >= 0) {
      if (a.vec_tail) {
        ha[i] = __bfloat162float(sh_tail[i][(low ? kDim : 0) + c]);
        if (low) hb[i] = __bfloat162float(sh_tail[i][2 * kDim + c]);
      } else {
        const int64_t base = (int64_t)n * a.tail.stride_b + (int64_t)r * a.tail.stride_t;
        ha[i] = load_any(a.tail.data, base + (int64_t)ch_a * a.tail.stride_h, a.tail.dtype);
        if (low) hb[i] = load_any(a.tail.data, base + (int64_t)ch_b * a.tail.stride_h, a.tail.dtype);
      }
    }
  }
  const float a_log_h = a.a_log[h], dt_bias_h = a.dt_bias[h];
  const float wo = load_any(a.o_norm, c, a.o_norm_dtype);
  // token inputs, loaded one token ahead (token 0's here, beside the state and tail loads)
  auto x_ab = [&](int t, float& xa, float& xb) {
    const int64_t xrow = (int64_t)n * a.qkv.stride_b + (int64_t)t * a.qkv.stride_t;
    xa = load_any(a.qkv.data, xrow + (int64_t)ch_a * a.qkv.stride_h, a.qkv.dtype);
    xb = low ? load_any(a.qkv.data, xrow + (int64_t)ch_b * a.qkv.stride_h, a.qkv.dtype) : 0.f;
  };
  // vector path: threads 0..47 load the token's three 256-byte channel segments
  auto x_vec = [&](int t) -> uint4 {
    const int seg = tid >> 4, ck = tid & 15;
    return *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.qkv.data) +
                                           (int64_t)n * a.qkv.stride_b + (int64_t)t * a.qkv.stride_t + seg_ch(seg) +
                                           8 * ck);
  };
  uint4 nxv = make_uint4(0u, 0u, 0u, 0u);
  auto gates = [&](int t, float& da, float& db, float& z) {
    const int64_t drow = (int64_t)n * a.decay.stride_b + (int64_t)t * a.decay.stride_t;
    da = load_any(a.decay.data, drow + (int64_t)h * a.decay.stride_h, a.decay.dtype);
    db = load_any(a.decay.data, drow + (int64_t)(a.hv + h) * a.decay.stride_h, a.decay.dtype);
    z = low ? load_any(a.gate.data, (int64_t)n * a.gate.stride_b + (int64_t)t * a.gate.stride_t +
                                        (int64_t)(h * kDim + c) * a.gate.stride_h,
                       a.gate.dtype)
            : 0.f;
  };
  float nxa = 0.f, nxb = 0.f, nda, ndb, nz;
  if (a.vec_x) {
    if (tid < 48) nxv = x_vec(0);
  } else {
    x_ab(0, nxa, nxb);
  }
  gates(0, nda, ndb, nz);

  for (int t = 0; t < a.seqlen; ++t) {
    // ---- conv + SiLU of this token's channels
    float xa = nxa, xb = nxb;
    const float da = nda, db = ndb, zt = nz;
    if (a.vec_x) {  // stage the row (every reader of the previous row has passed a barrier since)
      if (tid < 48) *reinterpret_cast<uint4*>(&sh_x[8 * tid]) = nxv;
      if (t + 1 < a.seqlen && tid < 48) nxv = x_vec(t + 1);
      __syncthreads();
      xa = __bfloat162float(sh_x[(low ? kDim : 0) + c]);
      xb = low ? __bfloat162float(sh_x[2 * kDim + c]) : 0.f;
    }
    if (t + 1 < a.seqlen) {
      if (!a.vec_x) x_ab(t + 1, nxa, nxb);
      gates(t + 1, nda, ndb, nz);
    }
    float ya = xa, yb = xb;
    if (conv) {
      ya = wa[KMAX - 1] * xa;
      yb = wb[KMAX - 1] * xb;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        ya = fmaf(wa[i], ha[i], ya);
        yb = fmaf(wb[i], hb[i], yb);
      }
#pragma unroll
      for (int i = 0; i + 1 < H; ++i) {
        ha[i] = ha[i + 1];
        hb[i] = hb[i + 1];
      }
      if (H > 0) {
        ha[H - 1] = xa;
        hb[H - 1] = xb;
      }
    }
    ya = silu_exact(ya);
    yb = silu_exact(yb);
    // ---- q / k L2 norm per head (k: warps 0-3, q: warps 4-7), then q's scale
    if (a.l2mode != 0) {
      const float ss = warp_sum(ya * ya);
      if (lane == 0) sh_norm[warp >> 2][warp & 3] = ss;
      __syncthreads();
      const int which = low ? 0 : 1;
      const float tot = sh_norm[which][0] + sh_norm[which][1] + sh_norm[which][2] + sh_norm[which][3];
      ya = a.l2mode == 1 ? ya / fmaxf(sqrtf(tot), a.l2_eps) : ya * rsqrtf(tot + a.l2_eps);
    }
    if (low) {
      sh_k[c] = ya;
      sh_v[c] = yb;
    } else {
      sh_q[c] = ya * a.scale;
    }
    // ---- gating (every thread computes the two scalars)
    const float xg = da + dt_bias_h;
    const float sp = xg > 20.f ? xg : log1pf(expf(xg));
    const float gam = expf(-expf(a_log_h) * sp);
    const float bet = 1.f / (1.f + expf(-db));
    __syncthreads();
    // ---- the recurrence step (gdn_decode.cu's register form); o into sh_o
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
      if (low) {
        float kv = 0.f, qv = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          kv += red[0][w][c];
          qv += red[1][w][c];
        }
        const float u = (sh_v[c] - kv) * bet;
        sh_u[c] = u;
        sh_o[c] = fmaf(sh_kq, u, qv);
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
        const int cc = warp + kWarps * i;  // value column of this register row
        s[i].x *= gam; s[i].y *= gam; s[i].z *= gam; s[i].w *= gam;
        const float pk = warp_sum(s[i].x * k4.x + s[i].y * k4.y + s[i].z * k4.z + s[i].w * k4.w);
        const float pq = warp_sum(s[i].x * q4.x + s[i].y * q4.y + s[i].z * q4.z + s[i].w * q4.w);
        const float u = (sh_v[cc] - pk) * bet;
        s[i].x = fmaf(k4.x, u, s[i].x); s[i].y = fmaf(k4.y, u, s[i].y);
        s[i].z = fmaf(k4.z, u, s[i].z); s[i].w = fmaf(k4.w, u, s[i].w);
        if (lane == 0) sh_o[cc] = fmaf(kq, u, pq);
      }
      __syncthreads();
    }
    // ---- output RMSNorm * o_norm * SiLU(gate) over the head's 128 values (warps 0-3)
    float o = 0.f;
    if (low) {
      o = sh_o[c];
      const float ss = warp_sum(o * o);
      if (lane == 0) sh_osq[warp] = ss;
    }
    __syncthreads();
    if (low) {
      const float ms = (sh_osq[0] + sh_osq[1] + sh_osq[2] + sh_osq[3]) * (1.f / kDim);
      const float y = o * rsqrtf(ms + a.norm_eps) * wo * silu_exact(zt);
      store_any(a.out.data, (int64_t)n * a.out.stride_b + (int64_t)t * a.out.stride_t + (int64_t)h * a.out.stride_h + c,
                a.out.dtype, y);
    }
    // the next token rewrites sh_k / sh_q / sh_v / sh_o only after its own first barrier,
    // which every thread reaches after finishing this token
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) st_f4_stream(S + (int64_t)(warp + kWarps * i) * kDim + 4 * lane, s[i]);

  // ---- the new tail: the last width - 1 inputs (history slots H - (K - 1) .. H - 1). The
  // cluster barrier sits here, after every read of the old tail has been consumed.
  if (conv && a.new_tail.data != nullptr) {
    if (a.cluster_sync) {
      cluster_arrive();
      cluster_wait();  // every CTA of the cluster has read the old tail
    }
    uint32_t rank = 0;
    if (a.cluster_sync) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    // q and k channels: the cluster's first CTA (or, without a cluster, the CTA whose value
    // head is the first of its key head); v channels: every CTA
    const bool lead = a.cluster_sync ? rank == 0 : (h % ratio) == 0;
    if (a.vec_tail) {  // through shared memory, 16-byte stores (sh_tail's last reads were long ago)
#pragma unroll
      for (int i = 0; i < H; ++i) {
        if (i < KMAX - K) continue;
        sh_tail[i][(low ? kDim : 0) + c] = __float2bfloat16_rn(ha[i]);
        if (low) sh_tail[i][2 * kDim + c] = __float2bfloat16_rn(hb[i]);
      }
      __syncthreads();
      __nv_bfloat16* nb = const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(a.new_tail.data));
      for (int e = tid; e < (K - 1) * 48; e += kThreads) {
        const int r = e / 48, rem = e - r * 48, seg = rem >> 4, ck = rem & 15;
        if (seg < 2 && !lead) continue;
        *reinterpret_cast<uint4*>(nb + (int64_t)n * a.new_tail.stride_b + (int64_t)r * a.new_tail.stride_t +
                                  seg_ch(seg) + 8 * ck) =
            *reinterpret_cast<const uint4*>(&sh_tail[r + (KMAX - K)][seg * kDim + 8 * ck]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const int r = i - (KMAX - K);
        if (r < 0) continue;
        const int64_t base = (int64_t)n * a.new_tail.stride_b + (int64_t)r * a.new_tail.stride_t;
        if (lead) store_any(a.new_tail.data, base + (int64_t)ch_a * a.new_tail.stride_h, a.new_tail.dtype, ha[i]);
        if (low) store_any(a.new_tail.data, base + (int64_t)ch_b * a.new_tail.stride_h, a.new_tail.dtype, hb[i]);
      }
    }
  }
}

template <int LAYOUT, int KMAX>
cudaError_t launch(const DecodeLayerArgs& a, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((int64_t)a.batch * a.hv));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (a.cluster_sync) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)(a.hv / a.hk);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, gdn_decode_layer_kernel<LAYOUT, KMAX>, a);
}

}  // namespace

cudaError_t launch_gdn_decode_layer(const pbk_gdn_layer_desc& d, cudaStream_t st) {
  DecodeLayerArgs a;
  a.batch = d.batch;
  a.seqlen = d.seqlen;
  a.hk = d.hk;
  a.hv = d.hv;
  a.width = d.conv_weight != nullptr ? d.width : 1;
  a.l2mode = d.l2mode;
  a.l2_eps = d.l2_eps;
  a.norm_eps = d.norm_eps;
  a.scale = d.scale;
  a.qkv = d.qkv;
  a.tail = d.tail;
  a.new_tail = d.new_tail;
  a.decay = d.decay;
  a.gate = d.gate;
  a.out = d.out;
  a.conv_weight = d.conv_weight;
  a.a_log = d.a_log;
  a.dt_bias = d.dt_bias;
  a.o_norm = d.o_norm;
  a.o_norm_dtype = d.o_norm_dtype;
  a.state = d.state;
  a.state_slot_stride = d.state_slot_stride;
  a.state_indices = d.state_indices;
  // a cluster only where CTAs share tail channels that are rewritten in place
  a.cluster_sync = (d.conv_weight != nullptr && d.width > 1 && d.new_tail.data != nullptr &&
                    d.new_tail.data == d.tail.data && d.hv / d.hk > 1)
                       ? 1
                       : 0;
  auto rows16 = [](const pbk_view& v) {  // bf16 rows of contiguous channels, 16-byte aligned
    return v.data != nullptr && v.dtype == PBK_BF16 && v.stride_h == 1 && v.stride_t % 8 == 0 &&
           v.stride_b % 8 == 0 && (reinterpret_cast<uintptr_t>(v.data) & 15) == 0;
  };
  a.vec_tail = rows16(d.tail) && (d.new_tail.data == nullptr || rows16(d.new_tail)) ? 1 : 0;
  a.vec_x = rows16(d.qkv) ? 1 : 0;
  const bool narrow = a.width <= 4;
  if (d.state_layout == PBK_STATE_KV)
    return narrow ? launch<PBK_STATE_KV, 4>(a, st) : launch<PBK_STATE_KV, 8>(a, st);
  return narrow ? launch<PBK_STATE_VK, 4>(a, st) : launch<PBK_STATE_VK, 8>(a, st);
}

}  // namespace pbk
