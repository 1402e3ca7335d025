// Per-token Quest scores, exact per-token rescoring and per-row ranks: the data-parallel
// parts of the serving path's per-token selector (pb27_vllm/memory.py:1009-1294). The
// selector scores every block for every query token separately (the maximum runs over the
// token's query heads of a key head only, :1080-1086), standardises each token's scores,
// and ranks them (_ranks, :881-885).
#include <cfloat>

#include "common.cuh"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 raw, float* out) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(p[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------------
// Per-token block scores (memory.py:1079-1086, 1094-1098): out[kv][t][j] = max over the key
// head's query heads g of sum_d q_{t,g,d} * (q > 0 ? kmax : kmin)_{b,d}, b = cand[kv][j] (or
// j), summed over d = 0 .. D - 1 in order; -inf for b >= full and for b in the hole. Thread =
// candidate; the rows of kTokRows / groups tokens sit in shared memory as fp32.
// ---------------------------------------------------------------------------------
constexpr int kTokThreads = 128;
constexpr int kTokRows = 32;  // query rows (token x head) per pass

template <int D>
__global__ void __launch_bounds__(kTokThreads) quest_token_score_kernel(const pbk_token_desc d) {
  __shared__ __align__(16) float qs[kTokRows][D];
  const int h = blockIdx.y, groups = d.h / d.kv;
  const int tpb = max(1, kTokRows / groups);  // tokens per pass
  const int t0 = blockIdx.z * tpb, nt = min(tpb, d.t - t0);
  const int rows = nt * groups;
  for (int e = threadIdx.x; e < rows * D; e += kTokThreads) {
    const int r = e / D, dd = e % D, ti = t0 + r / groups, g = r % groups;
    const bf16* qp = reinterpret_cast<const bf16*>(d.q) + ti * d.q_stride_t + (int64_t)(h * groups + g) * d.q_stride_h;
    qs[r][dd] = (d.rope_mask && dd < D / 4) ? 0.f : __bfloat162float(qp[dd]);
  }
  __syncthreads();
  const int j = blockIdx.x * kTokThreads + threadIdx.x;
  if (j >= d.n_pool) return;
  const int b = d.cand != nullptr ? d.cand[h * d.cand_stride_kv + j] : j;
  const bool masked = b < 0 || b >= d.full || (b >= d.hole_lo && b < d.hole_hi);
  const int bc = min(max(b, 0), d.full - 1);
  const bf16* bmax = reinterpret_cast<const bf16*>(d.kmax) + h * d.bnd_stride_kv + (int64_t)bc * d.bnd_stride_p;
  const bf16* bmin = reinterpret_cast<const bf16*>(d.kmin) + h * d.bnd_stride_kv + (int64_t)bc * d.bnd_stride_p;
  float acc[kTokRows];
#pragma unroll
  for (int r = 0; r < kTokRows; ++r) acc[r] = 0.f;
  for (int d0 = 0; d0 < D; d0 += 8) {
    float mx[8], mn[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmax + d0), mx);
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmin + d0), mn);
#pragma unroll
    for (int r = 0; r < kTokRows; ++r) {
      if (r < rows) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float qv = qs[r][d0 + jj];
          acc[r] = fmaf(qv, qv > 0.f ? mx[jj] : mn[jj], acc[r]);
        }
      }
    }
  }
  float* out = d.out + h * d.out_stride_kv + j;
  float best = -INFINITY;
#pragma unroll
  for (int r = 0; r < kTokRows; ++r) {  // rows are (token, head): the max runs over each token's heads
    if (r < rows) {
      best = fmaxf(best, acc[r]);
      if ((r + 1) % groups == 0) {
        out[(int64_t)(t0 + r / groups) * d.out_stride_t] = masked ? -INFINITY : best;
        best = -INFINITY;
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Per-token exact rescoring (memory.py:1192-1202): out[kv][t][j] = max over the key head's
// query heads and the block's tokens of q.k in fp32, block b = cand[kv][j] (or j) of keys.
// CTA = (8 candidates, key head, tokens of one pass); warp = candidate, lane = tokens lane,
// lane + 32, ...
// ---------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) quest_token_rerank_kernel(const pbk_token_desc d) {
  __shared__ __align__(16) float qs[kTokRows][D];
  const int h = blockIdx.y, groups = d.h / d.kv, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tpb = max(1, kTokRows / groups);
  const int t0 = blockIdx.z * tpb, nt = min(tpb, d.t - t0);
  const int rows = nt * groups;
  for (int e = threadIdx.x; e < rows * D; e += blockDim.x) {
    const int r = e / D, dd = e % D, ti = t0 + r / groups, g = r % groups;
    qs[r][dd] = __bfloat162float(reinterpret_cast<const bf16*>(d.q)[ti * d.q_stride_t +
                                                                     (int64_t)(h * groups + g) * d.q_stride_h + dd]);
  }
  __syncthreads();
  const int j = blockIdx.x * 8 + warp;
  if (j >= d.n_pool) return;
  const int b = d.cand != nullptr ? d.cand[h * d.cand_stride_kv + j] : j;
  const bf16* base = reinterpret_cast<const bf16*>(d.keys) + h * d.key_stride_kv + (int64_t)b * d.block * d.key_stride_n;
  float best[kTokRows];
#pragma unroll
  for (int r = 0; r < kTokRows; ++r) best[r] = -INFINITY;
  for (int s = lane; s < d.block; s += 32) {
    const bf16* kr = base + (int64_t)s * d.key_stride_n;
    float acc[kTokRows];
#pragma unroll
    for (int r = 0; r < kTokRows; ++r) acc[r] = 0.f;
#pragma unroll 1
    for (int h0 = 0; h0 < D; h0 += 64) {  // 64 dims (8 loads) of the key in flight, dims in order
      uint4 raw[8];
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) raw[c8] = *reinterpret_cast<const uint4*>(kr + h0 + 8 * c8);
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
      const int d0 = h0 + 8 * c8;
      float kf[8];
      bf16x8_to_f32(raw[c8], kf);
#pragma unroll
      for (int r = 0; r < kTokRows; ++r) {
        if (r < rows) {
          const float4 qa = *reinterpret_cast<const float4*>(&qs[r][d0]);
          const float4 qb = *reinterpret_cast<const float4*>(&qs[r][d0 + 4]);
          float a = acc[r];
          a = fmaf(qa.x, kf[0], a);
          a = fmaf(qa.y, kf[1], a);
          a = fmaf(qa.z, kf[2], a);
          a = fmaf(qa.w, kf[3], a);
          a = fmaf(qb.x, kf[4], a);
          a = fmaf(qb.y, kf[5], a);
          a = fmaf(qb.z, kf[6], a);
          a = fmaf(qb.w, kf[7], a);
          acc[r] = a;
        }
      }
      }
    }
#pragma unroll
    for (int r = 0; r < kTokRows; ++r) best[r] = fmaxf(best[r], acc[r]);
  }
  float* out = d.out + h * d.out_stride_kv + j;
#pragma unroll
  for (int r = 0; r < kTokRows; ++r) {
    if (r < rows) {
      float m = best[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      best[r] = m;
    }
  }
  if (lane == 0) {
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < kTokRows; ++r) {
      if (r < rows) {
        m = fmaxf(m, best[r]);
        if ((r + 1) % groups == 0) {
          out[(int64_t)(t0 + r / groups) * d.out_stride_t] = m;
          m = -INFINITY;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Ranks along a row (_ranks, memory.py:881-885): ranks[i] = position of x[i] in the row
// sorted descending, ties in index order. One CTA per row: a bitonic sort of (descending
// order key << 32 | index) in shared memory, padded to a power of two with keys that sort
// last.
// ---------------------------------------------------------------------------------
constexpr int kRankThreads = 1024;

__global__ void __launch_bounds__(kRankThreads) quest_row_rank_kernel(const float* x, int64_t x_stride, int n,
                                                                     int npow2, int32_t* ranks, int64_t r_stride) {
  extern __shared__ unsigned long long keys[];
  const float* row = x + blockIdx.x * x_stride;
  for (int i = threadIdx.x; i < npow2; i += kRankThreads)
    keys[i] = i < n ? ((unsigned long long)(~ordered_key(row[i])) << 32) | (unsigned)i : ~0ull;
  __syncthreads();
  for (int k = 2; k <= npow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < npow2; i += kRankThreads) {
        const int p = i ^ j;
        if (p > i) {
          const unsigned long long a = keys[i], b = keys[p];
          if ((a > b) == ((i & k) == 0)) {
            keys[i] = b;
            keys[p] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  int32_t* out = ranks + blockIdx.x * r_stride;
  for (int i = threadIdx.x; i < npow2; i += kRankThreads) {
    const unsigned idx = (unsigned)(keys[i] & 0xffffffffu);
    if (idx < (unsigned)n) out[idx] = i;
  }
}

int tokens_per_pass(const pbk_token_desc& d) { return max(1, kTokRows / (d.h / d.kv)); }

}  // namespace

cudaError_t launch_quest_token_scores(const pbk_token_desc& d, cudaStream_t st) {
  const int tpb = tokens_per_pass(d);
  const dim3 grid((unsigned)((d.n_pool + kTokThreads - 1) / kTokThreads), (unsigned)d.kv,
                  (unsigned)((d.t + tpb - 1) / tpb));
  if (d.d == 256) quest_token_score_kernel<256><<<grid, kTokThreads, 0, st>>>(d);
  else quest_token_score_kernel<128><<<grid, kTokThreads, 0, st>>>(d);
  return cudaGetLastError();
}

cudaError_t launch_quest_token_rerank(const pbk_token_desc& d, cudaStream_t st) {
  const int tpb = tokens_per_pass(d);
  const dim3 grid((unsigned)((d.n_pool + 7) / 8), (unsigned)d.kv, (unsigned)((d.t + tpb - 1) / tpb));
  if (d.d == 256) quest_token_rerank_kernel<256><<<grid, 256, 0, st>>>(d);
  else quest_token_rerank_kernel<128><<<grid, 256, 0, st>>>(d);
  return cudaGetLastError();
}

cudaError_t launch_quest_row_ranks(const float* x, int64_t x_stride, int rows, int n, int32_t* ranks,
                                   int64_t r_stride, cudaStream_t st) {
  int npow2 = 1;
  while (npow2 < n) npow2 <<= 1;
  const size_t smem = (size_t)npow2 * sizeof(unsigned long long);
  cudaError_t e = cudaFuncSetAttribute(quest_row_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  quest_row_rank_kernel<<<rows, kRankThreads, smem, st>>>(x, x_stride, n, npow2, ranks, r_stride);
  return cudaGetLastError();
}

}  // namespace pbk
