// Chunked gated delta rule on the 5th-generation tensor cores: bf16 operands, fp32 TMEM
// accumulators, fp32 state resident in TMEM for the whole sequence.
//
// Algorithm (pseudobrain/gated_deltanet.py:110-165), chunk C = 64, c = cumsum(g),
// gamma_t = exp(c_t), e_t = exp(c_C - c_t), D_ti = exp(c_t - c_i):
//   A = strict_lower(beta_t K K^T * D),  T = (I + A)^-1 (fp32)
//   W = T diag(beta gamma) K,  U' = T diag(beta) V
//   U = U' - W S;  O = diag(gamma scale) Q S + (scale Q K^T * D) U;  S <- gamma_C S + (diag(e) K)^T U
// Every product is one M=128 tcgen05.mma chain with the value dim (or the stacked K|Q
// rows) as M, so TMEM lane j of the CTA's 128 threads is "column j":
//   [K;Q] K^T  -> TMEM D1 (lanes 0-63 K K^T rows, 64-127 Q K^T rows)       K = dk
//   W^T  = K^T (T diag(beta gamma))^T -> TMEM D1        (A MN-major)      K = i
//   U'^T = V^T (T diag(beta))^T       -> TMEM UP        (A MN-major)      K = i
//   (WS)^T = S^T W^T -> TMEM WS;  (QS)^T = S^T Q^T -> TMEM QS               K = dk
//   (UM)^T = U^T M^T -> TMEM UM;  S^T += U^T (diag(e) K) -> TMEM S           K = i
// S^T (fp32, 128 TMEM columns) is loaded from h0 once, scaled by gamma_C through the
// register file each chunk (which also writes its bf16 copy, the A operand of the S
// products) and accumulated by the last MMA; it goes back to HBM once at the end.
//
// One CTA (128 threads, thread j <-> TMEM lane j) per (sequence, value head) chain walks
// its chunks in order; thread 0 issues TMA loads and MMAs. The chunk-local preparation of
// chunk n+1 (K K^T, the inverse, W, U') is interleaved with the tensor-core work of chunk
// n. q/k/v arrive by 4-D TMA ([B,T,H,128] with any strides; rows past T are zero-filled,
// the reference's identity padding); no multicast. Every mbarrier wait is bounded: on
// timeout the kernel records an error code, waits (bounded) for its own loads and MMAs,
// frees its TMEM and returns.
#include "common.cuh"
#include "tc.cuh"
#include "tma_host.h"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int C = 64;
constexpr int D = 128;
constexpr int NT = 128;
constexpr int PA = C + 4;  // fp32 row stride of A: 16-byte rows, conflict-free float4 row writes

// TMEM columns
constexpr uint32_t kColS = 0, kColD1 = 128, kColUP = 192, kColWS = 256, kColQS = 320, kColUM = 384;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) PrefillSmem {
  uint8_t kq[2][2][16384];   // [buf][dk atom][rows 0-63 K, 64-127 Q] x 64 bf16, SW128
  uint8_t v[2][8192];        // [dv atom][64 rows] x 64 bf16, SW128
  uint8_t st[2][16384];      // S^T bf16 [128 dv rows] x [dk atom] (A operand, K-major)
  uint8_t wt[16384];         // W^T bf16 [128 dk rows x 64 t] (B operand, MN-major)
  uint8_t m[2][8192];        // M bf16 [64 t x 64 i] (B operand, K-major)
  uint8_t tb[8192];          // T diag(beta) bf16 [64 t x 64 i]
  uint8_t tbg[8192];         // T diag(beta gamma) bf16 [64 t x 64 i]
  uint8_t ut[16384];         // U^T bf16 [128 dv rows x 64 t] (A operand, K-major)
  float a[C * PA];           // A fp32
  float cum[2][C], cum2[2][C], gam[2][C], ee[2][C], beta[2][C];
  uint64_t bar_kq[2], bar_v, bar_p1, bar_p3, bar_ws, bar_o, bar_s, bar_drain;
  uint32_t tmem_base;
};

struct PrefillArgs {
  int batch, seqlen, hk, hv;
  const void* g;
  int64_t g_sb, g_st, g_sh;
  int g_dtype;
  const void* beta;
  int64_t b_sb, b_st, b_sh;
  int b_dtype;
  void* o;
  int64_t o_sb, o_st, o_sh;
  const float* h0;
  float* state;
  int64_t slot_stride;
  int layout;
  const int32_t* state_indices;
  float scale;
  int* err;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Write 64 fp32 values as one 128-byte bf16 row of a 128B-swizzled tile.
__device__ __forceinline__ void store_row_bf16(uint8_t* tile, int row, const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    w.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    w.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    w.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, 8 * c)) = w;
  }
}

// 64 TMEM columns of this thread's lane into v[64].
__device__ __forceinline__ void tmem_row64(uint32_t taddr, float* v) {
  uint32_t r[32];
  tc::tmem_ld_32x32(taddr, r);
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  tc::tmem_ld_32x32(taddr + 32, r);
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(r[i]);
}

template <typename TOut>
__global__ void __launch_bounds__(NT, 1)
    gdn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const PrefillArgs p) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5;
  const int b = blockIdx.x / p.hv, h = blockIdx.x % p.hv;
  const int hk = h / (p.hv / p.hk);
  int64_t slot = b;
  if (p.state_indices != nullptr) {
    slot = p.state_indices[b];
    if (slot < 0) return;  // padding slot (uniform for the CTA)
  }
  const int nchunks = (p.seqlen + C - 1) / C;

  if (tid == 0) {
    tc::mbar_init(&sm.bar_kq[0], 1);
    tc::mbar_init(&sm.bar_kq[1], 1);
    tc::mbar_init(&sm.bar_v, 1);
    tc::mbar_init(&sm.bar_p1, 1);
    tc::mbar_init(&sm.bar_p3, 1);
    tc::mbar_init(&sm.bar_ws, 1);
    tc::mbar_init(&sm.bar_o, 1);
    tc::mbar_init(&sm.bar_s, 1);
    tc::mbar_init(&sm.bar_drain, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tm_q);
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
  }
  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);  // this thread's TMEM lane (row tid)

  // ------------------------------------------------------------ helpers
  auto issue_kq = [&](int n) {
    const int buf = n & 1;
    tc::mbar_expect_tx(&sm.bar_kq[buf], 4 * 8192);
    for (int a = 0; a < 2; ++a) {
      tc::tma_load_4d(sm.kq[buf][a], &tm_k, &sm.bar_kq[buf], 64 * a, n * C, hk, b);
      tc::tma_load_4d(sm.kq[buf][a] + 8192, &tm_q, &sm.bar_kq[buf], 64 * a, n * C, hk, b);
    }
  };
  auto issue_v = [&](int n) {
    tc::mbar_expect_tx(&sm.bar_v, 2 * 8192);
    for (int a = 0; a < 2; ++a) tc::tma_load_4d(sm.v[a], &tm_v, &sm.bar_v, 64 * a, n * C, h, b);
  };
  // Chunk scalars: cumulative log decay, gamma, e, beta (identity steps past the end).
  auto load_scalars = [&](int n) {
    const int buf = n & 1;
    if (tid < C) {
      const int t = n * C + tid;
      float gv = 0.f, bv = 0.f;
      if (t < p.seqlen) {
        gv = load_any(p.g, b * p.g_sb + (int64_t)t * p.g_st + h * p.g_sh, p.g_dtype);
        bv = load_any(p.beta, b * p.b_sb + (int64_t)t * p.b_st + h * p.b_sh, p.b_dtype);
      }
      float x = gv;  // inclusive scan over the 64 steps: warp scan, then carry
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if ((tid & 31) >= o) x += y;
      }
      sm.cum[buf][tid] = x;
      sm.beta[buf][tid] = bv;
    }
    __syncthreads();
    if (tid >= 32 && tid < C) sm.cum[buf][tid] += sm.cum[buf][31];
    __syncthreads();
    if (tid < C) {
      const float c = sm.cum[buf][tid];
      sm.gam[buf][tid] = expf(c);
      sm.ee[buf][tid] = expf(sm.cum[buf][C - 1] - c);
      sm.cum2[buf][tid] = c * 1.4426950408889634f;  // log2(e) c, for exp2 of differences
    }
  };

  int failed = 0;
  // Bounded wait by every thread; the outcome is made uniform across the CTA.
  auto wait_all = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    const bool ok = tc::mbar_wait(bar, parity);
    if (!__syncthreads_and(ok)) {
      if (tid == 0 && p.err) atomicCAS(p.err, 0, 200 + site);
      failed = 1;
      return false;
    }
    tc::fence_after_sync();
    return true;
  };
  // Last chunk whose K/Q (per buffer) and V load thread 0 issued, for a bounded drain on
  // failure. Barrier parities follow from chunk indices: buffer n&1 holds the (n>>1)-th
  // load of that buffer; V, P1 and P3 of chunk n are their barriers' n-th completions.
  int last_kq[2] = {-1, -1}, last_v = -1;

  const uint32_t i_kk = tc::idesc_bf16_f32(128, 64, false, false);   // A K-major, B K-major, N=64
  const uint32_t i_kmn = tc::idesc_bf16_f32(128, 64, false, true);   // A K-major, B MN-major, N=64
  const uint32_t i_mnk = tc::idesc_bf16_f32(128, 64, true, false);   // A MN-major, B K-major, N=64
  const uint32_t i_s = tc::idesc_bf16_f32(128, 128, false, true);    // S update, N=128

  // Prep MMAs of chunk n (thread 0): [K;Q] K^T -> D1.
  auto mma_p1 = [&](int n) {
    const int buf = n & 1;
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t base = tc::smem_u32(sm.kq[buf][kk >> 2]) + (kk & 3) * 32;
      tc::mma_f16(tmem + kColD1, tc::sdesc_sw128(base, 16, 1024), tc::sdesc_sw128(base, 16, 1024), i_kk, kk != 0);
    }
    tc::mma_commit(&sm.bar_p1);
  };
  // W^T = K^T TBG^T -> D1;  U'^T = V^T TB^T -> UP.
  auto mma_p3 = [&](int n) {
    const int buf = n & 1;
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][0]) + kk * 2048, 16384, 1024);
      const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sm.tbg) + kk * 32, 16, 1024);
      tc::mma_f16(tmem + kColD1, ad, bd, i_mnk, kk != 0);
    }
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.v[0]) + kk * 2048, 8192, 1024);
      const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sm.tb) + kk * 32, 16, 1024);
      tc::mma_f16(tmem + kColUP, ad, bd, i_mnk, kk != 0);
    }
    tc::mma_commit(&sm.bar_p3);
  };

  // P1 epilogue of chunk n: A (fp32) from K K^T rows, M (bf16) from Q K^T rows.
  auto p1_epilogue = [&](int n) {
    const int buf = n & 1;
    float v[64];
    tmem_row64(lane_addr + kColD1, v);
    const float* c2 = sm.cum2[buf];
    if (tid < C) {
      const int t = tid;
      const float bt = sm.beta[buf][t], ct = c2[t];
#pragma unroll
      for (int i = 0; i < C; i += 4) {
        float4 w;
        w.x = i + 0 < t ? bt * v[i + 0] * exp2f(ct - c2[i + 0]) : 0.f;
        w.y = i + 1 < t ? bt * v[i + 1] * exp2f(ct - c2[i + 1]) : 0.f;
        w.z = i + 2 < t ? bt * v[i + 2] * exp2f(ct - c2[i + 2]) : 0.f;
        w.w = i + 3 < t ? bt * v[i + 3] * exp2f(ct - c2[i + 3]) : 0.f;
        *reinterpret_cast<float4*>(&sm.a[t * PA + i]) = w;
      }
    } else {
      const int t = tid - C;
      const float ct = c2[t];
#pragma unroll
      for (int i = 0; i < C; ++i) v[i] = i <= t ? p.scale * v[i] * exp2f(ct - c2[i]) : 0.f;
      store_row_bf16(sm.m[buf], t, v);
    }
  };

  // T = (I + A)^-1 by forward substitution, one column of T per thread in registers
  // (threads 0..63; rows of A are shared-memory broadcasts): x_i = -sum_{m<i} A_im x_m
  // for i > col, x_col = 1, x_i = 0 above. Then TB = T diag(beta), TBG = T diag(beta gamma)
  // as bf16 [t][i] tiles.
  auto inverse = [&](int n) {
    const int buf = n & 1;
    if (tid < C) {
      const int col = tid;
      float x[C];
#pragma unroll
      for (int i = 0; i < C; ++i) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int m = 0; m + 3 < i; m += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(&sm.a[i * PA + m]);
          s0 = fmaf(a4.x, x[m], s0);
          s1 = fmaf(a4.y, x[m + 1], s1);
          s0 = fmaf(a4.z, x[m + 2], s0);
          s1 = fmaf(a4.w, x[m + 3], s1);
        }
#pragma unroll
        for (int m = i & ~3; m < i; ++m) s0 = fmaf(sm.a[i * PA + m], x[m], s0);
        x[i] = i < col ? 0.f : (i == col ? 1.f : -(s0 + s1));
      }
      const float bc = sm.beta[buf][col], bgc = bc * sm.gam[buf][col];
#pragma unroll
      for (int t = 0; t < C; ++t) {
        const uint32_t off = tc::sw128_offset(t, col);
        *reinterpret_cast<bf16*>(sm.tb + off) = __float2bfloat16_rn(x[t] * bc);
        *reinterpret_cast<bf16*>(sm.tbg + off) = __float2bfloat16_rn(x[t] * bgc);
      }
    }
  };

  // W^T (TMEM D1, lane = dk) -> wt smem; then scale the chunk's K rows by e_i in place
  // (the K operand of the state update).
  auto w_epilogue = [&](int n) {
    const int buf = n & 1;
    float v[64];
    tmem_row64(lane_addr + kColD1, v);
    store_row_bf16(sm.wt, tid, v);
    const int i = tid >> 1, a = tid & 1;
    const float e = sm.ee[buf][i];
    uint8_t* row = sm.kq[buf][a] + i * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 w = *reinterpret_cast<uint4*>(row + 16 * c);
      __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h2[j]);
        h2[j] = __floats2bfloat162_rn(f.x * e, f.y * e);
      }
      *reinterpret_cast<uint4*>(row + 16 * c) = w;
    }
  };

  // ------------------------------------------------------------ state in
  {
    const float* h0 = p.h0 != nullptr ? p.h0 + slot * p.slot_stride + (int64_t)h * D * D : nullptr;
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x = 0.f;
        if (h0 != nullptr) x = p.layout == PBK_STATE_KV ? h0[(c0 + i) * D + tid] : h0[tid * D + c0 + i];
        r[i] = __float_as_uint(x);
      }
      tc::tmem_st_32x32(lane_addr + kColS + c0, r);
    }
    tc::tmem_st_wait();
  }

  // ------------------------------------------------------------ prologue: prep of chunk 0
  if (tid == 0) {
    issue_kq(0);
    last_kq[0] = 0;
    if (nchunks > 1) { issue_kq(1); last_kq[1] = 1; }
    issue_v(0);
    last_v = 0;
  }
  load_scalars(0);
  if (wait_all(&sm.bar_kq[0], 0, 1)) {
    if (tid == 0) mma_p1(0);
  }
  if (!failed && wait_all(&sm.bar_p1, 0, 2)) {
    p1_epilogue(0);
    __syncthreads();
    inverse(0);
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (wait_all(&sm.bar_v, 0, 3)) {
      if (tid == 0) mma_p3(0);
      if (wait_all(&sm.bar_p3, 0, 4)) {
        w_epilogue(0);
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (tid == 0 && nchunks > 1) { issue_v(1); last_v = 1; }
      }
    }
  }

  // ------------------------------------------------------------ chunk loop
  TOut* out = reinterpret_cast<TOut*>(p.o) + b * p.o_sb + h * p.o_sh + tid;
  for (int n = 0; n < nchunks && !failed; ++n) {
    const int buf = n & 1;
    const uint32_t par = n & 1;
    const bool more = n + 1 < nchunks;
    // (1) S^T -> bf16 A operand; S^T *= gamma_C in TMEM
    {
      const float gl = sm.gam[buf][C - 1];
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32(lane_addr + kColS + c0, r);
        tc::tmem_ld_wait();
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(r[i]);
        uint8_t* tile = sm.st[c0 >> 6];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 w;
          w.x = pack_bf16x2(f[8 * c + 0], f[8 * c + 1]);
          w.y = pack_bf16x2(f[8 * c + 2], f[8 * c + 3]);
          w.z = pack_bf16x2(f[8 * c + 4], f[8 * c + 5]);
          w.w = pack_bf16x2(f[8 * c + 6], f[8 * c + 7]);
          *reinterpret_cast<uint4*>(tile + tc::sw128_offset(tid, (c0 & 63) + 8 * c)) = w;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(f[i] * gl);
        tc::tmem_st_32x32(lane_addr + kColS + c0, r);
      }
      tc::tmem_st_wait();
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // (2) WS^T = S^T W^T, QS^T = S^T Q^T
    if (tid == 0) {
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.st[kk >> 2]) + (kk & 3) * 32, 16, 1024);
        const uint64_t bw = tc::sdesc_sw128(tc::smem_u32(sm.wt) + kk * 2048, 16, 1024);
        tc::mma_f16(tmem + kColWS, ad, bw, i_kmn, kk != 0);
      }
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.st[kk >> 2]) + (kk & 3) * 32, 16, 1024);
        const uint64_t bq = tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][kk >> 2]) + 8192 + (kk & 3) * 32, 16, 1024);
        tc::mma_f16(tmem + kColQS, ad, bq, i_kk, kk != 0);
      }
      tc::mma_commit(&sm.bar_ws);
    }
    // (3) prep of chunk n+1, part 1: scalars and [K;Q] K^T
    if (more) {
      load_scalars(n + 1);
      if (!wait_all(&sm.bar_kq[buf ^ 1], ((n + 1) >> 1) & 1, 5)) break;
      if (tid == 0) mma_p1(n + 1);
    }
    // (4) U = U' - WS  ->  U^T bf16
    if (!wait_all(&sm.bar_ws, par, 6)) break;
    {
      float ws[64], up[64];
      tmem_row64(lane_addr + kColWS, ws);
      tmem_row64(lane_addr + kColUP, up);
#pragma unroll
      for (int i = 0; i < 64; ++i) up[i] -= ws[i];
      store_row_bf16(sm.ut, tid, up);
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // (5) UM^T = U^T M^T;  S^T += U^T (diag(e) K)
    if (tid == 0) {
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.ut) + kk * 32, 16, 1024);
        const uint64_t bm = tc::sdesc_sw128(tc::smem_u32(sm.m[buf]) + kk * 32, 16, 1024);
        tc::mma_f16(tmem + kColUM, ad, bm, i_kk, kk != 0);
      }
      tc::mma_commit(&sm.bar_o);
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.ut) + kk * 32, 16, 1024);
        const uint64_t bk = tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][0]) + kk * 2048, 16384, 1024);
        tc::mma_f16(tmem + kColS, ad, bk, i_s, 1);
      }
      tc::mma_commit(&sm.bar_s);
    }
    // (6)-(8) prep of chunk n+1: A, M, inverse, W^T and U'^T
    if (more) {
      if (!wait_all(&sm.bar_p1, (n + 1) & 1, 7)) break;
      p1_epilogue(n + 1);
      __syncthreads();
      inverse(n + 1);
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncthreads();
      if (!wait_all(&sm.bar_v, (n + 1) & 1, 8)) break;
      if (tid == 0) mma_p3(n + 1);
    }
    // (9) O = gamma scale QS + UM
    if (!wait_all(&sm.bar_o, par, 9)) break;
    {
      float qs[64], um[64];
      tmem_row64(lane_addr + kColQS, qs);
      tmem_row64(lane_addr + kColUM, um);
      const int tmax = min(C, p.seqlen - n * C);
      const float* gm = sm.gam[buf];
      TOut* oc = out + (int64_t)(n * C) * p.o_st;
#pragma unroll
      for (int t = 0; t < C; ++t)
        if (t < tmax) oc[(int64_t)t * p.o_st] = from_f32<TOut>(fmaf(gm[t] * p.scale, qs[t], um[t]));
    }
    // (10) W^T of chunk n+1 -> smem; K(n+1) rows scaled by e; next V load
    if (more) {
      if (!wait_all(&sm.bar_p3, (n + 1) & 1, 10)) break;
      w_epilogue(n + 1);
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncthreads();
      if (tid == 0 && n + 2 < nchunks) { issue_v(n + 2); last_v = n + 2; }
    }
    // (11) state update done: the chunk's K/Q buffer is free for chunk n+2
    if (!wait_all(&sm.bar_s, par, 11)) break;
    if (tid == 0 && n + 2 < nchunks) { issue_kq(n + 2); last_kq[buf] = n + 2; }
  }

  if (failed) {
    // ------------------------------------------------------------ bounded drain
    if (tid == 0) {
      // Our loads land in the order of their barriers' phases: wait for the last of each.
      for (int bb = 0; bb < 2; ++bb)
        if (last_kq[bb] >= 0) tc::mbar_wait(&sm.bar_kq[bb], (last_kq[bb] >> 1) & 1, 200000000ull);
      if (last_v >= 0) tc::mbar_wait(&sm.bar_v, last_v & 1, 200000000ull);
      // One more commit tracks every MMA this thread issued.
      tc::mma_commit(&sm.bar_drain);
      tc::mbar_wait(&sm.bar_drain, 0, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ state out
    float* st = p.state + slot * p.slot_stride + (int64_t)h * D * D;
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
      tc::tmem_ld_32x32(lane_addr + kColS + c0, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (p.layout == PBK_STATE_KV) st[(c0 + i) * D + tid] = __uint_as_float(r[i]);
        else st[tid * D + c0 + i] = __uint_as_float(r[i]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

constexpr size_t kSmemBytes = sizeof(PrefillSmem) + 1024;

bool make_map(CUtensorMap* m, const pbk_view& v, int heads, const pbk_gdn_desc& d) {
  const uint64_t dims[4] = {128, (uint64_t)d.seqlen, (uint64_t)heads, (uint64_t)d.batch};
  const uint64_t strides[3] = {(uint64_t)v.stride_t * 2, (uint64_t)v.stride_h * 2, (uint64_t)v.stride_b * 2};
  const uint32_t box[4] = {64, 64, 1, 1};
  return make_tmap_bf16_sw128(m, v.data, 4, dims, strides, box);
}

}  // namespace

bool gdn_prefill_tc_supported(const pbk_gdn_desc& d) {
  auto ok16 = [](const pbk_view& v) {
    return (reinterpret_cast<uintptr_t>(v.data) & 15) == 0 && v.stride_t % 8 == 0 && v.stride_h % 8 == 0 &&
           v.stride_b % 8 == 0 && v.stride_t > 0 && v.stride_h > 0 && v.stride_b > 0;
  };
  return d.q.dtype == PBK_BF16 && d.dk == 128 && d.dv == 128 && d.seqlen > 0 && ok16(d.q) && ok16(d.k) &&
         ok16(d.v);
}

cudaError_t launch_gdn_prefill_tc(const pbk_gdn_desc& d, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, d.q, d.hk, d) || !make_map(&mk, d.k, d.hk, d) || !make_map(&mv, d.v, d.hv, d))
    return cudaErrorInvalidValue;
  PrefillArgs a;
  a.batch = d.batch;
  a.seqlen = d.seqlen;
  a.hk = d.hk;
  a.hv = d.hv;
  a.g = d.g.data;
  a.g_sb = d.g.stride_b;
  a.g_st = d.g.stride_t;
  a.g_sh = d.g.stride_h;
  a.g_dtype = d.g.dtype;
  a.beta = d.beta.data;
  a.b_sb = d.beta.stride_b;
  a.b_st = d.beta.stride_t;
  a.b_sh = d.beta.stride_h;
  a.b_dtype = d.beta.dtype;
  a.o = const_cast<void*>(d.o.data);
  a.o_sb = d.o.stride_b;
  a.o_st = d.o.stride_t;
  a.o_sh = d.o.stride_h;
  a.h0 = d.h0;
  a.state = d.state;
  a.slot_stride = d.state_slot_stride;
  a.layout = d.state_layout;
  a.state_indices = d.state_indices;
  a.scale = d.scale;
  a.err = device_error_word();
  const dim3 grid((unsigned)((int64_t)d.batch * d.hv));
  if (d.o.dtype == PBK_BF16) {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_tc_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    gdn_prefill_tc_kernel<bf16><<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_tc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    gdn_prefill_tc_kernel<float><<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, a);
  }
  return cudaGetLastError();
}

}  // namespace pbk
