// Chunked gated delta rule on the 5th-generation tensor cores: bf16 operands, fp32 TMEM
// accumulators, fp32 state resident in TMEM for the whole sequence.
//
// Algorithm (pseudobrain/gated_deltanet.py:110-165), chunk C = 64, c = cumsum(g),
// gamma_t = exp(c_t), e_t = exp(c_C - c_t), D_ti = exp(c_t - c_i):
//   A = strict_lower(beta_t K K^T * D),  T = (I + A)^-1 (fp32)
//   W = T diag(beta gamma) K,  U' = T diag(beta) V
//   U = U' - W S;  O = diag(gamma scale) Q S + (scale Q K^T * D) U;  S <- gamma_C S + (diag(e) K)^T U
// Every product is one M=128 tcgen05.mma chain with the value dim (or the stacked K|Q
// rows) as M, so TMEM lane j is "column j" for the warpgroup that reads it:
//   [K;Q] K^T  -> TMEM D1 (lanes 0-63 K K^T rows, 64-127 Q K^T rows)       K = dk
//   W^T  = K^T (T diag(beta gamma))^T -> TMEM D1        (A MN-major)      K = i
//   U'^T = V^T (T diag(beta))^T       -> TMEM UP[n&1]   (A MN-major)      K = i
//   (WS)^T = S^T W^T -> TMEM WS;  (QS)^T = S^T Q^T -> TMEM QS               K = dk
//   (UM)^T = U^T M^T -> TMEM UM;  S^T += U^T (diag(e) K) -> TMEM S           K = i
//
// One CTA per (sequence, value head) chain, warp-specialised:
//   warps 0-3 (serial): state step of chunk n -- S^T to bf16 and S^T *= gamma_C through
//     the registers, then U = U' - WS, then the outputs; their thread 0 issues the S MMAs.
//   warps 4-7 (prep): chunk n+1's scalars, K K^T, A and M, the inverse (16x16 diagonal
//     blocks by substitution, off-diagonal blocks by tf32 mma.sync products), then W^T and
//     U'^T; their thread 0 issues the prep MMAs.
//   warp 8 (producer): TMA loads of K|Q and V (4-D maps over [B,T,H,128], any strides,
//     rows past T zero-filled = the reference's identity padding; no multicast), and the
//     TMEM allocation.
// The roles meet on mbarriers; every wait is bounded: on timeout the kernel records an
// error code, stops issuing, waits (bounded) for its own loads and MMAs, frees its TMEM
// and returns.
#include "common.cuh"
#include "tc.cuh"
#include "tma_host.h"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int C = 64;
constexpr int D = 128;
constexpr int NT = 288;    // 2 warpgroups + producer warp
constexpr int PA = C + 4;  // fp32 row stride of A (16-byte rows)

// TMEM columns
constexpr uint32_t kColS = 0, kColD1 = 128, kColUP = 192, kColWS = 320, kColQS = 384, kColUM = 448;
constexpr uint32_t kTmemCols = 512;

struct __align__(1024) PrefillSmem {
  uint8_t kq[2][2][16384];   // [buf][dk atom][rows 0-63 K, 64-127 Q] x 64 bf16, SW128
  uint8_t v[2][8192];        // [dv atom][64 rows] x 64 bf16, SW128
  uint8_t st[2][16384];      // S^T bf16 [128 dv rows] x [dk atom] (A operand, K-major)
  uint8_t wt[2][16384];      // [buf] W^T bf16 [128 dk rows x 64 t] (B, MN-major); also T scratch
  uint8_t m[2][8192];        // [buf] M bf16 [64 t x 64 i] (B operand, K-major)
  uint8_t tb[8192];          // T diag(beta) bf16 [64 t x 64 i]; also mma.sync scratch
  uint8_t tbg[8192];         // T diag(beta gamma) bf16 [64 t x 64 i]
  uint8_t ut[16384];         // U^T bf16 [128 dv rows x 64 t] (A operand); also output staging
  float a[C * PA];           // A fp32
  float cum[3][C], cum2[3][C], gam[3][C], ee[3][C], beta[3][C];
  uint64_t bar_kq[2], bar_v, bar_p1, bar_p3, bar_ws, bar_s, prep_ready, drain_s, drain_p;
  uint32_t tmem_base;
  volatile int abort;
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

// 64 TMEM columns of this thread's lane into v[64] (two loads in flight, one wait).
__device__ __forceinline__ void tmem_row64(uint32_t taddr, float* v) {
  uint32_t r0[32], r1[32];
  tc::tmem_ld_32x32(taddr, r0);
  tc::tmem_ld_32x32(taddr + 32, r1);
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __uint_as_float(r0[i]);
    v[32 + i] = __uint_as_float(r1[i]);
  }
}

// Named barrier over one warpgroup (id 1: serial, 2: prep), and its AND-reduction.
__device__ __forceinline__ void wg_sync(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
__device__ __forceinline__ bool wg_and(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id)
      : "memory");
  return r != 0;
}

// fp32 T scratch (64 x 64) with an XOR swizzle that keeps the mma.sync fragment loads
// conflict-free: element (r, c) at r * 64 + (c ^ ((r & 3) << 3)).
__device__ __forceinline__ int tidx(int r, int c) { return r * 64 + (c ^ ((r & 3) << 3)); }

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// acc (a 16x16 block as two m16n8 tiles) += X (16x16) * Y (16x16); x(r, c), y(r, c) read
// the operands. Fragment layout of m16n8k8 tf32: groupID g = lane / 4, t = lane % 4.
template <typename FX, typename FY>
__device__ __forceinline__ void block_mma(float (&acc)[2][4], FX x, FY y, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < 16; k0 += 8) {
    const uint32_t a[4] = {to_tf32(x(g, k0 + t)), to_tf32(x(g + 8, k0 + t)), to_tf32(x(g, k0 + t + 4)),
                           to_tf32(x(g + 8, k0 + t + 4))};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const uint32_t b[2] = {to_tf32(y(k0 + t, 8 * nt + g)), to_tf32(y(k0 + t + 4, 8 * nt + g))};
      mma_tf32(acc[nt], a, b);
    }
  }
}
// Store acc (scaled by s) through st(r, c, value).
template <typename FS>
__device__ __forceinline__ void block_store(const float (&acc)[2][4], float s, FS st, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    st(g, 8 * nt + 2 * t, s * acc[nt][0]);
    st(g, 8 * nt + 2 * t + 1, s * acc[nt][1]);
    st(g + 8, 8 * nt + 2 * t, s * acc[nt][2]);
    st(g + 8, 8 * nt + 2 * t + 1, s * acc[nt][3]);
  }
}

template <typename TOut>
__global__ void __launch_bounds__(NT, 1)
    gdn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                          const PrefillArgs p) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
    tc::mbar_init(&sm.bar_s, 1);
    tc::mbar_init(&sm.prep_ready, 128);
    tc::mbar_init(&sm.drain_s, 1);
    tc::mbar_init(&sm.drain_p, 1);
    sm.abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // TMEM lane of row (tid % 128)

  const uint32_t i_kk = tc::idesc_bf16_f32(128, 64, false, false);   // A K-major, B K-major, N=64
  const uint32_t i_kmn = tc::idesc_bf16_f32(128, 64, false, true);   // A K-major, B MN-major, N=64
  const uint32_t i_mnk = tc::idesc_bf16_f32(128, 64, true, false);   // A MN-major, B K-major, N=64
  const uint32_t i_s = tc::idesc_bf16_f32(128, 128, false, true);    // S update, N=128

  if (warp == 8) {
    // ================================================================ producer
    if (lane == 0) {
      tc::prefetch_tmap(&tm_q);
      tc::prefetch_tmap(&tm_k);
      tc::prefetch_tmap(&tm_v);
      tc::prefetch_tmap(&tm_o);
      int last_kq[2] = {-1, -1}, last_v = -1;
      for (int m = 0; m < nchunks && !sm.abort; ++m) {
        // K|Q of chunk m reuse the buffer of chunk m-2: its state update must be done.
        if (m >= 2 && !tc::mbar_wait(&sm.bar_s, (m - 2) & 1)) {
          if (p.err) atomicCAS(p.err, 0, 301);
          sm.abort = 1;
          break;
        }
        const int buf = m & 1;
        tc::mbar_expect_tx(&sm.bar_kq[buf], 4 * 8192);
        for (int a = 0; a < 2; ++a) {
          tc::tma_load_4d(sm.kq[buf][a], &tm_k, &sm.bar_kq[buf], 64 * a, m * C, hk, b);
          tc::tma_load_4d(sm.kq[buf][a] + 8192, &tm_q, &sm.bar_kq[buf], 64 * a, m * C, hk, b);
        }
        last_kq[buf] = m;
        // V of chunk m reuses the V buffer: the U' product of chunk m-1 must be done.
        if (m >= 1 && !tc::mbar_wait(&sm.bar_p3, (m - 1) & 1)) {
          if (p.err) atomicCAS(p.err, 0, 302);
          sm.abort = 1;
          break;
        }
        tc::mbar_expect_tx(&sm.bar_v, 2 * 8192);
        for (int a = 0; a < 2; ++a) tc::tma_load_4d(sm.v[a], &tm_v, &sm.bar_v, 64 * a, m * C, h, b);
        last_v = m;
      }
      // our loads in flight land before the CTA exits (bounded)
      for (int bb = 0; bb < 2; ++bb)
        if (last_kq[bb] >= 0) tc::mbar_wait(&sm.bar_kq[bb], (last_kq[bb] >> 1) & 1, 200000000ull);
      if (last_v >= 0) tc::mbar_wait(&sm.bar_v, last_v & 1, 200000000ull);
    }
  } else if (warp >= 4) {
    // ================================================================ prep warpgroup
    const int pt = tid - 128, pw = warp - 4;  // thread / warp within the group
    bool ok = true;
    auto fail = [&](int site) {
      if (pt == 0) {
        if (p.err) atomicCAS(p.err, 0, 200 + site);
        sm.abort = 1;
      }
      ok = false;
    };
    // bounded wait by every prep thread, outcome uniform across the group
    auto pwait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool got = wg_and(2, tc::mbar_wait(bar, parity) && !sm.abort);
      if (!got) fail(site);
      tc::fence_after_sync();
      return got;
    };
    // g and beta of the next chunk are loaded one chunk ahead (registers of warp 4: lane
    // l holds steps 2l and 2l+1).
    float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
    auto fetch_scalars = [&](int m) {
      g0 = g1 = b0 = b1 = 0.f;
      if (pw == 0 && m < nchunks) {
        const int t = m * C + 2 * lane;
        if (t < p.seqlen) {
          g0 = load_any(p.g, b * p.g_sb + (int64_t)t * p.g_st + h * p.g_sh, p.g_dtype);
          b0 = load_any(p.beta, b * p.b_sb + (int64_t)t * p.b_st + h * p.b_sh, p.b_dtype);
        }
        if (t + 1 < p.seqlen) {
          g1 = load_any(p.g, b * p.g_sb + (int64_t)(t + 1) * p.g_st + h * p.g_sh, p.g_dtype);
          b1 = load_any(p.beta, b * p.b_sb + (int64_t)(t + 1) * p.b_st + h * p.b_sh, p.b_dtype);
        }
      }
    };
    fetch_scalars(0);
    for (int m = 0; m < nchunks && ok; ++m) {
      const int buf = m & 1, sb = m % 3;
      // ---- scalars: cumulative log decay c, gamma = e^c, e = e^(c_C - c), beta
      if (pw == 0) {
        constexpr float kLog2e = 1.4426950408889634f;
        const float pair = g0 + g1;
        float incl = pair;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const float c0 = incl - pair + g0, c1 = incl;
        const float clast = __shfl_sync(0xffffffffu, incl, 31);
        sm.cum2[sb][2 * lane] = c0 * kLog2e;
        sm.cum2[sb][2 * lane + 1] = c1 * kLog2e;
        sm.gam[sb][2 * lane] = exp2f(c0 * kLog2e);
        sm.gam[sb][2 * lane + 1] = exp2f(c1 * kLog2e);
        sm.ee[sb][2 * lane] = exp2f((clast - c0) * kLog2e);
        sm.ee[sb][2 * lane + 1] = exp2f((clast - c1) * kLog2e);
        sm.beta[sb][2 * lane] = b0;
        sm.beta[sb][2 * lane + 1] = b1;
      }
      fetch_scalars(m + 1);
      wg_sync(2);
      // ---- [K;Q] K^T
      if (!pwait(&sm.bar_kq[buf], (m >> 1) & 1, 1)) break;
      if (pt == 0) {
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t base = tc::smem_u32(sm.kq[buf][kk >> 2]) + (kk & 3) * 32;
          tc::mma_f16(tmem + kColD1, tc::sdesc_sw128(base, 16, 1024), tc::sdesc_sw128(base, 16, 1024), i_kk,
                      kk != 0);
        }
        tc::mma_commit(&sm.bar_p1);
      }
      if (!pwait(&sm.bar_p1, m & 1, 2)) break;
      // ---- A (fp32) from K K^T rows (lanes 0-63), M (bf16) from Q K^T rows (lanes 64-127)
      {
        float v[64];
        tmem_row64(lane_addr + kColD1, v);
        const float* c2 = sm.cum2[sb];
        if (pt < C) {
          const int t = pt;
          const float bt = sm.beta[sb][t], ct = c2[t];
          const int lim = pw == 0 ? 32 : 64;  // rows 0-31 have no terms past column 31
#pragma unroll
          for (int i = 0; i < C; i += 4) {
            float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < lim) {
              w.x = i + 0 < t ? bt * v[i + 0] * exp2f(ct - c2[i + 0]) : 0.f;
              w.y = i + 1 < t ? bt * v[i + 1] * exp2f(ct - c2[i + 1]) : 0.f;
              w.z = i + 2 < t ? bt * v[i + 2] * exp2f(ct - c2[i + 2]) : 0.f;
              w.w = i + 3 < t ? bt * v[i + 3] * exp2f(ct - c2[i + 3]) : 0.f;
            }
            *reinterpret_cast<float4*>(&sm.a[t * PA + i]) = w;
          }
        } else {
          const int t = pt - C;
          const float ct = c2[t];
          const int lim = pw == 2 ? 32 : 64;
#pragma unroll
          for (int i = 0; i < C; ++i) v[i] = (i < lim && i <= t) ? p.scale * v[i] * exp2f(ct - c2[i]) : 0.f;
          store_row_bf16(sm.m[buf], t, v);
        }
      }
      tc::fence_before_sync();
      wg_sync(2);
      // ---- T = (I + A)^-1, blocked: diagonal 16x16 blocks by forward substitution
      float* ts = reinterpret_cast<float*>(sm.wt[buf]);  // fp32 T scratch (free: W^T(m-2) consumed)
      {
        const int blk = pw, col = lane & 15, r0 = 16 * blk;
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float s = 0.f;
#pragma unroll
          for (int mm = 0; mm + 3 < i; mm += 4) {
            const float4 a4 = *reinterpret_cast<const float4*>(&sm.a[(r0 + i) * PA + r0 + mm]);
            s = fmaf(a4.x, x[mm], s);
            s = fmaf(a4.y, x[mm + 1], s);
            s = fmaf(a4.z, x[mm + 2], s);
            s = fmaf(a4.w, x[mm + 3], s);
          }
#pragma unroll
          for (int mm = i & ~3; mm < i; ++mm) s = fmaf(sm.a[(r0 + i) * PA + r0 + mm], x[mm], s);
          x[i] = i < col ? 0.f : (i == col ? 1.f : -s);
        }
        if (lane < 16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) ts[tidx(r0 + i, r0 + col)] = x[i];
        }
      }
      wg_sync(2);
      // off-diagonal blocks: T_ij = -T_ii (sum_{k=j}^{i-1} A_ik T_kj), in three levels:
      // the two 32x32 diagonal halves (T_10, T_32), then the lower-left 32x32 quarter as
      // X = A_21 T_1 (four 16x16 blocks, one per warp) and T_21 = -T_2 X.
      {
        float* scr = reinterpret_cast<float*>(sm.tb);  // 4 x (16 x 24) fp32 scratch blocks
        auto sread = [&](int w) { return [=](int r, int c) { return scr[w * 384 + r * 24 + c]; }; };
        auto swrite = [&](int w) { return [=](int r, int c, float x) { scr[w * 384 + r * 24 + c] = x; }; };
        auto at = [&](int bi, int bj) {
          return [=, &sm](int r, int c) { return sm.a[(16 * bi + r) * PA + 16 * bj + c]; };
        };
        auto tt = [&](int bi, int bj) { return [=](int r, int c) { return ts[tidx(16 * bi + r, 16 * bj + c)]; }; };
        auto twrite = [&](int bi, int bj) {
          return [=](int r, int c, float x) { ts[tidx(16 * bi + r, 16 * bj + c)] = x; };
        };
        if (pw < 2) {  // T_10 (warp 0), T_32 (warp 1)
          const int j = 2 * pw, i = j + 1;
          float acc[2][4] = {};
          block_mma(acc, at(i, j), tt(j, j), lane);
          block_store(acc, 1.f, swrite(pw), lane);
          __syncwarp();
          float acc2[2][4] = {};
          block_mma(acc2, tt(i, i), sread(pw), lane);
          block_store(acc2, -1.f, twrite(i, j), lane);
        }
        wg_sync(2);
        const int r = 2 + (pw >> 1), c = pw & 1;
        {  // X_rc = sum_{k=c}^{1} A_rk T_kc
          float acc[2][4] = {};
          for (int k = c; k < 2; ++k) block_mma(acc, at(r, k), tt(k, c), lane);
          block_store(acc, 1.f, swrite(pw), lane);
        }
        wg_sync(2);
        {  // T_rc = -sum_{k=2}^{r} T_rk X_kc
          float acc[2][4] = {};
          for (int k = 2; k <= r; ++k) block_mma(acc, tt(r, k), sread(2 * (k - 2) + c), lane);
          block_store(acc, -1.f, twrite(r, c), lane);
        }
        wg_sync(2);
      }
      // ---- TB = T diag(beta), TBG = T diag(beta gamma), bf16 rows (zero above the blocks)
      {
        const int t = pt >> 1, half = pt & 1;
        float vb[32], vbg[32];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int i = 32 * half + jj;
          const float x = (i >> 4) <= (t >> 4) ? ts[tidx(t, i)] * sm.beta[sb][i] : 0.f;
          vb[jj] = x;
          vbg[jj] = x * sm.gam[sb][i];
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 w1, w2;
          w1.x = pack_bf16x2(vb[8 * c], vb[8 * c + 1]);
          w1.y = pack_bf16x2(vb[8 * c + 2], vb[8 * c + 3]);
          w1.z = pack_bf16x2(vb[8 * c + 4], vb[8 * c + 5]);
          w1.w = pack_bf16x2(vb[8 * c + 6], vb[8 * c + 7]);
          w2.x = pack_bf16x2(vbg[8 * c], vbg[8 * c + 1]);
          w2.y = pack_bf16x2(vbg[8 * c + 2], vbg[8 * c + 3]);
          w2.z = pack_bf16x2(vbg[8 * c + 4], vbg[8 * c + 5]);
          w2.w = pack_bf16x2(vbg[8 * c + 6], vbg[8 * c + 7]);
          const uint32_t off = tc::sw128_offset(t, 32 * half + 8 * c);
          *reinterpret_cast<uint4*>(sm.tb + off) = w1;  // the tb scratch reads ended at the last barrier
          *reinterpret_cast<uint4*>(sm.tbg + off) = w2;
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      // ---- W^T = K^T TBG^T -> D1; U'^T = V^T TB^T -> UP[buf]
      if (!pwait(&sm.bar_v, m & 1, 3)) break;
      if (pt == 0) {
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][0]) + kk * 2048, 16384, 1024);
          const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sm.tbg) + kk * 32, 16, 1024);
          tc::mma_f16(tmem + kColD1, ad, bd, i_mnk, kk != 0);
        }
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.v[0]) + kk * 2048, 8192, 1024);
          const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sm.tb) + kk * 32, 16, 1024);
          tc::mma_f16(tmem + kColUP + 64 * buf, ad, bd, i_mnk, kk != 0);
        }
        tc::mma_commit(&sm.bar_p3);
      }
      if (!pwait(&sm.bar_p3, m & 1, 4)) break;
      // ---- W^T -> wt[buf] (bf16, MN-major rows)
      {
        float v[64];
        tmem_row64(lane_addr + kColD1, v);
        store_row_bf16(sm.wt[buf], pt, v);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      // The serial group must have taken chunk m-1 (its first MMA commit) before chunk m is
      // announced, so the two phases of prep_ready never alias.
      if (m >= 1 && !pwait(&sm.bar_ws, (m - 1) & 1, 5)) break;
      tc::mbar_arrive(&sm.prep_ready);
    }
    if (pt == 0) {  // every MMA this thread issued completes before TMEM is freed
      tc::mma_commit(&sm.drain_p);
      tc::mbar_wait(&sm.drain_p, 0, 200000000ull);
    }
  } else {
    // ================================================================ serial warpgroup
    bool ok = true;
    auto fail = [&](int site) {
      if (tid == 0) {
        if (p.err) atomicCAS(p.err, 0, 250 + site);
        sm.abort = 1;
      }
      ok = false;
    };
    auto swait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool got = wg_and(1, tc::mbar_wait(bar, parity) && !sm.abort);
      if (!got) fail(site);
      tc::fence_after_sync();
      return got;
    };
    // state in: S^T in TMEM, row = this thread's value column
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
    // S step of chunk n: S^T -> bf16 operand tile; S^T *= gamma_C in TMEM. Then the
    // S products of chunk n (thread 0).
    auto state_step = [&](int n) {
      const int buf = n & 1, sb = n % 3;
      const float gl = sm.gam[sb][C - 1];
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 64) {
        float f[64];
        tmem_row64(lane_addr + kColS + c0, f);
        uint8_t* tile = sm.st[c0 >> 6];
        store_row_bf16(tile, tid, f);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(f[32 * half + i] * gl);
          tc::tmem_st_32x32(lane_addr + kColS + c0 + 32 * half, r);
        }
      }
      tc::tmem_st_wait();
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      wg_sync(1);
      if (tid == 0) {
        tc::fence_after_sync();
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.st[kk >> 2]) + (kk & 3) * 32, 16, 1024);
          const uint64_t bw = tc::sdesc_sw128(tc::smem_u32(sm.wt[buf]) + kk * 2048, 16, 1024);
          tc::mma_f16(tmem + kColWS, ad, bw, i_kmn, kk != 0);
        }
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.st[kk >> 2]) + (kk & 3) * 32, 16, 1024);
          const uint64_t bq =
              tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][kk >> 2]) + 8192 + (kk & 3) * 32, 16, 1024);
          tc::mma_f16(tmem + kColQS, ad, bq, i_kk, kk != 0);
        }
        tc::mma_commit(&sm.bar_ws);
      }
    };
    if (swait(&sm.prep_ready, 0, 1)) state_step(0);
    for (int n = 0; n < nchunks && ok; ++n) {
      const int buf = n & 1, sb = n % 3;
      // U = U' - WS -> U^T bf16; then UM^T = U^T M^T and S^T += (U diag(e))^T K
      if (tid == 0) tc::bulk_wait_read0();  // the output store of chunk n-1 has read ut
      if (!swait(&sm.bar_ws, n & 1, 2)) break;
      {
        float ws[64], up[64];
        tmem_row64(lane_addr + kColWS, ws);
        tmem_row64(lane_addr + kColUP + 64 * buf, up);
#pragma unroll
        for (int i = 0; i < 64; ++i) up[i] -= ws[i];
        store_row_bf16(sm.ut, tid, up);
        // U diag(e) -> st[0] (free: the S^T products of this chunk are done), the A
        // operand of the state update
        const float* ee = sm.ee[sb];
#pragma unroll
        for (int i = 0; i < 64; ++i) up[i] *= ee[i];
        store_row_bf16(sm.st[0], tid, up);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      wg_sync(1);
      if (tid == 0) {
        tc::fence_after_sync();
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.ut) + kk * 32, 16, 1024);
          const uint64_t bm = tc::sdesc_sw128(tc::smem_u32(sm.m[buf]) + kk * 32, 16, 1024);
          tc::mma_f16(tmem + kColUM, ad, bm, i_kk, kk != 0);
        }
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = tc::sdesc_sw128(tc::smem_u32(sm.st[0]) + kk * 32, 16, 1024);
          const uint64_t bk = tc::sdesc_sw128(tc::smem_u32(sm.kq[buf][0]) + kk * 2048, 16384, 1024);
          tc::mma_f16(tmem + kColS, ad, bk, i_s, 1);
        }
        tc::mma_commit(&sm.bar_s);
      }
      if (!swait(&sm.bar_s, n & 1, 3)) break;
      // O = gamma scale QS + UM (registers), then the next chunk's state step, then the
      // stores of O through shared memory (ut is free: U products are done).
      float o[64];
      {
        float um[64];
        tmem_row64(lane_addr + kColQS, o);
        tmem_row64(lane_addr + kColUM, um);
        const float* gm = sm.gam[sb];
#pragma unroll
        for (int t = 0; t < 64; ++t) o[t] = fmaf(gm[t] * p.scale, o[t], um[t]);
      }
      tc::fence_before_sync();
      if (n + 1 < nchunks) {
        if (!swait(&sm.prep_ready, (n + 1) & 1, 4)) break;
        state_step(n + 1);
      }
      // O through shared memory (ut, row-major [rows][128]) and a TMA store; rows past
      // the sequence end fall outside the tensor and are not written.
      constexpr int kRows = sizeof(TOut) == 2 ? 64 : 32;  // 16 KB per pass
      TOut* stage = reinterpret_cast<TOut*>(sm.ut);
#pragma unroll
      for (int t0 = 0; t0 < 64; t0 += kRows) {
        if (t0 > 0) {
          if (tid == 0) tc::bulk_wait_read0();
          wg_sync(1);
        }
#pragma unroll
        for (int t = 0; t < kRows; ++t) stage[t * D + tid] = from_f32<TOut>(o[t0 + t]);
        tc::fence_proxy_async_smem();
        wg_sync(1);
        if (tid == 0) {
          tc::tma_store_4d(&tm_o, stage, 0, n * C + t0, h, b);
          tc::bulk_commit();
        }
      }
    }
    if (tid == 0) tc::bulk_wait0();
    if (tid == 0) {  // every MMA this thread issued completes before TMEM is freed
      tc::mma_commit(&sm.drain_s);
      tc::mbar_wait(&sm.drain_s, 0, 200000000ull);
    }
    if (ok) {
      // state out
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
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 8) {
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
  // the output is written with 16-byte vectors along the value dim
  const bool out_ok = (reinterpret_cast<uintptr_t>(d.o.data) & 15) == 0 &&
                      d.o.stride_t % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0 &&
                      d.o.stride_h % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0 &&
                      d.o.stride_b % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0;
  return d.q.dtype == PBK_BF16 && d.dk == 128 && d.dv == 128 && d.seqlen > 0 && ok16(d.q) && ok16(d.k) &&
         ok16(d.v) && out_ok;
}

cudaError_t launch_gdn_prefill_tc(const pbk_gdn_desc& d, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, d.q, d.hk, d) || !make_map(&mk, d.k, d.hk, d) || !make_map(&mv, d.v, d.hv, d))
    return cudaErrorInvalidValue;
  {
    const bool obf = d.o.dtype == PBK_BF16;
    const uint64_t es = obf ? 2 : 4;
    const uint64_t dims[4] = {128, (uint64_t)d.seqlen, (uint64_t)d.hv, (uint64_t)d.batch};
    const uint64_t strides[3] = {(uint64_t)d.o.stride_t * es, (uint64_t)d.o.stride_h * es,
                                 (uint64_t)d.o.stride_b * es};
    const uint32_t box[4] = {128, obf ? 64u : 32u, 1, 1};
    if (!make_tmap_plain(&mo, d.o.data, obf, 4, dims, strides, box)) return cudaErrorInvalidValue;
  }
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
    gdn_prefill_tc_kernel<bf16><<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, mo, a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(gdn_prefill_tc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    gdn_prefill_tc_kernel<float><<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, mo, a);
  }
  return cudaGetLastError();
}

}  // namespace pbk
