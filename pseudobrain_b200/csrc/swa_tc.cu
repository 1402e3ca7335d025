// Causal sliding-window attention with sinks and GQA, forward, on tcgen05 (sm_100a).
//
// Computes pseudobrain/transplant.py:417-436 (`causal_attention`, with the chunked exact
// path of :346-362): query t of head h sees key s of key head h / G when
//     s <= t  and  (window <= 0  or  t - s < window  or  s < sinks),
// softmax(scale * q k^T) over the visible keys, times V. The reference runs SDPA on query
// chunks of 4096; the result is the same function.
//
// One CTA = (batch, key head, 128-query block, pair of query heads of that key head): the
// two heads share every K and V tile in shared memory. Per key tile j of 128 keys:
//   S_h = Q_h K_j^T           (tcgen05, M=128 queries, N=128 keys, K=128 dims; TMEM)
//   P_h = exp2(S_h c - m_h)   (softmax warps, one query row per thread, bf16 to smem)
//   O_h += P_h V_j            (tcgen05, N=128 dims, V as an MN-major operand; TMEM)
// with an online softmax whose running maximum is only raised when a row's maximum grows
// by more than 2^8 (then O and l are rescaled in place), so P stays below 256 and the
// final O / l is exact up to rounding. Key tiles are those of the sinks followed by those
// of the window; only tiles that cross the diagonal, the window edge or T are masked.
//
// Warps: 0 = TMA producer (Q once; K and V tiles through a 3-slot ring, each slot two
// 128B-swizzled 64-column halves), 1 = TMEM owner and MMA issuer, 2-5 = softmax of head A,
// 6-9 = softmax of head B (warp w reads TMEM lane quadrant w % 4). TMEM: S_A 0-127,
// O_A 128-255, S_B 256-383, O_B 384-511. Every wait is bounded; on timeout the kernel
// records an error code, stops issuing, drains its own loads and MMAs, frees TMEM and
// returns. No multicast loads.
#include "common.cuh"
#include "swa.cuh"
#include "tc.cuh"
#include "tma_host.h"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int BQ = 128;
constexpr int BK = 128;
constexpr int kStages = 3;
constexpr int NT = 320;
constexpr uint32_t kTileBytes = BK * 128 * 2;  // 32 KB: two 16 KB halves of 64 columns
constexpr uint32_t kHalfBytes = kTileBytes / 2;
constexpr uint32_t kTmemCols = 512;
constexpr float kRaise = 8.f;                  // log2 headroom of the stale running maximum

struct SwaSmem {
  alignas(1024) uint8_t q[2][kTileBytes];
  alignas(1024) uint8_t p[2][kTileBytes];
  alignas(1024) uint8_t ring[kStages][kTileBytes];
  uint64_t bar_q, full[kStages], empty[kStages], s_full[2], s_free[2], p_full[2], o_done[2], drain;
  uint32_t tmem_base;
  volatile int abort;
};

struct SwaArgs {
  int seqlen, kv, groups, pairs, nqb;
  int window, sinks;
  float scale_log2;
  void* o;
  int64_t o_sb, o_st, o_sh;
  int o_bf16;
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Load sequence of the ring: K0, then (K_j, V_{j-1}) for j = 1..n-1, then V_{n-1}.
__device__ __forceinline__ int seq_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int seq_v(int j, int n) { return min(2 * j + 2, 2 * n - 1); }

__global__ void __launch_bounds__(NT, 1)
    swa_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                  const __grid_constant__ CUtensorMap mv, const SwaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  SwaSmem& sm = *reinterpret_cast<SwaSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  int bid = blockIdx.x;
  const int pair = bid % a.pairs;
  bid /= a.pairs;
  const int qb = bid % a.nqb;
  bid /= a.nqb;
  const int kvh = bid % a.kv;
  const int b = bid / a.kv;
  const int h_a = kvh * a.groups + 2 * pair;
  const int nh = (2 * pair + 1 < a.groups) ? 2 : 1;
  const int q0 = qb * BQ;
  const int qlast = min(q0 + BQ - 1, a.seqlen - 1);
  const int hi = qlast / BK;
  const int lo = a.window > 0 ? max(0, q0 - (a.window - 1)) / BK : 0;
  const int ns = a.sinks > 0 ? min((a.sinks + BK - 1) / BK, lo) : 0;
  const int n = ns + (hi - lo + 1);

  if (tid == 0) {
    tc::mbar_init(&sm.bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&sm.full[s], 1);
      tc::mbar_init(&sm.empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      tc::mbar_init(&sm.s_full[h], 1);
      tc::mbar_init(&sm.s_free[h], 128);
      tc::mbar_init(&sm.p_full[h], 128);
      tc::mbar_init(&sm.o_done[h], 1);
    }
    tc::mbar_init(&sm.drain, 1);
    sm.abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  auto fail = [&](int site) {
    if (a.err) atomicCAS(a.err, 0, 300 + site);
    sm.abort = 1;
  };
  auto wait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
    if (tc::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = tc::globaltimer_ns();
    while (!tc::mbar_try_wait(bar, parity)) {
      if (sm.abort || tc::globaltimer_ns() - t0 > 2000000000ull) {
        fail(site);
        return false;
      }
    }
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tc::prefetch_tmap(&mq);
      tc::prefetch_tmap(&mk);
      tc::prefetch_tmap(&mv);
      tc::mbar_expect_tx(&sm.bar_q, nh * kTileBytes);
      for (int hh = 0; hh < nh; ++hh)
        for (int half = 0; half < 2; ++half)
          tc::tma_load_4d(sm.q[hh] + half * kHalfBytes, &mq, &sm.bar_q, half * 64, q0, h_a + hh, b);
      const int total = 2 * n;
      int issued = 0;
      for (int L = 0; L < total; ++L) {
        bool is_k;
        int j;
        if (L == 0) {
          is_k = true, j = 0;
        } else if (L == total - 1) {
          is_k = false, j = n - 1;
        } else if (L & 1) {
          is_k = true, j = (L + 1) >> 1;
        } else {
          is_k = false, j = (L >> 1) - 1;
        }
        const int s = L % kStages, r = L / kStages;
        if (r > 0 && !wait(&sm.empty[s], (r - 1) & 1, 1)) break;
        const int kt = j < ns ? j : lo + (j - ns);
        tc::mbar_expect_tx(&sm.full[s], kTileBytes);
        for (int half = 0; half < 2; ++half)
          tc::tma_load_4d(sm.ring[s] + half * kHalfBytes, is_k ? &mk : &mv, &sm.full[s], half * 64, kt * BK, kvh, b);
        issued = L + 1;
      }
      // our loads land before the CTA exits
      tc::mbar_wait(&sm.bar_q, 0, 200000000ull);
      for (int L = max(0, issued - kStages); L < issued; ++L)
        tc::mbar_wait(&sm.full[L % kStages], (L / kStages) & 1, 200000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t i_qk = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t i_pv = tc::idesc_bf16_f32(128, 128, false, true);
      bool ok = wait(&sm.bar_q, 0, 2);
      tc::fence_after_sync();
      auto issue_s = [&](int j) -> bool {
        const int L = seq_k(j), s = L % kStages;
        if (!wait(&sm.full[s], (L / kStages) & 1, 3)) return false;
        tc::fence_after_sync();
        for (int hh = 0; hh < nh; ++hh) {
          if (j > 0 && !wait(&sm.s_free[hh], (j - 1) & 1, 4)) return false;
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
            tc::mma_f16(tmem + hh * 256, tc::sdesc_sw128(tc::smem_u32(sm.q[hh]) + off, 16, 1024),
                        tc::sdesc_sw128(tc::smem_u32(sm.ring[s]) + off, 16, 1024), i_qk, kk != 0);
          }
          tc::mma_commit(&sm.s_full[hh]);
        }
        tc::mma_commit(&sm.empty[s]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int L = seq_v(j, n), s = L % kStages;
        if (!wait(&sm.full[s], (L / kStages) & 1, 5)) return false;
        tc::fence_after_sync();
        for (int hh = 0; hh < nh; ++hh) {
          if (!wait(&sm.p_full[hh], j & 1, 6)) return false;
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad =
                tc::sdesc_sw128(tc::smem_u32(sm.p[hh]) + (kk >> 2) * kHalfBytes + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = tc::sdesc_sw128(tc::smem_u32(sm.ring[s]) + kk * 2048, kHalfBytes, 1024);
            tc::mma_f16(tmem + hh * 256 + 128, ad, bd, i_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&sm.o_done[hh]);
        }
        tc::mma_commit(&sm.empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 1; ok && j < n; ++j) ok = issue_s(j) && issue_pv(j - 1);
      if (ok) issue_pv(n - 1);
      // every MMA issued here completes before the CTA exits
      tc::mma_commit(&sm.drain);
      tc::mbar_wait(&sm.drain, 0, 200000000ull);
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int hh = (warp - 2) >> 2;
    if (hh < nh) {
      const int quad = warp & 3;
      const int row = quad * 32 + lane;
      const int qpos = q0 + row;
      const uint32_t t_s = tmem + ((uint32_t)(quad * 32) << 16) + hh * 256;
      const uint32_t t_o = t_s + 128;
      const uint32_t p_row = tc::smem_u32(sm.p[hh]) + row * 128;
      const float c = a.scale_log2;
      float m = -INFINITY;  // running maximum of the raw scores (unscaled)
      float l = 0.f;
      bool ok = true;
      // warp-uniform outcome: the tcgen05.ld/st that follow need the whole warp
      auto wwait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
        return __all_sync(0xffffffffu, wait(bar, parity, site));
      };
      for (int j = 0; j < n; ++j) {
        if (!wwait(&sm.s_full[hh], j & 1, 7)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        uint32_t r[128];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          tc::tmem_ld_32x32(t_s + 32 * cc, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * cc]));
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        tc::mbar_arrive(&sm.s_free[hh]);

        const int kt = j < ns ? j : lo + (j - ns);
        const int k0 = kt * BK;
        const bool interior = (k0 + BK - 1 <= q0) && (k0 + BK - 1 < a.seqlen) &&
                              (a.window <= 0 || k0 >= q0 + BQ - 1 - (a.window - 1));
        float mx = -INFINITY;
        if (interior) {
#pragma unroll
          for (int i = 0; i < 128; ++i) mx = fmaxf(mx, __uint_as_float(r[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int kpos = k0 + i;
            const bool vis = kpos <= qpos && kpos < a.seqlen &&
                             (a.window <= 0 || qpos - kpos < a.window || kpos < a.sinks);
            const float x = vis ? __uint_as_float(r[i]) : -INFINITY;
            r[i] = __float_as_uint(x);
            mx = fmaxf(mx, x);
          }
        }
        // raise the running maximum only when this tile exceeds it by more than 2^kRaise
        const bool raise = mx * c > m * c + kRaise || (m == -INFINITY && mx != -INFINITY);
        const float m_new = raise ? mx : m;
        const float off = m_new == -INFINITY ? 0.f : m_new * c;
        uint32_t pk[64];
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          const float p0 = ex2(fmaf(__uint_as_float(r[i]), c, -off));
          const float p1 = ex2(fmaf(__uint_as_float(r[i + 1]), c, -off));
          const float p2 = ex2(fmaf(__uint_as_float(r[i + 2]), c, -off));
          const float p3 = ex2(fmaf(__uint_as_float(r[i + 3]), c, -off));
          s0 += p0;
          s1 += p1;
          s2 += p2;
          s3 += p3;
          pk[i >> 1] = pack_bf16x2(p0, p1);
          pk[(i >> 1) + 1] = pack_bf16x2(p2, p3);
        }
        const float factor = raise ? (m == -INFINITY ? 0.f : ex2((m - m_new) * c)) : 1.f;
        l = l * factor + ((s0 + s1) + (s2 + s3));
        m = m_new;
        // PV(j-1) has finished reading P and writing O
        if (j > 0) {
          if (!wwait(&sm.o_done[hh], (j - 1) & 1, 8)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          if (__any_sync(0xffffffffu, raise)) {
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
              uint32_t o[32];
              tc::tmem_ld_32x32(t_o + 32 * cc, o);
              tc::tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
              tc::tmem_st_32x32(t_o + 32 * cc, o);
            }
            tc::tmem_st_wait();
          }
        }
        // P row (128 keys) into the K-major, 128B-swizzled A operand: two 64-key halves
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const uint32_t addr =
              p_row + (ch >> 3) * kHalfBytes + ((((uint32_t)ch & 7u) ^ ((uint32_t)row & 7u)) << 4);
          st_shared_v4(addr, pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        tc::mbar_arrive(&sm.p_full[hh]);
      }
      if (ok && wwait(&sm.o_done[hh], (n - 1) & 1, 9)) {
        tc::fence_after_sync();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int h = h_a + hh;
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t o[32];
          tc::tmem_ld_32x32(t_o + 32 * cc, o);  // whole warp; rows past T are not stored
          tc::tmem_ld_wait();
          if (qpos >= a.seqlen) continue;
          if (a.o_bf16) {
            bf16* dst = reinterpret_cast<bf16*>(a.o) + b * a.o_sb + (int64_t)qpos * a.o_st + (int64_t)h * a.o_sh +
                        32 * cc;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
              *reinterpret_cast<uint4*>(dst + i) = v;
            }
          } else {
            float* dst = reinterpret_cast<float*>(a.o) + b * a.o_sb + (int64_t)qpos * a.o_st + (int64_t)h * a.o_sh +
                         32 * cc;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + i) =
                  make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                              __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

constexpr size_t kSmemBytes = sizeof(SwaSmem) + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory above the sm_100 per-block opt-in limit");

bool make_map(CUtensorMap* m, const pbk_view& v, int seqlen, int heads, int batch) {
  const uint64_t dims[4] = {128, (uint64_t)seqlen, (uint64_t)heads, (uint64_t)batch};
  const uint64_t strides[3] = {(uint64_t)v.stride_t * 2, (uint64_t)v.stride_h * 2, (uint64_t)v.stride_b * 2};
  const uint32_t box[4] = {64, 128, 1, 1};
  return make_tmap_bf16_sw128(m, v.data, 4, dims, strides, box);
}

}  // namespace

cudaError_t launch_swa_tc(const pbk_swa_desc& d, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, d.q, d.seqlen, d.h, d.batch) || !make_map(&mk, d.k, d.seqlen, d.kv, d.batch) ||
      !make_map(&mv, d.v, d.seqlen, d.kv, d.batch))
    return cudaErrorInvalidValue;
  SwaArgs a;
  a.seqlen = d.seqlen;
  a.kv = d.kv;
  a.groups = d.h / d.kv;
  a.pairs = (a.groups + 1) / 2;
  a.nqb = (d.seqlen + BQ - 1) / BQ;
  a.window = d.window;
  a.sinks = d.sinks;
  a.scale_log2 = d.scale * 1.4426950408889634f;
  a.o = const_cast<void*>(d.o.data);
  a.o_sb = d.o.stride_b;
  a.o_st = d.o.stride_t;
  a.o_sh = d.o.stride_h;
  a.o_bf16 = d.o.dtype == PBK_BF16;
  a.err = device_error_word();
  const int64_t blocks = (int64_t)a.pairs * a.nqb * d.kv * d.batch;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(swa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  swa_tc_kernel<<<(unsigned)blocks, NT, kSmemBytes, st>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

}  // namespace pbk
