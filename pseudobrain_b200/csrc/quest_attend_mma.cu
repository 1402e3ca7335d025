// Split-key exact attention of the Quest path on tensor cores (mma.sync m16n8k16, bf16 in,
// fp32 accumulate): the same virtual keys, masks and workspace partials as the SIMT
// quest_attend_kernel in quest.cu, for up to 16 query rows per key head.
//
// A warp owns one split of 256 virtual keys and walks it in sub-tiles of 32: the keys' and
// values' rows are staged in the warp's shared memory with cp.async (16-byte chunks, XOR
// swizzled so ldmatrix reads are conflict-free), S = Q K^T comes from ldmatrix'ed K and Q
// fragments held in registers, the online softmax (base 2, rows g and g + 8 of the warp's
// 16-row tile) rescales the running O, and O += P V reuses S's accumulator layout as the P
// operand with V read by ldmatrix.trans. The warp writes (m, l, O) for its split; the
// combine kernel merges the splits.
#include <cuda_bf16.h>

#include "common.cuh"
#include "quest.cuh"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kD = 128;
constexpr int kSplit = 256;   // virtual keys per warp (= the SIMT kernel's split)
constexpr int kSub = 32;      // keys per sub-tile
constexpr int kWarps = 4;
constexpr int kSinkTag = -(1 << 30);  // same key encoding as quest.cu
constexpr int kRowBytes = kD * 2;     // 256 bytes per key row

struct WarpSmem {
  uint8_t k[kSub * kRowBytes];  // 8 KB, row r at r * 256, 16-byte chunk c at (c ^ (r & 7))
  uint8_t v[kSub * kRowBytes];
  int kidx[kSub];
  int kpos[kSub];  // window keys' positions (for the mask)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// byte offset of 16-byte chunk c of row r in a swizzled 256-byte-row tile
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return r * kRowBytes + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ bool visible(int kp, int qp, int window, int sinks) {
  return kp <= qp && ((qp - kp) < window || kp < sinks);
}

__global__ void __launch_bounds__(32 * kWarps) quest_attend_mma_kernel(const pbk_quest_desc d, int k, int tail,
                                                                       int splits, float* part, SinkKeys sk) {
  extern __shared__ __align__(16) uint8_t attn_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpSmem& ws = reinterpret_cast<WarpSmem*>(attn_raw)[warp];
  const int split = blockIdx.x * kWarps + warp, n = blockIdx.y / d.kv, h = blockIdx.y % d.kv;
  if (split >= splits) return;
  const int g = lane >> 2, t = lane & 3;
  const int groups = d.h / d.kv, rows = d.t * groups;
  const int n_ret = sk.n + k * d.page + tail, sr = (n_ret + kSplit - 1) / kSplit;
  const bool win_split = split >= sr;
  const int j0 = win_split ? (split - sr) * kSplit : split * kSplit;
  const int nkeys = min(kSplit, (win_split ? d.n_win : n_ret) - j0);
  const bf16* keys = reinterpret_cast<const bf16*>(d.keys);
  const bf16* vals = reinterpret_cast<const bf16*>(d.values);
  const bf16* wkeys = reinterpret_cast<const bf16*>(d.win_keys);
  const bf16* wvals = reinterpret_cast<const bf16*>(d.win_values);
  const bf16* q = reinterpret_cast<const bf16*>(d.q);
  const float sl2 = d.scale * 1.4426950408889634f;

  // Q fragments (rows g and g + 8 of the 16-row tile; rows past `rows` are zero): for k-step
  // kk, a0 = (g, 16kk + 2t..), a1 = (g + 8, ..), a2 = (g, 16kk + 8 + 2t..), a3 = (g + 8, ..)
  uint32_t qa[8][4];
  int qpos_r[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = g + 8 * hr;
    const bool ok = r < rows;
    const int ti = ok ? r / groups : 0, gg = ok ? r % groups : 0;
    const bf16* qr = q + n * d.q_stride_n + ti * d.q_stride_t + (int64_t)(h * groups + gg) * d.q_stride_h;
    qpos_r[hr] = ok ? d.qpos[n * d.t + ti] : 0;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qa[kk][hr] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 2 * t) : 0u;
      qa[kk][2 + hr] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8 + 2 * t) : 0u;
    }
  }

  float o[16][4];  // O rows (g, g + 8) x dims 8 nt + 2t, +1
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int s0 = 0; s0 < nkeys; s0 += kSub) {
    // key index of this sub-tile's key `lane`
    {
      const int vj = j0 + s0 + lane;
      int idx = 0;
      if (s0 + lane < nkeys) {
        if (win_split) idx = -1 - vj;
        else if (vj < sk.n) idx = kSinkTag - vj;
        else if (vj - sk.n < k * d.page) {
          const int r = vj - sk.n;
          idx = d.pages[((int64_t)n * d.kv + h) * k + r / d.page] * d.page + r % d.page;
        } else {
          idx = (d.n_arch / d.page) * d.page + (vj - sk.n - k * d.page);
        }
      } else {
        idx = INT32_MIN;  // past the split's keys: masked, rows zero
      }
      ws.kidx[lane] = idx;
      ws.kpos[lane] = (idx < 0 && idx > kSinkTag) ? d.kpos[-1 - idx] : 0;
    }
    __syncwarp();
    // stage the 32 key and value rows (16 chunks each); rows past the split are zeroed (their
    // probabilities are 0, and 0 * (stale bits) could be NaN)
#pragma unroll 4
    for (int it = 0; it < kSub * 16 / 32; ++it) {
      const int c = it * 32 + lane, r = c >> 4, ch = c & 15;
      const int idx = ws.kidx[r];
      if (idx == INT32_MIN) {
        *reinterpret_cast<uint4*>(ws.k + sw_off(r, ch)) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(ws.v + sw_off(r, ch)) = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      const bf16 *kr, *vr;
      if (idx >= 0) {
        kr = keys + h * d.arc_stride_kv + (int64_t)idx * d.arc_stride_n;
        vr = vals + h * d.arc_stride_kv + (int64_t)idx * d.arc_stride_n;
      } else if (idx > kSinkTag) {
        kr = wkeys + h * d.win_stride_kv + (int64_t)(-1 - idx) * d.win_stride_n;
        vr = wvals + h * d.win_stride_kv + (int64_t)(-1 - idx) * d.win_stride_n;
      } else {
        kr = sk.k + h * sk.s_kv + (int64_t)(kSinkTag - idx) * sk.s_n;
        vr = sk.v + h * sk.s_kv + (int64_t)(kSinkTag - idx) * sk.s_n;
      }
      cp_async16(smem_u32(ws.k) + sw_off(r, ch), kr + 8 * ch);
      cp_async16(smem_u32(ws.v) + sw_off(r, ch), vr + 8 * ch);
    }
    cp_async_wait_all();
    __syncwarp();

    // S = Q K^T for the sub-tile's 4 n-tiles of 8 keys
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {  // two k-steps (32 dims) per ldmatrix.x4
        // matrices: (keys 8j.., dims 32kq + 0..7 | 8..15 | 16..23 | 24..31); lane -> row
        const int mi = lane >> 3, row = 8 * j + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(ws.k) + sw_off(row, 4 * kq + mi), b0, b1, b2, b3);
        mma_bf16(sc[j], qa[2 * kq][0], qa[2 * kq][1], qa[2 * kq][2], qa[2 * kq][3], b0, b1);
        mma_bf16(sc[j], qa[2 * kq + 1][0], qa[2 * kq + 1][1], qa[2 * kq + 1][2], qa[2 * kq + 1][3], b2, b3);
      }
    }
    // mask, scale (base 2), online softmax per row (g: elements 0,1; g + 8: elements 2,3)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = 8 * j + 2 * t + (e & 1), hr = e >> 1;
        const int idx = ws.kidx[key];
        bool vis = idx != INT32_MIN;
        if (vis && idx < 0 && idx > kSinkTag) vis = visible(ws.kpos[key], qpos_r[hr], d.window, d.sinks);
        const float x = vis ? sc[j][e] * sl2 : -INFINITY;
        sc[j][e] = x;
        mx[hr] = fmaxf(mx[hr], x);
      }
    float fac[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float m_new = fmaxf(m_run[hr], mx[hr]);
      fac[hr] = m_run[hr] == -INFINITY ? 0.f : exp2f(m_run[hr] - m_new);
      m_run[hr] = m_new;
    }
    uint32_t pa[2][4];  // P as A fragments for the two 16-key k-steps
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = m_run[e >> 1];
        p[e] = m == -INFINITY ? 0.f : exp2f(sc[j][e] - m);
        ls[e >> 1] += p[e];
      }
      // n-tile j covers keys 8j..: k-step j / 2, low (j even) or high (j odd) half
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p[0], p[1]);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p[2], p[3]);
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) l_run[hr] = l_run[hr] * fac[hr] + ls[hr];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= fac[0];
      o[nt][1] *= fac[0];
      o[nt][2] *= fac[1];
      o[nt][3] *= fac[1];
    }
    // O += P V: k-step kv2 (keys 16 kv2..), n-tile pairs (dims 16 dp..)
#pragma unroll
    for (int kv2 = 0; kv2 < 2; ++kv2) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        // matrices: (keys 16kv2 + 0..7, dims 16dp..+7), (keys +8..15, same), (keys 0..7, dims +8..15), (8..15, +8..)
        const int mi = lane >> 3, row = 16 * kv2 + (mi & 1) * 8 + (lane & 7), ch = 2 * dp + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(ws.v) + sw_off(row, ch), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], pa[kv2][0], pa[kv2][1], pa[kv2][2], pa[kv2][3], b0, b1);
        mma_bf16(o[2 * dp + 1], pa[kv2][0], pa[kv2][1], pa[kv2][2], pa[kv2][3], b2, b3);
      }
    }
    __syncwarp();  // the smem tiles are rewritten by the next sub-tile
  }
  // row sums over the 4 lanes of a row, then the partials of rows g and g + 8
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 1);
    l_run[hr] += __shfl_xor_sync(0xffffffffu, l_run[hr], 2);
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = g + 8 * hr;
    if (r >= rows) continue;
    const int ti = r / groups, gg = r % groups;
    const int64_t prow = (((int64_t)n * d.t + ti) * d.h + h * groups + gg) * splits + split;
    float* pp = part + prow * (kD + 2);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<float2*>(pp + 8 * nt + 2 * t) = make_float2(o[nt][2 * hr], o[nt][2 * hr + 1]);
    if (t == 0) pp[kD] = m_run[hr], pp[kD + 1] = l_run[hr];
  }
}

}  // namespace

bool quest_attend_mma_supported(const pbk_quest_desc& d) { return d.t * (d.h / d.kv) <= 16; }

cudaError_t launch_quest_attend_mma(const pbk_quest_desc& d, int k, int tail, int splits, float* part,
                                    const SinkKeys& sk, cudaStream_t st) {
  const size_t smem = sizeof(WarpSmem) * kWarps;
  cudaError_t e = cudaFuncSetAttribute(quest_attend_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  quest_attend_mma_kernel<<<dim3((splits + kWarps - 1) / kWarps, d.nq * d.kv), 32 * kWarps, smem, st>>>(
      d, k, tail, splits, part, sk);
  return cudaGetLastError();
}

}  // namespace pbk
