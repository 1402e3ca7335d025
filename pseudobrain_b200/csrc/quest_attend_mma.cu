// Split-key exact attention of the Quest path on tensor cores (mma.sync m16n8k16, bf16 in,
// fp32 accumulate): the same virtual keys, masks and workspace partials as the SIMT
// quest_attend_kernel in quest.cu, for up to 16 query rows per key head.
//
// A warp owns one split of S virtual keys (S a multiple of 16 in [256, 512], chosen per
// launch so that the grid fills one wave of resident blocks where it can) and walks it in
// tiles of 16 keys through a two-stage ring: while the math runs on tile s, the cp.async
// copies of tile s + 1 are in flight (16-byte chunks, XOR swizzled so ldmatrix reads are
// conflict-free; window keys' positions ride along as 4-byte copies). The split's key
// indices are resolved once, before the first copy. S = Q K^T comes from ldmatrix'ed K and
// Q fragments held in registers, the online softmax (base 2, rows g and g + 8 of the warp's
// 16-row tile) rescales the running O only when a row maximum rose, and O += P V reuses
// S's accumulator layout as the P operand with V read by ldmatrix.trans. The warp writes
// (m, l, O) for its split; the combine kernel merges the splits.
#include <cuda_bf16.h>

#include "common.cuh"
#include "quest.cuh"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kD = 128;
constexpr int kMinSplit = 256;  // = the SIMT kernel's split: the workspace holds its count
constexpr int kMaxSplit = 512;
constexpr int kTile = 16;       // keys per stage
constexpr int kStages = 2;
constexpr int kWarps = 4;
constexpr int kSinkTag = -(1 << 30);  // same key encoding as quest.cu

// A warp's staging ring for head dim D: row r at r * 2D bytes, 16-byte chunk c at (c ^ (r & 7)).
template <int D>
struct WarpSmemT {
  uint8_t k[kStages][kTile * D * 2];
  uint8_t v[kStages][kTile * D * 2];
  int kpos[kStages][kTile];  // window keys' positions (for the mask)
  int kidx[kMaxSplit];       // the split's key indices (encoding as in quest.cu)
};
using WarpSmem = WarpSmemT<kD>;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
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
// byte offset of 16-byte chunk c of row r in a swizzled tile of 2D-byte rows
template <int D = kD>
__device__ __forceinline__ uint32_t sw_off(int r, int c) { return r * (2 * D) + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ bool visible(int kp, int qp, int window, int sinks) {
  return kp <= qp && ((qp - kp) < window || kp < sinks);
}

// Key index of virtual key vj of key head h of query n (vj < the part's length).
__device__ __forceinline__ int key_index(const pbk_quest_desc& d, int k, const SinkKeys& sk, bool win, int vj, int n,
                                         int h) {
  if (win) return -1 - vj;
  if (vj < sk.n) return kSinkTag - vj;
  const int r = vj - sk.n;
  if (r < k * d.page) return d.pages[((int64_t)n * d.kv + h) * k + r / d.page] * d.page + r % d.page;
  return (d.n_arch / d.page) * d.page + (r - k * d.page);
}

// Tile s of the warp's split into stage b: 16 key and 16 value rows of 16 chunks (8 of each
// per lane), and the window keys' positions; rows past the split are zeroed (their
// probabilities are 0, and 0 * (stale bits) could be NaN). One cp.async group per tile.
template <int D>
__device__ __forceinline__ void stage_tile(WarpSmemT<D>& ws, int s, int b, int lane, const pbk_quest_desc& d,
                                           const SinkKeys& sk, int h) {
  constexpr int kChunks = D / 8;  // 16-byte chunks per row
  const bf16* keys = reinterpret_cast<const bf16*>(d.keys);
  const bf16* vals = reinterpret_cast<const bf16*>(d.values);
  const bf16* wkeys = reinterpret_cast<const bf16*>(d.win_keys);
  const bf16* wvals = reinterpret_cast<const bf16*>(d.win_values);
#pragma unroll
  for (int it = 0; it < kTile * kChunks / 32; ++it) {
    const int c = it * 32 + lane, r = c / kChunks, ch = c % kChunks;
    const int idx = ws.kidx[s * kTile + r];
    const uint32_t ko = smem_u32(ws.k[b]) + sw_off<D>(r, ch), vo = smem_u32(ws.v[b]) + sw_off<D>(r, ch);
    if (idx == INT32_MIN) {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(ko), "r"(0u) : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vo), "r"(0u) : "memory");
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
    cp_async16(ko, kr + 8 * ch);
    cp_async16(vo, vr + 8 * ch);
  }
  if (lane < kTile) {
    const int idx = ws.kidx[s * kTile + lane];
    if (idx < 0 && idx > kSinkTag) cp_async4(smem_u32(&ws.kpos[b][lane]), d.kpos + (-1 - idx));
    else ws.kpos[b][lane] = 0;
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(32 * kWarps, 3)
    quest_attend_mma_kernel(const pbk_quest_desc d, int k, int tail, int split_keys, int sr, int splits, float* part,
                            SinkKeys sk, int task0, int task_end) {
  extern __shared__ __align__(16) uint8_t attn_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpSmem& ws = reinterpret_cast<WarpSmem*>(attn_raw)[warp];
  // tasks: the retrieved splits of every (query, key head), then their window splits
  const int task = task0 + blockIdx.x * kWarps + warp;
  if (task >= task_end) return;
  const int ret_tasks = d.nq * d.kv * sr, sw = splits - sr;
  int split, pair;
  if (task < ret_tasks) {
    split = task % sr;
    pair = task / sr;
  } else {
    split = sr + (task - ret_tasks) % sw;
    pair = (task - ret_tasks) / sw;
  }
  const int n = pair / d.kv, h = pair % d.kv;
  const int g = lane >> 2, t = lane & 3;
  const int groups = d.h / d.kv, rows = d.t * groups;
  const int n_ret = sk.n + k * d.page + tail;
  const bool win_split = split >= sr;
  const int j0 = win_split ? (split - sr) * split_keys : split * split_keys;
  const int nkeys = min(split_keys, (win_split ? d.n_win : n_ret) - j0);
  const int ntiles = (nkeys + kTile - 1) / kTile;
  const bf16* q = reinterpret_cast<const bf16*>(d.q);
  const float sl2 = d.scale * 1.4426950408889634f;

  // the split's key indices; keys past the split (up to the tile edge) are INT32_MIN: masked,
  // rows zero
  for (int i = lane; i < ntiles * kTile; i += 32)
    ws.kidx[i] = i < nkeys ? key_index(d, k, sk, win_split, j0 + i, n, h) : INT32_MIN;
  __syncwarp();

  auto issue = [&](int s, int b) { stage_tile(ws, s, b, lane, d, sk, h); };

  // Q fragments (rows g and g + 8 of the 16-row tile; rows past `rows` are zero): for k-step
  // kk, a0 = (g, 16kk + 2t..), a1 = (g + 8, ..), a2 = (g, 16kk + 8 + 2t..), a3 = (g + 8, ..)
  issue(0, 0);
  if (ntiles > 1) issue(1, 1);
  else cp_async_commit();
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

  for (int s = 0; s < ntiles; ++s) {
    const int b = s & 1;
    cp_async_wait_prev();  // tile s's group is complete (only tile s + 1's may be pending)
    __syncwarp();
    const uint32_t kb = smem_u32(ws.k[b]), vb = smem_u32(ws.v[b]);
    // S = Q K^T for the tile's 2 n-tiles of 8 keys; even and odd k-steps accumulate apart
    // (two independent chains per n-tile)
    float sc[2][4], sc2[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] = sc2[j][e] = 0.f;
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {  // two k-steps (32 dims) per ldmatrix.x4
        // matrices: (keys 8j.., dims 32kq + 0..7 | 8..15 | 16..23 | 24..31); lane -> row
        const int mi = lane >> 3, row = 8 * j + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + sw_off(row, 4 * kq + mi), b0, b1, b2, b3);
        mma_bf16(sc[j], qa[2 * kq][0], qa[2 * kq][1], qa[2 * kq][2], qa[2 * kq][3], b0, b1);
        mma_bf16(sc2[j], qa[2 * kq + 1][0], qa[2 * kq + 1][1], qa[2 * kq + 1][2], qa[2 * kq + 1][3], b2, b3);
      }
    }
    // mask, scale (base 2), online softmax per row (g: elements 0,1; g + 8: elements 2,3)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = 8 * j + 2 * t + (e & 1), hr = e >> 1;
        const int idx = ws.kidx[s * kTile + key];
        bool vis = idx != INT32_MIN;
        if (vis && idx < 0 && idx > kSinkTag) vis = visible(ws.kpos[b][key], qpos_r[hr], d.window, d.sinks);
        const float x = vis ? (sc[j][e] + sc2[j][e]) * sl2 : -INFINITY;
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
    uint32_t pa[4];  // P as the A fragment of the tile's one 16-key k-step
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = m_run[e >> 1];
        p[e] = m == -INFINITY ? 0.f : exp2f(sc[j][e] - m);
        ls[e >> 1] += p[e];
      }
      // n-tile j covers keys 8j..: the low (j = 0) or high (j = 1) half of the k-step
      pa[j * 2 + 0] = pack_bf16(p[0], p[1]);
      pa[j * 2 + 1] = pack_bf16(p[2], p[3]);
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) l_run[hr] = l_run[hr] * fac[hr] + ls[hr];
    if (__any_sync(0xffffffffu, fac[0] != 1.f || fac[1] != 1.f)) {
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][0] *= fac[0];
        o[nt][1] *= fac[0];
        o[nt][2] *= fac[1];
        o[nt][3] *= fac[1];
      }
    }
    // O += P V: n-tile pairs (dims 16 dp..)
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      // matrices: (keys 0..7, dims 16dp..+7), (keys 8..15, same), (keys 0..7, dims +8..15), (8..15, +8..)
      const int mi = lane >> 3, row = (mi & 1) * 8 + (lane & 7), ch = 2 * dp + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vb + sw_off(row, ch), b0, b1, b2, b3);
      mma_bf16(o[2 * dp], pa[0], pa[1], pa[2], pa[3], b0, b1);
      mma_bf16(o[2 * dp + 1], pa[0], pa[1], pa[2], pa[3], b2, b3);
    }
    __syncwarp();  // stage b is rewritten by tile s + 2
    if (s + 2 < ntiles) issue(s + 2, b);
    else cp_async_commit();  // an empty group keeps "all but the newest" meaning tile s + 1
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


__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// Up to 8 query rows per task: the keys are the MMA's M dimension. S^T = K Q^T (m16n8k16: A = a
// 16-key tile by ldmatrix, B = Q^T fragments in registers, 8 rows as N), the online softmax
// runs per row over the key lanes, P^T goes from the accumulator layout to the B layout of
// the next product with two movmatrix transposes, and O^T += V^T P^T (A = V^T by
// ldmatrix.trans, 8 m-tiles of 16 dims). Half the MMAs of the 16-row kernel for these
// shapes, and a quarter of its O registers. A window task serves every query of a
// group of qpg = 8 / rows-per-query queries at once: the window keys are the same for all
// queries of a key head (only the mask differs), so they are staged once per group.
template <int D>
__global__ void __launch_bounds__(32 * kWarps, D == 128 ? 3 : 1)
    quest_attend_n8_kernel(const pbk_quest_desc d, int k, int tail, int split_keys, int sr, int sw, int qpg,
                           float* part, SinkKeys sk, int task0, int task_end) {
  constexpr int kK = D / 16;  // k-steps of S^T = K Q^T, m-tiles of O^T
  extern __shared__ __align__(16) uint8_t attn_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpSmemT<D>& ws = reinterpret_cast<WarpSmemT<D>*>(attn_raw)[warp];
  const int task = task0 + blockIdx.x * kWarps + warp;
  const int ret_tasks = d.nq * d.kv * sr;
  if (task >= task_end) return;
  const bool win_split = task >= ret_tasks;
  int n0, h, split, nqt;  // first query, key head, split index, queries in the task
  if (!win_split) {
    split = task % sr;
    n0 = task / sr / d.kv;
    h = task / sr % d.kv;
    nqt = 1;
  } else {
    const int wt = task - ret_tasks;
    split = sr + wt % sw;
    n0 = wt / sw / d.kv * qpg;
    h = wt / sw % d.kv;
    nqt = min(qpg, d.nq - n0);
  }
  const int g = lane >> 2, t = lane & 3;
  const int groups = d.h / d.kv, rpq = d.t * groups, rows = nqt * rpq;
  const int n_ret = sk.n + k * d.page + tail;
  const int j0 = (win_split ? split - sr : split) * split_keys;
  const int nkeys = min(split_keys, (win_split ? d.n_win : n_ret) - j0);
  const int ntiles = (nkeys + kTile - 1) / kTile;
  const bf16* q = reinterpret_cast<const bf16*>(d.q);
  const float sl2 = d.scale * 1.4426950408889634f;

  for (int i = lane; i < ntiles * kTile; i += 32)
    ws.kidx[i] = i < nkeys ? key_index(d, k, sk, win_split, j0 + i, n0, h) : INT32_MIN;
  __syncwarp();
  auto issue = [&](int s, int b) { stage_tile(ws, s, b, lane, d, sk, h); };
  issue(0, 0);
  if (ntiles > 1) issue(1, 1);
  else cp_async_commit();

  // row r of the task: query n0 + r / rpq, token (r % rpq) / groups, head h groups + r % groups
  auto row_q = [&](int r) {
    const int n = n0 + r / rpq, rem = r % rpq;
    return q + n * d.q_stride_n + (rem / groups) * d.q_stride_t + (int64_t)(h * groups + rem % groups) * d.q_stride_h;
  };
  auto row_pos = [&](int r) { return d.qpos[(n0 + r / rpq) * d.t + (r % rpq) / groups]; };
  // Q^T fragments (B: k = dims, n = row g): b0 = Q[g][16kk + 2t..], b1 = Q[g][16kk + 8 + 2t..]
  uint32_t qb[kK][2];
  {
    const bool ok = g < rows;
    const bf16* qr = ok ? row_q(g) : q;
#pragma unroll
    for (int kk = 0; kk < kK; ++kk) {
      qb[kk][0] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 2 * t) : 0u;
      qb[kk][1] = ok ? *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8 + 2 * t) : 0u;
    }
  }
  int qp[2];  // positions of this lane's rows 2t, 2t + 1
#pragma unroll
  for (int e = 0; e < 2; ++e) qp[e] = 2 * t + e < rows ? row_pos(2 * t + e) : 0;

  float o[kK][4];  // O^T: dims 16 mt + g (+ 8) x rows 2t, 2t + 1
#pragma unroll
  for (int mt = 0; mt < kK; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // rows 2t, 2t + 1 (lane partial l)

  for (int s = 0; s < ntiles; ++s) {
    const int b = s & 1;
    cp_async_wait_prev();
    __syncwarp();
    const uint32_t kb = smem_u32(ws.k[b]), vb = smem_u32(ws.v[b]);
    // S^T = K Q^T: keys g, g + 8 (c0/c1 and c2/c3) x rows 2t, 2t + 1; even and odd k-steps apart
    float sc[4] = {0.f, 0.f, 0.f, 0.f}, sc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < kK; ++kk) {
      // matrices: (keys 0-7, dims 16kk..+7), (keys 8-15, same), (keys 0-7, +8..15), (keys 8-15, +8..15)
      const int mi = lane >> 3, row = (mi & 1) * 8 + (lane & 7);
      uint32_t a0, a1, a2, a3;
      ldsm_x4(kb + sw_off<D>(row, 2 * kk + (mi >> 1)), a0, a1, a2, a3);
      if (kk & 1) mma_bf16(sc2, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      else mma_bf16(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = g + 8 * (e >> 1), r = e & 1;
      const int idx = ws.kidx[s * kTile + key];
      bool vis = idx != INT32_MIN;
      if (vis && idx < 0 && idx > kSinkTag) vis = visible(ws.kpos[b][key], qp[r], d.window, d.sinks);
      const float x = vis ? (sc[e] + sc2[e]) * sl2 : -INFINITY;
      sc[e] = x;
      mx[r] = fmaxf(mx[r], x);
    }
    float fac[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {  // max over the 8 key lanes (g) of each row
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 4));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 8));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 16));
      const float m_new = fmaxf(m_run[r], mx[r]);
      fac[r] = m_run[r] == -INFINITY ? 0.f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float m = m_run[e & 1];
      p[e] = m == -INFINITY ? 0.f : exp2f(sc[e] - m);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * fac[r] + (p[r] + p[2 + r]);
    if (__any_sync(0xffffffffu, fac[0] != 1.f || fac[1] != 1.f)) {
#pragma unroll
      for (int mt = 0; mt < kK; ++mt) {
        o[mt][0] *= fac[0];
        o[mt][1] *= fac[1];
        o[mt][2] *= fac[0];
        o[mt][3] *= fac[1];
      }
    }
    // P^T (keys x rows) in the accumulator layout -> B fragments (k = keys 2t.., n = row g)
    const uint32_t pb0 = movmatrix_t(pack_bf16(p[0], p[1])), pb1 = movmatrix_t(pack_bf16(p[2], p[3]));
    // O^T += V^T P^T: A = V^T (dims 16 mt .. x keys) by ldmatrix.trans of the V rows
#pragma unroll
    for (int mt = 0; mt < kK; ++mt) {
      // matrices: (keys 0-7, dims 16mt..+7), (keys 0-7, +8..15), (keys 8-15, ..+7), (keys 8-15, +8..15)
      const int mi = lane >> 3, row = (mi >> 1) * 8 + (lane & 7), ch = 2 * mt + (mi & 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vb + sw_off<D>(row, ch), a0, a1, a2, a3);
      mma_bf16(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();  // stage b is rewritten by tile s + 2
    if (s + 2 < ntiles) issue(s + 2, b);
    else cp_async_commit();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {  // row sums over the 8 key lanes
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 4);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 8);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 16);
  }
  const int splits = sr + sw;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = 2 * t + e;
    if (r >= rows) continue;
    const int n = n0 + r / rpq, rem = r % rpq, ti = rem / groups, gg = rem % groups;
    const int64_t prow = (((int64_t)n * d.t + ti) * d.h + h * groups + gg) * splits + split;
    float* pp = part + prow * (D + 2);
#pragma unroll
    for (int mt = 0; mt < kK; ++mt) {
      pp[16 * mt + g] = o[mt][e];
      pp[16 * mt + 8 + g] = o[mt][2 + e];
    }
    if (g == 0) pp[D] = m_run[e], pp[D + 1] = l_run[e];
  }
}

}  // namespace

// Head dim 128: up to 16 query rows per key head (8-row and 16-row kernels); head dim 256: up
// to 8 (the 8-row kernel).
bool quest_attend_mma_supported(const pbk_quest_desc& d) {
  const int rpq = d.t * (d.h / d.kv);
  return (d.d == 128 && rpq <= 16) || (d.d == 256 && rpq <= 8);
}

// Split length S in [256, 512] (a multiple of 16) that minimises waves x S, the launch's
// length in key tiles: with `slots` resident blocks, the fewest waves, then the shortest
// splits. Returns the number of splits per (query, key head) through *splits_out.
static int slots_for(const void* kernel, size_t smem, cudaError_t* err) {
  static int slots[3][64] = {};  // resident blocks per device (SMs x blocks per SM), per kernel
  const int which = kernel == (const void*)quest_attend_n8_kernel<128> ? 1
                    : kernel == (const void*)quest_attend_n8_kernel<256> ? 2 : 0;
  int dev = 0;
  if ((*err = cudaGetDevice(&dev)) != cudaSuccess) return 0;
  if (dev >= 64) return 148;
  if (slots[which][dev] == 0) {
    int sms = 0, per_sm = 0;
    if ((*err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return 0;
    if ((*err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32 * kWarps, smem)) != cudaSuccess)
      return 0;
    slots[which][dev] = sms * (per_sm > 0 ? per_sm : 1);
  }
  return slots[which][dev];
}

cudaError_t launch_quest_attend_mma(const pbk_quest_desc& d, int k, int tail, float* part, const SinkKeys& sk,
                                    int parts, int* splits_out, cudaStream_t st) {
  const bool wide = d.d == 256;
  const size_t smem = (wide ? sizeof(WarpSmemT<256>) : sizeof(WarpSmem)) * kWarps;
  const int rpq = d.t * (d.h / d.kv);
  const bool n8 = rpq <= 8;
  const void* kernel = wide ? (const void*)quest_attend_n8_kernel<256>
                       : n8 ? (const void*)quest_attend_n8_kernel<128> : (const void*)quest_attend_mma_kernel;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int slots = slots_for(kernel, smem, &e);
  if (e != cudaSuccess) return e;
  // Split length S in [256, 512] (a multiple of 16) that minimises waves x S, the launch's
  // length in key tiles: with `slots` resident blocks, the fewest waves, then the shortest
  // splits. The 8-row kernel's window tasks serve qpg queries each. A function of d only, so
  // launches of the retrieved and the window tasks apart agree on it.
  const int n_ret = sk.n + k * d.page + tail;
  const int qpg = n8 ? 8 / rpq : 1;
  const int64_t pairs = (int64_t)d.nq * d.kv, wpairs = (int64_t)((d.nq + qpg - 1) / qpg) * d.kv;
  int best = kMinSplit;
  int64_t best_cost = INT64_MAX;
  for (int sl = kMinSplit; sl <= kMaxSplit; sl += kTile) {
    const int64_t tasks = pairs * ((n_ret + sl - 1) / sl) + wpairs * ((d.n_win + sl - 1) / sl);
    const int64_t blocks = (tasks + kWarps - 1) / kWarps;
    const int64_t cost = (blocks + slots - 1) / slots * sl;
    if (cost < best_cost) best_cost = cost, best = sl;
  }
  const int sr = (n_ret + best - 1) / best, sw = (d.n_win + best - 1) / best;
  *splits_out = sr + sw;
  const int ret_tasks = (int)(pairs * sr), all_tasks = (int)(pairs * sr + wpairs * sw);
  const int task0 = (parts & 1) ? 0 : ret_tasks, task_end = (parts & 2) ? all_tasks : ret_tasks;
  if (task_end <= task0) return cudaSuccess;
  const unsigned blocks = (unsigned)((task_end - task0 + kWarps - 1) / kWarps);
  if (wide)
    quest_attend_n8_kernel<256><<<blocks, 32 * kWarps, smem, st>>>(d, k, tail, best, sr, sw, qpg, part, sk, task0,
                                                                   task_end);
  else if (n8)
    quest_attend_n8_kernel<128><<<blocks, 32 * kWarps, smem, st>>>(d, k, tail, best, sr, sw, qpg, part, sk, task0,
                                                                   task_end);
  else
    quest_attend_mma_kernel<<<blocks, 32 * kWarps, smem, st>>>(d, k, tail, best, sr, sr + sw, part, sk, task0,
                                                               task_end);
  return cudaGetLastError();
}

}  // namespace pbk
