// Quest page-bounded exact memory: page bounds, page scores, exact top-k page
// selection, page gather and split-key exact attention (flat mode of
// pseudobrain/exact_memory.py:43-152 and the attention of pseudobrain/transplant.py:612-628).
#include <cfloat>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "quest.cuh"

namespace pbk {
namespace {

// Head dims of the tensor-core score path and of the top-k's refinement (which only runs on
// tensor-core scores); the SIMT kernels below take the head dim as a template parameter
// (128 or 256).
constexpr int kD = 128;
using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 raw, float* out) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(p[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

// A row of D bf16 spread over a warp: lane l holds dims kPer l .. kPer l + kPer - 1 (kPer =
// D / 32: 4 or 8), moved as one 8- or 16-byte vector.
template <int D>
struct WarpRow {
  static constexpr int kPer = D / 32;
  using Vec = typename std::conditional<kPer == 4, uint2, uint4>::type;
  __device__ static Vec raw(const bf16* p) { return *reinterpret_cast<const Vec*>(p); }
  __device__ static void put(bf16* p, const Vec& v) { *reinterpret_cast<Vec*>(p) = v; }
  __device__ static void unpack(const Vec& v, float (&x)[kPer]) {
    const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < kPer / 2; ++i) {
      const float2 f = __bfloat1622float2(pr[i]);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
  __device__ static Vec pack(const float (&x)[kPer]) {
    Vec v;
    uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
    for (int i = 0; i < kPer / 2; ++i) w[i] = bf16x2_bits(x[2 * i], x[2 * i + 1]);
    return v;
  }
  __device__ static void load(const bf16* p, float (&x)[kPer]) { unpack(raw(p), x); }
  __device__ static void store(bf16* p, const float (&x)[kPer]) { put(p, pack(x)); }
};

// ---------------------------------------------------------------------------------
// Page bounds: one warp per (page, key head); lane l owns dims kPer l .. kPer l + kPer - 1.
// ---------------------------------------------------------------------------------
template <int D>
__global__ void quest_bounds_kernel(const bf16* keys, int n, int page, int64_t ks_kv, int64_t ks_n, bf16* kmax,
                                    bf16* kmin, int64_t bs_kv, int64_t bs_p, int first_page, int npages) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= npages) return;
  const int p = first_page + warp, h = blockIdx.y;
  const int t0 = p * page, t1 = min(t0 + page, n);
  float mx[P], mn[P], v[P];
#pragma unroll
  for (int i = 0; i < P; ++i) mx[i] = -FLT_MAX, mn[i] = FLT_MAX;
  for (int t = t0; t < t1; ++t) {
    R::load(keys + h * ks_kv + (int64_t)t * ks_n + P * lane, v);
#pragma unroll
    for (int i = 0; i < P; ++i) mx[i] = fmaxf(mx[i], v[i]), mn[i] = fminf(mn[i], v[i]);
  }
  // max/min of bf16 values are bf16 values: exact
  R::store(kmax + h * bs_kv + (int64_t)p * bs_p + P * lane, mx);
  R::store(kmin + h * bs_kv + (int64_t)p * bs_p + P * lane, mn);
}

// ---------------------------------------------------------------------------------
// Page scores. Thread = page; the group's query rows sit in shared memory as fp32.
// score[n][kv][p] = max over rows r of group n of sum_d q_rd * (q_rd > 0 ? kmax_pd : kmin_pd)
// (each product of two bf16 values is exact in fp32).
// ---------------------------------------------------------------------------------
constexpr int kScoreThreads = 128;
constexpr int kRowBlock = 4;

template <int D>
__global__ void __launch_bounds__(kScoreThreads) quest_score_kernel(const pbk_quest_desc d, int npages, float* scores,
                                                                   float* segmax, int nseg) {
  extern __shared__ __align__(16) float qs[];  // [rows of one key head][D]
  const int h = blockIdx.y, groups = d.h / d.kv, rows_per_group = d.t * groups;
  const int rows = d.nq * rows_per_group;
  for (int e = threadIdx.x; e < rows * D; e += kScoreThreads) {
    const int r = e / D, dd = e % D;
    const int n = r / rows_per_group, rem = r % rows_per_group, ti = rem / groups, g = rem % groups;
    const bf16* qp = reinterpret_cast<const bf16*>(d.q) + n * d.q_stride_n + ti * d.q_stride_t +
                     (int64_t)(h * groups + g) * d.q_stride_h;
    qs[e] = __bfloat162float(qp[dd]);
  }
  __syncthreads();
  const int p = blockIdx.x * kScoreThreads + threadIdx.x;
  const bool valid = p < npages;
  const int pc = valid ? p : npages - 1;  // invalid lanes compute on a valid page, then drop it
  const bf16* bmax = reinterpret_cast<const bf16*>(d.kmax) + h * d.bnd_stride_kv + (int64_t)pc * d.bnd_stride_p;
  const bf16* bmin = reinterpret_cast<const bf16*>(d.kmin) + h * d.bnd_stride_kv + (int64_t)pc * d.bnd_stride_p;
  for (int n = 0; n < d.nq; ++n) {
    float best = -INFINITY;
    for (int r0 = 0; r0 < rows_per_group; r0 += kRowBlock) {
      const int nr = min(kRowBlock, rows_per_group - r0);
      const float* qb = qs + (n * rows_per_group + r0) * D;
      float acc[kRowBlock] = {0.f, 0.f, 0.f, 0.f};
      for (int d0 = 0; d0 < D; d0 += 8) {
        float mx[8], mn[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmax + d0), mx);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmin + d0), mn);
#pragma unroll
        for (int r = 0; r < kRowBlock; ++r) {
          if (r < nr) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float qv = qb[r * D + d0 + j];
              acc[r] = fmaf(qv, qv > 0.f ? mx[j] : mn[j], acc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRowBlock; ++r)
        if (r < nr) best = fmaxf(best, acc[r]);
    }
    if (valid) scores[((int64_t)n * d.kv + h) * npages + p] = best;
    if (segmax != nullptr) {  // max over this warp's 32 consecutive pages
      float m = valid ? best : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if ((threadIdx.x & 31) == 0 && (p >> 5) < nseg) segmax[((int64_t)n * d.kv + h) * nseg + (p >> 5)] = m;
    }
  }
}

// ---------------------------------------------------------------------------------
// Exact top-k per row (one CTA per (group, key head)): radix select over the order-
// preserving 32-bit keys of the fp32 scores, one 8-bit digit per pass, then one pass
// that writes the selected page indices in ascending order (ties at the threshold go
// to the lowest indices).
// ---------------------------------------------------------------------------------
constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kSegMinPages = 1024;  // rows this long get segment maxima and the candidate path

__device__ __forceinline__ uint32_t ordered_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int N>
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  // scratch: >= N/32 + 1 ints
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < N / 32 ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < N / 32) scratch[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int base = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[N / 32 - 1];
  __syncthreads();
  return base + x - v;
}

// Radix select over n keys key_of(i): the k-th largest key (`prefix` on return) and how
// many elements equal to it belong to the top k (`kk`). Three digits (11, 11, 10 bits),
// warp-aggregated shared-memory histograms; each digit's bin comes from a block-wide scan
// of the bin counts (thread t owns 2 or 1 consecutive bins, highest bins first).
constexpr int kBins = 2048;
struct SelectSmem {
  uint32_t hist[kBins];
  uint32_t prefix, kk;
  int warp_tot[2][kTopkWarps];
};

// With passes = 2 only the top 22 bits are resolved: `prefix` (low 10 bits zero) is then a
// lower bound of the k-th largest key, tight to 2^-13 relative for finite scores.
template <typename KeyOf>
__device__ __forceinline__ void radix_select(KeyOf key_of, int n, uint32_t k, SelectSmem& ss, uint32_t& prefix_out,
                                             uint32_t& kk_out, int passes = 3) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0, mask = 0, kk = k;
  const int shifts[3] = {21, 10, 0}, widths[3] = {11, 11, 10};
#pragma unroll
  for (int pass = 0; pass < 3; ++pass) {
    if (pass >= passes) break;
    const int shift = shifts[pass];
    const uint32_t dmask = (1u << widths[pass]) - 1u;
    const int nb = 1 << widths[pass];
    for (int i = tid; i < kBins; i += kTopkThreads) ss.hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += kTopkThreads) {
      const int i = base + tid;
      uint32_t bin = 0xFFFFFFFFu;
      if (i < n) {
        const uint32_t u = key_of(i);
        if ((u & mask) == prefix) bin = (u >> shift) & dmask;
      }
      const uint32_t same = __match_any_sync(0xffffffffu, bin);
      if (bin != 0xFFFFFFFFu && lane == __ffs(same) - 1) atomicAdd(&ss.hist[bin], (uint32_t)__popc(same));
    }
    if (tid == 0) {  // default, overwritten below whenever the count reaches kk
      ss.prefix = prefix;
      ss.kk = kk;
    }
    __syncthreads();
    // thread tid owns the `per` bins from hi = nb - 1 - per * tid down (highest bins first):
    // a block-wide scan of the per-thread counts finds the bin holding the kk-th largest key
    const int per = nb / kTopkThreads;
    const int hi = nb - 1 - per * tid;
    int own = 0;
    for (int j = 0; j < per; ++j) own += (int)ss.hist[hi - j];
    int total;
    const uint32_t excl = (uint32_t)block_exclusive_scan<kTopkThreads>(own, ss.warp_tot[0], &total);
    if (excl < kk && kk <= excl + (uint32_t)own) {
      uint32_t above = excl;
      int b = hi;
      for (int j = 0; j < per - 1; ++j, --b) {
        if (above + ss.hist[b] >= kk) break;
        above += ss.hist[b];
      }
      ss.prefix = prefix | ((uint32_t)b << shift);
      ss.kk = kk - above;
    }
    __syncthreads();
    prefix = ss.prefix;
    kk = ss.kk;
    mask |= dmask << shift;
    __syncthreads();
  }
  prefix_out = prefix;
  kk_out = kk;
}

// Warp-contiguous ranges: warp w owns [w R, (w+1) R) of n elements, read 32 at a time
// (coalesced); R = ceil(n / warps) rounded up to a multiple of 32.
__device__ __forceinline__ int warp_range(int n) { return ((n + kTopkWarps - 1) / kTopkWarps + 31) / 32 * 32; }

// Exclusive prefix over the 32 warps of per-warp totals a (and b); returns this warp's bases.
__device__ __forceinline__ void warp_bases(int a, int b, SelectSmem& ss, int& base_a, int& base_b, int& tot_a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    ss.warp_tot[0][warp] = a;
    ss.warp_tot[1][warp] = b;
  }
  __syncthreads();
  // every warp scans the warp totals itself (lane l holds warp l's): inclusive sums by shuffles
  int x = lane < kTopkWarps ? ss.warp_tot[0][lane] : 0, y = lane < kTopkWarps ? ss.warp_tot[1][lane] : 0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int tx = __shfl_up_sync(0xffffffffu, x, o), ty = __shfl_up_sync(0xffffffffu, y, o);
    if (lane >= o) x += tx, y += ty;
  }
  base_a = __shfl_sync(0xffffffffu, x, warp) - a;
  base_b = __shfl_sync(0xffffffffu, y, warp) - b;
  tot_a = __shfl_sync(0xffffffffu, x, 31);
  __syncthreads();
}

// Write the top-k of n elements given in ascending index order (key_of(i), idx_of(i)) to
// out[0..k) in that order: an element's output position is (#greater before it) +
// min(#equal before it, kk), so ties at the threshold go to the lowest indices.
template <typename KeyOf, typename IdxOf>
__device__ __forceinline__ void collect_in_order(KeyOf key_of, IdxOf idx_of, int n, uint32_t prefix, uint32_t kk,
                                                 SelectSmem& ss, int32_t* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int R = warp_range(n);
  const int lo = min(warp * R, n), hi = min(lo + R, n);
  int n_gt = 0, n_eq = 0;
  for (int j = lo; j < hi; j += 32) {
    const int i = j + lane;
    const uint32_t u = i < hi ? key_of(i) : 0u;
    n_gt += __popc(__ballot_sync(0xffffffffu, i < hi && u > prefix));
    n_eq += __popc(__ballot_sync(0xffffffffu, i < hi && u == prefix));
  }
  int gt_before, eq_before, unused;
  warp_bases(n_gt, n_eq, ss, gt_before, eq_before, unused);
  for (int j = lo; j < hi; j += 32) {
    const int i = j + lane;
    const uint32_t u = i < hi ? key_of(i) : 0u;
    const bool gt = i < hi && u > prefix, eq = i < hi && u == prefix;
    const uint32_t bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    const int g_rank = gt_before + __popc(bg & lt), e_rank = eq_before + __popc(be & lt);
    if (gt) out[g_rank + min(e_rank, (int)kk)] = idx_of(i);
    else if (eq && e_rank < (int)kk) out[g_rank + e_rank] = idx_of(i);
    gt_before += __popc(bg);
    eq_before += __popc(be);
  }
}

constexpr int kCandCap = 4096;  // candidates held in shared memory
constexpr int kSegCap = 4096;   // segment maxima held in shared memory (131072 pages)
constexpr int kSegRegs = 16;    // candidate segments a warp keeps in registers per pass
constexpr int kRefineRows = 64; // query rows per (group, key head) the refinement holds (the tensor-core limit)

// Canonical page score: the maximum over a group's query rows r of
//   fl( ... fl(fl(t_r0 + 0) + t_r1) ... + t_r127 ),  t_rd = q_rd * (q_rd > 0 ? kmax_d : kmin_d),
// an fp32 sum in dimension order 0..127 (each product of two bf16 values is exact in fp32, so an
// fma chain and a multiply-then-add chain agree bit for bit). The SIMT score, candidate and
// rerank kernels produce it directly. The tensor-core scores differ from it by at most
// c ||q_r||_1 max|bound| (the rounding of both sums); the top-k re-scores, in this order, every
// page within twice that of its threshold, so every selection is exactly the selection of the
// canonical scores, which a CPU restatement reproduces bit for bit.
struct RefineArgs {
  const bf16* q;             // null: the scores are canonical already (no refinement)
  int64_t q_stride_n, q_stride_t, q_stride_h;
  const bf16* kmax;
  const bf16* kmin;
  int64_t bnd_stride_kv, bnd_stride_p;
  const float* tile_abs;     // [kv][abs_per_kv] largest |bound| per tile part (the score kernel's)
  int abs_per_kv;
  int kv, groups, t;
};

// Relative weight of the error bound. Each page score is a sum of 256 exact products whose
// magnitudes add up to at most U = ||q_r||_1 max|bound|. Every partial sum, and so every
// rounding step, is at most U in magnitude; the tensor cores round each of the 256 additions
// once (possibly by truncation: one ulp), so their sum differs from the exact one by at most
// 256 * 2^-23 U = 2^-15 U, and the canonical fp32 sum by at most 128 * 2^-24 U = 2^-17 U.
// 2^-14 U covers both (1.25 * 2^-15 U) with a margin of 1.6; the measured difference at
// config 3 is 2^-23 U.
constexpr int kRefineEpsExp = -14;

__device__ __forceinline__ float canonical_row_sum(const float* qrow, const bf16* bmax, const bf16* bmin) {
  float acc = 0.f;
  for (int d0 = 0; d0 < kD; d0 += 16) {
    uint4 rx[2], rn[2];  // 16 dims of both bounds in flight at once
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      rx[c] = *reinterpret_cast<const uint4*>(bmax + d0 + 8 * c);
      rn[c] = *reinterpret_cast<const uint4*>(bmin + d0 + 8 * c);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float mx[8], mn[8];
      bf16x8_to_f32(rx[c], mx);
      bf16x8_to_f32(rn[c], mn);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float qv = qrow[d0 + 8 * c + j];
        acc = fmaf(qv, qv > 0.f ? mx[j] : mn[j], acc);
      }
    }
  }
  return acc;
}

__device__ __forceinline__ float ordered_key_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Canonical keys of the listed pages: ckey[u] = ordered key of the max over the rpg query
// rows of page list[u]'s canonical sum. The pages' bounds are staged in shared memory
// kStagePages at a time (one coalesced 512-byte load per page: lanes 0-15 kmax, 16-31 kmin;
// rows padded by 4 bytes so 32 pages sit in 32 banks), then one thread per (page, row) --
// pages fastest within a warp, so a warp reads one query row as a broadcast -- runs the sum
// in dimension order from shared memory.
constexpr int kStagePages = 128;
constexpr int kStageRow = 2 * kD + 2;  // bf16 per staged page: kmax | kmin | pad
__device__ __forceinline__ void canonical_keys(const RefineArgs& rf, const float (*qs)[kD], int rpg, int h,
                                               const int32_t* list, int n, uint32_t* ckey, bf16* stage) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int u = threadIdx.x; u < n; u += kTopkThreads) ckey[u] = 0u;
  for (int base = 0; base < n; base += kStagePages) {
    const int np = min(kStagePages, n - base);
    for (int u = warp; u < np; u += kTopkWarps) {
      const int64_t off = h * rf.bnd_stride_kv + (int64_t)list[base + u] * rf.bnd_stride_p + 8 * (lane & 15);
      const uint4 raw = *reinterpret_cast<const uint4*>((lane < 16 ? rf.kmax : rf.kmin) + off);
      uint32_t* dst = reinterpret_cast<uint32_t*>(stage + u * kStageRow + (lane < 16 ? 0 : kD) + 8 * (lane & 15));
      dst[0] = raw.x, dst[1] = raw.y, dst[2] = raw.z, dst[3] = raw.w;  // 4-byte stores: rows are 4-aligned
    }
    __syncthreads();
    for (int w = threadIdx.x; w < np * rpg; w += kTopkThreads) {
      const int u = w % np, r = w / np;
      const bf16* bx = stage + u * kStageRow;
      const float* qrow = qs[r];
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < kD; ++d) {
        const float qv = qrow[d];
        acc = fmaf(qv, __bfloat162float(bx[qv > 0.f ? d : kD + d]), acc);
      }
      atomicMax(&ckey[base + u], ordered_key(acc));
    }
    __syncthreads();
  }
}

// The final selection from the band: the n_in pages above it are in; of the nb band pages
// (ckey, page) the need = k - n_in best by canonical key (ties to the lowest page) join them:
// key[pos[u]] (key[u] without pos) = MAX for those, 0 for the rest. Each page's rank is the
// count of band pages ahead of it, on packed 64-bit keys (ckey high, ~page low: larger is
// better). Returns false (nothing written) when the band is too large for this pairwise count.
constexpr int kRankCap = 1024;
__device__ __forceinline__ bool rank_band(const uint32_t* ckey, const int32_t* page, int nb, int need,
                                          const int32_t* pos, uint32_t* key, uint64_t* packed) {
  if (nb > kRankCap) return false;
  for (int u = threadIdx.x; u < nb; u += kTopkThreads)
    packed[u] = ((uint64_t)ckey[u] << 32) | (uint32_t)~page[u];
  __syncthreads();
  for (int u = threadIdx.x; u < nb; u += kTopkThreads) {
    const uint64_t c = packed[u];
    int rank = 0;
#pragma unroll 8
    for (int v = 0; v < nb; ++v) rank += packed[v] > c;
    key[pos != nullptr ? pos[u] : u] = rank < need ? 0xFFFFFFFFu : 0u;
  }
  __syncthreads();
  return true;
}

struct TopkSmem {
  SelectSmem ss;
  uint32_t seg_key[kSegCap];  // ordered keys of the row's segment maxima; then canonical keys
  int32_t cseg[kSegCap];      // candidate segments, ascending; then the pages to re-score
  uint32_t cand_key[kCandCap];
  int32_t cand_idx[kCandCap];
  float qs[kRefineRows][kD];  // the row's query rows (refinement)
  int32_t band_page[kCandCap]; // pages of the band (candidate path)
  __align__(16) bf16 stage[kStagePages * kStageRow];  // staged bounds of band pages; packed rank keys
  float red[kTopkWarps];
  float qs_l1[kTopkWarps];
  float eps2;                 // twice the error bound of the row's scores
  int n_unc, n_in;
};

// The refinement's set-up, in two halves around a barrier the caller places: refine_load
// issues the loads (the group's query rows into shared memory; per warp, the largest bound
// magnitude of the key head's tiles), refine_finish forms eps2 = 2 eps,
// eps = 2^kRefineEpsExp max_r ||q_r||_1 max|bound|.
__device__ __forceinline__ void refine_load(const RefineArgs& rf, int row, TopkSmem& ts) {
  const int n = row / rf.kv, h = row % rf.kv, rpg = rf.t * rf.groups;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < rpg * kD; e += kTopkThreads) {
    const int r = e / kD, dd = e % kD, ti = r / rf.groups, g = r % rf.groups;
    ts.qs[r][dd] = __bfloat162float(rf.q[n * rf.q_stride_n + ti * rf.q_stride_t +
                                         (int64_t)(h * rf.groups + g) * rf.q_stride_h + dd]);
  }
  float babs = 0.f;
  for (int i = threadIdx.x; i < rf.abs_per_kv; i += kTopkThreads)
    babs = fmaxf(babs, rf.tile_abs[(int64_t)h * rf.abs_per_kv + i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) babs = fmaxf(babs, __shfl_xor_sync(0xffffffffu, babs, o));
  if (lane == 0) ts.red[warp] = babs;
}

__device__ __forceinline__ void refine_finish(const RefineArgs& rf, TopkSmem& ts) {
  const int rpg = rf.t * rf.groups, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this warp's largest ||q_r||_1; the product of the two maxima bounds every page
  float l1 = 0.f;
  for (int r = warp; r < rpg; r += kTopkWarps) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < kD / 32; ++j) a += fabsf(ts.qs[r][lane + 32 * j]);
    l1 = fmaxf(l1, warp_sum(a));
  }
  if (lane == 0) ts.qs_l1[warp] = l1;
  __syncthreads();
  if (threadIdx.x == 0) {
    float bm = 0.f, lm = 0.f;
    for (int w = 0; w < kTopkWarps; ++w) bm = fmaxf(bm, ts.red[w]), lm = fmaxf(lm, ts.qs_l1[w]);
    // an fp32 sum of 128 magnitudes may round below the exact sum: 2^-20 relative covers it;
    // the other steps round up, so eps2 is a bound, not an estimate
    lm = __fmul_ru(lm, 1.f + 0x1p-20f);
    ts.eps2 = __fmul_ru(2.f, ldexpf(__fmul_ru(lm, bm), kRefineEpsExp));
  }
  __syncthreads();
}

// Band of the tensor-core keys around the threshold key `prefix`: pages above hi are in the
// canonical top k whatever their rounding, pages below lo are out; the band in between is
// re-scored. -inf scores (masked pages) are exact and stay as they are.
__device__ __forceinline__ void refine_band(uint32_t prefix, float eps2, uint32_t& lo, uint32_t& hi) {
  const float tau = ordered_key_inv(prefix);
  hi = ordered_key(__fadd_ru(tau, eps2));
  lo = ordered_key(__fadd_rd(tau, -eps2));
}

// One CTA per (group, key head) row of scores. With segment maxima (the max of every 32
// consecutive pages), the k-th largest segment maximum bounds the k-th largest page score
// from below (the top k segments hold k distinct pages scoring at least that), and so does
// any tau below it (here: its top 22 bits, less the refinement band), so the top k are
// among the pages scoring >= tau, all inside segments whose maximum is >= tau. Those
// segments are listed in index order, only their pages are read (one warp-wide load per
// segment, in registers), the pages scoring >= tau are placed in index order into shared
// memory, and the exact selection runs there. When there are too few segments, too many
// segments or too many candidates, the selection runs over the whole row.
// With rf.q set (tensor-core scores), the pages within the error band of the threshold get
// their canonical scores and the final selection runs on keys: MAX for the pages above the
// band, the canonical key inside it, 0 below it (n above < k <= n above + n inside).
__global__ void __launch_bounds__(kTopkThreads) quest_topk_kernel(const float* scores, const float* segmax, int npages,
                                                                  int nseg, int k, int32_t* pages,
                                                                  const RefineArgs rf) {
  extern __shared__ __align__(16) uint8_t topk_raw[];
  TopkSmem& ts = *reinterpret_cast<TopkSmem*>(topk_raw);
  SelectSmem& ss = ts.ss;
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* s = scores + (int64_t)row * npages;
  int32_t* out = pages + (int64_t)row * k;
  const uint32_t lt = (1u << lane) - 1u;
  const bool refine = rf.q != nullptr;
  const int rh = refine ? row % rf.kv : 0, rpg = refine ? rf.t * rf.groups : 0;
  const bool seg_path = segmax != nullptr && nseg >= k && nseg <= kSegCap;
  if (refine) refine_load(rf, row, ts);
  if (seg_path) {
    const float* sg = segmax + (int64_t)row * nseg;
    for (int i = threadIdx.x; i < nseg; i += kTopkThreads) ts.seg_key[i] = ordered_key(sg[i]);
  }
  __syncthreads();
  if (refine) refine_finish(rf, ts);
  const float eps2 = refine ? ts.eps2 : 0.f;
  uint32_t prefix, kk;
  if (seg_path) {
    // tau: a lower bound of the k-th largest segment maximum (two digits: any bound at or
    // below it keeps every top-k page among the candidates, the exact select comes later),
    // lowered by the refinement band so the band's pages are candidates too
    uint32_t tau, unused;
    radix_select([&](int i) { return ts.seg_key[i]; }, nseg, (uint32_t)k, ss, tau, unused, 2);
    if (refine) {
      const float t0 = ordered_key_inv(tau);
      if (t0 != -INFINITY) tau = ordered_key(__fadd_rd(t0, -eps2));
    }
    // candidate segments (key >= tau) in index order
    {
      const int R = warp_range(nseg);
      const int lo = min(warp * R, nseg), hi = min(lo + R, nseg);
      int cnt = 0;
      for (int j = lo; j < hi; j += 32) {
        const int i = j + lane;
        cnt += __popc(__ballot_sync(0xffffffffu, i < hi && ts.seg_key[i] >= tau));
      }
      int pos, zero, total;
      warp_bases(cnt, 0, ss, pos, zero, total);
      for (int j = lo; j < hi; j += 32) {
        const int i = j + lane;
        const bool c = i < hi && ts.seg_key[i] >= tau;
        const uint32_t bc = __ballot_sync(0xffffffffu, c);
        if (c) ts.cseg[pos + __popc(bc & lt)] = i;
        pos += __popc(bc);
      }
      __syncthreads();
      // pages of the candidate segments: warp w takes candidate segments [w P, (w+1) P),
      // lane = page within the segment
      const int nc = total, P = (nc + kTopkWarps - 1) / kTopkWarps;
      const int c0 = min(warp * P, nc), c1 = min(c0 + P, nc);
      // The scores read here are kept in shared memory for the placement pass (the staging
      // area of the band's bounds is idle until then) when the candidate segments fit, so the
      // placement reads them back without a second global round trip.
      float* seg_scores = reinterpret_cast<float*>(ts.stage);
      const bool staged = nc * 32 * (int)sizeof(float) <= (int)sizeof(ts.stage);
      int pcnt = 0;
      for (int b0 = c0; b0 < c1; b0 += kSegRegs) {
        float x[kSegRegs];
#pragma unroll
        for (int u = 0; u < kSegRegs; ++u) {
          const int page = b0 + u < c1 ? ts.cseg[b0 + u] * 32 + lane : npages;
          x[u] = page < npages ? s[page] : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < kSegRegs; ++u) {
          pcnt += __popc(__ballot_sync(0xffffffffu, b0 + u < c1 && ordered_key(x[u]) >= tau &&
                                                        ts.cseg[min(b0 + u, c1 - 1)] * 32 + lane < npages));
          if (staged && b0 + u < c1) seg_scores[(b0 + u) * 32 + lane] = x[u];
        }
      }
      int ppos, pzero, ptotal;
      warp_bases(pcnt, 0, ss, ppos, pzero, ptotal);
      if (ptotal <= kCandCap) {
        for (int b0 = c0; b0 < c1; b0 += kSegRegs) {
          float x[kSegRegs];
#pragma unroll
          for (int u = 0; u < kSegRegs; ++u) {
            const int page = b0 + u < c1 ? ts.cseg[b0 + u] * 32 + lane : npages;
            x[u] = page >= npages ? -INFINITY : (staged ? seg_scores[(b0 + u) * 32 + lane] : s[page]);
          }
#pragma unroll
          for (int u = 0; u < kSegRegs; ++u) {
            const int page = b0 + u < c1 ? ts.cseg[b0 + u] * 32 + lane : npages;
            const uint32_t key = ordered_key(x[u]);
            const bool c = page < npages && key >= tau;
            const uint32_t bc = __ballot_sync(0xffffffffu, c);
            if (c) {
              const int at = ppos + __popc(bc & lt);
              ts.cand_key[at] = key;
              ts.cand_idx[at] = page;
            }
            ppos += __popc(bc);
          }
        }
        __syncthreads();
        radix_select([&](int i) { return ts.cand_key[i]; }, ptotal, (uint32_t)k, ss, prefix, kk);
        const uint32_t ninf = ordered_key(-INFINITY);
        if (refine && prefix != ninf) {  // (a -inf threshold: every finite page is in, exactly)
          // the band's pages: listed (any order) with their page indices, re-scored in the
          // canonical order; the pages above the band are counted
          uint32_t lo, hi;
          refine_band(prefix, eps2, lo, hi);
          if (threadIdx.x == 0) ts.n_unc = ts.n_in = 0;
          __syncthreads();
          for (int base = 0; base < ptotal; base += kTopkThreads) {
            const int i = base + threadIdx.x;
            const uint32_t key = i < ptotal ? ts.cand_key[i] : ninf;
            const bool above = key != ninf && key > hi;
            const uint32_t ba = __ballot_sync(0xffffffffu, above);
            if (lane == 0 && ba) atomicAdd(&ts.n_in, __popc(ba));
            if (key == ninf) continue;  // masked (or past the end): exact already
            if (above) ts.cand_key[i] = 0xFFFFFFFFu;
            else if (key >= lo) {
              const int at = atomicAdd(&ts.n_unc, 1);
              ts.cseg[at] = i;
              ts.band_page[at] = ts.cand_idx[i];
            } else {
              ts.cand_key[i] = 0u;
            }
          }
          __syncthreads();
          const int nu = ts.n_unc;
          canonical_keys(rf, ts.qs, rpg, rh, ts.band_page, nu, ts.seg_key, ts.stage);
          if (rank_band(ts.seg_key, ts.band_page, nu, k - ts.n_in, ts.cseg, ts.cand_key,
                        reinterpret_cast<uint64_t*>(ts.stage))) {
            // exactly k keys are MAX now: collect them in index order
            prefix = 0xFFFFFFFFu;
            kk = (uint32_t)k;
          } else {
            for (int u = threadIdx.x; u < nu; u += kTopkThreads) ts.cand_key[ts.cseg[u]] = ts.seg_key[u];
            __syncthreads();
            radix_select([&](int i) { return ts.cand_key[i]; }, ptotal, (uint32_t)k, ss, prefix, kk);
          }
        }
        collect_in_order([&](int i) { return ts.cand_key[i]; }, [&](int i) { return ts.cand_idx[i]; }, ptotal,
                         prefix, kk, ss, out);
        return;
      }
    }
  }
  radix_select([&](int i) { return ordered_key(s[i]); }, npages, (uint32_t)k, ss, prefix, kk);
  const uint32_t ninf = ordered_key(-INFINITY);
  if (refine && prefix != ninf) {  // (a -inf threshold: every finite page is in, exactly)
    // whole row: the band's pages listed in index order, their canonical keys computed once
    // (read back by binary search) and, for a band of at most kRankCap pages, ranked into
    // MAX / 0 selection keys; a band too large for shared memory computes its keys where they
    // are read
    uint32_t lo, hi;
    refine_band(prefix, eps2, lo, hi);
    auto in_band = [&](uint32_t key) { return key != ninf && key >= lo && key <= hi; };
    const int R = warp_range(npages);
    const int lo_i = min(warp * R, npages), hi_i = min(lo_i + R, npages);
    if (threadIdx.x == 0) ts.n_in = 0;
    int cnt = 0, above = 0;
    for (int j = lo_i; j < hi_i; j += 32) {
      const int i = j + lane;
      const uint32_t key = i < hi_i ? ordered_key(s[i]) : ninf;
      cnt += __popc(__ballot_sync(0xffffffffu, in_band(key)));
      above += __popc(__ballot_sync(0xffffffffu, key != ninf && key > hi));
    }
    int pos, zero, nb;
    warp_bases(cnt, 0, ss, pos, zero, nb);  // (its barriers also order the n_in reset)
    if (lane == 0 && above) atomicAdd(&ts.n_in, above);
    const bool listed = nb <= kSegCap;
    bool ranked = false;
    if (listed) {
      for (int j = lo_i; j < hi_i; j += 32) {
        const int i = j + lane;
        const bool c = i < hi_i && in_band(ordered_key(s[i]));
        const uint32_t bc = __ballot_sync(0xffffffffu, c);
        if (c) ts.cseg[pos + __popc(bc & lt)] = i;
        pos += __popc(bc);
      }
      __syncthreads();
      canonical_keys(rf, ts.qs, rpg, rh, ts.cseg, nb, ts.seg_key, ts.stage);
      ranked = rank_band(ts.seg_key, ts.cseg, nb, k - ts.n_in, nullptr,
                         reinterpret_cast<uint32_t*>(ts.band_page), reinterpret_cast<uint64_t*>(ts.stage));
    }
    auto key2 = [&](int i) -> uint32_t {
      const uint32_t key = ordered_key(s[i]);
      if (key == ninf) return key;
      if (key > hi) return 0xFFFFFFFFu;
      if (key < lo) return 0u;
      if (listed) {  // cseg[0 .. nb) ascending: find i
        int a = 0, b = nb - 1;
        while (a < b) {
          const int m = (a + b) >> 1;
          if (ts.cseg[m] < i) a = m + 1;
          else b = m;
        }
        return ranked ? reinterpret_cast<const uint32_t*>(ts.band_page)[a] : ts.seg_key[a];
      }
      const int64_t off = rh * rf.bnd_stride_kv + (int64_t)i * rf.bnd_stride_p;
      float best = -INFINITY;
      for (int r = 0; r < rpg; ++r) best = fmaxf(best, canonical_row_sum(ts.qs[r], rf.kmax + off, rf.kmin + off));
      return ordered_key(best);
    };
    if (ranked) {  // exactly k keys are MAX: collect them in index order
      prefix = 0xFFFFFFFFu;
      kk = (uint32_t)k;
    } else {
      radix_select(key2, npages, (uint32_t)k, ss, prefix, kk);
    }
    collect_in_order(key2, [&](int i) { return i; }, npages, prefix, kk, ss, out);
    return;
  }
  collect_in_order([&](int i) { return ordered_key(s[i]); }, [&](int i) { return i; }, npages, prefix, kk, ss, out);
}

// ---------------------------------------------------------------------------------
// Gather of the selected pages + partial tail (what retrieve() returns).
// ---------------------------------------------------------------------------------
template <int D>
__global__ void quest_gather_kernel(const pbk_quest_desc d, int k, int tail, bf16* ok, bf16* ov) {
  constexpr int kParts = D / 8;  // 16-byte parts per row
  const int n = blockIdx.z, h = blockIdx.y;
  const int rows = k * d.page + tail;
  const int row = blockIdx.x * (blockDim.x / kParts) + threadIdx.x / kParts, part = threadIdx.x % kParts;
  if (row >= rows) return;
  int src;
  if (row < k * d.page) src = d.pages[((int64_t)n * d.kv + h) * k + row / d.page] * d.page + row % d.page;
  else src = (d.n_arch / d.page) * d.page + (row - k * d.page);
  const int64_t so = h * d.arc_stride_kv + (int64_t)src * d.arc_stride_n + part * 8;
  const int64_t dst = (((int64_t)n * d.kv + h) * rows + row) * D + part * 8;
  *reinterpret_cast<uint4*>(ok + dst) = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(d.keys) + so);
  *reinterpret_cast<uint4*>(ov + dst) = *reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(d.values) + so);
}

// ---------------------------------------------------------------------------------
// Split-key exact attention. Virtual key j of a (group, key head):
//   j <  k*page          : archive token pages[j / page] * page + j % page (visible)
//   j <  k*page + tail   : archive tail token (visible)
//   otherwise            : window key j - R (visible per the window mask)
// CTA = (split of kSplitKeys virtual keys, group*kv + key head), 256 threads. Logits: one
// key per thread (its 256-byte row in 16-byte loads). P V: warp w takes keys 32w..32w+31,
// lane l dims 4l..4l+3, so each V row is one coalesced 256-byte warp load; the eight warps'
// partial sums meet in shared memory. Partials (m, l, acc[d]) go to the workspace;
// quest_combine_kernel merges them.
// ---------------------------------------------------------------------------------
constexpr int kAttThreads = 256;
constexpr int kAttWarps = kAttThreads / 32;
constexpr int kSplitKeys = 256;
// query rows per pass: 4, or 8 when a key head has more than 4 query rows (the serving
// layout's 6), so that every key and value row is read once per CTA
constexpr int kSinkTag = -(1 << 30);  // kidx encoding of always-visible leading keys: kSinkTag - i

__device__ __forceinline__ bool key_visible(int kp, int qp, int window, int sinks) {
  return kp <= qp && ((qp - kp) < window || kp < sinks);
}

template <int D, int kAttRows>
__global__ void __launch_bounds__(kAttThreads, 2) quest_attend_kernel(const pbk_quest_desc d, int k, int tail, int splits,
                                                                     float* part, int split0, const SinkKeys sk) {
  __shared__ __align__(16) float qs[kAttRows][D];
  __shared__ float prob[kAttRows][kSplitKeys];
  __shared__ int kidx[kSplitKeys];     // archive token, or -1 - window index
  __shared__ float red[kAttRows][kAttWarps];
  __shared__ float sh_m[kAttRows], sh_l[kAttRows];
  // the warps' partial P V sums, [kAttWarps][kAttRows][D] in dynamic shared memory (64 KB at
  // 8 rows x 256 dims, past the 48 KB of static shared memory)
  extern __shared__ __align__(16) float accs_raw[];
  auto accs = reinterpret_cast<float (*)[kAttRows][D]>(accs_raw);
  const int split = split0 + blockIdx.x, n = blockIdx.y / d.kv, h = blockIdx.y % d.kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int groups = d.h / d.kv, rows = d.t * groups;
  // splits [0, sr) hold the retrieved keys (leading keys, pages, tail), splits [sr, splits)
  // the window keys
  const int n_ret = sk.n + k * d.page + tail, sr = (n_ret + kSplitKeys - 1) / kSplitKeys;
  const bool win_split = split >= sr;
  const int j0 = win_split ? (split - sr) * kSplitKeys : split * kSplitKeys;
  const int nkeys = min(kSplitKeys, (win_split ? d.n_win : n_ret) - j0);
  const bf16* keys = reinterpret_cast<const bf16*>(d.keys);
  const bf16* vals = reinterpret_cast<const bf16*>(d.values);
  const bf16* wkeys = reinterpret_cast<const bf16*>(d.win_keys);
  const bf16* wvals = reinterpret_cast<const bf16*>(d.win_values);
  const float sl2 = d.scale * 1.4426950408889634f;  // softmax in base 2
  {
    const int vj = j0 + tid;
    int idx = 0;
    if (tid < nkeys) {
      if (win_split) idx = -1 - vj;
      else if (vj < sk.n) idx = kSinkTag - vj;
      else if (vj - sk.n < k * d.page) {
        const int r = vj - sk.n;
        idx = d.pages[((int64_t)n * d.kv + h) * k + r / d.page] * d.page + r % d.page;
      } else {
        idx = (d.n_arch / d.page) * d.page + (vj - sk.n - k * d.page);
      }
    }
    kidx[tid] = idx;
  }
  for (int r0 = 0; r0 < rows; r0 += kAttRows) {
    const int nr = min(kAttRows, rows - r0);
    __syncthreads();
    for (int e = tid; e < kAttRows * D; e += kAttThreads) {
      const int r = e / D, dd = e % D;
      float v = 0.f;
      if (r < nr) {
        const int rr = r0 + r, ti = rr / groups, g = rr % groups;
        v = __bfloat162float(reinterpret_cast<const bf16*>(d.q)[n * d.q_stride_n + ti * d.q_stride_t +
                                                                 (int64_t)(h * groups + g) * d.q_stride_h + dd]);
      }
      qs[r][dd] = v;
    }
    __syncthreads();
    // logits of key `tid`
    float lg[kAttRows];
    {
      float acc[kAttRows] = {};
      const int idx = kidx[tid];
      if (tid < nkeys) {
        const bf16* kr = idx >= 0         ? keys + h * d.arc_stride_kv + (int64_t)idx * d.arc_stride_n
                         : idx > kSinkTag ? wkeys + h * d.win_stride_kv + (int64_t)(-1 - idx) * d.win_stride_n
                                          : sk.k + h * sk.s_kv + (int64_t)(kSinkTag - idx) * sk.s_n;
#pragma unroll
        for (int c0 = 0; c0 < D / 8; c0 += 16) {  // 128 dims (16 loads) in flight at a time
          uint4 raw[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) raw[c] = *reinterpret_cast<const uint4*>(kr + 8 * (c0 + c));
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            float kv8[8];
            bf16x8_to_f32(raw[c], kv8);
#pragma unroll
            for (int r = 0; r < kAttRows; ++r) {
              const float4 qa = *reinterpret_cast<const float4*>(&qs[r][8 * (c0 + c)]);
              const float4 qb = *reinterpret_cast<const float4*>(&qs[r][8 * (c0 + c) + 4]);
              acc[r] = fmaf(qa.x, kv8[0], acc[r]); acc[r] = fmaf(qa.y, kv8[1], acc[r]);
              acc[r] = fmaf(qa.z, kv8[2], acc[r]); acc[r] = fmaf(qa.w, kv8[3], acc[r]);
              acc[r] = fmaf(qb.x, kv8[4], acc[r]); acc[r] = fmaf(qb.y, kv8[5], acc[r]);
              acc[r] = fmaf(qb.z, kv8[6], acc[r]); acc[r] = fmaf(qb.w, kv8[7], acc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kAttRows; ++r) {
        bool vis = tid < nkeys && r < nr;
        if (vis && idx < 0 && idx > kSinkTag) {
          const int rr = r0 + r, ti = rr / groups;
          vis = key_visible(d.kpos[-1 - idx], d.qpos[n * d.t + ti], d.window, d.sinks);
        }
        lg[r] = vis ? acc[r] * sl2 : -INFINITY;
      }
    }
    // row max over the split
#pragma unroll
    for (int r = 0; r < kAttRows; ++r) {
      float x = lg[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
      if (lane == 0) red[r][warp] = x;
    }
    __syncthreads();
    if (tid < kAttRows) {
      float x = red[tid][0];
      for (int w = 1; w < kAttWarps; ++w) x = fmaxf(x, red[tid][w]);
      sh_m[tid] = x;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kAttRows; ++r) {
      const float m = sh_m[r];
      const float p = m == -INFINITY ? 0.f : exp2f(lg[r] - m);
      prob[r][tid] = p;
      const float s = warp_sum(p);
      if (lane == 0) red[r][warp] = s;
    }
    __syncthreads();
    if (tid < kAttRows) {
      float x = 0.f;
      for (int w = 0; w < kAttWarps; ++w) x += red[tid][w];
      sh_l[tid] = x;
    }
    // P V: warp keys 32 warp .., lane dims 4 lane .. of each 128-dim half
    const int jb = 32 * warp, kn = min(32, nkeys - jb);
#pragma unroll
    for (int half = 0; half < D / 128; ++half) {  // all 32 value rows of the warp in flight at once
      float acc[kAttRows][4] = {};
      uint2 raw[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        raw[u] = make_uint2(0u, 0u);
        if (u < kn) {
          const int idx = kidx[jb + u];
          const bf16* vr = idx >= 0         ? vals + h * d.arc_stride_kv + (int64_t)idx * d.arc_stride_n
                           : idx > kSinkTag ? wvals + h * d.win_stride_kv + (int64_t)(-1 - idx) * d.win_stride_n
                                            : sk.v + h * sk.s_kv + (int64_t)(kSinkTag - idx) * sk.s_n;
          raw[u] = *reinterpret_cast<const uint2*>(vr + 128 * half + 4 * lane);
        }
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float v0 = __uint_as_float(raw[u].x << 16), v1 = __uint_as_float(raw[u].x & 0xffff0000u);
        const float v2 = __uint_as_float(raw[u].y << 16), v3 = __uint_as_float(raw[u].y & 0xffff0000u);
#pragma unroll
        for (int r = 0; r < kAttRows; ++r) {
          const float pr = u < kn ? prob[r][jb + u] : 0.f;
          acc[r][0] = fmaf(pr, v0, acc[r][0]);
          acc[r][1] = fmaf(pr, v1, acc[r][1]);
          acc[r][2] = fmaf(pr, v2, acc[r][2]);
          acc[r][3] = fmaf(pr, v3, acc[r][3]);
        }
      }
#pragma unroll
      for (int r = 0; r < kAttRows; ++r)
        *reinterpret_cast<float4*>(&accs[warp][r][128 * half + 4 * lane]) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    }
    __syncthreads();
    for (int e = tid; e < nr * D; e += kAttThreads) {
      const int r = e / D, dd = e % D;
      float x = 0.f;
#pragma unroll
      for (int w = 0; w < kAttWarps; ++w) x += accs[w][r][dd];
      const int rr = r0 + r, ti = rr / groups, g = rr % groups;
      const int64_t row = (((int64_t)n * d.t + ti) * d.h + h * groups + g) * splits + split;
      float* pp = part + row * (D + 2);
      pp[dd] = x;
      if (dd == 0) pp[D] = sh_m[r], pp[D + 1] = sh_l[r];
    }
  }
}

// One CTA (128 threads) per (output row, 32 output dims): the split weights exp2(m_s - M)
// in shared memory (max and sum over the splits in parallel), then each warp sums a quarter
// of the splits for the 32 dims (lane = dim, eight independent loads in flight) and the
// four partial sums meet in shared memory.
template <int D>
__global__ void __launch_bounds__(128) quest_combine_kernel(const pbk_quest_desc d, int splits, const float* part) {
  extern __shared__ float w[];  // [splits]
  __shared__ float red[4];
  __shared__ float accs[4][32];
  const int row = blockIdx.x;  // (n, ti, head); blockIdx.y: dims 32 y .. 32 y + 31
  const int head = row % d.h, ti = (row / d.h) % d.t, n = row / (d.h * d.t);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* pp = part + (int64_t)row * splits * (D + 2);
  float m = -INFINITY;
  for (int s = tid; s < splits; s += 128) m = fmaxf(m, pp[s * (D + 2) + D]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float l = 0.f;
  for (int s = tid; s < splits; s += 128) {
    const float ms = pp[s * (D + 2) + D];
    const float ws = ms == -INFINITY ? 0.f : exp2f(ms - M);
    w[s] = ws;
    l = fmaf(pp[s * (D + 2) + D + 1], ws, l);
  }
  l = warp_sum(l);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  const float L = (red[0] + red[1]) + (red[2] + red[3]);
  // warp w sums splits w, w + 4, ..., eight loads in flight per lane; lane = one dim
  const float* pd = pp + 32 * blockIdx.y + lane;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int s = warp;
  for (; s + 28 < splits; s += 32) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = pd[(s + 4 * u) * (D + 2)];
#pragma unroll
    for (int u = 0; u < 8; ++u) acc[u] = fmaf(x[u], w[s + 4 * u], acc[u]);
  }
  for (; s < splits; s += 4) acc[0] = fmaf(pd[s * (D + 2)], w[s], acc[0]);
  accs[warp][lane] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
  __syncthreads();
  if (warp == 0) {
    const float o = ((accs[0][lane] + accs[1][lane]) + (accs[2][lane] + accs[3][lane])) / L;
    const int64_t off = n * d.out_stride_n + ti * d.out_stride_t + head * d.out_stride_h + 32 * blockIdx.y + lane;
    if (d.out_dtype == PBK_BF16) reinterpret_cast<bf16*>(d.out)[off] = __float2bfloat16_rn(o);
    else reinterpret_cast<float*>(d.out)[off] = o;
  }
}

}  // namespace

// ---------------------------------------------------------------------------------
// Exact rerank (pb27_vllm/memory.py:854-872): the score of candidate page c is the max
// over the key head's query rows and the page's tokens of q.k in fp32. CTA = (8
// candidates, group*kv + key head), warp = one candidate page, lane = tokens lane,
// lane + 32, ...; the query rows sit in shared memory.
// ---------------------------------------------------------------------------------
// kRows query rows per pass (8, 16 or 32: the launch picks the smallest that holds the key
// head's rows, so the unrolled row loop does no dead iterations).
template <int D, int kRows>
__global__ void __launch_bounds__(256) quest_rerank_kernel(const pbk_quest_desc d, const int32_t* cand, int c,
                                                           float* exact) {
  __shared__ __align__(16) float qs[kRows][D];
  const int n = blockIdx.y / d.kv, h = blockIdx.y % d.kv, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = d.h / d.kv, rows = d.t * groups;
  const int ci = blockIdx.x * 8 + warp;
  const int page = ci < c ? cand[((int64_t)n * d.kv + h) * c + ci] : 0;
  const bf16* base = reinterpret_cast<const bf16*>(d.keys) + h * d.arc_stride_kv;
  float best = -INFINITY;
  for (int r0 = 0; r0 < rows; r0 += kRows) {
    const int nr = min(kRows, rows - r0);
    __syncthreads();
    for (int e = threadIdx.x; e < nr * D; e += blockDim.x) {
      const int r = e / D, dd = e % D, ti = (r0 + r) / groups, g = (r0 + r) % groups;
      qs[r][dd] = __bfloat162float(reinterpret_cast<const bf16*>(d.q)[n * d.q_stride_n + ti * d.q_stride_t +
                                                                        (int64_t)(h * groups + g) * d.q_stride_h + dd]);
    }
    __syncthreads();
    if (ci >= c) continue;
    for (int s = lane; s < d.page; s += 32) {
      const bf16* kr = base + ((int64_t)page * d.page + s) * d.arc_stride_n;
      float acc[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
#pragma unroll 1
      for (int h0 = 0; h0 < D; h0 += 64) {  // 64 dims (8 loads) of the key in flight
        uint4 raw[8];
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) raw[c8] = *reinterpret_cast<const uint4*>(kr + h0 + 8 * c8);
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {  // dims in order
          float kf[8];
          bf16x8_to_f32(raw[c8], kf);
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            if (r < nr) {
              const float4 qa = *reinterpret_cast<const float4*>(&qs[r][h0 + 8 * c8]);
              const float4 qb = *reinterpret_cast<const float4*>(&qs[r][h0 + 8 * c8 + 4]);
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
      for (int r = 0; r < kRows; ++r)
        if (r < nr) best = fmaxf(best, acc[r]);
    }
  }
  if (ci >= c) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) exact[((int64_t)n * d.kv + h) * c + ci] = best;
}

// pages[i] = cand[row][pages[i]]: the selected candidate positions become page indices.
__global__ void quest_map_kernel(const int32_t* cand, int c, int k, int nrows, int32_t* pages) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nrows * k) return;
  pages[i] = cand[(int64_t)(i / k) * c + pages[i]];
}

// ---------------------------------------------------------------------------------
// Super-block bounds (exact_memory.py:53-63, memory.py:280-306): warp per (super-block,
// key head), lane l owns dims 4l..4l+3; max of the blocks' maxima, min of their minima.
// ---------------------------------------------------------------------------------
template <int D>
__global__ void quest_superbounds_kernel(const bf16* kmax, const bf16* kmin, int64_t bs_kv, int64_t bs_p, int n_blk,
                                         int sblk, bf16* smax, bf16* smin, int64_t ss_kv, int64_t ss_p, int first_sb,
                                         int nsb) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= nsb) return;
  const int s = first_sb + warp, h = blockIdx.y;
  const int b0 = s * sblk, b1 = min(b0 + sblk, n_blk);
  float mx[P], mn[P], va[P], vb[P];
#pragma unroll
  for (int i = 0; i < P; ++i) mx[i] = -FLT_MAX, mn[i] = FLT_MAX;
  for (int b = b0; b < b1; ++b) {
    const int64_t off = h * bs_kv + (int64_t)b * bs_p + P * lane;
    R::load(kmax + off, va);
    R::load(kmin + off, vb);
#pragma unroll
    for (int i = 0; i < P; ++i) mx[i] = fmaxf(mx[i], va[i]), mn[i] = fminf(mn[i], vb[i]);
  }
  // max/min of bf16 values are bf16 values: exact
  R::store(smax + h * ss_kv + (int64_t)s * ss_p + P * lane, mx);
  R::store(smin + h * ss_kv + (int64_t)s * ss_p + P * lane, mn);
}

// ---------------------------------------------------------------------------------
// Candidate scores of the two-level selection (exact_memory.py:113-121, memory.py:814-835):
// candidate c of row (group n, key head h) is page idx = min(raw, full - 1), raw =
// top_sb[c / sblk] * sblk + c % sblk; its score is the page bound score, -inf when raw >=
// full or idx lies in [hole0, hole1). top_sb ascending makes the candidates' pages
// non-decreasing in c. CTA = (128 candidates, row); thread = candidate; the group's query
// rows pass through shared memory 32 at a time.
// ---------------------------------------------------------------------------------
constexpr int kSubRows = 32;
template <int D>
__global__ void __launch_bounds__(kScoreThreads) quest_sub_score_kernel(const pbk_quest_desc d, const int32_t* top_sb,
                                                                       int m_sb, int sblk, int full, int hole0,
                                                                       int hole1, float* scores, int32_t* cand) {
  __shared__ __align__(16) float qs[kSubRows][D];
  const int row = blockIdx.y, n = row / d.kv, h = row % d.kv, groups = d.h / d.kv, rows = d.t * groups;
  const int nc = m_sb * sblk, c = blockIdx.x * kScoreThreads + threadIdx.x;
  const bool live = c < nc;
  const int cc = live ? c : nc - 1;
  const int raw = top_sb[(int64_t)row * m_sb + cc / sblk] * sblk + cc % sblk;
  const int idx = min(raw, full - 1);
  const bool valid = raw < full && !(idx >= hole0 && idx < hole1);
  const bf16* bmax = reinterpret_cast<const bf16*>(d.kmax) + h * d.bnd_stride_kv + (int64_t)idx * d.bnd_stride_p;
  const bf16* bmin = reinterpret_cast<const bf16*>(d.kmin) + h * d.bnd_stride_kv + (int64_t)idx * d.bnd_stride_p;
  float best = -INFINITY;
  for (int r0 = 0; r0 < rows; r0 += kSubRows) {
    const int nr = min(kSubRows, rows - r0);
    __syncthreads();
    for (int e = threadIdx.x; e < nr * D; e += kScoreThreads) {
      const int r = e / D, dd = e % D, ti = (r0 + r) / groups, g = (r0 + r) % groups;
      qs[r][dd] = __bfloat162float(reinterpret_cast<const bf16*>(d.q)[n * d.q_stride_n + ti * d.q_stride_t +
                                                                        (int64_t)(h * groups + g) * d.q_stride_h + dd]);
    }
    __syncthreads();
    for (int rb = 0; rb < nr; rb += kRowBlock) {
      const int nb = min(kRowBlock, nr - rb);
      float acc[kRowBlock] = {0.f, 0.f, 0.f, 0.f};
      for (int d0 = 0; d0 < D; d0 += 8) {
        float mx[8], mn[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmax + d0), mx);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(bmin + d0), mn);
#pragma unroll
        for (int r = 0; r < kRowBlock; ++r) {
          if (r < nb) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float qv = qs[rb + r][d0 + j];
              acc[r] = fmaf(qv, qv > 0.f ? mx[j] : mn[j], acc[r]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRowBlock; ++r)
        if (r < nb) best = fmaxf(best, acc[r]);
    }
  }
  if (!live) return;
  scores[(int64_t)row * nc + c] = valid ? best : -INFINITY;
  cand[(int64_t)row * nc + c] = idx;
}

// ---------------------------------------------------------------------------------
// RoPE repositioning (pb27_vllm/memory.py:574-677). One warp per key head computes every
// block's shift in the reference's fp32 operation order (each product, quotient and sum
// rounded apart; integer positions are exact in fp32 below 2^24); mode 1 needs the running
// sum of the gaps between consecutive blocks (a warp scan, 32 blocks per step).
// ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(32) quest_rope_delta_kernel(const pbk_rope_gather_desc d) {
  const int h = blockIdx.x, lane = threadIdx.x;
  const int32_t* idx = d.blocks + (int64_t)h * d.n_blk;
  float* out = d.delta + (int64_t)h * d.n_blk;
  const float ref = (float)d.ref_pos, blk = (float)d.block;
  auto pos_of = [&](int j) { return (float)((int64_t)d.origin + (int64_t)idx[j] * d.block); };
  if (d.mode == 2) {
    for (int j = lane; j < d.n_blk; j += 32) {
      const float orig = pos_of(j);
      const float target = __fadd_rn(orig, rintf(__fmul_rn(fmaxf(__fsub_rn(ref, orig), 0.f), d.scale)));
      out[j] = fmaxf(__fsub_rn(target, orig), 0.f);
    }
    return;
  }
  // mode 1
  const int64_t nb = (int64_t)d.n_blk * d.block;
  const int64_t eff_span = max((int64_t)d.arc_span, nb);
  const int64_t base_i = max((int64_t)d.origin, (int64_t)d.ref_pos - eff_span);
  const float base_start = (float)base_i;
  const float slack = (float)max((int64_t)0, ((int64_t)d.ref_pos - base_i) - nb);
  const float g_pre = fmaxf(__fsub_rn(pos_of(0), (float)d.origin), 0.f);
  auto gap = [&](int i) {  // g_mid[i], i < n_blk - 1
    return (float)((int64_t)max(idx[i + 1] - idx[i] - 1, 0) * d.block);
  };
  float total = 0.f;  // sum of g_mid
  for (int i = lane; i < d.n_blk - 1; i += 32) total = __fadd_rn(total, gap(i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total = __fadd_rn(total, __shfl_xor_sync(0xffffffffu, total, o));
  const float g_post = fmaxf(__fsub_rn(ref, __fadd_rn(pos_of(d.n_blk - 1), blk)), 0.f);
  const float g_tot = fmaxf(__fadd_rn(__fadd_rn(g_pre, total), g_post), 1.f);
  const float ratio = __fdiv_rn(slack, g_tot);
  float carry = g_pre;  // g_cum of the first block of this step
  for (int j0 = 0; j0 < d.n_blk; j0 += 32) {
    const int j = j0 + lane;
    // g_cum[j] = g_pre + sum_{i < j} g_mid[i]: inclusive scan of g_mid[j - 1] (0 for j = 0)
    float x = (j > 0 && j < d.n_blk) ? gap(j - 1) : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = __fadd_rn(x, y);
    }
    const float g_cum = __fadd_rn(carry, x);
    if (j < d.n_blk) {
      const float target = __fadd_rn(__fadd_rn(base_start, (float)((int64_t)j * d.block)), rintf(__fmul_rn(g_cum, ratio)));
      out[j] = fmaxf(__fsub_rn(target, pos_of(j)), 0.f);
    }
    carry = __shfl_sync(0xffffffffu, g_cum, 31);
  }
}

// Gather (and rotate) the rows of one (block, key head) per CTA, after its cos / sin table
// (D / 8 pairs, computed once per block); warp = row, lane l holds dims P l .. P l + P - 1
// (P = D / 32), so the rotated pairs (i, i + D / 8), i < D / 8, sit in lanes l and l + 4 for
// l < 4. The tail rows (unrotated) are the CTAs past the blocks, kTailRows rows each.
constexpr int kTailRows = 64;
template <int D>
__global__ void __launch_bounds__(256) quest_rope_gather_kernel(const pbk_rope_gather_desc d) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer, kHalf = D / 8;
  __shared__ float cs[2][kHalf];
  const int h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nb = (int64_t)d.n_blk * d.block;
  const bool in_blocks = (int)blockIdx.x < d.n_blk;
  int64_t src0, out0, nrows;
  bool rot = false;
  if (in_blocks) {
    const int j = blockIdx.x;
    const int b = d.blocks ? d.blocks[(int64_t)h * d.n_blk + j] : j;
    src0 = (int64_t)d.origin + (int64_t)b * d.block;
    out0 = (int64_t)j * d.block;
    nrows = d.block;
    rot = d.mode != 0;
    if (rot && threadIdx.x < kHalf) {
      const float dl = d.mode == 3 ? d.const_delta : d.delta[(int64_t)h * d.n_blk + j];
      const float ang = __fmul_rn(dl, d.inv_freq[threadIdx.x]);
      cs[0][threadIdx.x] = cosf(ang);
      cs[1][threadIdx.x] = sinf(ang);
    }
    __syncthreads();
  } else {
    const int64_t t = (int64_t)(blockIdx.x - d.n_blk) * kTailRows;
    src0 = (int64_t)d.tail0 + t;
    out0 = nb + t;
    nrows = min((int64_t)kTailRows, (int64_t)d.tail_n - t);
  }
  float c[P], sn[P];
#pragma unroll
  for (int e = 0; e < P; ++e) c[e] = 1.f, sn[e] = 0.f;
  if (rot && lane < 8) {
#pragma unroll
    for (int e = 0; e < P; ++e) c[e] = cs[0][P * (lane & 3) + e], sn[e] = cs[1][P * (lane & 3) + e];
  }
  const bf16* kin = reinterpret_cast<const bf16*>(d.keys);
  const bf16* vin = reinterpret_cast<const bf16*>(d.values);
  bf16* kout = reinterpret_cast<bf16*>(d.out_keys) + (int64_t)h * (nb + d.tail_n) * D;
  bf16* vout = d.out_values ? reinterpret_cast<bf16*>(d.out_values) + (int64_t)h * (nb + d.tail_n) * D : nullptr;
  for (int64_t s = warp; s < nrows; s += 8) {
    const int64_t src = src0 + s;
    const bool ok = src >= 0 && src < d.n_rows;
    const int64_t at = h * d.stride_kv + src * d.stride_n + P * lane;
    typename R::Vec kr{}, vr{};
    if (ok) {
      kr = R::raw(kin + at);
      if (vout) vr = R::raw(vin + at);
    }
    if (rot) {
      typename R::Vec pr;
      const uint32_t* kw = reinterpret_cast<const uint32_t*>(&kr);
      uint32_t* pw = reinterpret_cast<uint32_t*>(&pr);
#pragma unroll
      for (int w = 0; w < P / 2; ++w) pw[w] = __shfl_xor_sync(0xffffffffu, kw[w], 4);
      if (lane < 8) {
        float own[P], other[P], r[P];
        R::unpack(kr, own);
        R::unpack(pr, other);
#pragma unroll
        for (int e = 0; e < P; ++e)  // lanes 0-3: r1 = x1 cos - x2 sin; lanes 4-7: r2 = x2 cos + x1 sin
          r[e] = lane < 4 ? __fsub_rn(__fmul_rn(own[e], c[e]), __fmul_rn(other[e], sn[e]))
                          : __fadd_rn(__fmul_rn(own[e], c[e]), __fmul_rn(other[e], sn[e]));
        kr = R::pack(r);
      }
    }
    const int64_t o = (out0 + s) * D + P * lane;
    R::put(kout + o, kr);
    if (vout) R::put(vout + o, vr);
  }
}

// ---------------------------------------------------------------------------------
// Archive write (pb27_vllm/memory.py:310-430). Rows that no summarised block covers are
// copied by one warp per (row, key head); each summarised block is one warp per (block, key
// head) that reads its rows once (new rows from the input, which it also writes, older rows
// from the archive) and keeps max, min and the fp32 sums of keys and values in registers.
// ---------------------------------------------------------------------------------
// Input rows [i0, i1) of the write (all of them for a scattered write).
template <int D>
__global__ void __launch_bounds__(256) quest_archive_copy_kernel(const pbk_archive_write_desc d, int i0, int i1) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer;
  const int h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = i0 + blockIdx.x * 8 + warp;
  if (i >= i1) return;
  const int64_t r = d.pos ? (int64_t)d.pos[i] : (int64_t)d.p0 + i;
  if (r < 0 || r >= d.cap) return;
  if (r >= d.origin) {  // rows of a summarised block are written by its warp
    const int64_t b = (r - d.origin) / d.block;
    if (b >= d.blk_lo && b <= d.blk_hi) return;
  }
  const int64_t src = (int64_t)i * d.in_stride_n + h * d.in_stride_kv + P * lane;
  const int64_t dst = h * d.arc_stride_kv + r * d.arc_stride_n + P * lane;
  R::put(reinterpret_cast<bf16*>(d.keys) + dst, R::raw(reinterpret_cast<const bf16*>(d.k) + src));
  R::put(reinterpret_cast<bf16*>(d.values) + dst, R::raw(reinterpret_cast<const bf16*>(d.v) + src));
}

template <int D>
__global__ void __launch_bounds__(256) quest_archive_block_kernel(const pbk_archive_write_desc d, int nblocks) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer;
  const int h = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = blockIdx.x * 8 + warp;
  if (w >= nblocks) return;
  const int64_t b = (int64_t)d.blk_lo + w;
  const int64_t r0 = d.origin + b * d.block;
  const int64_t end = d.pos ? (int64_t)d.size : max((int64_t)d.size, (int64_t)d.p0 + d.n);
  const int64_t r1 = min(r0 + d.block, min(end, (int64_t)d.cap));
  if (r1 <= r0) return;  // nothing written in this block yet
  const bf16* in_k = reinterpret_cast<const bf16*>(d.k);
  const bf16* in_v = reinterpret_cast<const bf16*>(d.v);
  bf16* ak = reinterpret_cast<bf16*>(d.keys);
  bf16* av = reinterpret_cast<bf16*>(d.values);
  float mx[P], mn[P], sk[P], sv[P], kl[P], vl[P];
#pragma unroll
  for (int e = 0; e < P; ++e) mx[e] = -FLT_MAX, mn[e] = FLT_MAX, sk[e] = 0.f, sv[e] = 0.f;
  constexpr int kBatch = 8;  // rows loaded before any is stored: eight loads of each in flight
  for (int64_t rb = r0; rb < r1; rb += kBatch) {
    typename R::Vec kr[kBatch], vr[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t r = rb + u;
      if (r >= r1) break;
      const bool fresh = d.pos == nullptr && r >= d.p0 && r < (int64_t)d.p0 + d.n;
      const bf16* sk_ = fresh ? in_k + (r - d.p0) * d.in_stride_n + h * d.in_stride_kv + P * lane
                              : ak + h * d.arc_stride_kv + r * d.arc_stride_n + P * lane;
      const bf16* sv_ = fresh ? in_v + (r - d.p0) * d.in_stride_n + h * d.in_stride_kv + P * lane
                              : av + h * d.arc_stride_kv + r * d.arc_stride_n + P * lane;
      kr[u] = R::raw(sk_);
      vr[u] = R::raw(sv_);
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t r = rb + u;
      if (r >= r1) break;
      if (d.pos == nullptr && r >= d.p0 && r < (int64_t)d.p0 + d.n) {  // bf16 in, bf16 out: the row as it came
        const int64_t at = h * d.arc_stride_kv + r * d.arc_stride_n + P * lane;
        R::put(ak + at, kr[u]);
        R::put(av + at, vr[u]);
      }
      R::unpack(kr[u], kl);
      R::unpack(vr[u], vl);
#pragma unroll
      for (int e = 0; e < P; ++e) {
        mx[e] = fmaxf(mx[e], kl[e]), mn[e] = fminf(mn[e], kl[e]);
        sk[e] += kl[e], sv[e] += vl[e];
      }
    }
  }
  const float pad = (float)(r0 + d.block - r1);  // a partial block counts its last row again
  const int64_t bo = h * d.bnd_stride_kv + b * d.bnd_stride_p + P * lane;
  float km[P], vm[P];
#pragma unroll
  for (int e = 0; e < P; ++e) {
    km[e] = (sk[e] + pad * kl[e]) / (float)d.block;
    vm[e] = (sv[e] + pad * vl[e]) / (float)d.block;
  }
  R::store(reinterpret_cast<bf16*>(d.kmax) + bo, mx);
  R::store(reinterpret_cast<bf16*>(d.kmin) + bo, mn);
  if (d.kmean) R::store(reinterpret_cast<bf16*>(d.kmean) + bo, km);
  if (d.vmean) R::store(reinterpret_cast<bf16*>(d.vmean) + bo, vm);
}

// Super-block means (memory.py:296-306): warp per (super-block, key head).
template <int D>
__global__ void quest_supermeans_kernel(const bf16* bmean, int64_t bs_kv, int64_t bs_p, int n_blk, int sblk,
                                        bf16* smean, int64_t ss_kv, int64_t ss_p, int first_sb, int nsb) {
  using R = WarpRow<D>;
  constexpr int P = R::kPer;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= nsb) return;
  const int s = first_sb + warp, h = blockIdx.y;
  const int b0 = s * sblk, b1 = min(b0 + sblk, n_blk);
  float acc[P], x[P];
#pragma unroll
  for (int e = 0; e < P; ++e) acc[e] = 0.f;
  for (int b = b0; b < b1; ++b) {
    R::load(bmean + h * bs_kv + (int64_t)b * bs_p + P * lane, x);
#pragma unroll
    for (int e = 0; e < P; ++e) acc[e] += x[e];
  }
#pragma unroll
  for (int e = 0; e < P; ++e) acc[e] /= (float)(b1 - b0);
  R::store(smean + h * ss_kv + (int64_t)s * ss_p + P * lane, acc);
}

// Pages [lo, hi) of every score row score -inf (the archive hole, memory.py:852-853).
__global__ void quest_hole_kernel(float* scores, int npages, int nrows, int lo, int hi) {
  const int w = hi - lo;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)nrows * w) return;
  scores[(i / w) * npages + lo + i % w] = -INFINITY;
}

// ---------------------------------------------------------------------------------
// Launch helpers (called from capi.cu after validation).
// ---------------------------------------------------------------------------------
namespace {
// f(std::integral_constant<int, D>{}) for head dim d (128 or 256; the entry points admit no
// other).
template <typename F>
cudaError_t with_dim(int d, F&& f) {
  if (d == 256) return f(std::integral_constant<int, 256>{});
  return f(std::integral_constant<int, 128>{});
}
}  // namespace

int quest_k(const pbk_quest_desc& d) { return min(d.budget, d.n_arch / d.page); }
// Splits of the retrieved keys (pages and tail) and of the window keys.
int quest_ret_splits(const pbk_quest_desc& d, int n_sink) {
  return (n_sink + quest_k(d) * d.page + (d.n_arch % d.page) + kSplitKeys - 1) / kSplitKeys;
}
int quest_splits(const pbk_quest_desc& d, int n_sink) {
  return quest_ret_splits(d, n_sink) + (d.n_win + kSplitKeys - 1) / kSplitKeys;
}
// Segment maxima are kept for rows of at least kSegMinPages pages (ceil(pages / 32) each).
int quest_nseg(const pbk_quest_desc& d) {
  const int npages = d.n_arch / d.page;
  return npages >= kSegMinPages ? (npages + 31) / 32 : 0;
}
// Largest bound magnitude per (key head, 128-page tile), written by the tensor-core score
// kernel for the top-k's refinement.
size_t quest_tile_abs_floats(const pbk_quest_desc& d) {
  return quest_score_tc_supported(d) ? (size_t)d.kv * quest_score_tc_tiles(d) * quest_score_tc_abs_slots() : 0;
}
// Scratch of one select call, in floats: the scores (unless the caller keeps them in
// desc.scores), then the segment maxima, then the tile bound magnitudes.
size_t quest_select_floats(const pbk_quest_desc& d) {
  const size_t rows = (size_t)d.nq * d.kv;
  return (d.scores ? 0 : rows * (d.n_arch / d.page)) + rows * quest_nseg(d) + quest_tile_abs_floats(d);
}

namespace {
// The top-k's refinement arguments for scores of desc `d` (tile_abs null: canonical scores).
RefineArgs refine_args(const pbk_quest_desc& d, const float* tile_abs) {
  RefineArgs r{};
  if (tile_abs == nullptr) return r;
  r.q = static_cast<const bf16*>(d.q);
  r.q_stride_n = d.q_stride_n;
  r.q_stride_t = d.q_stride_t;
  r.q_stride_h = d.q_stride_h;
  r.kmax = static_cast<const bf16*>(d.kmax);
  r.kmin = static_cast<const bf16*>(d.kmin);
  r.bnd_stride_kv = d.bnd_stride_kv;
  r.bnd_stride_p = d.bnd_stride_p;
  r.tile_abs = tile_abs;
  r.abs_per_kv = quest_score_tc_tiles(d) * quest_score_tc_abs_slots();
  r.kv = d.kv;
  r.groups = d.h / d.kv;
  r.t = d.t;
  return r;
}
}  // namespace
size_t quest_score_bytes(const pbk_quest_desc& d) { return quest_select_floats(d) * sizeof(float); }
size_t quest_partial_bytes(const pbk_quest_desc& d, int n_sink) {
  return (size_t)d.nq * d.t * d.h * quest_splits(d, n_sink) * (d.d + 2) * sizeof(float);
}

cudaError_t launch_quest_select(const pbk_quest_desc& d, float* scratch, cudaStream_t st) {
  return launch_quest_select_parts(d, scratch, 3, st);
}

// parts (bit mask): 1 the page scores (and segment maxima) into the workspace, 2 the top-k
// selection from them.
cudaError_t launch_quest_select_parts(const pbk_quest_desc& d, float* scratch, int parts, cudaStream_t st) {
  const int npages = d.n_arch / d.page, k = quest_k(d);
  if (npages == 0 || k == 0) return cudaSuccess;
  float* scores = d.scores ? d.scores : scratch;
  const int nseg = quest_nseg(d);
  float* after_scores = scratch + (d.scores ? 0 : (size_t)d.nq * d.kv * npages);
  float* segmax = nseg ? after_scores : nullptr;
  float* tile_abs = quest_score_tc_supported(d) ? after_scores + (size_t)d.nq * d.kv * nseg : nullptr;
  if (!(parts & 1)) {
  } else if (quest_score_tc_supported(d)) {
    // Up to 64 query rows per key head: tensor-core scores (tcgen05, TMA-fed).
    cudaError_t e = launch_quest_score_tc(d, scores, segmax, nseg, tile_abs, st);
    if (e != cudaSuccess) return e;
  } else {
    const int rows = d.nq * d.t * (d.h / d.kv);
    const size_t smem = (size_t)rows * d.d * sizeof(float);
    cudaError_t e = with_dim(d.d, [&](auto D) {
      constexpr int kDim = decltype(D)::value;
      if (smem > 48 * 1024) {
        cudaError_t e2 = cudaFuncSetAttribute(quest_score_kernel<kDim>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem);
        if (e2 != cudaSuccess) return e2;
      }
      quest_score_kernel<kDim><<<dim3((npages + kScoreThreads - 1) / kScoreThreads, d.kv), kScoreThreads, smem, st>>>(
          d, npages, scores, segmax, nseg);
      return cudaGetLastError();
    });
    if (e != cudaSuccess) return e;
  }
  if (!(parts & 2)) return cudaGetLastError();
  {
    cudaError_t e = cudaFuncSetAttribute(quest_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(TopkSmem));
    if (e != cudaSuccess) return e;
  }
  quest_topk_kernel<<<d.nq * d.kv, kTopkThreads, sizeof(TopkSmem), st>>>(scores, segmax, npages, nseg, k, d.pages,
                                                                          refine_args(d, tile_abs));
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------
// Scratch of pbk_quest_select_noalloc: a fixed array in device memory, so the entry point
// needs no allocation. Host code must not use the symbol's name as a device address; its
// address is looked up once per device (that device current) with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_scores[kNoAllocFloats];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

cudaError_t launch_quest_select_noalloc(const pbk_quest_desc& d, cudaStream_t st) {
  float* scratch = nullptr;  // page scores (unless desc.scores is given) and segment maxima
  {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scores);
      if (e != cudaSuccess) return e;
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  return launch_quest_select(d, scratch, st);
}

cudaError_t launch_quest_attend(const pbk_quest_desc& d, float* part, const SinkKeys& sk, int parts, cudaStream_t st) {
  const int k = quest_k(d), tail = d.n_arch % d.page;
  int splits = quest_splits(d, sk.n);
  if (splits == 0) return cudaSuccess;
  if (quest_attend_mma_supported(d)) {
    cudaError_t e = launch_quest_attend_mma(d, k, tail, part, sk, parts & 3, &splits, st);
    if (e != cudaSuccess) return e;
  } else if (parts & 3) {
    // SIMT kernel: splits [0, sr) retrieved, [sr, splits) window
    const int sr = quest_ret_splits(d, sk.n);
    const int s0 = (parts & 1) ? 0 : sr, s1 = (parts & 2) ? splits : sr;
    if (s1 > s0) {
      const dim3 grid(s1 - s0, d.nq * d.kv);
      const bool eight = d.t * (d.h / d.kv) > 4;  // 8 query rows per pass, else 4
      auto go = [&](auto kernel, int rows_per_pass) {
        const size_t smem = (size_t)kAttWarps * rows_per_pass * d.d * sizeof(float);
        if (smem > 48 * 1024) {
          cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
          if (e != cudaSuccess) return e;
        }
        kernel<<<grid, kAttThreads, smem, st>>>(d, k, tail, splits, part, s0, sk);
        return cudaGetLastError();
      };
      cudaError_t e = d.d == 256 ? (eight ? go(quest_attend_kernel<256, 8>, 8) : go(quest_attend_kernel<256, 4>, 4))
                                 : (eight ? go(quest_attend_kernel<128, 8>, 8) : go(quest_attend_kernel<128, 4>, 4));
      if (e != cudaSuccess) return e;
    }
  }
  if (!(parts & 4)) return cudaGetLastError();
  const int wbytes = splits * (int)sizeof(float);
  return with_dim(d.d, [&](auto D) {
    constexpr int kDim = decltype(D)::value;
    if (wbytes > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(quest_combine_kernel<kDim>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           wbytes);
      if (e != cudaSuccess) return e;
    }
    quest_combine_kernel<kDim><<<dim3(d.nq * d.t * d.h, kDim / 32), 128, wbytes, st>>>(d, splits, part);
    return cudaGetLastError();
  });
}

cudaError_t launch_quest_rerank(const pbk_quest_desc& d, const int32_t* cand, int c, float* exact, cudaStream_t st) {
  const int k = min(d.budget, c), nrows = d.nq * d.kv;
  if (k <= 0) return cudaSuccess;
  const int rows = d.t * (d.h / d.kv);
  with_dim(d.d, [&](auto D) {
    constexpr int kDim = decltype(D)::value;
    const dim3 grid((c + 7) / 8, nrows);
    if (rows <= 8) quest_rerank_kernel<kDim, 8><<<grid, 256, 0, st>>>(d, cand, c, exact);
    else if (rows <= 16) quest_rerank_kernel<kDim, 16><<<grid, 256, 0, st>>>(d, cand, c, exact);
    else quest_rerank_kernel<kDim, 32><<<grid, 256, 0, st>>>(d, cand, c, exact);
    return cudaSuccess;
  });
  cudaError_t e = cudaFuncSetAttribute(quest_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(TopkSmem));
  if (e != cudaSuccess) return e;
  quest_topk_kernel<<<nrows, kTopkThreads, sizeof(TopkSmem), st>>>(exact, nullptr, c, 0, k, d.pages,
                                                                    RefineArgs{});  // canonical rerank scores
  quest_map_kernel<<<(nrows * k + 255) / 256, 256, 0, st>>>(cand, c, k, nrows, d.pages);
  return cudaGetLastError();
}

cudaError_t launch_quest_gather(const pbk_quest_desc& d, int sel, void* ok, void* ov, cudaStream_t st) {
  const int k = sel, tail = d.n_arch % d.page, rows = k * d.page + tail;
  if (rows == 0) return cudaSuccess;
  return with_dim(d.d, [&](auto D) {
    constexpr int kDim = decltype(D)::value, kRowsPerCta = 256 / (kDim / 8);
    quest_gather_kernel<kDim><<<dim3((rows + kRowsPerCta - 1) / kRowsPerCta, d.kv, d.nq), 256, 0, st>>>(
        d, k, tail, static_cast<bf16*>(ok), static_cast<bf16*>(ov));
    return cudaGetLastError();
  });
}

cudaError_t launch_quest_bounds(const void* keys, int kv, int n, int dim, int page, int64_t ks_kv, int64_t ks_n,
                                void* kmax, void* kmin, int64_t bs_kv, int64_t bs_p, int first_page, cudaStream_t st) {
  const int npages = (n + page - 1) / page - first_page;
  if (npages <= 0) return cudaSuccess;
  return with_dim(dim, [&](auto D) {
    quest_bounds_kernel<decltype(D)::value><<<dim3((npages + 7) / 8, kv), 256, 0, st>>>(
        static_cast<const bf16*>(keys), n, page, ks_kv, ks_n, static_cast<bf16*>(kmax), static_cast<bf16*>(kmin),
        bs_kv, bs_p, first_page, npages);
    return cudaGetLastError();
  });
}


// ---------------------------------------------------------------------------------
// Two-level and hole-masked selection (pbk_quest_select_levels).
// ---------------------------------------------------------------------------------
namespace {
size_t round_ws(size_t bytes) { return (bytes + 255) / 256 * 256; }

// The super-block descriptor: the page-score pass over smax/smin, m_sb kept into top_sb.
pbk_quest_desc superblock_desc(const pbk_quest_desc& d, const pbk_quest_levels& lv, int32_t* top_sb) {
  const int full = d.n_arch / d.page, n_sb = (full + lv.sblk - 1) / lv.sblk;
  pbk_quest_desc ds = d;
  ds.kmax = lv.smax;
  ds.kmin = lv.smin;
  ds.bnd_stride_kv = lv.sb_stride_kv;
  ds.bnd_stride_p = lv.sb_stride_p;
  ds.n_arch = n_sb * d.page;
  ds.budget = lv.m_sb;
  ds.pages = top_sb;
  ds.scores = nullptr;
  return ds;
}

cudaError_t launch_topk(const float* scores, int npages, int k, int nrows, int32_t* pages, const RefineArgs& rf,
                        cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(quest_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sizeof(TopkSmem));
  if (e != cudaSuccess) return e;
  quest_topk_kernel<<<nrows, kTopkThreads, sizeof(TopkSmem), st>>>(scores, nullptr, npages, 0, k, pages, rf);
  return cudaGetLastError();
}
}  // namespace

size_t quest_levels_bytes(const pbk_quest_desc& d, const pbk_quest_levels& lv) {
  const size_t rows = (size_t)d.nq * d.kv;
  const int full = d.n_arch / d.page;
  if (lv.smax == nullptr) {  // scores, then the segment maxima and tile bound magnitudes of the score pass
    pbk_quest_desc dd = d;
    dd.scores = reinterpret_cast<float*>(16);  // kept apart: the scratch holds the rest
    return round_ws(rows * full * sizeof(float)) + round_ws(quest_select_floats(dd) * sizeof(float));
  }
  const pbk_quest_desc ds = superblock_desc(d, lv, nullptr);
  const size_t nc = (size_t)lv.m_sb * lv.sblk;
  return round_ws(quest_score_bytes(ds)) + round_ws(rows * lv.m_sb * sizeof(int32_t)) +
         round_ws(rows * nc * sizeof(float)) + round_ws(rows * nc * sizeof(int32_t));
}

cudaError_t launch_quest_select_levels(const pbk_quest_desc& d, const pbk_quest_levels& lv, uint8_t* ws,
                                       cudaStream_t st) {
  const int full = d.n_arch / d.page, k = quest_k(d), nrows = d.nq * d.kv;
  if (full == 0 || k == 0 || nrows == 0) return cudaSuccess;
  if (lv.smax == nullptr) {
    float* scores = reinterpret_cast<float*>(ws);
    pbk_quest_desc dd = d;
    dd.scores = scores;
    float* segmax = reinterpret_cast<float*>(ws + round_ws((size_t)nrows * full * sizeof(float)));
    cudaError_t e = launch_quest_select_parts(dd, segmax, 1, st);
    if (e != cudaSuccess) return e;
    const int lo = max(lv.hole_lo, 0), hi = min(lv.hole_hi, full);
    if (hi > lo) {
      const int64_t n = (int64_t)nrows * (hi - lo);
      quest_hole_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(scores, full, nrows, lo, hi);
    }
    // segment maxima may hold hole pages: not used; the tile bound magnitudes follow them
    const float* tile_abs = quest_score_tc_supported(dd) ? segmax + (size_t)nrows * quest_nseg(dd) : nullptr;
    return launch_topk(scores, full, k, nrows, d.pages, refine_args(dd, tile_abs), st);
  }
  const int nc = lv.m_sb * lv.sblk, k2 = min(k, nc);
  const pbk_quest_desc probe = superblock_desc(d, lv, nullptr);
  uint8_t* p = ws;
  float* sb_scratch = reinterpret_cast<float*>(p);
  p += round_ws(quest_score_bytes(probe));
  int32_t* top_sb = reinterpret_cast<int32_t*>(p);
  p += round_ws((size_t)nrows * lv.m_sb * sizeof(int32_t));
  float* sub = reinterpret_cast<float*>(p);
  p += round_ws((size_t)nrows * nc * sizeof(float));
  int32_t* cand = reinterpret_cast<int32_t*>(p);
  cudaError_t e = launch_quest_select_parts(superblock_desc(d, lv, top_sb), sb_scratch, 3, st);
  if (e != cudaSuccess) return e;
  with_dim(d.d, [&](auto D) {
    quest_sub_score_kernel<decltype(D)::value>
        <<<dim3((nc + kScoreThreads - 1) / kScoreThreads, nrows), kScoreThreads, 0, st>>>(
            d, top_sb, lv.m_sb, lv.sblk, full, lv.hole_lo, lv.hole_hi, sub, cand);
    return cudaSuccess;
  });
  e = launch_topk(sub, nc, k2, nrows, d.pages, RefineArgs{}, st);  // canonical candidate scores
  if (e != cudaSuccess) return e;
  quest_map_kernel<<<(nrows * k2 + 255) / 256, 256, 0, st>>>(cand, nc, k2, nrows, d.pages);
  return cudaGetLastError();
}

cudaError_t launch_quest_superbounds(const void* kmax, const void* kmin, int kv, int n_blk, int dim, int sblk,
                                     int64_t bs_kv, int64_t bs_p, void* smax, void* smin, int64_t ss_kv, int64_t ss_p,
                                     int first_sb, int end_sb, cudaStream_t st) {
  const int nsb = min(end_sb, (n_blk + sblk - 1) / sblk) - first_sb;
  if (nsb <= 0) return cudaSuccess;
  return with_dim(dim, [&](auto D) {
    quest_superbounds_kernel<decltype(D)::value><<<dim3((nsb + 7) / 8, kv), 256, 0, st>>>(
        static_cast<const bf16*>(kmax), static_cast<const bf16*>(kmin), bs_kv, bs_p, n_blk, sblk,
        static_cast<bf16*>(smax), static_cast<bf16*>(smin), ss_kv, ss_p, first_sb, nsb);
    return cudaGetLastError();
  });
}

cudaError_t launch_quest_rope_gather(const pbk_rope_gather_desc& d, cudaStream_t st) {
  const int64_t rows = (int64_t)d.n_blk * d.block + d.tail_n;
  if (rows == 0) return cudaSuccess;
  if ((d.mode == 1 || d.mode == 2) && d.n_blk > 0) quest_rope_delta_kernel<<<d.kv, 32, 0, st>>>(d);
  const int64_t ctas = (int64_t)d.n_blk + (d.tail_n + kTailRows - 1) / kTailRows;
  return with_dim(d.d, [&](auto D) {
    quest_rope_gather_kernel<decltype(D)::value><<<dim3((unsigned)ctas, d.kv), 256, 0, st>>>(d);
    return cudaGetLastError();
  });
}

namespace {
template <int D>
cudaError_t archive_write_dim(const pbk_archive_write_desc& d, cudaStream_t st) {
  auto copy = [&](int i0, int i1) {
    if (i1 > i0) quest_archive_copy_kernel<D><<<dim3((unsigned)((i1 - i0 + 7) / 8), d.kv), 256, 0, st>>>(d, i0, i1);
  };
  if (d.pos != nullptr || d.blk_hi < d.blk_lo) {
    copy(0, d.n);
  } else {  // only the rows outside the summarised blocks (whose warps write their own rows)
    const int64_t c0 = (int64_t)d.origin + (int64_t)d.blk_lo * d.block;
    const int64_t c1 = (int64_t)d.origin + ((int64_t)d.blk_hi + 1) * d.block;
    const int64_t lo = min(max(c0 - d.p0, (int64_t)0), (int64_t)d.n), hi = min(max(c1 - d.p0, lo), (int64_t)d.n);
    copy(0, (int)lo);
    copy((int)hi, d.n);
  }
  const int nblocks = d.blk_hi - d.blk_lo + 1;
  if (nblocks > 0)
    quest_archive_block_kernel<D><<<dim3((unsigned)((nblocks + 7) / 8), d.kv), 256, 0, st>>>(d, nblocks);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_quest_archive_write(const pbk_archive_write_desc& d, cudaStream_t st) {
  return with_dim(d.d, [&](auto D) { return archive_write_dim<decltype(D)::value>(d, st); });
}

cudaError_t launch_quest_supermeans(const void* bmean, int kv, int n_blk, int dim, int sblk, int64_t bs_kv,
                                    int64_t bs_p, void* smean, int64_t ss_kv, int64_t ss_p, int first_sb, int end_sb,
                                    cudaStream_t st) {
  const int nsb = min(end_sb, (n_blk + sblk - 1) / sblk) - first_sb;
  if (nsb <= 0) return cudaSuccess;
  return with_dim(dim, [&](auto D) {
    quest_supermeans_kernel<decltype(D)::value><<<dim3((nsb + 7) / 8, kv), 256, 0, st>>>(
        static_cast<const bf16*>(bmean), bs_kv, bs_p, n_blk, sblk, static_cast<bf16*>(smean), ss_kv, ss_p, first_sb,
        nsb);
    return cudaGetLastError();
  });
}

}  // namespace pbk
