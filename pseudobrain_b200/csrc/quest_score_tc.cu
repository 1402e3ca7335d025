// Quest page scores on the 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA).
//
// For one key head the scores of a tile of 128 pages against all R query rows of that
// head are one GEMM:  D[p][r] = sum_k A[p][k] B[r][k]  with
//   A[p] = [kmax_p (128) | kmin_p (128)]   (the page bounds, bf16, streamed by TMA)
//   B[r] = [max(q_r, 0) (128) | min(q_r, 0) (128)]   (exact in bf16)
// so D[p][r] = sum_d max(q_rd kmax_pd, q_rd kmin_pd) (exact_memory.py:97-98,124-125), and
// the page score of query group n is the max of D[p][r] over that group's rows. The
// bounds are read from HBM once for every query; the kernel is HBM-bound.
//
// Persistent CTAs, each owning a contiguous range of (key head, page tile) items:
//   warp 0: TMA producer (3-stage ring of 64 KB stages, 128B swizzle, no multicast)
//   warp 1: TMEM allocation and the MMA issuer (M=128 pages, N=R rounded to 16, K=256)
//   warps 2-9: two epilogue warpgroups, one per TMEM accumulator buffer (even / odd
//              tiles): read D from TMEM, reduce per query group and store the scores; the
//              group that meets a key head's first tile builds B for it.
//   warps 12-13: the tile's largest bound magnitude max |kmax|, |kmin| (read from the staged
//              tile in shared memory, half each) into tile_abs. Warps 12 and 13 run on SM
//              sub-partitions 0 and 1, beside the producer and MMA warps, which issue little
//              (on sub-partition 2, beside two epilogue warps, this work slowed the kernel by
//              15%); warps 10-11 have no role. It bounds the
//              rounding error of the tensor-core sums, |D - exact| <= c ||q||_1 max|bound|,
//              which the top-k uses to re-score the pages near its threshold in the
//              canonical order (quest.cu), so the selection is bit-exact.
// Every mbarrier wait is bounded: on timeout the kernel records an error code in the
// library's device error word and winds down (waiting, bounded, for its own loads and
// MMAs), frees its TMEM and returns.
#include "common.cuh"
#include "quest.cuh"
#include "tc.cuh"
#include "tma_host.h"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int kTileP = 128;                     // pages per tile = MMA M
constexpr int kStages = 3;
constexpr int kMaxRows = 64;                    // query rows per key head = MMA N (max)
constexpr int kAtomBytes = kTileP * 128;        // [128 rows x 64 bf16] swizzled atom
constexpr int kStageBytes = 4 * kAtomBytes;     // kmax d0-63 | kmax d64-127 | kmin d0-63 | kmin d64-127
constexpr int kBAtomBytes = kMaxRows * 128;
constexpr int kAbsWarps = 2;                    // warps 12-13: bound magnitudes of each tile
constexpr int kAbsWarp0 = 12;
constexpr int kThreads = 32 * (kAbsWarp0 + kAbsWarps);
constexpr int kTmemCols = 2 * kMaxRows;         // two accumulator buffers

struct __align__(1024) ScoreSmem {
  uint8_t a[kStages][kStageBytes];
  uint8_t b[4 * kBAtomBytes];
  uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2], b_ready;
  uint32_t tmem_base;
  volatile int abort;
};

struct ScoreArgs {
  const bf16* q;
  int64_t q_stride_n, q_stride_t, q_stride_h;
  float* scores;
  float* segmax;  // max of every 32 consecutive pages per (group, key head), or null
  float* tile_abs;  // [kv * tiles_per_kv][kAbsWarps] largest |bound| of each tile half, or null
  int nseg;
  int* err;
  int nq, t, groups, kv, npages, rows, n_pad, tiles_per_kv, total_tiles;
};

__device__ __forceinline__ void record_error(int* err, int site, ScoreSmem& sm) {
  if (err) atomicCAS(err, 0, 100 + site);
  sm.abort = 1;
}

// Order-preserving map of fp32 to uint32 (and back), for integer warp reductions.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_key_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Page score of every query group (the max of its RPG consecutive rows, RPG = 0: any
// rows-per-group at run time), stored for page p; and, per group, the max over this
// warp's 32 pages as one segment maximum.
template <int RPG>
__device__ __forceinline__ void group_max_store(const uint32_t (&v)[kMaxRows], const ScoreArgs& args, int kvh, int p,
                                                int lane) {
  const bool valid = p < args.npages;
  const int rpg = RPG > 0 ? RPG : args.t * args.groups;
  constexpr int kGroups = RPG > 0 ? kMaxRows / RPG : kMaxRows;
#pragma unroll
  for (int n = 0; n < kGroups; ++n) {
    if (n >= args.nq) break;  // uniform across the CTA
    float best = -INFINITY;
    if (RPG > 0) {
#pragma unroll
      for (int j = 0; j < (RPG > 0 ? RPG : 1); ++j) best = fmaxf(best, __uint_as_float(v[n * (RPG > 0 ? RPG : 1) + j]));
    } else {
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r)
        if (r >= n * rpg && r < (n + 1) * rpg) best = fmaxf(best, __uint_as_float(v[r]));
    }
    if (valid) args.scores[((int64_t)n * args.kv + kvh) * args.npages + p] = best;
    if (args.segmax != nullptr) {  // this warp's 32 pages form one segment: one warp max
      const uint32_t m = __reduce_max_sync(0xffffffffu, order_key(valid ? best : -INFINITY));
      if (lane == 0 && (p >> 5) < args.nseg)
        args.segmax[((int64_t)n * args.kv + kvh) * args.nseg + (p >> 5)] = order_key_inv(m);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    quest_score_tc_kernel(const __grid_constant__ CUtensorMap tmap_max, const __grid_constant__ CUtensorMap tmap_min,
                          const ScoreArgs args) {
  extern __shared__ uint8_t smem_raw[];
  ScoreSmem& sm = *reinterpret_cast<ScoreSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (args.total_tiles + gridDim.x - 1) / gridDim.x;
  const int t_begin = min(args.total_tiles, (int)blockIdx.x * per);
  const int t_end = min(args.total_tiles, t_begin + per);
  const int ntiles = t_end - t_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&sm.full[s], 1);
      // the MMA commit, plus one arrival per bound-magnitude warp once it has read the stage
      tc::mbar_init(&sm.empty[s], 1 + (args.tile_abs != nullptr ? kAbsWarps : 0));
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&sm.acc_full[b], 1);
      tc::mbar_init(&sm.acc_empty[b], 4);  // one arrival per warp of the buffer's epilogue group
    }
    tc::mbar_init(&sm.b_ready, 128);       // every thread of the building group, after its B writes
    sm.abort = 0;
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmap_max);
    tc::prefetch_tmap(&tmap_min);
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < ntiles && !sm.abort; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !tc::mbar_wait(&sm.empty[s], ((i / kStages) & 1) ^ 1)) {
          record_error(args.err, 1, sm);
          break;
        }
        const int tile = t_begin + i, kvh = tile / args.tiles_per_kv, p0 = (tile % args.tiles_per_kv) * kTileP;
        tc::mbar_expect_tx(&sm.full[s], kStageBytes);
        tc::tma_load_3d(sm.a[s] + 0 * kAtomBytes, &tmap_max, &sm.full[s], 0, p0, kvh);
        tc::tma_load_3d(sm.a[s] + 1 * kAtomBytes, &tmap_max, &sm.full[s], 64, p0, kvh);
        tc::tma_load_3d(sm.a[s] + 2 * kAtomBytes, &tmap_min, &sm.full[s], 0, p0, kvh);
        tc::tma_load_3d(sm.a[s] + 3 * kAtomBytes, &tmap_min, &sm.full[s], 64, p0, kvh);
        issued = i + 1;
      }
      // Our own loads in flight must land before the CTA exits (bounded).
      for (int i = max(0, issued - kStages); i < issued; ++i)
        if (!tc::mbar_wait(&sm.full[i % kStages], (i / kStages) & 1, 200000000ull)) record_error(args.err, 2, sm);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(128, args.n_pad, false, false);
      int cur_kv = -1, issued = 0;
      uint32_t bphase = 0;
      for (int i = 0; i < ntiles && !sm.abort; ++i) {
        const int s = i % kStages, acc = i & 1;
        const int kvh = (t_begin + i) / args.tiles_per_kv;
        if (kvh != cur_kv) {
          if (!tc::mbar_wait(&sm.b_ready, bphase)) { record_error(args.err, 3, sm); break; }
          bphase ^= 1;
          cur_kv = kvh;
        }
        if (!tc::mbar_wait(&sm.full[s], (i / kStages) & 1)) { record_error(args.err, 4, sm); break; }
        if (i >= 2 && !tc::mbar_wait(&sm.acc_empty[acc], ((i >> 1) & 1) ^ 1)) { record_error(args.err, 5, sm); break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + acc * kMaxRows;
        const uint32_t a0 = tc::smem_u32(sm.a[s]), b0 = tc::smem_u32(sm.b);
#pragma unroll
        for (int atom = 0; atom < 4; ++atom) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = tc::sdesc_sw128(a0 + atom * kAtomBytes + kk * 32, 16, 1024);
            const uint64_t bd = tc::sdesc_sw128(b0 + atom * kBAtomBytes + kk * 32, 16, 1024);
            tc::mma_f16(d, ad, bd, idesc, (atom | kk) != 0);
          }
        }
        tc::mma_commit(&sm.empty[s]);
        tc::mma_commit(&sm.acc_full[acc]);
        issued = i + 1;
      }
      // Our MMAs must complete before TMEM is freed (bounded).
      if (issued > 0 && !tc::mbar_wait(&sm.acc_full[(issued - 1) & 1], ((issued - 1) >> 1) & 1, 200000000ull))
        record_error(args.err, 6, sm);
    }
  } else if (warp >= kAbsWarp0) {
    // ---------------- bound magnitudes: warps 12-13, half of every stage each ----------------
    // |x| of a bf16 is its bit pattern with the sign cleared, and for non-NaN values the
    // order of those patterns as unsigned integers is the order of |x|: a packed 16-bit
    // integer max over the staged bytes (their swizzled order does not matter).
    if (args.tile_abs != nullptr) {
      const int aw = warp - kAbsWarp0;
      for (int i = 0; i < ntiles; ++i) {
        if (__any_sync(0xffffffffu, sm.abort)) break;  // warp-uniform exit
        const int s = i % kStages;
        const bool ok = tc::mbar_wait(&sm.full[s], (i / kStages) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
          record_error(args.err, 9, sm);
          break;
        }
        const uint4* src = reinterpret_cast<const uint4*>(sm.a[s] + aw * (kStageBytes / kAbsWarps));
        uint32_t m0 = 0, m1 = 0;
#pragma unroll 8
        for (int j = lane; j < kStageBytes / kAbsWarps / 16; j += 32) {
          const uint4 x = src[j];
          m0 = __vmaxu2(m0, x.x & 0x7fff7fffu);
          m1 = __vmaxu2(m1, x.y & 0x7fff7fffu);
          m0 = __vmaxu2(m0, x.z & 0x7fff7fffu);
          m1 = __vmaxu2(m1, x.w & 0x7fff7fffu);
        }
        const uint32_t m2 = __vmaxu2(m0, m1);
        uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16));
        m = min(m, 0x7f80u);  // NaN patterns count as +inf
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&sm.empty[s]);  // this warp is done with the stage
          args.tile_abs[(int64_t)(t_begin + i) * kAbsWarps + aw] = __uint_as_float(m << 16);  // bf16 -> fp32
        }
      }
    }
  } else if (warp < 10) {
    // ---------------- epilogue: warps 2..9, group eg takes tiles i = eg, eg + 2, ... ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    const int eg = (warp - 2) >> 2, etid = (threadIdx.x - 64) & 127;
    const int rpg = args.t * args.groups;
    for (int i = eg; i < ntiles; i += 2) {
      if (__any_sync(0xffffffffu, sm.abort)) break;  // warp-uniform exit
      const int tile = t_begin + i, kvh = tile / args.tiles_per_kv, p0 = (tile % args.tiles_per_kv) * kTileP;
      if (i == 0 || (tile - 1) / args.tiles_per_kv != kvh) {
        // B = [max(q,0) | min(q,0)] for this key head's rows, once the MMAs that read the
        // old B completed: the last of them is tile i-1's (the other group's buffer; its
        // next phase needs this B, so the phase cannot move on before the wait).
        if (i > 0) {
          const bool ok = tc::mbar_wait(&sm.acc_full[(i - 1) & 1], ((i - 1) >> 1) & 1);
          if (!__all_sync(0xffffffffu, ok)) {
            record_error(args.err, 8, sm);
            break;
          }
        }
        for (int e = etid; e < args.rows * 16; e += 128) {
          const int r = e >> 4, c = e & 15;  // 16-byte chunk c of row r (8 dims)
          const int n = r / rpg, rem = r % rpg, ti = rem / args.groups, g = rem % args.groups;
          const bf16* src = args.q + n * args.q_stride_n + ti * args.q_stride_t +
                            (int64_t)(kvh * args.groups + g) * args.q_stride_h + c * 8;
          const uint4 raw = *reinterpret_cast<const uint4*>(src);
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
          const __nv_bfloat162 zero = __float2bfloat162_rn(0.f);
          uint4 pos, neg;
          __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&pos);
          __nv_bfloat162* n2 = reinterpret_cast<__nv_bfloat162*>(&neg);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            p2[j] = __hmax2(h2[j], zero);
            n2[j] = __hmin2(h2[j], zero);
          }
          const int atom = c >> 3, kin = (c & 7) * 8;  // dims 0-63 -> atom 0, 64-127 -> atom 1
          *reinterpret_cast<uint4*>(sm.b + atom * kBAtomBytes + tc::sw128_offset(r, kin)) = pos;
          *reinterpret_cast<uint4*>(sm.b + (2 + atom) * kBAtomBytes + tc::sw128_offset(r, kin)) = neg;
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&sm.b_ready);
      }
      const int acc = i & 1;
      const bool ok = tc::mbar_wait(&sm.acc_full[acc], (i >> 1) & 1);
      if (!__all_sync(0xffffffffu, ok)) {  // the TMEM load below is warp-collective
        record_error(args.err, 7, sm);
        break;
      }
      tc::fence_after_sync();
      uint32_t v[kMaxRows];
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + acc * kMaxRows;
      tc::tmem_ld_32x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      if (args.n_pad > 32) tc::tmem_ld_32x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tc::tmem_ld_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.acc_empty[acc]);
      const int p = p0 + quad * 32 + lane;
      switch (rpg) {  // rows per query group: compile-time for the common shapes
        case 1: group_max_store<1>(v, args, kvh, p, lane); break;
        case 2: group_max_store<2>(v, args, kvh, p, lane); break;
        case 4: group_max_store<4>(v, args, kvh, p, lane); break;
        case 8: group_max_store<8>(v, args, kvh, p, lane); break;
        case 16: group_max_store<16>(v, args, kvh, p, lane); break;
        case 32: group_max_store<32>(v, args, kvh, p, lane); break;
        case 64: group_max_store<64>(v, args, kvh, p, lane); break;
        default: group_max_store<0>(v, args, kvh, p, lane); break;
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

constexpr size_t kSmemBytes = sizeof(ScoreSmem) + 1024;

}  // namespace

bool quest_score_tc_supported(const pbk_quest_desc& d) {
  const int rows = d.nq * d.t * (d.h / d.kv);
  return d.d == 128 && rows <= kMaxRows && d.n_arch / d.page > 0;
}

int quest_score_tc_tiles(const pbk_quest_desc& d) { return (d.n_arch / d.page + kTileP - 1) / kTileP; }
int quest_score_tc_abs_slots() { return kAbsWarps; }

cudaError_t launch_quest_score_tc(const pbk_quest_desc& d, float* scores, float* segmax, int nseg, float* tile_abs,
                                  cudaStream_t st) {
  const int npages = d.n_arch / d.page;
  CUtensorMap tmax, tmin;
  const uint64_t dims[3] = {128, (uint64_t)npages, (uint64_t)d.kv};
  const uint64_t strides[2] = {(uint64_t)d.bnd_stride_p * 2, (uint64_t)d.bnd_stride_kv * 2};
  const uint32_t box[3] = {64, kTileP, 1};
  if (!make_tmap_bf16_sw128(&tmax, d.kmax, 3, dims, strides, box) ||
      !make_tmap_bf16_sw128(&tmin, d.kmin, 3, dims, strides, box))
    return cudaErrorInvalidValue;
  ScoreArgs a;
  a.q = static_cast<const bf16*>(d.q);
  a.q_stride_n = d.q_stride_n;
  a.q_stride_t = d.q_stride_t;
  a.q_stride_h = d.q_stride_h;
  a.scores = scores;
  a.segmax = segmax;
  a.tile_abs = tile_abs;
  a.nseg = nseg;
  a.err = device_error_word();
  a.nq = d.nq;
  a.t = d.t;
  a.groups = d.h / d.kv;
  a.kv = d.kv;
  a.npages = npages;
  a.rows = d.nq * d.t * a.groups;
  a.n_pad = ((a.rows + 15) / 16) * 16;
  a.tiles_per_kv = (npages + kTileP - 1) / kTileP;
  a.total_tiles = a.tiles_per_kv * d.kv;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaFuncSetAttribute(quest_score_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  const int grid = a.total_tiles < sms ? a.total_tiles : sms;
  quest_score_tc_kernel<<<grid, kThreads, kSmemBytes, st>>>(tmax, tmin, a);
  return cudaGetLastError();
}

}  // namespace pbk
