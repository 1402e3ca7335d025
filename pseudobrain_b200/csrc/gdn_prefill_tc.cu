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
//   warps 0-7 (serial): state step of chunk n -- S^T to bf16 and S^T *= gamma_C through
//     the registers, then U = U' - WS, then the outputs; their thread 0 issues the S MMAs.
//   warps 8-15 (prep): chunk n+1's scalars, K K^T, A and M, the inverse (16x16 diagonal
//     blocks by substitution, off-diagonal blocks by tf32 mma.sync products), then W^T and
//     U'^T; their thread 0 issues the prep MMAs.
// Warp w of a role reads TMEM lane quadrant w % 4 and half w / 4 of each row's columns.
// K|Q and V arrive by TMA (4-D maps over [B,T,H,128], any strides; rows past T are
// zero-filled, the reference's identity padding; no multicast), issued by the leaders.
// The roles meet on mbarriers; every wait is bounded: on timeout the kernel records an
// error code, stops issuing, waits (bounded) for its own loads and MMAs, frees its TMEM
// and returns.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "tc.cuh"
#include "tma_host.h"

namespace pbk {
namespace {

using bf16 = __nv_bfloat16;
constexpr int C = 64;
constexpr int D = 128;
constexpr int kRoleWarps = 8;                 // warps per role (serial, prep)
constexpr int kRoleThreads = 32 * kRoleWarps;
constexpr int NT = 2 * kRoleThreads;          // serial role, prep role
constexpr int PA = C + 4;  // fp32 row stride of A (16-byte rows)

// TMEM columns
constexpr uint32_t kColS = 0, kColD1 = 128, kColUP = 192, kColWS = 320, kColQS = 384, kColUM = 448;
constexpr uint32_t kTmemCols = 512;

// A chunk's decay scalars (log2 units): cumulative decay c2, gamma = exp2(c2), e =
// exp2(c2_last - c2), the factored decay da = exp2(c2 - c2_31), db = exp2(c2_31 - c2) and
// whether the chunk's span (< 60) allows it, and beta. The solve kernel writes one per chunk
// after TB | TBG, and the recurrence copies it in with them.
struct ChunkScalars {
  float cum2[C], gam[C], ee[C], da[C], db[C], beta[C];
  int factored;
  int pad_[3];
};

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
  ChunkScalars cs[4];        // chunk m's scalars in slot m & 3
  float gs[4][C], bs[4][C];  // raw g and beta, staged 3 chunks ahead by a serial warp (in-line solve)
  uint64_t bar_kq[2], bar_v, bar_tb, bar_p1, bar_p3, bar_ws, bar_s, prep_ready, drain_s, drain_p, scal[4];
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
  void* o;  // NULL: final state only, no outputs written
  int64_t o_sb, o_st, o_sh;
  const float* h0;
  float* state;
  int64_t slot_stride;
  int layout;
  const int32_t* state_indices;
  float scale;
  int* err;
  const uint8_t* solve;  // TB | TBG of every (sequence, chunk, value head), or NULL: solved here
  // varlen (packed [1, T, H, 128]): sequence s = rows cu_seqlens[s] .. cu_seqlens[s+1],
  // its chunks at solve slots chunk_off[s] ..; NULL: dense [B, T, H, 128]
  const int32_t* cu_seqlens;
  const int32_t* chunk_off;
  int solve_slots;  // chunk slots of the varlen workspace (bound on cbase + nchunks)
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Named barrier over one role's threads (id 1: serial, 2: prep), and its AND-reduction.
__device__ __forceinline__ void role_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "n"(kRoleThreads) : "memory");
}
__device__ __forceinline__ bool role_and(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "n"(kRoleThreads)
      : "memory");
  return r != 0;
}

// 32 TMEM columns of this thread's lane into v[32].
__device__ __forceinline__ void tmem_row32(uint32_t taddr, float* v) {
  uint32_t r[32];
  tc::tmem_ld_32x32(taddr, r);
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 TMEM columns at each of two addresses of this thread's lane, one wait for both.
__device__ __forceinline__ void tmem_row32x2(uint32_t ta, float* va, uint32_t tb, float* vb) {
  uint32_t ra[32], rb[32];
  tc::tmem_ld_32x32(ta, ra);
  tc::tmem_ld_32x32(tb, rb);
  tc::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) va[i] = __uint_as_float(ra[i]), vb[i] = __uint_as_float(rb[i]);
}

// 32 fp32 values as bf16 into half `half` (elements 32 half .. 32 half + 31) of a 64-element
// row of a 128B-swizzled tile.
__device__ __forceinline__ void store_half_row_bf16(uint8_t* tile, int row, int half, const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    w.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    w.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    w.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, 32 * half + 8 * c)) = w;
  }
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
// acc (the 16x8 n-tile nt of a 16x16 block) += X (16x16) * Y (16x16)[:, 8 nt ..]; x(r, c),
// y(r, c) read the operands. m16n8k8 tf32 fragments: groupID g = lane / 4, t = lane % 4.
template <typename FX, typename FY>
__device__ __forceinline__ void tile_mma(float (&acc)[4], FX x, FY y, int nt, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int k0 = 0; k0 < 16; k0 += 8) {
    const uint32_t a[4] = {to_tf32(x(g, k0 + t)), to_tf32(x(g + 8, k0 + t)), to_tf32(x(g, k0 + t + 4)),
                           to_tf32(x(g + 8, k0 + t + 4))};
    const uint32_t bb[2] = {to_tf32(y(k0 + t, 8 * nt + g)), to_tf32(y(k0 + t + 4, 8 * nt + g))};
    mma_tf32(acc, a, bb);
  }
}
// Store the n-tile (scaled by s) through st(r, c, value).
template <typename FS>
__device__ __forceinline__ void tile_store(const float (&acc)[4], float s, FS st, int nt, int lane) {
  const int g = lane >> 2, t = lane & 3;
  st(g, 8 * nt + 2 * t, s * acc[0]);
  st(g, 8 * nt + 2 * t + 1, s * acc[1]);
  st(g + 8, 8 * nt + 2 * t, s * acc[2]);
  st(g + 8, 8 * nt + 2 * t + 1, s * acc[3]);
}


// T = (I + A)^-1 for the strictly lower 64 x 64 fp32 A (row stride PA) into the fp32
// scratch ts (tidx layout), by 8 warps (w = 0..7) that meet at sync(); scr holds 4 x (16 x
// 24) fp32 blocks. Diagonal 16x16 blocks (warps 0-3, one block each, lane = column) by
// right-looking substitution: v[r] accumulates sum_{m<r} A_rm x_m and becomes x_r when its
// turn comes (one FMA on the chain per step). Off-diagonal blocks T_ij = -T_ii (sum_{k=j}^{i-1}
// A_ik T_kj) in three levels: the two 32x32 diagonal halves (T_10, T_32), then the lower-left
// 32x32 quarter as X = A_21 T_1 and T_21 = -T_2 X; each warp computes one 16x8 tile (n-tile
// nt) with tf32 mma.sync. Ends with a sync().
template <typename Sync>
__device__ __forceinline__ void invert_unit_lower(const float* a, float* ts, float* scr, int w, int lane, Sync sync) {
  if (w < 4) {
    const int col = lane & 15, r0 = 16 * w;
    float v[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) v[r] = 0.f;
#pragma unroll
    for (int mm = 0; mm < 16; ++mm) {
      const float x = mm < col ? 0.f : (mm == col ? 1.f : -v[mm]);
      v[mm] = x;
#pragma unroll
      for (int r = mm + 1; r < 16; ++r) v[r] = fmaf(a[(r0 + r) * PA + r0 + mm], x, v[r]);
    }
    if (lane < 16) {
#pragma unroll
      for (int r = 0; r < 16; ++r) ts[tidx(r0 + r, r0 + col)] = v[r];
    }
  }
  sync();
  auto sread = [&](int b) { return [=](int r, int c) { return scr[b * 384 + r * 24 + c]; }; };
  auto swrite = [&](int b) { return [=](int r, int c, float x) { scr[b * 384 + r * 24 + c] = x; }; };
  auto at = [&](int bi, int bj) { return [=](int r, int c) { return a[(16 * bi + r) * PA + 16 * bj + c]; }; };
  auto tt = [&](int bi, int bj) { return [=](int r, int c) { return ts[tidx(16 * bi + r, 16 * bj + c)]; }; };
  auto twrite = [&](int bi, int bj) {
    return [=](int r, int c, float x) { ts[tidx(16 * bi + r, 16 * bj + c)] = x; };
  };
  const int blk = w >> 1, nt = w & 1;
  if (blk < 2) {  // T_10 (warps 0-1), T_32 (warps 2-3)
    const int j = 2 * blk, i = j + 1;
    float acc[4] = {};
    tile_mma(acc, at(i, j), tt(j, j), nt, lane);
    tile_store(acc, 1.f, swrite(blk), nt, lane);
    __syncwarp();
    float acc2[4] = {};
    tile_mma(acc2, tt(i, i), sread(blk), nt, lane);
    tile_store(acc2, -1.f, twrite(i, j), nt, lane);
  }
  sync();
  const int r = 2 + (blk >> 1), c = blk & 1;
  {  // X_rc = sum_{k=c}^{1} A_rk T_kc
    float acc[4] = {};
    for (int k = c; k < 2; ++k) tile_mma(acc, at(r, k), tt(k, c), nt, lane);
    tile_store(acc, 1.f, swrite(blk), nt, lane);
  }
  sync();
  {  // T_rc = -sum_{k=2}^{r} T_rk X_kc
    float acc[4] = {};
    for (int k = 2; k <= r; ++k) tile_mma(acc, tt(r, k), sread(2 * (k - 2) + c), nt, lane);
    tile_store(acc, -1.f, twrite(r, c), nt, lane);
  }
  sync();
}

// TB = T diag(beta), TBG = T diag(beta gamma) as bf16 128B-swizzled [64 t x 64 i] tiles
// (zero above the diagonal blocks); this thread: row t, columns 16 q .. 16 q + 15. The
// destinations may be shared or global memory (the same byte image either way).
__device__ __forceinline__ void store_tb_tbg(const float* ts, const float* beta, const float* gam, int t, int q,
                                             uint8_t* tb, uint8_t* tbg) {
  float vb[16], vbg[16];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int i = 16 * q + jj;
    const float x = q <= (t >> 4) ? ts[tidx(t, i)] * beta[i] : 0.f;
    vb[jj] = x;
    vbg[jj] = x * gam[i];
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint4 w1, w2;
    w1.x = pack_bf16x2(vb[8 * c], vb[8 * c + 1]);
    w1.y = pack_bf16x2(vb[8 * c + 2], vb[8 * c + 3]);
    w1.z = pack_bf16x2(vb[8 * c + 4], vb[8 * c + 5]);
    w1.w = pack_bf16x2(vb[8 * c + 6], vb[8 * c + 7]);
    w2.x = pack_bf16x2(vbg[8 * c], vbg[8 * c + 1]);
    w2.y = pack_bf16x2(vbg[8 * c + 2], vbg[8 * c + 3]);
    w2.z = pack_bf16x2(vbg[8 * c + 4], vbg[8 * c + 5]);
    w2.w = pack_bf16x2(vbg[8 * c + 6], vbg[8 * c + 7]);
    const uint32_t off = tc::sw128_offset(t, 16 * q + 8 * c);
    *reinterpret_cast<uint4*>(tb + off) = w1;
    *reinterpret_cast<uint4*>(tbg + off) = w2;
  }
}

// ------------------------------------------------------------------ chunk solve kernel
// The state-independent part of every chunk, for all chunks of all (sequence, value head)
// chains at once: one CTA per (chunk, group of G value heads sharing a key head, sequence)
// computes K K^T once (bf16 mma.sync, fp32 accumulate, 16x16 blocks) and, per value head in
// a group of 4 warps, the chunk's cumulative decay, A = strict_lower(beta_t K K^T * D),
// T = (I + A)^-1 (diagonal blocks by substitution in fp32, the off-diagonal blocks by tf32
// mma.sync products in three levels, the same arithmetic as the in-kernel solve), and writes
// TB and TBG (16 KB: the two bf16 tiles in the byte image the prefill kernel's MMAs read) to
// workspace slot (sequence, chunk, head). The prefill kernel then only copies them in. G = 2
// when the value heads per key head are even (the two heads of a pair share K and K K^T),
// else 1.
constexpr int kSolveThreads = 128;  // per value head
// TB | TBG | ChunkScalars per (sequence, chunk, value head)
constexpr uint32_t kSolveBytes = 2 * 8192 + sizeof(ChunkScalars);
static_assert(sizeof(ChunkScalars) % 16 == 0, "bulk copies move multiples of 16 bytes");

// 16x16 fp32 blocks (1 KB): element (r, c) at r * 16 + (c ^ bsw(r)). The swizzle keeps both
// mma.sync tf32 operand patterns (A: rows g, columns t; B: rows t, columns g) free of bank
// conflicts and 4-column groups contiguous (float4 row reads).
__device__ __forceinline__ int bsw(int r) { return (((r >> 1) & 1) << 3) | (((r >> 2) & 1) << 2); }
__device__ __forceinline__ int bidx(int r, int c) { return r * 16 + (c ^ bsw(r)); }
// Off-diagonal block (i > j) number: (1,0) 0, (2,0) 1, (2,1) 2, (3,0) 3, (3,1) 4, (3,2) 5.
__host__ __device__ constexpr int oidx(int i, int j) { return i * (i - 1) / 2 + j; }

struct SolveTX {       // one value head's inverse blocks
  float t[10][256];    // T blocks: diagonal b at b, off-diagonal (i, j) at 4 + oidx(i, j)
  float x[4][256];     // X_20, X_21, X_30, X_31 (level 1 scratch in x[0], x[1])
};
struct SolveHead {     // one value head's A and scalars
  float at[4][16][20]; // diagonal blocks of A, transposed: at[b][m][r] = A[16b + r][16b + m]; rows
                       // padded to 20 so the epilogue's column-group stores hit distinct banks
  float ao[6][256];    // off-diagonal blocks of A
  float c2[C], gam[C], beta[C];
};
template <int G>
struct SolveSmem {
  union {
    uint8_t k[C * 256];  // K rows of the chunk, 16-byte chunk c of row r at (c ^ (r & 7))
    SolveTX w;           // after K K^T: head 0's inverse
  };
  SolveTX w_more[G - 1];  // heads 1 .. G-1
  SolveHead hd[G];
  __device__ __forceinline__ SolveTX& tx(int g) { return g == 0 ? w : w_more[g - 1]; }
};
template <>
struct SolveSmem<1> {
  union {
    uint8_t k[C * 256];
    SolveTX w;
  };
  SolveHead hd[1];
  __device__ __forceinline__ SolveTX& tx(int) { return w; }
};

struct SolveArgs {
  const bf16* k;
  int64_t k_sb, k_st, k_sh;
  const void* g;
  int64_t g_sb, g_st, g_sh;
  int g_dtype;
  const void* beta;
  int64_t b_sb, b_st, b_sh;
  int b_dtype;
  int seqlen, hk, hv;
  uint8_t* ws;
  // varlen (packed [1, T, H, 128] inputs): sequence s spans rows cu_seqlens[s] ..
  // cu_seqlens[s+1], its chunks take workspace slots chunk_off[s] .. chunk_off[s+1]; NULL: dense
  const int32_t* cu_seqlens;
  const int32_t* chunk_off;
  int num_seqs;
  // optional chunk outputs (pbk_gdn_prefill_aux): the in-chunk cumulative g (fp32) and the rows
  // of T = (I + A)^-1, [B, T, Hv] and [B, T, Hv, 64] views; null: not written
  float* gc;
  int64_t gc_sb, gc_st, gc_sh;
  void* ta;
  int64_t ta_sb, ta_st, ta_sh;
  int ta_dtype;
};

// The layer's producer stages fused into the chunk solve (pbk_gdn_prefill_layer, dense
// sequences only): each CTA makes its own chunk's q, k and v from the input projection's
// channels -- short_convolution with the carried tail and SiLU (gated_deltanet.py:314-338),
// the q/k L2 norm (:59-70) -- and its g and beta from the raw gate inputs (:427-429), so the
// standalone conv and gating passes disappear. k goes straight into the solve's shared K tile;
// q, k and v are also written (bf16, dense [B, T, H, 128]) for the recurrence kernel.
struct SolveConvArgs {
  const bf16* x;              // [B, T, (2 hk + hv) 128] channels contiguous; NULL: the plain solve
  int64_t x_sb, x_st;
  const void* tail;           // [B, width - 1, channels] (NULL: zeros)
  int64_t tl_sb, tl_st, tl_sc;
  int tl_dtype;
  void* new_tail;             // [B, width - 1, channels] (NULL: not written); never `tail`
  int64_t nt_sb, nt_st, nt_sc;
  int nt_dtype;
  const float* conv_w;        // [channels, width] (NULL: SiLU only)
  int width, l2mode;
  float l2_eps;
  bf16* qo;                   // [B, T, hk, 128]
  bf16* ko;                   // [B, T, hk, 128]
  bf16* vo;                   // [B, T, hv, 128]
  const void* decay;          // [B, T, 2 hv]: a | b
  int64_t d_sb, d_st, d_sh;
  int d_dtype;
  const float* a_log;
  const float* dt_bias;
  const int32_t* state_indices;  // a sequence whose index is negative is skipped (no tail write)
  int* err;                       // the device error word (a copy that never landed)
};
constexpr int kConvMaxWidth = 8;

// Rows [t0, t0 + len) of packed sequence s, clamped into [0, T] (offsets out of order or out of
// range read nothing outside the tensors; they are caller errors).
__device__ __forceinline__ void seq_rows(const int32_t* cu_seqlens, int s, int T, int& t0, int& len) {
  t0 = min(max(cu_seqlens[s], 0), T);
  len = min(max(cu_seqlens[s + 1], t0), T) - t0;
}

// Sequence of global chunk c (chunk_off ascending, num_seqs + 1 entries): the last s with
// chunk_off[s] <= c.
__device__ __forceinline__ int seq_of_chunk(const int32_t* chunk_off, int num_seqs, int c) {
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_off[mid] <= c) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// chunk_off[s] = sum over s' < s of ceil(len_s' / C) for s = 0 .. num_seqs (one 1024-thread
// block: each thread sums a run of sequences, then a block scan).
__global__ void __launch_bounds__(1024) gdn_chunk_offsets_kernel(const int32_t* cu_seqlens, int num_seqs, int T,
                                                                  int32_t* chunk_off) {
  __shared__ int warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (num_seqs + 1023) / 1024, s0 = min(num_seqs, tid * per), s1 = min(num_seqs, s0 + per);
  int own = 0;
  int t0, len;
  for (int s = s0; s < s1; ++s) {
    seq_rows(cu_seqlens, s, T, t0, len);
    own += (len + C - 1) / C;
  }
  int x = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;
  }
  __syncthreads();
  int run = (warp > 0 ? warp_tot[warp - 1] : 0) + x - own;  // chunks before sequence s0
  for (int s = s0; s < s1; ++s) {
    chunk_off[s] = run;
    seq_rows(cu_seqlens, s, T, t0, len);
    run += (len + C - 1) / C;
  }
  if (tid == 1023) chunk_off[num_seqs] = warp_tot[31];
}

// Barrier of the 4 warps of value-head group g (named barrier 1 + g), or of the CTA when it
// holds one group.
template <int G>
__device__ __forceinline__ void group_sync(int g) {
  static_assert(G <= 2, "named barriers 1 and 2");
  if constexpr (G == 1) {
    __syncthreads();
  } else if (g == 0) {
    asm volatile("bar.sync 1, %0;" ::"n"(kSolveThreads) : "memory");
  } else {
    asm volatile("bar.sync 2, %0;" ::"n"(kSolveThreads) : "memory");
  }
}

// The conv producer of one CTA (kConv). Per 128-channel head of its chunk -- k first (into
// the shared K tile), q (by the CTA of the key head's first value-head group), then its value
// heads -- one TMA copy brings the head's 64 rows and the 7 before them (zero outside the
// sequence) into one of two 18 KB buffers, the next head's copy in flight while this one is
// computed; the first chunk patches the steps before the sequence from the carried tail. A
// half-warp per row then convolves (lane: 8 channels, its taps' weights in registers), applies
// SiLU, normalises q and k (one half-warp sum), rounds to bf16 and stores 16 bytes per lane. The CTA
// of the sequence's last chunk writes the new tail from the same tile. Rows past the end are
// zero in the K tile and not stored. Returns false (error code recorded) if a copy never lands.
constexpr int kRawRows = C + kConvMaxWidth - 1;         // the chunk's rows and the 7 before them
constexpr uint32_t kRawBytes = kRawRows * D * 2;        // 18,176 bytes per head
static_assert(kRawBytes % 128 == 0, "TMA destinations stay 128-byte aligned");
// KM: the compiled tap count (4 or 8; the layer's width right-aligned in it).
template <int G, int KM>
__device__ bool solve_conv_produce(const SolveArgs& p, const SolveConvArgs& cv, const CUtensorMap* xmap,
                                   uint8_t* smem, uint64_t* bars, int b, int m, int hkh, int h0) {
  constexpr int NT = kSolveThreads * G, kWarps = NT / 32, kHalo = kConvMaxWidth - 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.seqlen;
  const bool conv = cv.conv_w != nullptr;
  const int K = conv ? cv.width : 1;
  const bool qk_writer = (h0 % (p.hv / p.hk)) == 0;
  const int npass = 1 + (qk_writer ? 1 : 0) + G;
  const int t_first = m * C - kHalo;  // the step of raw row 0
  // pass 0: k; then q (writer only); then value heads h0 .. h0 + G - 1. kind: 0 q, 1 k, 2 v
  auto head_of = [&](int pass, int& kind, int& vh) {
    kind = pass == 0 ? 1 : (qk_writer && pass == 1 ? 0 : 2);
    vh = h0 + pass - (qk_writer ? 2 : 1);
    return (kind == 0 ? hkh : (kind == 1 ? p.hk + hkh : 2 * p.hk + vh)) * D;
  };
  auto buf_of = [&](int pass) { return smem + C * 256 + (pass & 1) * kRawBytes; };
  auto issue = [&](int pass) {
    int kind, vh;
    const int hc = head_of(pass, kind, vh);
    tc::mbar_expect_tx(&bars[pass & 1], kRawBytes);
    tc::tma_load_3d(buf_of(pass), xmap, &bars[pass & 1], hc, t_first, b);
  };
  if (tid == 0) {
    issue(0);
    if (npass > 1) issue(1);
  }
  for (int pass = 0; pass < npass; ++pass) {
    int kind, vh;
    const int hc = head_of(pass, kind, vh);
    bf16* raw = reinterpret_cast<bf16*>(buf_of(pass));
    const bool landed = tc::mbar_wait(&bars[pass & 1], (pass >> 1) & 1);
    if (__syncthreads_or(!landed)) {  // a copy never landed: record it, drain, give up
      if (tid == 0 && cv.err != nullptr) atomicCAS(cv.err, 0, 280);
      for (int q = pass; q < min(npass, pass + 2); ++q) tc::mbar_wait(&bars[q & 1], (q >> 1) & 1);
      return false;
    }
    if (conv && t_first < 0) {  // the first chunk: steps before the sequence from the tail
      for (int e = tid; e < (K - 1) * D; e += NT) {
        const int jj = e / D, c = e - jj * D;  // tail row jj holds step jj - (K - 1)
        const float val = cv.tail != nullptr ? load_any(cv.tail, b * cv.tl_sb + (int64_t)jj * cv.tl_st +
                                                                      (int64_t)(hc + c) * cv.tl_sc,
                                                        cv.tl_dtype)
                                             : 0.f;
        raw[(jj - (K - 1) - t_first) * D + c] = __float2bfloat16_rn(val);
      }
      __syncthreads();
    }
    // half-warp per row (lane: 8 channels, 16 bytes), two rows per warp and step; the lane's
    // weights in registers, tap i right-aligned (weight column i - (KM - K))
    const int l16 = lane & 15, half = lane >> 4;
    float w[8][KM];
    if (conv && K == KM && KM == 4) {  // rows of 4 taps: one 16-byte load per channel
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const float4 w4 = *reinterpret_cast<const float4*>(cv.conv_w + (int64_t)(hc + 8 * l16 + c8) * 4);
        w[c8][0] = w4.x, w[c8][1] = w4.y, w[c8][2] = w4.z, w[c8][3] = w4.w;
      }
    } else {
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
#pragma unroll
        for (int i = 0; i < KM; ++i) {
          const int j = i - (KM - K);
          w[c8][i] = conv ? (j >= 0 ? cv.conv_w[(int64_t)(hc + 8 * l16 + c8) * K + j] : 0.f)
                          : (i == KM - 1 ? 1.f : 0.f);
        }
    }
    for (int r = 2 * warp + half; r < C; r += 2 * kWarps) {
      float y[8];
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) y[c8] = 0.f;
#pragma unroll
      for (int i = 0; i < KM; ++i) {
        if (i < KM - K) continue;  // taps left of the layer's width
        const uint4 xv =  // raw row of step m C + r - (KM - 1 - i)
            *reinterpret_cast<const uint4*>(raw + (r + i + kHalo - (KM - 1)) * D + 8 * l16);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[q2]));
          y[2 * q2] = fmaf(w[2 * q2][i], f.x, y[2 * q2]);
          y[2 * q2 + 1] = fmaf(w[2 * q2 + 1][i], f.y, y[2 * q2 + 1]);
        }
      }
      // SiLU as h (1 + tanh h), h = y / 2, on the hardware tanh (one special-function
      // instruction; relative error about 2^-11, below the bf16 rounding of q, k and v)
      float ss = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const float hh = 0.5f * y[c8];
        float th;
        asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(hh));
        y[c8] = fmaf(hh, th, hh);
        ss = fmaf(y[c8], y[c8], ss);
      }
      if (kind != 2 && cv.l2mode != 0) {  // the row's sum over its half-warp
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float sc = cv.l2mode == 1 ? 1.f / fmaxf(sqrtf(ss), cv.l2_eps) : rsqrtf(ss + cv.l2_eps);
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) y[c8] *= sc;
      }
      const int tt = m * C + r;
      uint4 pk = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                            pack_bf16x2(y[6], y[7]));
      if (tt >= T) pk = make_uint4(0u, 0u, 0u, 0u);
      if (kind == 1)  // the K tile: 16-byte chunk c of row r at (c ^ (r & 7))
        *reinterpret_cast<uint4*>(smem + r * 256 + ((l16 ^ (r & 7)) << 4)) = pk;
      if (tt < T && (kind == 2 || qk_writer)) {
        bf16* dst = kind == 0 ? cv.qo + ((int64_t)b * T + tt) * p.hk * D + hkh * D
                    : kind == 1 ? cv.ko + ((int64_t)b * T + tt) * p.hk * D + hkh * D
                                : cv.vo + ((int64_t)b * T + tt) * p.hv * D + (int64_t)vh * D;
        *reinterpret_cast<uint4*>(dst + 8 * l16) = pk;
      }
    }
    // the new tail (the last width - 1 inputs), by the CTA of the last chunk, from the tile
    if (cv.new_tail != nullptr && conv && (m + 1) * C >= T && (kind == 2 || qk_writer)) {
      for (int e = tid; e < (K - 1) * D; e += NT) {
        const int j = e / D, c = e - j * D;
        const float val = __bfloat162float(raw[(T - (K - 1) + j - t_first) * D + c]);
        const int64_t o = b * cv.nt_sb + (int64_t)j * cv.nt_st + (int64_t)(hc + c) * cv.nt_sc;
        if (cv.nt_dtype == PBK_BF16) static_cast<bf16*>(cv.new_tail)[o] = __float2bfloat16_rn(val);
        else static_cast<float*>(cv.new_tail)[o] = val;
      }
    }
    __syncthreads();  // the tile has been read: its buffer takes the pass after next
    if (tid == 0 && pass + 2 < npass) {
      tc::fence_proxy_async_smem();
      issue(pass + 2);
    }
  }
  return true;
}

// The solve's body. kConvW: 0 the plain solve (gdn_solve_kernel); 4 or 8 with the conv
// producer compiled for that many taps (gdn_solve_conv_kernel).
template <int G, int kConvW>
__device__ __forceinline__ void solve_body(const SolveArgs& p, const SolveConvArgs& cv, const CUtensorMap* xmap) {
  extern __shared__ __align__(128) uint8_t solve_raw[];
  SolveSmem<G>& sm = *reinterpret_cast<SolveSmem<G>*>(solve_raw);
  constexpr int NT = kSolveThreads * G, kWarps = NT / 32;
  const int b = blockIdx.z;
  // this CTA's chunk m of a sequence at rows t0 .. t0 + len, workspace slot `cslot`
  int m = blockIdx.x, t0 = 0, len = p.seqlen;
  int64_t cslot = (int64_t)b * gridDim.x + m;
  if (p.cu_seqlens != nullptr) {
    if (m >= p.chunk_off[p.num_seqs]) return;  // the grid covers an upper bound of the chunks
    const int s = seq_of_chunk(p.chunk_off, p.num_seqs, m);
    seq_rows(p.cu_seqlens, s, p.seqlen, t0, len);
    cslot = m;
    m -= p.chunk_off[s];
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // value-head group: warps 4 gi .. 4 gi + 3 (threads gt = 0..127 of it) own head h; the G
  // heads of the CTA are consecutive and share key head hkh
  const int gi = warp >> 2, gw = warp & 3, gt = tid & (kSolveThreads - 1);
  const int h = blockIdx.y * G + gi;
  const int hkh = (blockIdx.y * G) / (p.hv / p.hk);
  SolveHead& hd = sm.hd[gi];
  constexpr bool kConv = kConvW != 0;
  if constexpr (kConv) {
    if (cv.state_indices != nullptr && cv.state_indices[b] < 0) return;  // the recurrence skips it too
    __shared__ uint64_t conv_bars[2];
    if (tid == 0) {
      tc::mbar_init(&conv_bars[0], 1);
      tc::mbar_init(&conv_bars[1], 1);
      tc::fence_barrier_init();
    }
    __syncthreads();
    if (!solve_conv_produce<G, kConvW>(p, cv, xmap, solve_raw, conv_bars, b, m, hkh, blockIdx.y * G)) return;
  }
  // K rows (zero past the sequence end, the reference's padding)
  for (int c = tid; c < C * 16 && !kConv; c += NT) {
    const int r = c >> 4, ch = c & 15, t = m * C + r;
    const uint32_t dst = tc::smem_u32(sm.k) + r * 256 + ((ch ^ (r & 7)) << 4);
    if (t < len) {
      const bf16* src = p.k + b * p.k_sb + (int64_t)(t0 + t) * p.k_st + hkh * p.k_sh + 8 * ch;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // cumulative log2 decay and gamma (the group's first warp; lane l: steps 2l, 2l + 1; zero
  // past the end)
  if (gw == 0) {
    constexpr float kLog2e = 1.4426950408889634f;
    const int t = m * C + 2 * lane;
    const int64_t tg = t0 + t;  // row in the (packed) tensor
    float g0 = 0.f, g1 = 0.f, b0 = 0.f, b1 = 0.f;
    if constexpr (kConv) {  // g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
      const float al = -expf(cv.a_log[h]), db = cv.dt_bias[h];
      auto gate = [&](int64_t row, float& gv, float& bv) {
        const int64_t o = b * cv.d_sb + row * cv.d_st;
        const float xa = load_any(cv.decay, o + h * cv.d_sh, cv.d_dtype) + db;
        gv = al * (xa > 20.f ? xa : log1pf(expf(xa)));
        bv = 1.f / (1.f + expf(-load_any(cv.decay, o + (int64_t)(p.hv + h) * cv.d_sh, cv.d_dtype)));
      };
      if (t < len) gate(tg, g0, b0);
      if (t + 1 < len) gate(tg + 1, g1, b1);
    } else {
      if (t < len) {
        g0 = load_any(p.g, b * p.g_sb + tg * p.g_st + h * p.g_sh, p.g_dtype);
        b0 = load_any(p.beta, b * p.b_sb + tg * p.b_st + h * p.b_sh, p.b_dtype);
      }
      if (t + 1 < len) {
        g1 = load_any(p.g, b * p.g_sb + (tg + 1) * p.g_st + h * p.g_sh, p.g_dtype);
        b1 = load_any(p.beta, b * p.b_sb + (tg + 1) * p.b_st + h * p.b_sh, p.b_dtype);
      }
    }
    const float pair = g0 + g1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (p.gc != nullptr) {  // the in-chunk cumulative g (natural log units)
      float* gcp = p.gc + b * p.gc_sb + tg * p.gc_st + h * p.gc_sh;
      if (t < len) gcp[0] = incl - pair + g0;
      if (t + 1 < len) gcp[p.gc_st] = incl;
    }
    const float c0 = (incl - pair + g0) * kLog2e, c1 = incl * kLog2e;
    const float ga0 = exp2f(c0), ga1 = exp2f(c1);
    hd.c2[2 * lane] = c0;
    hd.c2[2 * lane + 1] = c1;
    hd.gam[2 * lane] = ga0;
    hd.gam[2 * lane + 1] = ga1;
    hd.beta[2 * lane] = b0;
    hd.beta[2 * lane + 1] = b1;
    // the chunk's scalar record for the recurrence kernel (after TB | TBG): e = exp2(c_last -
    // c), and the factored decay about c_ref = c_31 while the log2 span stays below 60
    ChunkScalars* rec = reinterpret_cast<ChunkScalars*>(p.ws + (cslot * p.hv + h) * kSolveBytes + 2 * 8192);
    const float clast = __shfl_sync(0xffffffffu, c1, 31), ref = __shfl_sync(0xffffffffu, c1, 15);
    float hi = fmaxf(c0, c1), lo = fminf(c0, c1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    }
    *reinterpret_cast<float2*>(&rec->cum2[2 * lane]) = make_float2(c0, c1);
    *reinterpret_cast<float2*>(&rec->gam[2 * lane]) = make_float2(ga0, ga1);
    *reinterpret_cast<float2*>(&rec->ee[2 * lane]) = make_float2(exp2f(clast - c0), exp2f(clast - c1));
    *reinterpret_cast<float2*>(&rec->da[2 * lane]) = make_float2(exp2f(c0 - ref), exp2f(c1 - ref));
    *reinterpret_cast<float2*>(&rec->db[2 * lane]) = make_float2(exp2f(ref - c0), exp2f(ref - c1));
    *reinterpret_cast<float2*>(&rec->beta[2 * lane]) = make_float2(b0, b1);
    if (lane == 0) rec->factored = (hi - lo) < 60.f;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int g = lane >> 2, t4 = lane & 3, mi = lane >> 3;
  // ---- K K^T on the 10 lower 16x16 blocks (rb, cb), cb <= rb, numbered row by row; warp w
  // takes blocks w, w + kWarps, ... Epilogue, for each head of the CTA: A = beta_t K K^T
  // exp2(c_t - c_i) below the diagonal, zero on and above it; diagonal blocks stored
  // transposed (substitution), the others in the block layout (mma operands).
  {
    constexpr int kQ = (10 + kWarps - 1) / kWarps;
    auto rb_of = [](int j) { return j >= 6 ? 3 : (j >= 3 ? 2 : (j >= 1 ? 1 : 0)); };
    auto cb_of = [&](int j) { return j - rb_of(j) * (rb_of(j) + 1) / 2; };
    const uint32_t kb = tc::smem_u32(sm.k);
    float acc[kQ][2][4];
#pragma unroll
    for (int q = 0; q < kQ; ++q)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc[q][nt][0] = acc[q][nt][1] = acc[q][nt][2] = acc[q][nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {  // k-steps of 16 dims
#pragma unroll
      for (int q = 0; q < kQ; ++q) {
        const int j = warp + kWarps * q;
        if (j >= 10) continue;
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        {  // A: rows 16 rb + (0..7 | 8..15), dims 16 kk + (0..7 | 8..15)
          const int r = 16 * rb_of(j) + (mi & 1) * 8 + (lane & 7), ch = 2 * kk + (mi >> 1);
          ldsm_x4(kb + r * 256 + ((ch ^ (r & 7)) << 4), a0, a1, a2, a3);
        }
        {  // B (n = K rows 16 cb ..): (rows 0-7, dims lo | hi) for n-tile 0, rows 8-15 for n-tile 1
          const int r = 16 * cb_of(j) + (mi >> 1) * 8 + (lane & 7), ch = 2 * kk + (mi & 1);
          ldsm_x4(kb + r * 256 + ((ch ^ (r & 7)) << 4), b0, b1, b2, b3);
        }
        mma_bf16_16816(acc[q][0], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(acc[q][1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      const int j = warp + kWarps * q;
      if (j >= 10) continue;
      const int rb = rb_of(j), cb = cb_of(j);
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        SolveHead& ho = sm.hd[hh];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = g + 8 * (e >> 1), c = 8 * nt + 2 * t4 + (e & 1);
            const int t = 16 * rb + r, i = 16 * cb + c;
            const float a = i < t ? ho.beta[t] * acc[q][nt][e] * exp2f(ho.c2[t] - ho.c2[i]) : 0.f;
            if (rb == cb) ho.at[rb][c][r] = a;
            else ho.ao[oidx(rb, cb)][bidx(r, c)] = a;
          }
      }
    }
  }
  __syncthreads();  // K is dead: its space holds head 0's T and X blocks from here
  // From here each group of 4 warps inverts its own head's (I + A).
  SolveTX& w = sm.tx(gi);
  auto rd = [](const float* blk) { return [=](int r, int c) { return blk[bidx(r, c)]; }; };
  auto wr = [](float* blk) { return [=](int r, int c, float x) { blk[bidx(r, c)] = x; }; };
  // ---- diagonal blocks T_bb (group warps 0-1, lane = column c of block 2 gw + lane / 16):
  // right-looking substitution, v[r] accumulates sum_{m<r} A_rm x_m and becomes x_r when its
  // turn comes
  if (gw < 2) {
    const int bb = 2 * gw + (lane >> 4), c = lane & 15;
    float v[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) v[r] = 0.f;
#pragma unroll
    for (int mm = 0; mm < 16; ++mm) {
      const float x = mm < c ? 0.f : (mm == c ? 1.f : -v[mm]);
      v[mm] = x;
      const float4* col = reinterpret_cast<const float4*>(hd.at[bb][mm]);
#pragma unroll
      for (int q4 = (mm + 1) / 4; q4 < 4; ++q4) {
        const float4 a4 = col[q4];
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * q4 + e > mm) v[4 * q4 + e] = fmaf(av[e], x, v[4 * q4 + e]);
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) w.t[bb][bidx(r, c)] = v[r];
  }
  group_sync<G>(gi);
  // ---- off-diagonal blocks, T_ij = -T_ii (sum_{k=j}^{i-1} A_ik T_kj): warp = (block, n-tile)
  {  // level 1: T_10 (group warps 0-1), T_32 (group warps 2-3) via Y = A_ij T_jj
    const int blk = gw >> 1, nt = gw & 1, i = 2 * blk + 1, j = 2 * blk;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma(acc, rd(hd.ao[oidx(i, j)]), rd(w.t[j]), nt, lane);
    tile_store(acc, 1.f, wr(w.x[blk]), nt, lane);
    __syncwarp();
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
    tile_mma(acc2, rd(w.t[i]), rd(w.x[blk]), nt, lane);
    tile_store(acc2, -1.f, wr(w.t[4 + oidx(i, j)]), nt, lane);
  }
  group_sync<G>(gi);
#pragma unroll
  for (int q = 0; q < 2; ++q) {  // level 2: X_rc = sum_{k=c}^{1} A_rk T_kc, r = 2, 3; c = 0, 1
    const int u = gw + 4 * q, xb = u >> 1, nt = u & 1, r = 2 + (xb >> 1), c = xb & 1;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = c; k < 2; ++k)
      tile_mma(acc, rd(hd.ao[oidx(r, k)]), rd(k == c ? w.t[k] : w.t[4 + oidx(1, 0)]), nt, lane);
    tile_store(acc, 1.f, wr(w.x[xb]), nt, lane);
  }
  group_sync<G>(gi);
#pragma unroll
  for (int q = 0; q < 2; ++q) {  // level 3: T_rc = -sum_{k=2}^{r} T_rk X_kc
    const int u = gw + 4 * q, xb = u >> 1, nt = u & 1, r = 2 + (xb >> 1), c = xb & 1;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 2; k <= r; ++k)
      tile_mma(acc, rd(k == r ? w.t[r] : w.t[4 + oidx(3, 2)]), rd(w.x[2 * (k - 2) + c]), nt, lane);
    tile_store(acc, -1.f, wr(w.t[4 + oidx(r, c)]), nt, lane);
  }
  group_sync<G>(gi);
  // ---- TB = T diag(beta), TBG = T diag(beta gamma) as bf16 128B-swizzled [64 t x 64 i]
  // tiles (zero above the diagonal blocks) into the workspace; thread: row t, columns
  // 32 hh .. 32 hh + 31
  {
    uint8_t* dst = p.ws + (cslot * p.hv + h) * kSolveBytes;
    const int t = gt >> 1, hh = gt & 1, rb = t >> 4, rl = t & 15;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int cb = 2 * hh + cc;
      float v[16];
      if (cb <= rb) {
        const float* blk = cb == rb ? w.t[rb] : w.t[4 + oidx(rb, cb)];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 x = *reinterpret_cast<const float4*>(blk + rl * 16 + ((4 * q4) ^ bsw(rl)));
          v[4 * q4] = x.x, v[4 * q4 + 1] = x.y, v[4 * q4 + 2] = x.z, v[4 * q4 + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.f;
      }
      if (p.ta != nullptr && m * C + t < len) {  // row t of T, columns 16 cb ..
        const int64_t o = b * p.ta_sb + (int64_t)(t0 + m * C + t) * p.ta_st + h * p.ta_sh + 16 * cb;
        if (p.ta_dtype == PBK_BF16) {
          uint4 wv[2];
          uint32_t* wp = reinterpret_cast<uint32_t*>(wv);
#pragma unroll
          for (int e = 0; e < 8; ++e) wp[e] = pack_bf16x2(v[2 * e], v[2 * e + 1]);
          *reinterpret_cast<uint4*>(static_cast<bf16*>(p.ta) + o) = wv[0];
          *reinterpret_cast<uint4*>(static_cast<bf16*>(p.ta) + o + 8) = wv[1];
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            *reinterpret_cast<float4*>(static_cast<float*>(p.ta) + o + 4 * e) =
                make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float vb[8], vbg[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = 16 * cb + 8 * u + e;
          vb[e] = v[8 * u + e] * hd.beta[i];
          vbg[e] = vb[e] * hd.gam[i];
        }
        uint4 w1, w2;
        w1.x = pack_bf16x2(vb[0], vb[1]);
        w1.y = pack_bf16x2(vb[2], vb[3]);
        w1.z = pack_bf16x2(vb[4], vb[5]);
        w1.w = pack_bf16x2(vb[6], vb[7]);
        w2.x = pack_bf16x2(vbg[0], vbg[1]);
        w2.y = pack_bf16x2(vbg[2], vbg[3]);
        w2.z = pack_bf16x2(vbg[4], vbg[5]);
        w2.w = pack_bf16x2(vbg[6], vbg[7]);
        const uint32_t off = tc::sw128_offset(t, 16 * cb + 8 * u);
        *reinterpret_cast<uint4*>(dst + off) = w1;
        *reinterpret_cast<uint4*>(dst + 8192 + off) = w2;
      }
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kSolveThreads * G) gdn_solve_kernel(const SolveArgs p) {
  solve_body<G, 0>(p, SolveConvArgs{}, nullptr);
}
template <int G, int kConvW>
__global__ void __launch_bounds__(kSolveThreads * G, 8 / G)
    gdn_solve_conv_kernel(const SolveArgs p, const SolveConvArgs cv, const __grid_constant__ CUtensorMap xmap) {
  solve_body<G, kConvW>(p, cv, &xmap);
}

template <typename TOut, bool kOffload>
__global__ void __launch_bounds__(NT, 1)
    gdn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                          const PrefillArgs p) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // sequence `seq` of this CTA: rows t0 .. t0 + len of tensor batch b (b = 0 when packed),
  // its chunks at solve slots cbase ..
  const int seq = blockIdx.x / p.hv, h = blockIdx.x % p.hv;
  const bool varlen = p.cu_seqlens != nullptr;
  const int b = varlen ? 0 : seq;
  int t0 = 0, len = p.seqlen;
  if (varlen) seq_rows(p.cu_seqlens, seq, p.seqlen, t0, len);
  const int hk = h / (p.hv / p.hk);
  int64_t slot = seq;
  if (p.state_indices != nullptr) {
    slot = p.state_indices[seq];
    if (slot < 0) return;  // padding slot (uniform for the CTA)
  }
  const int nchunks = (len + C - 1) / C;
  const int64_t cbase = varlen ? (p.chunk_off != nullptr ? p.chunk_off[seq] : 0) : (int64_t)b * nchunks;
  if (varlen && cbase + nchunks > p.solve_slots) {  // offsets inconsistent with the workspace sizing
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, 270);
    return;
  }
  if (nchunks == 0) {  // an empty packed sequence: the final state is the initial one
    float* st = p.state + slot * p.slot_stride + (int64_t)h * D * D;
    const float* h0 = p.h0 != nullptr ? p.h0 + slot * p.slot_stride + (int64_t)h * D * D : nullptr;
    if (h0 != st)
      for (int i = threadIdx.x; i < D * D; i += NT) st[i] = h0 != nullptr ? h0[i] : 0.f;
    return;
  }

  if (tid == 0) {
    tc::mbar_init(&sm.bar_kq[0], 1);
    tc::mbar_init(&sm.bar_kq[1], 1);
    tc::mbar_init(&sm.bar_v, 1);
    tc::mbar_init(&sm.bar_tb, 1);
    tc::mbar_init(&sm.bar_p1, 1);
    tc::mbar_init(&sm.bar_p3, 1);
    tc::mbar_init(&sm.bar_ws, 1);
    tc::mbar_init(&sm.bar_s, 1);
    tc::mbar_init(&sm.prep_ready, kRoleThreads);
    tc::mbar_init(&sm.drain_s, 1);
    tc::mbar_init(&sm.drain_p, 1);
    for (int i = 0; i < 4; ++i) tc::mbar_init(&sm.scal[i], 1);
    sm.abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&sm.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  // Role layout: warp w of a role reads TMEM lanes 32 (w % 4) .. + 31 (its operand rows)
  // and owns half hf = w / 4 of each row's columns.
  const int quad = warp & 3, hf = (warp >> 2) & 1;
  const int row = 32 * quad + lane;
  const uint32_t lane_addr = tmem + ((uint32_t)(32 * quad) << 16);

  const uint32_t i_kk = tc::idesc_bf16_f32(128, 64, false, false);   // A K-major, B K-major, N=64
  const uint32_t i_kmn = tc::idesc_bf16_f32(128, 64, false, true);   // A K-major, B MN-major, N=64
  const uint32_t i_mnk = tc::idesc_bf16_f32(128, 64, true, false);   // A MN-major, B K-major, N=64
  const uint32_t i_s = tc::idesc_bf16_f32(128, 128, false, true);    // S update, N=128
  // Operand descriptors: one 128B-swizzle descriptor per leading-byte offset at the start of
  // the shared struct; a tile's descriptor adds its byte offset / 16 (the 14-bit address
  // field never carries: shared addresses stay below 256 KB). Rebuilding a descriptor from a
  // runtime address at every MMA costs the issuing thread more than the MMA itself.
  const uint32_t s_base = tc::smem_u32(&sm);
  const uint64_t d16 = tc::sdesc_sw128(s_base, 16, 1024);      // K-major; MN-major one atom wide
  const uint64_t d16k = tc::sdesc_sw128(s_base, 16384, 1024);  // MN-major over the two K|Q atoms
  const uint64_t d8k = tc::sdesc_sw128(s_base, 8192, 1024);    // MN-major over the two V atoms
  auto kq_desc = [&](uint64_t base, int buf) { return base + ((offsetof(PrefillSmem, kq) + (size_t)buf * 32768) >> 4); };

  // TMA loads (4-D maps over [B,T,H,128], rows past T zero-filled, no multicast). K|Q of
  // chunk m go to buffer m&1 (issued by the serial leader once chunk m-2's state update is
  // done), V to the single V buffer (issued by the prep leader once U' of chunk m-1 is done).
  auto issue_kq = [&](int m) {
    const int buf = m & 1;
    tc::mbar_expect_tx(&sm.bar_kq[buf], 4 * 8192);
    for (int a = 0; a < 2; ++a) {
      tc::tma_load_4d(sm.kq[buf][a], &tm_k, &sm.bar_kq[buf], 64 * a, t0 + m * C, hk, b);
      tc::tma_load_4d(sm.kq[buf][a] + 8192, &tm_q, &sm.bar_kq[buf], 64 * a, t0 + m * C, hk, b);
    }
  };
  auto issue_v = [&](int m) {
    tc::mbar_expect_tx(&sm.bar_v, 2 * 8192);
    for (int a = 0; a < 2; ++a) tc::tma_load_4d(sm.v[a], &tm_v, &sm.bar_v, 64 * a, t0 + m * C, h, b);
  };
  // With the solve offloaded: chunk m's TB | TBG (16 KB, contiguous in sm.tb, sm.tbg) and its
  // scalars (slot m & 3, last read for chunk m-4) by bulk copies, issued by the prep leader
  // once chunk m-1's U' and W^T products are done.
  auto issue_tb = [&](int m) {
    const uint8_t* src = p.solve + ((cbase + m) * p.hv + h) * kSolveBytes;
    tc::mbar_expect_tx(&sm.bar_tb, kSolveBytes);
    tc::bulk_load(sm.tb, src, 2 * 8192, &sm.bar_tb);
    tc::bulk_load(&sm.cs[m & 3], src + 2 * 8192, sizeof(ChunkScalars), &sm.bar_tb);
  };
  if (tid == 0) {
    tc::prefetch_tmap(&tm_q);
    tc::prefetch_tmap(&tm_k);
    tc::prefetch_tmap(&tm_v);
    if (p.o != nullptr) tc::prefetch_tmap(&tm_o);
    issue_kq(0);
    if (nchunks > 1) issue_kq(1);
    issue_v(0);
    if (kOffload) issue_tb(0);
  }

  if (warp >= kRoleWarps) {
    // ================================================================ prep role
    const int pt = tid - kRoleThreads, pw = warp - kRoleWarps;  // thread / warp within the role
    bool ok = true;
    auto fail = [&](int site) {
      if (pt == 0) {
        if (p.err) atomicCAS(p.err, 0, 200 + site);
        sm.abort = 1;
      }
      ok = false;
    };
    // bounded wait by every prep thread, outcome uniform across the role
    auto pwait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool got = role_and(2, tc::mbar_wait(bar, parity) && !sm.abort);
      if (!got) fail(site);
      tc::fence_after_sync();
      return got;
    };
    int last_v = 0;  // last V load issued (for the bounded drain)
    for (int m = 0; m < nchunks && ok; ++m) {
      const int buf = m & 1, sb = m & 3;
      // (No L2 prefetch of later chunks: issuing it queues behind this SM's loads in the TMA
      // unit and delays the prep leader by more than it saves.)
      // ---- [K;Q] K^T first: the scalar scan below runs under the MMA
      if (!pwait(&sm.bar_kq[buf], (m >> 1) & 1, 1)) break;
      if (pt == 0) {
        const uint64_t kd = kq_desc(d16, buf);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t dsc = kd + (kk >> 2) * 1024 + (kk & 3) * 2;
          tc::mma_f16(tmem + kColD1, dsc, dsc, i_kk, kk != 0);
        }
        tc::mma_commit(&sm.bar_p1);
      }
      // the copied-in TB | TBG and scalars of chunk m (offloaded solve)
      if (kOffload && !pwait(&sm.bar_tb, m & 1, 6)) break;
      // ---- scalars: cumulative log decay c, gamma = e^c, e = e^(c_C - c), beta
      if (!kOffload && pw == 0) {
        constexpr float kLog2e = 1.4426950408889634f;
        // g and beta of chunk m, staged in shared memory by a serial warp
        if (!tc::mbar_wait(&sm.scal[m & 3], (m >> 2) & 1)) {
          if (p.err) atomicCAS(p.err, 0, 210);
          sm.abort = 1;
        }
        const float g0 = sm.gs[m & 3][2 * lane], g1 = sm.gs[m & 3][2 * lane + 1];
        const float b0 = sm.bs[m & 3][2 * lane], b1 = sm.bs[m & 3][2 * lane + 1];
        const float pair = g0 + g1;
        float incl = pair;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const float c0 = incl - pair + g0, c1 = incl;
        const float clast = __shfl_sync(0xffffffffu, incl, 31);
        sm.cs[sb].cum2[2 * lane] = c0 * kLog2e;
        sm.cs[sb].cum2[2 * lane + 1] = c1 * kLog2e;
        sm.cs[sb].gam[2 * lane] = exp2f(c0 * kLog2e);
        sm.cs[sb].gam[2 * lane + 1] = exp2f(c1 * kLog2e);
        sm.cs[sb].ee[2 * lane] = exp2f((clast - c0) * kLog2e);
        sm.cs[sb].ee[2 * lane + 1] = exp2f((clast - c1) * kLog2e);
        sm.cs[sb].beta[2 * lane] = b0;
        sm.cs[sb].beta[2 * lane + 1] = b1;
        // decay factors exp2(c_t - c_i) = da_t db_i about c_ref = c_31, exact enough while
        // the chunk's log2 decay spans less than 60 (no factor leaves fp32's normal range)
        const float l0 = c0 * kLog2e, l1 = c1 * kLog2e;
        const float ref = __shfl_sync(0xffffffffu, l1, 15);
        float hi = fmaxf(l0, l1), lo = fminf(l0, l1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
          lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        }
        sm.cs[sb].da[2 * lane] = exp2f(l0 - ref);
        sm.cs[sb].da[2 * lane + 1] = exp2f(l1 - ref);
        sm.cs[sb].db[2 * lane] = exp2f(ref - l0);
        sm.cs[sb].db[2 * lane + 1] = exp2f(ref - l1);
        if (lane == 0) sm.cs[sb].factored = (hi - lo) < 60.f;
      }
      if (!pwait(&sm.bar_p1, m & 1, 2)) break;
      // ---- A (fp32) from K K^T rows (lanes 0-63), M (bf16) from Q K^T rows (lanes 64-127);
      // this thread: row `row`, columns 32 hf .. 32 hf + 31. With the solve offloaded only
      // M is needed (warp-uniform: warps of quadrants 0-1 hold the K K^T rows).
      if (!kOffload || row >= C) {
        const float* c2 = sm.cs[sb].cum2;
        const int t = row & 63, i0 = 32 * hf;
        const bool zero = t < 32 && hf == 1;  // rows 0-31 have no terms past column 31
        float v[32];
        if (!zero) tmem_row32(lane_addr + kColD1 + i0, v);
        // decay D_ti = exp2(c_t - c_i) for i <= t: factored (one multiply) or direct
        if (!zero) {
          const float ct = c2[t];
          if (sm.cs[sb].factored) {
            const float dt = sm.cs[sb].da[t];
            const float* dbi = sm.cs[sb].db + i0;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= dt * dbi[i];
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= i0 + i <= t ? exp2f(ct - c2[i0 + i]) : 0.f;
          }
        }
        if (row < C) {
          const float bt = sm.cs[sb].beta[t];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
            if (!zero) {
              w.x = i0 + i + 0 < t ? bt * v[i + 0] : 0.f;
              w.y = i0 + i + 1 < t ? bt * v[i + 1] : 0.f;
              w.z = i0 + i + 2 < t ? bt * v[i + 2] : 0.f;
              w.w = i0 + i + 3 < t ? bt * v[i + 3] : 0.f;
            }
            *reinterpret_cast<float4*>(&sm.a[t * PA + i0 + i]) = w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = (!zero && i0 + i <= t) ? p.scale * v[i] : 0.f;
          store_half_row_bf16(sm.m[buf], t, hf, v);
        }
      }
      if constexpr (!kOffload) {
        tc::fence_before_sync();
        role_sync(2);
        // ---- T = (I + A)^-1 into the fp32 scratch (free: W^T(m-2) consumed), then TB, TBG
        float* ts = reinterpret_cast<float*>(sm.wt[buf]);
        invert_unit_lower(sm.a, ts, reinterpret_cast<float*>(sm.tb), pw, lane, [] { role_sync(2); });
        // the tb scratch reads ended at the inverse's last barrier
        store_tb_tbg(ts, sm.cs[sb].beta, sm.cs[sb].gam, pt >> 2, pt & 3, sm.tb, sm.tbg);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      // ---- W^T = K^T TBG^T -> D1; U'^T = V^T TB^T -> UP[buf]
      if (!pwait(&sm.bar_v, m & 1, 3)) break;
      if (pt == 0) {
        const uint64_t kmn = kq_desc(d16k, buf), tbg = d16 + (offsetof(PrefillSmem, tbg) >> 4);
        const uint64_t vmn = d8k + (offsetof(PrefillSmem, v) >> 4), tb = d16 + (offsetof(PrefillSmem, tb) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc::mma_f16(tmem + kColD1, kmn + kk * 128, tbg + kk * 2, i_mnk, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f16(tmem + kColUP + 64 * buf, vmn + kk * 128, tb + kk * 2, i_mnk, kk != 0);
        tc::mma_commit(&sm.bar_p3);
      }
      if (!pwait(&sm.bar_p3, m & 1, 4)) break;
      if (pt == 0 && m + 1 < nchunks) {
        issue_v(m + 1);
        if (kOffload) issue_tb(m + 1);
        last_v = m + 1;
      }
      // ---- W^T -> wt[buf] (bf16, MN-major rows): row = dk index, columns 32 hf ..
      {
        float v[32];
        tmem_row32(lane_addr + kColD1 + 32 * hf, v);
        store_half_row_bf16(sm.wt[buf], row, hf, v);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      // The serial role must have taken chunk m-1 (its first MMA commit) before chunk m is
      // announced, so the two phases of prep_ready never alias.
      if (m >= 1 && !pwait(&sm.bar_ws, (m - 1) & 1, 5)) break;
      tc::mbar_arrive(&sm.prep_ready);
    }
    if (pt == 0) {  // our loads land and every MMA this thread issued completes before exit
      tc::mbar_wait(&sm.bar_v, last_v & 1, 200000000ull);
      if (kOffload) tc::mbar_wait(&sm.bar_tb, last_v & 1, 200000000ull);
      tc::mma_commit(&sm.drain_p);
      tc::mbar_wait(&sm.drain_p, 0, 200000000ull);
    }
  } else {
    // ================================================================ serial role
    bool ok = true;
    auto fail = [&](int site) {
      if (tid == 0) {
        if (p.err) atomicCAS(p.err, 0, 250 + site);
        sm.abort = 1;
      }
      ok = false;
    };
    auto swait = [&](uint64_t* bar, uint32_t parity, int site) -> bool {
      const bool got = role_and(1, tc::mbar_wait(bar, parity) && !sm.abort);
      if (!got) fail(site);
      tc::fence_after_sync();
      return got;
    };
    const int j = row;  // this thread's value column (TMEM lane); state columns 64 hf .. + 63
    // state in: S^T in TMEM
    {
      const float* h0 = p.h0 != nullptr ? p.h0 + slot * p.slot_stride + (int64_t)h * D * D : nullptr;
      for (int c0 = 64 * hf; c0 < 64 * hf + 64; c0 += 32) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = 0.f;
          if (h0 != nullptr) x = p.layout == PBK_STATE_KV ? h0[(c0 + i) * D + j] : h0[j * D + c0 + i];
          r[i] = __float_as_uint(x);
        }
        tc::tmem_st_32x32(lane_addr + kColS + c0, r);
      }
      tc::tmem_st_wait();
    }
    // State step of chunk n: S^T -> bf16 operand tile (atom hf holds dk 64 hf ..); S^T *=
    // gamma_C in TMEM. Then the S products of chunk n (thread 0).
    // The state decays lazily: S^T = big_g * (TMEM S) with big_g the product of the chunk
    // decays since the last renormalisation; chunk n's update adds K^T U diag(e) / big_g, and
    // TMEM is rescaled only when big_g would fall below 2^-100 (fp32 keeps the ratio exact).
    float big_g = 1.f, inv_next = 1.f;
    // (QS)^T = S^T Q^T of chunk n (thread 0): the state's bf16 copy in st, Q in chunk n's K|Q.
    // Its TMEM columns must have been read for chunk n-1, and st stays unchanged until the
    // chunk's S update commits (which covers QS: commits track every earlier MMA).
    const uint64_t st_d = d16 + (offsetof(PrefillSmem, st) >> 4);
    auto issue_qs = [&](int n) {
      const uint64_t qd = kq_desc(d16, n & 1) + (8192 >> 4);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t o = (kk >> 2) * 1024 + (kk & 3) * 2;
        tc::mma_f16(tmem + kColQS, st_d + o, qd + o, i_kk, kk != 0);
      }
    };
    auto state_step = [&](int n) {
      const int buf = n & 1, sb = n & 3;
      const float gnext = big_g * sm.cs[sb].gam[C - 1];
      const bool renorm = gnext < 0x1p-100f;  // identical in every thread of the role
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float f[32];
        tmem_row32(lane_addr + kColS + 64 * hf + 32 * c, f);
        if (renorm) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(f[i] * gnext);
          tc::tmem_st_32x32(lane_addr + kColS + 64 * hf + 32 * c, r);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] *= big_g;
        store_half_row_bf16(sm.st[hf], j, c, f);
      }
      if (renorm) tc::tmem_st_wait();
      big_g = renorm ? 1.f : gnext;
      inv_next = 1.f / big_g;
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      role_sync(1);
      if (tid == 0) {
        tc::fence_after_sync();
        const uint64_t wd = d16 + ((offsetof(PrefillSmem, wt) + (size_t)buf * 16384) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::mma_f16(tmem + kColWS, st_d + (kk >> 2) * 1024 + (kk & 3) * 2, wd + kk * 128, i_kmn, kk != 0);
        // With U diag(e) in its own buffer (offloaded solve) QS leaves the critical path: it
        // is issued once the previous chunk's outputs have been read (issue_qs below).
        if (!kOffload) issue_qs(n);
        tc::mma_commit(&sm.bar_ws);
      }
    };
    int last_kq[2] = {0, nchunks > 1 ? 1 : -1};  // last K|Q load per buffer (for the drain)
    // g and beta of chunk m into slot m & 3 (the role's last warp; lane l: steps 2l, 2l+1).
    // Slot m & 3 last held chunk m - 4, which the prep role scanned before announcing
    // chunk m - 3, so the slot is free once the serial role has taken chunk m - 3. The loads
    // run one call ahead: a call stores the values loaded by the previous call (chunk m) and
    // issues the loads of chunk m + 1, so the warp never waits on them before a role barrier.
    float pend[4] = {0.f, 0.f, 0.f, 0.f};
    auto load_scalars = [&](int m) {
      const int t = m * C + 2 * lane;
      const int64_t tg = t0 + t;
      pend[0] = pend[1] = pend[2] = pend[3] = 0.f;
      if (m < nchunks && t < len) {
        pend[0] = load_any(p.g, b * p.g_sb + tg * p.g_st + h * p.g_sh, p.g_dtype);
        pend[2] = load_any(p.beta, b * p.b_sb + tg * p.b_st + h * p.b_sh, p.b_dtype);
      }
      if (m < nchunks && t + 1 < len) {
        pend[1] = load_any(p.g, b * p.g_sb + (tg + 1) * p.g_st + h * p.g_sh, p.g_dtype);
        pend[3] = load_any(p.beta, b * p.b_sb + (tg + 1) * p.b_st + h * p.b_sh, p.b_dtype);
      }
    };
    auto stage_scalars = [&](int m) {
      if (kOffload || warp != kRoleWarps - 1 || m >= nchunks) return;
      sm.gs[m & 3][2 * lane] = pend[0];
      sm.gs[m & 3][2 * lane + 1] = pend[1];
      sm.bs[m & 3][2 * lane] = pend[2];
      sm.bs[m & 3][2 * lane + 1] = pend[3];
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.scal[m & 3]);
      load_scalars(m + 1);
    };
    if (!kOffload && warp == kRoleWarps - 1) load_scalars(0);
    stage_scalars(0);
    stage_scalars(1);
    stage_scalars(2);
    // U diag(e), the A operand of the state update: its own tile when the solve is offloaded
    // (the unused A scratch), else st[0] once the S^T products are done
    uint8_t* const ue = kOffload ? reinterpret_cast<uint8_t*>(sm.a) : sm.st[0];
    const uint64_t ue_d = d16 + ((kOffload ? offsetof(PrefillSmem, a) : offsetof(PrefillSmem, st)) >> 4);
    if (swait(&sm.prep_ready, 0, 1)) {
      state_step(0);
      if (kOffload && p.o != nullptr && tid == 0) issue_qs(0);
    }
    for (int n = 0; n < nchunks && ok; ++n) {
      const int buf = n & 1, sb = n & 3;
      // U = U' - WS -> U^T bf16 (ut) and U diag(e) (st[0], free: the S^T products are
      // done); then UM^T = U^T M^T and S^T += (U diag(e))^T K. This thread: t = 32 hf ..
      if (tid == 0) tc::bulk_wait_read0();  // the output store of chunk n-1 has read ut
      if (!swait(&sm.bar_ws, n & 1, 2)) break;
      {
        float ws[32], up[32];
        tmem_row32x2(lane_addr + kColWS + 32 * hf, ws, lane_addr + kColUP + 64 * buf + 32 * hf, up);
#pragma unroll
        for (int i = 0; i < 32; ++i) up[i] -= ws[i];
        store_half_row_bf16(sm.ut, j, hf, up);
        const float* ee = sm.cs[sb].ee + 32 * hf;
#pragma unroll
        for (int i = 0; i < 32; ++i) up[i] *= ee[i] * inv_next;
        store_half_row_bf16(ue, j, hf, up);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      role_sync(1);
      if (tid == 0) {
        tc::fence_after_sync();
        const uint64_t ud = d16 + (offsetof(PrefillSmem, ut) >> 4);
        const uint64_t md = d16 + ((offsetof(PrefillSmem, m) + (size_t)buf * 8192) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc::mma_f16(tmem + kColUM, ud + kk * 2, md + kk * 2, i_kk, kk != 0);
        const uint64_t kmn = kq_desc(d16k, buf);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) tc::mma_f16(tmem + kColS, ue_d + kk * 2, kmn + kk * 128, i_s, 1);
        tc::mma_commit(&sm.bar_s);
      }
      if (!swait(&sm.bar_s, n & 1, 3)) break;
      if (tid == 0 && n + 2 < nchunks) {  // chunk n's K|Q buffer is free for chunk n+2
        issue_kq(n + 2);
        last_kq[buf] = n + 2;
      }
      // O = gamma scale QS + UM (registers; t = 32 hf + i) and the next chunk's state step;
      // then O through shared memory and a TMA store. With the solve offloaded the state step
      // comes first, so that O's reads and store run while WS of chunk n+1 executes.
      float o[32];
      auto compute_o = [&]() {
        float um[32];
        tmem_row32x2(lane_addr + kColQS + 32 * hf, o, lane_addr + kColUM + 32 * hf, um);
        const float* gm = sm.cs[sb].gam + 32 * hf;
#pragma unroll
        for (int t = 0; t < 32; ++t) o[t] = fmaf(gm[t] * p.scale, o[t], um[t]);
      };
      if (!kOffload && p.o != nullptr) compute_o();
      tc::fence_before_sync();
      stage_scalars(n + 3);  // chunk n took the prep role's announcement of chunk n
      if (n + 1 < nchunks) {
        if (!swait(&sm.prep_ready, (n + 1) & 1, 4)) break;
        state_step(n + 1);
      }
      // staging in ut as row-major [rows][128]; rows past the sequence end fall outside
      // the tensor and are not written by the TMA store. A packed sequence's last, partial
      // chunk is copied out row by row instead (its next rows belong to the next sequence).
      if (p.o == nullptr) continue;
      if (kOffload) compute_o();
      constexpr int kRows = sizeof(TOut) == 2 ? 64 : 32;  // 16 KB per pass
      TOut* stage = reinterpret_cast<TOut*>(sm.ut);
      const bool partial = varlen && n * C + C > len;
#pragma unroll
      for (int r0 = 0; r0 < 64; r0 += kRows) {
        if (r0 > 0) {
          if (tid == 0) tc::bulk_wait_read0();
          role_sync(1);
        }
        if (32 * hf >= r0 && 32 * hf < r0 + kRows) {
#pragma unroll
          for (int t = 0; t < 32; ++t) stage[(32 * hf - r0 + t) * D + j] = from_f32<TOut>(o[t]);
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();  // every thread's TMEM reads of QS, UM precede QS(n+1)
        role_sync(1);
        if (partial) {
          constexpr int kVec = 16 / (int)sizeof(TOut), kRowVecs = D / kVec;
          const int valid = min(kRows, len - n * C - r0);
          TOut* out = static_cast<TOut*>(p.o);
          for (int e = tid; e < valid * kRowVecs; e += kRoleThreads) {
            const int r = e / kRowVecs, c = (e % kRowVecs) * kVec;
            const int64_t off = (int64_t)b * p.o_sb + (int64_t)(t0 + n * C + r0 + r) * p.o_st + (int64_t)h * p.o_sh + c;
            *reinterpret_cast<uint4*>(out + off) = *reinterpret_cast<const uint4*>(stage + r * D + c);
          }
        }
        if (tid == 0) {
          if (!partial) {
            tc::tma_store_4d(&tm_o, stage, 0, t0 + n * C + r0, h, b);
            tc::bulk_commit();
          }
          if (kOffload && r0 == 0 && n + 1 < nchunks) {
            tc::fence_after_sync();
            issue_qs(n + 1);
          }
        }
      }
    }
    if (tid == 0) tc::bulk_wait0();
    if (tid == 0) {  // our loads land and every MMA this thread issued completes before exit
      for (int bb = 0; bb < 2; ++bb)
        if (last_kq[bb] >= 0) tc::mbar_wait(&sm.bar_kq[bb], (last_kq[bb] >> 1) & 1, 200000000ull);
      tc::mma_commit(&sm.drain_s);
      tc::mbar_wait(&sm.drain_s, 0, 200000000ull);
    }
    if (ok) {
      // state out: columns 64 hf .. + 63 of row j of S^T
      float* st = p.state + slot * p.slot_stride + (int64_t)h * D * D;
      for (int c0 = 64 * hf; c0 < 64 * hf + 64; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld_32x32(lane_addr + kColS + c0, r);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (p.layout == PBK_STATE_KV) st[(c0 + i) * D + j] = __uint_as_float(r[i]) * big_g;
          else st[j * D + c0 + i] = __uint_as_float(r[i]) * big_g;
        }
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
static_assert(offsetof(PrefillSmem, a) % 1024 == 0 && sizeof(PrefillSmem::a) >= 16384,
              "the A scratch doubles as the U diag(e) operand tile (SW128, 1024-byte aligned)");

bool make_map(CUtensorMap* m, const pbk_view& v, int heads, const pbk_gdn_desc& d) {
  const uint64_t dims[4] = {128, (uint64_t)d.seqlen, (uint64_t)heads, (uint64_t)d.batch};
  const uint64_t strides[3] = {(uint64_t)v.stride_t * 2, (uint64_t)v.stride_h * 2, (uint64_t)v.stride_b * 2};
  const uint32_t box[4] = {64, 64, 1, 1};
  return make_tmap_bf16_sw128(m, v.data, 4, dims, strides, box);
}

void fill_args(PrefillArgs& a, const pbk_gdn_desc& d) {
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
  a.solve = nullptr;
  a.cu_seqlens = nullptr;
  a.chunk_off = nullptr;
  a.solve_slots = 0;
}

// The chunk solve over grid (chunks, value-head groups, sequences): two value heads per CTA
// (sharing K and K K^T) when the heads per key head are even, else one.
cudaError_t launch_solve(const SolveArgs& sa, unsigned chunks, unsigned seqs, int hv, int hk, cudaStream_t st,
                         const SolveConvArgs* cv = nullptr, const CUtensorMap* xmap = nullptr) {
  auto go = [&](auto kern, int g, size_t smem) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3(chunks, (unsigned)(hv / g), seqs), kSolveThreads * g, smem, st>>>(sa);
    return cudaGetLastError();
  };
  auto go_conv = [&](auto kern, int g, size_t smem) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<dim3(chunks, (unsigned)(hv / g), seqs), kSolveThreads * g, smem, st>>>(sa, *cv, *xmap);
    return cudaGetLastError();
  };
  // the conv producer's smem: the K tile, then two raw tiles over the inverse's scratch
  constexpr size_t kConvSmem = C * 256 + 2 * kRawBytes;
  const size_t conv2 = std::max(sizeof(SolveSmem<2>), kConvSmem);
  const size_t conv1 = std::max(sizeof(SolveSmem<1>), kConvSmem);
  const bool narrow = cv != nullptr && (cv->conv_w == nullptr || cv->width <= 4);
  if ((hv / hk) % 2 == 0) {
    if (cv == nullptr) return go(gdn_solve_kernel<2>, 2, sizeof(SolveSmem<2>));
    return narrow ? go_conv(gdn_solve_conv_kernel<2, 4>, 2, conv2) : go_conv(gdn_solve_conv_kernel<2, 8>, 2, conv2);
  }
  if (cv == nullptr) return go(gdn_solve_kernel<1>, 1, sizeof(SolveSmem<1>));
  return narrow ? go_conv(gdn_solve_conv_kernel<1, 4>, 1, conv1) : go_conv(gdn_solve_conv_kernel<1, 8>, 1, conv1);
}

}  // namespace

bool gdn_prefill_tc_supported(const pbk_gdn_desc& d) {
  auto ok16 = [](const pbk_view& v) {
    return (reinterpret_cast<uintptr_t>(v.data) & 15) == 0 && v.stride_t % 8 == 0 && v.stride_h % 8 == 0 &&
           v.stride_b % 8 == 0 && v.stride_t > 0 && v.stride_h > 0 && v.stride_b > 0;
  };
  // the output is written with 16-byte vectors along the value dim
  const bool out_ok = d.o.data == nullptr ||
                      ((reinterpret_cast<uintptr_t>(d.o.data) & 15) == 0 &&
                      d.o.stride_t % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0 &&
                      d.o.stride_h % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0 &&
                      d.o.stride_b % (d.o.dtype == PBK_BF16 ? 8 : 4) == 0);
  return d.q.dtype == PBK_BF16 && d.dk == 128 && d.dv == 128 && d.seqlen > 0 && ok16(d.q) && ok16(d.k) &&
         ok16(d.v) && out_ok;
}

size_t gdn_prefill_tc_workspace(const pbk_gdn_desc& d) {
  return (size_t)d.batch * ((d.seqlen + C - 1) / C) * d.hv * kSolveBytes;
}

// The chunk solve of every (sequence, chunk, value head) of d into ws
// (gdn_prefill_tc_workspace(d) bytes, 16-byte aligned).
cudaError_t launch_gdn_chunk_solve(const pbk_gdn_desc& d, void* ws, cudaStream_t st, const pbk_view* gc,
                                   const pbk_view* ta) {
  SolveArgs sa;
  sa.gc = gc != nullptr ? static_cast<float*>(const_cast<void*>(gc->data)) : nullptr;
  sa.gc_sb = gc ? gc->stride_b : 0;
  sa.gc_st = gc ? gc->stride_t : 0;
  sa.gc_sh = gc ? gc->stride_h : 0;
  sa.ta = ta != nullptr ? const_cast<void*>(ta->data) : nullptr;
  sa.ta_sb = ta ? ta->stride_b : 0;
  sa.ta_st = ta ? ta->stride_t : 0;
  sa.ta_sh = ta ? ta->stride_h : 0;
  sa.ta_dtype = ta ? ta->dtype : PBK_F32;
  sa.k = static_cast<const bf16*>(d.k.data);
  sa.k_sb = d.k.stride_b;
  sa.k_st = d.k.stride_t;
  sa.k_sh = d.k.stride_h;
  sa.g = d.g.data;
  sa.g_sb = d.g.stride_b;
  sa.g_st = d.g.stride_t;
  sa.g_sh = d.g.stride_h;
  sa.g_dtype = d.g.dtype;
  sa.beta = d.beta.data;
  sa.b_sb = d.beta.stride_b;
  sa.b_st = d.beta.stride_t;
  sa.b_sh = d.beta.stride_h;
  sa.b_dtype = d.beta.dtype;
  sa.seqlen = d.seqlen;
  sa.hk = d.hk;
  sa.hv = d.hv;
  sa.ws = static_cast<uint8_t*>(ws);
  sa.cu_seqlens = nullptr;
  sa.chunk_off = nullptr;
  sa.num_seqs = 0;
  return launch_solve(sa, (unsigned)((d.seqlen + C - 1) / C), (unsigned)d.batch, d.hv, d.hk, st);
}

// solve_ws: gdn_prefill_tc_workspace(d) bytes (16-byte aligned) holding the chunk solve of d
// (launch_gdn_chunk_solve) when `solved`, filled here first otherwise; NULL to solve each
// chunk inside the prefill kernel.
cudaError_t launch_gdn_prefill_tc(const pbk_gdn_desc& d, void* solve_ws, bool solved, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, d.q, d.hk, d) || !make_map(&mk, d.k, d.hk, d) || !make_map(&mv, d.v, d.hv, d))
    return cudaErrorInvalidValue;
  memset(&mo, 0, sizeof(mo));  // unused when only the final state is wanted
  if (d.o.data != nullptr) {
    const bool obf = d.o.dtype == PBK_BF16;
    const uint64_t es = obf ? 2 : 4;
    const uint64_t dims[4] = {128, (uint64_t)d.seqlen, (uint64_t)d.hv, (uint64_t)d.batch};
    const uint64_t strides[3] = {(uint64_t)d.o.stride_t * es, (uint64_t)d.o.stride_h * es,
                                 (uint64_t)d.o.stride_b * es};
    const uint32_t box[4] = {128, obf ? 64u : 32u, 1, 1};
    if (!make_tmap_plain(&mo, d.o.data, obf, 4, dims, strides, box)) return cudaErrorInvalidValue;
  }
  PrefillArgs a;
  fill_args(a, d);
  a.solve = static_cast<const uint8_t*>(solve_ws);
  if (solve_ws != nullptr && !solved) {
    cudaError_t e = launch_gdn_chunk_solve(d, solve_ws, st, nullptr, nullptr);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid((unsigned)((int64_t)d.batch * d.hv));
  auto go = [&](auto kernel) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    kernel<<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, mo, a);
    return cudaGetLastError();
  };
  if (d.o.dtype == PBK_BF16)
    return solve_ws ? go(gdn_prefill_tc_kernel<bf16, true>) : go(gdn_prefill_tc_kernel<bf16, false>);
  return solve_ws ? go(gdn_prefill_tc_kernel<float, true>) : go(gdn_prefill_tc_kernel<float, false>);
}

// Packed varlen prefill: d describes [1, T, H, 128] tensors (batch 1, seqlen = T), sequence s
// = rows cu_seqlens[s] .. cu_seqlens[s+1] (device array, ascending, cu_seqlens[0] = 0 is not
// required), its state at slot state_indices[s] (or s). Workspace: the solve slots of at most
// ceil(T / C) + num_seqs chunks, then the chunk offsets.
size_t gdn_prefill_varlen_workspace(const pbk_gdn_desc& d, int num_seqs) {
  const size_t slots = (size_t)((d.seqlen + C - 1) / C + num_seqs) * d.hv * kSolveBytes;
  return slots + ((size_t)(num_seqs + 1) * sizeof(int32_t) + 15) / 16 * 16;
}

cudaError_t launch_gdn_prefill_varlen(const pbk_gdn_desc& d, const int32_t* cu_seqlens, int num_seqs, void* ws,
                                      cudaStream_t st) {
  const int max_chunks = (d.seqlen + C - 1) / C + num_seqs;
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int32_t* chunk_off = reinterpret_cast<int32_t*>(wsb + (size_t)max_chunks * d.hv * kSolveBytes);
  gdn_chunk_offsets_kernel<<<1, 1024, 0, st>>>(cu_seqlens, num_seqs, d.seqlen, chunk_off);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  SolveArgs sa;
  sa.k = static_cast<const bf16*>(d.k.data);
  sa.k_sb = d.k.stride_b;
  sa.k_st = d.k.stride_t;
  sa.k_sh = d.k.stride_h;
  sa.g = d.g.data;
  sa.g_sb = d.g.stride_b;
  sa.g_st = d.g.stride_t;
  sa.g_sh = d.g.stride_h;
  sa.g_dtype = d.g.dtype;
  sa.beta = d.beta.data;
  sa.b_sb = d.beta.stride_b;
  sa.b_st = d.beta.stride_t;
  sa.b_sh = d.beta.stride_h;
  sa.b_dtype = d.beta.dtype;
  sa.seqlen = d.seqlen;
  sa.hk = d.hk;
  sa.hv = d.hv;
  sa.ws = wsb;
  sa.cu_seqlens = cu_seqlens;
  sa.chunk_off = chunk_off;
  sa.num_seqs = num_seqs;
  sa.gc = nullptr;
  sa.ta = nullptr;
  if ((e = launch_solve(sa, (unsigned)max_chunks, 1, d.hv, d.hk, st)) != cudaSuccess) return e;
  // the recurrence: one CTA per (sequence, value head) over the packed tensors
  pbk_gdn_desc dv = d;
  dv.batch = num_seqs;  // CTAs and state slots per sequence; the tensors stay [1, T, H, 128]
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, d.q, d.hk, d) || !make_map(&mk, d.k, d.hk, d) || !make_map(&mv, d.v, d.hv, d))
    return cudaErrorInvalidValue;
  memset(&mo, 0, sizeof(mo));
  if (d.o.data != nullptr) {
    const bool obf = d.o.dtype == PBK_BF16;
    const uint64_t es = obf ? 2 : 4;
    const uint64_t dims[4] = {128, (uint64_t)d.seqlen, (uint64_t)d.hv, 1};
    const uint64_t strides[3] = {(uint64_t)d.o.stride_t * es, (uint64_t)d.o.stride_h * es, (uint64_t)d.o.stride_b * es};
    const uint32_t box[4] = {128, obf ? 64u : 32u, 1, 1};
    if (!make_tmap_plain(&mo, d.o.data, obf, 4, dims, strides, box)) return cudaErrorInvalidValue;
  }
  PrefillArgs a;
  fill_args(a, dv);
  a.solve = wsb;
  a.cu_seqlens = cu_seqlens;
  a.chunk_off = chunk_off;
  a.solve_slots = max_chunks;
  const dim3 grid((unsigned)((int64_t)num_seqs * d.hv));
  auto go = [&](auto kernel) {
    cudaError_t e2 = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e2 != cudaSuccess) return e2;
    kernel<<<grid, NT, kSmemBytes, st>>>(mq, mk, mv, mo, a);
    return cudaGetLastError();
  };
  return d.o.dtype == PBK_BF16 ? go(gdn_prefill_tc_kernel<bf16, true>) : go(gdn_prefill_tc_kernel<float, true>);
}

// ------------------------------------------------------------------ the layer's prefill
cudaError_t launch_gdn_out_norm(const pbk_out_norm_desc& d, cudaStream_t st);

namespace {
// Workspace of pbk_gdn_prefill_layer: the chunk records, then q, k, v and o (bf16, dense).
struct LayerWs {
  size_t rec, q, k, v, o, total;
};
LayerWs layer_ws(const pbk_gdn_layer_desc& d) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const size_t rows = (size_t)d.batch * d.seqlen;
  LayerWs w;
  w.rec = 0;
  w.q = up((size_t)d.batch * ((d.seqlen + C - 1) / C) * d.hv * kSolveBytes);
  w.k = w.q + up(rows * d.hk * D * 2);
  w.v = w.k + up(rows * d.hk * D * 2);
  w.o = w.v + up(rows * d.hv * D * 2);
  w.total = w.o + up(rows * d.hv * D * 2);
  return w;
}
pbk_view dense_view(const void* p, int heads, int seqlen) {
  pbk_view v;
  v.data = p;
  v.stride_h = D;
  v.stride_t = (int64_t)heads * D;
  v.stride_b = (int64_t)seqlen * heads * D;
  v.dtype = PBK_BF16;
  v.pad_ = 0;
  return v;
}
}  // namespace

size_t gdn_prefill_layer_workspace(const pbk_gdn_layer_desc& d) { return layer_ws(d).total; }

// GatedDeltaNetLayer.forward over a prefill (gated_deltanet.py:411-440): the conv-fused chunk
// solve (q, k, v, g, beta and the chunk records from the projection's channels), the
// recurrence from those records, then the gated output norm.
cudaError_t launch_gdn_prefill_layer(const pbk_gdn_layer_desc& d, void* ws, cudaStream_t st) {
  const LayerWs w = layer_ws(d);
  uint8_t* base = static_cast<uint8_t*>(ws);
  bf16* qb = reinterpret_cast<bf16*>(base + w.q);
  bf16* kb = reinterpret_cast<bf16*>(base + w.k);
  bf16* vb = reinterpret_cast<bf16*>(base + w.v);
  bf16* ob = reinterpret_cast<bf16*>(base + w.o);
  // the recurrence's problem over the produced tensors (its g / beta are never read: the
  // records carry the chunk scalars; they point at the gate inputs only to be valid)
  pbk_gdn_desc g;
  memset(&g, 0, sizeof(g));
  g.batch = d.batch;
  g.seqlen = d.seqlen;
  g.hk = d.hk;
  g.hv = d.hv;
  g.dk = g.dv = D;
  g.q = dense_view(qb, d.hk, d.seqlen);
  g.k = dense_view(kb, d.hk, d.seqlen);
  g.v = dense_view(vb, d.hv, d.seqlen);
  g.g = d.decay;
  g.beta = d.decay;
  g.o = dense_view(ob, d.hv, d.seqlen);
  g.h0 = d.state;
  g.state = d.state;
  g.state_slot_stride = d.state_slot_stride;
  g.state_layout = d.state_layout;
  g.state_indices = d.state_indices;
  g.scale = d.scale;

  SolveArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.k = kb;
  sa.seqlen = d.seqlen;
  sa.hk = d.hk;
  sa.hv = d.hv;
  sa.ws = base + w.rec;
  SolveConvArgs cv;
  memset(&cv, 0, sizeof(cv));
  cv.x = static_cast<const bf16*>(d.qkv.data);
  cv.x_sb = d.qkv.stride_b;
  cv.x_st = d.qkv.stride_t;
  cv.tail = d.tail.data;
  cv.tl_sb = d.tail.stride_b;
  cv.tl_st = d.tail.stride_t;
  cv.tl_sc = d.tail.stride_h;
  cv.tl_dtype = d.tail.dtype;
  cv.new_tail = const_cast<void*>(d.new_tail.data);
  cv.nt_sb = d.new_tail.stride_b;
  cv.nt_st = d.new_tail.stride_t;
  cv.nt_sc = d.new_tail.stride_h;
  cv.nt_dtype = d.new_tail.dtype;
  cv.conv_w = d.conv_weight;
  cv.width = d.conv_weight != nullptr ? d.width : 1;
  cv.l2mode = d.l2mode;
  cv.l2_eps = d.l2_eps;
  cv.qo = qb;
  cv.ko = kb;
  cv.vo = vb;
  cv.decay = d.decay.data;
  cv.d_sb = d.decay.stride_b;
  cv.d_st = d.decay.stride_t;
  cv.d_sh = d.decay.stride_h;
  cv.d_dtype = d.decay.dtype;
  cv.a_log = d.a_log;
  cv.dt_bias = d.dt_bias;
  cv.state_indices = d.state_indices;
  cv.err = device_error_word();
  // x as [B, T, channels] bf16; boxes of 128 channels x 71 steps (zero outside the tensor)
  CUtensorMap xmap;
  const uint64_t xdims[3] = {(uint64_t)(2 * d.hk + d.hv) * D, (uint64_t)d.seqlen, (uint64_t)d.batch};
  const uint64_t xstrides[2] = {(uint64_t)d.qkv.stride_t * 2, (uint64_t)d.qkv.stride_b * 2};
  const uint32_t xbox[3] = {(uint32_t)D, (uint32_t)kRawRows, 1};
  if (!make_tmap_plain(&xmap, d.qkv.data, true, 3, xdims, xstrides, xbox)) return cudaErrorInvalidValue;
  cudaError_t e =
      launch_solve(sa, (unsigned)((d.seqlen + C - 1) / C), (unsigned)d.batch, d.hv, d.hk, st, &cv, &xmap);
  if (e != cudaSuccess) return e;
  if ((e = launch_gdn_prefill_tc(g, base + w.rec, true, st)) != cudaSuccess) return e;
  pbk_out_norm_desc on;
  memset(&on, 0, sizeof(on));
  on.batch = d.batch;
  on.seqlen = d.seqlen;
  on.hv = d.hv;
  on.weight_dtype = d.o_norm_dtype;
  on.eps = d.norm_eps;
  on.o = g.o;
  on.gate = d.gate;
  on.gate.stride_h = d.gate.stride_h * D;  // [B, T, hv 128] channels -> [B, T, hv, 128]
  on.out = d.out;
  on.weight = d.o_norm;
  return launch_gdn_out_norm(on, st);
}

}  // namespace pbk
