// Chunked gated delta rule in exact fp32 on the CUDA cores (the fp32 path).
//
// Algorithm: the chunkwise WY form of pseudobrain/gated_deltanet.py:110-165. Per chunk
// of C = 64 steps with cumulative log decay c_t (gamma_t = exp(c_t)):
//   A_ti = beta_t (k_t . k_i) exp(c_t - c_i)  (i < t);   T = (I + A)^-1
//   W = T (K * beta gamma);   U' = T (V * beta)
//   U = U' - W S;   O = (Q gamma scale) S + (scale Q K^T * D) U;   S <- gamma_C S + (exp(c_C - c_i) k_i)^T U
// Padded steps past the sequence end are identity steps (k = v = 0, g = 0, beta = 0).
//
// One CTA of 256 threads owns one (sequence, value head, value-column slice of DVB)
// chain and walks its chunks in order; everything lives in shared memory as fp32, so
// the result differs from the reference only by summation order. The (I + A)^-1
// forward substitution runs four threads per column. This kernel is the precision
// reference of the build (the bf16 inputs path runs on the tensor cores).
#include "common.cuh"

namespace pbk {
namespace {

constexpr int C = 64;        // chunk
constexpr int D = 128;       // dk == dv
constexpr int NT = 256;      // threads
constexpr int PD = D + 1;    // padded row strides (conflict-free column access)
constexpr int PC = C + 1;

template <int DVB>
struct Smem {
  float K[C * PD], Q[C * PD], W[C * PD];
  float V[C * (DVB + 1)], U[C * (DVB + 1)];
  float S[D * (DVB + 1)];
  float A[C * PC], M[C * PC], T[C * PC];
  float cum[C], gam[C], beta[C], tail[C];
};

// C[M x N] = sum_k a(m, k) b(k, n), then out(m, n, r, c, acc) with (r, c) the
// thread-local tile index of (m, n). Thread (ty, tx) owns rows
// ty + TY r and columns tx + TX c, so a warp reads b along n (consecutive words) and
// a as a broadcast.
template <int M, int N, int K, int RM, int RN, typename FA, typename FB, typename FO>
__device__ __forceinline__ void simt_gemm(FA a, FB b, FO out) {
  constexpr int TX = N / RN, TY = M / RM;
  static_assert(TX * TY == NT, "tile map must cover 256 threads");
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  float acc[RM][RN];
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) acc[r][c] = 0.f;
#pragma unroll 4
  for (int k = 0; k < K; ++k) {
    float av[RM], bv[RN];
#pragma unroll
    for (int r = 0; r < RM; ++r) av[r] = a(ty + TY * r, k);
#pragma unroll
    for (int c = 0; c < RN; ++c) bv[c] = b(k, tx + TX * c);
#pragma unroll
    for (int r = 0; r < RM; ++r)
#pragma unroll
      for (int c = 0; c < RN; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
  }
#pragma unroll
  for (int r = 0; r < RM; ++r)
#pragma unroll
    for (int c = 0; c < RN; ++c) out(ty + TY * r, tx + TX * c, r, c, acc[r][c]);
}

// Optional chunk outputs (pbk_gdn_prefill_aux), written by the first value-column slice: the
// in-chunk cumulative g [B, T, Hv] fp32 and the rows of T = (I + A)^-1 [B, T, Hv, 64].
struct ChunkAux {
  float* gc;
  int64_t gc_sb, gc_st, gc_sh;
  void* ta;
  int64_t ta_sb, ta_st, ta_sh;
  int ta_dtype;
};

template <typename TIn, typename TOut, int DVB>
__global__ void __launch_bounds__(NT, 1) gdn_prefill_simt_kernel(const pbk_gdn_desc d, const ChunkAux aux) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem<DVB>& sm = *reinterpret_cast<Smem<DVB>*>(smem_raw);
  const int j0 = blockIdx.x * DVB;
  const int b = blockIdx.y / d.hv, h = blockIdx.y % d.hv;
  const int hk = h / (d.hv / d.hk);
  const int tid = threadIdx.x;
  int64_t slot = b;
  if (d.state_indices != nullptr) {
    slot = d.state_indices[b];
    if (slot < 0) return;
  }
  const int64_t tile = slot * d.state_slot_stride + (int64_t)h * D * D;
  const bool vk = d.state_layout == PBK_STATE_VK;
  // S[dk][j] for this CTA's value columns.
  for (int e = tid; e < D * DVB; e += NT) {
    const int dd = e / DVB, j = e % DVB;
    const int64_t off = vk ? (int64_t)(j0 + j) * D + dd : (int64_t)dd * D + j0 + j;
    sm.S[dd * (DVB + 1) + j] = d.h0 != nullptr ? d.h0[tile + off] : 0.f;
  }
  const TIn* qg = reinterpret_cast<const TIn*>(d.q.data) + b * d.q.stride_b + hk * d.q.stride_h;
  const TIn* kg = reinterpret_cast<const TIn*>(d.k.data) + b * d.k.stride_b + hk * d.k.stride_h;
  const TIn* vg = reinterpret_cast<const TIn*>(d.v.data) + b * d.v.stride_b + h * d.v.stride_h + j0;
  TOut* og = reinterpret_cast<TOut*>(const_cast<void*>(d.o.data)) + b * d.o.stride_b + h * d.o.stride_h + j0;
  const float scale = d.scale;
  const int nchunks = (d.seqlen + C - 1) / C;

  for (int n = 0; n < nchunks; ++n) {
    const int t0 = n * C;
    // ---- load the chunk (identity padding past the end) ----
    for (int e = tid; e < C * D; e += NT) {
      const int t = e / D, dd = e % D;
      const bool in = t0 + t < d.seqlen;
      sm.K[t * PD + dd] = in ? to_f32(kg[(int64_t)(t0 + t) * d.k.stride_t + dd]) : 0.f;
      sm.Q[t * PD + dd] = in ? to_f32(qg[(int64_t)(t0 + t) * d.q.stride_t + dd]) : 0.f;
    }
    for (int e = tid; e < C * DVB; e += NT) {
      const int t = e / DVB, j = e % DVB;
      sm.V[t * (DVB + 1) + j] = t0 + t < d.seqlen ? to_f32(vg[(int64_t)(t0 + t) * d.v.stride_t + j]) : 0.f;
    }
    if (tid < C) {
      const bool in = t0 + tid < d.seqlen;
      const int64_t gi = b * d.g.stride_b + (int64_t)(t0 + tid) * d.g.stride_t + h * d.g.stride_h;
      const int64_t bi = b * d.beta.stride_b + (int64_t)(t0 + tid) * d.beta.stride_t + h * d.beta.stride_h;
      sm.cum[tid] = in ? load_any(d.g.data, gi, d.g.dtype) : 0.f;
      sm.beta[tid] = in ? load_any(d.beta.data, bi, d.beta.dtype) : 0.f;
    }
    __syncthreads();
    if (tid == 0) {  // inclusive cumsum, sequential like torch.cumsum
      float c = 0.f;
      for (int t = 0; t < C; ++t) {
        c += sm.cum[t];
        sm.cum[t] = c;
      }
    }
    __syncthreads();
    if (tid < C) sm.gam[tid] = expf(sm.cum[tid]);
    if (tid >= C && tid < 2 * C) sm.tail[tid - C] = expf(sm.cum[C - 1] - sm.cum[tid - C]);
    // T = I (filled below the diagonal by the substitution).
    for (int e = tid; e < C * C; e += NT) sm.T[(e / C) * PC + e % C] = (e / C == e % C) ? 1.f : 0.f;
    __syncthreads();

    // ---- A = strict_lower(beta_t K K^T D), M = lower(scale Q K^T D) ----
    simt_gemm<C, C, D, 4, 4>(
        [&](int t, int k) { return sm.K[t * PD + k]; }, [&](int k, int i) { return sm.K[i * PD + k]; },
        [&](int t, int i, int, int, float acc) {
          sm.A[t * PC + i] = i < t ? sm.beta[t] * acc * expf(sm.cum[t] - sm.cum[i]) : 0.f;
        });
    simt_gemm<C, C, D, 4, 4>(
        [&](int t, int k) { return sm.Q[t * PD + k]; }, [&](int k, int i) { return sm.K[i * PD + k]; },
        [&](int t, int i, int, int, float acc) {
          sm.M[t * PC + i] = i <= t ? scale * acc * expf(sm.cum[t] - sm.cum[i]) : 0.f;
        });
    __syncthreads();

    // ---- T = (I + A)^-1, forward substitution, 4 threads per column ----
    {
      const int col = tid >> 2, r = tid & 3;
      for (int i = 1; i < C; ++i) {
        float s = 0.f;  // empty sum for rows at or above the diagonal (i <= col)
        for (int m = col + r; m < i; m += 4) s = fmaf(sm.A[i * PC + m], sm.T[m * PC + col], s);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (r == 0 && i > col) sm.T[i * PC + col] = -s;
        __syncwarp();
      }
    }
    __syncthreads();
    if (blockIdx.x == 0 && (aux.gc != nullptr || aux.ta != nullptr)) {
      for (int e = tid; e < C * C; e += NT) {
        const int t = e / C, i = e % C;
        if (t0 + t >= d.seqlen) continue;
        if (aux.ta != nullptr) {
          const int64_t o = b * aux.ta_sb + (int64_t)(t0 + t) * aux.ta_st + h * aux.ta_sh + i;
          const float x = sm.T[t * PC + i];
          if (aux.ta_dtype == PBK_BF16) static_cast<__nv_bfloat16*>(aux.ta)[o] = __float2bfloat16_rn(x);
          else static_cast<float*>(aux.ta)[o] = x;
        }
        if (aux.gc != nullptr && i == 0)
          aux.gc[b * aux.gc_sb + (int64_t)(t0 + t) * aux.gc_st + h * aux.gc_sh] = sm.cum[t];
      }
    }

    // ---- W = T (K beta gamma) [C x D];  U' = T (V beta) [C x DVB] ----
    simt_gemm<C, D, C, 4, 8>(
        [&](int t, int i) { return sm.T[t * PC + i]; },
        [&](int i, int dd) { return sm.beta[i] * sm.gam[i] * sm.K[i * PD + dd]; },
        [&](int t, int dd, int, int, float acc) { sm.W[t * PD + dd] = acc; });
    simt_gemm<C, DVB, C, 4, DVB / 16>(
        [&](int t, int i) { return sm.T[t * PC + i]; },
        [&](int i, int j) { return sm.beta[i] * sm.V[i * (DVB + 1) + j]; },
        [&](int t, int j, int, int, float acc) { sm.U[t * (DVB + 1) + j] = acc; });
    __syncthreads();

    // ---- U = U' - W S ----
    simt_gemm<C, DVB, D, 4, DVB / 16>(
        [&](int t, int dd) { return sm.W[t * PD + dd]; },
        [&](int dd, int j) { return sm.S[dd * (DVB + 1) + j]; },
        [&](int t, int j, int, int, float acc) { sm.U[t * (DVB + 1) + j] -= acc; });
    __syncthreads();

    // ---- O = (Q gamma scale) S + M U ----
    {
      constexpr int RN = DVB / 16;
      float part[4][RN];
      simt_gemm<C, DVB, D, 4, RN>(
          [&](int t, int dd) { return sm.Q[t * PD + dd]; },
          [&](int dd, int j) { return sm.S[dd * (DVB + 1) + j]; },
          [&](int t, int, int r, int c, float acc) { part[r][c] = acc * sm.gam[t] * scale; });
      simt_gemm<C, DVB, C, 4, RN>(
          [&](int t, int i) { return sm.M[t * PC + i]; },
          [&](int i, int j) { return sm.U[i * (DVB + 1) + j]; },
          [&](int t, int j, int r, int c, float acc) {
            if (t0 + t < d.seqlen)
              og[(int64_t)(t0 + t) * d.o.stride_t + j] = from_f32<TOut>(part[r][c] + acc);
          });
    }
    __syncthreads();

    // ---- S = gamma_C S + (tail K)^T U ----
    {
      const float gl = sm.gam[C - 1];
      simt_gemm<D, DVB, C, 8, DVB / 16>(
          [&](int dd, int i) { return sm.tail[i] * sm.K[i * PD + dd]; },
          [&](int i, int j) { return sm.U[i * (DVB + 1) + j]; },
          [&](int dd, int j, int, int, float acc) { sm.S[dd * (DVB + 1) + j] = fmaf(gl, sm.S[dd * (DVB + 1) + j], acc); });
    }
    __syncthreads();
  }
  float* st = d.state + tile;
  for (int e = tid; e < D * DVB; e += NT) {
    const int dd = e / DVB, j = e % DVB;
    const int64_t off = vk ? (int64_t)(j0 + j) * D + dd : (int64_t)dd * D + j0 + j;
    st[off] = sm.S[dd * (DVB + 1) + j];
  }
}

template <typename TIn, typename TOut, int DVB>
cudaError_t launch_split(const pbk_gdn_desc& d, const ChunkAux& aux, cudaStream_t st) {
  auto kern = gdn_prefill_simt_kernel<TIn, TOut, DVB>;
  const int bytes = (int)sizeof(Smem<DVB>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  kern<<<dim3(D / DVB, (unsigned)((int64_t)d.batch * d.hv)), NT, bytes, st>>>(d, aux);
  return cudaGetLastError();
}

template <typename TIn, typename TOut>
cudaError_t launch_types(const pbk_gdn_desc& d, const ChunkAux& aux, cudaStream_t st) {
  // Few chains: split the value columns four ways so more SMs work; many: two.
  if ((int64_t)d.batch * d.hv * 2 < 148) return launch_split<TIn, TOut, 32>(d, aux, st);
  return launch_split<TIn, TOut, 64>(d, aux, st);
}

}  // namespace

cudaError_t launch_gdn_prefill_simt(const pbk_gdn_desc& d, cudaStream_t st, const pbk_view* gc,
                                    const pbk_view* ta) {
  ChunkAux aux{};
  if (gc != nullptr) {
    aux.gc = static_cast<float*>(const_cast<void*>(gc->data));
    aux.gc_sb = gc->stride_b;
    aux.gc_st = gc->stride_t;
    aux.gc_sh = gc->stride_h;
  }
  if (ta != nullptr) {
    aux.ta = const_cast<void*>(ta->data);
    aux.ta_sb = ta->stride_b;
    aux.ta_st = ta->stride_t;
    aux.ta_sh = ta->stride_h;
    aux.ta_dtype = ta->dtype;
  }
  const bool in_bf16 = d.q.dtype == PBK_BF16, out_bf16 = d.o.dtype == PBK_BF16;
  if (in_bf16 && out_bf16) return launch_types<__nv_bfloat16, __nv_bfloat16>(d, aux, st);
  if (in_bf16) return launch_types<__nv_bfloat16, float>(d, aux, st);
  if (out_bf16) return launch_types<float, __nv_bfloat16>(d, aux, st);
  return launch_types<float, float>(d, aux, st);
}

cudaError_t launch_gdn_prefill_simt(const pbk_gdn_desc& d, cudaStream_t st) {
  return launch_gdn_prefill_simt(d, st, nullptr, nullptr);
}

}  // namespace pbk
