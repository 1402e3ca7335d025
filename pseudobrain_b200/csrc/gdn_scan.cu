// Segment scan of the chunked gated delta rule split along the sequence.
//
// Over a segment of whole 64-token chunks the recurrence of delta_rule_chunked
// (pseudobrain/gated_deltanet.py:157-163: U = U' - W S; S' = gamma_C S + tail^T U) is
// affine in the segment's initial state, S_out = A S_in + b, with A = prod(gamma_C I -
// tail^T W) over its chunks. Running a segment from zeros gives b and from the identity
// gives m = A + b, and both runs are independent of every other segment, so all
// segments of a long sequence run in parallel; this kernel then chains them:
//   starts[0] = h0,  starts[p + 1] = (m[p] - b[p]) starts[p] + b[p],
// exactly in fp32, after which every segment is run again from its true start.
//
// Grid (batch x value head, 4 column slices of 32); 256 threads, thread = (row, 16
// columns); the current start slice [128 x 32] lives in shared memory.
#include "common.cuh"

namespace pbk {
namespace {

constexpr int D = 128;
constexpr int kCols = 32;  // columns per CTA

__global__ void __launch_bounds__(256) gdn_segment_scan_kernel(const float* __restrict__ bseg,
                                                               const float* __restrict__ mseg,
                                                               const float* __restrict__ h0, float* __restrict__ starts,
                                                               int nseg, int hv) {
  __shared__ __align__(16) float s[D][kCols];
  const int bh = blockIdx.x;  // batch * hv + head
  const int batch = bh / hv, head = bh % hv;
  const int row = threadIdx.x >> 1;
  const int cl = (threadIdx.x & 1) * 16;  // local column of this thread's 16
  const int c0 = blockIdx.y * kCols + cl;
  const int64_t mat = (int64_t)D * D;
  // element (p, row, col) of a [batch, n, hv, D, D] array
  auto at = [&](int n, int p) { return ((int64_t)(batch * n + p) * hv + head) * mat + (int64_t)row * D + c0; };

  float acc[16];
  if (h0 != nullptr) {
    const float4* src = reinterpret_cast<const float4*>(h0 + ((int64_t)batch * hv + head) * mat + (int64_t)row * D + c0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 x = src[i];
      acc[4 * i] = x.x, acc[4 * i + 1] = x.y, acc[4 * i + 2] = x.z, acc[4 * i + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  }
  for (int p = 0;; ++p) {
    // acc holds starts[p] (row, c0..c0+15)
    float4* dst = reinterpret_cast<float4*>(starts + at(nseg, p));
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
    if (p + 1 >= nseg) break;
    __syncthreads();  // the previous step's readers of s are done
#pragma unroll
    for (int i = 0; i < 16; ++i) s[row][cl + i] = acc[i];
    __syncthreads();
    const float* brow = bseg + at(nseg - 1, p) - c0;  // row `row` of b[p]
    const float* mrow = mseg + at(nseg - 1, p) - c0;
    {
      const float4* bb = reinterpret_cast<const float4*>(brow + c0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 x = bb[i];
        acc[4 * i] = x.x, acc[4 * i + 1] = x.y, acc[4 * i + 2] = x.z, acc[4 * i + 3] = x.w;
      }
    }
#pragma unroll 2
    for (int j = 0; j < D; j += 4) {
      const float4 mm = *reinterpret_cast<const float4*>(mrow + j);
      const float4 bv = *reinterpret_cast<const float4*>(brow + j);
      const float a[4] = {mm.x - bv.x, mm.y - bv.y, mm.z - bv.z, mm.w - bv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4* sr = reinterpret_cast<const float4*>(&s[j + u][cl]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 x = sr[i];
          acc[4 * i] = fmaf(a[u], x.x, acc[4 * i]);
          acc[4 * i + 1] = fmaf(a[u], x.y, acc[4 * i + 1]);
          acc[4 * i + 2] = fmaf(a[u], x.z, acc[4 * i + 2]);
          acc[4 * i + 3] = fmaf(a[u], x.w, acc[4 * i + 3]);
        }
      }
    }
  }
}

}  // namespace

cudaError_t launch_gdn_segment_scan(const float* b, const float* m, const float* h0, float* starts, int batch,
                                    int nseg, int hv, cudaStream_t st) {
  const dim3 grid((unsigned)(batch * hv), D / kCols);
  gdn_segment_scan_kernel<<<grid, 256, 0, st>>>(b, m, h0, starts, nseg, hv);
  return cudaGetLastError();
}

}  // namespace pbk
