// The extern "C" entry points of libpbk: host-side validation, then one launch.
// Nothing here allocates device memory or synchronises the host.
#include <cstdint>

#include "common.cuh"
#include "quest.cuh"
#include "swa.cuh"

namespace pbk {
cudaError_t launch_gdn_decode(const pbk_gdn_desc& d, cudaStream_t st);
cudaError_t launch_gdn_decode_ext(const pbk_gdn_desc& d, const pbk_decode_ext& e, cudaStream_t st);
cudaError_t launch_gdn_prefill_simt(const pbk_gdn_desc& d, cudaStream_t st);
bool gdn_prefill_tc_supported(const pbk_gdn_desc& d);
size_t gdn_prefill_tc_workspace(const pbk_gdn_desc& d);
cudaError_t launch_gdn_chunk_solve(const pbk_gdn_desc& d, void* ws, cudaStream_t st, const pbk_view* gc = nullptr,
                                   const pbk_view* ta = nullptr);
cudaError_t launch_gdn_prefill_simt(const pbk_gdn_desc& d, cudaStream_t st, const pbk_view* gc,
                                    const pbk_view* ta);
size_t gdn_prefill_varlen_workspace(const pbk_gdn_desc& d, int num_seqs);
cudaError_t launch_gdn_conv_norm(const pbk_conv_desc& d, cudaStream_t st);
cudaError_t launch_gdn_gating(const pbk_gating_desc& d, cudaStream_t st);
cudaError_t launch_gdn_out_norm(const pbk_out_norm_desc& d, cudaStream_t st);
cudaError_t launch_gdn_decode_layer(const pbk_gdn_layer_desc& d, cudaStream_t st);
size_t gdn_prefill_layer_workspace(const pbk_gdn_layer_desc& d);
cudaError_t launch_gdn_prefill_layer(const pbk_gdn_layer_desc& d, void* ws, cudaStream_t st);
cudaError_t launch_gdn_l2norm(const pbk_view& x, const pbk_view& out, int batch, int seqlen, int heads, int mode,
                              float eps, cudaStream_t st);
bool gdn_conv_width_ok(int width);
cudaError_t launch_gdn_prefill_varlen(const pbk_gdn_desc& d, const int32_t* cu_seqlens, int num_seqs, void* ws,
                                      cudaStream_t st);
cudaError_t launch_gdn_prefill_tc(const pbk_gdn_desc& d, void* solve_ws, bool solved, cudaStream_t st);
cudaError_t launch_quest_token_scores(const pbk_token_desc& d, cudaStream_t st);
cudaError_t launch_quest_token_rerank(const pbk_token_desc& d, cudaStream_t st);
cudaError_t launch_quest_row_ranks(const float* x, int64_t x_stride, int rows, int n, int32_t* ranks,
                                   int64_t r_stride, cudaStream_t st);
cudaError_t launch_gdn_segment_scan(const float* b, const float* m, const float* h0, float* starts, int batch,
                                    int nseg, int hv, cudaStream_t st);
}

namespace {

bool dtype_ok(int32_t dt) { return dt == PBK_F32 || dt == PBK_BF16; }

// The CUDA error behind this thread's last PBK_ERR_LAUNCH (cudaSuccess if none).
thread_local cudaError_t g_last_launch_error = cudaSuccess;

int launch_status(cudaError_t e) {
  if (e == cudaSuccess) return PBK_OK;
  g_last_launch_error = e;
  return PBK_ERR_LAUNCH;
}

// Compute capability 10.x, checked once per device and cached (immutable afterwards).
int check_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PBK_ERR_DEVICE;
  return pbk_device_check(dev);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// allow_null_o: prefill may run for its final state only (o.data == NULL).
int validate_gdn(const pbk_gdn_desc* d, bool allow_null_o = false) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->batch < 0 || d->seqlen < 0 || d->hk < 1 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->hv % d->hk != 0) return PBK_ERR_SHAPE;
  if (d->dk != 128 || d->dv != 128) return PBK_ERR_SHAPE;
  if (d->batch > 0) {
    if (!d->q.data || !d->k.data || !d->v.data || !d->g.data || !d->beta.data || !d->state) return PBK_ERR_INVALID;
    if (!d->o.data && !allow_null_o) return PBK_ERR_INVALID;
  }
  if (!dtype_ok(d->q.dtype) || d->k.dtype != d->q.dtype || d->v.dtype != d->q.dtype) return PBK_ERR_DTYPE;
  if (!dtype_ok(d->g.dtype) || !dtype_ok(d->beta.dtype) || !dtype_ok(d->o.dtype)) return PBK_ERR_DTYPE;
  if (d->state_layout != PBK_STATE_KV && d->state_layout != PBK_STATE_VK) return PBK_ERR_INVALID;
  if (d->state_slot_stride < (int64_t)d->hv * d->dk * d->dv) return PBK_ERR_INVALID;
  if (!aligned16(d->state) || (d->h0 && !aligned16(d->h0)) || (d->state_slot_stride & 3)) return PBK_ERR_ALIGN;
  if ((int64_t)d->batch * d->hv > INT32_MAX) return PBK_ERR_SHAPE;
  return PBK_OK;
}

constexpr size_t kWsAlign = 256;
size_t round_up(size_t x) { return (x + kWsAlign - 1) / kWsAlign * kWsAlign; }
bool aligned_elems(int64_t stride, int64_t elems) { return stride % elems == 0; }

// Head dims of the Quest, serving and per-token kernels (128: tensor-core scores and
// attention; 256: the SIMT kernels).
bool quest_dim_ok(int d) { return d == 128 || d == 256; }

int validate_swa(const pbk_swa_desc* d) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->batch < 0 || d->seqlen < 0 || d->h < 1 || d->kv < 1 || d->sinks < 0 || !(d->scale > 0.f))
    return PBK_ERR_INVALID;
  if (d->h % d->kv != 0 || d->d != 128) return PBK_ERR_SHAPE;
  if (d->q.dtype != PBK_BF16 || d->k.dtype != PBK_BF16 || d->v.dtype != PBK_BF16 || !dtype_ok(d->o.dtype))
    return PBK_ERR_DTYPE;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  const pbk_view* in[3] = {&d->q, &d->k, &d->v};
  for (const pbk_view* v : in) {
    if (v->data == nullptr) return PBK_ERR_INVALID;
    if (v->stride_b <= 0 || v->stride_t <= 0 || v->stride_h <= 0) return PBK_ERR_INVALID;
    if (!aligned16(v->data) || v->stride_b % 8 || v->stride_t % 8 || v->stride_h % 8) return PBK_ERR_ALIGN;
  }
  const int64_t ev = d->o.dtype == PBK_BF16 ? 8 : 4;  // elements per 16 bytes
  if (d->o.data == nullptr) return PBK_ERR_INVALID;
  if (!aligned16(d->o.data) || d->o.stride_b % ev || d->o.stride_t % ev || d->o.stride_h % ev) return PBK_ERR_ALIGN;
  return PBK_OK;
}

// Shapes, pointers and alignment shared by the Quest entry points. `need` selects
// which tensors must be present: 1 select, 2 attend, 4 gather.
int validate_quest(const pbk_quest_desc* d, int need) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->nq < 0 || d->t < 1 || d->kv < 1 || d->h < d->kv || d->page < 1 || d->n_arch < 0 || d->budget < 0 ||
      d->n_win < 0)
    return PBK_ERR_INVALID;
  if (d->h % d->kv != 0) return PBK_ERR_SHAPE;
  if (!quest_dim_ok(d->d)) return PBK_ERR_SHAPE;
  const int64_t rows_per_head = (int64_t)d->nq * d->t * (d->h / d->kv);
  if (rows_per_head * d->d * 4 > 220 * 1024) return PBK_ERR_SHAPE;  // query rows of one key head in shared memory
  if (!d->q || !d->pages) return PBK_ERR_INVALID;
  if (!aligned16(d->q) || !aligned_elems(d->q_stride_n, 8) || !aligned_elems(d->q_stride_t, 8) ||
      !aligned_elems(d->q_stride_h, 8))
    return PBK_ERR_ALIGN;
  const int npages = d->n_arch / d->page;
  if ((need & 1) && npages > 0) {
    if (!d->kmax || !d->kmin) return PBK_ERR_INVALID;
    if (!aligned16(d->kmax) || !aligned16(d->kmin) || !aligned_elems(d->bnd_stride_kv, 8) ||
        !aligned_elems(d->bnd_stride_p, 8))
      return PBK_ERR_ALIGN;
  }
  if (need & 6) {
    if (d->n_arch > 0 && (!d->keys || !d->values)) return PBK_ERR_INVALID;
    if (!aligned16(d->keys) || !aligned16(d->values) || !aligned_elems(d->arc_stride_kv, 8) ||
        !aligned_elems(d->arc_stride_n, 8))
      return PBK_ERR_ALIGN;
  }
  if (need & 2) {
    if (d->n_win > 0 && (!d->win_keys || !d->win_values || !d->kpos)) return PBK_ERR_INVALID;
    if (!aligned16(d->win_keys) || !aligned16(d->win_values) || !aligned_elems(d->win_stride_kv, 8) ||
        !aligned_elems(d->win_stride_n, 8))
      return PBK_ERR_ALIGN;
    if (!d->qpos || !d->out) return PBK_ERR_INVALID;
    if (d->out_dtype != PBK_F32 && d->out_dtype != PBK_BF16) return PBK_ERR_DTYPE;
  }
  return PBK_OK;
}

}  // namespace

extern "C" {

int pbk_abi_version(void) { return PBK_ABI_VERSION; }

const char* pbk_last_launch_error(void) { return cudaGetErrorString(g_last_launch_error); }

const char* pbk_status_string(int status) {
  switch (status) {
    case PBK_OK: return "ok";
    case PBK_ERR_INVALID: return "invalid argument";
    case PBK_ERR_SHAPE: return "unsupported shape";
    case PBK_ERR_DTYPE: return "unsupported dtype";
    case PBK_ERR_ALIGN: return "misaligned pointer or stride";
    case PBK_ERR_DEVICE: return "device is not sm_100 (B200)";
    case PBK_ERR_LAUNCH: return "CUDA launch failed";
    case PBK_ERR_TIMEOUT: return "device-side wait timed out";
    case PBK_ERR_WORKSPACE: return "workspace missing or too small";
    case PBK_ERR_TOO_LARGE: return "problem exceeds the fixed scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

int pbk_device_check(int device) {
  static int cached[64] = {0};  // 0 unknown, 1 ok, 2 not sm_100
  if (device < 0) return PBK_ERR_DEVICE;
  if (device < 64 && cached[device]) return cached[device] == 1 ? PBK_OK : PBK_ERR_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return PBK_ERR_DEVICE;
  }
  const int ok = (major == 10) ? 1 : 2;
  if (device < 64) cached[device] = ok;
  return ok == 1 ? PBK_OK : PBK_ERR_DEVICE;
}

int pbk_gdn_decode(const pbk_gdn_desc* desc, void* stream) {
  int st = validate_gdn(desc);
  if (st != PBK_OK) return st;
  if (desc->h0 != nullptr && desc->h0 != desc->state) {
    // Out-of-place: the kernel reads h0 and writes state; they must not overlap.
    const int64_t n = ((int64_t)desc->batch - 1) * desc->state_slot_stride + (int64_t)desc->hv * 128 * 128;
    const char* a = reinterpret_cast<const char*>(desc->h0);
    const char* b = reinterpret_cast<const char*>(desc->state);
    if (desc->state_indices == nullptr && a < b + n * 4 && b < a + n * 4) return PBK_ERR_INVALID;
  }
  if (desc->batch == 0) return PBK_OK;  // seqlen 0 still copies h0 into state
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_decode(*desc, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_decode_ext(const pbk_gdn_desc* desc, const pbk_decode_ext* ext, void* stream) {
  if (ext == nullptr) return PBK_ERR_INVALID;
  pbk_gdn_desc d = *desc;
  if (ext->gating) {  // desc->g / desc->beta are not read: let validation see the gate inputs
    d.g = ext->a;
    d.beta = ext->b;
  }
  if (ext->cu_seqlens != nullptr) d.seqlen = 1;  // rows come from cu_seqlens (validated on the device side)
  int st = validate_gdn(&d);
  if (st != PBK_OK) return st;
  if (desc->h0 != nullptr && desc->h0 != desc->state) return PBK_ERR_INVALID;  // the pool is updated in place
  if (ext->l2norm < 0 || ext->l2norm > 2 || !(ext->eps >= 0.f)) return PBK_ERR_INVALID;
  if (ext->gating) {
    if (!ext->a.data || !ext->b.data || !ext->a_log || !ext->dt_bias) return PBK_ERR_INVALID;
    if (!dtype_ok(ext->a.dtype) || !dtype_ok(ext->b.dtype) || !dtype_ok(ext->a_log_dtype) ||
        !dtype_ok(ext->dt_bias_dtype))
      return PBK_ERR_DTYPE;
    if (!(ext->softplus_beta > 0.f)) return PBK_ERR_INVALID;
  }
  if (ext->index_stride < 0 || (ext->index_stride > 0 && desc->state_indices == nullptr)) return PBK_ERR_INVALID;
  if (ext->num_accepted != nullptr && ext->index_stride == 0) return PBK_ERR_INVALID;
  if (desc->batch == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_decode_ext(*desc, *ext, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_prefill(const pbk_gdn_desc* desc, void* stream) {
  int st = validate_gdn(desc, true);
  if (st != PBK_OK) return st;
  if (desc->batch == 0) return PBK_OK;
  // state-only runs (no output) exist on the tensor-core path
  if (desc->o.data == nullptr && !pbk::gdn_prefill_tc_supported(*desc)) return PBK_ERR_INVALID;
  if ((st = check_current_device()) != PBK_OK) return st;
  // bf16 inputs: tensor-core kernel (bf16 operands, fp32 state and accumulation);
  // fp32 inputs: the exact fp32 kernel.
  const cudaError_t e = pbk::gdn_prefill_tc_supported(*desc)
                            ? pbk::launch_gdn_prefill_tc(*desc, nullptr, false, static_cast<cudaStream_t>(stream))
                            : pbk::launch_gdn_prefill_simt(*desc, static_cast<cudaStream_t>(stream));
  return launch_status(e);
}

size_t pbk_gdn_prefill_workspace(const pbk_gdn_desc* desc) {
  if (validate_gdn(desc, true) != PBK_OK || !pbk::gdn_prefill_tc_supported(*desc)) return 0;
  return pbk::gdn_prefill_tc_workspace(*desc);
}

int pbk_gdn_prefill_ws(const pbk_gdn_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  int st = validate_gdn(desc, true);
  if (st != PBK_OK) return st;
  if (desc->batch == 0) return PBK_OK;
  if (!pbk::gdn_prefill_tc_supported(*desc)) {  // no workspace use off the tensor-core path
    if (desc->o.data == nullptr) return PBK_ERR_INVALID;
    if ((st = check_current_device()) != PBK_OK) return st;
    return launch_status(pbk::launch_gdn_prefill_simt(*desc, static_cast<cudaStream_t>(stream)));
  }
  if (workspace == nullptr || workspace_bytes < pbk::gdn_prefill_tc_workspace(*desc)) return PBK_ERR_INVALID;
  if (!aligned16(workspace)) return PBK_ERR_ALIGN;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_prefill_tc(*desc, workspace, false, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_prefill_aux(const pbk_gdn_desc* desc, const pbk_view* gc, const pbk_view* a, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int st = validate_gdn(desc);
  if (st != PBK_OK) return st;
  if (gc == nullptr || a == nullptr || gc->data == nullptr || a->data == nullptr) return PBK_ERR_INVALID;
  if (gc->dtype != PBK_F32 || !dtype_ok(a->dtype)) return PBK_ERR_DTYPE;
  if (!aligned16(a->data) || a->stride_b % 8 || a->stride_t % 8 || a->stride_h % 8) return PBK_ERR_ALIGN;
  if (desc->batch == 0) return PBK_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!pbk::gdn_prefill_tc_supported(*desc)) {
    if ((st = check_current_device()) != PBK_OK) return st;
    return launch_status(pbk::launch_gdn_prefill_simt(*desc, s, gc, a));
  }
  if (workspace == nullptr || workspace_bytes < pbk::gdn_prefill_tc_workspace(*desc)) return PBK_ERR_INVALID;
  if (!aligned16(workspace)) return PBK_ERR_ALIGN;
  if ((st = check_current_device()) != PBK_OK) return st;
  cudaError_t e = pbk::launch_gdn_chunk_solve(*desc, workspace, s, gc, a);
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(pbk::launch_gdn_prefill_tc(*desc, workspace, true, s));
}

// The two halves of pbk_gdn_prefill_ws (tensor-core path only).
static int check_solve_ws(const pbk_gdn_desc* desc, const void* workspace, size_t workspace_bytes) {
  int st = validate_gdn(desc, true);
  if (st != PBK_OK) return st;
  if (!pbk::gdn_prefill_tc_supported(*desc)) return PBK_ERR_INVALID;
  if (workspace == nullptr || workspace_bytes < pbk::gdn_prefill_tc_workspace(*desc)) return PBK_ERR_INVALID;
  if (!aligned16(workspace)) return PBK_ERR_ALIGN;
  return check_current_device();
}

int pbk_gdn_chunk_solve(const pbk_gdn_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  if (desc != nullptr && desc->batch == 0) return PBK_OK;
  const int st = check_solve_ws(desc, workspace, workspace_bytes);
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_chunk_solve(*desc, workspace, static_cast<cudaStream_t>(stream)));
}

// ---- layer pieces around the recurrence
static bool view_ok(const pbk_view& v) { return v.data != nullptr && dtype_ok(v.dtype); }

int pbk_gdn_conv_norm(const pbk_conv_desc* d, void* stream) {
  if (d == nullptr || d->batch < 0 || d->seqlen < 0 || d->hk < 1 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->weight != nullptr && !pbk::gdn_conv_width_ok(d->width)) return PBK_ERR_SHAPE;
  if (d->l2mode < 0 || d->l2mode > 2 || !(d->eps >= 0.f)) return PBK_ERR_INVALID;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (!view_ok(d->x) || !view_ok(d->q) || !view_ok(d->k) || !view_ok(d->v)) return PBK_ERR_INVALID;
  if (d->tail.data != nullptr && !dtype_ok(d->tail.dtype)) return PBK_ERR_DTYPE;
  if (d->new_tail.data != nullptr && (!dtype_ok(d->new_tail.dtype) || d->new_tail.data == d->tail.data))
    return PBK_ERR_INVALID;
  if (d->batch > 65535 || 2 * d->hk + d->hv > 65535) return PBK_ERR_SHAPE;  // grid y, z
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_conv_norm(*d, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_gating(const pbk_gating_desc* d, void* stream) {
  if (d == nullptr || d->batch < 0 || d->seqlen < 0 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (!view_ok(d->decay) || !view_ok(d->g) || !view_ok(d->beta) || !d->a_log || !d->dt_bias) return PBK_ERR_INVALID;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_gating(*d, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_out_norm(const pbk_out_norm_desc* d, void* stream) {
  if (d == nullptr || d->batch < 0 || d->seqlen < 0 || d->hv < 1 || !(d->eps >= 0.f)) return PBK_ERR_INVALID;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (!view_ok(d->o) || !view_ok(d->gate) || !view_ok(d->out) || !d->weight || !dtype_ok(d->weight_dtype))
    return PBK_ERR_INVALID;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_out_norm(*d, static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_decode_layer(const pbk_gdn_layer_desc* d, void* stream) {
  if (d == nullptr || d->batch < 0 || d->seqlen < 0 || d->hk < 1 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->hv % d->hk != 0) return PBK_ERR_SHAPE;
  if (d->conv_weight != nullptr && !pbk::gdn_conv_width_ok(d->width)) return PBK_ERR_SHAPE;
  if (d->l2mode < 0 || d->l2mode > 2 || !(d->l2_eps >= 0.f) || !(d->norm_eps >= 0.f)) return PBK_ERR_INVALID;
  if (d->state_layout != PBK_STATE_KV && d->state_layout != PBK_STATE_VK) return PBK_ERR_INVALID;
  if ((int64_t)d->batch * d->hv > INT32_MAX) return PBK_ERR_SHAPE;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (!view_ok(d->qkv) || !view_ok(d->decay) || !view_ok(d->gate) || !view_ok(d->out)) return PBK_ERR_INVALID;
  if (!d->a_log || !d->dt_bias || !d->o_norm || !d->state) return PBK_ERR_INVALID;
  if (!dtype_ok(d->o_norm_dtype)) return PBK_ERR_DTYPE;
  if (d->tail.data != nullptr && !dtype_ok(d->tail.dtype)) return PBK_ERR_DTYPE;
  if (d->new_tail.data != nullptr && !dtype_ok(d->new_tail.dtype)) return PBK_ERR_DTYPE;
  const bool in_place = d->conv_weight != nullptr && d->width > 1 && d->new_tail.data != nullptr &&
                        d->new_tail.data == d->tail.data;
  if (in_place && (d->hv / d->hk > 8 || d->new_tail.dtype != d->tail.dtype ||
                   d->new_tail.stride_b != d->tail.stride_b || d->new_tail.stride_t != d->tail.stride_t ||
                   d->new_tail.stride_h != d->tail.stride_h))
    return PBK_ERR_SHAPE;  // in place: one cluster (at most 8 CTAs) per key head, identical views
  if (d->state_slot_stride < (int64_t)d->hv * 128 * 128) return PBK_ERR_INVALID;
  if (!aligned16(d->state) || (d->state_slot_stride & 3)) return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_decode_layer(*d, static_cast<cudaStream_t>(stream)));
}

// The prefill layer: the decode layer's checks plus the producer's (bf16 projection channels,
// contiguous, rows 16-byte aligned for its TMA copies; a separate new tail).
static int check_prefill_layer(const pbk_gdn_layer_desc* d) {
  if (d == nullptr || d->batch < 0 || d->seqlen < 0 || d->hk < 1 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->hv % d->hk != 0) return PBK_ERR_SHAPE;
  if (d->conv_weight != nullptr && !pbk::gdn_conv_width_ok(d->width)) return PBK_ERR_SHAPE;
  if (d->l2mode < 0 || d->l2mode > 2 || !(d->l2_eps >= 0.f) || !(d->norm_eps >= 0.f)) return PBK_ERR_INVALID;
  if (d->state_layout != PBK_STATE_KV && d->state_layout != PBK_STATE_VK) return PBK_ERR_INVALID;
  if (d->batch > 65535 || d->hv > 65535 || (int64_t)d->batch * d->hv > INT32_MAX) return PBK_ERR_SHAPE;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (!view_ok(d->qkv) || !view_ok(d->decay) || !view_ok(d->gate) || !view_ok(d->out)) return PBK_ERR_INVALID;
  if (!d->a_log || !d->dt_bias || !d->o_norm || !d->state) return PBK_ERR_INVALID;
  if (d->qkv.dtype != PBK_BF16 || !dtype_ok(d->o_norm_dtype)) return PBK_ERR_DTYPE;
  if (d->qkv.stride_h != 1 || (d->qkv.stride_t & 7) || (d->qkv.stride_b & 7) || d->qkv.stride_t <= 0 ||
      d->qkv.stride_b <= 0 || !aligned16(d->qkv.data) || d->gate.stride_h != 1)
    return PBK_ERR_ALIGN;  // the producer's TMA copies: 16-byte aligned rows
  if (d->tail.data != nullptr && !dtype_ok(d->tail.dtype)) return PBK_ERR_DTYPE;
  if (d->new_tail.data != nullptr && (!dtype_ok(d->new_tail.dtype) || d->new_tail.data == d->tail.data))
    return PBK_ERR_INVALID;  // the prefill's tail is read and written by different CTAs
  if (d->state_slot_stride < (int64_t)d->hv * 128 * 128) return PBK_ERR_INVALID;
  if (!aligned16(d->state) || (d->state_slot_stride & 3)) return PBK_ERR_ALIGN;
  return PBK_OK;
}

size_t pbk_gdn_prefill_layer_workspace(const pbk_gdn_layer_desc* d) {
  if (check_prefill_layer(d) != PBK_OK) return 0;
  return pbk::gdn_prefill_layer_workspace(*d);
}

int pbk_gdn_prefill_layer(const pbk_gdn_layer_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_prefill_layer(d);
  if (st != PBK_OK) return st;
  if (d->batch == 0 || d->seqlen == 0) return PBK_OK;
  if (workspace == nullptr || workspace_bytes < pbk::gdn_prefill_layer_workspace(*d)) return PBK_ERR_WORKSPACE;
  if (!aligned16(workspace)) return PBK_ERR_ALIGN;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_prefill_layer(*d, workspace, static_cast<cudaStream_t>(stream)));
}

int pbk_l2norm(pbk_view x, pbk_view out, int32_t batch, int32_t seqlen, int32_t heads, int32_t mode, float eps,
               void* stream) {
  if (batch < 0 || seqlen < 0 || heads < 1 || (mode != 1 && mode != 2) || !(eps >= 0.f)) return PBK_ERR_INVALID;
  if (batch == 0 || seqlen == 0) return PBK_OK;
  if (!view_ok(x) || !view_ok(out)) return PBK_ERR_INVALID;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_l2norm(x, out, batch, seqlen, heads, mode, eps, static_cast<cudaStream_t>(stream)));
}

// Packed varlen prefill (tensor-core path): desc describes [1, T, H, 128] tensors.
static int check_varlen(const pbk_gdn_desc* desc, const int32_t* cu_seqlens, int32_t num_seqs) {
  const int st = validate_gdn(desc, true);
  if (st != PBK_OK) return st;
  if (desc->batch != 1 || num_seqs < 0 || (num_seqs > 0 && cu_seqlens == nullptr)) return PBK_ERR_INVALID;
  if ((int64_t)num_seqs * desc->hv > INT32_MAX) return PBK_ERR_SHAPE;
  if (!pbk::gdn_prefill_tc_supported(*desc)) return PBK_ERR_INVALID;
  return PBK_OK;
}

size_t pbk_gdn_prefill_varlen_workspace(const pbk_gdn_desc* desc, int32_t num_seqs) {
  if (check_varlen(desc, nullptr, 0) != PBK_OK || num_seqs < 0) return 0;
  return round_up(pbk::gdn_prefill_varlen_workspace(*desc, num_seqs));
}

int pbk_gdn_prefill_varlen(const pbk_gdn_desc* desc, const int32_t* cu_seqlens, int32_t num_seqs, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int st = check_varlen(desc, cu_seqlens, num_seqs);
  if (st != PBK_OK) return st;
  if (num_seqs == 0 || desc->seqlen == 0) return PBK_OK;
  if (workspace == nullptr || workspace_bytes < pbk::gdn_prefill_varlen_workspace(*desc, num_seqs))
    return PBK_ERR_INVALID;
  if (!aligned16(workspace) || !aligned16(cu_seqlens)) return PBK_ERR_ALIGN;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_prefill_varlen(*desc, cu_seqlens, num_seqs, workspace,
                                                      static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_prefill_solved(const pbk_gdn_desc* desc, const void* workspace, size_t workspace_bytes, void* stream) {
  if (desc != nullptr && desc->batch == 0) return PBK_OK;
  const int st = check_solve_ws(desc, workspace, workspace_bytes);
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_gdn_prefill_tc(*desc, const_cast<void*>(workspace), true,
                                                  static_cast<cudaStream_t>(stream)));
}

int pbk_gdn_segment_scan(const float* b, const float* m, const float* h0, float* starts, int32_t batch, int32_t nseg,
                         int32_t hv, void* stream) {
  if (batch < 0 || nseg < 1 || hv < 1) return PBK_ERR_INVALID;
  if ((int64_t)batch * hv > INT32_MAX) return PBK_ERR_SHAPE;
  if (batch == 0) return PBK_OK;
  if (starts == nullptr || (nseg > 1 && (b == nullptr || m == nullptr))) return PBK_ERR_INVALID;
  if (!aligned16(starts) || (b && !aligned16(b)) || (m && !aligned16(m)) || (h0 && !aligned16(h0)))
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(
      pbk::launch_gdn_segment_scan(b, m, h0, starts, batch, nseg, hv, static_cast<cudaStream_t>(stream)));
}

size_t pbk_quest_select_workspace(const pbk_quest_desc* desc) {
  if (validate_quest(desc, 1) != PBK_OK) return 0;
  return round_up(pbk::quest_score_bytes(*desc));
}

size_t pbk_quest_attend_workspace(const pbk_quest_desc* desc) {
  if (validate_quest(desc, 2) != PBK_OK) return 0;
  return round_up(pbk::quest_partial_bytes(*desc, 0));
}

size_t pbk_quest_attend_sinks_workspace(const pbk_quest_desc* desc, int32_t n_sink) {
  if (validate_quest(desc, 2) != PBK_OK || n_sink < 0) return 0;
  return round_up(pbk::quest_partial_bytes(*desc, n_sink));
}

size_t pbk_quest_rerank_workspace(const pbk_quest_desc* desc, int32_t c) {
  if (desc == nullptr || c < 1 || desc->nq < 0 || desc->kv < 1) return 0;
  return round_up((size_t)desc->nq * desc->kv * c * sizeof(float));
}

int pbk_quest_select_parts(const pbk_quest_desc* desc, int32_t parts, void* workspace, size_t workspace_bytes,
                           void* stream) {
  int st = validate_quest(desc, 1);  // the full select descriptor for either part
  if (st != PBK_OK) return st;
  if (parts < 1 || parts > 3) return PBK_ERR_INVALID;
  const size_t need = pbk::quest_score_bytes(*desc);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return PBK_ERR_WORKSPACE;
  if (desc->nq == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  // workspace: the page scores (unless desc->scores keeps them), then the segment maxima
  return launch_status(pbk::launch_quest_select_parts(*desc, static_cast<float*>(workspace), parts,
                                                      static_cast<cudaStream_t>(stream)));
}

int pbk_quest_select(const pbk_quest_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  return pbk_quest_select_parts(desc, 3, workspace, workspace_bytes, stream);
}

int pbk_quest_select_noalloc(const pbk_quest_desc* desc, void* stream) {
  int st = validate_quest(desc, 1);
  if (st != PBK_OK) return st;
  const int64_t nscores = (int64_t)desc->nq * desc->kv * (desc->n_arch / desc->page);
  if (desc->scores == nullptr && nscores > PBK_QUEST_NOALLOC_MAX_SCORES) return PBK_ERR_TOO_LARGE;
  if (pbk::quest_select_floats(*desc) > pbk::kNoAllocFloats) return PBK_ERR_TOO_LARGE;
  if (desc->nq == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_quest_select_noalloc(*desc, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_attend_sinks(const pbk_quest_desc* desc, const void* sink_keys, const void* sink_values, int32_t n_sink,
                           int64_t sink_stride_kv, int64_t sink_stride_n, void* workspace, size_t workspace_bytes,
                           void* stream) {
  return pbk_quest_attend_parts(desc, sink_keys, sink_values, n_sink, sink_stride_kv, sink_stride_n, 7, workspace,
                                workspace_bytes, stream);
}

int pbk_quest_attend_parts(const pbk_quest_desc* desc, const void* sink_keys, const void* sink_values, int32_t n_sink,
                           int64_t sink_stride_kv, int64_t sink_stride_n, int32_t parts, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int st = validate_quest(desc, 2);
  if (st != PBK_OK) return st;
  if (n_sink < 0 || parts < 1 || parts > 7) return PBK_ERR_INVALID;
  if (n_sink > 0) {
    if (!sink_keys || !sink_values) return PBK_ERR_INVALID;
    if (!aligned16(sink_keys) || !aligned16(sink_values) || !aligned_elems(sink_stride_kv, 8) ||
        !aligned_elems(sink_stride_n, 8))
      return PBK_ERR_ALIGN;
  }
  const size_t need = pbk::quest_partial_bytes(*desc, n_sink);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return PBK_ERR_WORKSPACE;
  if (desc->nq == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  pbk::SinkKeys sk;
  sk.k = static_cast<const __nv_bfloat16*>(sink_keys);
  sk.v = static_cast<const __nv_bfloat16*>(sink_values);
  sk.s_kv = sink_stride_kv;
  sk.s_n = sink_stride_n;
  sk.n = n_sink;
  return launch_status(
      pbk::launch_quest_attend(*desc, static_cast<float*>(workspace), sk, parts, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_attend(const pbk_quest_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  return pbk_quest_attend_sinks(desc, nullptr, nullptr, 0, 0, 0, workspace, workspace_bytes, stream);
}

int pbk_quest_rerank(const pbk_quest_desc* desc, const int32_t* cand, int32_t c, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (desc == nullptr || cand == nullptr || c < 1) return PBK_ERR_INVALID;
  if (desc->nq < 0 || desc->t < 1 || desc->kv < 1 || desc->h % desc->kv != 0 || desc->page < 1 || desc->budget < 1)
    return PBK_ERR_INVALID;
  if (!quest_dim_ok(desc->d)) return PBK_ERR_SHAPE;
  if (!desc->q || !desc->keys || !desc->pages) return PBK_ERR_INVALID;
  if (!aligned16(desc->q) || !aligned_elems(desc->q_stride_n, 8) || !aligned_elems(desc->q_stride_t, 8) ||
      !aligned_elems(desc->q_stride_h, 8) || !aligned16(desc->keys) || !aligned_elems(desc->arc_stride_kv, 8) ||
      !aligned_elems(desc->arc_stride_n, 8))
    return PBK_ERR_ALIGN;
  const size_t need = (size_t)desc->nq * desc->kv * c * sizeof(float);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return PBK_ERR_WORKSPACE;
  if (desc->nq == 0) return PBK_OK;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(
      pbk::launch_quest_rerank(*desc, cand, c, static_cast<float*>(workspace), static_cast<cudaStream_t>(stream)));
}

int pbk_quest_gather(const pbk_quest_desc* desc, int32_t sel, void* out_keys, void* out_values, void* stream) {
  int st = validate_quest(desc, 4);
  if (st != PBK_OK) return st;
  if (sel < 0 || (sel > 0 && desc->n_arch / desc->page == 0)) return PBK_ERR_INVALID;
  if (!aligned16(out_keys) || !aligned16(out_values)) return PBK_ERR_ALIGN;
  if (desc->nq == 0) return PBK_OK;
  if (!out_keys || !out_values) return PBK_ERR_INVALID;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_quest_gather(*desc, sel, out_keys, out_values, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_bounds(const void* keys, int32_t kv, int32_t n, int32_t d, int32_t page, int64_t key_stride_kv,
                     int64_t key_stride_n, void* kmax, void* kmin, int64_t bnd_stride_kv, int64_t bnd_stride_p,
                     int32_t first_page, void* stream) {
  if (kv < 1 || n < 0 || page < 1 || first_page < 0) return PBK_ERR_INVALID;
  if (!quest_dim_ok(d)) return PBK_ERR_SHAPE;
  if (n == 0 || first_page * (int64_t)page >= n) return PBK_OK;
  if (!keys || !kmax || !kmin) return PBK_ERR_INVALID;
  if (!aligned16(keys) || !aligned16(kmax) || !aligned16(kmin) || key_stride_n % 8 || key_stride_kv % 8 ||
      bnd_stride_kv % 8 || bnd_stride_p % 8)
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_bounds(keys, kv, n, d, page, key_stride_kv, key_stride_n, kmax, kmin, bnd_stride_kv,
                                  bnd_stride_p, first_page, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_superbounds(const void* kmax, const void* kmin, int32_t kv, int32_t n_blk, int32_t d, int32_t sblk,
                          int64_t bnd_stride_kv, int64_t bnd_stride_p, void* smax, void* smin, int64_t sb_stride_kv,
                          int64_t sb_stride_p, int32_t first_sb, int32_t end_sb, void* stream) {
  if (kv < 1 || n_blk < 0 || sblk < 1 || first_sb < 0) return PBK_ERR_INVALID;
  if (!quest_dim_ok(d)) return PBK_ERR_SHAPE;
  if (n_blk == 0 || end_sb <= first_sb || first_sb * (int64_t)sblk >= n_blk) return PBK_OK;
  if (!kmax || !kmin || !smax || !smin) return PBK_ERR_INVALID;
  if (!aligned16(kmax) || !aligned16(kmin) || !aligned16(smax) || !aligned16(smin) || bnd_stride_kv % 8 ||
      bnd_stride_p % 8 || sb_stride_kv % 8 || sb_stride_p % 8)
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_superbounds(kmax, kmin, kv, n_blk, d, sblk, bnd_stride_kv, bnd_stride_p, smax,
                                                     smin, sb_stride_kv, sb_stride_p, first_sb, end_sb,
                                                     static_cast<cudaStream_t>(stream)));
}

int pbk_quest_rope_gather(const pbk_rope_gather_desc* d, void* stream) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->kv < 1 || d->block < 1 || d->n_blk < 0 || d->tail_n < 0 || d->n_rows < 0 || d->mode < 0 || d->mode > 3)
    return PBK_ERR_INVALID;
  if (!quest_dim_ok(d->d)) return PBK_ERR_SHAPE;
  if ((int64_t)d->n_blk * d->block + d->tail_n > INT32_MAX) return PBK_ERR_SHAPE;
  if ((int64_t)d->n_blk * d->block + d->tail_n == 0) return PBK_OK;
  if (!d->keys || !d->out_keys || (d->out_values && !d->values)) return PBK_ERR_INVALID;
  if (d->mode != 0 && d->n_blk > 0 && !d->inv_freq) return PBK_ERR_INVALID;
  if ((d->mode == 1 || d->mode == 2) && d->n_blk > 0 && (!d->blocks || !d->delta)) return PBK_ERR_INVALID;
  if (!aligned16(d->keys) || !aligned16(d->out_keys) || (d->values && !aligned16(d->values)) ||
      (d->out_values && !aligned16(d->out_values)) || !aligned_elems(d->stride_kv, 8) || !aligned_elems(d->stride_n, 8))
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_rope_gather(*d, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_archive_write(const pbk_archive_write_desc* d, void* stream) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->kv < 1 || d->block < 1 || d->origin < 0 || d->cap < 0 || d->size < 0 || d->n < 0 || d->p0 < 0)
    return PBK_ERR_INVALID;
  if (!quest_dim_ok(d->d)) return PBK_ERR_SHAPE;
  const bool blocks = d->blk_hi >= d->blk_lo;
  if (blocks && (d->blk_lo < 0 || (int64_t)d->origin + ((int64_t)d->blk_hi + 1) * d->block > (int64_t)d->cap + d->block))
    return PBK_ERR_INVALID;  // summarised blocks start inside the archive
  if (d->pos == nullptr && (int64_t)d->p0 + d->n > d->cap) return PBK_ERR_INVALID;
  if (d->n == 0 && !blocks) return PBK_OK;
  if (!d->keys || !d->values) return PBK_ERR_INVALID;
  if (d->n > 0 && (!d->k || !d->v)) return PBK_ERR_INVALID;
  if (blocks && (!d->kmax || !d->kmin)) return PBK_ERR_INVALID;
  if (!aligned16(d->keys) || !aligned16(d->values) || !aligned_elems(d->arc_stride_kv, 8) ||
      !aligned_elems(d->arc_stride_n, 8))
    return PBK_ERR_ALIGN;
  if (d->n > 0 && (!aligned16(d->k) || !aligned16(d->v) || !aligned_elems(d->in_stride_n, 8) ||
                   !aligned_elems(d->in_stride_kv, 8)))
    return PBK_ERR_ALIGN;
  if (blocks && (!aligned16(d->kmax) || !aligned16(d->kmin) || (d->kmean && !aligned16(d->kmean)) ||
                 (d->vmean && !aligned16(d->vmean)) || !aligned_elems(d->bnd_stride_kv, 8) ||
                 !aligned_elems(d->bnd_stride_p, 8)))
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_archive_write(*d, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_supermeans(const void* bmean, int32_t kv, int32_t n_blk, int32_t d, int32_t sblk, int64_t bnd_stride_kv,
                         int64_t bnd_stride_p, void* smean, int64_t sb_stride_kv, int64_t sb_stride_p,
                         int32_t first_sb, int32_t end_sb, void* stream) {
  if (kv < 1 || n_blk < 0 || sblk < 1 || first_sb < 0) return PBK_ERR_INVALID;
  if (!quest_dim_ok(d)) return PBK_ERR_SHAPE;
  if (n_blk == 0 || end_sb <= first_sb || first_sb * (int64_t)sblk >= n_blk) return PBK_OK;
  if (!bmean || !smean) return PBK_ERR_INVALID;
  if (!aligned16(bmean) || !aligned16(smean) || bnd_stride_kv % 8 || bnd_stride_p % 8 || sb_stride_kv % 8 ||
      sb_stride_p % 8)
    return PBK_ERR_ALIGN;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_supermeans(bmean, kv, n_blk, d, sblk, bnd_stride_kv, bnd_stride_p, smean,
                                                    sb_stride_kv, sb_stride_p, first_sb, end_sb,
                                                    static_cast<cudaStream_t>(stream)));
}

namespace {
int validate_levels(const pbk_quest_desc* d, const pbk_quest_levels* lv) {
  int st = validate_quest(d, 1);
  if (st != PBK_OK) return st;
  if (lv == nullptr) return PBK_ERR_INVALID;
  if (lv->smax == nullptr) return lv->smin == nullptr ? PBK_OK : PBK_ERR_INVALID;
  const int full = d->n_arch / d->page;
  if (!lv->smin || lv->sblk < 2) return PBK_ERR_INVALID;
  const int n_sb = (full + lv->sblk - 1) / lv->sblk;
  if (full > 0 && (lv->m_sb < 1 || lv->m_sb > n_sb)) return PBK_ERR_INVALID;
  if ((int64_t)lv->m_sb * lv->sblk > INT32_MAX / 2) return PBK_ERR_SHAPE;
  if (!aligned16(lv->smax) || !aligned16(lv->smin) || !aligned_elems(lv->sb_stride_kv, 8) ||
      !aligned_elems(lv->sb_stride_p, 8))
    return PBK_ERR_ALIGN;
  return PBK_OK;
}
}  // namespace

size_t pbk_quest_select_levels_workspace(const pbk_quest_desc* desc, const pbk_quest_levels* lv) {
  if (validate_levels(desc, lv) != PBK_OK) return 0;
  return round_up(pbk::quest_levels_bytes(*desc, *lv));
}

int pbk_quest_select_levels(const pbk_quest_desc* desc, const pbk_quest_levels* lv, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int st = validate_levels(desc, lv);
  if (st != PBK_OK) return st;
  if (desc->nq == 0 || desc->n_arch / desc->page == 0 || desc->budget == 0) return PBK_OK;
  const size_t need = pbk::quest_levels_bytes(*desc, *lv);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) return PBK_ERR_WORKSPACE;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_quest_select_levels(*desc, *lv, static_cast<uint8_t*>(workspace),
                                                       static_cast<cudaStream_t>(stream)));
}

int pbk_swa_prefill(const pbk_swa_desc* desc, void* stream) {
  int st = validate_swa(desc);
  if (st != PBK_OK || desc->batch == 0 || desc->seqlen == 0) return st;
  st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_swa_tc(*desc, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

// ------------------------------------------------------------------ per-token selection
namespace {
// `need`: 1 scores (bounds), 2 rescoring (keys).
int validate_token(const pbk_token_desc* d, int need) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->t < 0 || d->kv < 1 || d->h < d->kv || d->n_pool < 0) return PBK_ERR_INVALID;
  if (d->h % d->kv != 0 || d->h / d->kv > 32) return PBK_ERR_SHAPE;
  if (!quest_dim_ok(d->d)) return PBK_ERR_SHAPE;
  if (d->t == 0 || d->n_pool == 0) return PBK_OK;
  if (!d->q || !d->out) return PBK_ERR_INVALID;
  if (!aligned16(d->q) || !aligned_elems(d->q_stride_t, 8) || !aligned_elems(d->q_stride_h, 8)) return PBK_ERR_ALIGN;
  if (need & 1) {
    if (d->full < 1 || !d->kmax || !d->kmin) return PBK_ERR_INVALID;
    if (!aligned16(d->kmax) || !aligned16(d->kmin) || !aligned_elems(d->bnd_stride_kv, 8) ||
        !aligned_elems(d->bnd_stride_p, 8))
      return PBK_ERR_ALIGN;
  }
  if (need & 2) {
    if (d->block < 1 || !d->keys) return PBK_ERR_INVALID;
    if (!aligned16(d->keys) || !aligned_elems(d->key_stride_kv, 8) || !aligned_elems(d->key_stride_n, 8))
      return PBK_ERR_ALIGN;
  }
  return PBK_OK;
}
}  // namespace

extern "C" {

int pbk_quest_token_scores(const pbk_token_desc* desc, void* stream) {
  int st = validate_token(desc, 1);
  if (st != PBK_OK) return st;
  if (desc->t == 0 || desc->n_pool == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_quest_token_scores(*desc, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_token_rerank(const pbk_token_desc* desc, void* stream) {
  int st = validate_token(desc, 2);
  if (st != PBK_OK) return st;
  if (desc->t == 0 || desc->n_pool == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  return launch_status(pbk::launch_quest_token_rerank(*desc, static_cast<cudaStream_t>(stream)));
}

int pbk_quest_row_ranks(const float* x, int64_t x_stride, int32_t rows, int32_t n, int32_t* ranks,
                        int64_t ranks_stride, void* stream) {
  if (rows < 0 || n < 0 || n > 16384) return n > 16384 ? PBK_ERR_SHAPE : PBK_ERR_INVALID;
  if (rows == 0 || n == 0) return PBK_OK;
  if (x == nullptr || ranks == nullptr || x_stride < n || ranks_stride < n) return PBK_ERR_INVALID;
  int st = check_current_device();
  if (st != PBK_OK) return st;
  return launch_status(pbk::launch_quest_row_ranks(x, x_stride, rows, n, ranks, ranks_stride,
                                                   static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
