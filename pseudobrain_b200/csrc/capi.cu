// The extern "C" entry points of libpbk: host-side validation, then one launch.
// Nothing here allocates device memory or synchronises the host.
#include <cstdint>

#include "common.cuh"

namespace pbk {
cudaError_t launch_gdn_decode(const pbk_gdn_desc& d, cudaStream_t st);
cudaError_t launch_gdn_prefill_simt(const pbk_gdn_desc& d, cudaStream_t st);
}

namespace {

bool dtype_ok(int32_t dt) { return dt == PBK_F32 || dt == PBK_BF16; }

// Compute capability 10.x, checked once per device and cached (immutable afterwards).
int check_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PBK_ERR_DEVICE;
  return pbk_device_check(dev);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int validate_gdn(const pbk_gdn_desc* d) {
  if (d == nullptr) return PBK_ERR_INVALID;
  if (d->batch < 0 || d->seqlen < 0 || d->hk < 1 || d->hv < 1) return PBK_ERR_INVALID;
  if (d->hv % d->hk != 0) return PBK_ERR_SHAPE;
  if (d->dk != 128 || d->dv != 128) return PBK_ERR_SHAPE;
  if (d->batch > 0) {
    if (!d->q.data || !d->k.data || !d->v.data || !d->g.data || !d->beta.data || !d->o.data || !d->state)
      return PBK_ERR_INVALID;
  }
  if (!dtype_ok(d->q.dtype) || d->k.dtype != d->q.dtype || d->v.dtype != d->q.dtype) return PBK_ERR_DTYPE;
  if (!dtype_ok(d->g.dtype) || !dtype_ok(d->beta.dtype) || !dtype_ok(d->o.dtype)) return PBK_ERR_DTYPE;
  if (d->state_layout != PBK_STATE_KV && d->state_layout != PBK_STATE_VK) return PBK_ERR_INVALID;
  if (d->state_slot_stride < (int64_t)d->hv * d->dk * d->dv) return PBK_ERR_INVALID;
  if (!aligned16(d->state) || (d->h0 && !aligned16(d->h0)) || (d->state_slot_stride & 3)) return PBK_ERR_ALIGN;
  if ((int64_t)d->batch * d->hv > INT32_MAX) return PBK_ERR_SHAPE;
  return PBK_OK;
}

}  // namespace

extern "C" {

int pbk_abi_version(void) { return PBK_ABI_VERSION; }

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
  return pbk::launch_gdn_decode(*desc, static_cast<cudaStream_t>(stream)) == cudaSuccess ? PBK_OK
                                                                                         : PBK_ERR_LAUNCH;
}

int pbk_gdn_prefill(const pbk_gdn_desc* desc, void* stream) {
  int st = validate_gdn(desc);
  if (st != PBK_OK) return st;
  if (desc->batch == 0) return PBK_OK;
  if ((st = check_current_device()) != PBK_OK) return st;
  return pbk::launch_gdn_prefill_simt(*desc, static_cast<cudaStream_t>(stream)) == cudaSuccess ? PBK_OK
                                                                                               : PBK_ERR_LAUNCH;
}

}  // extern "C"
