// Host entry of the sliding-window attention kernel (swa_tc.cu); arguments are
// validated by the C ABI (capi.cu) before this is called.
#pragma once

#include <cuda_runtime.h>

#include "../../include/pbk.h"

namespace pbk {

cudaError_t launch_swa_tc(const pbk_swa_desc& d, cudaStream_t st);

}  // namespace pbk
