// Tensor-core (tcgen05) forward: placeholder until the sm_100a kernel lands.
#include "common.cuh"
#include "kernels.h"

namespace sdk {
bool fwd_tensorcore_supports(const FwdLaunch&) { return false; }
int fwd_tensorcore(const FwdLaunch&) { return SDK_ERR_UNSUPPORTED; }
}  // namespace sdk
