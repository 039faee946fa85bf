// tcgen05 tensor-core SSD (bf16 inputs): placeholder until the kernel lands.
#include "common.cuh"
#include "kernels.h"

namespace alloy {
bool ssd_tc_supported(const SsdArgs&) { return false; }
int ssd_tc(const SsdArgs&, cudaStream_t) {
  return fail(ALLOY_ERR_UNSUPPORTED, "ssd_tc: not available");
}
}  // namespace alloy
