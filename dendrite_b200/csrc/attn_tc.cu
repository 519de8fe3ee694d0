// tcgen05 (TMEM-accumulator) path for cascade nodes with many query rows.
#include "dd_device.cuh"

extern "C" int dd_tc_available(void) { return 0; }

namespace dd {
int launch_attn_tc(const AttnArgs&, int64_t, int, cudaStream_t) {
  return fail(DD_ERR_NOT_AVAILABLE, "tcgen05 path not built");
}
}  // namespace dd
