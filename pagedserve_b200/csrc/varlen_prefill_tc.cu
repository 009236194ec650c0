// placeholder, replaced by the tcgen05 kernel
#include "varlen_prefill.h"
#include "../../include/pagedserve_b200.h"
namespace psb {
bool prefill_tc_supported(const PrefillParams&, int) { return false; }
int prefill_tc_launch(const PrefillParams&, int, cudaStream_t) { return PSB_ERR_UNSUPPORTED; }
}  // namespace psb
