// bf16 / f16 flash attention on tcgen05.  Until the tensor-core kernel is in place this unit
// reports every request as "not handled", so the SIMT flash kernel runs.
#include "runtime.h"

namespace mt {

MT_STATUS_READER(read_status_attention)

size_t sdpa_tc_workspace(const mt_sdpa_desc&) { return 0; }

int run_sdpa_tc(const mt_sdpa_desc&, void*, size_t, cudaStream_t, bool* handled) {
  *handled = false;
  return MT_OK;
}

}  // namespace mt
