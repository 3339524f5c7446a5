// tcgen05 + TMA decode attention (sm_100a). Not built yet: every shape goes to
// the CUDA-core kernel.
#include "decode_tc.h"
#include "../../include/pagedkv.h"

namespace pagedkv {

bool tc_eligible(int32_t, int32_t, int32_t, int32_t) { return false; }

size_t tc_workspace_bytes(int32_t, int32_t, int32_t, int32_t, int32_t, int32_t) { return 0; }

int tc_launch(DecodeParams &, int, void *, size_t, int32_t, cudaStream_t, int *launches,
              std::string *error) {
  *launches = 0;
  *error = "tensor-core decode kernel not built";
  return PAGEDKV_ERR_UNSUPPORTED;
}

}  // namespace pagedkv
