// tcgen05 (5th-generation tensor core) matmul for sm_100a: placeholder until the TMA/TMEM pipeline lands; every
// call is routed to the SIMT kernel of matmul.cu.
#include "common.cuh"

namespace nvb200 {

int matmul_tc_launch(void *, const void *, const void *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                     int64_t, int64_t, int64_t, int, int32_t *, cudaStream_t) {
  return NVB200_ERR_UNSUPPORTED;
}

}  // namespace nvb200
