// tcgen05 BF16 GEMM (placeholder until the tensor-core kernel lands: every
// call is routed to the SIMT kernel by gemm_tc_supported()).
#include "kernels.h"

namespace ppocr {

bool gemm_tc_supported(const GemmParams&) { return false; }

cudaError_t launch_gemm_tc(const GemmParams&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace ppocr
