// GEMM dispatch: the tcgen05 tensor-core kernel for BF16 storage when the
// operand shapes allow it, otherwise the FP32 SIMT kernel.
#include "kernels.h"

namespace ppocr {

cudaError_t launch_gemm_simt(const GemmParams& p, cudaStream_t stream);
cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream);

cudaError_t launch_gemm(const GemmParams& p, cudaStream_t stream) {
    if (p.w_tc && gemm_tc_supported(p)) return launch_gemm_tc(p, stream);
    if (rows_gemm_supported(p)) return launch_rows_gemm(p, stream);
    return launch_gemm_simt(p, stream);
}

}  // namespace ppocr
