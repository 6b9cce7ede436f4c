// GEMM dispatch: the tcgen05 tensor-core kernel for BF16 storage when the
// operand shapes allow it.  FP32: the streaming kernel for thin outputs
// (n <= 32, where its persistent row tiles measured fastest), otherwise the
// register-tiled SIMT kernel.  BF16 without tensor cores: the row kernel
// where its accumulators fit, else the SIMT kernel.
#include <mutex>
#include <set>
#include <utility>

#include "kernels.h"

namespace ppocr {

cudaError_t allow_dynamic_smem(const void* func, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({func, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({func, dev});
    return e;
}

cudaError_t launch_gemm(const GemmParams& p, cudaStream_t stream) {
    if (p.w_tc && gemm_tc_supported(p)) return launch_gemm_tc(p, stream);
    if (p.dtype == DT_F32) {
        if (p.n <= 32 && gemm_stream_supported(p)) return launch_gemm_stream(p, stream);
        return launch_gemm_simt(p, stream);
    }
    if (rows_gemm_supported(p)) return launch_rows_gemm(p, stream);
    return launch_gemm_simt(p, stream);
}

}  // namespace ppocr
