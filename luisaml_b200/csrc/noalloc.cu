// lcml_fp8_gemm_rowquant_noalloc: the GEMM + per-row quantization entry point
// for callers that cannot give this library any device memory to use as
// scratch. Its only scratch, the per-row max |value| buffer, lives in a
// static device array compiled into the library.
#include "lcml_internal.h"

// Scratch rows available to the no-allocation entry point. 65536 rows x 4 B
// = 256 KiB, which every GPU that loads this library holds until the process
// exits. Every call shares this one array (it keeps the previous call's row
// maxima; each call zeroes the rows it uses before the GEMM writes them), so
// calls that overlap on the GPU, e.g. on two streams, race on it.
static constexpr int64_t kNoAllocMaxRows = 65536;
static __device__ __align__(256) float g_noalloc_row_amax[kNoAllocMaxRows];

namespace {

// The device address of g_noalloc_row_amax on the current device. In host
// code the array's name only stands in for the device symbol, and its address
// is not a device address: handing it to a kernel would fault, or on a system
// where the GPU can reach host memory silently use the wrong memory. The
// address is looked up on every call rather than cached: after a
// cudaDeviceReset the module is loaded again, possibly elsewhere, and a cached
// address would dangle. Once the module is loaded the lookup is a table read.
int noalloc_scratch(float **out) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_row_amax);
    if (e != cudaSuccess)
        return lcml::set_error(LCML_ERR_CUDA, "no-allocation scratch: cudaGetSymbolAddress failed: %s",
                               cudaGetErrorString(e));
    *out = static_cast<float *>(p);
    return LCML_OK;
}

}// namespace

extern "C" int lcml_fp8_gemm_rowquant_noalloc(const lcml_fp8_gemm_desc *desc, uint8_t *q, float *q_scale,
                                              lcml_stream_t stream) {
    LCML_CHECK_ARG(desc != nullptr, "lcml_fp8_gemm_rowquant_noalloc: desc is NULL");
    if (desc->M > kNoAllocMaxRows)
        return lcml::set_error(LCML_ERR_INVALID_ARGUMENT,
                               "lcml_fp8_gemm_rowquant_noalloc: M = %lld rows exceeds the %lld-row scratch built "
                               "into the library; split the rows or use lcml_fp8_gemm_rowquant with a workspace",
                               static_cast<long long>(desc->M), static_cast<long long>(kNoAllocMaxRows));
    float *scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != LCML_OK) return rc;
    return lcml_fp8_gemm_rowquant(desc, q, q_scale, scratch, stream);
}
