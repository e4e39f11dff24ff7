// dw_static.cu -- the weight gradient of actcomp_cg_dw without a caller
// workspace: the decoded activation goes to a file-scope device array owned by
// the library (ACTCOMP_DW_STATIC_SCRATCH_BYTES per device).  No device memory
// is allocated on the call path.
#include <mutex>

#include "common.cuh"

// Scratch for the reconstructed activation (T x H bf16).  Every byte the GEMM
// reads is written by the decode of the same call first, so nothing in it has
// to start at zero.
static __device__ __align__(256) unsigned char g_dw_scratch[ACTCOMP_DW_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_addr[kMaxDevices];  // device address of g_dw_scratch, looked up on the first call per device
}  // namespace

extern "C" int actcomp_cg_dw_static(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw,
                                    int32_t dw_dtype, int64_t lddw, void *stream) {
    ACT_CHECK(d, ACT_E_INVALID);
    const size_t need = actcomp_cg_dw_workspace(d, N);
    ACT_CHECK(need > 0, ACT_E_INVALID);
    ACT_CHECK(need <= ACTCOMP_DW_STATIC_SCRATCH_BYTES, ACT_E_WORKSPACE);  // T * H * 2 bytes must fit
    int dev = 0;
    ACT_CUDA_TRY(cudaGetDevice(&dev));
    ACT_CHECK(dev >= 0 && dev < kMaxDevices, ACT_E_UNSUPPORTED);
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            void *p = nullptr;
            ACT_CUDA_TRY(cudaGetSymbolAddress(&p, g_dw_scratch));  // this device is current
            g_scratch_addr[dev] = p;
        }
        scratch = g_scratch_addr[dev];
    }
    return actcomp_cg_dw(d, dy, N, lddy, dw, dw_dtype, lddw, scratch, ACTCOMP_DW_STATIC_SCRATCH_BYTES, stream);
}
