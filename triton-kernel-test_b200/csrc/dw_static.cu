// dw_static.cu -- the weight gradient of actcomp_cg_dw without a caller
// workspace: the decoded activation goes to a file-scope device array owned by
// the library (ACTCOMP_DW_STATIC_SCRATCH_BYTES per device).  No device memory
// is allocated on the call path.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

// Scratch for the reconstructed activation (T x H bf16).  Every byte the GEMM
// reads is written by the decode of the same call first, so nothing in it has
// to start at zero.
static __device__ __align__(256) unsigned char g_dw_scratch[ACTCOMP_DW_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_addr[kMaxDevices];            // device address of g_dw_scratch in the context below
unsigned long long g_scratch_ctx[kMaxDevices];  // unique id of the context the address belongs to

// Unique id of the calling thread's current CUDA context (driver API through
// the runtime's entry-point query, so the library needs no libcuda at link
// time), or 0 when the driver cannot tell.  A context destroyed and created
// again (cudaDeviceReset, then any runtime call) gets a new id, and with it
// the module's device arrays move, so the cached address is looked up again.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static bool tried = false;
    if (!tried) {  // called under g_scratch_mu
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}
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
        const unsigned long long ctx = current_context_id();
        // first call on this device, its context was re-created since the lookup, or the
        // driver cannot identify the context (then the cheap host-side lookup runs every call)
        if (!g_scratch_addr[dev] || ctx != g_scratch_ctx[dev] || ctx == 0) {
            void *p = nullptr;
            ACT_CUDA_TRY(cudaGetSymbolAddress(&p, g_dw_scratch));  // this device is current
            g_scratch_addr[dev] = p;
            g_scratch_ctx[dev] = ctx;
        }
        scratch = g_scratch_addr[dev];
    }
    return actcomp_cg_dw(d, dy, N, lddy, dw, dw_dtype, lddw, scratch, ACTCOMP_DW_STATIC_SCRATCH_BYTES, stream);
}
