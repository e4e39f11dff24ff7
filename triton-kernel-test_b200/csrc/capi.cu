// capi.cu -- C ABI entry points of libactcomp that dispatch between kernels,
// plus status strings and the device error word.
#include <mutex>

#include "tc_ptx.cuh"

namespace act {
__device__ uint32_t g_device_error = 0;

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int validate_desc(const actcomp_cg_desc *d);
int gemm_launch(const actcomp_gemm_args *g, cudaStream_t stream);
}  // namespace act

int act_cg_encode_simt(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s);
int act_cg_consume_simt(const actcomp_cg_desc *d, int op, const uint16_t *y, int64_t ldy, uint16_t *out,
                        int64_t ldo, cudaStream_t s);
int act_cg_consume_tc(const actcomp_cg_desc *d, int op, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                      cudaStream_t s);
int act_cg_encode_rows(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s);
int act_cg_encode_split(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s);
int act_cg_softmax_simt(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld, int causal,
                        cudaStream_t s);
size_t act_cg_softmax_tc_workspace(const actcomp_cg_desc *d);
int act_cg_decode_rows(const actcomp_cg_desc *d, uint16_t *out, int64_t ldo, cudaStream_t s);
int act_cg_softmax_tc(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld, int causal,
                      void *workspace, cudaStream_t s);

using namespace act;

extern "C" const char *actcomp_strerror(int status) {
    switch (status) {
        case ACT_OK: return "ok";
        case ACT_E_INVALID: return "invalid argument";
        case ACT_E_UNSUPPORTED: return "unsupported configuration";
        case ACT_E_ALIGN: return "misaligned pointer or stride";
        case ACT_E_CUDA: return "CUDA runtime error";
        case ACT_E_NODEVICE: return "no usable sm_100 device";
        case ACT_E_WORKSPACE: return "workspace missing or too small";
        case ACT_E_TIMEOUT: return "device-side wait timed out";
        case ACT_E_BOUNDS: return "device-side index check failed (bounds-checked build)";
        default: return "unknown status";
    }
}

extern "C" int actcomp_abi_version(void) { return ACTCOMP_ABI_VERSION; }

extern "C" int actcomp_last_device_error(void *stream, uint32_t *word) {
    ACT_CHECK(word, ACT_E_INVALID);
    ACT_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    ACT_CUDA_TRY(cudaMemcpyFromSymbol(word, g_device_error, sizeof(uint32_t)));
    if (*word & DEV_ERR_MBAR_TIMEOUT) return ACT_E_TIMEOUT;
    return (*word & DEV_ERR_BOUNDS) ? ACT_E_BOUNDS : ACT_OK;
}

namespace act {
// One CTA waits on an mbarrier with the library's bounded wait cut to `polls`
// polls.  Without an arrival nothing completes the barrier, the wait gives up,
// sets the device error word and the kernel returns; with one, the wait ends
// at once and the word is left alone.
__global__ void selftest_wait_kernel(uint32_t polls, int arrive) {
    __shared__ uint64_t bar;
    __shared__ int abort_word;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        abort_word = 0;
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) tc::mbar_arrive(&bar);
        (void)tc::mbar_wait(&bar, 0, &abort_word, polls);
    }
}
}  // namespace act

extern "C" int actcomp_selftest_bounded_wait(uint32_t polls, int32_t arrive, void *stream) {
    ACT_CHECK(polls >= 1 && polls <= (1u << 24), ACT_E_INVALID);
    act::selftest_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(polls, arrive);
    return launch_status();
}

extern "C" int actcomp_clear_device_error(void *stream) {
    const uint32_t zero = 0;
    ACT_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    ACT_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(uint32_t)));
    return ACT_OK;
}

// Decode: the row kernel where it covers the format, else the piece kernel
// (narrow H), else the CUDA-core kernel.  Each declines (ACT_E_UNSUPPORTED,
// before launching anything) what it does not cover.
static int decode_tc(const actcomp_cg_desc *d, uint16_t *xhat, int64_t ldo, cudaStream_t s) {
    int st = act_cg_decode_rows(d, xhat, ldo, s);
    if (st != ACT_E_UNSUPPORTED) return st;
    st = act_cg_consume_tc(d, ACT_OP_DECODE, nullptr, 0, xhat, ldo, s);
    if (st != ACT_E_UNSUPPORTED) return st;
    return act_cg_consume_simt(d, ACT_OP_DECODE, nullptr, 0, xhat, ldo, s);
}

// Vector access requirements shared by the encode/decode kernels.
static int check_rows(const void *p, int64_t ld, int64_t H) {
    ACT_CHECK(p, ACT_E_INVALID);
    ACT_CHECK(ld >= H, ACT_E_INVALID);
    ACT_CHECK(aligned(p, 16) && ld % 8 == 0, ACT_E_ALIGN);
    return ACT_OK;
}

extern "C" int actcomp_cg_encode(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, void *stream) {
    int st = validate_desc(d);
    if (st) return st;
    if ((st = check_rows(x, ldx, d->channels))) return st;
    if (d->rank) ACT_CHECK(d->basis_t && aligned(d->basis_t, 16), ACT_E_ALIGN);
    // the two-kernel encode (projection, then quantisation: rank 16 or 32,
    // groups of 32 or 64, no rotation, one slice, H a multiple of 128), else
    // the two-pass row encode (1024 <= H <= 16384, a multiple of 128), else the
    // CUDA-core encode; each tensor-core encode declines (ACT_E_UNSUPPORTED,
    // before launching) what it does not cover
    st = act_cg_encode_split(d, x, ldx, as_stream(stream));
    if (st != ACT_E_UNSUPPORTED) return st;
    st = act_cg_encode_rows(d, x, ldx, as_stream(stream));
    if (st != ACT_E_UNSUPPORTED) return st;
    return act_cg_encode_simt(d, x, ldx, as_stream(stream));
}

extern "C" int actcomp_cg_decode(const actcomp_cg_desc *d, uint16_t *xhat, int64_t ldo, void *stream) {
    int st = validate_desc(d);
    if (st) return st;
    if ((st = check_rows(xhat, ldo, d->channels))) return st;
    return decode_tc(d, xhat, ldo, as_stream(stream));
}

extern "C" int actcomp_cg_consume(const actcomp_cg_desc *d, int32_t op, const uint16_t *y, int64_t ldy,
                                  uint16_t *out, int64_t ldo, void *stream) {
    int st = validate_desc(d);
    if (st) return st;
    ACT_CHECK(op >= ACT_OP_DECODE && op <= ACT_OP_GELU_BWD, ACT_E_INVALID);
    if ((st = check_rows(out, ldo, d->channels))) return st;
    if (op != ACT_OP_DECODE && (st = check_rows(y, ldy, d->channels))) return st;
    if (op == ACT_OP_DECODE) return decode_tc(d, out, ldo, as_stream(stream));
    st = act_cg_consume_tc(d, op, y, ldy, out, ldo, as_stream(stream));
    if (st != ACT_E_UNSUPPORTED) return st;
    return act_cg_consume_simt(d, op, y, ldy, out, ldo, as_stream(stream));
}

extern "C" size_t actcomp_cg_softmax_workspace(const actcomp_cg_desc *d) {
    if (!d || d->tokens <= 0 || d->channels <= 0 || d->batch <= 0) return 0;
    return act_cg_softmax_tc_workspace(d);
}

extern "C" int actcomp_cg_softmax_bwd(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld,
                                      int32_t causal, void *workspace, size_t workspace_bytes, void *stream) {
    int st = validate_desc(d);
    if (st) return st;
    ACT_CHECK(d->tokens == d->channels, ACT_E_INVALID);
    if ((st = check_rows(dp, ld, d->channels)) || (st = check_rows(ds, ld, d->channels))) return st;
    if (!workspace) return act_cg_softmax_simt(d, dp, ds, ld, causal != 0, as_stream(stream));
    ACT_CHECK(workspace_bytes >= act_cg_softmax_tc_workspace(d), ACT_E_WORKSPACE);
    ACT_CHECK(aligned(workspace, 16), ACT_E_ALIGN);
    st = act_cg_softmax_tc(d, dp, ds, ld, causal != 0, workspace, as_stream(stream));
    if (st != ACT_E_UNSUPPORTED) return st;
    return act_cg_softmax_simt(d, dp, ds, ld, causal != 0, as_stream(stream));
}

extern "C" size_t actcomp_cg_dw_workspace(const actcomp_cg_desc *d, int64_t N) {
    (void)N;
    if (!d || d->tokens <= 0 || d->channels <= 0) return 0;
    // the reconstructed activation, T x H bf16, 256-byte aligned
    return (size_t)(((d->tokens * d->channels * 2) + 255) / 256 * 256);
}

extern "C" int actcomp_cg_dw(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw,
                             int32_t dw_dtype, int64_t lddw, void *workspace, size_t workspace_bytes, void *stream) {
    int st = validate_desc(d);
    if (st) return st;
    ACT_CHECK(d->batch == 1, ACT_E_UNSUPPORTED);
    ACT_CHECK(dy && dw && N > 0 && lddy >= N && lddw >= N, ACT_E_INVALID);
    ACT_CHECK(dw_dtype == 0 || dw_dtype == 1, ACT_E_INVALID);
    ACT_CHECK(d->channels % 8 == 0 && N % 8 == 0 && lddy % 8 == 0 && aligned(dy, 16), ACT_E_ALIGN);
    const size_t need = actcomp_cg_dw_workspace(d, N);
    ACT_CHECK(workspace && workspace_bytes >= need, ACT_E_WORKSPACE);
    ACT_CHECK(aligned(workspace, 256), ACT_E_ALIGN);
    cudaStream_t s = as_stream(stream);
    uint16_t *xhat = static_cast<uint16_t *>(workspace);
    if ((st = decode_tc(d, xhat, d->channels, s))) return st;
    actcomp_gemm_args g{};
    g.M = d->channels;
    g.N = N;
    g.K = d->tokens;
    g.batch = 1;
    g.in_dtype = 0;
    g.c_dtype = dw_dtype == 0 ? 0 : 1;
    g.activation = 0;
    g.a_kmajor = 0;  // xhat is T x H: A^T given
    g.b_kmajor = 0;  // dy is T x N
    g.A = xhat;
    g.lda = d->channels;
    g.B = dy;
    g.ldb = lddy;
    g.C = dw;
    g.ldc = lddw;
    return gemm_launch(&g, s);
}

extern "C" int actcomp_cg_copy(const actcomp_cg_desc *dst, const actcomp_cg_desc *src, void *stream) {
    ACT_CHECK(dst && src, ACT_E_INVALID);
    ACT_CHECK(dst->tokens == src->tokens && dst->channels == src->channels && dst->bits == src->bits &&
                  dst->group == src->group && dst->rank == src->rank && dst->n_outlier == src->n_outlier &&
                  dst->batch == src->batch,
              ACT_E_INVALID);
    cudaStream_t s = as_stream(stream);
    const int64_t T = src->tokens * src->batch, H = src->channels;
    auto cp = [&](void *d, const void *sp, int64_t bytes) -> int {
        if (bytes <= 0) return ACT_OK;
        ACT_CHECK(d && sp, ACT_E_INVALID);
        ACT_CUDA_TRY(cudaMemcpyAsync(d, sp, (size_t)bytes, cudaMemcpyDefault, s));
        return ACT_OK;
    };
    int st;
    if ((st = cp(dst->codes, src->codes, T * H * src->bits / 8))) return st;
    if ((st = cp(dst->scales, src->scales, T * (H / src->group) * 4))) return st;
    if (src->rank && (st = cp(dst->lowrank, src->lowrank, T * src->rank * 4))) return st;
    if (src->n_outlier && (st = cp(dst->outliers, src->outliers, T * src->n_outlier * 2))) return st;
    return ACT_OK;
}
