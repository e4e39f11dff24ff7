/*
 * actcomp.h -- C ABI of libactcomp.so, the B200 (sm_100a) activation-compression
 * kernels.  Plain pointers, sizes and strides; no C++ or torch types.
 *
 * Every entry point
 *   - returns ACT_OK (0) or a negative ACT_E_* code and never throws or exits;
 *   - validates its arguments on the host before launching anything;
 *   - launches only on the stream it is given (cudaStream_t passed as void*,
 *     NULL = legacy default stream) and does not synchronise;
 *   - reads and writes caller-owned device memory only (no allocation), unless
 *     the comment says otherwise.
 * bf16 tensors are passed as uint16_t* holding the raw bits.
 *
 * Each declaration names the reference function it replaces
 * (Ther-nullptr/Triton-Kernel-Test, file:line).  Two data formats exist:
 *   rc = reference-compatible: the reference's own layout (low-rank factors
 *        l (M,K), r (K,N) as inputs, per-column scale s, threshold outliers as a
 *        dense tensor, codes packed in 32-column blocks);
 *   cg = channel-group: projection onto a basis V (H x r), top-k outlier
 *        channels kept verbatim, optional 128-wide Walsh-Hadamard rotation,
 *        int4/int8 codes with per-token group-absmax scales.
 */
#ifndef ACTCOMP_H
#define ACTCOMP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ACTCOMP_ABI_VERSION 2

enum actcomp_status {
    ACT_OK = 0,
    ACT_E_INVALID = -1,     /* null pointer, bad shape or size, bad enum value */
    ACT_E_UNSUPPORTED = -2, /* well-formed but outside what the kernels implement */
    ACT_E_ALIGN = -3,       /* pointer or stride misaligned for vector/TMA access */
    ACT_E_CUDA = -4,        /* a CUDA runtime call or launch failed */
    ACT_E_NODEVICE = -5,    /* no usable sm_100 device */
    ACT_E_WORKSPACE = -6,   /* workspace missing or too small */
    ACT_E_TIMEOUT = -7,     /* a bounded device-side wait gave up (see actcomp_last_device_error) */
    ACT_E_BOUNDS = -8       /* bounds-checked build: a device-side index check failed */
};

/* Human-readable name of a status code (static storage). */
const char *actcomp_strerror(int status);
/* ACTCOMP_ABI_VERSION of the loaded library. */
int actcomp_abi_version(void);
/* Device-side error word of the current device: 0 when no bounded wait has
 * timed out (bit 0) and, in the bounds-checked build, no index check has failed
 * (bit 2) since the last call to actcomp_clear_device_error.  Synchronises the
 * given stream; returns ACT_E_TIMEOUT when the word records a timed-out wait,
 * ACT_E_BOUNDS when it records a failed index check, else ACT_OK (or a CUDA
 * error). */
int actcomp_last_device_error(void *stream, uint32_t *word);
int actcomp_clear_device_error(void *stream);
/* Failure-detection self-test (no reference counterpart): one CTA waits on an
 * mbarrier with the kernels' bounded wait cut to `polls` (1..2^24) polls.
 * With arrive == 0 nothing completes the barrier: the wait gives up, records
 * the timeout in the device error word and the kernel returns (no trap, no
 * hang); with arrive != 0 the wait completes and the word is untouched. */
int actcomp_selftest_bounded_wait(uint32_t polls, int32_t arrive, void *stream);

/* ========================================================= channel-group format
 * One compressed activation: `batch` independent slices, each a T x H bf16
 * matrix X (T tokens / rows, H channels / columns), stored as
 *   X = L . V^T + R,   L = X . V  (the projection onto a rank-r basis V),
 * with R the residual, its outlier channels kept verbatim and the rest
 * (optionally rotated by a 128-point Walsh-Hadamard transform per 128-channel
 * block) quantised to int4/int8 codes with per-token group-absmax scales.
 * All buffers hold the slices back to back, slice i at offset i * (per-slice size):
 *   codes       uint8   T x (H*bits/8)   int4: channel 2j in the low nibble
 *   scales      float   T x (H/group)    per-token group absmax / qmax
 *   lowrank     float   T x rank         L = X . V, float32 (may be NULL if rank == 0)
 *   outliers    bf16    T x n_outlier    verbatim values of the outlier channels
 *   outlier_idx int32   n_outlier        ascending channel indices
 *   basis_t     bf16    rank x H         V^T (the projection reads it)
 *   basis       bf16    H x rank         V (the CUDA-core reconstruction reads it)
 *   basis_tile  bf16    tile operand     V in the tensor-core kernels' shared-memory
 *                                        layout (may be NULL: the CUDA-core kernels run)
 * The basis is bf16: V is rounded to bf16 once, by actcomp_cg_basis_prepare,
 * and every kernel (and any checker) uses those values.  The low-rank term
 * L . V^T enters the arithmetic in float32; the tensor cores form it from L
 * split exactly into three bf16 pieces, L = hi + mid + lo (hi = bf16(L),
 * mid = bf16(L - hi), lo = L - hi - mid), each multiplied by the bf16 basis
 * with float32 accumulation.
 * Tile operand: per slice ceil(H/128) tiles of 128 channels; tile t row `row`
 * (channel 128 t + row) holds the row's rank values in W = 2 * RK bytes, RK =
 * rank rounded up to 16, 32 or 64, value j at byte 2 j, with the 16-byte chunk
 * c of the row stored at chunk c ^ s(row), s = (row >> 2) & 1 for W = 32,
 * (row >> 1) & 3 for W = 64, row & 7 for W = 128 (the swizzled K-major layout
 * tcgen05.mma reads), zero beyond the rank and beyond H.  Size: batch *
 * ceil(H/128) * 128 * W bytes.
 * bits in {4, 8}; group in {32, 64, 128} dividing H; rank in {0, 16, 32, 48, 64};
 * 0 <= n_outlier <= 64; wht requires H % 128 == 0 and group <= 128.          */
typedef struct actcomp_cg_desc {
    int64_t tokens;
    int64_t channels;
    int32_t bits;
    int32_t group;
    int32_t rank;
    int32_t n_outlier;
    int32_t wht;
    int32_t batch;
    uint8_t *codes;
    float *scales;
    float *lowrank;
    uint16_t *outliers;
    const int32_t *outlier_idx;
    const uint16_t *basis_t;
    const uint16_t *basis;
    const uint16_t *basis_tile;
} actcomp_cg_desc;

/* Round a basis V (batch x H x rank, float32 row-major) to bf16 and write it as
 * basis_t (batch x rank x H), basis (batch x H x rank) and, if non-NULL, the
 * tile operand basis_tile (layout above, padding included).  No reference
 * counterpart (the reference takes its factors l, r as given,
 * low_rank_extraction_fuse_compression_quantization.py:118). */
int actcomp_cg_basis_prepare(const float *V, int64_t H, int32_t rank, int32_t batch, uint16_t *basis_t,
                             uint16_t *basis, uint16_t *basis_tile, void *stream);

/* Encode x (batch x T x H bf16, row stride ldx elements, slice stride T*ldx)
 * into the buffers of d.  Replaces low_rank_addition_fuse_compression_quantization
 * (low_rank_extraction_fuse_compression_quantization.py:118) for the
 * channel-group format, with the outlier split of extraction_outlier_channel.py:11-14
 * and the optional block Walsh-Hadamard rotation. */
int actcomp_cg_encode(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, void *stream);

/* Reconstruct xhat (batch x T x H bf16, row stride ldo).  Replaces
 * low_rank_addition_fuse_decompression_dequantization
 * (low_rank_extraction_fuse_decompression_dequantization.py:116). */
int actcomp_cg_decode(const actcomp_cg_desc *d, uint16_t *xhat, int64_t ldo, void *stream);

/* Fused consumers: reconstruct xhat tile by tile and apply, never writing xhat.
 *   ACT_OP_MUL      out = xhat * y                 (extraction_fuse_hadamard.py:185, triton_hadamard_fuse_extraction)
 *   ACT_OP_SILU_BWD out = y * s(1 + xhat(1 - s))   (extraction_fuse_silu_backward.py:192; silu_backward.py:6)
 *   ACT_OP_GELU_BWD out = tanh-GELU'(xhat) * y     (gelu_backward.py:14,73)
 * y and out: batch x T x H bf16 with row strides ldy / ldo. */
enum actcomp_op { ACT_OP_DECODE = 0, ACT_OP_MUL = 1, ACT_OP_SILU_BWD = 2, ACT_OP_GELU_BWD = 3 };
int actcomp_cg_consume(const actcomp_cg_desc *d, int32_t op, const uint16_t *y, int64_t ldy, uint16_t *out,
                       int64_t ldo, void *stream);

/* Softmax backward with the saved probabilities read from compressed form:
 * dS = (dP - rowsum(dP * P^)) * P^ per row (softmax_backward.py:6,45).  Each
 * slice is one (batch, head) S x S probability matrix (T == H == S); causal != 0
 * forces P^[i][j] = 0 for j > i.  dp / ds: batch x S x S bf16, row stride ld.
 * With a workspace of actcomp_cg_softmax_workspace() bytes (per-row partial
 * dot products and row sums) P^ is formed by the tensor-core decode in two
 * passes; with workspace == NULL a CUDA-core kernel reconstructs P^ itself. */
size_t actcomp_cg_softmax_workspace(const actcomp_cg_desc *d);
int actcomp_cg_softmax_bwd(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld, int32_t causal,
                           void *workspace, size_t workspace_bytes, void *stream);

/* Weight gradient dW = xhat^T * dy with xhat reconstructed inside the GEMM
 * (extraction_fuse_matmul.py:224 triton_matmul_decompress, consumer math of
 * low_rank_system_profile_backward.py:14-18).  d->batch must be 1.
 * dy: T x N bf16 (row stride lddy); dw: H x N, dw_dtype 0 = float32, 1 = bf16,
 * row stride lddw.  workspace: actcomp_cg_dw_workspace() bytes of device memory. */
size_t actcomp_cg_dw_workspace(const actcomp_cg_desc *d, int64_t N);
int actcomp_cg_dw(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw, int32_t dw_dtype,
                  int64_t lddw, void *workspace, size_t workspace_bytes, void *stream);

/* Allocation-free variant of actcomp_cg_dw.  No reference counterpart: the
 * reference allocates its outputs with torch.empty and has no such entry point.
 * The decoded activation goes to a device array of
 * ACTCOMP_DW_STATIC_SCRATCH_BYTES (32 MiB) that the library reserves per device
 * when its kernels load, instead of a caller workspace.  For callers that cannot
 * allocate device memory on the call path: plain C / ctypes callers without an
 * allocator of their own, and code that must not call cudaMalloc / cudaFree
 * (both can synchronise the device).
 *   Limit: actcomp_cg_dw_workspace(d, N) -- T * H * 2 bytes rounded up to 256,
 *   e.g. 4096 tokens x 4096 channels -- must not exceed
 *   ACTCOMP_DW_STATIC_SCRATCH_BYTES; larger calls return ACT_E_WORKSPACE and
 *   launch nothing (use actcomp_cg_dw with a workspace).
 *   Nothing in the scratch has to start at zero: the decode writes all of it
 *   before the GEMM reads it.
 *   The scratch is shared by every call on a device: calls that overlap in time
 *   (on other streams or host threads) race on it -- serialise them.
 *   The first call on each device, with that device current, looks up the
 *   scratch's address (cudaGetSymbolAddress); make that first call before any
 *   stream capture.  The address is cached per device together with the id of
 *   the context it belongs to: after cudaDeviceReset the next call sees a new
 *   context and looks the address up again (so that call, too, should come
 *   before any capture). */
#define ACTCOMP_DW_STATIC_SCRATCH_BYTES ((size_t)32 << 20)
int actcomp_cg_dw_static(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw,
                         int32_t dw_dtype, int64_t lddw, void *stream);

/* dW = xhat^T * dy with the dequantisation inside the GEMM's producer, as
 * triton_matmul_decompress (extraction_fuse_matmul.py:224) reconstructs its
 * tiles while loading them (:151-221).  The GEMM follows the format instead of
 * rebuilding xhat: dW = Q^T dy + V (L^T dy), Q = bf16((u - 2^(b-1)) * s) made
 * from the codes in shared memory by dequantising warps (zero in the outlier
 * channels), V (L^T dy) a second K segment of the same accumulator (exact
 * bf16 pieces of the float32 L^T dy), and the outlier channels' rows
 * overwritten by outliers^T dy.  No T x H reconstruction is written.  The
 * result differs from actcomp_cg_dw (the GEMM of the bf16 reconstruction) by
 * the bf16 rounding of the residual instead of that of L V^T + R: about 5e-4
 * relative, both equally far (about 4e-3) from the GEMM of the uncompressed x.
 * Same arguments as actcomp_cg_dw; ACT_E_UNSUPPORTED for batch > 1, the
 * rotated format, H % 64 != 0, H < 256, T < 64 or n_outlier % 8 != 0.  workspace:
 * actcomp_cg_dw_fused_workspace() bytes (the low-rank and outlier terms:
 * (T + 2 H) * 3r * 2 + 3r * N * 6 + n_outlier * N * 4 bytes, rounded). */
size_t actcomp_cg_dw_fused_workspace(const actcomp_cg_desc *d, int64_t N);
int actcomp_cg_dw_fused(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw,
                        int32_t dw_dtype, int64_t lddw, void *workspace, size_t workspace_bytes, void *stream);

/* Column absmax of x (T x H, row stride ldx) and the k largest channels
 * (score descending, ties to the lower index), returned ascending in idx.
 * score_ws: H floats of device scratch.  Selection rule for the outlier
 * channels of extraction_outlier_channel.py:11-14 (which takes the list as input). */
int actcomp_cg_channel_topk(const uint16_t *x, int64_t T, int64_t H, int64_t ldx, int32_t k, int32_t *idx,
                            float *score_ws, void *stream);

/* Copy every buffer of a compressed activation between two descriptors with
 * identical shapes (device -> pinned host or back), one cudaMemcpyAsync per
 * buffer on `stream`.  Replaces the synchronous o.cpu()/q.cpu() of
 * offload_forward.py:55 and the reload of offload_backward.py:63. */
int actcomp_cg_copy(const actcomp_cg_desc *dst, const actcomp_cg_desc *src, void *stream);

/* ========================================================= reference-compatible
 * Shapes follow the reference wrappers: x (B,M,N) with strides (sxb, sxm, 1);
 * l (M,K) and r (K,N) contiguous (K <= 64); s (s_rows,N) bf16; codes q
 * (B,M,N*bits/8) contiguous; o dense bf16 (B,M,N) contiguous.  bits in
 * {1,2,4,8}; N % 32 == 0 when bits < 8. */
#define ACT_RC_TWIN_LOWRANK 1  /* round l@r to bf16 before subtracting (PyTorch twin)      */
#define ACT_RC_HALF_EVEN 2     /* torch.round instead of round-half-away (Triton kernel)   */
#define ACT_RC_SCALE_BATCH 4   /* use s[b,:] per batch instead of s[0,:] for every batch    */
#define ACT_RC_ROW_PACK 8      /* pack across the whole row instead of 32-column blocks     */
#define ACT_RC_OUTLIER_BF16 16 /* compare |x| > bf16(outlier) instead of the float value    */

typedef struct actcomp_rc_args {
    int64_t B, M, N;
    int32_t K;
    int32_t bits;
    int32_t flags;
    float outlier;
    const uint16_t *l;
    const uint16_t *r;
    const uint16_t *s;
    int64_t s_rows;
    const uint16_t *x; /* encode input / consumer second operand (b) */
    int64_t sxb, sxm;
    uint16_t *o;       /* encode output / decode input; may be NULL for decode */
    uint8_t *q;
    uint16_t *out;     /* decode / consumer output, contiguous (B,M,N) */
} actcomp_rc_args;

/* low_rank_addition_fuse_compression_quantization,
 * low_rank_extraction_fuse_compression_quantization.py:118 (kernel :13). */
int actcomp_rc_encode(const actcomp_rc_args *a, void *stream);
/* low_rank_addition_fuse_decompression_dequantization,
 * low_rank_extraction_fuse_decompression_dequantization.py:116 (kernel :13);
 * with op != ACT_OP_DECODE and a->x as the second operand:
 * triton_hadamard_fuse_extraction (extraction_fuse_hadamard.py:185) and
 * triton_silu_backward_fuse_extraction (extraction_fuse_silu_backward.py:192). */
int actcomp_rc_decode(const actcomp_rc_args *a, int32_t op, void *stream);

/* low_rank_addition, low_rank_extraction_speed.py:113 (kernel :12): out
 * (B,M,N contiguous) = bf16(x + l@r), uses l, r, K, x, sxb, sxm, out. */
int actcomp_rc_lowrank_add(const actcomp_rc_args *a, void *stream);

/* ========================================================= dense helpers
 * 3-D tensors (B,M,N) with per-tensor strides (b, m) in elements, unit stride in N. */
typedef struct actcomp_ew_args {
    int64_t B, M, N;
    const uint16_t *x;
    int64_t sxb, sxm;
    const uint16_t *g;
    int64_t sgb, sgm;
    uint16_t *out;
    int64_t sob, som;
} actcomp_ew_args;
/* triton_silu_backward (silu_backward.py:54), triton_gelu_backward
 * (gelu_backward.py:73), triton_hadamard (extraction_fuse_hadamard.py:62). */
int actcomp_elementwise(const actcomp_ew_args *a, int32_t op, void *stream);
/* triton_softmax_backward (softmax_backward.py:45): rows of length n. */
int actcomp_softmax_bwd(const uint16_t *y, const uint16_t *g, uint16_t *out, int64_t rows, int64_t n, int64_t ld,
                        void *stream);
/* torch_extract_unstructured (extraction_outlier_channel.py:5): outlier = x
 * where |x| > thr else 0, rest = x - outlier; n contiguous elements. */
int actcomp_extract_unstructured(const uint16_t *x, int64_t n, float thr, uint16_t *outlier, uint16_t *rest,
                                 void *stream);
/* torch_extract_channel (extraction_outlier_channel.py:11): gathers x[:, idx, :]
 * of a contiguous (B,M,N) tensor into out (B,k,N) and zeroes those rows of x. */
int actcomp_extract_channel(uint16_t *x, int64_t B, int64_t M, int64_t N, const int32_t *idx, int32_t k,
                            uint16_t *out, void *stream);

/* Dense GEMM on the tcgen05 tensor cores: C (batch x M x N) = A (M x K) * B (K x N)
 * per batch, fp32 accumulation.  a_kmajor: A stored M x K with row stride lda
 * (else K x M, i.e. A^T given); b_kmajor: B stored N x K with row stride ldb
 * (else K x N).  in_dtype 0 = bf16, 1 = fp16; c_dtype 0 = float32, 1 = bf16,
 * 2 = fp16; activation 0 = none, 1 = leaky_relu(0.01).  Batch strides in
 * elements (0 broadcasts).  matmul (triton_matmul.py:178), triton_batched_matmul
 * (extraction_fuse_matmul.py:59).  Requires M, N, K multiples of 8 for 16-byte
 * aligned rows. */
typedef struct actcomp_gemm_args {
    int64_t M, N, K;
    int32_t batch;
    int32_t in_dtype, c_dtype, activation;
    int32_t a_kmajor, b_kmajor;
    const void *A;
    int64_t lda, sa_batch;
    const void *B;
    int64_t ldb, sb_batch;
    void *C;
    int64_t ldc, sc_batch;
    /* Optional second K segment: C = A * B + A2 * B2, A2 (M x K2) and B2
     * (K2 x N) stored like A and B (same major-ness, row strides lda2, ldb2),
     * batch 1 only; K2 = 0 for none.  One accumulator in TMEM over K + K2:
     * compute_lora_gradient's dx = dy (w^T + b^T a^T) as dy w^T + (dy b^T) a^T
     * without forming w^T + b^T a^T (low_rank_system_profile_backward.py:15). */
    int64_t K2;
    const void *A2;
    int64_t lda2;
    const void *B2;
    int64_t ldb2;
} actcomp_gemm_args;
int actcomp_gemm(const actcomp_gemm_args *g, void *stream);

/* ========================================================= NF4 base weight
 * F.dequantize_4bit(w.t(), quant_state, quant_type='nf4') of bitsandbytes as
 * low_rank_system_profile_backward.py:58 calls it on the frozen LinearNF4 base
 * weight (:31) before compute_lora_gradient.  n values (the weight flattened
 * row-major), blocks of `blocksize` consecutive values (a power of two >= 8);
 * packed: ceil(n/2) bytes, value 2j in the high nibble of byte j, 2j+1 in the
 * low; code: 16 floats (the data type's values, quant_state.code).  Block
 * statistics, exactly one of:
 *   absmax (float per block), or
 *   absmax_q (uint8 per block) with absmax2 (float per blocksize2 blocks),
 *   code2 (256 floats) and offset (one float; device memory, like every
 *   pointer here): absmax_b = code2[absmax_q[b]] * absmax2[b / blocksize2] +
 *   *offset (float32, product then sum; the nested statistics of
 *   compress_statistics=True).
 * out[i] = bf16(code[q_i] * absmax_{i / blocksize}) (float32 product, round to
 * nearest even).  packed 4-byte aligned, out 16-byte aligned (ACT_E_ALIGN). */
int actcomp_nf4_dequant(const uint8_t *packed, int64_t n, int64_t blocksize, const float *code,
                        const float *absmax, const uint8_t *absmax_q, const float *absmax2,
                        const float *code2, int64_t blocksize2, const float *offset, uint16_t *out, void *stream);

/* Error statistics of a reconstruction against its original (n bf16 values):
 * out[0] += sum (a-b)^2, out[1] += sum b^2, out[2] = max(out[2], max|a-b|),
 * out[3] += count(a != b); out: 4 doubles of device memory (accumulated into,
 * so several tensors can share one vector before an all-reduce). */
int actcomp_error_stats(const uint16_t *a, const uint16_t *b, int64_t n, double *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* ACTCOMP_H */
