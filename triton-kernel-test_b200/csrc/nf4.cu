// nf4.cu -- NF4 base-weight dequantisation (the frozen LoRA base weight of
// low_rank_system_profile_backward.py:31, dequantised at :58 by bitsandbytes'
// F.dequantize_4bit(..., quant_type='nf4') before compute_lora_gradient).
//
// Format (bitsandbytes' 4-bit blockwise format, restated from its published
// description): the weight is flattened row-major into n values; consecutive
// blocks of `blocksize` values share one absolute maximum; value i is a 4-bit
// index into a 16-entry code table (the NF4 data type), two indices a byte,
// value 2j in the high nibble of byte j and value 2j+1 in the low nibble.
// The block statistics are either float32 (one per block) or nested: one
// 8-bit index per block into a 256-entry table, scaled per `blocksize2`
// blocks by a float32 and shifted by a float32 offset.
//
//   absmax_b = absmax[b]                                   (plain)
//   absmax_b = fl(fl(code2[absmax_q[b]] * absmax2[b / blocksize2]) + offset)   (nested)
//   out[i]   = bf16_rn(fl(code[q_i] * absmax_{i / blocksize}))
//
// fl() is float32 rounding; the reference's dequantisation produces float32
// (the weight's original dtype) and converts it to bf16 with .to(bfloat16),
// round to nearest even, which is what the one cvt.rn here does.
//
// HBM-bound: n/2 bytes of indices in (plus n/blocksize statistics), 2n bytes
// of bf16 out.  A thread turns one 4-byte word (8 values) into one 16-byte
// store, so each warp reads 128 contiguous bytes and writes 512; four words
// a thread are in flight per loop trip.  The code table sits in shared memory:
// its 16 floats fill 16 distinct banks, so a warp's 32 lookups never conflict.
#include "common.cuh"

namespace act {
namespace nf4 {

constexpr int THREADS = 256;
constexpr int UNROLL = 4;

struct Params {
    const uint32_t *words;      // packed indices as 4-byte words
    const uint8_t *bytes;       // the same, bytewise (tail)
    int64_t n, nwords;          // values; whole 8-value words
    int bshift;                 // log2(blocksize)
    const float *code;          // 16 entries
    const float *absmax;        // plain statistics, or null
    const uint8_t *absmax_q;    // nested statistics
    const float *absmax2;
    const float *code2;         // 256 entries
    int b2shift;                // log2(blocksize2)
    const float *offset;        // device, one float
    uint4 *out;                 // 8 bf16 a store
    uint16_t *out16;            // tail
};

template <bool NESTED>
__device__ __forceinline__ float block_absmax(const Params &p, const float *code2_s, float offset, int64_t b) {
    if constexpr (NESTED) {
        const float a = __fmul_rn(code2_s[__ldg(p.absmax_q + b)], __ldg(p.absmax2 + (b >> p.b2shift)));
        return __fadd_rn(a, offset);
    } else {
        return __ldg(p.absmax + b);
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

template <bool NESTED>
__global__ void __launch_bounds__(THREADS) nf4_dequant_kernel(Params p) {
    __shared__ float code_s[16];
    __shared__ float code2_s[NESTED ? 256 : 1];
    if (threadIdx.x < 16) code_s[threadIdx.x] = __ldg(p.code + threadIdx.x);
    if constexpr (NESTED)
        for (int i = threadIdx.x; i < 256; i += THREADS) code2_s[i] = __ldg(p.code2 + i);
    __syncthreads();
    const float offset = NESTED ? __ldg(p.offset) : 0.f;
    const int64_t stride = (int64_t)gridDim.x * THREADS;
    int64_t w = (int64_t)blockIdx.x * THREADS + threadIdx.x;
    for (; w + (UNROLL - 1) * stride < p.nwords; w += UNROLL * stride) {
        uint32_t q[UNROLL];
        float am[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            q[u] = __ldcs(p.words + w + u * stride);  // read once: streaming
            am[u] = block_absmax<NESTED>(p, code2_s, offset, ((w + u * stride) * 8) >> p.bshift);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t byte = (q[u] >> (8 * j)) & 0xffu;  // values 2j (high nibble), 2j+1 (low)
                o[j] = pack_bf16x2(__fmul_rn(code_s[byte >> 4], am[u]), __fmul_rn(code_s[byte & 15u], am[u]));
            }
            __stcs(p.out + w + u * stride, make_uint4(o[0], o[1], o[2], o[3]));
        }
    }
    for (; w < p.nwords; w += stride) {
        const uint32_t q = __ldcs(p.words + w);
        const float am = block_absmax<NESTED>(p, code2_s, offset, (w * 8) >> p.bshift);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t byte = (q >> (8 * j)) & 0xffu;
            o[j] = pack_bf16x2(__fmul_rn(code_s[byte >> 4], am), __fmul_rn(code_s[byte & 15u], am));
        }
        __stcs(p.out + w, make_uint4(o[0], o[1], o[2], o[3]));
    }
    // the values after the last whole word (fewer than 8): the grid's first thread
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        for (int64_t i = p.nwords * 8; i < p.n; ++i) {
            const uint32_t byte = p.bytes[i >> 1];
            const uint32_t idx = (i & 1) ? (byte & 15u) : (byte >> 4);
            const float v = __fmul_rn(code_s[idx], block_absmax<NESTED>(p, code2_s, offset, i >> p.bshift));
            p.out16[i] = (uint16_t)(pack_bf16x2(v, 0.f) & 0xffffu);
        }
    }
}

}  // namespace nf4
}  // namespace act

extern "C" int actcomp_nf4_dequant(const uint8_t *packed, int64_t n, int64_t blocksize, const float *code,
                                   const float *absmax, const uint8_t *absmax_q, const float *absmax2,
                                   const float *code2, int64_t blocksize2, const float *offset, uint16_t *out,
                                   void *stream) {
    using namespace act;
    ACT_CHECK(n >= 0, ACT_E_INVALID);
    if (n == 0) return ACT_OK;
    ACT_CHECK(packed && code && out, ACT_E_INVALID);
    ACT_CHECK(blocksize >= 8 && blocksize <= (1 << 20) && (blocksize & (blocksize - 1)) == 0, ACT_E_INVALID);
    const bool nested = absmax_q != nullptr;
    ACT_CHECK(nested != (absmax != nullptr), ACT_E_INVALID);  // exactly one kind of statistics
    if (nested) {
        ACT_CHECK(absmax2 && code2 && offset, ACT_E_INVALID);
        ACT_CHECK(blocksize2 >= 1 && blocksize2 <= (1 << 20) && (blocksize2 & (blocksize2 - 1)) == 0, ACT_E_INVALID);
    }
    ACT_CHECK(aligned(packed, 4) && aligned(out, 16), ACT_E_ALIGN);
    nf4::Params p{};
    p.words = reinterpret_cast<const uint32_t *>(packed);
    p.bytes = packed;
    p.n = n;
    p.nwords = n / 8;
    p.bshift = 63 - __builtin_clzll((unsigned long long)blocksize);
    p.code = code;
    p.absmax = absmax;
    p.absmax_q = absmax_q;
    p.absmax2 = absmax2;
    p.code2 = code2;
    p.b2shift = nested ? 63 - __builtin_clzll((unsigned long long)blocksize2) : 0;
    p.offset = offset;
    p.out = reinterpret_cast<uint4 *>(out);
    p.out16 = out;
    const int64_t need = (p.nwords + nf4::UNROLL - 1) / nf4::UNROLL;
    const int64_t cap = (int64_t)num_sms() * 8;
    const int64_t blocks = (need + nf4::THREADS - 1) / nf4::THREADS;
    const int grid = (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
    cudaStream_t s = as_stream(stream);
    if (nested) nf4::nf4_dequant_kernel<true><<<grid, nf4::THREADS, 0, s>>>(p);
    else nf4::nf4_dequant_kernel<false><<<grid, nf4::THREADS, 0, s>>>(p);
    return launch_status();
}
