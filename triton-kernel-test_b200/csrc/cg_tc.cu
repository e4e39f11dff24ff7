// cg_tc.cu -- tensor-core (tcgen05) kernels of the channel-group format:
// decode and the fused consumers (elementwise product, SiLU and GELU backward).
//
// One tile = 128 tokens x 128 channels.  Per tile:
//   TMA warp   loads the low-rank codes of the 128 tokens (128 x r int8), the
//              quantised basis rows of the 128 channels (128 x r int8), the
//              residual codes (128 x 64 B for int4) and, for a consumer, the
//              second operand (128 x 128 bf16) into a 2-3 stage ring;
//   MMA warp   issues one tcgen05.mma kind::i8 (M=128, N=128, K=32) per 32
//              basis vectors: I = Lq . Vq^T, an exact int32 accumulator in TMEM
//              (double-buffered, 2 x 128 columns);
//   epilogue   (8 warps, or 4 with the Walsh-Hadamard rotation; one token row
//              per thread) reads I with tcgen05.ld, forms
//              xhat = bf16((u - 2^(b-1)) * s + I * sL) exactly as the oracle,
//              puts the outlier channels back, applies the consumer op, writes
//              the tile to a 128B-swizzled staging buffer and stores it by TMA.
// The kernel is persistent: one CTA per SM walks the tiles with a fixed stride.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgtc {

constexpr int CH = 128;    // channels per tile (MMA N)
constexpr int ROWS = 128;  // tokens per tile (MMA M)

struct DecParams {
    int64_t T, H;
    int rank, k, group, batch;
    const float *scales;
    const float *lr_scale;
    const uint16_t *outliers;
    const int32_t *idx;
    int ntb, ncc;
    int64_t ntiles;
};

template <int BITS, int OP, bool WHT, int RB>
struct DecLayout {
    static constexpr int LQ = RB ? ROWS * RB : 0;
    static constexpr int VQ = RB ? CH * RB : 0;
    static constexpr int CODES = ROWS * CH * BITS / 8;
    static constexpr int Y = OP == ACT_OP_DECODE ? 0 : ROWS * CH * 2;
    static constexpr int STAGE = LQ + VQ + CODES + Y;
    static constexpr int OUT = ROWS * CH * 2;
    static constexpr int S = (3 * STAGE + 2 * OUT <= 200 * 1024) ? 3 : 2;
    static constexpr int EW = WHT ? 4 : 8;  // epilogue warps
    static constexpr int THREADS = 64 + 32 * EW;
    static constexpr int BAR_OFF = S * STAGE + 2 * OUT;
    static constexpr int TOTAL = BAR_OFF + 512 + 1024;
    static constexpr int CODE_ROW = CH * BITS / 8;  // bytes of one token's codes in the tile
};

// byte offset of 16-byte chunk `c` of row `r` in a TMA tile with the given
// swizzle (row pitch = swizzle span)
template <int PITCH>
__device__ __forceinline__ int swz(int r, int c) {
    if constexpr (PITCH == 128) return r * 128 + ((c ^ (r & 7)) << 4);
    else if constexpr (PITCH == 64) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    else return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
}

__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf(float a, float b) {
    return (uint32_t)f2bf(a) | ((uint32_t)f2bf(b) << 16);
}

// 128-point unnormalised Walsh-Hadamard on registers (stages m = 1..64 as the oracle).
__device__ __forceinline__ void wht128_reg(float (&v)[128]) {
#pragma unroll
    for (int m = 1; m < 128; m <<= 1) {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
            if (!(i & m)) {
                float a = v[i], b = v[i + m];
                v[i] = __fadd_rn(a, b);
                v[i + m] = __fsub_rn(a, b);
            }
        }
    }
}

template <int BITS, int OP, bool WHT, int RB>
__global__ void __launch_bounds__(DecLayout<BITS, OP, WHT, RB>::THREADS, 1)
    cg_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_lq, const __grid_constant__ CUtensorMap tm_vq,
                        const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_y,
                        const __grid_constant__ CUtensorMap tm_out, DecParams p) {
    using L = DecLayout<BITS, OP, WHT, RB>;
    constexpr int off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *empty = full + L::S;
    uint64_t *tfull = empty + L::S;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::S; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], L::EW + (RB ? 1 : 0));
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], L::EW);
        }
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (RB && warp == 1) {
        tc::tmem_alloc(tmem_slot, 2 * CH);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = RB ? *tmem_slot : 0;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            if (RB) {
                tc::prefetch_tmap(&tm_lq);
                tc::prefetch_tmap(&tm_vq);
            }
            tc::prefetch_tmap(&tm_codes);
            int i = 0;
            for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++i) {
                const int s = i % L::S;
                const uint32_t ph = (i / L::S) & 1;
                if (!tc::mbar_wait(&empty[s], ph ^ 1, abort)) break;
                const int cc = (int)(tile % p.ncc);
                const int64_t bt = tile / p.ncc;
                const int tb = (int)(bt % p.ntb), b = (int)(bt / p.ntb);
                uint8_t *st = smem + s * L::STAGE;
                tc::mbar_arrive_expect_tx(&full[s], L::STAGE);
                if constexpr (RB > 0) {
                    tc::tma_load_3d(st, &tm_lq, &full[s], 0, tb * ROWS, b);
                    tc::tma_load_3d(st + L::LQ, &tm_vq, &full[s], 0, cc * CH, b);
                }
                tc::tma_load_3d(st + L::LQ + L::VQ, &tm_codes, &full[s], cc * L::CODE_ROW, tb * ROWS, b);
                if constexpr (OP != ACT_OP_DECODE) {
                    uint8_t *y = st + L::LQ + L::VQ + L::CODES;
                    tc::tma_load_3d(y, &tm_y, &full[s], cc * CH, tb * ROWS, b);
                    tc::tma_load_3d(y + ROWS * 128, &tm_y, &full[s], cc * CH + 64, tb * ROWS, b);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if constexpr (RB > 0) {
            if (lane == 0) {
                constexpr uint32_t idesc = tc::idesc_i8(ROWS, CH);
                constexpr tc::Swizzle SW = RB == 32 ? tc::SW_32B : tc::SW_64B;
                int i = 0;
                for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++i) {
                    const int s = i % L::S, b = i & 1;
                    const uint32_t ph = (i / L::S) & 1, bph = (i >> 1) & 1;
                    if (!tc::mbar_wait(&full[s], ph, abort)) break;
                    if (!tc::mbar_wait(&tempty[b], bph ^ 1, abort)) break;
                    tc::tc_fence_after();
                    uint8_t *st = smem + s * L::STAGE;
#pragma unroll
                    for (int kk = 0; kk < RB / 32; ++kk) {
                        const uint64_t ad = tc::smem_desc(st + kk * 32, 16, 8 * RB, SW);
                        const uint64_t bd = tc::smem_desc(st + L::LQ + kk * 32, 16, 8 * RB, SW);
                        tc::mma_i8(tmem + b * CH, ad, bd, idesc, kk > 0);
                    }
                    tc::mma_commit(&tfull[b]);
                    tc::mma_commit(&empty[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 2;
        const int q = warp & 3;              // TMEM lane quadrant of this warp
        const int h = WHT ? 0 : ew >> 2;     // column half (64 columns) when 8 warps
        constexpr int NC = WHT ? 128 : 64;   // columns per thread
        constexpr int NP = NC / 32;          // 32-column pieces per thread
        const int r = q * 32 + lane;         // row of the tile
        const int ngr = (int)(p.H / p.group);
        const bool leader = (ew == 0 && lane == 0);
        int32_t *sidx = reinterpret_cast<int32_t *>(tmem_slot + 8);  // outlier channels of the current slice
        int cur_slice = -1;

        // per-row scalars of a tile, loaded one tile ahead so their latency hides
        float nsc[NP], nsl = 0.f;
        auto prefetch = [&](int64_t tile) {
#pragma unroll
            for (int j = 0; j < NP; ++j) nsc[j] = 0.f;
            nsl = 0.f;
            if (tile >= p.ntiles) return;
            const int cc = (int)(tile % p.ncc);
            const int64_t bt = tile / p.ncc;
            const int tb = (int)(bt % p.ntb), sb = (int)(bt / p.ntb);
            const int64_t t = (int64_t)tb * ROWS + r;
            if (t >= p.T) return;
            const int64_t trow = (int64_t)sb * p.T + t;
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const int64_t c = (int64_t)cc * CH + h * 64 + 32 * j;
                if (c < p.H) nsc[j] = __ldg(p.scales + trow * ngr + c / p.group);
            }
            if (RB) nsl = __ldg(p.lr_scale + trow);
        };
        prefetch(blockIdx.x);

        int i = 0;
        for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++i) {
            const int s = i % L::S, b = i & 1, ob = i & 1;
            const uint32_t ph = (i / L::S) & 1, bph = (i >> 1) & 1;
            const int cc = (int)(tile % p.ncc);
            const int64_t bt = tile / p.ncc;
            const int tb = (int)(bt % p.ntb), sl_b = (int)(bt / p.ntb);
            float sc[NP];
#pragma unroll
            for (int j = 0; j < NP; ++j) sc[j] = nsc[j];
            const float sl = nsl;
            prefetch(tile + gridDim.x);

            // outlier channels of this slice, in shared memory
            if (p.k && sl_b != cur_slice) {
                tc::named_bar(2, 32 * L::EW);
                for (int j = ew * 32 + lane; j < p.k; j += 32 * L::EW) sidx[j] = __ldg(p.idx + (int64_t)sl_b * p.k + j);
                tc::named_bar(2, 32 * L::EW);
                cur_slice = sl_b;
            }
            bool ok = tc::mbar_wait(&full[s], ph, abort);
            if (RB) ok = ok && tc::mbar_wait(&tfull[b], bph, abort);
            if (!ok) break;
            tc::tc_fence_after();
            const int64_t t = (int64_t)tb * ROWS + r;
            const bool rv = t < p.T;
            const int64_t trow = (int64_t)sl_b * p.T + t;
            const int64_t c_first = (int64_t)cc * CH + h * 64;

            // low-rank term I: read up front without the rotation (its latency
            // overlaps the residual), piece by piece after it (registers)
            uint32_t I[WHT ? 32 : NC];
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + b * CH + h * 64;
            if constexpr (RB > 0 && !WHT) {
#pragma unroll
                for (int j = 0; j < NP; ++j)
                    tc::tmem_ld32(taddr + 32 * j, *reinterpret_cast<uint32_t(*)[32]>(&I[32 * j]));
            }

            // residual: w = (u - 2^(b-1)) * s
            const uint8_t *ct = smem + s * L::STAGE + L::LQ + L::VQ;
            float w[NC];
            constexpr float UOFF = 8388608.0f + (float)off;
#pragma unroll
            for (int c16 = 0; c16 < NC * BITS / 128; ++c16) {  // 16-byte code chunks
                const int chunk = (h * 64 * BITS / 8) / 16 + c16;
                const uint4 v = *reinterpret_cast<const uint4 *>(ct + swz<L::CODE_ROW>(r, chunk));
                const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 128 / BITS; ++e) {
                    const int col = c16 * (128 / BITS) + e;
                    const uint32_t u = (wd[e / (32 / BITS)] >> ((e % (32 / BITS)) * BITS)) & ((1u << BITS) - 1u);
                    w[col] = __fmul_rn(u2f_minus(u, UOFF), sc[col / 32]);
                }
            }
            if constexpr (WHT) {
                wht128_reg(w);
#pragma unroll
                for (int j = 0; j < NC; ++j) w[j] = __fmul_rn(w[j], 0.0078125f);
            }
            // xhat = fma(I, sL, w), in place
            if constexpr (RB > 0) {
                if constexpr (WHT) {
#pragma unroll
                    for (int j = 0; j < NP; ++j) {
                        tc::tmem_ld32(taddr + 32 * j, *reinterpret_cast<uint32_t(*)[32]>(&I[0]));
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) w[32 * j + e] = __fmaf_rn(i2f_exact((int)I[e]), sl, w[32 * j + e]);
                    }
                } else {
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < NC; ++j) w[j] = __fmaf_rn(i2f_exact((int)I[j]), sl, w[j]);
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[b]);
            }
            // outlier channels inside my columns (uniform over the warp): a mask
            // built from the shared copy of the slice's indices with two ballots
            uint64_t om[NC / 64];
            int olo[NC / 64];
#pragma unroll
            for (int g = 0; g < NC / 64; ++g) {
                om[g] = 0;
                olo[g] = 0;
                if (p.k) {
                    const int64_t lo_c = c_first + 64 * g;
                    uint64_t bits = 0;
                    int below = 0;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int j = lane + 32 * half;
                        const int64_t c = j < p.k ? (int64_t)sidx[j] : INT64_MAX;
                        below += __popc(__ballot_sync(0xffffffffu, c < lo_c));
                        if (c >= lo_c && c < lo_c + 64) bits |= 1ull << (c - lo_c);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) bits |= __shfl_xor_sync(0xffffffffu, bits, o);
                    om[g] = bits;
                    olo[g] = below;
                }
            }
            // bf16 reconstruction (the consumer ops take it as their input)
            if constexpr (OP != ACT_OP_DECODE) {
#pragma unroll
                for (int j = 0; j < NC; ++j) w[j] = rne_bf(w[j]);
            }
#pragma unroll
            for (int g = 0; g < NC / 64; ++g) {
                if (om[g]) {
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        if ((om[g] >> e) & 1ull) {
                            const int slot = olo[g] + __popcll(om[g] & ((1ull << e) - 1ull));
                            w[g * 64 + e] = rv ? bf2f(p.outliers[trow * p.k + slot]) : 0.f;
                        }
                    }
                }
            }
            // second operand and consumer op
            if constexpr (OP != ACT_OP_DECODE) {
                const uint8_t *yt = smem + s * L::STAGE + L::LQ + L::VQ + L::CODES;
#pragma unroll
                for (int g = 0; g < NC / 64; ++g) {
                    const uint8_t *box = yt + (h + g) * ROWS * 128;
#pragma unroll
                    for (int c16 = 0; c16 < 8; ++c16) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(box + swz<128>(r, c16));
                        const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int j = g * 64 + c16 * 8 + 2 * e;
                            w[j] = apply_op<OP>(w[j], lo_bf(wd[e]));
                            w[j + 1] = apply_op<OP>(w[j + 1], hi_bf(wd[e]));
                        }
                    }
                }
            }
            // this stage is no longer read by the epilogue
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);

            // staging buffer ob: free once the store issued two tiles ago has read it
            uint8_t *stg = smem + L::S * L::STAGE + ob * L::OUT;
            if (leader) tc::bulk_wait_read<1>();
            tc::named_bar(1, 32 * L::EW);
#pragma unroll
            for (int g = 0; g < NC / 64; ++g) {
                uint8_t *box = stg + (h + g) * ROWS * 128;
#pragma unroll
                for (int c16 = 0; c16 < 8; ++c16) {
                    const int j = g * 64 + c16 * 8;
                    uint4 v;
                    v.x = pack_bf16x2(w[j], w[j + 1]);
                    v.y = pack_bf16x2(w[j + 2], w[j + 3]);
                    v.z = pack_bf16x2(w[j + 4], w[j + 5]);
                    v.w = pack_bf16x2(w[j + 6], w[j + 7]);
                    *reinterpret_cast<uint4 *>(box + swz<128>(r, c16)) = v;
                }
            }
            tc::fence_proxy_async();
            tc::named_bar(1, 32 * L::EW);
            if (leader) {
                tc::tma_store_3d(&tm_out, stg, cc * CH, tb * ROWS, sl_b);
                tc::tma_store_3d(&tm_out, stg + ROWS * 128, cc * CH + 64, tb * ROWS, sl_b);
                tc::bulk_commit();
            }
        }
        if (leader) tc::bulk_wait<0>();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (RB && warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * CH);
    }
}

template <int BITS, int OP, bool WHT, int RB>
int launch_decode(const actcomp_cg_desc *d, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                  cudaStream_t stream) {
    using L = DecLayout<BITS, OP, WHT, RB>;
    const int64_t T = d->tokens, H = d->channels, B = d->batch;
    const int r = d->rank;
    CUtensorMap m_lq{}, m_vq{}, m_codes{}, m_y{}, m_out{};
    int st;
    const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (RB) {
        const auto sw = RB == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
        if ((st = make_map_3d(&m_lq, d->lr_codes, U8, 1, r, T, B, r, T * r, RB, ROWS, sw))) return st;
        if ((st = make_map_3d(&m_vq, d->basis_q, U8, 1, r, H, B, r, H * r, RB, CH, sw))) return st;
    }
    const int64_t rowb = H * BITS / 8;
    if ((st = make_map_3d(&m_codes, d->codes, U8, 1, rowb, T, B, rowb, T * rowb, L::CODE_ROW, ROWS,
                          BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if (OP != ACT_OP_DECODE &&
        (st = make_map_3d(&m_y, y, BF, 2, H, T, B, ldy, T * ldy, 64, ROWS, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_map_3d(&m_out, out, BF, 2, H, T, B, ldo, T * ldo, 64, ROWS, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    DecParams p{};
    p.T = T;
    p.H = H;
    p.rank = r;
    p.k = d->n_outlier;
    p.group = d->group;
    p.batch = d->batch;
    p.scales = d->scales;
    p.lr_scale = d->lr_scale;
    p.outliers = d->outliers;
    p.idx = d->outlier_idx;
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.ncc = (int)((H + CH - 1) / CH);
    p.ntiles = (int64_t)p.ntb * p.ncc * B;
    auto kern = cg_decode_tc_kernel<BITS, OP, WHT, RB>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    const int grid = (int)(p.ntiles < num_sms() ? p.ntiles : num_sms());
    kern<<<grid, L::THREADS, L::TOTAL, stream>>>(m_lq, m_vq, m_codes, m_y, m_out, p);
    return launch_status();
}

template <int BITS, int OP>
int dispatch_rb(const actcomp_cg_desc *d, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                cudaStream_t s) {
    const int rb = d->rank == 0 ? 0 : (d->rank <= 32 ? 32 : 64);
    if (d->wht) {
        if (rb == 0) return launch_decode<BITS, OP, true, 0>(d, y, ldy, out, ldo, s);
        if (rb == 32) return launch_decode<BITS, OP, true, 32>(d, y, ldy, out, ldo, s);
        return launch_decode<BITS, OP, true, 64>(d, y, ldy, out, ldo, s);
    }
    if (rb == 0) return launch_decode<BITS, OP, false, 0>(d, y, ldy, out, ldo, s);
    if (rb == 32) return launch_decode<BITS, OP, false, 32>(d, y, ldy, out, ldo, s);
    return launch_decode<BITS, OP, false, 64>(d, y, ldy, out, ldo, s);
}

}  // namespace cgtc
}  // namespace act

// Tensor-core decode / consumer path.  Requirements beyond the descriptor
// checks: 16-byte aligned row strides (ld % 8 == 0) and base pointers.
int act_cg_consume_tc(const actcomp_cg_desc *d, int op, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                      cudaStream_t s) {
    using namespace act::cgtc;
    if (d->tokens == 0) return ACT_OK;
    if (d->bits == 4) {
        switch (op) {
            case ACT_OP_DECODE: return dispatch_rb<4, ACT_OP_DECODE>(d, y, ldy, out, ldo, s);
            case ACT_OP_MUL: return dispatch_rb<4, ACT_OP_MUL>(d, y, ldy, out, ldo, s);
            case ACT_OP_SILU_BWD: return dispatch_rb<4, ACT_OP_SILU_BWD>(d, y, ldy, out, ldo, s);
            default: return dispatch_rb<4, ACT_OP_GELU_BWD>(d, y, ldy, out, ldo, s);
        }
    }
    switch (op) {
        case ACT_OP_DECODE: return dispatch_rb<8, ACT_OP_DECODE>(d, y, ldy, out, ldo, s);
        case ACT_OP_MUL: return dispatch_rb<8, ACT_OP_MUL>(d, y, ldy, out, ldo, s);
        case ACT_OP_SILU_BWD: return dispatch_rb<8, ACT_OP_SILU_BWD>(d, y, ldy, out, ldo, s);
        default: return dispatch_rb<8, ACT_OP_GELU_BWD>(d, y, ldy, out, ldo, s);
    }
}
