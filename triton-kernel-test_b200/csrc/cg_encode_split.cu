// cg_encode_split.cu -- channel-group encode as two streaming kernels.
//
// Kernel 1, projection (cg_proj_kernel): L = X . V for one block of 128
// tokens per CTA.  Warp 0 streams X[128 x 64] and V^T[r x 64] boxes by TMA
// through an 8-stage ring (about 160 KB in flight per SM, what a single SM
// needs to pull its share of the HBM bandwidth), warp 1 issues tcgen05.mma
// kind::f16 (M=128, N=r) into one of two TMEM accumulators, warps 2-5 store L
// (float32, one token row per thread).
//
// Kernel 2, quantisation (cg_quant_kernel): 128-token x 128-channel tiles,
// persistent, each CTA a contiguous range of the tiles in the order the
// projection read them (least recently read first: under L2's LRU eviction
// the lines this kernel has used up go before the ones it still needs).
// Warp 0 streams each tile's X[128 x 128] by TMA (marked evict-first in L2,
// so that these loads do not push out the lines the projection left behind)
// and its prepared basis tile into a 3-stage
// ring; warp 2 splits each token block's L into three exact bf16 pieces (two
// buffered slots); warp 1 issues P = L . V^T (kind::f16, three pieces,
// float32 accumulation) into one of three TMEM accumulators; twelve epilogue
// warps in three groups of four take the tiles round-robin, a thread one
// token row x 128 channels: residual x - P with x from the ring, outlier
// channels copied out and zeroed, group absmax and scale, codes stored from
// registers (a thread's 64 bytes of its row per tile).  X reaches the SMs
// twice (once from HBM, once mostly from L2) and the two kernels split the
// work over every SM.
// Arithmetic is that of oracle/actcomp_oracle.c (cg_encode_given_lr) given the
// projection; the tensor cores sum L and P in float32 in their own order.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgsplit {

constexpr int ROWS = 128, KC = 64, CH = 128;

// ======================================================================== projection
constexpr int P_STAGES = 8;
constexpr int P_THREADS = 6 * 32;

struct ProjParams {
    int64_t T, H;
    int rank, ntb;
    float *lr;
};

template <int RK>
__global__ void __launch_bounds__(P_THREADS, 1)
    cg_proj_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_vt, ProjParams p) {
    constexpr int XB = ROWS * 128;                // X box: 128 rows x 64 bf16
    constexpr int SLOT = XB + RK * 128;           // + V^T box: RK rows x 64 bf16
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P_STAGES * SLOT);
    uint64_t *empty = full + P_STAGES;
    uint64_t *afull = empty + P_STAGES;  // [2]
    uint64_t *aempty = afull + 2;        // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(aempty + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = p.rank;
    const int nk = (int)(p.H / KC);

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(&afull[a], 1);
            tc::mbar_init(&aempty[a], 4);
        }
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 64);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tc::prefetch_tmap(&tm_x);
            tc::prefetch_tmap(&tm_vt);
            int i = 0;
            bool ok = true;
            for (int blk = blockIdx.x; blk < p.ntb && ok; blk += gridDim.x)
                for (int kb = 0; kb < nk; ++kb, ++i) {
                    const int s = i % P_STAGES;
                    if (!(ok = tc::mbar_wait(&empty[s], ((i / P_STAGES) & 1) ^ 1, abort))) break;
                    uint8_t *st = smem + s * SLOT;
                    tc::mbar_arrive_expect_tx(&full[s], XB + r * 128);
                    tc::tma_load_3d(st, &tm_x, &full[s], kb * KC, blk * ROWS, 0);
                    tc::tma_load_3d(st + XB, &tm_vt, &full[s], kb * KC, 0, 0);
                }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_f16(ROWS, r, true, false, false);
            int i = 0, nb = 0;
            bool ok = true;
            for (int blk = blockIdx.x; blk < p.ntb && ok; blk += gridDim.x, ++nb) {
                const int a = nb & 1;
                if (!(ok = tc::mbar_wait(&aempty[a], ((nb >> 1) & 1) ^ 1, abort))) break;
                tc::tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, ++i) {
                    const int s = i % P_STAGES;
                    if (!(ok = tc::mbar_wait(&full[s], (i / P_STAGES) & 1, abort))) break;
                    tc::tc_fence_after();
                    uint8_t *st = smem + s * SLOT;
#pragma unroll
                    for (int kk = 0; kk < KC / 16; ++kk) {
                        const uint64_t ad = tc::smem_desc(st + kk * 32, 16, 1024, tc::SW_128B);
                        const uint64_t bd = tc::smem_desc(st + XB + kk * 32, 16, 1024, tc::SW_128B);
                        tc::mma_f16(tmem + 32 * a, ad, bd, idesc, (kb | kk) != 0);
                    }
                    tc::mma_commit(&empty[s]);
                }
                if (ok) tc::mma_commit(&afull[a]);
            }
        }
    } else {
        // warps 2..5: TMEM lane quarter = warp % 4
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int nb = 0;
        for (int blk = blockIdx.x; blk < p.ntb; blk += gridDim.x, ++nb) {
            const int a = nb & 1;
            if (!tc::mbar_wait(&afull[a], (nb >> 1) & 1, abort)) break;
            tc::tc_fence_after();
            uint32_t v[32];
            tc::tmem_ld32(tmem + 32 * a + ((uint32_t)(q * 32) << 16), v);
            tc::tmem_ld_wait();
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&aempty[a]);
            const int64_t t = (int64_t)blk * ROWS + row;
            if (t < p.T) {
                float4 *dst = reinterpret_cast<float4 *>(p.lr + t * r);
#pragma unroll
                for (int e = 0; e < RK / 4; ++e)
                    if (4 * e < r && ACT_DCHECK(4 * e + 4 <= r)) dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                                        __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 64);
    }
}

// ======================================================================== quantisation
constexpr int NG = 3;                 // epilogue groups = TMEM accumulators
constexpr int Q_THREADS = (3 + 4 * NG) * 32;
constexpr int Q_STAGES = 4;           // tiles in flight (X tile + basis tile each)

struct QuantParams {
    int64_t T, H;
    int rank, k, group;
    int ntb, ncc;
    int64_t ntiles;
    int tq, trem;                     // tiles per CTA: tq, one more for the first trem CTAs
    const float *lr;
    float *scales;
    uint16_t *outl;
    const int32_t *idx;
    const uint16_t *vtile;
    uint8_t *codes;
};

template <int PITCH>
__device__ __forceinline__ int swz(int r, int c) {
    if constexpr (PITCH == 128) return r * 128 + ((c ^ (r & 7)) << 4);
    else if constexpr (PITCH == 64) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    else return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
}
template <int PITCH>
__host__ __device__ constexpr tc::Swizzle swz_mode() {
    return PITCH == 128 ? tc::SW_128B : (PITCH == 64 ? tc::SW_64B : tc::SW_32B);
}
template <int PITCH>
constexpr CUtensorMapSwizzle tma_swz() {
    return PITCH == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                        : (PITCH == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// Packs 8 int4 codes (4 pairs) or 4 int8 codes (2 pairs) into one word, channel
// order low to high.  Each input is fma(w, rs, 1.5 * 2^23 + 2^(b-1)): the
// nearest integer of the exact w * rs plus the code offset sits in the low
// mantissa bits with zeros up to bit 21 (|w * rs| <= qmax (1 + 2^-24)).
template <int BITS>
__device__ __forceinline__ uint32_t pack_codes(float2 t0, float2 t1, float2 t2, float2 t3) {
    const uint32_t a0 = __float_as_uint(t0.x), a1 = __float_as_uint(t0.y), a2 = __float_as_uint(t1.x),
                   a3 = __float_as_uint(t1.y);
    if constexpr (BITS == 4) {
        const uint32_t a4 = __float_as_uint(t2.x), a5 = __float_as_uint(t2.y), a6 = __float_as_uint(t3.x),
                       a7 = __float_as_uint(t3.y);
        const uint32_t b0 = a1 * 16u + a0, b1 = a3 * 16u + a2, b2 = a5 * 16u + a4, b3 = a7 * 16u + a6;
        return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    } else {
        return __byte_perm(__byte_perm(a0, a1, 0x0040), __byte_perm(a2, a3, 0x0040), 0x5410);
    }
}

// Tile v of the walk: token block v / ncc, channel tile v % ncc (first channels first).
struct Walk {
    int tb, cc, ncc;
    __device__ Walk(int64_t v, int64_t ntiles, int ncc_) : ncc(ncc_) {
        (void)ntiles;
        tb = (int)(v / ncc);
        cc = (int)(v - (int64_t)tb * ncc);
    }
    __device__ __forceinline__ void next() {
        if (++cc == ncc) {
            cc = 0;
            ++tb;
        }
    }
};

template <int BITS, int RK>
struct QLayout {
    static constexpr int LB = 2 * RK;
    static constexpr int XT = ROWS * CH * 2;         // X tile: two 64-channel boxes of 128 rows (SW128)
    static constexpr int VT = CH * LB;               // basis tile of 128 channels
    static constexpr int STAGE = XT + VT;
    static constexpr int PT = 3 * ROWS * LB;         // piece tiles of a token block
    static constexpr int CROW = CH * BITS / 8;       // code bytes of one token row of a tile
    static constexpr int OFF_ST = 0;
    static constexpr int OFF_PT = OFF_ST + Q_STAGES * STAGE;
    static constexpr int OFF_STG = OFF_PT + 2 * PT;
    static constexpr int OFF_OT = OFF_STG;  // outlier table: per 32 channels (mask, below)
    __host__ __device__ static int bar_off(int n32) { return (OFF_OT + n32 * 8 + 1023) & ~1023; }
    __host__ __device__ static int total(int n32) { return bar_off(n32) + 1024 + 1024; }
};

template <int BITS, int RK>
__global__ void __launch_bounds__(Q_THREADS, 1)
    cg_quant_kernel(const __grid_constant__ CUtensorMap tm_x, QuantParams p) {
    using L = QLayout<BITS, RK>;
    constexpr int LB = L::LB;
    constexpr int qmax = (1 << (BITS - 1)) - 1, off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int n32 = (int)(p.H / 32);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::bar_off(n32));
    uint64_t *empty = full + Q_STAGES;
    uint64_t *tfull = empty + Q_STAGES;   // [NG]
    uint64_t *tempty = tfull + NG;        // [NG]
    uint64_t *pready = tempty + NG;       // [2] piece tiles of a token block written
    uint64_t *pfree = pready + 2;         // [2] ... and read by the MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pfree + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint32_t *otab = reinterpret_cast<uint32_t *>(smem + L::OFF_OT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = p.rank;
    const int64_t v_lo = (int64_t)blockIdx.x * p.tq + (blockIdx.x < p.trem ? blockIdx.x : p.trem);
    const int64_t v_hi = v_lo + p.tq + (blockIdx.x < p.trem ? 1 : 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < Q_STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1 + 4);  // the MMA (basis tile) and the tile's four epilogue warps (X)
        }
        for (int g = 0; g < NG; ++g) {
            tc::mbar_init(&tfull[g], 1);
            tc::mbar_init(&tempty[g], 4);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&pready[i], 1);
            tc::mbar_init(&pfree[i], 1);
        }
        *abort = 0;
        tc::fence_mbar_init();
    }
    // outlier table: per 32-channel group of H, the mask of its outlier channels
    // and the number of outlier channels below it (indices ascending)
    for (int e = threadIdx.x; e < n32; e += Q_THREADS) {
        const int64_t lo = 32 * (int64_t)e;
        uint32_t m = 0;
        int below = 0;
        for (int j = 0; j < p.k; ++j) {
            const int64_t c = __ldg(p.idx + j);
            below += c < lo;
            if (c >= lo && c < lo + 32) m |= 1u << (c - lo);
        }
        otab[2 * e] = m;
        otab[2 * e + 1] = (uint32_t)below;
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ X tiles and basis tiles
        if (lane == 0) {
            tc::prefetch_tmap(&tm_x);
            const uint64_t pol = tc::l2_policy_evict_first();
            int i = 0;
            Walk w(v_lo, p.ntiles, p.ncc);
            for (int64_t v = v_lo; v < v_hi; ++v, ++i, w.next()) {
                const int s = i % Q_STAGES;
                if (!tc::mbar_wait(&empty[s], ((i / Q_STAGES) & 1) ^ 1, abort)) break;
                uint8_t *st = smem + L::OFF_ST + s * L::STAGE;
                tc::mbar_arrive_expect_tx(&full[s], L::STAGE);
                tc::tma_load_3d_hint(st, &tm_x, &full[s], w.cc * CH, w.tb * ROWS, 0, pol);
                tc::tma_load_3d_hint(st + L::XT / 2, &tm_x, &full[s], w.cc * CH + 64, w.tb * ROWS, 0, pol);
                tc::bulk_load(st + L::XT, p.vtile + (int64_t)w.cc * (L::VT / 2), L::VT, &full[s]);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ L -> piece tiles, per token block
        Walk w(v_lo, p.ntiles, p.ncc);
        int m = 0;
        bool ok = true;
        for (int64_t v = v_lo; v < v_hi && ok; ++v, w.next()) {
            if (v != v_lo && w.cc != 0) continue;  // not the first tile of a token block
            if (m == 0) {  // the range's first block: built by the epilogue warps
                ++m;
                continue;
            }
            const int slot = m & 1;
            if (!(ok = tc::mbar_wait(&pfree[slot], ((m >> 1) & 1) ^ 1, abort))) break;
            uint8_t *dst = smem + L::OFF_PT + slot * L::PT;
            const int64_t t0 = (int64_t)w.tb * ROWS;
            build_piece_tiles<ROWS, LB>(p.lr, t0, p.T - t0, r, dst, lane);
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&pready[slot]);
            ++m;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ low-rank MMA
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(ROWS, CH, true, false, false);
            constexpr tc::Swizzle SW = swz_mode<LB>();
            const int nkq = r / 16;
            int i = 0, m = -1;
            bool ok = true;
            Walk w(v_lo, p.ntiles, p.ncc);
            for (int64_t v = v_lo; v < v_hi && ok; ++v, ++i, w.next()) {
                const int s = i % Q_STAGES, acc = i % NG;
                if (v == v_lo || w.cc == 0) {  // a new token block: its piece tiles
                    ++m;
                    if (!(ok = tc::mbar_wait(&pready[m & 1], (m >> 1) & 1, abort))) break;
                }
                if (!(ok = tc::mbar_wait(&full[s], (i / Q_STAGES) & 1, abort))) break;
                if (!(ok = tc::mbar_wait(&tempty[acc], ((i / NG) & 1) ^ 1, abort))) break;
                tc::tc_fence_after();
                const uint8_t *a = smem + L::OFF_PT + (m & 1) * L::PT;
                const uint8_t *b = smem + L::OFF_ST + s * L::STAGE + L::XT;
                for (int pc = 0; pc < 3; ++pc)
                    for (int kk = 0; kk < nkq; ++kk) {
                        const uint64_t ad = tc::smem_desc(a + pc * ROWS * LB + kk * 32, 16, 8 * LB, SW);
                        const uint64_t bd = tc::smem_desc(b + kk * 32, 16, 8 * LB, SW);
                        tc::mma_f16(tmem + acc * CH, ad, bd, idesc, (pc | kk) != 0);
                    }
                tc::mma_commit(&tfull[acc]);
                tc::mma_commit(&empty[s]);
                // the last tile of this token block in the range: the piece slot frees with these MMAs
                if (w.cc == p.ncc - 1 || v == v_hi - 1) tc::mma_commit(&pfree[m & 1]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 3;           // 0 .. 4 NG - 1
        const int g = ew >> 2;             // group: tiles g, g + NG, ... of the range
        const int q = warp & 3;            // TMEM lane quarter = row quarter
        const int row = q * 32 + lane;
        const int G = p.group;
        const int gshift = 31 - __clz(G);
        const int ngr = (int)(p.H / G);
        const int64_t crow = p.H * BITS / 8;  // code bytes per token row
        // the piece tiles of the range's first token block, by all epilogue
        // warps (idle until its P exists): one memory round trip instead of the
        // builder warp's several
        if (v_lo < v_hi) {
            const int64_t t0 = (v_lo / p.ncc) * ROWS;
            build_piece_tiles_team<ROWS, LB, 32 * 4 * NG>(p.lr, t0, p.T - t0, r, smem + L::OFF_PT,
                                                          (int)threadIdx.x - 96);
            tc::fence_proxy_async();
            tc::named_bar(1, 32 * 4 * NG);
            if (threadIdx.x == 96) tc::mbar_arrive(&pready[0]);
        }
        int j = 0;
        bool ok = true;
        Walk w(v_lo, p.ntiles, p.ncc);
        for (int e = 0; e < g; ++e) w.next();
        for (int64_t v = v_lo + g; v < v_hi && ok; v += NG, ++j) {
            const int tb = w.tb, cc = w.cc;
            for (int e = 0; e < NG; ++e) w.next();
            const int64_t t = (int64_t)tb * ROWS + row;
            const bool rv = t < p.T;
            const int64_t c0 = (int64_t)cc * CH;
            const int i = (int)(v - v_lo), s = i % Q_STAGES;
            // every thread observes both: the X tile's TMA writes, and P complete
            if (!(ok = tc::mbar_wait(&full[s], (i / Q_STAGES) & 1, abort) && tc::mbar_wait(&tfull[g], j & 1, abort)))
                break;
            tc::tc_fence_after();
            const uint32_t acc = tmem + g * CH + ((uint32_t)(q * 32) << 16);
            const uint8_t *xt = smem + L::OFF_ST + s * L::STAGE;
            const uint32_t *ot = otab + 2 * (c0 >> 5);
            uint8_t *cdst = p.codes + t * crow + c0 * BITS / 8;  // this row's codes of the tile
            // this warp's code staging (two buffers) is free once the store issued
            // two tiles ago has read it
            __syncwarp();
            float scv[4];
            // groups of G channels: G / 32 pieces of 32 held as residuals in registers
#pragma unroll 1
            for (int gi = 0; gi < CH / 64; ++gi) {  // two 64-channel halves
                float2 w2[2][16];
                float am[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int pc = 2 * gi + h;
                    uint32_t P[32];
                    tc::tmem_ld32(acc + 32 * pc, P);
                    uint4 xv[4];
                    const uint8_t *box = xt + (pc >> 1) * (L::XT / 2);  // 64-channel half of the tile
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16)
                        xv[c16] = *reinterpret_cast<const uint4 *>(box + swz<128>(row, (pc & 1) * 4 + c16));
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16) {
                        const uint32_t wd[4] = {xv[c16].x, xv[c16].y, xv[c16].z, xv[c16].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            w2[h][4 * c16 + e] =
                                sub2(make_float2(__uint_as_float(wd[e] << 16), __uint_as_float(wd[e] & 0xffff0000u)),
                                     make_float2(__uint_as_float(P[8 * c16 + 2 * e]), __uint_as_float(P[8 * c16 + 2 * e + 1])));
                    }
                    const uint32_t om = ot[2 * pc];
                    if (om) {  // warp-uniform: verbatim values out, residual zeroed
                        const int below = (int)ot[2 * pc + 1];
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            if ((om >> e) & 1u) {
                                const int slot = below + __popc(om & ((1u << e) - 1u));
                                const int c16 = e >> 3, wi = (e & 7) >> 1;
                                const uint32_t word =
                                    wi == 0 ? xv[c16].x : (wi == 1 ? xv[c16].y : (wi == 2 ? xv[c16].z : xv[c16].w));
                                const uint16_t xb = (uint16_t)(e & 1 ? (word >> 16) : (word & 0xffffu));
                                if (rv && ACT_DCHECK(slot < p.k)) p.outl[t * p.k + slot] = xb;
                                if (e & 1) w2[h][e >> 1].y = 0.f;
                                else w2[h][e >> 1].x = 0.f;
                            }
                        }
                    }
                    float a = 0.f;
#pragma unroll
                    for (int e = 0; e < 16; ++e) a = fmaxf(a, fmaxf(fabsf(w2[h][e].x), fabsf(w2[h][e].y)));
                    am[h] = a;
                }
                // scales: one correctly rounded division each, as the oracle
                float sc[2], rs[2];
                if (G == 32) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        sc[h] = __fdiv_rn(am[h], (float)qmax);
                        rs[h] = am[h] > 0.f ? __fdiv_rn((float)qmax, am[h]) : 0.f;
                    }
                } else {
                    const float a = fmaxf(am[0], am[1]);
                    sc[0] = sc[1] = __fdiv_rn(a, (float)qmax);
                    rs[0] = rs[1] = a > 0.f ? __fdiv_rn((float)qmax, a) : 0.f;
                }
                scv[2 * gi] = sc[0];
                scv[2 * gi + 1] = sc[1];
                constexpr float MAGIC = 12582912.0f + (float)off;
                const float2 magic2 = make_float2(MAGIC, MAGIC);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int pc = 2 * gi + h;
                    const float2 rs2 = make_float2(rs[h], rs[h]);
                    if constexpr (BITS == 4) {
                        uint32_t pk[4];
#pragma unroll
                        for (int wd = 0; wd < 4; ++wd)
                            pk[wd] = pack_codes<4>(fma2(w2[h][4 * wd], rs2, magic2), fma2(w2[h][4 * wd + 1], rs2, magic2),
                                                   fma2(w2[h][4 * wd + 2], rs2, magic2),
                                                   fma2(w2[h][4 * wd + 3], rs2, magic2));
                        if (rv) *reinterpret_cast<uint4 *>(cdst + 16 * pc) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    } else {
                        const float2 z = make_float2(0.f, 0.f);
                        uint32_t pk[8];
#pragma unroll
                        for (int wd = 0; wd < 8; ++wd)
                            pk[wd] = pack_codes<8>(fma2(w2[h][2 * wd], rs2, magic2), fma2(w2[h][2 * wd + 1], rs2, magic2),
                                                   z, z);
                        if (rv) {
                            *reinterpret_cast<uint4 *>(cdst + 32 * pc) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            *reinterpret_cast<uint4 *>(cdst + 32 * pc + 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                        }
                    }
                }
            }
            // P and the X tile have been read
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&tempty[g]);
                tc::mbar_arrive(&empty[s]);
            }
            if (rv && ACT_DCHECK((c0 >> gshift) + (G == 32 ? 4 : 2) <= ngr)) {
                float *sp = p.scales + t * ngr + (c0 >> gshift);
                if (G == 32) *reinterpret_cast<float4 *>(sp) = make_float4(scv[0], scv[1], scv[2], scv[3]);
                else *reinterpret_cast<float2 *>(sp) = make_float2(scv[0], scv[2]);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

template <int RK>
int launch_proj(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t stream) {
    const int64_t T = d->tokens, H = d->channels;
    const int r = d->rank;
    CUtensorMap m_x{}, m_vt{};
    int st;
    if ((st = make_map_3d(&m_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, T, 1, ldx, T * ldx, KC, ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_map_3d(&m_vt, d->basis_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, r, 1, H, (int64_t)r * H, KC, r,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    ProjParams p{};
    p.T = T;
    p.H = H;
    p.rank = r;
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.lr = d->lowrank;
    const int smem = P_STAGES * (ROWS * 128 + RK * 128) + 1024 + 1024;
    auto kern = cg_proj_kernel<RK>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int grid = p.ntb < num_sms() ? p.ntb : num_sms();
    kern<<<grid, P_THREADS, smem, stream>>>(m_x, m_vt, p);
    return launch_status();
}

template <int BITS, int RK>
int launch_quant(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t stream) {
    using L = QLayout<BITS, RK>;
    const int64_t T = d->tokens, H = d->channels;
    CUtensorMap m_x{};
    int st;
    if ((st = make_map_3d(&m_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, T, 1, ldx, T * ldx, 64, ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    QuantParams p{};
    p.T = T;
    p.H = H;
    p.rank = d->rank;
    p.k = d->n_outlier;
    p.group = d->group;
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.ncc = (int)(H / CH);
    p.ntiles = (int64_t)p.ntb * p.ncc;
    p.lr = d->lowrank;
    p.scales = d->scales;
    p.outl = d->outliers;
    p.idx = d->outlier_idx;
    p.vtile = d->basis_tile;
    p.codes = d->codes;
    const int smem = L::total((int)(H / 32));
    if (smem > 227 * 1024) return ACT_E_UNSUPPORTED;
    auto kern = cg_quant_kernel<BITS, RK>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int grid = (int)(p.ntiles < num_sms() ? p.ntiles : num_sms());
    p.tq = (int)(p.ntiles / grid);
    p.trem = (int)(p.ntiles % grid);
    kern<<<grid, Q_THREADS, smem, stream>>>(m_x, p);
    return launch_status();
}

}  // namespace cgsplit
}  // namespace act

// Two-kernel encode (projection, then quantisation), or ACT_E_UNSUPPORTED
// (before launching) for formats it does not cover: batch > 1, the rotation,
// groups of 128, a rank other than 16 or 32, H not a multiple of 128, no
// basis tile, unaligned buffers.
int act_cg_encode_split(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s) {
    using namespace act::cgsplit;
    if (d->tokens == 0) return ACT_OK;
    if (d->batch != 1 || d->wht || d->group > 64 || !(d->rank == 16 || d->rank == 32) || !d->basis_tile)
        return ACT_E_UNSUPPORTED;
    if (d->channels % CH || ldx % 8 || !act::aligned(x, 16)) return ACT_E_UNSUPPORTED;
    if (!act::aligned(d->scales, 16) || !act::aligned(d->codes, 16) || !act::aligned(d->lowrank, 16) ||
        !act::aligned(d->basis_tile, 16))
        return ACT_E_UNSUPPORTED;
    // the quantisation's shared memory must fit before anything is launched
    const int n32 = (int)(d->channels / 32);
    const int qsmem = d->bits == 4 ? (d->rank == 16 ? QLayout<4, 16>::total(n32) : QLayout<4, 32>::total(n32))
                                   : (d->rank == 16 ? QLayout<8, 16>::total(n32) : QLayout<8, 32>::total(n32));
    if (qsmem > 227 * 1024) return ACT_E_UNSUPPORTED;
    int st = d->rank == 16 ? launch_proj<16>(d, x, ldx, s) : launch_proj<32>(d, x, ldx, s);
    if (st) return st;
    if (d->bits == 4) return d->rank == 16 ? launch_quant<4, 16>(d, x, ldx, s) : launch_quant<4, 32>(d, x, ldx, s);
    return d->rank == 16 ? launch_quant<8, 16>(d, x, ldx, s) : launch_quant<8, 32>(d, x, ldx, s);
}
