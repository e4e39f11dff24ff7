// cg_encode_rows.cu -- channel-group encode with whole chunk rows per thread
// (the encode for 1024..16384 channels, with or without the rotation).
//
// One CTA per block of 128 tokens at a time (grid-stride over blocks).  Roles:
//   warp 0      phase-1 producer: TMA streams X[128 x 64] and V^T[r x 64]
//               steps into a projection ring;
//   warp 1      projection MMA: tcgen05.mma kind::f16 (M=128, N=r) accumulates
//               L = X . V in TMEM;
//   warp 2      phase-2 producer: per 128-channel chunk (backward over the
//               channels, so that it starts on the columns the projection left
//               in L2) TMA re-reads X[128 x 128] and bulk-copies the chunk's
//               prepared bf16 basis tile;
//   warp 3      low-rank MMA: P = L . V^T (kind::f16, L as its three exact bf16
//               pieces against the bf16 basis, fp32 accumulation) into one of
//               three TMEM accumulators;
//   warps 4-15  epilogue: three groups of four warps; group g takes chunks
//               g, g+3, g+6, ... (counted over all blocks of the CTA); a thread
//               owns one token row of a chunk and all its 128 channels.  Pass 1,
//               per 32-channel piece: residual x - P, outlier channels
//               copied out and zeroed, piece absmax, residual written back over
//               P in TMEM.  With the rotation, pass 1 also applies the butterfly
//               stages 1..16 inside each piece, and stages 32 and 64 then combine
//               the four pieces eight TMEM columns at a time (oracle stage order).
//               Pass 2: group scales (one correctly rounded division
//               each, as the oracle), residual read back, codes packed and staged;
//               each warp stores its 32 rows of codes with one TMA store and
//               writes its rows' scales directly.
//   Group 0 also stores the projection L (float32) and writes its three bf16
//   pieces as the low-rank MMA's operand tiles (double-buffered).
// No two epilogue warps exchange data inside a chunk: no named barriers on the
// chunk path.  Arithmetic is that of oracle/actcomp_oracle.c
// (cg_encode_given_lr) given the projection, except that the tensor cores sum
// the low-rank term in their own order (a few float32 ulps).
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgencr {

constexpr int ROWS = 128, KC = 64, CH = 128;
constexpr int NGR = 3;            // epilogue groups = residual accumulators
constexpr int EW = 4 * NGR;       // epilogue warps
constexpr int THREADS = 128 + 32 * EW;
constexpr int MAXNA = 6, MAXNB = 4;

struct Params {
    int64_t T, H;
    int rank, k, group, batch;
    float *scales;
    float *lr;
    uint16_t *outl;
    const int32_t *idx;
    const uint16_t *vtile;
    int nk2;          // 128-channel chunks per block
    int ntb;          // token blocks per slice
    int64_t nblocks;
    int ngrid;        // CTAs (grid stride over blocks)
    int na, nb;       // ring stages
    int ngs;          // 64-channel groups of H (outlier table entries)
    int ostage;       // outlier values staged per block (else written directly)
    int off_ringB, off_lqt, off_bar, off_stg, off_ot, off_ost, off_sv;
};

template <int BITS, int RK>
struct Layout {
    static constexpr int LB = 2 * RK;
    static constexpr int SLOT_A = 16 * 1024 + RK * 128;
    static constexpr int SLOT_B = 32 * 1024 + CH * LB;
    static constexpr int LQT = 3 * ROWS * LB;  // the three bf16 pieces of L, one tile each
    static constexpr int CROW = CH * BITS / 8;  // code bytes of one token row of a chunk
    static constexpr int WSTG = 32 * CROW;      // one warp's code staging (32 rows)
    // alias: every CTA encodes one block, so the residual ring may reuse the
    // projection ring's memory (phase-2 loads start after the projection MMAs
    // have completed)
    static int plan(Params &p, int na, int nb, bool alias, int k, int ostage) {
        p.na = na;
        p.nb = nb;
        p.ostage = ostage;
        p.off_ringB = alias ? 0 : na * SLOT_A;
        const int ring = alias ? (na * SLOT_A > nb * SLOT_B ? na * SLOT_A : nb * SLOT_B) : na * SLOT_A + nb * SLOT_B;
        p.off_lqt = ring;
        p.off_bar = p.off_lqt + 2 * LQT;
        p.off_stg = p.off_bar + 1024;
        p.off_ot = p.off_stg + EW * WSTG;
        p.off_ost = p.off_ot + ((p.ngs * 12 + 15) & ~15);
        p.off_sv = p.off_ost + (ostage ? ((ROWS * k * 2 + 15) & ~15) : 0);
        return p.off_sv + 1024;
    }
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

// Packs 8 int4 codes (4 pairs) or 4 int8 codes (2 pairs) into one word,
// channel order low to high.  Each input is fma(w, rs, 1.5 * 2^23 + 2^(b-1)):
// the nearest integer of the exact w * rs plus the code offset sits in the
// low mantissa bits with zeros up to bit 21 (|w * rs| <= qmax (1 + 2^-24)).
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

template <int BITS, int RK, bool WHT>
__global__ void __launch_bounds__(THREADS, 1)
    cg_encode_rows_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_vt,
                          const __grid_constant__ CUtensorMap tm_c, Params p) {
    using L = Layout<BITS, RK>;
    constexpr int LB = L::LB;
    constexpr int CROW = L::CROW;
    constexpr int qmax = (1 << (BITS - 1)) - 1, off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NA = p.na, NB = p.nb;
    uint8_t *ringA = smem, *ringB = smem + p.off_ringB;
    uint8_t *lqt = smem + p.off_lqt;  // [2] x 3 bf16 piece tiles of L
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *emptyA = fullA + MAXNA;
    uint64_t *fullB = emptyA + MAXNA;
    uint64_t *emptyB = fullB + MAXNB;
    uint64_t *tfull = emptyB + MAXNB;  // [NGR]
    uint64_t *tempty = tfull + NGR;    // [NGR]
    uint64_t *lqready = tempty + NGR;  // [2] the piece tiles of a block written (by group 0)
    uint64_t *lqfree = lqready + 2;    // [2] the low-rank MMAs of a block have read its piece tiles
    uint64_t *lfull = lqfree + 2;      // projection accumulator complete
    uint64_t *lempty = lfull + 1;      // ... and read
    uint64_t *lseen = lempty + 1;      // the phase-2 producer has observed lfull of the block
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(lseen + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = p.rank;
    const int nk1 = (int)(p.H / KC), nk2 = p.nk2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NA; ++s) {
            tc::mbar_init(&fullA[s], 1);
            tc::mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < NB; ++s) {
            tc::mbar_init(&fullB[s], 1);
            tc::mbar_init(&emptyB[s], 1 + 4);  // the MMA (basis tile) and the chunk's four epilogue warps (X)
        }
        for (int g = 0; g < NGR; ++g) {
            tc::mbar_init(&tfull[g], 1);
            tc::mbar_init(&tempty[g], 4);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&lqready[i], 4);
            tc::mbar_init(&lqfree[i], 1);
        }
        tc::mbar_init(lfull, 1);
        tc::mbar_init(lempty, 4);
        tc::mbar_init(lseen, 1);
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, 512);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tm_l = tmem;        // projection accumulator, columns [0, 64)
    const uint32_t tm_p = tmem + 128;  // residual accumulators, [128, 512)

    if (warp == 0) {
        // ------------------------------------------------------------ phase-1 producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_x);
            tc::prefetch_tmap(&tm_vt);
            int i = 0;
            bool ok = true;
            for (int64_t blk = blockIdx.x; blk < p.nblocks && ok; blk += p.ngrid) {
                const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
                for (int ks = 0; ks < nk1; ++ks, ++i) {
                    const int s = i % NA;
                    if (!(ok = tc::mbar_wait(&emptyA[s], ((i / NA) & 1) ^ 1, abort))) break;
                    uint8_t *st = ringA + s * L::SLOT_A;
                    tc::mbar_arrive_expect_tx(&fullA[s], ROWS * 128 + r * 128);
                    tc::tma_load_3d(st, &tm_x, &fullA[s], ks * KC, tb * ROWS, b);
                    tc::tma_load_3d(st + 16 * 1024, &tm_vt, &fullA[s], ks * KC, 0, b);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ projection MMA
        if (lane == 0) {
            const uint32_t id_proj = tc::idesc_f16(ROWS, r, true, false, false);
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = blockIdx.x; blk < p.nblocks && ok; blk += p.ngrid, ++nb) {
                if (!(ok = tc::mbar_wait(lempty, (nb & 1) ^ 1, abort))) break;
                tc::tc_fence_after();
                for (int ks = 0; ks < nk1; ++ks, ++i) {
                    const int s = i % NA;
                    if (!(ok = tc::mbar_wait(&fullA[s], (i / NA) & 1, abort))) break;
                    tc::tc_fence_after();
                    uint8_t *st = ringA + s * L::SLOT_A;
#pragma unroll
                    for (int kk = 0; kk < KC / 16; ++kk) {
                        const uint64_t ad = tc::smem_desc(st + kk * 32, 16, 1024, tc::SW_128B);
                        const uint64_t bd = tc::smem_desc(st + 16 * 1024 + kk * 32, 16, 1024, tc::SW_128B);
                        tc::mma_f16(tm_l, ad, bd, id_proj, (ks | kk) != 0);
                    }
                    tc::mma_commit(&emptyA[s]);
                }
                // lfull must not run two phases ahead of the phase-2 producer's parity wait
                if (ok && nb > 0) ok = tc::mbar_wait(lseen, (nb - 1) & 1, abort);
                if (ok) tc::mma_commit(lfull);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ phase-2 producer
        if (lane == 0) {
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = blockIdx.x; blk < p.nblocks && ok; blk += p.ngrid, ++nb) {
                const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
                // re-read X only after phase 1 of this block has streamed it into L2
                if (!(ok = tc::mbar_wait(lfull, nb & 1, abort))) break;
                tc::mbar_arrive(lseen);
                for (int ck = 0; ck < nk2; ++ck, ++i) {
                    const int s = i % NB;
                    if (!(ok = tc::mbar_wait(&emptyB[s], ((i / NB) & 1) ^ 1, abort))) break;
                    uint8_t *st = ringB + s * L::SLOT_B;
                    tc::mbar_arrive_expect_tx(&fullB[s], 2 * ROWS * 128 + CH * LB);
                    const int x = (nk2 - 1 - ck) * CH;  // backward sweep
                    tc::tma_load_3d(st, &tm_x, &fullB[s], x, tb * ROWS, b);
                    tc::tma_load_3d(st + ROWS * 128, &tm_x, &fullB[s], x + 64, tb * ROWS, b);
                    tc::bulk_load(st + 32 * 1024, p.vtile + ((int64_t)b * nk2 + x / CH) * (CH * LB / 2), CH * LB,
                                  &fullB[s]);
                }
            }
        }
    } else if (warp == 3) {
        // ------------------------------------------------------------ low-rank MMA
        if (lane == 0) {
            constexpr uint32_t id_q = tc::idesc_f16(ROWS, CH, true, false, false);
            constexpr tc::Swizzle SWQ = swz_mode<LB>();
            const int nkq = (r + 15) / 16;
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = blockIdx.x; blk < p.nblocks && ok; blk += p.ngrid, ++nb) {
                const int ls = nb & 1;
                if (!(ok = tc::mbar_wait(&lqready[ls], (nb >> 1) & 1, abort))) break;
                tc::tc_fence_after();
                const uint8_t *a = lqt + ls * L::LQT;
                for (int ck = 0; ck < nk2; ++ck, ++i) {
                    const int s = i % NB, acc = i % NGR;
                    if (!(ok = tc::mbar_wait(&fullB[s], (i / NB) & 1, abort))) break;
                    if (!(ok = tc::mbar_wait(&tempty[acc], ((i / NGR) & 1) ^ 1, abort))) break;
                    tc::tc_fence_after();
                    uint8_t *st = ringB + s * L::SLOT_B;
                    // P = hi . V^T + mid . V^T + lo . V^T
                    for (int pc = 0; pc < 3; ++pc)
                        for (int kk = 0; kk < nkq; ++kk) {
                            const uint64_t ad = tc::smem_desc(a + pc * ROWS * LB + kk * 32, 16, 8 * LB, SWQ);
                            const uint64_t bd = tc::smem_desc(st + 32 * 1024 + kk * 32, 16, 8 * LB, SWQ);
                            tc::mma_f16(tm_p + acc * CH, ad, bd, id_q, (pc | kk) > 0);
                        }
                    tc::mma_commit(&tfull[acc]);
                    tc::mma_commit(&emptyB[s]);
                }
                if (ok) tc::mma_commit(&lqfree[ls]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 4;
        const int g = ew >> 2;
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int etid = threadIdx.x - 128;
        constexpr int ETH = 32 * EW;
        const int G = p.group;
        const int gshift = 31 - __clz(G);
        const int ppg = G >> 5;  // 32-channel pieces per group
        const int ngr = (int)(p.H / G);
        uint64_t *omask = reinterpret_cast<uint64_t *>(smem + p.off_ot);  // outlier table
        int32_t *obelow = reinterpret_cast<int32_t *>(omask + p.ngs);
        uint16_t *ost = reinterpret_cast<uint16_t *>(smem + p.off_ost);
        uint8_t *cb = smem + p.off_stg + ew * L::WSTG;
        int cur_slice = -1;
        int j = 0, nb = 0;  // chunks of this CTA so far (all blocks), blocks so far
        // After a failed wait (abort set) the warps keep walking the blocks so
        // that every epilogue warp reaches every named barrier; all later waits
        // return at once and the work is skipped.
        bool ok = true;
        for (int64_t blk = blockIdx.x; blk < p.nblocks; blk += p.ngrid, ++nb) {
            const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
            const int64_t t = (int64_t)tb * ROWS + row;
            const bool rv = t < p.T;
            const int64_t trow = (int64_t)b * p.T + t;
            const int nrows = (int)((p.T - (int64_t)tb * ROWS) < ROWS ? (p.T - (int64_t)tb * ROWS) : ROWS);
            const int ls = nb & 1;
            if (g == 0 && ok) do {
                // ---- projection -> L (float32, stored) and its three bf16 pieces
                // (group 0: one token row per thread)
                if (!(ok = tc::mbar_wait(lfull, nb & 1, abort))) break;
                // the piece tiles' slot is free once the low-rank MMAs of block nb - 2 completed
                if (nb >= 2 && !(ok = tc::mbar_wait(&lqfree[ls], ((nb >> 1) & 1) ^ 1, abort))) break;
                tc::tc_fence_after();
                uint8_t *lq = lqt + ls * L::LQT;
                // 32 coefficients at a time: L to global memory, pieces to the tiles
#pragma unroll
                for (int jj = 0; jj < (RK + 31) / 32; ++jj) {
                    constexpr int NC = RK < 32 ? RK : 32;
                    uint32_t v[32];
                    tc::tmem_ld32(tm_l + ((uint32_t)(q * 32) << 16) + 32 * jj, v);
                    tc::tmem_ld_wait();
                    float Lr[NC];
#pragma unroll
                    for (int e = 0; e < NC; ++e) Lr[e] = 32 * jj + e < r ? __uint_as_float(v[e]) : 0.f;
                    if (rv) {
                        float4 *dst = reinterpret_cast<float4 *>(p.lr + trow * r + 32 * jj);
#pragma unroll
                        for (int e = 0; e < NC / 4; ++e)
                            if (32 * jj + 4 * e < r)
                                dst[e] = make_float4(Lr[4 * e], Lr[4 * e + 1], Lr[4 * e + 2], Lr[4 * e + 3]);
                    }
#pragma unroll
                    for (int c8 = 0; c8 < NC / 8; ++c8) {  // 8 coefficients = one 16-byte chunk per piece
                        uint32_t ph[4], pm[4], pl[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float h0, m0, l0, h1, m1, l1;
                            split3_bf16(Lr[8 * c8 + 2 * e], h0, m0, l0);
                            split3_bf16(Lr[8 * c8 + 2 * e + 1], h1, m1, l1);
                            ph[e] = pack_bf16x2(h0, h1);
                            pm[e] = pack_bf16x2(m0, m1);
                            pl[e] = pack_bf16x2(l0, l1);
                        }
                        const int o = swz<LB>(row, 4 * jj + c8);
                        *reinterpret_cast<uint4 *>(lq + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
                        *reinterpret_cast<uint4 *>(lq + ROWS * LB + o) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
                        *reinterpret_cast<uint4 *>(lq + 2 * ROWS * LB + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(lempty);
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&lqready[ls]);
            } while (0);
            // ---- outlier table of slice b (indices ascending), rebuilt when the slice changes
            if (p.k && b != cur_slice) {
                tc::named_bar(2, ETH);  // the previous slice's table is no longer read
                for (int gi = etid; gi < p.ngs; gi += ETH) {
                    const int64_t lo = 64 * (int64_t)gi;
                    uint64_t m = 0;
                    int below = 0;
                    for (int jx = 0; jx < p.k; ++jx) {
                        const int64_t c = __ldg(p.idx + (int64_t)b * p.k + jx);
                        below += c < lo;
                        if (c >= lo && c < lo + 64) m |= 1ull << (c - lo);
                    }
                    omask[gi] = m;
                    obelow[gi] = below;
                }
                tc::named_bar(2, ETH);
                cur_slice = b;
            }
            // ---- residual codes: this group's chunks of the block
            for (int ck = 0; ck < nk2; ++ck, ++j) {
                if (j % NGR != g || !ok) continue;
                const int s = j % NB;
                const uint32_t acc = tm_p + (uint32_t)(g * CH) + ((uint32_t)(q * 32) << 16);
                if (!(ok = tc::mbar_wait(&fullB[s], (j / NB) & 1, abort))) continue;
                if (!(ok = tc::mbar_wait(&tfull[g], (j / NGR) & 1, abort))) continue;
                tc::tc_fence_after();
                const int cx = nk2 - 1 - ck;  // chunk index (backward sweep)
                const int64_t c0 = (int64_t)cx * CH;
                const uint8_t *xt = ringB + s * L::SLOT_B;
                float am0 = 0.f, am1 = 0.f, am2 = 0.f, am3 = 0.f;
                // ---- pass 1: residual, outliers, piece absmax; residual back into TMEM
#pragma unroll 1
                for (int k = 0; k < 4; ++k) {
                    uint32_t I[32];
                    tc::tmem_ld32(acc + 32 * k, I);
                    const uint8_t *box = xt + (k >> 1) * ROWS * 128;  // 64-channel half of the chunk
                    uint4 xv4[4];
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16)
                        xv4[c16] = *reinterpret_cast<const uint4 *>(box + swz<128>(row, (k & 1) * 4 + c16));
                    tc::tmem_ld_wait();
                    float2 w[16];
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16) {
                        const uint32_t wd[4] = {xv4[c16].x, xv4[c16].y, xv4[c16].z, xv4[c16].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 xv = make_float2(__uint_as_float(wd[e] << 16), __uint_as_float(wd[e] & 0xffff0000u));
                            const float2 iv = make_float2(__uint_as_float(I[8 * c16 + 2 * e]),
                                                          __uint_as_float(I[8 * c16 + 2 * e + 1]));
                            w[4 * c16 + e] = sub2(xv, iv);  // x - P, one rounding
                        }
                    }
                    // outlier channels of this piece (warp-uniform mask): verbatim copy, residual zeroed
                    if (p.k) {
                        const int gi = (int)((c0 + 32 * k) >> 6);
                        const uint64_t om64 = omask[gi];
                        const uint32_t om = (uint32_t)(om64 >> (32 * (k & 1)));
                        if (om) {
                            const int below = obelow[gi] + ((k & 1) ? __popc((uint32_t)om64) : 0);
#pragma unroll
                            for (int c8 = 0; c8 < 4; ++c8) {
                                const uint32_t m8 = (om >> (8 * c8)) & 0xffu;
                                if (!m8) continue;
#pragma unroll
                                for (int e8 = 0; e8 < 8; ++e8) {
                                    if ((m8 >> e8) & 1u) {
                                        const int e = 8 * c8 + e8;
                                        const int slot = below + __popc(om & ((1u << e) - 1u));
                                        const uint16_t bits = *reinterpret_cast<const uint16_t *>(
                                            box + swz<128>(row, (k & 1) * 4 + c8) + 2 * e8);
                                        if (p.ostage) ost[row * p.k + slot] = bits;
                                        else if (rv) p.outl[trow * p.k + slot] = bits;
                                        if (e & 1) w[e >> 1].y = 0.f;
                                        else w[e >> 1].x = 0.f;
                                    }
                                }
                            }
                        }
                    }
                    if constexpr (WHT) {
                        // rotation stages m = 1..16 inside the piece, (a, b) -> (a + b, a - b)
                        // in the oracle's stage order; stages 32 and 64 combine the pieces
                        // after pass 1, through TMEM
                        float(&v)[32] = *reinterpret_cast<float(*)[32]>(&w[0]);
#pragma unroll
                        for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                if (!(e & m)) {
                                    const float a = v[e], c = v[e + m];
                                    v[e] = __fadd_rn(a, c);
                                    v[e + m] = __fsub_rn(a, c);
                                }
                            }
                        }
                    } else {
                        float a[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) a[e] = fmaxf(fabsf(w[e].x), fabsf(w[e].y));
#pragma unroll
                        for (int st = 8; st > 0; st >>= 1)
#pragma unroll
                            for (int e = 0; e < st; ++e) a[e] = fmaxf(a[e], a[e + st]);
                        am0 = k == 0 ? a[0] : am0;
                        am1 = k == 1 ? a[0] : am1;
                        am2 = k == 2 ? a[0] : am2;
                        am3 = k == 3 ? a[0] : am3;
                    }
                    uint32_t wr[32];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        wr[2 * e] = __float_as_uint(w[e].x);
                        wr[2 * e + 1] = __float_as_uint(w[e].y);
                    }
                    tc::tmem_st32(acc + 32 * k, wr);
                }
                // the X tile of this chunk has been read
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&emptyB[s]);
                tc::tmem_st_wait();
                if constexpr (WHT) {
                    // rotation stages 32 (pieces 0-1, 2-3) and 64 (0-2, 1-3), eight
                    // columns of every piece at a time; piece absmax of the result
#pragma unroll 1
                    for (int jj = 0; jj < 4; ++jj) {
                        uint32_t u0[8], u1[8], u2[8], u3[8];
                        tc::tmem_ld8(acc + 8 * jj, u0);
                        tc::tmem_ld8(acc + 32 + 8 * jj, u1);
                        tc::tmem_ld8(acc + 64 + 8 * jj, u2);
                        tc::tmem_ld8(acc + 96 + 8 * jj, u3);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float a0 = __uint_as_float(u0[i]), a1 = __uint_as_float(u1[i]);
                            const float a2 = __uint_as_float(u2[i]), a3 = __uint_as_float(u3[i]);
                            const float s01 = __fadd_rn(a0, a1), d01 = __fsub_rn(a0, a1);
                            const float s23 = __fadd_rn(a2, a3), d23 = __fsub_rn(a2, a3);
                            const float o0 = __fadd_rn(s01, s23), o1 = __fadd_rn(d01, d23);
                            const float o2 = __fsub_rn(s01, s23), o3 = __fsub_rn(d01, d23);
                            am0 = fmaxf(am0, fabsf(o0));
                            am1 = fmaxf(am1, fabsf(o1));
                            am2 = fmaxf(am2, fabsf(o2));
                            am3 = fmaxf(am3, fabsf(o3));
                            u0[i] = __float_as_uint(o0);
                            u1[i] = __float_as_uint(o1);
                            u2[i] = __float_as_uint(o2);
                            u3[i] = __float_as_uint(o3);
                        }
                        tc::tmem_st8(acc + 8 * jj, u0);
                        tc::tmem_st8(acc + 32 + 8 * jj, u1);
                        tc::tmem_st8(acc + 64 + 8 * jj, u2);
                        tc::tmem_st8(acc + 96 + 8 * jj, u3);
                    }
                    tc::tmem_st_wait();
                }
                // ---- pass 2: group scales (one correctly rounded division each), codes
                float scv[4], rsv[4];
                {
                    float ga[4];
                    if (ppg == 1) {
                        ga[0] = am0; ga[1] = am1; ga[2] = am2; ga[3] = am3;
                    } else if (ppg == 2) {
                        ga[0] = ga[1] = fmaxf(am0, am1);
                        ga[2] = ga[3] = fmaxf(am2, am3);
                    } else {
                        ga[0] = ga[1] = ga[2] = ga[3] = fmaxf(fmaxf(am0, am1), fmaxf(am2, am3));
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (k == 0 || ppg == 1 || (ppg == 2 && k == 2)) {
                            scv[k] = __fdiv_rn(ga[k], (float)qmax);
                            rsv[k] = ga[k] > 0.f ? __fdiv_rn((float)qmax, ga[k]) : 0.f;
                        } else {
                            scv[k] = scv[k - 1];
                            rsv[k] = rsv[k - 1];
                        }
                    }
                }
                // the staging rows are free once this warp's previous code store has read them
                if (lane == 0) tc::bulk_wait_read<0>();
                __syncwarp();
                constexpr float MAGIC = 12582912.0f + (float)off;
                const float2 magic2 = make_float2(MAGIC, MAGIC);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    uint32_t v[32];
                    tc::tmem_ld32(acc + 32 * k, v);
                    tc::tmem_ld_wait();
                    const float2 rs2 = make_float2(rsv[k], rsv[k]);
                    uint32_t pk[BITS];
                    if constexpr (BITS == 4) {
#pragma unroll
                        for (int wd = 0; wd < 4; ++wd) {
                            float2 t[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                t[e] = fma2(make_float2(__uint_as_float(v[8 * wd + 2 * e]), __uint_as_float(v[8 * wd + 2 * e + 1])),
                                            rs2, magic2);
                            pk[wd] = pack_codes<4>(t[0], t[1], t[2], t[3]);
                        }
                        *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, k)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    } else {
                        const float2 z = make_float2(0.f, 0.f);
#pragma unroll
                        for (int wd = 0; wd < 8; ++wd)
                            pk[wd] = pack_codes<8>(
                                fma2(make_float2(__uint_as_float(v[4 * wd]), __uint_as_float(v[4 * wd + 1])), rs2, magic2),
                                fma2(make_float2(__uint_as_float(v[4 * wd + 2]), __uint_as_float(v[4 * wd + 3])), rs2, magic2),
                                z, z);
                        *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, 2 * k)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, 2 * k + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                    }
                }
                // the accumulator has been read
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[g]);
                // scales of my row: 128 / G values, contiguous
                if (rv) {
                    float *sp = p.scales + trow * ngr + (c0 >> gshift);
                    if (ppg == 1) *reinterpret_cast<float4 *>(sp) = make_float4(scv[0], scv[1], scv[2], scv[3]);
                    else if (ppg == 2) *reinterpret_cast<float2 *>(sp) = make_float2(scv[0], scv[2]);
                    else *sp = scv[0];
                }
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    tc::tma_store_3d(&tm_c, cb, (int)(c0 * BITS / 8), tb * ROWS + 32 * q, b);
                    tc::bulk_commit();
                }
            }
            if (p.k && p.ostage) {
                // the block's outliers: every group has staged its chunks' values
                tc::named_bar(3, ETH);
                for (int i = etid; i < nrows * p.k; i += ETH) {
                    const int rr = i / p.k;
                    p.outl[((int64_t)b * p.T + (int64_t)tb * ROWS + rr) * p.k + (i - rr * p.k)] = ost[i];
                }
                tc::named_bar(3, ETH);  // read out before the next block stages its outliers
            }
        }
        if (lane == 0) tc::bulk_wait<0>();  // code stores complete before the CTA exits
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

template <int BITS, int RK, bool WHT>
int launch(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t stream) {
    using L = Layout<BITS, RK>;
    const int64_t T = d->tokens, H = d->channels, B = d->batch;
    const int r = d->rank;
    const int64_t rowb = H * BITS / 8;
    CUtensorMap m_x{}, m_vt{}, m_c{};
    int st;
    if ((st = make_map_3d(&m_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, T, B, ldx, T * ldx, 64, ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_map_3d(&m_vt, d->basis_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, r, B, H, (int64_t)r * H, 64, r,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    // codes leave per warp: 32 token rows x one chunk's code bytes
    if ((st = make_map_3d(&m_c, d->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowb, T, B, rowb, T * rowb, L::CROW, 32,
                          tma_swz<L::CROW>())))
        return st;
    Params p{};
    p.T = T;
    p.H = H;
    p.rank = r;
    p.k = d->n_outlier;
    p.group = d->group;
    p.batch = d->batch;
    p.scales = d->scales;
    p.lr = d->lowrank;
    p.outl = d->outliers;
    p.idx = d->outlier_idx;
    p.vtile = d->basis_tile;
    p.nk2 = (int)(H / CH);
    p.ngs = (int)(H / 64);
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.nblocks = (int64_t)p.ntb * B;
    p.ngrid = (int)(p.nblocks < num_sms() ? p.nblocks : num_sms());
    const int k = d->n_outlier;
    constexpr int SMEM_MAX = 227 * 1024;
    // One block per CTA: the residual ring reuses the projection ring's memory
    // and both are as deep as it allows.  Otherwise the rings are separate so
    // that the next block's projection streams during this block's residual pass.
    const bool alias = p.nblocks <= p.ngrid;
    int na = MAXNA, nb = alias ? MAXNB : 3, ostage = k > 0;
    while (L::plan(p, na, nb, alias, k, ostage) > SMEM_MAX) {
        if (alias && nb > 3) --nb;
        else if (na > 3) --na;
        else if (ostage) ostage = 0;
        else if (nb > 2) --nb;
        else if (na > 2) --na;
        else return ACT_E_UNSUPPORTED;
    }
    const int smem = L::plan(p, na, nb, alias, k, ostage);
    auto kern = cg_encode_rows_kernel<BITS, RK, WHT>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<p.ngrid, THREADS, smem, stream>>>(m_x, m_vt, m_c, p);
    return launch_status();
}

}  // namespace cgencr
}  // namespace act

// Row encode, or ACT_E_UNSUPPORTED (before launching) for formats it does not
// cover: a rank outside 16..64, no basis tile operand, H outside
// 1024..16384 or not a multiple of 128 (an epilogue group must have a chunk in
// every block, and one CTA covers a block's channels), unaligned scales.
int act_cg_encode_rows(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s) {
    using namespace act::cgencr;
    if (d->tokens == 0) return ACT_OK;
    if (d->rank < 16 || d->rank > 64 || d->rank % 16 || !d->basis_tile) return ACT_E_UNSUPPORTED;
    if (d->channels % CH || d->channels < 1024 || d->channels > 16384) return ACT_E_UNSUPPORTED;
    if (!act::aligned(d->scales, 16) || !act::aligned(d->basis_tile, 16)) return ACT_E_UNSUPPORTED;
    const int rk = d->rank <= 16 ? 16 : (d->rank <= 32 ? 32 : 64);
#define ACT_ENCR_RK(B, W)                                     \
    do {                                                      \
        if (rk == 16) return launch<B, 16, W>(d, x, ldx, s);  \
        if (rk == 32) return launch<B, 32, W>(d, x, ldx, s);  \
        return launch<B, 64, W>(d, x, ldx, s);                \
    } while (0)
    if (d->bits == 4) {
        if (d->wht) ACT_ENCR_RK(4, true);
        ACT_ENCR_RK(4, false);
    }
    if (d->wht) ACT_ENCR_RK(8, true);
    ACT_ENCR_RK(8, false);
#undef ACT_ENCR_RK
}
