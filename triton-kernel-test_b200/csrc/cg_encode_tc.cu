// cg_encode_tc.cu -- channel-group encode on the tcgen05 tensor cores.
//
// A cluster of C CTAs owns one block of 128 tokens at a time; CTA c of the
// cluster owns a contiguous, group-aligned slice of the channels.  Per block:
//   phase 1  (warps 0, 1) TMA streams X[128 x slice] (64-channel steps) and
//            V^T[r x 64]; tcgen05.mma kind::f16 (M=128, N=r) accumulates the
//            partial projection L_c = X_slice . V_slice in TMEM;
//   exchange the epilogue pushes L_c to every peer with one bulk shared-to-
//            shared copy each (completing on the peer's mbarrier) and sums
//            all partials in rank order from local shared memory -- every CTA
//            gets the same L, from which it forms the per-token int8 low-rank
//            codes Lq and their scale sL (rank 0 stores them);
//   phase 2  (warps 2, 3, after phase 1 of the block completed) per
//            128-channel chunk: TMA re-reads the X chunk (the slice was read
//            moments ago and is still in L2) and the quantised basis rows as
//            bf16 integers; tcgen05.mma kind::f16 with those integer-valued
//            operands gives I = Lq . Vq^T exactly in fp32 (every product and
//            partial sum is an integer below 2^24); the epilogue (one token
//            row per thread, packed f32x2 arithmetic) forms the residual
//            fma(-I, sL, x), copies the outlier channels verbatim, optionally
//            rotates 128-channel blocks (Walsh-Hadamard), and forms int4/int8
//            codes with per-token group-absmax scales.  Codes go through a
//            shared-memory staging tile and leave with one TMA store per chunk;
//            scales and outlier values are staged and written with coalesced
//            stores (per FL chunks, per block), never one token row per thread.
// The two phases run on separate rings and issuers, so phase 1 of the next
// block streams from HBM while phase 2 of this block is quantised.
// X is read from HBM once; every other byte is written once.  Arithmetic
// matches oracle/actcomp_oracle.c (cg_encode_given_lr) bit for bit given L.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgenc {

constexpr int ROWS = 128;  // tokens per block (MMA M)
constexpr int KC = 64;     // channels per projection step
constexpr int CH = 128;    // channels per quantisation chunk (MMA N)

struct EncParams {
    int64_t T, H;
    int rank, k, group, batch;
    const float *basis_scale;
    uint8_t *codes;
    float *scales;
    int8_t *lrq;
    float *lrs;
    uint16_t *outl;
    const int32_t *idx;
    const uint16_t *vqb;  // basis_qb: bf16 tile operand (layout in include/actcomp.h)
    int C;         // CTAs per cluster
    int nunits;    // 128-channel chunks in H (the split unit)
    int ntb;       // token blocks per slice
    int64_t nblocks;
    int nclusters;
    int na;        // projection ring stages
    int ngs;       // 64-channel groups in the widest slice (outlier table entries)
    int ostage;    // outliers staged in shared memory and flushed per block
    // shared-memory offsets (bytes from the 1024-aligned base)
    int off_ringB, off_lqt, off_bar, off_cst, off_xch, off_ot, off_sst, off_ost, off_amx, off_wx, off_slr;
};

constexpr int NB = 2;      // residual ring: X 128x128 (32 KB) + Vq 128 x r bf16
constexpr int MAXNA = 6;   // projection ring: X 128x64 (16 KB) + V^T r x 64
constexpr int FL = 4;      // chunks per scale flush
constexpr int NT = 3;      // residual-term accumulators in TMEM (3 x 128 columns after the projection's 128):
                           // the MMA runs up to NT chunks ahead of the epilogue

constexpr int EW = 16;     // epilogue warps: 4 row quarters x 4 column quarters of a chunk

// RK: rank rounded up to 16, 32 or 64; LB = bytes of one bf16 row of Lq / Vq.
template <int BITS, bool WHT, int RK>
struct EncLayout {
    static constexpr int LB = 2 * RK;
    static constexpr int SLOT_A = 16 * 1024 + RK * 128;
    static constexpr int SLOT_B = 32 * 1024 + CH * LB;
    static constexpr int LQT = ROWS * LB;
    static constexpr int CROW = CH * BITS / 8;  // code bytes of one token row of a chunk
    static constexpr int QST = 32 * CROW;       // one row quarter's code staging buffer
    static constexpr int CST = 4 * 2 * QST;     // all quarters, double-buffered
    static constexpr int THREADS = 128 + 32 * EW;  // 2 producers, 2 MMA issuers, epilogue
    // Shared memory: projection ring, residual ring, low-rank code tile,
    // barriers, code staging (per row quarter, double-buffered, TMA-stored per
    // chunk), group-absmax exchange, per-row low-rank scales, the rotation
    // exchange (with WHT), then the sizes
    // that depend on the launch: projection exchange buffers (send + C-1
    // receive slots, 128 x r floats each), the outlier table of the current
    // slice (per 64-channel group: a mask of its outlier channels and the
    // number of outliers below it), the scale staging rows (FL chunks of
    // scales per token row, flushed with coalesced stores) and the outlier
    // staging rows (k values per token row, flushed per block).
    static int plan(EncParams &p, int na, int C, int r, int ngs, int group, int k, int ostage) {
        p.na = na;
        p.C = C;
        p.ngs = ngs;
        p.ostage = ostage;
        p.off_ringB = na * SLOT_A;
        p.off_lqt = p.off_ringB + NB * SLOT_B;
        p.off_bar = p.off_lqt + LQT;
        p.off_cst = p.off_bar + 1024;
        p.off_amx = p.off_cst + CST;                     // [2][4][128] floats
        p.off_slr = p.off_amx + 2 * 4 * ROWS * 4;        // [2][128] floats
        p.off_wx = p.off_slr + 2 * ROWS * 4;             // [4][128][32] floats with WHT
        p.off_xch = p.off_wx + (WHT ? 4 * ROWS * 32 * 4 : 0);
        p.off_ot = p.off_xch + (C > 1 ? C * ROWS * r * 4 : 0);
        p.off_sst = p.off_ot + ((ngs * 12 + 15) & ~15);
        const int spp = FL * (CH / group) + 4;
        p.off_ost = p.off_sst + ROWS * spp * 4;
        return p.off_ost + (ostage ? ((ROWS * k * 2 + 15) & ~15) : 0) + 1024;
    }
};

template <int PITCH>
__device__ __forceinline__ int swz(int r, int c) {
    if constexpr (PITCH == 128) return r * 128 + ((c ^ (r & 7)) << 4);
    else if constexpr (PITCH == 64) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    else return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
}
template <int PITCH>
constexpr tc::Swizzle swz_mode() {
    return PITCH == 128 ? tc::SW_128B : (PITCH == 64 ? tc::SW_64B : tc::SW_32B);
}
template <int PITCH>
constexpr CUtensorMapSwizzle tma_swz() {
    return PITCH == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                        : (PITCH == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

// byte offset of float4 chunk c (0 .. r/4-1) of row `row` in an exchange
// buffer: rows of r floats, chunks XOR-swizzled by the row (within aligned
// groups of 8 chunks, or of 4 when r/4 is not a multiple of 8) so that 32
// threads writing their rows' chunk c spread over the banks
__device__ __forceinline__ int xch_off(int row, int c, int r) {
    const int m = ((r / 4) % 8 == 0) ? 7 : 3;
    return row * r * 4 + ((c ^ (row & m)) << 4);
}

// 128-point unnormalised Walsh-Hadamard on 64 register pairs, stages m = 1..64
// in order, (a, b) -> (a + b, a - b) as the oracle; stages m >= 2 pair whole
// float2 elements and run as packed adds.
__device__ __forceinline__ void wht128_pairs(float2 (&v)[64]) {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        const float a = v[i].x, b = v[i].y;
        v[i] = make_float2(__fadd_rn(a, b), __fsub_rn(a, b));
    }
#pragma unroll
    for (int m2 = 1; m2 < 64; m2 <<= 1) {  // m = 2 * m2
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            if (!(i & m2)) {
                const float2 a = v[i], b = v[i + m2];
                v[i] = add2(a, b);
                v[i + m2] = sub2(a, b);
            }
        }
    }
}

// Codes: q = the exact product w * rs rounded to the nearest integer (ties to
// even) with rs = qmax / absmax (one correctly rounded division per group, as
// the oracle).  fma(w, rs, MAGIC) with MAGIC = 1.5 * 2^23 + 2^(b-1) does that
// rounding once and leaves q + 2^(b-1) in the low mantissa bits, with zeros up
// to bit 21.  Since |w| <= absmax, |w * rs| <= qmax (1 + 2^-24) < qmax + 1/2:
// the clamp never acts.  Packs 8 int4 codes (4 pairs) or 4 int8 codes (2 pairs)
// into one word, channel order low to high.
template <int BITS>
__device__ __forceinline__ uint32_t pack_codes(float2 t0, float2 t1, float2 t2, float2 t3) {
    const uint32_t a0 = __float_as_uint(t0.x), a1 = __float_as_uint(t0.y), a2 = __float_as_uint(t1.x),
                   a3 = __float_as_uint(t1.y);
    if constexpr (BITS == 4) {
        const uint32_t a4 = __float_as_uint(t2.x), a5 = __float_as_uint(t2.y), a6 = __float_as_uint(t3.x),
                       a7 = __float_as_uint(t3.y);
        // byte = u0 + 16 u1 (bits 4..21 of a0 are zero, so nothing carries into the low byte)
        const uint32_t b0 = a1 * 16u + a0, b1 = a3 * 16u + a2, b2 = a5 * 16u + a4, b3 = a7 * 16u + a6;
        return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
    } else {
        return __byte_perm(__byte_perm(a0, a1, 0x0040), __byte_perm(a2, a3, 0x0040), 0x5410);
    }
}

template <int BITS, bool WHT, int RK>
__global__ void __launch_bounds__(EncLayout<BITS, WHT, RK>::THREADS, 1)
    cg_encode_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_vt,
                        const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_cw,
                        EncParams p) {
    using L = EncLayout<BITS, WHT, RK>;
    constexpr int LB = L::LB;
    constexpr int qmax = (1 << (BITS - 1)) - 1, off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NA = p.na;
    uint8_t *ringA = smem, *ringB = smem + p.off_ringB;
    uint8_t *lqt = smem + p.off_lqt;
    uint8_t *xsend = smem + p.off_xch;  // this CTA's partial projection
    uint8_t *xrecv = xsend;             // + (slot + 1) * ROWS * r * 4: peers' partials
    uint64_t *fullA = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *emptyA = fullA + MAXNA;
    uint64_t *fullB = emptyA + MAXNA;
    uint64_t *emptyB = fullB + NB;
    uint64_t *tfull = emptyB + NB;  // [NT]
    uint64_t *tempty = tfull + NT;  // [NT]
    uint64_t *lfull = tempty + NT;
    uint64_t *lempty = lfull + 1;
    uint64_t *lqready = lempty + 1;
    uint64_t *pready = lqready + 1;  // peers' partials have landed (transaction bytes)
    uint64_t *pdone = pready + 1;    // peers have consumed our previous partial
    uint64_t *lseen = pdone + 1;     // phase-2 producer has observed lfull of the block
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(lseen + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = p.C;
    const uint32_t crank = C > 1 ? tc::cluster_rank() : 0;
    const int cluster = blockIdx.x / C;
    // my channel slice [c_lo, c_hi): a whole number of 128-channel chunks
    const int u_lo = (int)((int64_t)crank * p.nunits / C), u_hi = (int)((int64_t)(crank + 1) * p.nunits / C);
    const int64_t c_lo = (int64_t)u_lo * CH, c_hi = (int64_t)u_hi * CH;
    const int nk1 = (int)((c_hi - c_lo) / KC);
    const int nk2 = u_hi - u_lo;
    const int r = p.rank;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NA; ++s) {
            tc::mbar_init(&fullA[s], 1);
            tc::mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < NB; ++s) {
            tc::mbar_init(&fullB[s], 1);
            tc::mbar_init(&emptyB[s], 1 + EW);
        }
        for (int b = 0; b < NT; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], EW);
        }
        tc::mbar_init(lfull, 1);
        tc::mbar_init(lempty, 4);   // the 4 warps that read the projection (column quarter 0)
        tc::mbar_init(lqready, 4);
        tc::mbar_init(pready, 1);
        tc::mbar_init(pdone, C > 1 ? C - 1 : 1);
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
    if (C > 1) tc::cluster_sync();  // peers' barriers are initialised before any remote arrive
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tm_l = tmem;        // projection accumulator, columns [0, 64)
    const uint32_t tm_p = tmem + 128;  // NT residual-term accumulators, [128, 512)

    if (warp == 0) {
        // ------------------------------------------------------------ phase-1 producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_x);
            tc::prefetch_tmap(&tm_vt);
            int i = 0;
            bool ok = true;
            for (int64_t blk = cluster; blk < p.nblocks && ok; blk += p.nclusters) {
                const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
                for (int ks = 0; ks < nk1; ++ks, ++i) {
                    const int s = i % NA;
                    if (!(ok = tc::mbar_wait(&emptyA[s], ((i / NA) & 1) ^ 1, abort))) break;
                    uint8_t *st = ringA + s * L::SLOT_A;
                    tc::mbar_arrive_expect_tx(&fullA[s], ROWS * 128 + r * 128);
                    const int x = (int)(c_lo + ks * KC);
                    tc::tma_load_3d(st, &tm_x, &fullA[s], x, tb * ROWS, b);
                    tc::tma_load_3d(st + 16 * 1024, &tm_vt, &fullA[s], x, 0, b);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ projection MMA
        if (lane == 0) {
            const uint32_t id_proj = tc::idesc_f16(ROWS, r, true, false, false);
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = cluster; blk < p.nblocks && ok; blk += p.nclusters, ++nb) {
                // the epilogue has read the previous block's projection
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
            const int64_t ntile = p.H / CH;
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = cluster; blk < p.nblocks && ok; blk += p.nclusters, ++nb) {
                const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
                // re-read X only after phase 1 of this block has streamed it into L2
                if (!(ok = tc::mbar_wait(lfull, nb & 1, abort))) break;
                tc::mbar_arrive(lseen);
                for (int ck = 0; ck < nk2; ++ck, ++i) {
                    const int s = i % NB;
                    if (!(ok = tc::mbar_wait(&emptyB[s], ((i / NB) & 1) ^ 1, abort))) break;
                    uint8_t *st = ringB + s * L::SLOT_B;
                    tc::mbar_arrive_expect_tx(&fullB[s], 2 * ROWS * 128 + CH * LB);
                    // the residual sweep runs backwards over the slice: it starts on the
                    // X columns the projection sweep streamed last, still in L2
                    const int x = (int)(c_lo + (nk2 - 1 - ck) * CH);
                    tc::tma_load_3d(st, &tm_x, &fullB[s], x, tb * ROWS, b);
                    tc::tma_load_3d(st + ROWS * 128, &tm_x, &fullB[s], x + 64, tb * ROWS, b);
                    // the chunk's basis rows: one contiguous tile of the prepared operand
                    tc::bulk_load(st + 32 * 1024, p.vqb + ((int64_t)b * ntile + x / CH) * (CH * LB / 2), CH * LB,
                                  &fullB[s]);
                }
            }
        }
    } else if (warp == 3) {
        // ------------------------------------------------------------ residual-term MMA
        if (lane == 0) {
            constexpr uint32_t id_q = tc::idesc_f16(ROWS, CH, true, false, false);
            constexpr tc::Swizzle SWQ = swz_mode<LB>();
            const int nkq = (r + 15) / 16;
            int i = 0, nb = 0;
            bool ok = true;
            for (int64_t blk = cluster; blk < p.nblocks && ok; blk += p.nclusters, ++nb) {
                // low-rank codes of this block are in shared memory
                if (!(ok = tc::mbar_wait(lqready, nb & 1, abort))) break;
                tc::tc_fence_after();
                for (int ck = 0; ck < nk2; ++ck, ++i) {
                    const int s = i % NB, tb2 = i % NT;
                    if (!(ok = tc::mbar_wait(&fullB[s], (i / NB) & 1, abort))) break;
                    if (!(ok = tc::mbar_wait(&tempty[tb2], ((i / NT) & 1) ^ 1, abort))) break;
                    tc::tc_fence_after();
                    uint8_t *st = ringB + s * L::SLOT_B;
                    for (int kk = 0; kk < nkq; ++kk) {
                        const uint64_t ad = tc::smem_desc(lqt + kk * 32, 16, 8 * LB, SWQ);
                        const uint64_t bd = tc::smem_desc(st + 32 * 1024 + kk * 32, 16, 8 * LB, SWQ);
                        tc::mma_f16(tm_p + tb2 * CH, ad, bd, id_q, kk > 0);
                    }
                    tc::mma_commit(&tfull[tb2]);
                    tc::mma_commit(&emptyB[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // 16 warps: warp w (4..19) reads TMEM lanes 32 (w % 4).. (row quarter q)
        // and owns channels [32 h, 32 h + 32) of each 128-channel chunk,
        // h = (w - 4) / 4; one token row per thread.  The 4 warps of a row
        // quarter (a "q-group", 128 threads, named barrier 4 + q) share the
        // group absmax of groups wider than 32 channels, the rotation, the
        // code staging buffer and its TMA store.  Column quarter 0 (4 warps, one
        // thread per token row) also reads the projection and forms the
        // low-rank codes.
        const int ew = warp - 4;
        const int etid = threadIdx.x - 128;
        constexpr int ETH = 32 * EW;
        const int q = warp & 3;
        const int h = ew >> 2;
        const int qid = 4 + q;  // the q-group's named barrier
        constexpr int CROW = L::CROW;
        uint64_t *omask = reinterpret_cast<uint64_t *>(smem + p.off_ot);  // outlier table
        int32_t *obelow = reinterpret_cast<int32_t *>(omask + p.ngs);
        float *sst = reinterpret_cast<float *>(smem + p.off_sst);
        uint16_t *ost = reinterpret_cast<uint16_t *>(smem + p.off_ost);
        float *amx = reinterpret_cast<float *>(smem + p.off_amx);
        float *slr = reinterpret_cast<float *>(smem + p.off_slr);
        float *wx = reinterpret_cast<float *>(smem + p.off_wx);
        uint8_t *cst = smem + p.off_cst;
        const int ngs_mine = (int)((c_hi - c_lo) / 64);
        int cur_slice = -1;
        const int row = q * 32 + lane;
        const int G = p.group;
        const int ppg = G >> 5;        // 32-column pieces (threads) per group
        const int gpc = CH / G;        // groups per chunk
        const int spp = FL * gpc + 4;  // staged scales per token row (padded)
        const int ngr = (int)(p.H / G);
        const bool qleader = (h == 0 && lane == 0);  // issues the q-group's code stores
        // groups of 32 or 64 channels without rotation: every warp stores its own
        // codes and scales, and only the two warps of a 64-channel group meet
        const bool solo = !WHT && ppg <= 2;
        const int gshift = 31 - __clz(G);
        int j = 0, nb = 0;
        bool ok = true;
        for (int64_t blk = cluster; blk < p.nblocks && ok; blk += p.nclusters, ++nb) {
            const int b = (int)(blk / p.ntb), tb = (int)(blk % p.ntb);
            const int64_t t = (int64_t)tb * ROWS + row;
            const bool rv = t < p.T;
            const int64_t trow = (int64_t)b * p.T + t;
            const int nrows = (int)((p.T - (int64_t)tb * ROWS) < ROWS ? (p.T - (int64_t)tb * ROWS) : ROWS);
            if (h == 0) do {  // (a do-while so that a failed wait leaves this section, not the block loop)
                // ---- partial projection -> registers (column quarter 0 only)
                if (!(ok = tc::mbar_wait(lfull, nb & 1, abort))) break;
                tc::tc_fence_after();
                float Lr[RK];
                {
                    uint32_t v[32];
#pragma unroll
                    for (int jj = 0; jj < (RK + 31) / 32; ++jj) {
                        tc::tmem_ld32(tm_l + ((uint32_t)(q * 32) << 16) + 32 * jj, v);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (32 * jj + e < RK) Lr[32 * jj + e] = __uint_as_float(v[e]);
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(lempty);
                if (C > 1) {
                    // Exchange: every CTA pushes its 128 x r partial to each peer with one
                    // bulk copy (completing on the peer's pready), then sums all partials
                    // in rank order from local shared memory.  Lane 0 of each warp polls
                    // the cluster-scope barriers; the warp follows it.
                    const int PB = ROWS * r * 4;
                    if (nb > 0) {  // our buffers are free once every peer consumed the previous block
                        int okw = 1;
                        if (lane == 0) okw = tc::mbar_wait_cluster(pdone, (nb - 1) & 1, abort);
                        ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
                        if (!ok) break;
                    }
#pragma unroll
                    for (int e = 0; e < RK / 4; ++e)
                        if (4 * e < r)
                            *reinterpret_cast<float4 *>(xsend + xch_off(row, e, r)) =
                                make_float4(Lr[4 * e], Lr[4 * e + 1], Lr[4 * e + 2], Lr[4 * e + 3]);
                    tc::fence_proxy_async();
                    tc::named_bar(1, 128);
                    if (ew == 0 && lane == 0) {
                        tc::mbar_arrive_expect_tx(pready, (uint32_t)((C - 1) * PB));
                        for (int q2 = 0; q2 < C; ++q2) {
                            if (q2 == (int)crank) continue;
                            const int slot = (int)crank < q2 ? (int)crank : (int)crank - 1;  // our slot at q2
                            tc::bulk_copy_to_peer(tc::map_cluster(xrecv + (slot + 1) * PB, q2), xsend, (uint32_t)PB,
                                                  tc::map_cluster(pready, q2));
                        }
                    }
                    {
                        // a suspended try_wait on a barrier that only other CTAs complete
                        // sleeps out its whole interval: poll
                        int okw = 1;
                        if (lane == 0) okw = tc::mbar_wait_cluster(pready, nb & 1, abort);
                        ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
                        if (!ok) break;
                    }
                    // L = sum of the partials in rank order (identical in every CTA)
                    for (int pr = 0; pr < C; ++pr) {
                        const uint8_t *src =
                            pr == (int)crank ? xsend : xrecv + ((pr < (int)crank ? pr : pr - 1) + 1) * PB;
#pragma unroll
                        for (int e = 0; e < RK / 4; ++e) {
                            if (4 * e < r) {
                                const float4 v = *reinterpret_cast<const float4 *>(src + xch_off(row, e, r));
                                Lr[4 * e] = pr ? __fadd_rn(Lr[4 * e], v.x) : v.x;
                                Lr[4 * e + 1] = pr ? __fadd_rn(Lr[4 * e + 1], v.y) : v.y;
                                Lr[4 * e + 2] = pr ? __fadd_rn(Lr[4 * e + 2], v.z) : v.z;
                                Lr[4 * e + 3] = pr ? __fadd_rn(Lr[4 * e + 3], v.w) : v.w;
                            }
                        }
                    }
                    // tell every peer we have consumed its partial (the values are in registers)
                    tc::named_bar(1, 128);
                    if (ew == 0 && lane < C && lane != (int)crank) tc::mbar_arrive_remote(tc::map_cluster(pdone, lane));
                }
                // ---- per-token low-rank codes: Lq = nearest(L * sV * 127 / max|L * sV|), one fma
                float amax = 0.f;
#pragma unroll
                for (int e = 0; e < RK; ++e) {
                    if (e < r) {
                        Lr[e] = __fmul_rn(Lr[e], __ldg(p.basis_scale + (int64_t)b * r + e));
                        amax = fmaxf(amax, fabsf(Lr[e]));
                    }
                }
                const float sl = __fdiv_rn(amax, 127.0f);
                const float rsl = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
                constexpr float MAGIC_L = 12582912.0f + 128.0f;
                uint32_t lw[RK / 4];  // int8 codes, four per word
                uint32_t lb[RK / 2];  // the same codes as bf16 pairs (exact integers)
#pragma unroll
                for (int e = 0; e < RK / 4; ++e) lw[e] = 0;
#pragma unroll
                for (int e = 0; e < RK; e += 2) {
                    float f0 = 0.f, f1 = 0.f;
                    if (e < r) {
                        const float t0 = __fmaf_rn(Lr[e], rsl, MAGIC_L);
                        const float t1 = __fmaf_rn(Lr[e + 1], rsl, MAGIC_L);
                        const uint32_t u0 = __float_as_uint(t0) & 0xffu, u1 = __float_as_uint(t1) & 0xffu;  // q + 128
                        lw[e >> 2] |= ((u0 ^ 0x80u) << ((e & 3) * 8)) | ((u1 ^ 0x80u) << (((e + 1) & 3) * 8));
                        f0 = __fsub_rn(t0, MAGIC_L);
                        f1 = __fsub_rn(t1, MAGIC_L);
                    }
                    lb[e >> 1] = pack_bf16x2(f0, f1);
                }
#pragma unroll
                for (int c16 = 0; c16 < LB / 16; ++c16)
                    *reinterpret_cast<uint4 *>(lqt + swz<LB>(row, c16)) =
                        make_uint4(lb[4 * c16], lb[4 * c16 + 1], lb[4 * c16 + 2], lb[4 * c16 + 3]);
                if (crank == 0 && rv) {
                    uint32_t *dst = reinterpret_cast<uint32_t *>(p.lrq + trow * r);
#pragma unroll
                    for (int e = 0; e < RK / 4; ++e)
                        if (4 * e < r) dst[e] = lw[e];
                    p.lrs[trow] = sl;
                }
                slr[(nb & 1) * ROWS + row] = sl;
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(lqready);
            } while (0);
            // ---- the row's low-rank scale for every warp; outlier table of slice b
            // (indices ascending), rebuilt when the slice changes
            tc::named_bar(2, ETH);
            if (!ok) break;
            const float sl = slr[(nb & 1) * ROWS + row];
            if (p.k && b != cur_slice) {
                for (int gi = etid; gi < ngs_mine; gi += ETH) {
                    const int64_t lo = c_lo + 64 * (int64_t)gi;
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

            // ---- residual codes, chunk by chunk
            const float2 nsl2 = make_float2(-sl, -sl);
            for (int ck = 0; ck < nk2 && ok; ++ck, ++j) {
                const int s = j % NB, tb2 = j % NT;
                if (!(ok = tc::mbar_wait(&fullB[s], (j / NB) & 1, abort))) break;
                if (!(ok = tc::mbar_wait(&tfull[tb2], (j / NT) & 1, abort))) break;
                tc::tc_fence_after();
                const int cx = nk2 - 1 - ck;                          // chunk (backward sweep)
                const int64_t c0 = c_lo + (int64_t)cx * CH + 32 * h;  // my first channel
                const uint8_t *xt = ringB + s * L::SLOT_B;
                const uint8_t *box = xt + (h >> 1) * ROWS * 128;    // my X columns: box h / 2, chunks 4 (h & 1) ..
                float2 w[16];
                {
                    uint32_t I[32];
                    tc::tmem_ld32(tm_p + tb2 * CH + ((uint32_t)(q * 32) << 16) + 32 * h, I);
                    uint4 xv4[4];
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16)
                        xv4[c16] = *reinterpret_cast<const uint4 *>(box + swz<128>(row, (h & 1) * 4 + c16));
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16) {
                        const uint32_t wd[4] = {xv4[c16].x, xv4[c16].y, xv4[c16].z, xv4[c16].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 xv = make_float2(__uint_as_float(wd[e] << 16),
                                                          __uint_as_float(wd[e] & 0xffff0000u));
                            const float2 iv = make_float2(__uint_as_float(I[8 * c16 + 2 * e]),
                                                          __uint_as_float(I[8 * c16 + 2 * e + 1]));
                            w[4 * c16 + e] = fma2(iv, nsl2, xv);  // x - I * sL, one rounding
                        }
                    }
                }
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[tb2]);
                // outlier channels of my 32 (warp-uniform mask): verbatim copy, residual zeroed
                if (p.k) {
                    const int gi = (int)((c0 - c_lo) >> 6);
                    const uint64_t om64 = omask[gi];
                    const uint32_t om = (uint32_t)(om64 >> (32 * (h & 1)));
                    if (om) {
                        const int below = obelow[gi] + ((h & 1) ? __popc((uint32_t)om64) : 0);
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
                                        box + swz<128>(row, (h & 1) * 4 + c8) + 2 * e8);
                                    if (p.ostage) ost[row * p.k + slot] = bits;
                                    else if (rv) p.outl[trow * p.k + slot] = bits;
                                    if (e & 1) w[e >> 1].y = 0.f;
                                    else w[e >> 1].x = 0.f;
                                }
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&emptyB[s]);  // X and basis tile no longer needed
                if constexpr (WHT) {
                    // 128-point rotation over the q-group: stages m = 1..16 inside my 32
                    // channels, m = 32 and 64 across the 4 quarters through shared memory
                    float (&v)[32] = *reinterpret_cast<float(*)[32]>(&w[0]);
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
                    tc::named_bar(qid, 128);  // the previous chunk's exchange has been read
                    float *mine = wx + (h * ROWS + row) * 32;
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4)
                        *reinterpret_cast<float4 *>(mine + ((c4 ^ (row & 7)) << 2)) =
                            make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
                    tc::named_bar(qid, 128);
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4) {
                        float4 x4[4];
#pragma unroll
                        for (int hh = 0; hh < 4; ++hh)
                            x4[hh] = *reinterpret_cast<const float4 *>(wx + (hh * ROWS + row) * 32 + ((c4 ^ (row & 7)) << 2));
                        const float *a0 = &x4[0].x, *a1 = &x4[1].x, *a2 = &x4[2].x, *a3 = &x4[3].x;
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            const float s01 = __fadd_rn(a0[jj], a1[jj]), d01 = __fsub_rn(a0[jj], a1[jj]);
                            const float s23 = __fadd_rn(a2[jj], a3[jj]), d23 = __fsub_rn(a2[jj], a3[jj]);
                            float o;
                            if (h == 0) o = __fadd_rn(s01, s23);
                            else if (h == 1) o = __fadd_rn(d01, d23);
                            else if (h == 2) o = __fsub_rn(s01, s23);
                            else o = __fsub_rn(d01, d23);
                            v[4 * c4 + jj] = o;
                        }
                    }
                }
                // absmax of my 32 (balanced tree), then over the group's threads
                float am;
                {
                    float a[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) a[e] = fmaxf(fabsf(w[e].x), fabsf(w[e].y));
#pragma unroll
                    for (int st = 8; st > 0; st >>= 1)
#pragma unroll
                        for (int e = 0; e < st; ++e) a[e] = fmaxf(a[e], a[e + st]);
                    am = a[0];
                }
                float *ax = amx + (j & 1) * 4 * ROWS;
                float gam = am;
                if (solo) {
                    // groups of 64: the pair of warps (h, h ^ 1) shares its absmax; the
                    // slot (j & 1) is rewritten two chunks later, after the pair's next barrier
                    if (ppg == 2) {
                        ax[h * ROWS + row] = am;
                        tc::named_bar(4 + 2 * q + (h >> 1), 64);
                        gam = fmaxf(am, ax[(h ^ 1) * ROWS + row]);
                    }
                } else {
                    if (ppg > 1) ax[h * ROWS + row] = am;
                    // the q-group's staging buffer (j & 1) is free once its store of chunk j - 2 has read it
                    if (qleader) tc::bulk_wait_read<1>();
                    tc::named_bar(qid, 128);
                    if (ppg == 2) gam = fmaxf(am, ax[(h ^ 1) * ROWS + row]);
                    else if (ppg == 4)
                        gam = fmaxf(fmaxf(ax[row], ax[ROWS + row]), fmaxf(ax[2 * ROWS + row], ax[3 * ROWS + row]));
                }
                const float sc = __fdiv_rn(gam, (float)qmax);
                const float rs = gam > 0.f ? __fdiv_rn((float)qmax, gam) : 0.f;
                const float2 rs2 = make_float2(rs, rs);
                constexpr float MAGIC = 12582912.0f + (float)off;
                const float2 magic2 = make_float2(MAGIC, MAGIC);
                uint32_t pk[BITS];
                if constexpr (BITS == 4) {
#pragma unroll
                    for (int wd = 0; wd < 4; ++wd)
                        pk[wd] = pack_codes<4>(fma2(w[4 * wd], rs2, magic2), fma2(w[4 * wd + 1], rs2, magic2),
                                               fma2(w[4 * wd + 2], rs2, magic2), fma2(w[4 * wd + 3], rs2, magic2));
                } else {
                    const float2 z = make_float2(0.f, 0.f);
#pragma unroll
                    for (int wd = 0; wd < 8; ++wd)
                        pk[wd] = pack_codes<8>(fma2(w[2 * wd], rs2, magic2), fma2(w[2 * wd + 1], rs2, magic2), z, z);
                }
                if (solo) {
                    // this warp's 32 rows x 32 channels of codes leave by their own TMA
                    // store; buffer (j & 1) is free once the store of chunk j - 2 has read it
                    uint8_t *cb = cst + (ew * 2 + (j & 1)) * (L::QST / 4);
                    if (lane == 0) tc::bulk_wait_read<1>();
                    __syncwarp();
#pragma unroll
                    for (int c16 = 0; c16 < BITS / 4; ++c16)
                        *reinterpret_cast<uint4 *>(cb + lane * (CROW / 4) + 16 * c16) =
                            make_uint4(pk[4 * c16], pk[4 * c16 + 1], pk[4 * c16 + 2], pk[4 * c16 + 3]);
                    if ((h % ppg) == 0 && rv) p.scales[trow * ngr + (c0 >> gshift)] = sc;
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tc::tma_store_3d(&tm_cw, cb, (int)((c_lo + (int64_t)cx * CH) * BITS / 8) + h * (CROW / 4),
                                         tb * ROWS + 32 * q, b);
                        tc::bulk_commit();
                    }
                    continue;
                }
                uint8_t *cb = cst + (q * 2 + (j & 1)) * L::QST;
                if constexpr (BITS == 4) {
                    *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, h)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                } else {
                    *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, 2 * h)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    *reinterpret_cast<uint4 *>(cb + swz<CROW>(lane, 2 * h + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
                if ((h % ppg) == 0) sst[row * spp + (ck % FL) * gpc + (32 * h) / G] = sc;
                tc::fence_proxy_async();
                tc::named_bar(qid, 128);
                if (qleader) {
                    tc::tma_store_3d(&tm_c, cb, (int)((c_lo + (int64_t)cx * CH) * BITS / 8), tb * ROWS + 32 * q, b);
                    tc::bulk_commit();
                }
                if ((ck % FL) == FL - 1 || ck == nk2 - 1) {
                    // the q-group's staged scales of the last nch chunks: staging slot p
                    // holds chunk cx + (nch - 1 - p), so chunks cx .. cx + nch - 1 form one
                    // contiguous run per row; consecutive threads take consecutive scales
                    const int nch = ck % FL + 1, n = nch * gpc;
                    const int64_t g0 = (c_lo + (int64_t)cx * CH) / G;
                    const int qrows = nrows - 32 * q < 32 ? (nrows - 32 * q > 0 ? nrows - 32 * q : 0) : 32;
                    for (int i = h * 32 + lane; i < qrows * n; i += 128) {
                        const int rr = i / n, e = i - rr * n;
                        p.scales[((int64_t)b * p.T + (int64_t)tb * ROWS + 32 * q + rr) * ngr + g0 + e] =
                            sst[(32 * q + rr) * spp + (nch - 1 - e / gpc) * gpc + e % gpc];
                    }
                }
            }
            if (ok && p.k && p.ostage) {
                // the block's outliers of this slice: slots [s_lo, s_lo + s_n) of each row
                tc::named_bar(3, ETH);
                const int s_lo = obelow[0];
                const int s_n = obelow[ngs_mine - 1] + __popcll(omask[ngs_mine - 1]) - s_lo;
                if (s_n > 0)
                    for (int i = etid; i < nrows * s_n; i += ETH) {
                        const int rr = i / s_n, sl2 = s_lo + (i - rr * s_n);
                        p.outl[((int64_t)b * p.T + (int64_t)tb * ROWS + rr) * p.k + sl2] = ost[rr * p.k + sl2];
                    }
                tc::named_bar(3, ETH);  // read out before the next block stages its outliers
            }
        }
        if (lane == 0) tc::bulk_wait<0>();  // code stores complete before the CTA exits
        // do not exit while a peer may still read our partial buffer
        if (C > 1 && ok && nb > 0) {
            if (lane == 0) tc::mbar_wait_cluster(pdone, (nb - 1) & 1, abort);
            __syncwarp();
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
    // no CTA leaves while a peer may still read its shared memory
    if (C > 1) tc::cluster_sync();
}

template <int BITS, bool WHT, int RK>
int launch_encode(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t stream) {
    using L = EncLayout<BITS, WHT, RK>;
    const int64_t T = d->tokens, H = d->channels, B = d->batch;
    const int r = d->rank;
    const int64_t rowb = H * BITS / 8;
    CUtensorMap m_x{}, m_vt{}, m_c{}, m_cw{};
    int st;
    if ((st = make_map_3d(&m_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, T, B, ldx, T * ldx, 64, ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_map_3d(&m_vt, d->basis_t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, r, B, H, (int64_t)r * H, 64, r,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    // codes leave per row quarter: boxes of 32 token rows x one chunk's code bytes
    if ((st = make_map_3d(&m_c, d->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowb, T, B, rowb, T * rowb, L::CROW, 32,
                          tma_swz<L::CROW>())))
        return st;
    // ... or per warp: 32 token rows x 32 channels' code bytes
    if ((st = make_map_3d(&m_cw, d->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowb, T, B, rowb, T * rowb, L::CROW / 4, 32,
                          CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    EncParams p{};
    p.T = T;
    p.H = H;
    p.rank = r;
    p.k = d->n_outlier;
    p.group = d->group;
    p.batch = d->batch;
    p.basis_scale = d->basis_scale;
    p.codes = d->codes;
    p.scales = d->scales;
    p.lrq = d->lr_codes;
    p.lrs = d->lr_scale;
    p.outl = d->outliers;
    p.idx = d->outlier_idx;
    p.vqb = d->basis_qb;
    p.nunits = (int)(H / CH);
    const int k = d->n_outlier;
    constexpr int SMEM_MAX = 227 * 1024;
    // widest slice of a C-way split (ceil(nunits / C) chunks) in 64-channel groups
    auto ngs_of = [&](int c) { return (int)(((p.nunits + c - 1) / c) * (int64_t)CH / 64); };
    // the deepest projection ring (and outlier staging) that fits beside the rest
    auto fits = [&](int c) {
        EncParams t = p;
        return L::plan(t, 2, c, r, ngs_of(c), d->group, k, 0) <= SMEM_MAX;
    };
    // Cluster size: splitting a block's channels over C CTAs shortens each
    // CTA's sweep but costs a projection exchange per block (measured on B200
    // at 16384 x 4096: C = 1 115 us, 2 121 us, 4 190 us), so stay at one CTA
    // per block up to 8192 channels (2 MB per 128-token block) and split wider
    // activations in slices of at most 4096 channels, within 64 KB of exchange
    // buffers (C * 128 * r * 4 bytes) and the shared memory.
    int C = 1;
    while (C < 8 && H / C > 8192 / (C > 1 ? 2 : 1) && p.nunits / (C * 2) >= 1 && (2 * C) * ROWS * r * 4 <= 64 * 1024 &&
           fits(2 * C))
        C *= 2;
    if (C > p.nunits) C = p.nunits;
    // the deepest projection ring that fits (phase 1 streams X from HBM: the
    // more 16 KB steps in flight, the closer to the copy bandwidth)
    int na = MAXNA, ostage = k > 0;
    while (L::plan(p, na, C, r, ngs_of(C), d->group, k, ostage) > SMEM_MAX) {
        if (na > 3) --na;
        else if (ostage) ostage = 0;
        else if (na > 2) --na;
        else return ACT_E_UNSUPPORTED;
    }
    const int smem = L::plan(p, na, C, r, ngs_of(C), d->group, k, ostage);
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.nblocks = (int64_t)p.ntb * B;
    int maxc = num_sms() / C;
    p.nclusters = (int)(p.nblocks < maxc ? p.nblocks : maxc);
    auto kern = cg_encode_tc_kernel<BITS, WHT, RK>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(p.nclusters * C), 1, 1);
    cfg.blockDim = dim3(L::THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ACT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, m_x, m_vt, m_c, m_cw, p));
    return ACT_OK;
}

}  // namespace cgenc
}  // namespace act

// Tensor-core encode: needs a low-rank basis (rank 16..64, a multiple of 8, so
// that bf16 basis rows are 16-byte strided for TMA) with its bf16 copy,
// and H a multiple of 128 (the chunk the CTAs split H by).  Other shapes use
// the SIMT encode.
bool act_cg_encode_tc_supported(const actcomp_cg_desc *d) {
    if (d->rank < 16 || d->rank > 64 || d->rank % 8 || !d->basis_qb) return false;
    return d->channels % act::cgenc::CH == 0;
}

int act_cg_encode_tc(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s) {
    using namespace act::cgenc;
    if (d->tokens == 0) return ACT_OK;
#define ACT_ENC_RK(B, W)                                            \
    do {                                                            \
        if (rk == 16) return launch_encode<B, W, 16>(d, x, ldx, s); \
        if (rk == 32) return launch_encode<B, W, 32>(d, x, ldx, s); \
        return launch_encode<B, W, 64>(d, x, ldx, s);               \
    } while (0)
    const int rk = d->rank <= 16 ? 16 : (d->rank <= 32 ? 32 : 64);
    if (d->bits == 4) {
        if (d->wht) ACT_ENC_RK(4, true);
        ACT_ENC_RK(4, false);
    }
    if (d->wht) ACT_ENC_RK(8, true);
    ACT_ENC_RK(8, false);
#undef ACT_ENC_RK
}
