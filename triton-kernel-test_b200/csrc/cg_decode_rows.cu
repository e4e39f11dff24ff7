// cg_decode_rows.cu -- tensor-core decode of the channel-group format with
// whole tile rows per thread.
//
// One tile = 128 tokens x 128 channels; each CTA walks one contiguous range
// of tiles (persistent, one CTA per SM).  Roles:
//   warp 0      producer: per tile one bulk copy of the prepared bf16 basis
//               tile (128 channels x r) and one TMA load of the residual codes
//               into an S-stage ring; per token block one bulk copy of its
//               outlier values;
//   last warp   per token block, ahead of the MMAs, splits L (read from global
//               memory) into its three exact bf16 pieces: three swizzled operand
//               tiles in one of two slots;
//   warp 1      MMA: per tile tcgen05.mma kind::f16 (M=128, N=128, K=16 steps,
//               three pieces) gives the low-rank term P = L . V^T in float32 in
//               TMEM, one accumulator per epilogue group;
//   warps 2-17  epilogue: four groups of four warps, group g takes the tiles
//               g, g+4, g+8, ... of the range; a thread owns one token row of
//               the tile and all 128 channels, processed as four 32-channel
//               pieces: xhat = bf16(P + (u - 2^(b-1)) * s), outlier
//               channels verbatim; each warp stores its 32 rows x 64 channels
//               (two pieces) with one TMA store.
// Rotated formats run two epilogue groups (8 warps, up to 168 registers per
// thread): a thread dequantises its whole 128-channel row, applies the seven
// butterfly stages in registers and scales by 1/128, then adds the low-rank
// term piece by piece.
// Per-tile costs (waits, scalars, arrivals) are paid once per 128 channels of
// a row instead of once per 32.  Arithmetic is that of oracle/actcomp_oracle.c
// (cg_decode), except that the tensor cores sum the low-rank term in their own
// order (a few float32 ulps).
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgrow {

constexpr int ROWS = 128, CH = 128;
// Epilogue geometry: NG groups of four warps = NG TMEM accumulators of 128
// columns.  Unrotated: 4 groups, a thread works on 32 channels at a time.
// Rotated: 2 groups (up to 168 registers a thread: 10 warps put three on some
// SM sub-partitions).  Stages 1..32 of the 128-point transform stay inside each
// 64-channel half of a row, so a thread rotates one half at a time in registers
// and parks it in its warp's 128 TMEM scratch columns (after the accumulators),
// where stage 64 runs 8 columns at a time: 64 values live instead of the row.
template <bool WHT>
struct Geo {
    static constexpr int NG = WHT ? 2 : 4;
    static constexpr int EW = 4 * NG;
    static constexpr int THREADS = 64 + 32 * EW + 32;  // + the warp that prepares the piece tiles
};
// TMEM columns a block allocates: the accumulators, plus 128 scratch columns per
// group for the rotated formats
template <int RK, bool WHT>
constexpr uint32_t tmem_cols() {
    return WHT ? (RK ? 512u : 256u) : (RK ? 4u * 128u : 0u);
}

constexpr int WSTG = 32 * 128; // one warp's output staging: 32 rows x 64 bf16 (128-byte rows)
constexpr int PD = 2;          // per-row scalars prefetched PD group tiles ahead

struct RowParams {
    int64_t T, H;
    int rank, k, group, batch;
    int ntb, ncc;
    int64_t ntiles;
    int tq, trem;          // tiles per CTA: tq, one more for the first trem CTAs
    int S;                 // ring stages
    int n32;               // 32-channel groups of H
    int ostage;            // outlier values staged in shared memory per token block
    int ostb;              // bytes of one outlier slot
    const float *scales;
    const float *lr;       // projection L, T x rank float32 per slice
    const uint16_t *outliers;
    const int32_t *idx;
    const uint16_t *vtile; // basis tile operand
    int off_stg, off_lqb, off_ost, off_bar, off_ot;
};

template <int BITS, int RK>
struct RowLayout {
    static constexpr int LB = 2 * RK;                  // bytes of one bf16 operand row
    static constexpr int VQ = RK ? CH * LB : 0;         // basis tile
    static constexpr int CODE_ROW = CH * BITS / 8;      // code bytes of one token row of a tile
    static constexpr int CODES = ROWS * CODE_ROW;
    static constexpr int STAGE = VQ + CODES;
    static constexpr int LQB = RK ? 3 * ROWS * LB : 0;  // the three bf16 pieces of a token block's L
    // returns the shared-memory bytes, or 0 if S < 3 stages would fit
    static int plan(RowParams &p, int nsl, int EW) {
        const int fixed_no_ost = EW * WSTG + 2 * LQB + 1024 /*bars*/ +
                                 ((nsl * p.n32 * 8 + 15) & ~15) + 1024 /*align*/;
        const int ostb = (ROWS * p.k * 2 + 15) & ~15;
        for (int ost = p.k ? 1 : 0; ost >= 0; --ost) {
            const int fixed = fixed_no_ost + (ost ? 2 * ostb : 0);
            for (int S = 6; S >= 3; --S) {
                if (S * STAGE + fixed <= 227 * 1024) {
                    p.S = S;
                    p.ostage = ost;
                    p.ostb = ostb;
                    p.off_stg = S * STAGE;
                    p.off_lqb = p.off_stg + EW * WSTG;
                    p.off_ost = p.off_lqb + 2 * LQB;
                    p.off_bar = p.off_ost + (ost ? 2 * ostb : 0);
                    p.off_ot = p.off_bar + 1024;
                    return p.off_ot + ((nsl * p.n32 * 8 + 15) & ~15) + 1024;
                }
            }
        }
        return 0;
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

// Coordinates of consecutive tiles (channel chunk fastest), no divisions per step.
struct Walk {
    int cc, tb, b, ncc, ntb;
    __device__ Walk(int64_t first, int ncc_, int ntb_) : ncc(ncc_), ntb(ntb_) {
        cc = (int)(first % ncc);
        const int64_t bt = first / ncc;
        tb = (int)(bt % ntb);
        b = (int)(bt / ntb);
    }
    __device__ __forceinline__ void next() {
        if (++cc == ncc) {
            cc = 0;
            if (++tb == ntb) {
                tb = 0;
                ++b;
            }
        }
    }
    __device__ __forceinline__ int64_t block() const { return (int64_t)b * ntb + tb; }
};

// Outlier values of token block (tb, b): rows tb*128.. of the T x k matrix,
// one contiguous run; staged when its size and start are 16-byte multiples.
__device__ __forceinline__ uint32_t ost_bytes(const RowParams &p, int tb, int b, const uint16_t *&src) {
    const int64_t rows = (p.T - (int64_t)tb * ROWS) < ROWS ? (p.T - (int64_t)tb * ROWS) : ROWS;
    src = p.outliers + ((int64_t)b * p.T + (int64_t)tb * ROWS) * p.k;
    if (!p.ostage) return 0;
    const int64_t bytes = rows * p.k * 2;
    if ((bytes & 15) || (reinterpret_cast<uintptr_t>(src) & 15)) return 0;
    return (uint32_t)bytes;
}

// Residual of piece k (32 channels) of row r of a tile's codes:
// w = (u - 2^(b-1)) * s, the code u converted exactly to 2^23 + u by one byte
// permute against 0x4B000000 (int4 codes split into even and odd channels first).
template <int BITS, int OFF>
__device__ __forceinline__ void dequant_piece(const uint8_t *ct, int r, int k, float sc, float2 (&w)[16]) {
    uint32_t wd[BITS];
    if constexpr (BITS == 4) {
        const uint4 v = *reinterpret_cast<const uint4 *>(ct + swz<64>(r, k));
        wd[0] = v.x; wd[1] = v.y; wd[2] = v.z; wd[3] = v.w;
    } else {
        const uint4 v0 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * k));
        const uint4 v1 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * k + 1));
        wd[0] = v0.x; wd[1] = v0.y; wd[2] = v0.z; wd[3] = v0.w;
        wd[4] = v1.x; wd[5] = v1.y; wd[6] = v1.z; wd[7] = v1.w;
    }
    const float2 sc2 = make_float2(sc, sc);
    constexpr float UOFF = 8388608.0f + (float)OFF;
    const float2 uoff2 = make_float2(UOFF, UOFF);
    constexpr uint32_t K4B = 0x4B000000u;
#pragma unroll
    for (int wi = 0; wi < BITS; ++wi) {
        if constexpr (BITS == 4) {
            const uint32_t ev = wd[wi] & 0x0F0F0F0Fu, od = (wd[wi] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float2 f = make_float2(__uint_as_float(__byte_perm(ev, K4B, 0x7540u | m)),
                                             __uint_as_float(__byte_perm(od, K4B, 0x7540u | m)));
                w[4 * wi + m] = mul2(sub2(f, uoff2), sc2);
            }
        } else {
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const float2 f = make_float2(__uint_as_float(__byte_perm(wd[wi], K4B, 0x7540u | (2 * m))),
                                             __uint_as_float(__byte_perm(wd[wi], K4B, 0x7541u + 2 * m)));
                w[2 * wi + m] = mul2(sub2(f, uoff2), sc2);
            }
        }
    }
}

// Stages 1..32 of the oracle's butterfly order on one 64-channel half held as
// 32 channel pairs: stage 1 inside each pair, stage 2 * m2 between pairs i and
// i + m2.
__device__ __forceinline__ void wht_half(float2 (&w)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float a = w[i].x, c = w[i].y;
        w[i] = make_float2(__fadd_rn(a, c), __fsub_rn(a, c));
    }
#pragma unroll
    for (int m2 = 1; m2 < 32; m2 <<= 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (!(i & m2)) {
                const float2 a = w[i], c = w[i + m2];
                w[i] = add2(a, c);
                w[i + m2] = sub2(a, c);
            }
        }
    }
}

template <int BITS, int RK, bool WHT>
__global__ void __launch_bounds__(Geo<WHT>::THREADS, 1)
    cg_decode_rows_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_out,
                          RowParams p) {
    using L = RowLayout<BITS, RK>;
    constexpr int NG = Geo<WHT>::NG, EW = Geo<WHT>::EW;
    constexpr int LB = L::LB;
    constexpr int off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.S;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *empty = full + 6;
    uint64_t *tfull = empty + 6;
    uint64_t *tempty = tfull + NG;
    uint64_t *lqfull = tempty + NG;  // [2] token-block outlier slots loaded
    uint64_t *lqempty = lqfull + 2;  // [2] ... and no longer read
    uint64_t *pready = lqempty + 2;  // [2] piece tiles of a token block written
    uint64_t *pfree = pready + 2;    // [2] ... and read by the MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pfree + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint8_t *lqb = smem + p.off_lqb;
    uint8_t *ostbuf = smem + p.off_ost;
    const bool use_ost = p.k > 0 && p.ostage;
    const bool blockbuf = use_ost;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i_blk = blockIdx.x;
    const int64_t t_lo = (int64_t)i_blk * p.tq + (i_blk < p.trem ? i_blk : p.trem);
    const int64_t t_hi = t_lo + p.tq + (i_blk < p.trem ? 1 : 0);
    const int64_t tps = (int64_t)p.ntb * p.ncc;  // tiles per slice
    const int b_lo = (int)(t_lo / tps);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 4 + (RK ? 1 : 0));
        }
        for (int g = 0; g < NG; ++g) {
            tc::mbar_init(&tfull[g], 1);
            tc::mbar_init(&tempty[g], 4);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&lqfull[b], 1);
            // 4 arrivals per tile of the block (the warps of the group that decodes it)
            if (use_ost) tc::mbar_init(&lqempty[b], 4 * p.ncc);
            tc::mbar_init(&pready[b], 1);
            tc::mbar_init(&pfree[b], 1);
        }
        *abort = 0;
        tc::fence_mbar_init();
    }
    constexpr uint32_t TCOLS = tmem_cols<RK, WHT>();
    if (TCOLS && warp == 1) {
        tc::tmem_alloc(tmem_slot, TCOLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = TCOLS ? *tmem_slot : 0;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_codes);
            int i = 0, nlq = 0;
            Walk tw(t_lo, p.ncc, p.ntb);
            for (int64_t tile = t_lo; tile < t_hi; ++tile, ++i, tw.next()) {
                const int s = i % S;
                const uint32_t ph = (i / S) & 1;
                if (blockbuf && (tile == t_lo || tw.cc == 0)) {
                    const int ls = nlq & 1;
                    if (!tc::mbar_wait(&lqempty[ls], ((nlq >> 1) & 1) ^ 1, abort)) break;
                    const uint16_t *osrc = nullptr;
                    const uint32_t obytes = p.k ? ost_bytes(p, tw.tb, tw.b, osrc) : 0;
                    tc::mbar_arrive_expect_tx(&lqfull[ls], obytes);
                    if (obytes) tc::bulk_load(ostbuf + ls * p.ostb, osrc, obytes, &lqfull[ls]);
                    ++nlq;
                }
                if (!tc::mbar_wait(&empty[s], ph ^ 1, abort)) break;
                uint8_t *st = smem + s * L::STAGE;
                tc::mbar_arrive_expect_tx(&full[s], L::STAGE);
                if constexpr (RK > 0)
                    tc::bulk_load(st, p.vtile + ((int64_t)tw.b * p.ncc + tw.cc) * (CH * LB / 2), L::VQ, &full[s]);
                tc::tma_load_3d(st + L::VQ, &tm_codes, &full[s], tw.cc * L::CODE_ROW, tw.tb * ROWS, tw.b);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if constexpr (RK > 0) {
            constexpr uint32_t idesc = tc::idesc_f16(ROWS, CH, true, false, false);
            constexpr tc::Swizzle SW = swz_mode<LB>();
            const int nkq = (p.rank + 15) / 16;
            int i = 0, mlq = 0;
            bool ok = true;
            Walk tw(t_lo, p.ncc, p.ntb);
            for (int64_t tile = t_lo; tile < t_hi && ok; ++tile, ++i, tw.next()) {
                const int s = i % S, acc = i & (NG - 1);
                const uint32_t ph = (i / S) & 1, aph = (i / NG) & 1;
                if (tile == t_lo || tw.cc == 0) {
                    // a new token block: its piece tiles (prepared by the last warp)
                    const int ls = mlq & 1;
                    int okw = 1;
                    if (lane == 0) okw = tc::mbar_wait(&pready[ls], (mlq >> 1) & 1, abort);
                    if (!(ok = __shfl_sync(0xffffffffu, okw, 0) != 0)) break;
                    ++mlq;
                }
                const int ls = (mlq - 1) & 1;
                int okw = 1;
                if (lane == 0) {
                    okw = tc::mbar_wait(&full[s], ph, abort) && tc::mbar_wait(&tempty[acc], aph ^ 1, abort);
                    if (okw) {
                        tc::tc_fence_after();
                        const uint8_t *st = smem + s * L::STAGE;
                        const uint8_t *a = lqb + ls * L::LQB;
                        // P = hi . V^T + mid . V^T + lo . V^T
                        for (int pc = 0; pc < 3; ++pc)
                            for (int kk = 0; kk < nkq; ++kk) {
                                const uint64_t ad = tc::smem_desc(a + pc * ROWS * LB + kk * 32, 16, 8 * LB, SW);
                                const uint64_t bd = tc::smem_desc(st + kk * 32, 16, 8 * LB, SW);
                                tc::mma_f16(tmem + acc * CH, ad, bd, idesc, (pc | kk) > 0);
                            }
                        tc::mma_commit(&tfull[acc]);
                        tc::mma_commit(&empty[s]);
                        // last tile of this token block in the range: the slot frees when these MMAs complete
                        if (tw.cc == p.ncc - 1 || tile == t_hi - 1) tc::mma_commit(&pfree[ls]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
            }
        }
    } else if (warp == 2 + EW) {
        // ------------------------------------------------------------ L -> piece tiles, per token block
        if constexpr (RK > 0) {
            Walk tw(t_lo, p.ncc, p.ntb);
            int m = 0;
            bool ok = true;
            for (int64_t tile = t_lo; tile < t_hi && ok; ++tile, tw.next()) {
                if (tile != t_lo && tw.cc != 0) continue;  // not the first tile of a token block
                if (m == 0) {  // the range's first block: built by the epilogue warps
                    ++m;
                    continue;
                }
                const int ls = m & 1;
                if (!(ok = tc::mbar_wait(&pfree[ls], ((m >> 1) & 1) ^ 1, abort))) break;
                uint8_t *dst = lqb + ls * L::LQB;
                const int64_t t0 = (int64_t)tw.b * p.T + (int64_t)tw.tb * ROWS;  // first row of the block
                const int64_t rows_here = p.T - (int64_t)tw.tb * ROWS;
                build_piece_tiles<ROWS, LB>(p.lr, t0, rows_here, p.rank, dst, lane);
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&pready[ls]);
                ++m;
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int ew = warp - 2;
        const int g = ew >> 2;   // group: tiles g, g + 4, ...
        const int q = warp & 3;  // TMEM lane quadrant = row quarter
        const int r = q * 32 + lane;
        const int ngr = (int)(p.H / p.group);
        const int gshift = 31 - __clz(p.group);
        const uint32_t *otab = reinterpret_cast<const uint32_t *>(smem + p.off_ot);
        uint8_t *stg = smem + p.off_stg + ew * WSTG;
        // the piece tiles of the range's first token block, by all epilogue warps
        // (idle until its P exists): one memory round trip instead of the
        // builder warp's several
        if constexpr (RK > 0) {
            if (t_lo < t_hi) {
                const Walk fw(t_lo, p.ncc, p.ntb);
                const int64_t t0 = (int64_t)fw.b * p.T + (int64_t)fw.tb * ROWS;
                build_piece_tiles_team<ROWS, LB, 32 * EW>(p.lr, t0, p.T - (int64_t)fw.tb * ROWS, p.rank, lqb,
                                                          (int)threadIdx.x - 64);
                tc::fence_proxy_async();
            }
        }
        // outlier table of every slice this range touches: per 32-channel group a
        // mask of its outlier channels and the number of outliers below it (built
        // here, after the producer has started its loads)
        if (p.k) {
            uint32_t *omask = reinterpret_cast<uint32_t *>(smem + p.off_ot);
            const int b_hi = (int)((t_hi - 1) / tps);
            const int n = (b_hi - b_lo + 1) * p.n32;
            for (int e = threadIdx.x - 64; e < n; e += 32 * EW) {
                const int bs = b_lo + e / p.n32;
                const int64_t lo = 32 * (int64_t)(e % p.n32);
                uint32_t m = 0;
                int below = 0;
                for (int j = 0; j < p.k; ++j) {
                    const int64_t c = __ldg(p.idx + (int64_t)bs * p.k + j);
                    below += c < lo;
                    if (c >= lo && c < lo + 32) m |= 1u << (c - lo);
                }
                omask[2 * e] = m;
                omask[2 * e + 1] = (uint32_t)below;
            }
        }
        if (p.k || (RK > 0 && t_lo < t_hi)) {
            tc::named_bar(1, 32 * EW);  // the table and the first piece tiles complete
            if (RK > 0 && t_lo < t_hi && threadIdx.x == 64) tc::mbar_arrive(&pready[0]);
        }

        // per-row scalars of a tile: the group scales of its 128 channels,
        // loaded PD group tiles ahead
        float4 qsc[PD];
        auto load_scalars = [&](int64_t tile, const Walk &at, float4 &vsc) {
            vsc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (tile >= t_hi) return;
            const int64_t t = (int64_t)at.tb * ROWS + r;
            if (t >= p.T) return;
            const int64_t trow = (int64_t)at.b * p.T + t;
            const float *sp = p.scales + trow * ngr + (((int64_t)at.cc * CH) >> gshift);
            if (p.group == 32) {
                vsc = __ldg(reinterpret_cast<const float4 *>(sp));
            } else if (p.group == 64) {
                const float2 v = __ldg(reinterpret_cast<const float2 *>(sp));
                vsc = make_float4(v.x, v.x, v.y, v.y);
            } else {
                const float v = __ldg(sp);
                vsc = make_float4(v, v, v, v);
            }
        };
        auto step4 = [](Walk &w) {
#pragma unroll
            for (int e = 0; e < NG; ++e) w.next();
        };
        Walk tw(t_lo + g < t_hi ? t_lo + g : t_lo, p.ncc, p.ntb), nw = tw;
#pragma unroll
        for (int d = 0; d < PD; ++d) {
            load_scalars(t_lo + g + NG * d, nw, qsc[d]);
            step4(nw);
        }
        const int64_t blk_lo = t_lo / p.ncc;
        int64_t cur_blk = -1;
        const uint16_t *ovals = nullptr;
        int j = 0;
        for (int64_t tile = t_lo + g; tile < t_hi; tile += NG, ++j, step4(tw)) {
            const int i = (int)(tile - t_lo);
            const int s = i % S;
            const uint32_t ph = (i / S) & 1, aph = j & 1;
            const int cc = tw.cc, tb = tw.tb, b = tw.b;
            const float4 sc4 = qsc[0];
#pragma unroll
            for (int d = 0; d + 1 < PD; ++d) qsc[d] = qsc[d + 1];
            load_scalars(tile + NG * PD, nw, qsc[PD - 1]);
            step4(nw);

            const int64_t blk = tw.block();
            if (p.k && blk != cur_blk) {  // a new token block for this warp: where its outlier values are
                const uint16_t *osrc = nullptr;
                const uint32_t ob = ost_bytes(p, tb, b, osrc);
                ovals = osrc;
                if (use_ost) {
                    const int seq = (int)(blk - blk_lo);
                    if (!tc::mbar_wait(&lqfull[seq & 1], (seq >> 1) & 1, abort)) break;
                    if (ob) ovals = reinterpret_cast<const uint16_t *>(ostbuf + (seq & 1) * p.ostb);
                }
                cur_blk = blk;
            }
            bool ok = tc::mbar_wait(&full[s], ph, abort);
            if (RK) ok = ok && tc::mbar_wait(&tfull[g], aph, abort);
            if (!ok) break;
            tc::tc_fence_after();
            const int64_t t = (int64_t)tb * ROWS + r;
            const bool rv = t < p.T;
            const uint8_t *ct = smem + s * L::STAGE + L::VQ;
            const uint32_t *ot = otab + 2 * ((int64_t)(b - b_lo) * p.n32 + (((int64_t)cc * CH) >> 5));

            // rotated formats: the row's residual dequantised and rotated back in
            // the oracle's order (stages 1, 2, ..., 64, then * 1/128).  Each
            // 64-channel half takes stages 1..32 in registers and is parked in
            // this warp's 128 TMEM scratch columns; stage 64 and the scaling run
            // there 8 columns at a time, and the pieces come back like I.
            const uint32_t scr = tmem + ((uint32_t)(q * 32) << 16) + (RK ? NG * CH : 0) + CH * g;
            if constexpr (WHT) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float2 wh[32];
                    dequant_piece<BITS, off>(ct, r, 2 * h, h ? sc4.z : sc4.x,
                                             *reinterpret_cast<float2(*)[16]>(&wh[0]));
                    dequant_piece<BITS, off>(ct, r, 2 * h + 1, h ? sc4.w : sc4.y,
                                             *reinterpret_cast<float2(*)[16]>(&wh[16]));
                    if (h) {
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&empty[s]);  // the codes of this stage have been read
                    }
                    wht_half(wh);
                    tc::tmem_st32(scr + 64 * h, *reinterpret_cast<const uint32_t(*)[32]>(&wh[0]));
                    tc::tmem_st32(scr + 64 * h + 32, *reinterpret_cast<const uint32_t(*)[32]>(&wh[16]));
                }
                tc::tmem_st_wait();
                const float2 inv = make_float2(0.0078125f, 0.0078125f);
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {  // stage 64: channel c of the first half with c + 64
                    uint32_t A[8], C[8];
                    tc::tmem_ld8(scr + 8 * c8, A);
                    tc::tmem_ld8(scr + 64 + 8 * c8, C);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 a = make_float2(__uint_as_float(A[2 * e]), __uint_as_float(A[2 * e + 1]));
                        const float2 c = make_float2(__uint_as_float(C[2 * e]), __uint_as_float(C[2 * e + 1]));
                        const float2 lo = mul2(add2(a, c), inv), hi = mul2(sub2(a, c), inv);
                        A[2 * e] = __float_as_uint(lo.x);
                        A[2 * e + 1] = __float_as_uint(lo.y);
                        C[2 * e] = __float_as_uint(hi.x);
                        C[2 * e + 1] = __float_as_uint(hi.y);
                    }
                    tc::tmem_st8(scr + 8 * c8, A);
                    tc::tmem_st8(scr + 64 + 8 * c8, C);
                }
                tc::tmem_st_wait();
            }
#pragma unroll(WHT ? 4 : 1)
            for (int k = 0; k < 4; ++k) {
                uint32_t I[32];
                if constexpr (RK > 0) tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + g * CH + 32 * k, I);
                float2 w[16];
                if constexpr (WHT) {  // the piece, back from the scratch columns
                    uint32_t F[32];
                    tc::tmem_ld32(scr + 32 * k, F);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) w[e] = make_float2(__uint_as_float(F[2 * e]), __uint_as_float(F[2 * e + 1]));
                } else {
                uint32_t wd[BITS];
                if constexpr (BITS == 4) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(ct + swz<64>(r, k));
                    wd[0] = v.x; wd[1] = v.y; wd[2] = v.z; wd[3] = v.w;
                } else {
                    const uint4 v0 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * k));
                    const uint4 v1 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * k + 1));
                    wd[0] = v0.x; wd[1] = v0.y; wd[2] = v0.z; wd[3] = v0.w;
                    wd[4] = v1.x; wd[5] = v1.y; wd[6] = v1.z; wd[7] = v1.w;
                }
                if (k == 3) {  // the codes of this stage have been read
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(&empty[s]);
                }
                const float sc = k == 0 ? sc4.x : (k == 1 ? sc4.y : (k == 2 ? sc4.z : sc4.w));
                {
                    const float2 sc2 = make_float2(sc, sc);
                    constexpr float UOFF = 8388608.0f + (float)off;
                    const float2 uoff2 = make_float2(UOFF, UOFF);
                    // code u -> float 2^23 + u by one byte permute against 0x4B000000
                    constexpr uint32_t K4B = 0x4B000000u;
#pragma unroll
                    for (int wi = 0; wi < BITS; ++wi) {
                        if constexpr (BITS == 4) {
                            const uint32_t ev = wd[wi] & 0x0F0F0F0Fu, od = (wd[wi] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                            for (int m = 0; m < 4; ++m) {
                                const float2 f = make_float2(__uint_as_float(__byte_perm(ev, K4B, 0x7540u | m)),
                                                             __uint_as_float(__byte_perm(od, K4B, 0x7540u | m)));
                                w[4 * wi + m] = mul2(sub2(f, uoff2), sc2);
                            }
                        } else {
#pragma unroll
                            for (int m = 0; m < 2; ++m) {
                                const float2 f =
                                    make_float2(__uint_as_float(__byte_perm(wd[wi], K4B, 0x7540u | (2 * m))),
                                                __uint_as_float(__byte_perm(wd[wi], K4B, 0x7541u + 2 * m)));
                                w[2 * wi + m] = mul2(sub2(f, uoff2), sc2);
                            }
                        }
                    }
                }
                }  // unrotated
                if constexpr (RK > 0) {
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        w[e] = add2(make_float2(__uint_as_float(I[2 * e]), __uint_as_float(I[2 * e + 1])), w[e]);
                    if (k == 3) {  // the accumulator has been read
                        tc::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive(&tempty[g]);
                    }
                }
                // outlier channels of this piece (warp-uniform mask): verbatim values
                if (p.k) {
                    const uint32_t om = ot[2 * k];
                    if (om && (int64_t)cc * CH + 32 * k < p.H) {
                        const int below = (int)ot[2 * k + 1];
#pragma unroll
                        for (int c8 = 0; c8 < 4; ++c8) {
                            const uint32_t m8 = (om >> (8 * c8)) & 0xffu;
                            if (!m8) continue;
#pragma unroll
                            for (int e8 = 0; e8 < 8; ++e8) {
                                if ((m8 >> e8) & 1u) {
                                    const int e = 8 * c8 + e8;
                                    const int slot = below + __popc(om & ((1u << e) - 1u));
                                    const float v = rv ? bf2f(ovals[r * p.k + slot]) : 0.f;
                                    if (e & 1) w[e >> 1].y = v;
                                    else w[e >> 1].x = v;
                                }
                            }
                        }
                    }
                }
                // pieces 2h and 2h + 1 fill the warp's 32 rows x 64 channels
                // (128-byte swizzled rows) and leave by one TMA store; the buffer
                // is free once the previous half's store has read it
                uint8_t *buf = stg;
                if ((k & 1) == 0) {
                    if (lane == 0) tc::bulk_wait_read<0>();
                    __syncwarp();
                }
#pragma unroll
                for (int c16 = 0; c16 < 4; ++c16) {
                    const int e = 4 * c16;
                    uint4 v;
                    v.x = pack_bf16x2(w[e].x, w[e].y);
                    v.y = pack_bf16x2(w[e + 1].x, w[e + 1].y);
                    v.z = pack_bf16x2(w[e + 2].x, w[e + 2].y);
                    v.w = pack_bf16x2(w[e + 3].x, w[e + 3].y);
                    *reinterpret_cast<uint4 *>(buf + swz<128>(lane, 4 * (k & 1) + c16)) = v;
                }
                if (k & 1) {
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0 && ACT_DCHECK(cc * CH + 64 * (k >> 1) < p.H)) {
                        tc::tma_store_3d(&tm_out, buf, cc * CH + 64 * (k >> 1), tb * ROWS + 32 * q, b);
                        tc::bulk_commit();
                    }
                }
            }
            // the outlier slot of this block: 4 arrivals per tile, plus those of
            // the block's tiles outside the range (first and last tile of the range)
            if (use_ost && lane == 0) {
                uint32_t n = 1;
                if (tile == t_lo) n += (uint32_t)cc;
                if (tile == t_hi - 1) n += (uint32_t)(p.ncc - 1 - cc);
                tc::mbar_arrive_cnt(&lqempty[(int)(blk - blk_lo) & 1], n);
            }
        }
        if (lane == 0) tc::bulk_wait<0>();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (TCOLS && warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TCOLS);
    }
}

template <int BITS, int RK, bool WHT>
int launch(const actcomp_cg_desc *d, uint16_t *out, int64_t ldo, cudaStream_t stream) {
    using L = RowLayout<BITS, RK>;
    const int64_t T = d->tokens, H = d->channels, B = d->batch;
    CUtensorMap m_codes{}, m_out{};
    int st;
    const int64_t rowb = H * BITS / 8;
    if ((st = make_map_3d(&m_codes, d->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rowb, T, B, rowb, T * rowb,
                          L::CODE_ROW, ROWS, BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if ((st = make_map_3d(&m_out, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, H, T, B, ldo, T * ldo, 64, 32,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    RowParams p{};
    p.T = T;
    p.H = H;
    p.rank = d->rank;
    p.k = d->n_outlier;
    p.group = d->group;
    p.batch = d->batch;
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.ncc = (int)(H / CH);
    p.ntiles = (int64_t)p.ntb * p.ncc * B;
    p.n32 = (int)(H / 32);
    p.scales = d->scales;
    p.lr = d->lowrank;
    p.outliers = d->outliers;
    p.idx = d->outlier_idx;
    p.vtile = d->basis_tile;
    const int grid = (int)(p.ntiles < num_sms() ? p.ntiles : num_sms());
    p.tq = (int)(p.ntiles / grid);
    p.trem = (int)(p.ntiles % grid);
    const int64_t tps = (int64_t)p.ntb * p.ncc;
    const int64_t span = p.tq + (p.trem ? 1 : 0);
    const int nsl = (int)((span - 1) / tps + 2 < B ? (span - 1) / tps + 2 : B);
    const int smem = L::plan(p, nsl, Geo<WHT>::EW);
    if (!smem) return ACT_E_UNSUPPORTED;
    auto kern = cg_decode_rows_kernel<BITS, RK, WHT>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, Geo<WHT>::THREADS, smem, stream>>>(m_codes, m_out, p);
    return launch_status();
}

}  // namespace cgrow
}  // namespace act

// Decode through the row kernel, or ACT_E_UNSUPPORTED (before launching) for
// formats it does not cover: H not a multiple of 128 or below 512
// (with at least 4 tiles per token block no group of warps skips a block in
// the middle of its range, which the per-block barrier phases rely on), a
// rank without the basis tile operand, or an unaligned projection.
int act_cg_decode_rows(const actcomp_cg_desc *d, uint16_t *out, int64_t ldo, cudaStream_t s) {
    using namespace act::cgrow;
    if (d->tokens == 0) return ACT_OK;
    if (d->channels % CH != 0 || d->channels < 4 * CH || !act::aligned(d->scales, 16))
        return ACT_E_UNSUPPORTED;
    if (d->rank && (!d->basis_tile || !act::aligned(d->basis_tile, 16) || !act::aligned(d->lowrank, 16)))
        return ACT_E_UNSUPPORTED;
    const int rk = d->rank == 0 ? 0 : (d->rank <= 16 ? 16 : (d->rank <= 32 ? 32 : 64));
#define ACT_DECR(B, W)                                       \
    do {                                                     \
        switch (rk) {                                        \
            case 0: return launch<B, 0, W>(d, out, ldo, s);   \
            case 16: return launch<B, 16, W>(d, out, ldo, s); \
            case 32: return launch<B, 32, W>(d, out, ldo, s); \
            default: return launch<B, 64, W>(d, out, ldo, s); \
        }                                                    \
    } while (0)
    if (d->bits == 4) {
        if (d->wht) ACT_DECR(4, true);
        ACT_DECR(4, false);
    }
    if (d->wht) ACT_DECR(8, true);
    ACT_DECR(8, false);
#undef ACT_DECR
}
