// cg_tc.cu -- tensor-core (tcgen05) kernels of the channel-group format:
// decode and the fused consumers (elementwise product, SiLU and GELU backward).
//
// One tile = 128 tokens x 128 channels.  Per tile:
//   TMA warp   loads the prepared bf16 basis tile of the 128 channels, the
//              residual codes (128 x 64 B for int4) and, for a consumer, the
//              second operand (128 x 128 bf16) into a 2-6 stage ring; per token
//              block the outlier values;
//   last warp  per token block, ahead of the MMAs, splits L (read from global
//              memory) into its three exact bf16 pieces: three swizzled operand
//              tiles in one of two slots;
//   MMA warp   per tile tcgen05.mma kind::f16 (M=128, N=128, K=16 steps over
//              the three pieces) gives the low-rank term P = L . V^T in float32
//              in TMEM (4 accumulators of 128 columns, so the MMA runs ahead);
//   epilogue   (16 warps: 4 row quarters x 4 column quarters, one token row
//              and 32 channels per thread; the rotation exchanges quarters
//              through shared memory) reads P with tcgen05.ld, forms
//              xhat = bf16(P + (u - 2^(b-1)) * s) as the oracle does,
//              puts the outlier channels back and applies the consumer op.  The
//              decode writes the tile to a 64B-swizzled staging buffer and
//              stores it by TMA; the consumers store each thread's 64 bytes
//              straight from registers (no staging, so the ring stays deep).
// The kernel is persistent: one CTA per SM walks the tiles with a fixed stride.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
namespace cgtc {

constexpr int CH = 128;    // channels per tile (MMA N)
constexpr int ROWS = 128;  // tokens per tile (MMA M)
constexpr int NT = 4;      // TMEM accumulators (4 x 128 columns): the MMA runs up to NT tiles ahead
constexpr int WST = 32 * 64;  // one warp's output staging buffer: 32 rows x 32 bf16
// internal consumer ops of the softmax backward (outside the public op enum)
constexpr int OP_SMAX_DOT = 16;  // partial[row][tile][quarter] = sum over my 32 columns of P^ * dP
constexpr int OP_SMAX_BWD = 17;  // dS = (dP - rowsum) * P^
template <int OP>
constexpr bool is_smax() { return OP == OP_SMAX_DOT || OP == OP_SMAX_BWD; }

struct DecParams {
    int64_t T, H;
    int rank, k, group, batch;
    const float *scales;
    const float *lr;           // projection L, T x rank float32 per slice
    const uint16_t *outliers;
    const int32_t *idx;
    int ntb, ncc;
    int64_t ntiles;
    int n32;      // 32-channel groups of H (outlier table entries)
    int off_ot;   // shared-memory offset of the outlier table
    int tq, trem;              // tiles per CTA: tq, and one more for the first trem CTAs
    int off_ost, ostb;         // outlier staging: 2 slots of ostb bytes (128 rows x k bf16) at off_ost
    // softmax backward passes: per (row, tile, column quarter) partial dot
    // products of dP and P^, their per-row sums, causal mask of P^
    float *partials;
    const float *rowsum;
    int causal;
    int tri;                   // walk only the tiles on or below the diagonal (causal softmax passes)
    const uint16_t *vtile;     // basis tile operand (layout in include/actcomp.h)
    uint16_t *out;             // consumer output (direct stores), row stride ldo
    int64_t ldo;
};

template <int BITS, int OP, bool WHT, int RK>
struct DecLayout {
    static constexpr int LB = 2 * RK;              // bytes of one bf16 operand row
    static constexpr int PT = RK ? 3 * ROWS * LB : 0;  // the three bf16 piece tiles of a token block (2 slots)
    static constexpr int VQ = RK ? CH * LB : 0;        // basis tile
    static constexpr int CODES = ROWS * CH * BITS / 8;
    static constexpr int Y = OP == ACT_OP_DECODE ? 0 : ROWS * CH * 2;
    static constexpr int STAGE = VQ + CODES + Y;
    static constexpr int OUT = OP == ACT_OP_DECODE ? ROWS * CH * 2 : 0;  // decode output staging
    static constexpr int WX = WHT ? 4 * ROWS * 32 * 4 : 0;  // rotation exchange: 32 floats per thread
    static constexpr int FIXED = 2 * OUT + WX + 2 * PT + 1024;  // + barriers
    static constexpr int S = (6 * STAGE + FIXED <= 200 * 1024) ? 6 : (4 * STAGE + FIXED <= 200 * 1024) ? 4
                                                                  : ((3 * STAGE + FIXED <= 214 * 1024) ? 3 : 2);
    static constexpr int EW = 16;  // epilogue warps: 4 row quarters x 4 column quarters
    static constexpr int THREADS = 64 + 32 * EW + 32;  // + the warp that prepares the piece tiles
    static constexpr int OUT_OFF = S * STAGE;
    static constexpr int WX_OFF = OUT_OFF + 2 * OUT;
    static constexpr int PT_OFF = WX_OFF + WX;
    static constexpr int BAR_OFF = PT_OFF + 2 * PT;
    static constexpr int OT_OFF = BAR_OFF + 1024;
    static int ost_off(int n32) { return OT_OFF + ((n32 * 8 + 15) & ~15); }
    static int total(int n32, int k) { return ost_off(n32) + 2 * ((ROWS * k * 2 + 15) & ~15) + 1024; }
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

// Coordinates (channel chunk cc, token block tb, slice b) of consecutive
// tiles in cc-fastest order, advanced without divisions.  Each CTA walks one
// contiguous range of tiles, so consecutive tiles share their token block (and
// its low-rank codes) and read neighbouring code columns.  tri: only the tiles
// on or below the diagonal (cc <= tb) of square slices -- causal probabilities
// are zero above it, so the softmax passes never visit those tiles.
struct TileWalk {
    int cc, tb, b;
    int ncc, ntb;
    bool tri;
    __device__ TileWalk(int64_t first, int ncc_, int ntb_, bool tri_) : ncc(ncc_), ntb(ntb_), tri(tri_) {
        if (!tri) {
            cc = (int)(first % ncc);
            const int64_t bt = first / ncc;
            tb = (int)(bt % ntb);
            b = (int)(bt / ntb);
        } else {  // tile u of a slice: tb = the largest t with t (t + 1) / 2 <= u
            const int64_t per = (int64_t)ntb * (ntb + 1) / 2;
            b = (int)(first / per);
            const int64_t u = first % per;
            int t = (int)((sqrtf(8.0f * (float)u + 1.0f) - 1.0f) * 0.5f);
            while ((int64_t)(t + 1) * (t + 2) / 2 <= u) ++t;
            while (t > 0 && (int64_t)t * (t + 1) / 2 > u) --t;
            tb = t;
            cc = (int)(u - (int64_t)t * (t + 1) / 2);
        }
    }
    __device__ __forceinline__ int last_cc() const { return tri ? tb : ncc - 1; }
    __device__ __forceinline__ void next() {
        if (++cc > last_cc()) {
            cc = 0;
            if (++tb == ntb) {
                tb = 0;
                ++b;
            }
        }
    }
};
// The outlier values of token block (tb, b) are rows tb*128 .. of the T x k
// outlier matrix: one contiguous run, copied whole when its size and start
// are 16-byte multiples (always, except possibly for the last, partial block
// of a slice, whose values are then read from global memory).
__device__ __forceinline__ uint32_t ost_bytes(const DecParams &p, int tb, int b, const uint16_t *&src) {
    if (!p.k) return 0;
    const int64_t rows = (p.T - (int64_t)tb * ROWS) < ROWS ? (p.T - (int64_t)tb * ROWS) : ROWS;
    const int64_t bytes = rows * p.k * 2;
    src = p.outliers + ((int64_t)b * p.T + (int64_t)tb * ROWS) * p.k;
    if ((bytes & 15) || (reinterpret_cast<uintptr_t>(src) & 15)) return 0;
    return (uint32_t)bytes;
}
__device__ __forceinline__ void tile_range(const DecParams &p, int64_t &lo, int64_t &hi) {
    const int i = blockIdx.x;
    lo = (int64_t)i * p.tq + (i < p.trem ? i : p.trem);
    hi = lo + p.tq + (i < p.trem ? 1 : 0);
}

__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Epilogue geometry: 16 warps; warp w (2..17) reads TMEM lanes 32 (w % 4) ..
// (its row quarter q) and handles 32 channels [32 h, 32 h + 32) of the tile,
// h = (w - 2) / 4, one token row per thread: per tile a thread owns 32
// consecutive channels of one row, i.e. one int4 group of 32, half of a group
// of 64, a quarter of a group of 128 or of a rotation block.
template <int BITS, int OP, bool WHT, int RK>
__global__ void __launch_bounds__(DecLayout<BITS, OP, WHT, RK>::THREADS, 1)
    cg_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_codes, const __grid_constant__ CUtensorMap tm_y,
                        const __grid_constant__ CUtensorMap tm_out, DecParams p) {
    using L = DecLayout<BITS, OP, WHT, RK>;
    constexpr int LB = L::LB;
    constexpr int off = 1 << (BITS - 1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *empty = full + L::S;
    uint64_t *tfull = empty + L::S;
    uint64_t *tempty = tfull + NT;
    uint64_t *lqfull = tempty + NT;   // [2] token-block outlier slots loaded
    uint64_t *lqempty = lqfull + 2;  // [2] ... and no longer read
    uint64_t *pready = lqempty + 2;  // [2] piece tiles of a token block written
    uint64_t *pfree = pready + 2;    // [2] ... and read by the MMAs
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pfree + 2);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    uint8_t *ptile = smem + L::PT_OFF;
    uint8_t *ostbuf = smem + p.off_ost;
    const bool blockbuf = p.k > 0;  // per-token-block outlier slots in use
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t t_lo, t_hi;
    tile_range(p, t_lo, t_hi);

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::S; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], L::EW + (RK ? 1 : 0));
        }
        for (int b = 0; b < NT; ++b) {
            tc::mbar_init(&tfull[b], 1);
            tc::mbar_init(&tempty[b], L::EW);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&lqfull[b], 1);
            if (p.k) tc::mbar_init(&lqempty[b], L::EW);
            tc::mbar_init(&pready[b], 1);
            tc::mbar_init(&pfree[b], 1);
        }
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (RK && warp == 1) {
        tc::tmem_alloc(tmem_slot, NT * CH);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = RK ? *tmem_slot : 0;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tm_codes);
            int i = 0, nlq = 0;
            TileWalk tw(t_lo, p.ncc, p.ntb, p.tri != 0);
            for (int64_t tile = t_lo; tile < t_hi; ++tile, ++i, tw.next()) {
                const int s = i % L::S;
                const uint32_t ph = (i / L::S) & 1;
                const int cc = tw.cc, tb = tw.tb, b = tw.b;
                if (blockbuf && (tile == t_lo || cc == 0)) {
                    // a new token block: its outlier values into the free slot
                    const int ls = nlq & 1;
                    if (!tc::mbar_wait(&lqempty[ls], ((nlq >> 1) & 1) ^ 1, abort)) break;
                    const uint16_t *osrc = nullptr;
                    const uint32_t obytes = ost_bytes(p, tb, b, osrc);
                    tc::mbar_arrive_expect_tx(&lqfull[ls], obytes);
                    if (obytes) tc::bulk_load(ostbuf + ls * p.ostb, osrc, obytes, &lqfull[ls]);
                    ++nlq;
                }
                if (!tc::mbar_wait(&empty[s], ph ^ 1, abort)) break;
                uint8_t *st = smem + s * L::STAGE;
                tc::mbar_arrive_expect_tx(&full[s], L::STAGE);
                if constexpr (RK > 0)  // one contiguous tile of the prepared operand
                    tc::bulk_load(st, p.vtile + ((int64_t)b * p.ncc + cc) * (L::VQ / 2), L::VQ, &full[s]);
                tc::tma_load_3d(st + L::VQ, &tm_codes, &full[s], cc * L::CODE_ROW, tb * ROWS, b);
                if constexpr (OP != ACT_OP_DECODE) {
                    uint8_t *y = st + L::VQ + L::CODES;
                    tc::tma_load_3d(y, &tm_y, &full[s], cc * CH, tb * ROWS, b);
                    tc::tma_load_3d(y + ROWS * 128, &tm_y, &full[s], cc * CH + 64, tb * ROWS, b);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if constexpr (RK > 0) {
            constexpr uint32_t idesc = tc::idesc_f16(ROWS, CH, true, false, false);
            constexpr tc::Swizzle SW = LB == 32 ? tc::SW_32B : (LB == 64 ? tc::SW_64B : tc::SW_128B);
            const int nkq = (p.rank + 15) / 16;
            int i = 0, mlq = 0;
            bool ok = true;
            TileWalk tw(t_lo, p.ncc, p.ntb, p.tri != 0);
            for (int64_t tile = t_lo; tile < t_hi && ok; ++tile, ++i, tw.next()) {
                const int s = i % L::S, b = i % NT;
                const uint32_t ph = (i / L::S) & 1, bph = (i / NT) & 1;
                if (tile == t_lo || tw.cc == 0) {
                    // a new token block: its piece tiles (prepared by the last warp)
                    int okw = 1;
                    if (lane == 0) okw = tc::mbar_wait(&pready[mlq & 1], (mlq >> 1) & 1, abort);
                    if (!(ok = __shfl_sync(0xffffffffu, okw, 0) != 0)) break;
                    ++mlq;
                }
                const uint8_t *pts = ptile + ((mlq - 1) & 1) * L::PT;
                int okw = 1;
                if (lane == 0) {
                    okw = tc::mbar_wait(&full[s], ph, abort) && tc::mbar_wait(&tempty[b], bph ^ 1, abort);
                    if (okw) {
                        tc::tc_fence_after();
                        uint8_t *st = smem + s * L::STAGE;
                        // P = hi . V^T + mid . V^T + lo . V^T
                        for (int pc = 0; pc < 3; ++pc)
                            for (int kk = 0; kk < nkq; ++kk) {
                                const uint64_t ad = tc::smem_desc(pts + pc * ROWS * LB + kk * 32, 16, 8 * LB, SW);
                                const uint64_t bd = tc::smem_desc(st + kk * 32, 16, 8 * LB, SW);
                                tc::mma_f16(tmem + b * CH, ad, bd, idesc, (pc | kk) > 0);
                            }
                        tc::mma_commit(&tfull[b]);
                        tc::mma_commit(&empty[s]);
                        // last tile of this token block in my range: the piece tiles free once these MMAs complete
                        if (tw.cc == tw.last_cc() || tile == t_hi - 1) tc::mma_commit(&pfree[(mlq - 1) & 1]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
            }
        }
    } else if (warp == 2 + L::EW) {
        // ------------------------------------------------------------ L -> piece tiles, per token block
        if constexpr (RK > 0) {
            TileWalk tw(t_lo, p.ncc, p.ntb, p.tri != 0);
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
                uint8_t *dst = ptile + ls * L::PT;
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
        const int etid = threadIdx.x - 64;
        constexpr int ETH = 32 * L::EW;
        const int q = warp & 3;  // TMEM lane quadrant of this warp
        const int h = ew >> 2;   // 32-channel quarter of the tile
        const int r = q * 32 + lane;
        const int ngr = (int)(p.H / p.group);
        uint32_t *omask = reinterpret_cast<uint32_t *>(smem + p.off_ot);  // per 32-channel group of H
        int32_t *obelow = reinterpret_cast<int32_t *>(omask + p.n32);
        float *wx = reinterpret_cast<float *>(smem + L::WX_OFF);
        int cur_slice = -1;

        // per-row scalars of a tile (group scale, softmax row sum), loaded PD tiles
        // ahead into a register queue so the global-load latency (~1-2 us under
        // load) hides behind PD tiles of work
        constexpr int PD = 4;
        float qsc[PD], qrs[PD];
        TileWalk tw(t_lo, p.ncc, p.ntb, p.tri != 0), nw = tw;  // this tile, the one PD ahead
        // the piece tiles of the range's first token block, by all epilogue warps
        // (idle until its P exists): one memory round trip instead of the
        // builder warp's several
        if constexpr (RK > 0) {
            if (t_lo < t_hi) {
                const int64_t t0 = (int64_t)tw.b * p.T + (int64_t)tw.tb * ROWS;
                build_piece_tiles_team<ROWS, LB, ETH>(p.lr, t0, p.T - (int64_t)tw.tb * ROWS, p.rank, ptile, etid);
                tc::fence_proxy_async();
                tc::named_bar(3, ETH);
                if (etid == 0) tc::mbar_arrive(&pready[0]);
            }
        }
        const int gshift = 31 - __clz(p.group);
        auto load_scalars = [&](int64_t tile, const TileWalk &at, float &vsc, float &vrs) {
            vsc = 0.f;
            vrs = 0.f;
            if (tile >= t_hi) return;
            const int64_t t = (int64_t)at.tb * ROWS + r;
            if (t >= p.T) return;
            const int64_t trow = (int64_t)at.b * p.T + t;
            const int64_t c = (int64_t)at.cc * CH + 32 * h;
            if (c < p.H) vsc = __ldg(p.scales + trow * ngr + (c >> gshift));
            if constexpr (OP == OP_SMAX_BWD) vrs = __ldg(p.rowsum + trow);
        };
#pragma unroll
        for (int d = 0; d < PD; ++d) {
            load_scalars(t_lo + d, nw, qsc[d], qrs[d]);
            nw.next();
        }

        int i = 0, elq = 0;
        const uint16_t *ovals = nullptr;  // this token block's outlier values (shared or global)
        for (int64_t tile = t_lo; tile < t_hi; ++tile, ++i, tw.next()) {
            const int s = i % L::S, b = i % NT, ob = i & 1;
            const uint32_t ph = (i / L::S) & 1, bph = (i / NT) & 1;
            const int cc = tw.cc, tb = tw.tb, sl_b = tw.b;
            const float sc = qsc[0], rsum = qrs[0];
#pragma unroll
            for (int d = 0; d + 1 < PD; ++d) {
                qsc[d] = qsc[d + 1];
                qrs[d] = qrs[d + 1];
            }
            load_scalars(tile + PD, nw, qsc[PD - 1], qrs[PD - 1]);
            nw.next();

            // outlier table of the slice: per 32-channel group a mask and the
            // number of outlier channels below it (indices ascending)
            if (p.k && sl_b != cur_slice) {
                tc::named_bar(2, ETH);
                for (int g = etid; g < p.n32; g += ETH) {
                    const int64_t lo = 32 * (int64_t)g;
                    uint32_t m = 0;
                    int below = 0;
                    for (int j = 0; j < p.k; ++j) {
                        const int64_t c = __ldg(p.idx + (int64_t)sl_b * p.k + j);
                        below += c < lo;
                        if (c >= lo && c < lo + 32) m |= 1u << (c - lo);
                    }
                    omask[g] = m;
                    obelow[g] = below;
                }
                tc::named_bar(2, ETH);
                cur_slice = sl_b;
            }
            if (p.k && (tile == t_lo || tw.cc == 0)) {  // a new token block: its outlier values
                if (!tc::mbar_wait(&lqfull[elq & 1], (elq >> 1) & 1, abort)) break;
                const uint16_t *osrc = nullptr;
                ovals = ost_bytes(p, tb, sl_b, osrc) ? reinterpret_cast<const uint16_t *>(ostbuf + (elq & 1) * p.ostb)
                                                     : osrc;
                ++elq;
            }
            bool ok = tc::mbar_wait(&full[s], ph, abort);
            if (RK) ok = ok && tc::mbar_wait(&tfull[b], bph, abort);
            if (!ok) break;
            tc::tc_fence_after();
            const int64_t t = (int64_t)tb * ROWS + r;
            const bool rv = t < p.T;
            const int64_t trow = (int64_t)sl_b * p.T + t;
            const int64_t c_first = (int64_t)cc * CH + 32 * h;

            // low-rank term P (float32) for my 32 channels: issued first, waited for late
            uint32_t I[32];
            if constexpr (RK > 0) tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + b * CH + 32 * h, I);

            // residual: w = (u - 2^(b-1)) * s, exact conversion of the code
            const uint8_t *ct = smem + s * L::STAGE + L::VQ;
            float2 w[16];
            {
                const float2 sc2 = make_float2(sc, sc);
                constexpr float UOFF = 8388608.0f + (float)off;
                const float2 uoff2 = make_float2(UOFF, UOFF);
                uint32_t wd[BITS];  // BITS words hold my 32 codes
                if constexpr (BITS == 4) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(ct + swz<64>(r, h));
                    wd[0] = v.x; wd[1] = v.y; wd[2] = v.z; wd[3] = v.w;
                } else {
                    const uint4 v0 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * h));
                    const uint4 v1 = *reinterpret_cast<const uint4 *>(ct + swz<128>(r, 2 * h + 1));
                    wd[0] = v0.x; wd[1] = v0.y; wd[2] = v0.z; wd[3] = v0.w;
                    wd[4] = v1.x; wd[5] = v1.y; wd[6] = v1.z; wd[7] = v1.w;
                }
                // code u -> float 2^23 + u by one byte permute against 0x4B000000:
                // result bytes (code byte, 0, 0, 0x4B); int4 codes are first split
                // into even (low nibble) and odd channels, one byte per code
                constexpr uint32_t K4B = 0x4B000000u;
#pragma unroll
                for (int wi = 0; wi < BITS; ++wi) {
                    if constexpr (BITS == 4) {
                        const uint32_t ev = wd[wi] & 0x0F0F0F0Fu, od = (wd[wi] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                        for (int m = 0; m < 4; ++m) {  // channels 8 wi + 2 m, 8 wi + 2 m + 1
                            const float2 f = make_float2(__uint_as_float(__byte_perm(ev, K4B, 0x7540u | m)),
                                                         __uint_as_float(__byte_perm(od, K4B, 0x7540u | m)));
                            w[4 * wi + m] = mul2(sub2(f, uoff2), sc2);
                        }
                    } else {
#pragma unroll
                        for (int m = 0; m < 2; ++m) {  // channels 4 wi + 2 m, 4 wi + 2 m + 1
                            const float2 f = make_float2(__uint_as_float(__byte_perm(wd[wi], K4B, 0x7540u | (2 * m))),
                                                         __uint_as_float(__byte_perm(wd[wi], K4B, 0x7541u + 2 * m)));
                            w[2 * wi + m] = mul2(sub2(f, uoff2), sc2);
                        }
                    }
                }
            }
            if constexpr (WHT) {
                // 128-point rotation over the 4 column quarters of a row: stages
                // m = 1..16 inside my 32 channels, m = 32 and 64 across quarters
                // through shared memory (oracle stage order), then * 1/128
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
                tc::named_bar(4 + q, 128);  // the previous tile's exchange has been read
                float *mine = wx + (h * ROWS + r) * 32;
#pragma unroll
                for (int c4 = 0; c4 < 8; ++c4)
                    *reinterpret_cast<float4 *>(mine + ((c4 ^ (r & 7)) << 2)) =
                        make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
                tc::named_bar(4 + q, 128);
#pragma unroll
                for (int c4 = 0; c4 < 8; ++c4) {  // four channels of each quarter at a time
                    float4 x4[4];
#pragma unroll
                    for (int hh = 0; hh < 4; ++hh)
                        x4[hh] = *reinterpret_cast<const float4 *>(wx + (hh * ROWS + r) * 32 + ((c4 ^ (r & 7)) << 2));
                    const float *a0 = &x4[0].x, *a1 = &x4[1].x, *a2 = &x4[2].x, *a3 = &x4[3].x;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // stage 32 pairs quarters (0, 1) and (2, 3); stage 64 pairs (0', 2') and (1', 3')
                        const float s01 = __fadd_rn(a0[j], a1[j]), d01 = __fsub_rn(a0[j], a1[j]);
                        const float s23 = __fadd_rn(a2[j], a3[j]), d23 = __fsub_rn(a2[j], a3[j]);
                        float o;
                        if (h == 0) o = __fadd_rn(s01, s23);
                        else if (h == 1) o = __fadd_rn(d01, d23);
                        else if (h == 2) o = __fsub_rn(s01, s23);
                        else o = __fsub_rn(d01, d23);
                        v[4 * c4 + j] = __fmul_rn(o, 0.0078125f);
                    }
                }
            }
            // xhat = P + w
            if constexpr (RK > 0) {
                tc::tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    w[e] = add2(make_float2(__uint_as_float(I[2 * e]), __uint_as_float(I[2 * e + 1])), w[e]);
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&tempty[b]);
            }
            // bf16 reconstruction (the consumer ops take it as their input)
            if constexpr (OP != ACT_OP_DECODE) {
#pragma unroll
                for (int e = 0; e < 16; ++e) w[e] = make_float2(rne_bf(w[e].x), rne_bf(w[e].y));
            }
            // outlier channels of my 32 (warp-uniform mask): verbatim values
            if (p.k && c_first < p.H) {
                const int g32 = (int)(c_first >> 5);
                const uint32_t om = omask[g32];
                if (om) {
                    const int below = obelow[g32];
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
            if constexpr (is_smax<OP>()) {
                // causal probabilities: P^[t][c] = 0 above the diagonal (c > t)
                if (p.causal) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int64_t col = c_first + 2 * e;
                        if (col > t) w[e].x = 0.f;
                        if (col + 1 > t) w[e].y = 0.f;
                    }
                }
            }
            // second operand and consumer op
            // OP_SMAX_DOT: P^ . dP over my 32 columns, even and odd columns in two
            // running sums (packed), added at the end
            float2 dot2 = make_float2(0.f, 0.f);
            if constexpr (OP != ACT_OP_DECODE) {
                const uint8_t *box = smem + s * L::STAGE + L::VQ + L::CODES + (h >> 1) * ROWS * 128;
#pragma unroll
                for (int c16 = 0; c16 < 4; ++c16) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(box + swz<128>(r, (h & 1) * 4 + c16));
                    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float2 &x2 = w[4 * c16 + e];
                        if constexpr (OP == OP_SMAX_DOT) {
                            dot2 = fma2(x2, make_float2(lo_bf(wd[e]), hi_bf(wd[e])), dot2);
                        } else if constexpr (OP == OP_SMAX_BWD) {
                            x2 = mul2(sub2(make_float2(lo_bf(wd[e]), hi_bf(wd[e])), make_float2(rsum, rsum)), x2);
                        } else {
                            x2 = apply_op2<OP>(x2, make_float2(lo_bf(wd[e]), hi_bf(wd[e])));
                        }
                    }
                }
            }
            // this stage is no longer read by the epilogue
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&empty[s]);
                // last tile of this token block in my range: its outlier slot is free
                if (p.k && (tw.cc == tw.last_cc() || tile == t_hi - 1)) tc::mbar_arrive(&lqempty[(elq - 1) & 1]);
            }
            if constexpr (OP == OP_SMAX_DOT) {  // the partial goes out, no tile
                if (rv && ACT_DCHECK(cc < p.ncc && h < 4)) p.partials[trow * (4 * p.ncc) + 4 * cc + h] = __fadd_rn(dot2.x, dot2.y);
                continue;
            }

            if constexpr (OP != ACT_OP_DECODE) {  // 64 bytes of my row straight from registers
                if (rv && c_first < p.H && ACT_DCHECK(c_first + 32 <= p.ldo)) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + trow * p.ldo + c_first);
#pragma unroll
                    for (int c16 = 0; c16 < 4; ++c16) {
                        const int e = 4 * c16;
                        dst[c16] = make_uint4(pack_bf16x2(w[e].x, w[e].y), pack_bf16x2(w[e + 1].x, w[e + 1].y),
                                              pack_bf16x2(w[e + 2].x, w[e + 2].y), pack_bf16x2(w[e + 3].x, w[e + 3].y));
                    }
                }
                continue;
            }
            // decode: each warp stores its own 32 x 32 sub-tile; staging buffer ob of
            // the warp is free once the warp's store issued two tiles ago has read it
            uint8_t *stg = smem + L::OUT_OFF + ew * (2 * WST) + ob * WST;
            if (lane == 0) tc::bulk_wait_read<1>();
            __syncwarp();
#pragma unroll
            for (int c16 = 0; c16 < 4; ++c16) {
                const int e = 4 * c16;
                uint4 v;
                v.x = pack_bf16x2(w[e].x, w[e].y);
                v.y = pack_bf16x2(w[e + 1].x, w[e + 1].y);
                v.z = pack_bf16x2(w[e + 2].x, w[e + 2].y);
                v.w = pack_bf16x2(w[e + 3].x, w[e + 3].y);
                *reinterpret_cast<uint4 *>(stg + swz<64>(lane, c16)) = v;
            }
            tc::fence_proxy_async();
            __syncwarp();
            if (lane == 0 && ACT_DCHECK(cc * CH + 32 * h < p.H)) {
                tc::tma_store_3d(&tm_out, stg, cc * CH + 32 * h, tb * ROWS + 32 * q, sl_b);
                tc::bulk_commit();
            }
        }
        if (lane == 0) tc::bulk_wait<0>();
    }
    tc::tc_fence_before();
    __syncthreads();
    if (RK && warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, NT * CH);
    }
}

// softmax passes: where the partial dot products go / the row sums come from
struct SmaxArgs {
    float *partials = nullptr;
    const float *rowsum = nullptr;
    int causal = 0;
};

template <int BITS, int OP, bool WHT, int RK>
int launch_decode(const actcomp_cg_desc *d, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                  cudaStream_t stream, const SmaxArgs &sx = SmaxArgs()) {
    using L = DecLayout<BITS, OP, WHT, RK>;
    const int64_t T = d->tokens, H = d->channels, B = d->batch;
    CUtensorMap m_codes{}, m_y{}, m_out{};
    int st;
    const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const int64_t rowb = H * BITS / 8;
    if ((st = make_map_3d(&m_codes, d->codes, U8, 1, rowb, T, B, rowb, T * rowb, L::CODE_ROW, ROWS,
                          BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if (OP != ACT_OP_DECODE &&
        (st = make_map_3d(&m_y, y, BF, 2, H, T, B, ldy, T * ldy, 64, ROWS, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    // per-warp output boxes of the decode: 32 tokens x 32 channels (64-byte rows)
    if ((st = make_map_3d(&m_out, out, BF, 2, H, T, B, ldo, T * ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))) return st;
    DecParams p{};
    p.T = T;
    p.H = H;
    p.rank = d->rank;
    p.k = d->n_outlier;
    p.group = d->group;
    p.batch = d->batch;
    p.scales = d->scales;
    p.lr = d->lowrank;
    p.outliers = d->outliers;
    p.idx = d->outlier_idx;
    p.ntb = (int)((T + ROWS - 1) / ROWS);
    p.ncc = (int)((H + CH - 1) / CH);
    p.tri = is_smax<OP>() && sx.causal && T == H;
    p.ntiles = p.tri ? (int64_t)p.ntb * (p.ntb + 1) / 2 * B : (int64_t)p.ntb * p.ncc * B;
    p.n32 = (int)((H + 31) / 32);
    p.off_ot = L::OT_OFF;
    p.vtile = d->basis_tile;
    p.out = out;
    p.ldo = ldo;
    p.partials = sx.partials;
    p.rowsum = sx.rowsum;
    p.causal = sx.causal;
    p.off_ost = L::ost_off(p.n32);
    p.ostb = (ROWS * p.k * 2 + 15) & ~15;
    const int smem = L::total(p.n32, p.k);
    if (smem > 227 * 1024) return ACT_E_UNSUPPORTED;
    auto kern = cg_decode_tc_kernel<BITS, OP, WHT, RK>;
    ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int grid = (int)(p.ntiles < num_sms() ? p.ntiles : num_sms());
    p.tq = (int)(p.ntiles / grid);
    p.trem = (int)(p.ntiles % grid);
    kern<<<grid, L::THREADS, smem, stream>>>(m_codes, m_y, m_out, p);
    return launch_status();
}

template <int BITS, int OP>
int dispatch_rb(const actcomp_cg_desc *d, const uint16_t *y, int64_t ldy, uint16_t *out, int64_t ldo,
                cudaStream_t s, const SmaxArgs &sx = SmaxArgs()) {
    if (d->rank && (!d->basis_tile || !act::aligned(d->basis_tile, 16) || !act::aligned(d->lowrank, 16)))
        return ACT_E_UNSUPPORTED;
    const int rk = d->rank == 0 ? 0 : (d->rank <= 16 ? 16 : (d->rank <= 32 ? 32 : 64));
#define ACT_DTC(W)                                                                 \
    do {                                                                           \
        switch (rk) {                                                              \
            case 0: return launch_decode<BITS, OP, W, 0>(d, y, ldy, out, ldo, s, sx);   \
            case 16: return launch_decode<BITS, OP, W, 16>(d, y, ldy, out, ldo, s, sx); \
            case 32: return launch_decode<BITS, OP, W, 32>(d, y, ldy, out, ldo, s, sx); \
            default: return launch_decode<BITS, OP, W, 64>(d, y, ldy, out, ldo, s, sx); \
        }                                                                          \
    } while (0)
    if (d->wht) ACT_DTC(true);
    ACT_DTC(false);
#undef ACT_DTC
}

// row sums of the softmax partials, in a fixed order (deterministic)
// (causal: the partials of the tiles on or below the diagonal, the only ones written)
__global__ void smax_rowsum_kernel(const float *partials, int64_t rows, int per_row, int64_t T, int causal,
                                   float *rowsum) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    const float *pp = partials + i * per_row;
    const int n = causal ? 4 * (int)((i % T) / ROWS + 1) : per_row;
    float acc = 0.f;
    for (int j = 0; j < n; ++j) acc = __fadd_rn(acc, pp[j]);
    rowsum[i] = acc;
}

// dS = 0 above the diagonal blocks of causal probabilities (the tiles the
// second pass does not visit): columns [128 (t / 128 + 1), T) of every row,
// eight bf16 per 16-byte store where aligned
__global__ void smax_zero_upper_kernel(uint16_t *ds, int64_t ld, int64_t T, int64_t rows) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.y; i < rows; i += gridDim.y) {
        const int64_t c0 = ((i % T) / ROWS + 1) * ROWS;
        if (c0 >= T) continue;
        uint16_t *row = ds + i * ld;
        const int64_t n8 = (T - c0) / 8;
        for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n8; j += stride)
            reinterpret_cast<uint4 *>(row + c0)[j] = make_uint4(0u, 0u, 0u, 0u);
        for (int64_t c = c0 + 8 * n8 + blockIdx.x * blockDim.x + threadIdx.x; c < T; c += stride) row[c] = 0;
    }
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

// Softmax backward over compressed probabilities on the tensor-core decode:
// pass 1 forms P^ tile by tile and writes the partial dot products of each
// 32-column quarter with dP, a small kernel sums them per row in a fixed
// order, pass 2 forms P^ again and writes dS = (dP - rowsum) * P^.
size_t act_cg_softmax_tc_workspace(const actcomp_cg_desc *d) {
    const int64_t rows = d->batch * d->tokens, ncc = (d->channels + 127) / 128;
    return (size_t)(rows * (4 * ncc + 1) * 4);
}

int act_cg_softmax_tc(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld, int causal,
                      void *workspace, cudaStream_t s) {
    using namespace act::cgtc;
    if (d->tokens == 0) return ACT_OK;
    const int64_t rows = d->batch * d->tokens, ncc = (d->channels + 127) / 128;
    SmaxArgs sx;
    sx.partials = static_cast<float *>(workspace);
    float *rowsum = sx.partials + rows * 4 * ncc;
    sx.rowsum = rowsum;
    sx.causal = causal;
    int st = d->bits == 4 ? dispatch_rb<4, OP_SMAX_DOT>(d, dp, ld, ds, ld, s, sx)
                          : dispatch_rb<8, OP_SMAX_DOT>(d, dp, ld, ds, ld, s, sx);
    if (st) return st;
    const int tri = causal && d->tokens == d->channels;
    smax_rowsum_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(sx.partials, rows, (int)(4 * ncc), d->tokens,
                                                                      tri, rowsum);
    if ((st = act::launch_status())) return st;
    if (tri) {
        smax_zero_upper_kernel<<<dim3(2, (unsigned)(rows < 65535 ? rows : 65535)), 256, 0, s>>>(ds, ld, d->tokens, rows);
        if ((st = act::launch_status())) return st;
    }
    return d->bits == 4 ? dispatch_rb<4, OP_SMAX_BWD>(d, dp, ld, ds, ld, s, sx)
                        : dispatch_rb<8, OP_SMAX_BWD>(d, dp, ld, ds, ld, s, sx);
}
