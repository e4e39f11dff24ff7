// cg_dw_fused.cu -- weight gradient dW = X^T dY read from the compressed form
// inside the GEMM (triton_matmul_decompress, extraction_fuse_matmul.py:224,
// whose producer reconstructs each X tile as it loads it, :151-221).
//
// The reconstruction X = bf16(L V^T + R) is not rebuilt per tile: the GEMM is
// split along the format,
//   dW = Q^T dY  +  V (L^T dY)          (rows of the outlier channels: O^T dY)
// with Q = bf16((u - 2^(b-1)) * s) the dequantised residual, zero in the
// outlier channels.  Only Q needs the codes, and it is made inside the GEMM's
// producer; the low-rank term is a second, 3r-deep K segment of the same
// accumulator ([V | V | V] times the three exact bf16 pieces of the float32
// L^T dY), and the k outlier rows are a skinny GEMM written over their rows.
// Against the GEMM of the bf16 reconstruction this moves dW by the bf16
// rounding of the residual alone instead of that of L V^T + R (4.4e-4
// relative at config-4-like data; both are 4.2e-3 from the GEMM of the
// uncompressed X).
//
// Kernel dq_gemm_kernel: one CTA a 256 x 256 tile of dW (two M = 128 TMEM
// accumulators sharing each dY tile), grouped raster as gemm_kernel.
//   warp 0      TMA: dY tiles (and, in the second segment, [V|V|V] and the
//               pieces of L^T dY) into a 3-stage ring;
//   warp 1      TMEM allocation and tcgen05.mma (A MN-major in the first
//               segment, K-major in the second);
//   warps 2-5   epilogue (TMEM -> dW rows);
//   warps 6-13  dequantisation: per 64-token k-block each thread turns one
//               token's 64 channels of codes (and their group scales) into
//               one 128-byte row of the MN-major, 128-byte-swizzled A tile.
//               int4 codes come by TMA into a 3-slot ring of their own (one
//               64 x 128-byte swizzled box a k-block, with its own arrival
//               barrier); int8 codes and the scales are loaded by the
//               threads one k-block ahead.  The codes of a 256-channel slab (2 MB at 16384
//               tokens, int4) are read by every CTA of that M tile, mostly
//               from L2.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {
int validate_desc(const actcomp_cg_desc *d);
int gemm_launch(const actcomp_gemm_args *g, cudaStream_t stream);

namespace dwf {

constexpr int BM = 128, BN = 256, MA = 2, BK = 64;
constexpr int A_BYTES = BM * BK * 2;           // 16 KB per accumulator half
constexpr int B_BYTES = BN * BK * 2;           // 32 KB
constexpr int STAGE = MA * A_BYTES + B_BYTES;  // 64 KB
constexpr int STAGES = 3;
constexpr int DQ_WARPS = 8;
constexpr int THREADS = (6 + DQ_WARPS) * 32;
constexpr int CODE_BYTES = BK * 128;            // int4 codes of a k-block: 64 tokens x 256 channels
// int4: the codes come by TMA into their own 3-slot ring (128-byte swizzle)
template <int BITS>
constexpr int smem_bytes() { return STAGES * STAGE + (BITS == 4 ? STAGES * CODE_BYTES : 0) + 1024 + 256; }

struct Params {
    int64_t T, H, N;
    int kb1, kb2;           // k-blocks of the dequantised segment and of the low-rank segment
    int m_tiles, n_tiles;
    int group, k;
    const uint8_t *codes;   // T x H*BITS/8
    const float *scales;    // T x H/group
    const int32_t *idx;     // k outlier channels
    void *C;
    int64_t ldc;
};

// one token's 64 channels of codes and their scales
template <int BITS>
struct Row {
    uint4 v[BITS / 2];  // 32 (int4) or 64 (int8) bytes
    float s0, s1;       // scales of channels 0-31 and 32-63
};

template <int BITS>
__device__ __forceinline__ void load_row(const Params &p, int64_t t, int64_t c0, Row<BITS> &q) {
    if (t < p.T && c0 < p.H) {
        if constexpr (BITS == 8) {  // int4 codes arrive by TMA instead
            const uint4 *src = reinterpret_cast<const uint4 *>(p.codes + t * (p.H * BITS / 8) + c0 * BITS / 8);
#pragma unroll
            for (int i = 0; i < BITS / 2; ++i) q.v[i] = __ldg(src + i);
        }
        const int ngr = (int)(p.H / p.group);
        const int gshift = 31 - __clz(p.group);
        const float *sp = p.scales + t * ngr;
        q.s0 = __ldg(sp + (c0 >> gshift));
        q.s1 = __ldg(sp + ((c0 + 32) >> gshift));
    } else {
#pragma unroll
        for (int i = 0; i < BITS / 2; ++i) q.v[i] = make_uint4(0, 0, 0, 0);
        q.s0 = q.s1 = 0.f;  // rows beyond T and channels beyond H contribute zero
    }
}

template <typename T>
__device__ __forceinline__ T cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <int BITS, typename TOut>
__global__ void __launch_bounds__(THREADS, 1)
    dq_gemm_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmQ, Params p) {
    constexpr bool TMAC = BITS == 4;  // codes staged by TMA
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *cring = smem + STAGES * STAGE;  // int4 codes, one slot a stage
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE + (TMAC ? STAGES * CODE_BYTES : 0));
    uint64_t *empty = full + STAGES;
    uint64_t *cfull = empty + STAGES;        // [STAGES] a k-block's codes arrived
    uint64_t *acc_full = cfull + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    int m_t, n_t;  // grouped raster: up to 16 M tiles a group, M fastest
    {
        const int nm = p.m_tiles, nn = p.n_tiles, id = blockIdx.x;
        const int gsz = 16 * nn, grp = id / gsz, first = grp * 16;
        const int gm = nm - first < 16 ? nm - first : 16;
        const int in = id - grp * gsz;
        m_t = first + in % gm;
        n_t = in / gm;
    }
    const int m0 = m_t * BM * MA, n0 = n_t * BN;
    const int kblocks = p.kb1 + p.kb2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1 + DQ_WARPS);  // the TMA producer and every dequantising warp
            tc::mbar_init(&empty[s], 1);
            tc::mbar_init(&cfull[s], 1);
        }
        tc::mbar_init(acc_full, 1);
        *abort = 0;
        tc::fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, BN * MA);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tc::prefetch_tmap(&tmB);
            for (int kb = 0; kb < kblocks; ++kb) {
                const int s = kb % STAGES;
                if (!tc::mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1, abort)) break;
                uint8_t *a = smem + s * STAGE;
                uint8_t *b = a + MA * A_BYTES;
                if (kb < p.kb1) {
                    if constexpr (TMAC) {
                        tc::mbar_arrive_expect_tx(&cfull[s], CODE_BYTES);
                        tc::tma_load_3d(cring + s * CODE_BYTES, &tmQ, &cfull[s], m0 / 2, kb * BK, 0);
                    }
                    tc::mbar_arrive_expect_tx(&full[s], B_BYTES);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tc::tma_load_3d(b + j * 8192, &tmB, &full[s], n0 + 64 * j, kb * BK, 0);
                } else {
                    const int k0 = (kb - p.kb1) * BK;
                    tc::mbar_arrive_expect_tx(&full[s], STAGE);
#pragma unroll
                    for (int h = 0; h < MA; ++h) tc::tma_load_3d(a + h * A_BYTES, &tmA2, &full[s], k0, m0 + BM * h, 0);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tc::tma_load_3d(b + j * 8192, &tmB2, &full[s], n0 + 64 * j, k0, 0);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            constexpr uint32_t idesc_q = tc::idesc_f16(BM, BN, true, true, true);    // A MN-major (dequantised)
            constexpr uint32_t idesc_v = tc::idesc_f16(BM, BN, true, false, true);   // A K-major ([V|V|V])
            for (int kb = 0; kb < kblocks; ++kb) {
                const int s = kb % STAGES;
                if (!tc::mbar_wait(&full[s], (kb / STAGES) & 1, abort)) break;
                tc::tc_fence_after();
                uint8_t *a = smem + s * STAGE;
                uint8_t *b = a + MA * A_BYTES;
                const bool q = kb < p.kb1;
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t bd = tc::smem_desc(b + kk * 2048, 8192, 1024, tc::SW_128B);
#pragma unroll
                    for (int h = 0; h < MA; ++h) {
                        uint8_t *ah = a + h * A_BYTES;
                        const uint64_t ad = q ? tc::smem_desc(ah + kk * 2048, 8192, 1024, tc::SW_128B)
                                              : tc::smem_desc(ah + kk * 32, 16, 1024, tc::SW_128B);
                        tc::mma_f16(tmem + h * BN, ad, bd, q ? idesc_q : idesc_v, (kb | kk) != 0);
                    }
                }
                tc::mma_commit(&empty[s]);
            }
            tc::mma_commit(acc_full);
        }
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const bool ok = tc::mbar_wait(acc_full, 0, abort);
        tc::tc_fence_after();
        if (ok) {
            TOut *C = reinterpret_cast<TOut *>(p.C);
            const bool vec = (p.ldc * (int64_t)sizeof(TOut)) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.C) % 16) == 0;
#pragma unroll 1
            for (int hc = 0; hc < MA * (BN / 32); ++hc) {
                const int h = hc / (BN / 32), c = hc % (BN / 32);
                const int64_t row = m0 + BM * h + q * 32 + lane;
                uint32_t r[32];
                tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + h * BN + c * 32, r);
                tc::tmem_ld_wait();
                const int64_t col = n0 + c * 32;
                if (row >= p.H || col >= p.N) continue;
                TOut *dst = C + row * p.ldc + col;
                const int valid = p.N - col < 32 ? (int)(p.N - col) : 32;
                if (valid == 32 && vec) {
                    if constexpr (sizeof(TOut) == 4) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            reinterpret_cast<float4 *>(dst)[i] =
                                make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                            __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            uint32_t w[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                w[j] = pack_bf16x2(__uint_as_float(r[8 * i + 2 * j]), __uint_as_float(r[8 * i + 2 * j + 1]));
                            reinterpret_cast<uint4 *>(dst)[i] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (i < valid) dst[i] = cvt_out<TOut>(__uint_as_float(r[i]));
                }
            }
        }
    } else {
        // ------------------------------------------------------------ dequantisation
        const int dt = threadIdx.x - 6 * 32;  // 0 .. 255
        const int kk = dt >> 2;                // token row of the k-block
        const int at = dt & 3;                 // 64-channel atom of the 256-channel tile
        const int64_t c0 = m0 + 64 * at;
        uint64_t om = 0;                       // outlier channels among these 64
        for (int j = 0; j < p.k; ++j) {
            const int64_t c = (int64_t)__ldg(p.idx + j) - c0;
            if (c >= 0 && c < 64) om |= 1ull << c;
        }
        // where this thread's 128-byte row sits in a stage (MN-major, 128-byte swizzle:
        // 16-byte chunk j of row kk at chunk j ^ (kk & 7))
        const int dst_off = (at >> 1) * A_BYTES + (at & 1) * 8192 + kk * 128;
        Row<BITS> cur, nxt;
        load_row<BITS>(p, (int64_t)kk, c0, cur);
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % STAGES;
            if (kb + 1 < p.kb1) load_row<BITS>(p, (int64_t)(kb + 1) * BK + kk, c0, nxt);
            if (!tc::mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1, abort)) break;
            if (TMAC && kb < p.kb1 && !tc::mbar_wait(&cfull[s], (kb / STAGES) & 1, abort)) break;
            if (kb < p.kb1) {
                uint8_t *row = smem + s * STAGE + dst_off;
                if constexpr (TMAC) {  // this row's 32 code bytes: chunks 2 at, 2 at + 1 of the swizzled slot
                    const uint8_t *cr = cring + s * CODE_BYTES + kk * 128;
                    cur.v[0] = *reinterpret_cast<const uint4 *>(cr + (((2 * at) ^ (kk & 7)) << 4));
                    cur.v[1] = *reinterpret_cast<const uint4 *>(cr + (((2 * at + 1) ^ (kk & 7)) << 4));
                }
                uint32_t wd[BITS * 2];  // the row's code words, by constant index (no local copy)
#pragma unroll
                for (int i = 0; i < BITS / 2; ++i) {
                    wd[4 * i] = cur.v[i].x;
                    wd[4 * i + 1] = cur.v[i].y;
                    wd[4 * i + 2] = cur.v[i].z;
                    wd[4 * i + 3] = cur.v[i].w;
                }
                // code u -> the float 2^23 + u by one byte permute against 0x4B000000,
                // then (u - 2^(b-1)) exactly and one rounded product with the scale,
                // two channels at a time
                constexpr uint32_t K4B = 0x4B000000u;
                constexpr float UOFF = 8388608.0f + (float)(1 << (BITS - 1));
                const float2 uoff2 = make_float2(UOFF, UOFF);
#pragma unroll
                for (int j = 0; j < 8; ++j) {  // channels 8j .. 8j+7
                    const float sj = j < 4 ? cur.s0 : cur.s1;
                    const float2 s2 = make_float2(sj, sj);
                    uint32_t o[4];
                    if constexpr (BITS == 4) {  // channel 2i in the low nibble of byte i
                        const uint32_t ev = wd[j] & 0x0F0F0F0Fu, od = (wd[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = make_float2(__uint_as_float(__byte_perm(ev, K4B, 0x7540u | e)),
                                                         __uint_as_float(__byte_perm(od, K4B, 0x7540u | e)));
                            const float2 w = mul2(sub2(f, uoff2), s2);
                            o[e] = pack_bf16x2(w.x, w.y);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t w2 = wd[2 * j + (e >> 1)];
                            const uint32_t b0 = 2 * (e & 1);
                            const float2 f = make_float2(__uint_as_float(__byte_perm(w2, K4B, 0x7540u | b0)),
                                                         __uint_as_float(__byte_perm(w2, K4B, 0x7540u | (b0 + 1))));
                            const float2 w = mul2(sub2(f, uoff2), s2);
                            o[e] = pack_bf16x2(w.x, w.y);
                        }
                    }
                    const uint32_t m8 = (uint32_t)(om >> (8 * j)) & 0xffu;
                    if (m8) {  // outlier channels among these eight: zero
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            o[e] &= ((m8 >> (2 * e)) & 1u ? 0xffff0000u : 0xffffffffu) &
                                    ((m8 >> (2 * e + 1)) & 1u ? 0x0000ffffu : 0xffffffffu);
                    }
                    *reinterpret_cast<uint4 *>(row + ((j ^ (kk & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                tc::fence_proxy_async();
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&full[s]);
            cur = nxt;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, BN * MA);
    }
}

// L (T x r float32) -> its three exact bf16 pieces side by side, T x 3r
__global__ void l_pieces_kernel(const float *L, int64_t T, int r, uint16_t *P3) {
    const int64_t n = T * r;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / r;
        const int j = (int)(e - t * r);
        float hi, mid, lo;
        split3_bf16(L[e], hi, mid, lo);
        uint16_t *row = P3 + t * 3 * r;
        row[j] = f2bf(hi);
        row[r + j] = f2bf(mid);
        row[2 * r + j] = f2bf(lo);
    }
}
// G (3r x N float32: hi^T dY, mid^T dY, lo^T dY) -> L^T dY = (hi + mid) + lo
// parts, split again into three exact bf16 pieces, 3r x N
__global__ void sum_split_kernel(const float *G, int r, int64_t N, uint16_t *B2) {
    const int64_t n = (int64_t)r * N;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const float v = __fadd_rn(__fadd_rn(G[e], G[n + e]), G[2 * n + e]);
        float hi, mid, lo;
        split3_bf16(v, hi, mid, lo);
        B2[e] = f2bf(hi);
        B2[n + e] = f2bf(mid);
        B2[2 * n + e] = f2bf(lo);
    }
}
// V (H x r bf16) -> [V | V | V], H x 3r
__global__ void v3_kernel(const uint16_t *V, int64_t H, int r, uint16_t *V3) {
    const int64_t n = H * r;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = e / r;
        const int j = (int)(e - c * r);
        const uint16_t v = V[e];
        V3[c * 3 * r + j] = v;
        V3[c * 3 * r + r + j] = v;
        V3[c * 3 * r + 2 * r + j] = v;
    }
}
// rows idx[i] of C = R[i] (k x N float32), over what the GEMM wrote there
template <typename TOut>
__global__ void scatter_rows_kernel(const float *R, const int32_t *idx, int k, int64_t N, TOut *C, int64_t ldc) {
    const int64_t n = (int64_t)k * N;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e / N);
        const int64_t c = e - (int64_t)i * N;
        C[(int64_t)idx[i] * ldc + c] = cvt_out<TOut>(R[e]);
    }
}

struct Ws {  // workspace carve-up (each part 256-byte aligned)
    size_t p3, g1, b2, v3, orow, total;
};
static Ws carve(int64_t T, int64_t H, int64_t N, int r, int k) {
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    Ws w{};
    size_t o = 0;
    w.p3 = o;   o += r ? up((size_t)T * 3 * r * 2) : 0;
    w.g1 = o;   o += r ? up((size_t)3 * r * N * 4) : 0;
    w.b2 = o;   o += r ? up((size_t)3 * r * N * 2) : 0;
    w.v3 = o;   o += r ? up((size_t)H * 3 * r * 2) : 0;
    w.orow = o; o += k ? up((size_t)k * N * 4) : 0;
    w.total = o;
    return w;
}

static int grid_for(int64_t n) {
    const int64_t b = (n + 255) / 256, cap = (int64_t)num_sms() * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace dwf
}  // namespace act

extern "C" size_t actcomp_cg_dw_fused_workspace(const actcomp_cg_desc *d, int64_t N) {
    if (!d || d->tokens <= 0 || d->channels <= 0 || N <= 0) return 0;
    return act::dwf::carve(d->tokens, d->channels, N, d->rank, d->n_outlier).total;
}

extern "C" int actcomp_cg_dw_fused(const actcomp_cg_desc *d, const uint16_t *dy, int64_t N, int64_t lddy, void *dw,
                                   int32_t dw_dtype, int64_t lddw, void *workspace, size_t workspace_bytes,
                                   void *stream) {
    using namespace act;
    using namespace act::dwf;
    int st = validate_desc(d);
    if (st) return st;
    ACT_CHECK(dy && dw && N > 0 && lddy >= N && lddw >= N, ACT_E_INVALID);
    ACT_CHECK(dw_dtype == 0 || dw_dtype == 1, ACT_E_INVALID);
    ACT_CHECK(d->batch == 1 && !d->wht, ACT_E_UNSUPPORTED);  // the rotated residual is not Q in the channel basis
    const int64_t T = d->tokens, H = d->channels;
    const int r = d->rank, k = d->n_outlier;
    if (T == 0) return ACT_OK;
    ACT_CHECK(H % 64 == 0 && H >= 256 && T >= BK && T <= INT32_MAX && H <= INT32_MAX && N <= INT32_MAX,
              ACT_E_UNSUPPORTED);  // at least one whole TMA box of codes
    ACT_CHECK(N % 8 == 0 && lddy % 8 == 0 && aligned(dy, 16) && aligned(d->codes, 16), ACT_E_ALIGN);
    if (k) {  // the outliers enter a GEMM as a T x k operand: 16-byte rows
        ACT_CHECK(d->outliers && d->outlier_idx, ACT_E_INVALID);
        ACT_CHECK(k % 8 == 0 && aligned(d->outliers, 16), ACT_E_UNSUPPORTED);
    }
    if (r) ACT_CHECK(d->lowrank && d->basis, ACT_E_INVALID);
    const Ws w = carve(T, H, N, r, k);
    ACT_CHECK(w.total == 0 || (workspace && workspace_bytes >= w.total), ACT_E_WORKSPACE);
    ACT_CHECK(aligned(workspace, 256), ACT_E_ALIGN);
    cudaStream_t s = as_stream(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    uint16_t *P3 = reinterpret_cast<uint16_t *>(ws + w.p3), *B2 = reinterpret_cast<uint16_t *>(ws + w.b2);
    uint16_t *V3 = reinterpret_cast<uint16_t *>(ws + w.v3);
    float *G1 = reinterpret_cast<float *>(ws + w.g1), *OR = reinterpret_cast<float *>(ws + w.orow);

    // low-rank segment: B2 = pieces of L^T dY (3r x N), A2 = [V | V | V] (H x 3r)
    if (r) {
        l_pieces_kernel<<<grid_for(T * r), 256, 0, s>>>(d->lowrank, T, r, P3);
        if ((st = launch_status())) return st;
        actcomp_gemm_args g{};
        g.M = 3 * r; g.N = N; g.K = T; g.batch = 1; g.in_dtype = 0; g.c_dtype = 0;
        g.a_kmajor = 0; g.b_kmajor = 0;  // P3 is T x 3r (A^T given), dy is T x N
        g.A = P3; g.lda = 3 * r; g.B = dy; g.ldb = lddy; g.C = G1; g.ldc = N;
        if ((st = gemm_launch(&g, s))) return st;
        sum_split_kernel<<<grid_for((int64_t)r * N), 256, 0, s>>>(G1, r, N, B2);
        if ((st = launch_status())) return st;
        v3_kernel<<<grid_for(H * r), 256, 0, s>>>(d->basis, H, r, V3);
        if ((st = launch_status())) return st;
    }
    // outlier rows: O^T dY (k x N)
    if (k) {
        actcomp_gemm_args g{};
        g.M = k; g.N = N; g.K = T; g.batch = 1; g.in_dtype = 0; g.c_dtype = 0;
        g.a_kmajor = 0; g.b_kmajor = 0;
        g.A = d->outliers; g.lda = k; g.B = dy; g.ldb = lddy; g.C = OR; g.ldc = N;
        if ((st = gemm_launch(&g, s))) return st;
    }
    // the dequantising GEMM: Q^T dY (+ [V|V|V] B2)
    CUtensorMap tmB{}, tmA2{}, tmB2{};
    if ((st = make_map_3d(&tmB, dy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, T, 1, lddy, 0, 64, 64,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    tmA2 = tmB2 = tmB;  // copies never read without a low-rank segment
    CUtensorMap tmQ = tmB;  // int4 codes: T rows of H/2 bytes, 128 x 64 boxes
    if (d->bits == 4 && (st = make_map_3d(&tmQ, d->codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, H / 2, T, 1, H / 2, 0,
                                          128, 64, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if (r) {
        if ((st = make_map_3d(&tmA2, V3, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * r, H, 1, 3 * r, 0, 64, 128,
                              CU_TENSOR_MAP_SWIZZLE_128B)))
            return st;
        if ((st = make_map_3d(&tmB2, B2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, 3 * r, 1, N, 0, 64, 64,
                              CU_TENSOR_MAP_SWIZZLE_128B)))
            return st;
    }
    Params p{};
    p.T = T; p.H = H; p.N = N;
    p.kb1 = (int)((T + BK - 1) / BK);
    p.kb2 = r ? (3 * r + BK - 1) / BK : 0;
    p.m_tiles = (int)((H + BM * MA - 1) / (BM * MA));
    p.n_tiles = (int)((N + BN - 1) / BN);
    p.group = d->group; p.k = k;
    p.codes = d->codes; p.scales = d->scales; p.idx = d->outlier_idx;
    p.C = dw; p.ldc = lddw;
    const dim3 grid((unsigned)(p.m_tiles * p.n_tiles));
    auto launch = [&](auto kern, int smem) -> int {
        ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        kern<<<grid, THREADS, smem, s>>>(tmB, tmA2, tmB2, tmQ, p);
        return launch_status();
    };
    if (d->bits == 4)
        st = dw_dtype == 0 ? launch(dq_gemm_kernel<4, float>, smem_bytes<4>())
                           : launch(dq_gemm_kernel<4, __nv_bfloat16>, smem_bytes<4>());
    else
        st = dw_dtype == 0 ? launch(dq_gemm_kernel<8, float>, smem_bytes<8>())
                           : launch(dq_gemm_kernel<8, __nv_bfloat16>, smem_bytes<8>());
    if (st) return st;
    if (k) {
        if (dw_dtype == 0)
            scatter_rows_kernel<float><<<grid_for((int64_t)k * N), 256, 0, s>>>(OR, d->outlier_idx, k, N,
                                                                             static_cast<float *>(dw), lddw);
        else
            scatter_rows_kernel<__nv_bfloat16><<<grid_for((int64_t)k * N), 256, 0, s>>>(
                OR, d->outlier_idx, k, N, static_cast<__nv_bfloat16 *>(dw), lddw);
        if ((st = launch_status())) return st;
    }
    return ACT_OK;
}
