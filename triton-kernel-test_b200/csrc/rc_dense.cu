// rc_dense.cu -- reference-compatible encode/decode (the reference's own data
// layout) and the dense helper kernels (uncompressed consumers, outlier
// extraction, error statistics).
//
// Reference-compatible arithmetic, per element (defaults = Triton kernel
// semantics, flags = PyTorch-twin behaviour; see include/actcomp.h):
//   d   = sum_k l[m,k] r[k,n] as sequential binary32 FMAs from k = 0
//   res = bf16(x - d)                                  (TWIN_LOWRANK: bf16(x - bf16(d)))
//   o   = |res| > thr ? res : 0;  xr = res - o
//   t   = bf16(xr / s[0 or b, n]);  q = round(t) (half away; HALF_EVEN: rint)
//   q   = clamp(q, -2^(b-1), 2^(b-1)-1) + 2^(b-1), packed per 32-column block
// and for decode: w = bf16((u - off) * s); a = bf16(w + o); x = bf16(a + d).
// This is low_rank_extraction_fuse_compression_quantization.py:63-115 and
// low_rank_extraction_fuse_decompression_dequantization.py:76-113 with the
// scratch round trips (K2's o-buffer reuse, K3's uint8 x_temp) removed.
#include "common.cuh"

namespace act {

__device__ __forceinline__ void rc_pack_pos(int64_t n, int64_t N, int bits, int flags, int64_t &byte, int &shift) {
    const int epp = 8 / bits;
    if (flags & ACT_RC_ROW_PACK) {
        const int64_t w = N / epp;
        byte = n % w;
        shift = (int)(n / w) * bits;
    } else {
        const int64_t blk = n >> 5, within = n & 31, w = 32 / epp;
        byte = blk * w + within % w;
        shift = (int)(within / w) * bits;
    }
}

__device__ __forceinline__ float rc_dot(const uint16_t *l, const uint16_t *r, int64_t m, int64_t n, int K,
                                        int64_t N) {
    float d = 0.f;
    for (int k = 0; k < K; ++k) d = __fmaf_rn(bf2f(l[m * K + k]), bf2f(r[(int64_t)k * N + n]), d);
    return d;
}

// One thread per packed byte (all epp elements that share it).
__global__ void rc_encode_kernel(actcomp_rc_args a) {
    const int epp = 8 / a.bits;
    const int64_t W = a.N / epp;  // bytes per row
    const int64_t total = a.B * a.M * W;
    const int lo = -(1 << (a.bits - 1)), hi = (1 << (a.bits - 1)) - 1, off = 1 << (a.bits - 1);
    const float thr = (a.flags & ACT_RC_OUTLIER_BF16) ? rne_bf(a.outlier) : a.outlier;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = g % W, bm = g / W, m = bm % a.M, b = bm / a.M;
        const int64_t srow = (a.flags & ACT_RC_SCALE_BATCH) ? (a.s_rows > 1 ? b : 0) : 0;
        uint32_t byte = 0;
        for (int i = 0; i < epp; ++i) {
            int64_t n;
            if (a.flags & ACT_RC_ROW_PACK) n = w + (int64_t)i * W;
            else n = (w / (32 / epp)) * 32 + (w % (32 / epp)) + (int64_t)i * (32 / epp);
            const float xv = bf2f(a.x[b * a.sxb + m * a.sxm + n]);
            const float d = rc_dot(a.l, a.r, m, n, a.K, a.N);
            const float res = (a.flags & ACT_RC_TWIN_LOWRANK) ? rne_bf(__fsub_rn(xv, rne_bf(d))) : rne_bf(__fsub_rn(xv, d));
            const float ov = fabsf(res) > thr ? res : 0.f;
            a.o[(b * a.M + m) * a.N + n] = f2bf(ov);
            const float xr = __fsub_rn(res, ov);
            const float t = rne_bf(__fdiv_rn(xr, bf2f(a.s[srow * a.N + n])));
            float rq = (a.flags & ACT_RC_HALF_EVEN) ? rintf(t) : roundf(t);
            rq = fminf(fmaxf(rq, (float)lo), (float)hi);
            byte |= (uint32_t)((int)rq + off) << (i * a.bits);
        }
        a.q[bm * W + w] = (uint8_t)byte;
    }
}

// One thread per element; op selects decode or a fused consumer with a.x as
// its second operand.
template <int OP>
__global__ void rc_decode_kernel(actcomp_rc_args a) {
    const int64_t total = a.B * a.M * a.N;
    const int off = 1 << (a.bits - 1);
    const uint32_t mask = (1u << a.bits) - 1u;
    const int64_t W = a.N * a.bits / 8;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = g % a.N, bm = g / a.N, m = bm % a.M, b = bm / a.M;
        int64_t byte;
        int shift;
        rc_pack_pos(n, a.N, a.bits, a.flags, byte, shift);
        const uint32_t u = ((uint32_t)a.q[bm * W + byte] >> shift) & mask;
        const int64_t srow = (a.flags & ACT_RC_SCALE_BATCH) ? (a.s_rows > 1 ? b : 0) : 0;
        const float w = rne_bf(__fmul_rn(__int2float_rn((int)u - off), bf2f(a.s[srow * a.N + n])));
        const float av = a.o ? rne_bf(__fadd_rn(w, bf2f(a.o[g]))) : w;
        const float d = rc_dot(a.l, a.r, m, n, a.K, a.N);
        const float v = (a.flags & ACT_RC_TWIN_LOWRANK) ? rne_bf(__fadd_rn(av, rne_bf(d))) : rne_bf(__fadd_rn(av, d));
        if constexpr (OP == ACT_OP_DECODE) {
            a.out[g] = f2bf(v);
        } else {
            const float y = bf2f(a.x[b * a.sxb + m * a.sxm + n]);
            a.out[g] = f2bf(apply_op<OP>(v, y));
        }
    }
}

// low_rank_addition (low_rank_extraction_speed.py:12-110): out = bf16(x + l@r),
// the dot as sequential binary32 FMAs.
__global__ void rc_lowrank_add_kernel(actcomp_rc_args a) {
    const int64_t total = a.B * a.M * a.N;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = g % a.N, bm = g / a.N, m = bm % a.M, b = bm / a.M;
        const float d = rc_dot(a.l, a.r, m, n, a.K, a.N);
        a.out[g] = f2bf(__fadd_rn(bf2f(a.x[b * a.sxb + m * a.sxm + n]), d));
    }
}

// ---------------------------------------------------------------- tiled rc kernels
// A CTA takes a tile of RCT = 256 columns (8 packing blocks) of one batch and
// RCR rows of it, in passes of RPP rows.  Dynamic shared memory holds r[:, tile]
// reordered so that the epp values one packed byte needs for each k are
// contiguous (one vector load per k), the pass's rows of l, and the pass's
// coalesced tile: x in and o out of the encode (in place), o in and the output
// out of the decode (in place), plus y for the fused consumers.  A thread owns
// one packed byte in each of NRW rows of the pass: the epp elements of its
// block that share the byte.  Per element the arithmetic (sequential binary32
// FMAs over k from 0, the roundings) is the per-element kernels' above, bit
// for bit.
constexpr int RCT = 256, RCR = 128, NRW = 4;

template <int BITS>
struct RcTile {
    static constexpr int EPP = 8 / BITS;     // elements per packed byte
    static constexpr int BPB = 32 / EPP;     // bytes per 32-column block
    static constexpr int TPR = RCT / EPP;    // threads (bytes) per row of the tile
    static constexpr int RP = 256 / TPR;     // rows one sweep of the CTA covers
    static constexpr int RPP = RP * NRW;     // rows per pass
    // column of element i of tile byte w
    __device__ static int col(int w, int i) { return (w / BPB) * 32 + (w % BPB) + i * BPB; }
    // dynamic shared memory: r_s [K][RCT] floats, l_s [RPP][K] bf16, t_s [RPP][RCT] bf16, y_s [RPP][RCT] bf16,
    // s_s [RCT] floats
    __host__ __device__ static int off_l(int K) { return K * RCT * 4; }
    __host__ __device__ static int off_t(int K) { return (off_l(K) + RPP * K * 2 + 15) & ~15; }
    __host__ __device__ static int off_y(int K) { return off_t(K) + RPP * RCT * 2; }
    __host__ __device__ static int off_s(int K, bool y) { return off_y(K) + (y ? RPP * RCT * 2 : 0); }
    __host__ __device__ static int bytes(int K, bool y) { return off_s(K, y) + RCT * 4; }
};

// the EPP values (float, from bf16) one thread needs for one k, in vector loads
template <int EPP>
__device__ __forceinline__ void load_epp(const float *p, float (&v)[EPP]) {
    if constexpr (EPP == 8) {
        const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else if constexpr (EPP == 4) {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    } else if constexpr (EPP == 2) {
        const float2 a = *reinterpret_cast<const float2 *>(p);
        v[0] = a.x, v[1] = a.y;
    } else {
        v[0] = *p;
    }
}

// d[j][i] = sum_k l[row j][k] r[k][col(w, i)] for the thread's NRW rows, each
// a sequential binary32 FMA chain from k = 0 (the r values of one k serve all
// NRW rows)
template <int EPP, int RP>
__device__ __forceinline__ void rc_dots(const float *r_s, const uint16_t *l_s, int K, int rp0, int w,
                                        float (&d)[NRW][EPP]) {
#pragma unroll
    for (int j = 0; j < NRW; ++j)
#pragma unroll
        for (int i = 0; i < EPP; ++i) d[j][i] = 0.f;
    for (int k = 0; k < K; ++k) {
        float rv[EPP];
        load_epp<EPP>(r_s + k * RCT + w * EPP, rv);
#pragma unroll
        for (int j = 0; j < NRW; ++j) {
            const float lv = bf2f(l_s[(rp0 + j * RP) * K + k]);
#pragma unroll
            for (int i = 0; i < EPP; ++i) d[j][i] = __fmaf_rn(lv, rv[i], d[j][i]);
        }
    }
}

// r_s[k][w * EPP + i] = r[k][n0 + col(w, i)]; the scale row of the tile
template <int BITS>
__device__ __forceinline__ void rc_stage_tile(const actcomp_rc_args &a, float *r_s, float *s_s, int64_t n0,
                                              int64_t srow) {
    using R = RcTile<BITS>;
    for (int e = threadIdx.x; e < a.K * RCT; e += 256) {
        const int k = e / RCT, c = e - k * RCT, w = c / R::EPP, i = c - w * R::EPP;
        r_s[e] = bf2f(a.r[(int64_t)k * a.N + n0 + R::col(w, i)]);
    }
    for (int c = threadIdx.x; c < RCT; c += 256) s_s[c] = bf2f(a.s[srow * a.N + n0 + c]);
}

// rows [m0, m0 + RPP) of a (rows x ld) bf16 matrix, columns n0 .. n0 + RCT, into t (16-byte chunks)
__device__ __forceinline__ void rc_load_rows(uint16_t *t, const uint16_t *src, int64_t ld, int64_t m0, int64_t m_hi,
                                             int rpp, int64_t n0) {
    for (int e = threadIdx.x; e < rpp * (RCT / 8); e += 256) {
        const int r = e / (RCT / 8), c8 = e - r * (RCT / 8);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (src && m0 + r < m_hi) v = *reinterpret_cast<const uint4 *>(src + (m0 + r) * ld + n0 + 8 * c8);
        *reinterpret_cast<uint4 *>(t + r * RCT + 8 * c8) = v;
    }
}
__device__ __forceinline__ void rc_store_rows(uint16_t *dst, const uint16_t *t, int64_t ld, int64_t N, int64_t m0,
                                              int64_t m_hi, int rpp, int64_t n0) {
    for (int e = threadIdx.x; e < rpp * (RCT / 8); e += 256) {
        const int r = e / (RCT / 8), c8 = e - r * (RCT / 8);
        if (m0 + r < m_hi && ACT_DCHECK(n0 + 8 * c8 + 8 <= N))
            *reinterpret_cast<uint4 *>(dst + (m0 + r) * ld + n0 + 8 * c8) = *reinterpret_cast<const uint4 *>(t + r * RCT + 8 * c8);
    }
}

template <int BITS>
__global__ void __launch_bounds__(256, 4) rc_encode_tiled(actcomp_rc_args a) {
    using R = RcTile<BITS>;
    constexpr int EPP = R::EPP;
    extern __shared__ __align__(16) uint8_t rc_smem[];
    const int K = a.K, tid = threadIdx.x;
    float *r_s = reinterpret_cast<float *>(rc_smem);
    uint16_t *l_s = reinterpret_cast<uint16_t *>(rc_smem + R::off_l(K));
    uint16_t *t_s = reinterpret_cast<uint16_t *>(rc_smem + R::off_t(K));
    float *s_s = reinterpret_cast<float *>(rc_smem + R::off_s(K, false));
    const int64_t n0 = (int64_t)blockIdx.x * RCT, b = blockIdx.z;
    const int64_t m_lo = (int64_t)blockIdx.y * RCR;
    const int64_t m_hi = m_lo + RCR < a.M ? m_lo + RCR : a.M;
    const int lo = -(1 << (BITS - 1)), hi = (1 << (BITS - 1)) - 1, off = 1 << (BITS - 1);
    const float thr = (a.flags & ACT_RC_OUTLIER_BF16) ? rne_bf(a.outlier) : a.outlier;
    const int64_t srow = (a.flags & ACT_RC_SCALE_BATCH) ? (a.s_rows > 1 ? b : 0) : 0;
    const int64_t W = a.N * BITS / 8;
    rc_stage_tile<BITS>(a, r_s, s_s, n0, srow);
    const int rp0 = tid / R::TPR, w = tid - rp0 * R::TPR;
    for (int64_t m0 = m_lo; m0 < m_hi; m0 += R::RPP) {
        __syncthreads();  // the previous pass's o tile has gone out
        rc_load_rows(t_s, a.x + b * a.sxb, a.sxm, m0, m_hi, R::RPP, n0);
        for (int e = tid; e < R::RPP * K; e += 256) {
            const int r = e / K, k = e - r * K;
            l_s[e] = m0 + r < m_hi ? a.l[(m0 + r) * K + k] : (uint16_t)0;
        }
        __syncthreads();
        float dd[NRW][EPP];
        rc_dots<EPP, R::RP>(r_s, l_s, K, rp0, w, dd);
#pragma unroll
        for (int j = 0; j < NRW; ++j) {
            const int rp = rp0 + j * R::RP;
            const int64_t m = m0 + rp;
            if (m >= m_hi) break;
            const float (&d)[EPP] = dd[j];
            uint32_t byte = 0;
#pragma unroll
            for (int i = 0; i < EPP; ++i) {
                const int c = R::col(w, i);
                const float xv = bf2f(t_s[rp * RCT + c]);
                const float res = (a.flags & ACT_RC_TWIN_LOWRANK) ? rne_bf(__fsub_rn(xv, rne_bf(d[i])))
                                                                  : rne_bf(__fsub_rn(xv, d[i]));
                const float ov = fabsf(res) > thr ? res : 0.f;
                t_s[rp * RCT + c] = f2bf(ov);  // o over x, the same element of the same thread
                const float xr = __fsub_rn(res, ov);
                const float t = rne_bf(__fdiv_rn(xr, s_s[c]));
                float rq = (a.flags & ACT_RC_HALF_EVEN) ? rintf(t) : roundf(t);
                rq = fminf(fmaxf(rq, (float)lo), (float)hi);
                byte |= (uint32_t)((int)rq + off) << (i * BITS);
            }
            if (ACT_DCHECK(n0 * BITS / 8 + w < W)) a.q[(b * a.M + m) * W + n0 * BITS / 8 + w] = (uint8_t)byte;
        }
        __syncthreads();
        rc_store_rows(a.o + b * a.M * a.N, t_s, a.N, a.N, m0, m_hi, R::RPP, n0);
    }
}

template <int BITS, int OP>
__global__ void __launch_bounds__(256, 4) rc_decode_tiled(actcomp_rc_args a) {
    using R = RcTile<BITS>;
    constexpr int EPP = R::EPP;
    constexpr bool Y = OP != ACT_OP_DECODE;
    extern __shared__ __align__(16) uint8_t rc_smem[];
    const int K = a.K, tid = threadIdx.x;
    float *r_s = reinterpret_cast<float *>(rc_smem);
    uint16_t *l_s = reinterpret_cast<uint16_t *>(rc_smem + R::off_l(K));
    uint16_t *t_s = reinterpret_cast<uint16_t *>(rc_smem + R::off_t(K));
    uint16_t *y_s = reinterpret_cast<uint16_t *>(rc_smem + R::off_y(K));
    float *s_s = reinterpret_cast<float *>(rc_smem + R::off_s(K, Y));
    const int64_t n0 = (int64_t)blockIdx.x * RCT, b = blockIdx.z;
    const int64_t m_lo = (int64_t)blockIdx.y * RCR;
    const int64_t m_hi = m_lo + RCR < a.M ? m_lo + RCR : a.M;
    const int off = 1 << (BITS - 1);
    const uint32_t mask = (1u << BITS) - 1u;
    const int64_t srow = (a.flags & ACT_RC_SCALE_BATCH) ? (a.s_rows > 1 ? b : 0) : 0;
    const int64_t W = a.N * BITS / 8;
    rc_stage_tile<BITS>(a, r_s, s_s, n0, srow);
    const int rp0 = tid / R::TPR, w = tid - rp0 * R::TPR;
    for (int64_t m0 = m_lo; m0 < m_hi; m0 += R::RPP) {
        __syncthreads();  // the previous pass's output tile has gone out
        rc_load_rows(t_s, a.o ? a.o + b * a.M * a.N : nullptr, a.N, m0, m_hi, R::RPP, n0);
        if constexpr (Y) rc_load_rows(y_s, a.x + b * a.sxb, a.sxm, m0, m_hi, R::RPP, n0);
        for (int e = tid; e < R::RPP * K; e += 256) {
            const int r = e / K, k = e - r * K;
            l_s[e] = m0 + r < m_hi ? a.l[(m0 + r) * K + k] : (uint16_t)0;
        }
        __syncthreads();
        float dd[NRW][EPP];
        rc_dots<EPP, R::RP>(r_s, l_s, K, rp0, w, dd);
#pragma unroll
        for (int j = 0; j < NRW; ++j) {
            const int rp = rp0 + j * R::RP;
            const int64_t m = m0 + rp;
            if (m >= m_hi) break;
            const float (&d)[EPP] = dd[j];
            const uint32_t byte = a.q[(b * a.M + m) * W + n0 * BITS / 8 + w];
#pragma unroll
            for (int i = 0; i < EPP; ++i) {
                const int c = R::col(w, i);
                const uint32_t u = (byte >> (i * BITS)) & mask;
                const float wv = rne_bf(__fmul_rn(__int2float_rn((int)u - off), s_s[c]));
                const float av = a.o ? rne_bf(__fadd_rn(wv, bf2f(t_s[rp * RCT + c]))) : wv;
                float x = (a.flags & ACT_RC_TWIN_LOWRANK) ? rne_bf(__fadd_rn(av, rne_bf(d[i])))
                                                          : rne_bf(__fadd_rn(av, d[i]));
                if constexpr (Y) x = apply_op<OP>(x, bf2f(y_s[rp * RCT + c]));
                t_s[rp * RCT + c] = f2bf(x);  // the output over o, the same element of the same thread
            }
        }
        __syncthreads();
        rc_store_rows(a.out + b * a.M * a.N, t_s, a.N, a.N, m0, m_hi, R::RPP, n0);
    }
}

// The tiled kernels cover the 32-column block packing with whole 256-column
// tiles and 16-byte aligned rows; anything else takes the per-element kernels.
static bool rc_tiled_ok(const actcomp_rc_args *a, bool needs_x, bool needs_o) {
    if ((a->flags & ACT_RC_ROW_PACK) || a->N % RCT) return false;
    if (needs_x && (!aligned(a->x, 16) || a->sxb % 8 || a->sxm % 8)) return false;
    if (needs_o && a->o && !aligned(a->o, 16)) return false;
    return a->B <= 65535 && (a->M + RCR - 1) / RCR <= 65535;
}
static dim3 rc_tiled_grid(const actcomp_rc_args *a) {
    return dim3((unsigned)(a->N / RCT), (unsigned)((a->M + RCR - 1) / RCR), (unsigned)a->B);
}

// ---------------------------------------------------------------- dense helpers
template <int OP>
__global__ void elementwise_kernel(actcomp_ew_args a) {
    const int64_t total = a.B * a.M * a.N;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = g % a.N, bm = g / a.N, m = bm % a.M, b = bm / a.M;
        const float x = bf2f(a.x[b * a.sxb + m * a.sxm + n]);
        const float y = bf2f(a.g[b * a.sgb + m * a.sgm + n]);
        a.out[b * a.sob + m * a.som + n] = f2bf(apply_op<OP>(x, y));
    }
}

// One warp per row: out = (g - sum(g*y)) * y.
__global__ void softmax_bwd_kernel(const uint16_t *y, const uint16_t *g, uint16_t *out, int64_t rows, int64_t n,
                                   int64_t ld) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint16_t *yr = y + r * ld, *gr = g + r * ld;
        float acc = 0.f;
        for (int64_t c = lane; c < n; c += 32) acc = __fmaf_rn(bf2f(yr[c]), bf2f(gr[c]), acc);
        const float sum = warp_sum(acc);
        for (int64_t c = lane; c < n; c += 32)
            out[r * ld + c] = f2bf(__fmul_rn(__fsub_rn(bf2f(gr[c]), sum), bf2f(yr[c])));
    }
}

__global__ void extract_unstructured_kernel(const uint16_t *x, int64_t n, float thr, uint16_t *outl,
                                            uint16_t *rest) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = bf2f(x[i]);
        const float o = fabsf(v) > thr ? v : 0.f;
        outl[i] = f2bf(o);
        rest[i] = f2bf(__fsub_rn(v, o));
    }
}

__global__ void extract_channel_kernel(uint16_t *x, int64_t B, int64_t M, int64_t N, const int32_t *idx, int k,
                                       uint16_t *out) {
    const int64_t total = B * k * N;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = g % N, bj = g / N, j = bj % k, b = bj / k;
        const int64_t src = (b * M + idx[j]) * N + n;
        out[g] = x[src];
    }
}
__global__ void zero_channel_kernel(uint16_t *x, int64_t B, int64_t M, int64_t N, const int32_t *idx, int k) {
    const int64_t total = B * k * N;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = g % N, bj = g / N, j = bj % k, b = bj / k;
        x[(b * M + idx[j]) * N + n] = 0;
    }
}

__global__ void error_stats_kernel(const uint16_t *a, const uint16_t *b, int64_t n, double *out) {
    double se = 0.0, sr = 0.0, mx = 0.0, mis = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const double av = bf2f(a[i]), bv = bf2f(b[i]);
        const double e = av - bv;
        se += e * e;
        sr += bv * bv;
        mx = fmax(mx, fabs(e));
        mis += a[i] != b[i] ? 1.0 : 0.0;
    }
    for (int o = 16; o > 0; o >>= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        sr += __shfl_xor_sync(0xffffffffu, sr, o);
        mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mis += __shfl_xor_sync(0xffffffffu, mis, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(out + 0, se);
        atomicAdd(out + 1, sr);
        atomicMax(reinterpret_cast<unsigned long long *>(out + 2), (unsigned long long)__double_as_longlong(mx));
        atomicAdd(out + 3, mis);
    }
}

static unsigned blocks_for(int64_t n, int threads = 256) {
    int64_t b = (n + threads - 1) / threads;
    int64_t cap = (int64_t)num_sms() * 32;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace act

using namespace act;

static int rc_validate(const actcomp_rc_args *a) {
    ACT_CHECK(a && a->l && a->r && a->s && a->q, ACT_E_INVALID);
    ACT_CHECK(a->B >= 0 && a->M >= 0 && a->N > 0 && a->K >= 1 && a->K <= 64 && a->s_rows >= 1, ACT_E_INVALID);
    ACT_CHECK(a->bits == 1 || a->bits == 2 || a->bits == 4 || a->bits == 8, ACT_E_UNSUPPORTED);
    if (a->bits < 8) ACT_CHECK(a->N % 32 == 0, ACT_E_UNSUPPORTED);
    return ACT_OK;
}

extern "C" int actcomp_rc_encode(const actcomp_rc_args *a, void *stream) {
    int st = rc_validate(a);
    if (st) return st;
    ACT_CHECK(a->x && a->o, ACT_E_INVALID);
    const int64_t bytes = a->B * a->M * (a->N * a->bits / 8);
    if (bytes == 0) return ACT_OK;
    cudaStream_t s = as_stream(stream);
    if (rc_tiled_ok(a, true, true)) {
        const dim3 g = rc_tiled_grid(a);
        auto go = [&](auto kern, int smem) -> int {
            ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            kern<<<g, 256, smem, s>>>(*a);
            return launch_status();
        };
        switch (a->bits) {
            case 1: return go(rc_encode_tiled<1>, RcTile<1>::bytes(a->K, false));
            case 2: return go(rc_encode_tiled<2>, RcTile<2>::bytes(a->K, false));
            case 4: return go(rc_encode_tiled<4>, RcTile<4>::bytes(a->K, false));
            default: return go(rc_encode_tiled<8>, RcTile<8>::bytes(a->K, false));
        }
    }
    rc_encode_kernel<<<blocks_for(bytes), 256, 0, s>>>(*a);
    return launch_status();
}

extern "C" int actcomp_rc_decode(const actcomp_rc_args *a, int32_t op, void *stream) {
    int st = rc_validate(a);
    if (st) return st;
    ACT_CHECK(a->out, ACT_E_INVALID);
    ACT_CHECK(op >= ACT_OP_DECODE && op <= ACT_OP_GELU_BWD, ACT_E_INVALID);
    if (op != ACT_OP_DECODE) ACT_CHECK(a->x != nullptr, ACT_E_INVALID);
    const int64_t n = a->B * a->M * a->N;
    if (n == 0) return ACT_OK;
    cudaStream_t s = as_stream(stream);
    if (rc_tiled_ok(a, op != ACT_OP_DECODE, true)) {
        const dim3 g = rc_tiled_grid(a);
        const bool y = op != ACT_OP_DECODE;
        auto one = [&](auto kern, int smem) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return;
            kern<<<g, 256, smem, s>>>(*a);
        };
        auto go = [&](auto k1, auto k2, auto k4, auto k8) {
            switch (a->bits) {
                case 1: one(k1, RcTile<1>::bytes(a->K, y)); break;
                case 2: one(k2, RcTile<2>::bytes(a->K, y)); break;
                case 4: one(k4, RcTile<4>::bytes(a->K, y)); break;
                default: one(k8, RcTile<8>::bytes(a->K, y)); break;
            }
        };
        switch (op) {
            case ACT_OP_DECODE:
                go(rc_decode_tiled<1, ACT_OP_DECODE>, rc_decode_tiled<2, ACT_OP_DECODE>, rc_decode_tiled<4, ACT_OP_DECODE>,
                   rc_decode_tiled<8, ACT_OP_DECODE>);
                break;
            case ACT_OP_MUL:
                go(rc_decode_tiled<1, ACT_OP_MUL>, rc_decode_tiled<2, ACT_OP_MUL>, rc_decode_tiled<4, ACT_OP_MUL>,
                   rc_decode_tiled<8, ACT_OP_MUL>);
                break;
            case ACT_OP_SILU_BWD:
                go(rc_decode_tiled<1, ACT_OP_SILU_BWD>, rc_decode_tiled<2, ACT_OP_SILU_BWD>,
                   rc_decode_tiled<4, ACT_OP_SILU_BWD>, rc_decode_tiled<8, ACT_OP_SILU_BWD>);
                break;
            default:
                go(rc_decode_tiled<1, ACT_OP_GELU_BWD>, rc_decode_tiled<2, ACT_OP_GELU_BWD>,
                   rc_decode_tiled<4, ACT_OP_GELU_BWD>, rc_decode_tiled<8, ACT_OP_GELU_BWD>);
                break;
        }
        return launch_status();
    }
    switch (op) {
        case ACT_OP_DECODE: rc_decode_kernel<ACT_OP_DECODE><<<blocks_for(n), 256, 0, s>>>(*a); break;
        case ACT_OP_MUL: rc_decode_kernel<ACT_OP_MUL><<<blocks_for(n), 256, 0, s>>>(*a); break;
        case ACT_OP_SILU_BWD: rc_decode_kernel<ACT_OP_SILU_BWD><<<blocks_for(n), 256, 0, s>>>(*a); break;
        default: rc_decode_kernel<ACT_OP_GELU_BWD><<<blocks_for(n), 256, 0, s>>>(*a); break;
    }
    return launch_status();
}

extern "C" int actcomp_rc_lowrank_add(const actcomp_rc_args *a, void *stream) {
    ACT_CHECK(a && a->l && a->r && a->x && a->out, ACT_E_INVALID);
    ACT_CHECK(a->B >= 0 && a->M >= 0 && a->N > 0 && a->K >= 1 && a->K <= 64, ACT_E_INVALID);
    const int64_t n = a->B * a->M * a->N;
    if (n == 0) return ACT_OK;
    rc_lowrank_add_kernel<<<blocks_for(n), 256, 0, as_stream(stream)>>>(*a);
    return launch_status();
}

extern "C" int actcomp_elementwise(const actcomp_ew_args *a, int32_t op, void *stream) {
    ACT_CHECK(a && a->x && a->g && a->out, ACT_E_INVALID);
    ACT_CHECK(a->B >= 0 && a->M >= 0 && a->N >= 0, ACT_E_INVALID);
    ACT_CHECK(op >= ACT_OP_MUL && op <= ACT_OP_GELU_BWD, ACT_E_INVALID);
    const int64_t n = a->B * a->M * a->N;
    if (n == 0) return ACT_OK;
    cudaStream_t s = as_stream(stream);
    switch (op) {
        case ACT_OP_MUL: elementwise_kernel<ACT_OP_MUL><<<blocks_for(n), 256, 0, s>>>(*a); break;
        case ACT_OP_SILU_BWD: elementwise_kernel<ACT_OP_SILU_BWD><<<blocks_for(n), 256, 0, s>>>(*a); break;
        default: elementwise_kernel<ACT_OP_GELU_BWD><<<blocks_for(n), 256, 0, s>>>(*a); break;
    }
    return launch_status();
}

extern "C" int actcomp_softmax_bwd(const uint16_t *y, const uint16_t *g, uint16_t *out, int64_t rows, int64_t n,
                                   int64_t ld, void *stream) {
    ACT_CHECK(y && g && out && rows >= 0 && n > 0 && ld >= n, ACT_E_INVALID);
    if (rows == 0) return ACT_OK;
    softmax_bwd_kernel<<<blocks_for(rows * 32), 256, 0, as_stream(stream)>>>(y, g, out, rows, n, ld);
    return launch_status();
}

extern "C" int actcomp_extract_unstructured(const uint16_t *x, int64_t n, float thr, uint16_t *outlier,
                                            uint16_t *rest, void *stream) {
    ACT_CHECK(x && outlier && rest && n >= 0, ACT_E_INVALID);
    if (n == 0) return ACT_OK;
    extract_unstructured_kernel<<<blocks_for(n), 256, 0, as_stream(stream)>>>(x, n, thr, outlier, rest);
    return launch_status();
}

extern "C" int actcomp_extract_channel(uint16_t *x, int64_t B, int64_t M, int64_t N, const int32_t *idx, int32_t k,
                                       uint16_t *out, void *stream) {
    ACT_CHECK(x && out && idx && B >= 0 && M >= 0 && N >= 0 && k >= 0, ACT_E_INVALID);
    const int64_t n = B * k * N;
    if (n == 0) return ACT_OK;
    cudaStream_t s = as_stream(stream);
    extract_channel_kernel<<<blocks_for(n), 256, 0, s>>>(x, B, M, N, idx, k, out);
    ACT_CUDA_TRY(cudaGetLastError());
    zero_channel_kernel<<<blocks_for(n), 256, 0, s>>>(x, B, M, N, idx, k);
    return launch_status();
}

extern "C" int actcomp_error_stats(const uint16_t *a, const uint16_t *b, int64_t n, double *out, void *stream) {
    ACT_CHECK(a && b && out && n >= 0, ACT_E_INVALID);
    if (n == 0) return ACT_OK;
    error_stats_kernel<<<blocks_for(n), 256, 0, as_stream(stream)>>>(a, b, n, out);
    return launch_status();
}
