// cg_simt.cu -- channel-group format: basis preparation, top-k channel
// selection, and the warp-cooperative encode / decode / consumer kernels.
//
// Layout of the work: one warp handles one (token, 128-channel chunk) item;
// lane l owns the four consecutive channels chunk*128 + 4l .. 4l+3.  A 64- or
// 128-channel quantisation group is then 16 or 32 lanes (shuffle reductions),
// and one 128-point Walsh-Hadamard block is the whole warp (two in-register
// butterfly stages, five shuffle stages).
//
// Arithmetic follows oracle/actcomp_oracle.c step for step (single binary32
// operations, round-to-nearest-even, no contraction), and the two sums of the
// format -- the projection L = X . V and the low-rank term L . V^T -- are
// accumulated in binary64 (exact products, rounded once to binary32) like the
// oracle's, so codes, scales and reconstructions match it bit for bit.  These
// kernels serve the shapes the tensor-core kernels do not cover.
#include "common.cuh"

namespace act {

// ------------------------------------------------------------------ helpers
struct CgSlice {
    int64_t T, H;
    int bits, group, rank, k, wht;
    uint8_t *codes;
    float *scales;
    float *lr;
    uint16_t *outl;
    const int32_t *idx;
    const uint16_t *basis_t;
    const uint16_t *basis;
};

__device__ __forceinline__ CgSlice slice_of(const actcomp_cg_desc &d, int b) {
    CgSlice s;
    s.T = d.tokens;
    s.H = d.channels;
    s.bits = d.bits;
    s.group = d.group;
    s.rank = d.rank;
    s.k = d.n_outlier;
    s.wht = d.wht;
    const int64_t T = d.tokens, H = d.channels;
    s.codes = d.codes + (int64_t)b * T * (H * d.bits / 8);
    s.scales = d.scales + (int64_t)b * T * (H / d.group);
    s.lr = d.rank ? d.lowrank + (int64_t)b * T * d.rank : nullptr;
    s.outl = d.n_outlier ? d.outliers + (int64_t)b * T * d.n_outlier : nullptr;
    s.idx = d.n_outlier ? d.outlier_idx + (int64_t)b * d.n_outlier : nullptr;
    s.basis_t = d.rank ? d.basis_t + (int64_t)b * d.rank * H : nullptr;
    s.basis = d.rank ? d.basis + (int64_t)b * H * d.rank : nullptr;
    return s;
}

// low-rank term of channel c: sum_j L[j] * V[c, j], every product exact in
// binary64, the sum rounded once to binary32 (oracle lowrank_term)
__device__ __forceinline__ float lr_term(const float (&l)[64], const uint16_t *v_row, int rank) {
    double acc = 0.0;
    const uint4 *v = reinterpret_cast<const uint4 *>(v_row);
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) {
        if (w8 * 8 < rank) {
            const uint4 q = __ldg(v + w8);
            const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc += (double)l[w8 * 8 + 2 * i] * (double)__uint_as_float(qw[i] << 16);
                acc += (double)l[w8 * 8 + 2 * i + 1] * (double)__uint_as_float(qw[i] & 0xffff0000u);
            }
        }
    }
    return (float)acc;
}

__device__ __forceinline__ void load_lr_row(const CgSlice &s, int64_t t, float (&l)[64]) {
#pragma unroll
    for (int i = 0; i < 64; ++i) l[i] = 0.f;
    if (s.rank) {
        const float4 *p = reinterpret_cast<const float4 *>(s.lr + t * s.rank);
#pragma unroll
        for (int w4 = 0; w4 < 16; ++w4)
            if (w4 * 4 < s.rank) {
                const float4 q = __ldg(p + w4);
                l[4 * w4] = q.x;
                l[4 * w4 + 1] = q.y;
                l[4 * w4 + 2] = q.z;
                l[4 * w4 + 3] = q.w;
            }
    }
}

// 128-point unnormalised Walsh-Hadamard over a warp, lane owns v[0..3] =
// elements 4*lane .. 4*lane+3.  Stage m: pair (i, i+m), i has bit m clear,
// (a, b) -> (a + b, a - b); stages in increasing m, as in the oracle.
__device__ __forceinline__ void wht128_warp(float (&v)[4], int lane) {
    // m = 1: (0,1), (2,3)
    {
        float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
    // m = 2: (0,2), (1,3)
    {
        float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
    // m = 4 .. 64: partner lane = lane ^ (m / 4)
#pragma unroll
    for (int lm = 1; lm < 32; lm <<= 1) {
        const bool upper = (lane & lm) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float other = __shfl_xor_sync(0xffffffffu, v[i], lm);
            v[i] = upper ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
        }
    }
}

// first index j in [0, k) with idx[j] >= c (idx ascending)
__device__ __forceinline__ int lower_bound_idx(const int32_t *idx, int k, int64_t c) {
    int lo = 0, hi = k;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if ((int64_t)idx[mid] < c) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// ------------------------------------------------------------------ basis
// byte offset of value j (of `vbytes` bytes) of row `row` in a tile operand
// with W-byte rows (swizzled K-major layout, see include/actcomp.h)
__device__ __forceinline__ int64_t tile_operand_off(int64_t c, int j, int vbytes, int W) {
    const int row = (int)(c & 127);
    const int64_t tile = c >> 7;
    const int byte = j * vbytes;
    const int chunk = byte >> 4;
    const int s = W == 32 ? ((row >> 2) & 1) : (W == 64 ? ((row >> 1) & 3) : (row & 7));
    return (tile * 128 + row) * W + ((chunk ^ s) << 4) + (byte & 15);
}

// V rounded to bf16 and written in the three layouts of the format; one
// thread per (channel, basis vector).
__global__ void basis_prepare_kernel(const float *V, int64_t H, int rank, uint16_t *Vt, uint16_t *Vb,
                                     uint16_t *tile) {
    const int b = blockIdx.y;
    const int64_t n = H * rank;
    const int rk = rank <= 16 ? 16 : (rank <= 32 ? 32 : 64);  // tile operand: 2 * rk bytes per row
    const int64_t ntile = (H + 127) / 128;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = e / rank;
        const int j = (int)(e - c * rank);
        const uint16_t h = f2bf(V[(int64_t)b * n + e]);
        Vb[(int64_t)b * n + e] = h;
        Vt[(int64_t)b * n + (int64_t)j * H + c] = h;
        if (tile) tile[((int64_t)b * ntile * 128 * 2 * rk + tile_operand_off(c, j, 2, 2 * rk)) / 2] = h;
    }
}

// ------------------------------------------------------------------ top-k channels
__global__ void channel_absmax_kernel(const uint16_t *x, int64_t T, int64_t H, int64_t ldx, float *score) {
    int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= H) return;
    float m = 0.f;
    for (int64_t t = blockIdx.y; t < T; t += gridDim.y) m = fmaxf(m, fabsf(bf2f(x[t * ldx + c])));
    // scores are non-negative floats: their bit patterns order like unsigned ints
    atomicMax(reinterpret_cast<unsigned int *>(score) + c, __float_as_uint(m));
}

// One block: k rounds of arg-max over H scores (ties -> lower index), then
// the chosen set is written in ascending channel order.
__global__ void topk_kernel(float *score, int64_t H, int k, int32_t *idx) {
    __shared__ unsigned long long best[32];
    __shared__ int chosen[64];
    for (int round = 0; round < k; ++round) {
        // key: score bits high, inverted index low -> max key = max score, min index
        unsigned long long key = 0;
        for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
            float s = score[c];
            if (s < 0.f) continue;  // taken
            unsigned long long kk = ((unsigned long long)__float_as_uint(s) << 32) |
                                    (unsigned long long)(0xffffffffu - (uint32_t)c);
            key = kk > key ? kk : key;
        }
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = key;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long m = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = best[w] > m ? best[w] : m;
            int c = (int)(0xffffffffu - (uint32_t)(m & 0xffffffffu));
            chosen[round] = c;
            score[c] = -1.f;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        // insertion sort of <= 64 entries
        for (int i = 1; i < k; ++i) {
            int v = chosen[i], j = i - 1;
            while (j >= 0 && chosen[j] > v) {
                chosen[j + 1] = chosen[j];
                --j;
            }
            chosen[j + 1] = v;
        }
        for (int i = 0; i < k; ++i) idx[i] = chosen[i];
    }
}

// ------------------------------------------------------------------ encode
// Projection: one warp per token.  L = x . V with the products exact in
// binary64, lane-strided partial sums and a shuffle tree in binary64, rounded
// once to binary32 (oracle cg_project).
template <int RANK>
__global__ void __launch_bounds__(256) cg_project_kernel(actcomp_cg_desc d, const uint16_t *x, int64_t ldx) {
    const int b = blockIdx.y;
    const CgSlice s = slice_of(d, b);
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const uint16_t *xs = x + (int64_t)b * s.T * ldx;
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < s.T; t += warps) {
        double acc[RANK];
#pragma unroll
        for (int j = 0; j < RANK; ++j) acc[j] = 0.0;
        const uint16_t *xr = xs + t * ldx;
        for (int64_t c = (int64_t)lane * 8; c < s.H; c += 256) {
            const bool full = c + 8 <= s.H;
            float xf[8];
            if (full) {
                const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(xr + c));
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    xf[2 * i] = __uint_as_float(xw[i] << 16);
                    xf[2 * i + 1] = __uint_as_float(xw[i] & 0xffff0000u);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) xf[i] = c + i < s.H ? bf2f(xr[c + i]) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < RANK; ++j) {
                const uint16_t *vr = s.basis_t + (int64_t)j * s.H + c;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    if (full || c + i < s.H) acc[j] += (double)xf[i] * (double)bf2f(vr[i]);
            }
        }
        // lane j ends up with coefficient j (and j + 32 when RANK == 64)
        double mine0 = 0.0, mine1 = 0.0;
#pragma unroll
        for (int j = 0; j < RANK; ++j) {
            double v = acc[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (j == lane) mine0 = v;
            if (j == lane + 32) mine1 = v;
        }
        if (lane < RANK) s.lr[t * RANK + lane] = (float)mine0;
        if (lane + 32 < RANK) s.lr[t * RANK + lane + 32] = (float)mine1;
    }
}

// Residual codes: one warp per (token, 128-channel chunk).
template <int BITS>
__global__ void __launch_bounds__(256) cg_quant_kernel(actcomp_cg_desc d, const uint16_t *x, int64_t ldx) {
    const int b = blockIdx.y;
    const CgSlice s = slice_of(d, b);
    const int lane = threadIdx.x & 31;
    const int64_t nchunk = (s.H + 127) / 128;
    const int64_t items = s.T * nchunk;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int qmax = (1 << (BITS - 1)) - 1, off = 1 << (BITS - 1);
    const int glanes = s.group / 4;  // lanes per quantisation group
    const int64_t ngroups = s.H / s.group;
    const uint16_t *xs = x + (int64_t)b * s.T * ldx;
    for (int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
        const int64_t t = it / nchunk, ch = it % nchunk;
        const int64_t c0 = ch * 128 + lane * 4;
        const bool valid = c0 < s.H;
        float l[64];
        load_lr_row(s, t, l);
        float w[4] = {0.f, 0.f, 0.f, 0.f};
        uint2 xraw = make_uint2(0, 0);
        if (valid) {
            xraw = __ldg(reinterpret_cast<const uint2 *>(xs + t * ldx + c0));
            const uint32_t xw[2] = {xraw.x, xraw.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float xv = __uint_as_float(i & 1 ? (xw[i >> 1] & 0xffff0000u) : (xw[i >> 1] << 16));
                w[i] = s.rank ? __fsub_rn(xv, lr_term(l, s.basis + (c0 + i) * s.rank, s.rank)) : xv;
            }
        }
        // outlier channels of this chunk: verbatim copy, residual zeroed
        if (s.k) {
            const int64_t cs = ch * 128, ce = cs + 128;
            int j = lower_bound_idx(s.idx, s.k, cs);
            for (; j < s.k && s.idx[j] < ce; ++j) {
                const int64_t c = s.idx[j];
                if (c >= c0 && c < c0 + 4 && valid) {
                    const int i = (int)(c - c0);
                    const uint32_t word = i < 2 ? xraw.x : xraw.y;
                    s.outl[t * s.k + j] = (uint16_t)(i & 1 ? (word >> 16) : (word & 0xffffu));
                    w[i] = 0.f;
                }
            }
        }
        if (s.wht) wht128_warp(w, lane);
        float amax = fmaxf(fmaxf(fabsf(w[0]), fabsf(w[1])), fmaxf(fabsf(w[2]), fabsf(w[3])));
        amax = group_max(amax, glanes);
        const float sc = __fdiv_rn(amax, (float)qmax);
        const float rs = amax > 0.f ? __fdiv_rn((float)qmax, amax) : 0.f;
        if (!valid) continue;
        if ((lane % glanes) == 0) s.scales[t * ngroups + c0 / s.group] = sc;
        uint32_t u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) u[i] = (uint32_t)(nearest_code(w[i], rs, qmax) + off);
        if constexpr (BITS == 4) {
            uint16_t packed = (uint16_t)(u[0] | (u[1] << 4) | (u[2] << 8) | (u[3] << 12));
            *reinterpret_cast<uint16_t *>(s.codes + t * (s.H / 2) + c0 / 2) = packed;
        } else {
            uint32_t packed = u[0] | (u[1] << 8) | (u[2] << 16) | (u[3] << 24);
            *reinterpret_cast<uint32_t *>(s.codes + t * s.H + c0) = packed;
        }
    }
}

// ------------------------------------------------------------------ decode + consumers
// Reconstruct four channels of one token (bit-exact with cg_decode) into bf16.
template <int BITS>
__device__ __forceinline__ void reconstruct4(const CgSlice &s, int64_t t, int64_t ch, int lane, bool valid,
                                             const float (&l)[64], uint16_t (&xh)[4]) {
    const int off = 1 << (BITS - 1);
    const int64_t c0 = ch * 128 + lane * 4;
    float w[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
        uint32_t raw;
        if constexpr (BITS == 4) raw = *reinterpret_cast<const uint16_t *>(s.codes + t * (s.H / 2) + c0 / 2);
        else raw = *reinterpret_cast<const uint32_t *>(s.codes + t * s.H + c0);
        const float sc = s.scales[t * (s.H / s.group) + c0 / s.group];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int u = (int)((raw >> (i * BITS)) & ((1u << BITS) - 1u));
            w[i] = __fmul_rn(__int2float_rn(u - off), sc);
        }
    }
    if (s.wht) {
        wht128_warp(w, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = __fmul_rn(w[i], 0.0078125f);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float v = (s.rank && valid) ? __fadd_rn(lr_term(l, s.basis + (c0 + i) * s.rank, s.rank), w[i]) : w[i];
        xh[i] = f2bf(v);
    }
    if (s.k) {
        const int64_t cs = ch * 128, ce = cs + 128;
        int j = lower_bound_idx(s.idx, s.k, cs);
        for (; j < s.k && s.idx[j] < ce; ++j) {
            const int64_t c = s.idx[j];
            if (c >= c0 && c < c0 + 4) xh[c - c0] = s.outl[t * s.k + j];
        }
    }
}

template <int BITS, int OP>
__global__ void __launch_bounds__(256) cg_consume_kernel(actcomp_cg_desc d, const uint16_t *y, int64_t ldy,
                                                         uint16_t *out, int64_t ldo) {
    const int b = blockIdx.y;
    const CgSlice s = slice_of(d, b);
    const int lane = threadIdx.x & 31;
    const int64_t nchunk = (s.H + 127) / 128;
    const int64_t items = s.T * nchunk;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const uint16_t *ys = OP != ACT_OP_DECODE ? y + (int64_t)b * s.T * ldy : nullptr;
    uint16_t *os = out + (int64_t)b * s.T * ldo;
    for (int64_t it = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items; it += warps) {
        const int64_t t = it / nchunk, ch = it % nchunk;
        const int64_t c0 = ch * 128 + lane * 4;
        const bool valid = c0 < s.H;
        float l[64];
        load_lr_row(s, t, l);
        uint16_t xh[4];
        reconstruct4<BITS>(s, t, ch, lane, valid, l, xh);
        if (!valid) continue;
        uint16_t o[4];
        if constexpr (OP == ACT_OP_DECODE) {
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = xh[i];
        } else {
            uint2 yr = __ldg(reinterpret_cast<const uint2 *>(ys + t * ldy + c0));
            const uint32_t yw[2] = {yr.x, yr.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float yv = __uint_as_float(i & 1 ? (yw[i >> 1] & 0xffff0000u) : (yw[i >> 1] << 16));
                o[i] = f2bf(apply_op<OP>(bf2f(xh[i]), yv));
            }
        }
        uint2 packed;
        packed.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
        packed.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
        *reinterpret_cast<uint2 *>(os + t * ldo + c0) = packed;
    }
}

// Softmax backward over compressed probabilities: one warp per row, two
// sweeps (row sum of dP * P^, then the output).
template <int BITS>
__global__ void __launch_bounds__(256) cg_softmax_bwd_kernel(actcomp_cg_desc d, const uint16_t *dp, uint16_t *ds,
                                                             int64_t ld, int causal) {
    const int b = blockIdx.y;
    const CgSlice s = slice_of(d, b);
    const int lane = threadIdx.x & 31;
    const int64_t nchunk = (s.H + 127) / 128;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const uint16_t *dps = dp + (int64_t)b * s.T * ld;
    uint16_t *dss = ds + (int64_t)b * s.T * ld;
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < s.T; t += warps) {
        float l[64];
        load_lr_row(s, t, l);
        const int64_t last = causal ? t : s.H - 1;  // last column with P != 0
        const int64_t nch = causal ? (last / 128 + 1) : nchunk;
        float acc = 0.f;
        for (int64_t ch = 0; ch < nch; ++ch) {
            const int64_t c0 = ch * 128 + lane * 4;
            const bool valid = c0 < s.H;
            uint16_t xh[4];
            reconstruct4<BITS>(s, t, ch, lane, valid, l, xh);
            if (!valid) continue;
            uint2 g = __ldg(reinterpret_cast<const uint2 *>(dps + t * ld + c0));
            const uint32_t gw[2] = {g.x, g.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (c0 + i > last) continue;
                float gv = __uint_as_float(i & 1 ? (gw[i >> 1] & 0xffff0000u) : (gw[i >> 1] << 16));
                acc = __fmaf_rn(bf2f(xh[i]), gv, acc);
            }
        }
        const float sum = warp_sum(acc);
        for (int64_t ch = 0; ch < nchunk; ++ch) {
            const int64_t c0 = ch * 128 + lane * 4;
            const bool valid = c0 < s.H;
            uint16_t o[4] = {0, 0, 0, 0};
            if (ch < nch) {
                uint16_t xh[4];
                reconstruct4<BITS>(s, t, ch, lane, valid, l, xh);
                if (!valid) continue;
                uint2 g = __ldg(reinterpret_cast<const uint2 *>(dps + t * ld + c0));
                const uint32_t gw[2] = {g.x, g.y};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (c0 + i > last) continue;
                    float gv = __uint_as_float(i & 1 ? (gw[i >> 1] & 0xffff0000u) : (gw[i >> 1] << 16));
                    o[i] = f2bf(__fmul_rn(__fsub_rn(gv, sum), bf2f(xh[i])));
                }
            } else if (!valid) {
                continue;
            }
            uint2 packed;
            packed.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
            packed.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
            *reinterpret_cast<uint2 *>(dss + t * ld + c0) = packed;
        }
    }
}

// ------------------------------------------------------------------ validation
int validate_desc(const actcomp_cg_desc *d) {
    ACT_CHECK(d, ACT_E_INVALID);
    ACT_CHECK(d->tokens >= 0 && d->channels > 0 && d->batch >= 1, ACT_E_INVALID);
    ACT_CHECK(d->bits == 4 || d->bits == 8, ACT_E_UNSUPPORTED);
    ACT_CHECK(d->group == 32 || d->group == 64 || d->group == 128, ACT_E_UNSUPPORTED);
    ACT_CHECK(d->channels % d->group == 0, ACT_E_INVALID);
    ACT_CHECK(d->rank >= 0 && d->rank <= 64 && d->rank % 16 == 0, ACT_E_UNSUPPORTED);
    ACT_CHECK(d->n_outlier >= 0 && d->n_outlier <= 64 && d->n_outlier <= d->channels, ACT_E_UNSUPPORTED);
    ACT_CHECK(d->wht == 0 || d->wht == 1, ACT_E_INVALID);
    if (d->wht) ACT_CHECK(d->channels % 128 == 0, ACT_E_UNSUPPORTED);
    ACT_CHECK(d->codes && d->scales, ACT_E_INVALID);
    ACT_CHECK(aligned(d->codes, 4) && aligned(d->scales, 4), ACT_E_ALIGN);
    if (d->rank) {
        ACT_CHECK(d->lowrank && d->basis_t && d->basis, ACT_E_INVALID);
        ACT_CHECK(aligned(d->lowrank, 16) && aligned(d->basis, 16) && aligned(d->basis_t, 16), ACT_E_ALIGN);
        if (d->basis_tile) ACT_CHECK(aligned(d->basis_tile, 16), ACT_E_ALIGN);
    }
    if (d->n_outlier) ACT_CHECK(d->outliers && d->outlier_idx, ACT_E_INVALID);
    return ACT_OK;
}

static int grid_for(int64_t items_per_slice) {
    int64_t blocks = (items_per_slice + 7) / 8;
    int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    return (int)(blocks < 1 ? 1 : blocks);
}

}  // namespace act

using namespace act;

extern "C" int actcomp_cg_basis_prepare(const float *V, int64_t H, int32_t rank, int32_t batch, uint16_t *basis_t,
                                        uint16_t *basis, uint16_t *basis_tile, void *stream) {
    ACT_CHECK(V && basis_t && basis, ACT_E_INVALID);
    ACT_CHECK(H > 0 && rank > 0 && rank <= 64 && batch >= 1, ACT_E_INVALID);
    cudaStream_t s = as_stream(stream);
    const int64_t rows = batch * ((H + 127) / 128) * 128;
    const int rk = rank <= 16 ? 16 : (rank <= 32 ? 32 : 64);
    // padding (values past the rank, channels past H) reads as zero
    if (basis_tile) ACT_CUDA_TRY(cudaMemsetAsync(basis_tile, 0, (size_t)(rows * 2 * rk), s));
    const int64_t n = H * rank;
    dim3 grid((unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), (unsigned)batch);
    basis_prepare_kernel<<<grid, 256, 0, s>>>(V, H, rank, basis_t, basis, basis_tile);
    return launch_status();
}

extern "C" int actcomp_cg_channel_topk(const uint16_t *x, int64_t T, int64_t H, int64_t ldx, int32_t k,
                                       int32_t *idx, float *score_ws, void *stream) {
    ACT_CHECK(x && idx && score_ws, ACT_E_INVALID);
    ACT_CHECK(T > 0 && H > 0 && ldx >= H && k >= 0 && k <= 64 && k <= H, ACT_E_INVALID);
    if (k == 0) return ACT_OK;
    cudaStream_t s = as_stream(stream);
    ACT_CUDA_TRY(cudaMemsetAsync(score_ws, 0, sizeof(float) * H, s));
    dim3 grid((unsigned)((H + 255) / 256), (unsigned)(T < 64 ? T : 64));
    channel_absmax_kernel<<<grid, 256, 0, s>>>(x, T, H, ldx, score_ws);
    topk_kernel<<<1, 1024, 0, s>>>(score_ws, H, k, idx);
    return launch_status();
}

// Encode entry point: CUDA-core path.  (The tensor-core encode takes over for
// the shapes it supports; see actcomp_cg_encode in capi.cu.)
int act_cg_encode_simt(const actcomp_cg_desc *d, const uint16_t *x, int64_t ldx, cudaStream_t s) {
    if (d->tokens == 0) return ACT_OK;
    if (d->rank) {
        dim3 grid(grid_for(d->tokens), d->batch);
        switch (d->rank) {
            case 16: cg_project_kernel<16><<<grid, 256, 0, s>>>(*d, x, ldx); break;
            case 32: cg_project_kernel<32><<<grid, 256, 0, s>>>(*d, x, ldx); break;
            case 48: cg_project_kernel<48><<<grid, 256, 0, s>>>(*d, x, ldx); break;
            default: cg_project_kernel<64><<<grid, 256, 0, s>>>(*d, x, ldx); break;
        }
        ACT_CUDA_TRY(cudaGetLastError());
    }
    dim3 grid(grid_for(d->tokens * ((d->channels + 127) / 128)), d->batch);
    if (d->bits == 4) cg_quant_kernel<4><<<grid, 256, 0, s>>>(*d, x, ldx);
    else cg_quant_kernel<8><<<grid, 256, 0, s>>>(*d, x, ldx);
    return launch_status();
}

int act_cg_consume_simt(const actcomp_cg_desc *d, int op, const uint16_t *y, int64_t ldy, uint16_t *out,
                        int64_t ldo, cudaStream_t s) {
    if (d->tokens == 0) return ACT_OK;
    dim3 grid(grid_for(d->tokens * ((d->channels + 127) / 128)), d->batch);
#define ACT_LAUNCH_CONSUME(B)                                                                                 \
    switch (op) {                                                                                             \
        case ACT_OP_DECODE: cg_consume_kernel<B, ACT_OP_DECODE><<<grid, 256, 0, s>>>(*d, y, ldy, out, ldo); break; \
        case ACT_OP_MUL: cg_consume_kernel<B, ACT_OP_MUL><<<grid, 256, 0, s>>>(*d, y, ldy, out, ldo); break;       \
        case ACT_OP_SILU_BWD: cg_consume_kernel<B, ACT_OP_SILU_BWD><<<grid, 256, 0, s>>>(*d, y, ldy, out, ldo); break; \
        default: cg_consume_kernel<B, ACT_OP_GELU_BWD><<<grid, 256, 0, s>>>(*d, y, ldy, out, ldo); break;         \
    }
    if (d->bits == 4) {
        ACT_LAUNCH_CONSUME(4)
    } else {
        ACT_LAUNCH_CONSUME(8)
    }
#undef ACT_LAUNCH_CONSUME
    return launch_status();
}

int act_cg_softmax_simt(const actcomp_cg_desc *d, const uint16_t *dp, uint16_t *ds, int64_t ld, int causal,
                        cudaStream_t s) {
    if (d->tokens == 0) return ACT_OK;
    dim3 grid(grid_for(d->tokens), d->batch);
    if (d->bits == 4) cg_softmax_bwd_kernel<4><<<grid, 256, 0, s>>>(*d, dp, ds, ld, causal);
    else cg_softmax_bwd_kernel<8><<<grid, 256, 0, s>>>(*d, dp, ds, ld, causal);
    return launch_status();
}
