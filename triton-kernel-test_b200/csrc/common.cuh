// common.cuh -- shared helpers of libactcomp (sm_100a).
//
// The library is compiled with --fmad=false: every a*b+c written in these
// sources is a multiply and an add, each rounded to nearest-even, exactly as
// the CPU oracle evaluates it.  Where a fused multiply-add is wanted it is
// written as __fmaf_rn explicitly.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/actcomp.h"

#define ACT_CUDA_TRY(expr)                         \
    do {                                           \
        cudaError_t _e = (expr);                   \
        if (_e != cudaSuccess) return ACT_E_CUDA;  \
    } while (0)

#define ACT_CHECK(cond, code)     \
    do {                          \
        if (!(cond)) return code; \
    } while (0)

namespace act {

// Error word set by device-side bounded waits that give up and, in the
// bounds-checked build, by an index check that fails (never by a trap).
extern __device__ uint32_t g_device_error;
enum : uint32_t { DEV_ERR_MBAR_TIMEOUT = 1u, DEV_ERR_BAD_ARG = 2u, DEV_ERR_BOUNDS = 4u };

// ACT_DCHECK(cond): in the build with -DACT_BOUNDS_CHECK (libactcomp_bc.so), a
// false cond records DEV_ERR_BOUNDS and the guarded access is skipped; in the
// product build it is `true` and costs nothing.
#ifdef ACT_BOUNDS_CHECK
__device__ __forceinline__ bool act_dcheck(bool ok) {
    if (!ok) atomicOr(&g_device_error, DEV_ERR_BOUNDS);
    return ok;
}
#define ACT_DCHECK(cond) ::act::act_dcheck((cond))
#else
#define ACT_DCHECK(cond) true
#endif

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
static inline int launch_status() { return cudaGetLastError() == cudaSuccess ? ACT_OK : ACT_E_CUDA; }
static inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int num_sms();  // cached per device

// ---------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float rne_bf(float f) { return bf2f(f2bf(f)); }

// ---------------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// max over aligned groups of `width` lanes (width a power of two <= 32)
__device__ __forceinline__ float group_max(float v, int width) {
    for (int o = width >> 1; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------- exact int <-> float
// For |v| < 2^22, v + 1.5 * 2^23 is a float whose mantissa holds v exactly, so
// one integer add and one float subtract convert without the quarter-rate
// conversion pipe.
__device__ __forceinline__ float i2f_exact(int v) {
    return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}
// Quantisation code of v with reciprocal scale rs: the exact product v * rs
// rounded to the nearest integer (ties to even) by ONE fma against 1.5 * 2^23,
// whose bit pattern then holds 0x4B400000 + q; |v * rs| <= qmax + 1/2 < 2^22.
// A single explicit fma gives the same code whatever the compiler contracts.
__device__ __forceinline__ int nearest_code(float v, float rs, int qmax) {
    const int q = __float_as_int(__fmaf_rn(v, rs, 12582912.0f)) - 0x4B400000;
    return max(-qmax, min(qmax, q));
}
// (float)u for 0 <= u < 2^23, minus a constant folded into the subtraction.
__device__ __forceinline__ float u2f_minus(uint32_t u, float c_plus_2p23) {
    return __fsub_rn(__uint_as_float(0x4B000000u | u), c_plus_2p23);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
// v = hi + mid + lo exactly, each a bf16 value: hi = bf16(v), mid = bf16(v - hi),
// lo = v - hi - mid (both differences are exact in binary32, and the last one
// has at most 8 significant bits).  The tensor cores multiply the three pieces
// by a bf16 operand exactly, so a float32 factor enters an MMA at full precision.
__device__ __forceinline__ void split3_bf16(float v, float &hi, float &mid, float &lo) {
    hi = rne_bf(v);
    const float r1 = __fsub_rn(v, hi);
    mid = rne_bf(r1);
    lo = rne_bf(__fsub_rn(r1, mid));
}

// ---------------------------------------------------------------- consumer ops
// The derivative formulas of the reference twins, evaluated in binary32 in the
// order they are written there and rounded once to bf16.  exp and the
// reciprocal use the hardware approximations (ex2.approx, rcp.approx: a few
// ulp), so outputs agree with the libm-based oracle except where a bf16
// rounding boundary falls inside that error.
__device__ __forceinline__ float hw_exp(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, 1.4426950408889634f)));
    return y;
}
__device__ __forceinline__ float hw_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float silu_bwd_f(float x, float g) {
    // silu_backward.py:6-8
    const float s = hw_rcp(__fadd_rn(1.0f, hw_exp(-x)));
    return __fmul_rn(g, __fmul_rn(s, __fadd_rn(1.0f, __fmul_rn(x, __fsub_rn(1.0f, s)))));
}
__device__ __forceinline__ float gelu_bwd_f(float x, float g) {
    // gelu_backward.py:14-21 (tanh approximation); tanh(y) = 1 - 2 / (e^{2y} + 1)
    const float gamma = 0.7978845608028654f, kappa = 0.044715f;
    const float x2 = __fmul_rn(x, x);
    const float y = __fmul_rn(gamma, __fadd_rn(x, __fmul_rn(kappa, __fmul_rn(x2, x))));
    const float th = __fsub_rn(1.0f, __fmul_rn(2.0f, hw_rcp(__fadd_rn(hw_exp(__fmul_rn(2.0f, y)), 1.0f))));
    const float inner = __fmul_rn(__fmul_rn(__fsub_rn(1.0f, __fmul_rn(th, th)), gamma),
                                  __fadd_rn(1.0f, __fmul_rn(__fmul_rn(3.0f, kappa), x2)));
    const float d = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(1.0f, th), __fmul_rn(x, inner)));
    return __fmul_rn(d, g);
}
// packed fp32 pairs (sm_100 f32x2 instructions; each half correctly rounded)
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{.reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
        " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{.reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mul.rn.f32x2 rd, ra, rb;\n"
        " mov.b64 {%0, %1}, rd;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{.reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n add.rn.f32x2 rd, ra, rb;\n"
        " mov.b64 {%0, %1}, rd;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    float2 d;
    asm("{.reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n sub.rn.f32x2 rd, ra, rb;\n"
        " mov.b64 {%0, %1}, rd;}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// The same formulas on pairs of elements: every add / multiply is a packed
// f32x2 instruction (each half rounded exactly as the scalar one), exp and the
// reciprocal stay per element.
__device__ __forceinline__ float2 silu_bwd_f2(float2 x, float2 g) {
    const float2 one = make_float2(1.0f, 1.0f);
    const float2 s = make_float2(hw_rcp(__fadd_rn(1.0f, hw_exp(-x.x))), hw_rcp(__fadd_rn(1.0f, hw_exp(-x.y))));
    return mul2(g, mul2(s, add2(one, mul2(x, sub2(one, s)))));
}
__device__ __forceinline__ float2 gelu_bwd_f2(float2 x, float2 g) {
    const float gamma = 0.7978845608028654f, kappa = 0.044715f;
    const float2 one = make_float2(1.0f, 1.0f), two = make_float2(2.0f, 2.0f), half = make_float2(0.5f, 0.5f);
    const float2 gm = make_float2(gamma, gamma), kp = make_float2(kappa, kappa);
    const float tk = __fmul_rn(3.0f, kappa);
    const float2 tk2 = make_float2(tk, tk);
    const float2 x2 = mul2(x, x);
    const float2 y = mul2(gm, add2(x, mul2(kp, mul2(x2, x))));
    const float2 e = add2(make_float2(hw_exp(__fmul_rn(2.0f, y.x)), hw_exp(__fmul_rn(2.0f, y.y))), one);
    const float2 th = sub2(one, mul2(two, make_float2(hw_rcp(e.x), hw_rcp(e.y))));
    const float2 inner = mul2(mul2(sub2(one, mul2(th, th)), gm), add2(one, mul2(tk2, x2)));
    const float2 d = mul2(half, add2(add2(one, th), mul2(x, inner)));
    return mul2(d, g);
}

template <int OP>
__device__ __forceinline__ float apply_op(float xhat, float y) {
    if constexpr (OP == ACT_OP_MUL) return __fmul_rn(xhat, y);
    else if constexpr (OP == ACT_OP_SILU_BWD) return silu_bwd_f(xhat, y);
    else if constexpr (OP == ACT_OP_GELU_BWD) return gelu_bwd_f(xhat, y);
    else return xhat;
}
template <int OP>
__device__ __forceinline__ float2 apply_op2(float2 xhat, float2 y) {
    if constexpr (OP == ACT_OP_MUL) return mul2(xhat, y);
    else if constexpr (OP == ACT_OP_SILU_BWD) return silu_bwd_f2(xhat, y);
    else if constexpr (OP == ACT_OP_GELU_BWD) return gelu_bwd_f2(xhat, y);
    else return xhat;
}

// Row-swizzled K-major operand layout (PITCH bytes a row, 16-byte chunks
// XORed with the row as the 128/64/32-byte tcgen05 swizzles expect).
template <int PITCH>
__device__ __forceinline__ int kmajor_swz(int r, int c) {
    if constexpr (PITCH == 128) return r * 128 + ((c ^ (r & 7)) << 4);
    else if constexpr (PITCH == 64) return r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    else return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
}

// One warp splits ROWS rows of the float32 projection (rows t0 .., row
// stride `rank`; rows from `rows_here` on and coefficients from `rank` on are
// zero) into its three exact bf16 pieces (split3_bf16), written as three
// K-major operand tiles of LB bytes a row at dst, dst + ROWS*LB and
// dst + 2*ROWS*LB.  Each lane issues the loads of up to eight 8-coefficient
// chunks before converting any, so the warp waits for memory once per batch.
template <int ROWS, int LB>
__device__ __forceinline__ void build_piece_tiles(const float *lr, int64_t t0, int64_t rows_here, int rank,
                                                  uint8_t *dst, int lane) {
    constexpr int CPR = LB / 16;          // 16-byte chunks per operand row (8 coefficients)
    constexpr int N = ROWS * CPR / 32;    // chunks per lane
    constexpr int BATCH = N < 8 ? N : 8;
    static_assert((ROWS * CPR) % 32 == 0 && N % BATCH == 0, "whole chunks per lane");
#pragma unroll 1
    for (int j0 = 0; j0 < N; j0 += BATCH) {
        float4 v[BATCH][2];
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int e = lane + 32 * (j0 + j), row = e / CPR, c16 = e - row * CPR;
            if (8 * c16 < rank && row < rows_here) {
                const float4 *src = reinterpret_cast<const float4 *>(lr + (t0 + row) * rank + 8 * c16);
                v[j][0] = __ldg(src);
                v[j][1] = __ldg(src + 1);
            } else {
                v[j][0] = v[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int e = lane + 32 * (j0 + j), row = e / CPR, c16 = e - row * CPR;
            const float in[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w,
                                 v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
            uint32_t ph[4], pm[4], pl[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float h0, m0, l0, h1, m1, l1;
                split3_bf16(in[2 * h], h0, m0, l0);
                split3_bf16(in[2 * h + 1], h1, m1, l1);
                ph[h] = pack_bf16x2(h0, h1);
                pm[h] = pack_bf16x2(m0, m1);
                pl[h] = pack_bf16x2(l0, l1);
            }
            const int o = kmajor_swz<LB>(row, c16);
            *reinterpret_cast<uint4 *>(dst + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
            *reinterpret_cast<uint4 *>(dst + ROWS * LB + o) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
            *reinterpret_cast<uint4 *>(dst + 2 * ROWS * LB + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
        }
    }
}

// The same piece tiles built by a team of TEAM threads (tid 0 .. TEAM-1, whole
// warps): each thread loads all of its chunks (at most a few) before converting
// any, so a kernel's idle warps turn its first token block around in one
// memory round trip instead of the one builder warp's several.  The caller
// fences the async proxy and synchronises the team before the tiles are used.
template <int ROWS, int LB, int TEAM>
__device__ __forceinline__ void build_piece_tiles_team(const float *lr, int64_t t0, int64_t rows_here, int rank,
                                                       uint8_t *dst, int tid) {
    constexpr int CPR = LB / 16;
    constexpr int TOTAL = ROWS * CPR;
    constexpr int N = (TOTAL + TEAM - 1) / TEAM;
    float4 v[N][2];
#pragma unroll
    for (int j = 0; j < N; ++j) {
        const int e = tid + TEAM * j, row = e / CPR, c16 = e - row * CPR;
        if (e < TOTAL && 8 * c16 < rank && row < rows_here) {
            const float4 *src = reinterpret_cast<const float4 *>(lr + (t0 + row) * rank + 8 * c16);
            v[j][0] = __ldg(src);
            v[j][1] = __ldg(src + 1);
        } else {
            v[j][0] = v[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
        const int e = tid + TEAM * j, row = e / CPR, c16 = e - row * CPR;
        if (e >= TOTAL) continue;
        const float in[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w,
                             v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
        uint32_t ph[4], pm[4], pl[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            float h0, m0, l0, h1, m1, l1;
            split3_bf16(in[2 * h], h0, m0, l0);
            split3_bf16(in[2 * h + 1], h1, m1, l1);
            ph[h] = pack_bf16x2(h0, h1);
            pm[h] = pack_bf16x2(m0, m1);
            pl[h] = pack_bf16x2(l0, l1);
        }
        const int o = kmajor_swz<LB>(row, c16);
        *reinterpret_cast<uint4 *>(dst + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
        *reinterpret_cast<uint4 *>(dst + ROWS * LB + o) = make_uint4(pm[0], pm[1], pm[2], pm[3]);
        *reinterpret_cast<uint4 *>(dst + 2 * ROWS * LB + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    }
}

}  // namespace act
