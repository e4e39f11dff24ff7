// tc_gemm.cu -- dense GEMM on the 5th-generation tensor cores (tcgen05).
//
// C[b] = A[b] * B[b] with bf16/fp16 operands and fp32 accumulation in TMEM.
// One CTA computes one 128 x BN output tile, or (large problems) one 256 x 256
// tile as two M = 128 accumulators sharing each B tile:
//   warp 0      TMA producer: 128x64 A (one or two) and BNx64 B tiles
//               (128-byte swizzle) into a 4- or 3-stage shared-memory ring,
//               mbarrier complete_tx;
//   warp 1      TMEM allocator and MMA issuer (one elected thread issues
//               tcgen05.mma M=128 N=BN K=16 per accumulator, commits each stage
//               back to the producer and the finished tile to the epilogue);
//   warps 2..5  epilogue: tcgen05.ld 32x32b (one accumulator row per
//               thread), optional leaky_relu, convert, store.
// Both operands may be K-major or MN-major in global memory; the tile layout
// in shared memory is the canonical 128B-swizzled layout of that major-ness.
// No TMA multicast anywhere.
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace act {

// ------------------------------------------------------------------ tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 3-D tiled map over a (dim2 x dim1 x dim0) tensor of 16-bit elements,
// dim0 contiguous; strides in elements.  box = {box0, box1, 1}.
int make_map_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t dim0,
                uint64_t dim1, uint64_t dim2, uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1,
                CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return ACT_E_CUDA;
    cuuint64_t dims[3] = {dim0, dim1, dim2 ? dim2 : 1};
    cuuint64_t strides[2] = {stride1 * elem_bytes, (dim2 > 1 ? stride2 : stride1 * dim1) * elem_bytes};
    if (strides[1] == 0) strides[1] = strides[0];
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? ACT_OK : ACT_E_CUDA;
}

// The same with a box of {box0, box1, box2}: with dim2 a channel-chunk axis
// (stride 128 bytes) a single copy lands as box2 stacked 128-byte-swizzled
// atom columns of box1 rows.
int make_map_3d_box(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int elem_bytes, uint64_t dim0,
                    uint64_t dim1, uint64_t dim2, uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1,
                    uint32_t box2, CUtensorMapSwizzle sw) {
    auto fn = encode_fn();
    if (!fn) return ACT_E_CUDA;
    cuuint64_t dims[3] = {dim0, dim1, dim2};
    cuuint64_t strides[2] = {stride1 * elem_bytes, stride2 * elem_bytes};
    cuuint32_t box[3] = {box0, box1, box2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? ACT_OK : ACT_E_CUDA;
}

namespace gemm {

constexpr int BM = 128, BK = 64, THREADS = 192;

// MA = 1: one 128 x BN tile per CTA, 4 stages.  MA = 2: a 256 x BN tile as two
// M = 128 accumulators (2 x BN TMEM columns) that share every B tile, so each
// 64-deep K step moves 2 x 16 KB of A and one B tile for twice the MMAs
// (a third less operand traffic per FLOP from L2), 3 stages.
template <int BN, int MA>
struct Smem {
    static constexpr int A_BYTES = BM * BK * 2;  // 16 KB per accumulator
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE = MA * A_BYTES + B_BYTES;
    static constexpr int STAGES = MA == 1 ? 4 : 3;
    static constexpr int TILES = STAGE * STAGES;
    static constexpr int TOTAL = TILES + 1024 /*align slack*/ + 256 /*barriers*/;
};

struct Params {
    int64_t M, N, K;
    int kb2;  // k-blocks of the second segment (0: none)
    int m_tiles, n_tiles;
    int a_mn, b_mn;
    void *C;
    int64_t ldc, sc_batch;
    int c_dtype, activation;
};

template <typename T>
__device__ __forceinline__ T cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__device__ __forceinline__ void store_row32(T *dst, const float (&v)[32], int valid, bool vec_ok) {
    if (valid == 32 && vec_ok) {
        if constexpr (sizeof(T) == 4) {
            float4 *d = reinterpret_cast<float4 *>(dst);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
            uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    T lo = cvt_out<T>(v[8 * i + 2 * j]), hi = cvt_out<T>(v[8 * i + 2 * j + 1]);
                    w[j] = (uint32_t)(*reinterpret_cast<uint16_t *>(&lo)) |
                           ((uint32_t)(*reinterpret_cast<uint16_t *>(&hi)) << 16);
                }
                d[i] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    } else {
        for (int i = 0; i < valid; ++i) dst[i] = cvt_out<T>(v[i]);
    }
}

template <int BN, int MA, typename TOut>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, Params p, int bf16) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using S = Smem<BN, MA>;
    constexpr int STAGES = S::STAGES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::TILES);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Grouped raster: the tiles of a batch are numbered in groups of up to 16
    // M-tiles, M fastest inside a group, so that the CTAs resident at one time
    // cover a compact block of C and share their A rows and B columns in L2
    // (with N fastest every wave would stream all of B).
    int m_t, n_t;
    {
        const int nm = p.m_tiles, nn = p.n_tiles;
        const int id = blockIdx.x;
        const int gsz = 16 * nn;
        const int grp = id / gsz, first = grp * 16;
        const int gm = nm - first < 16 ? nm - first : 16;
        const int in = id - grp * gsz;
        m_t = first + in % gm;
        n_t = in / gm;
    }
    const int n0 = n_t * BN, m0 = m_t * (BM * MA), bz = blockIdx.z;
    const int kb1 = (int)((p.K + BK - 1) / BK);
    const int kblocks = kb1 + p.kb2;  // the second segment's k-blocks follow the first's

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
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

    if (warp == 0 && lane == 0) {
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % STAGES;
            const uint32_t ph = (kb / STAGES) & 1;
            if (!tc::mbar_wait(&empty[s], ph ^ 1, abort)) break;
            uint8_t *a = smem + s * S::STAGE;
            uint8_t *b = a + MA * S::A_BYTES;
            tc::mbar_arrive_expect_tx(&full[s], S::STAGE);
            const bool second = kb >= kb1;
            const CUtensorMap *ma = second ? &tmA2 : &tmA, *mb = second ? &tmB2 : &tmB;
            const int k0 = (second ? kb - kb1 : kb) * BK;
#pragma unroll
            for (int h = 0; h < MA; ++h) {
                uint8_t *ah = a + h * S::A_BYTES;
                const int mh = m0 + BM * h;
                if (!p.a_mn) {
                    tc::tma_load_3d(ah, ma, &full[s], k0, mh, bz);
                } else {
                    tc::tma_load_3d(ah, ma, &full[s], mh, k0, bz);
                    tc::tma_load_3d(ah + 8192, ma, &full[s], mh + 64, k0, bz);
                }
            }
            if (!p.b_mn) {
                tc::tma_load_3d(b, mb, &full[s], k0, n0, bz);
            } else {
#pragma unroll
                for (int j = 0; j < BN / 64; ++j) tc::tma_load_3d(b + j * 8192, mb, &full[s], n0 + 64 * j, k0, bz);
            }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = tc::idesc_f16(BM, BN, bf16 != 0, p.a_mn != 0, p.b_mn != 0);
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % STAGES;
            const uint32_t ph = (kb / STAGES) & 1;
            if (!tc::mbar_wait(&full[s], ph, abort)) break;
            tc::tc_fence_after();
            uint8_t *a = smem + s * S::STAGE;
            uint8_t *b = a + MA * S::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t bd = p.b_mn ? tc::smem_desc(b + kk * 2048, 8192, 1024, tc::SW_128B)
                                           : tc::smem_desc(b + kk * 32, 16, 1024, tc::SW_128B);
#pragma unroll
                for (int h = 0; h < MA; ++h) {
                    uint8_t *ah = a + h * S::A_BYTES;
                    const uint64_t ad = p.a_mn ? tc::smem_desc(ah + kk * 2048, 8192, 1024, tc::SW_128B)
                                               : tc::smem_desc(ah + kk * 32, 16, 1024, tc::SW_128B);
                    tc::mma_f16(tmem + h * BN, ad, bd, idesc, (kb | kk) != 0);
                }
            }
            tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(acc_full);
    } else if (warp >= 2) {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const bool ok = tc::mbar_wait(acc_full, 0, abort);
        tc::tc_fence_after();
        if (ok) {
            TOut *C = reinterpret_cast<TOut *>(p.C) + (int64_t)bz * p.sc_batch;
            const bool vec_ok = ((p.ldc * (int64_t)sizeof(TOut)) % 16 == 0) &&
                                (reinterpret_cast<uintptr_t>(p.C) % 16 == 0) &&
                                ((p.sc_batch * (int64_t)sizeof(TOut)) % 16 == 0);
#pragma unroll 1
            for (int hc = 0; hc < MA * (BN / 32); ++hc) {
                const int h = hc / (BN / 32), c = hc % (BN / 32);
                const int row = m0 + BM * h + q * 32 + lane;
                uint32_t r[32];
                tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + h * BN + c * 32, r);
                tc::tmem_ld_wait();
                const int col = n0 + c * 32;
                if (row >= p.M || col >= p.N) continue;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float x = __uint_as_float(r[i]);
                    if (p.activation == 1) x = x >= 0.f ? x : __fmul_rn(0.01f, x);
                    v[i] = x;
                }
                const int valid = p.N - col < 32 ? (int)(p.N - col) : 32;
                store_row32<TOut>(C + (int64_t)row * p.ldc + col, v, valid, vec_ok);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, BN * MA);
    }
}

}  // namespace gemm

int gemm_launch(const actcomp_gemm_args *g, cudaStream_t stream) {
    using namespace gemm;
    const bool bf16 = g->in_dtype == 0;
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int a_mn = g->a_kmajor ? 0 : 1, b_mn = g->b_kmajor ? 0 : 1;
    const int BN = g->N <= 128 ? 128 : 256;
    // two accumulators per CTA where M fills them and there are enough tiles
    // to keep every SM busy
    const bool two = BN == 256 && g->M > 128 &&
                     ((g->N + 255) / 256) * ((g->M + 255) / 256) * g->batch >= 2 * num_sms();
    CUtensorMap tmA, tmB;
    int st;
    const uint64_t batch = (uint64_t)g->batch;
    // A: K-major -> dims {K, M}; MN-major (K x M stored) -> dims {M, K}
    if (!a_mn)
        st = make_map_3d(&tmA, g->A, dt, 2, g->K, g->M, g->sa_batch ? batch : 1, g->lda, g->sa_batch, 64, 128,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    else
        st = make_map_3d(&tmA, g->A, dt, 2, g->M, g->K, g->sa_batch ? batch : 1, g->lda, g->sa_batch, 64, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    if (!b_mn)
        st = make_map_3d(&tmB, g->B, dt, 2, g->K, g->N, g->sb_batch ? batch : 1, g->ldb, g->sb_batch, 64, BN,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    else
        st = make_map_3d(&tmB, g->B, dt, 2, g->N, g->K, g->sb_batch ? batch : 1, g->ldb, g->sb_batch, 64, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // the second K segment (or, without one, copies of the first maps that are never read)
    CUtensorMap tmA2 = tmA, tmB2 = tmB;
    if (g->K2 > 0) {
        if (!a_mn)
            st = make_map_3d(&tmA2, g->A2, dt, 2, g->K2, g->M, 1, g->lda2, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
        else
            st = make_map_3d(&tmA2, g->A2, dt, 2, g->M, g->K2, 1, g->lda2, 0, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        if (!b_mn)
            st = make_map_3d(&tmB2, g->B2, dt, 2, g->K2, g->N, 1, g->ldb2, 0, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
        else
            st = make_map_3d(&tmB2, g->B2, dt, 2, g->N, g->K2, 1, g->ldb2, 0, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    const int kb2 = g->K2 > 0 ? (int)((g->K2 + 63) / 64) : 0;
    const int m_tiles = (int)((g->M + BM * (two ? 2 : 1) - 1) / (BM * (two ? 2 : 1)));
    const int n_tiles = (int)((g->N + BN - 1) / BN);
    Params p{g->M, g->N, g->K, kb2, m_tiles, n_tiles, a_mn, b_mn, g->C, g->ldc, g->sc_batch, g->c_dtype, g->activation};
    if ((int64_t)m_tiles * n_tiles > INT32_MAX) return ACT_E_UNSUPPORTED;
    dim3 grid((unsigned)(m_tiles * n_tiles), 1, (unsigned)g->batch);
    auto launch = [&](auto kern, int smem) -> int {
        ACT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        kern<<<grid, THREADS, smem, stream>>>(tmA, tmB, tmA2, tmB2, p, bf16 ? 1 : 0);
        return launch_status();
    };
    if (BN == 128) {
        const int smem = Smem<128, 1>::TOTAL;
        if (g->c_dtype == 0) return launch(gemm_kernel<128, 1, float>, smem);
        if (g->c_dtype == 1) return launch(gemm_kernel<128, 1, __nv_bfloat16>, smem);
        return launch(gemm_kernel<128, 1, __half>, smem);
    }
    if (two) {
        const int smem = Smem<256, 2>::TOTAL;
        if (g->c_dtype == 0) return launch(gemm_kernel<256, 2, float>, smem);
        if (g->c_dtype == 1) return launch(gemm_kernel<256, 2, __nv_bfloat16>, smem);
        return launch(gemm_kernel<256, 2, __half>, smem);
    }
    const int smem = Smem<256, 1>::TOTAL;
    if (g->c_dtype == 0) return launch(gemm_kernel<256, 1, float>, smem);
    if (g->c_dtype == 1) return launch(gemm_kernel<256, 1, __nv_bfloat16>, smem);
    return launch(gemm_kernel<256, 1, __half>, smem);
}

}  // namespace act

extern "C" int actcomp_gemm(const actcomp_gemm_args *g, void *stream) {
    using namespace act;
    ACT_CHECK(g && g->A && g->B && g->C, ACT_E_INVALID);
    ACT_CHECK(g->M > 0 && g->N > 0 && g->K > 0 && g->batch >= 1, ACT_E_INVALID);
    ACT_CHECK(g->in_dtype == 0 || g->in_dtype == 1, ACT_E_INVALID);
    ACT_CHECK(g->c_dtype >= 0 && g->c_dtype <= 2 && (g->activation == 0 || g->activation == 1), ACT_E_INVALID);
    ACT_CHECK(g->M <= INT32_MAX && g->N <= INT32_MAX && g->K <= INT32_MAX, ACT_E_UNSUPPORTED);
    // TMA: 16-byte aligned base and row strides
    ACT_CHECK(aligned(g->A, 16) && aligned(g->B, 16), ACT_E_ALIGN);
    ACT_CHECK(g->lda % 8 == 0 && g->ldb % 8 == 0 && g->sa_batch % 8 == 0 && g->sb_batch % 8 == 0, ACT_E_ALIGN);
    ACT_CHECK(g->lda >= (g->a_kmajor ? g->K : g->M) && g->ldb >= (g->b_kmajor ? g->K : g->N), ACT_E_INVALID);
    ACT_CHECK(g->ldc >= g->N, ACT_E_INVALID);
    // a broadcast (stride 0) operand is only supported for batch == 1 maps;
    // otherwise every batched operand needs its own slice
    if (g->batch > 1) ACT_CHECK(g->sa_batch != 0 && g->sb_batch != 0 && g->sc_batch != 0, ACT_E_UNSUPPORTED);
    ACT_CHECK(g->K2 >= 0 && g->K2 <= INT32_MAX, ACT_E_INVALID);
    if (g->K2 > 0) {
        ACT_CHECK(g->batch == 1, ACT_E_UNSUPPORTED);
        ACT_CHECK(g->A2 && g->B2, ACT_E_INVALID);
        ACT_CHECK(aligned(g->A2, 16) && aligned(g->B2, 16) && g->lda2 % 8 == 0 && g->ldb2 % 8 == 0, ACT_E_ALIGN);
        ACT_CHECK(g->lda2 >= (g->a_kmajor ? g->K2 : g->M) && g->ldb2 >= (g->b_kmajor ? g->K2 : g->N), ACT_E_INVALID);
    }
    return gemm_launch(g, as_stream(stream));
}
