// gemm.cu -- W4A4 NVFP4 GEMM on the sm_100a tensor cores (tcgen05.mma kind::mxf4nvf4, e4m3 scale per 16).
//
// Replaces the reference's cuBLASLt call (kernels/fp4_gemm.cu:113-162): D = alpha * A[M,K] @ B[N,K]^T with A, B
// packed e2m1 (K-major) plus e4m3 block scales in the 128x4-tile layout, fp32 accumulation.
//
// Structure (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer: per K-tile of 256 elements, a 2-D tensor load of A (128 rows x 128 B) and B (BN rows
//               x 128 B), both 128-byte swizzled, and 1-D bulk loads of the matching scale tiles.  The scale
//               layout already groups 128 rows x 4 blocks into 512 contiguous bytes and tiles run along K, so the
//               scales of one (128-row, 256-K) block are 2 KB of contiguous global memory.
//   warp 1      TMEM owner and MMA issuer (one thread): copies each stage's scale tiles smem -> TMEM with
//               tcgen05.cp 32x128b.warpx4 (a 512-byte tile is exactly 32 rows x 16 bytes, replicated to the four
//               lane quadrants as the MMA expects), then four 128 x BN x 64 MMAs per stage, and tcgen05.commit to
//               release the stage; a commit per output tile hands the accumulator to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lane quadrant w % 4), multiply by
//               alpha, convert and store.  Two accumulator buffers in TMEM let tile i+1's MMAs run while tile i
//               drains.
// TMEM columns: [0, 2*BN) accumulators, then per pipeline stage 16 columns of A scales + BN/8 columns of B scales.
// Every wait is bounded (sm100::mbar_wait): a stuck pipeline records an error in a device flag and the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemm.cuh"
#include "sm100.cuh"

namespace nvfp4b {

__device__ int g_device_error = 0;

namespace {

using namespace sm100;

template <int BN_, int STAGES_, int ACC_BUFS_>
struct Cfg {
    static constexpr int BM = 128, BN = BN_, STAGES = STAGES_, ACC_BUFS = ACC_BUFS_;
    static constexpr int KT_BYTES = 128;                 // one K-tile = 256 e2m1 values = 128 bytes per row
    static constexpr int A_BYTES = BM * KT_BYTES;        // 16 KB
    static constexpr int B_BYTES = BN * KT_BYTES;
    static constexpr int SFA_BYTES = 4 * 512;            // 4 K-steps of 64 x one 128-row scale tile
    static constexpr int SFB_TILES = BN / 128;
    static constexpr int SFB_BYTES = SFB_TILES * 4 * 512;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr int SF_COLS_A = 16, SF_COLS_B = 4 * (BN / 32);
    static constexpr int TMEM_COLS_USED = ACC_BUFS * BN + STAGES * (SF_COLS_A + SF_COLS_B);
    static constexpr int TMEM_COLS = 512;
    static constexpr int BAR_BYTES = (2 * STAGES + 2 * ACC_BUFS) * 8 + 16;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    static_assert(TMEM_COLS_USED <= TMEM_COLS, "TMEM budget");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(BN % 128 == 0 && BN <= 256, "BN");
};

template <int OUT>
__device__ __forceinline__ void store_chunk(const GemmParams& p, long long m, int n0, const uint32_t (&r)[32],
                                            float alpha) {
    if (m >= p.M) return;
    if constexpr (OUT == NVFP4B_OUT_BF16_ROWMAJOR) {
        __nv_bfloat16* D = static_cast<__nv_bfloat16*>(p.d) + m * p.ldd + n0;
        if (n0 + 32 <= p.N && (p.ldd & 7) == 0) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __nv_bfloat162 h = __floats2bfloat162_rn(alpha * __uint_as_float(r[8 * v + 2 * i]),
                                                                   alpha * __uint_as_float(r[8 * v + 2 * i + 1]));
                    w[i] = *reinterpret_cast<const uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(D + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) D[i] = __float2bfloat16_rn(alpha * __uint_as_float(r[i]));
        }
    } else if constexpr (OUT == NVFP4B_OUT_F32_COLMAJOR) {
        float* D = static_cast<float*>(p.d) + m;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (n0 + i < p.N) D[(long long)(n0 + i) * p.ldd] = alpha * __uint_as_float(r[i]);
    } else {
        float* D = static_cast<float*>(p.d) + m * p.ldd + n0;
        if (n0 + 32 <= p.N && (p.ldd & 3) == 0) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
                *reinterpret_cast<float4*>(D + 4 * v) =
                    make_float4(alpha * __uint_as_float(r[4 * v]), alpha * __uint_as_float(r[4 * v + 1]),
                                alpha * __uint_as_float(r[4 * v + 2]), alpha * __uint_as_float(r[4 * v + 3]));
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < p.N) D[i] = alpha * __uint_as_float(r[i]);
        }
    }
}

template <class C, int OUT>
__global__ void __launch_bounds__(192, 1)
    gemm_nvf4_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + C::STAGES * C::A_BYTES;
    uint8_t* sSFA = sB + C::STAGES * C::B_BYTES;
    uint8_t* sSFB = sSFA + C::STAGES * C::SFA_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + C::STAGES * C::SFB_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + C::ACC_BUFS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + C::ACC_BUFS);
    volatile int* sflag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < C::ACC_BUFS; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 128); }
        *sflag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tma_a); prefetch_tmap(&tma_b); }
    if (warp == 1) { tmem_alloc(tmem_slot, C::TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int num_tiles = p.m_tiles * p.n_tiles;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int mb = t % p.m_tiles, nb = t / p.m_tiles;
                for (int kt = 0; kt < p.k_tiles; ++kt) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, sflag, kErrTimeoutProducer)) { ok = false; break; }
                    const int ks0 = kt * 4;
                    const int nks = min(4, p.ksteps - ks0);
                    const uint32_t sf_bytes = (uint32_t)nks * 512u;
                    int b_tiles = 0;
#pragma unroll
                    for (int h = 0; h < C::SFB_TILES; ++h) b_tiles += (nb * C::SFB_TILES + h < p.b_row_tiles);
                    mbar_arrive_expect_tx(&full[stage],
                                          (uint32_t)(C::A_BYTES + C::B_BYTES) + sf_bytes * (1u + (uint32_t)b_tiles));
                    tma_load_2d(sA + stage * C::A_BYTES, &tma_a, &full[stage], kt * C::KT_BYTES, mb * C::BM);
                    tma_load_2d(sB + stage * C::B_BYTES, &tma_b, &full[stage], kt * C::KT_BYTES, nb * C::BN);
                    bulk_load(sSFA + stage * C::SFA_BYTES, p.sfa + ((long long)mb * p.tile_cols + ks0) * 512,
                              sf_bytes, &full[stage]);
#pragma unroll
                    for (int h = 0; h < C::SFB_TILES; ++h) {
                        const int rt = nb * C::SFB_TILES + h;
                        if (rt < p.b_row_tiles)
                            bulk_load(sSFB + stage * C::SFB_BYTES + h * 2048,
                                      p.sfb + ((long long)rt * p.tile_cols + ks0) * 512, sf_bytes, &full[stage]);
                    }
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0, abuf = 0;
            uint32_t phase = 0, aphase = 0;
            bool ok = true;
            const uint32_t idesc = idesc_nvf4(C::BM, C::BN);
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(&tempty[abuf], aphase ^ 1u, sflag, kErrTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(abuf * C::BN);
                for (int kt = 0; kt < p.k_tiles; ++kt) {
                    if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                    tc_fence_after();
                    const int nks = min(4, p.ksteps - kt * 4);
                    const uint32_t sfa_col =
                        tmem + (uint32_t)(C::ACC_BUFS * C::BN + stage * (C::SF_COLS_A + C::SF_COLS_B));
                    const uint32_t sfb_col = sfa_col + C::SF_COLS_A;
                    const uint32_t a_base = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * C::B_BYTES);
                    const uint32_t sfa_base = smem_u32(sSFA + stage * C::SFA_BYTES);
                    const uint32_t sfb_base = smem_u32(sSFB + stage * C::SFB_BYTES);
                    for (int j = 0; j < nks; ++j) {
                        tmem_cp_32x128b_x4(sfa_col + 4 * j, desc_sf_32x16(sfa_base + j * 512));
#pragma unroll
                        for (int h = 0; h < C::SFB_TILES; ++h)
                            tmem_cp_32x128b_x4(sfb_col + (C::BN / 32) * j + 4 * h,
                                               desc_sf_32x16(sfb_base + h * 2048 + j * 512));
                    }
                    for (int j = 0; j < nks; ++j)
                        mma_nvf4(d_tmem, desc_kmajor_sw128(a_base + 32 * j), desc_kmajor_sw128(b_base + 32 * j),
                                 idesc, sfa_col + 4 * j, sfb_col + (C::BN / 32) * j, (kt | j) != 0 ? 1u : 0u);
                    tc_commit(&empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(&tfull[abuf]);
                if (++abuf == C::ACC_BUFS) { abuf = 0; aphase ^= 1u; }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quad = warp & 3;
        int abuf = 0;
        uint32_t aphase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const int mb = t % p.m_tiles, nb = t / p.m_tiles;
            if (!mbar_wait(&tfull[abuf], aphase, sflag, kErrTimeoutEpilogue)) break;
            tc_fence_after();
            const float alpha = p.d_a_amax ? __fdiv_rn(p.b_dequant, gscale_from_amax(__ldg(p.d_a_amax))) : p.alpha;
            const long long m = (long long)mb * C::BM + quad * 32 + lane;
            const uint32_t row_addr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(abuf * C::BN);
#pragma unroll 1
            for (int c = 0; c < C::BN; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(row_addr + c, r);
                tmem_wait_ld();
                store_chunk<OUT>(p, m, nb * C::BN + c, r, alpha);
            }
            tc_fence_before();
            mbar_arrive(&tempty[abuf]);
            if (++abuf == C::ACC_BUFS) { abuf = 0; aphase ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if (threadIdx.x == 0 && *sflag != 0) atomicCAS(&g_device_error, 0, *sflag);
}

// ---- host side -------------------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

template <class C, int OUT>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, cudaStream_t stream) {
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_nvf4_kernel<C, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::SMEM_BYTES);
        if (e != cudaSuccess) return record_cuda_error(e);
        attr_done[dev] = true;
    }
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_nvf4_kernel<C, OUT><<<grid, 192, C::SMEM_BYTES, stream>>>(ma, mb, p);
    return launch_status();
}

}  // namespace

// 2-D K-major tensor map over `rows` rows of `row_bytes` bytes, box = 128 bytes x box_rows, 128-byte swizzle.
int make_kmajor_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return record_cuda_error(cudaErrorNotSupported);
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NVFP4B_OK : NVFP4B_ERR_ALIGN;
}

int gemm_dense(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, GemmParams p,
               cudaStream_t stream) {
    using C = Cfg<128, 6, 2>;
    CUtensorMap ma, mb;
    int st = make_kmajor_map(&ma, a, p.M, p.K / 2, C::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, b, p.N, p.K / 2, C::BN);
    if (st) return st;
    p.sfa = a_sf;
    p.sfb = b_sf;
    p.m_tiles = (p.M + C::BM - 1) / C::BM;
    p.n_tiles = (p.N + C::BN - 1) / C::BN;
    p.tile_cols = (p.K / 16 + 3) / 4;
    p.ksteps = p.tile_cols;
    p.k_tiles = (p.ksteps + 3) / 4;
    p.b_row_tiles = (p.N + 127) / 128;
    switch (p.out_kind) {
        case NVFP4B_OUT_BF16_ROWMAJOR: return launch_gemm<C, NVFP4B_OUT_BF16_ROWMAJOR>(ma, mb, p, stream);
        case NVFP4B_OUT_F32_COLMAJOR: return launch_gemm<C, NVFP4B_OUT_F32_COLMAJOR>(ma, mb, p, stream);
        case NVFP4B_OUT_F32_ROWMAJOR: return launch_gemm<C, NVFP4B_OUT_F32_ROWMAJOR>(ma, mb, p, stream);
        default: return NVFP4B_ERR_ARG;
    }
}

}  // namespace nvfp4b

using namespace nvfp4b;

extern "C" int nvfp4b_gemm(const uint8_t* a, const uint8_t* a_scales, float a_dequant, const float* d_a_amax,
                           const uint8_t* b, const uint8_t* b_scales, float b_dequant, int M, int N, int K, void* d,
                           int out_kind, long long ldd, void* stream) {
    if (!a || !a_scales || !b || !b_scales || !d) return NVFP4B_ERR_NULL;
    if (M <= 0 || N <= 0 || K <= 0 || (K & 31)) return NVFP4B_ERR_SHAPE;
    if (out_kind < 0 || out_kind > 2) return NVFP4B_ERR_ARG;
    if (out_kind == NVFP4B_OUT_F32_COLMAJOR ? ldd < M : ldd < N) return NVFP4B_ERR_SHAPE;
    if (!aligned16(a) || !aligned16(b) || !aligned16(a_scales) || !aligned16(b_scales)) return NVFP4B_ERR_ALIGN;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.alpha = a_dequant * b_dequant;
    p.b_dequant = b_dequant;
    p.d_a_amax = d_a_amax;
    p.d = d;
    p.ldd = ldd;
    p.out_kind = out_kind;
    return gemm_dense(a, a_scales, b, b_scales, p, (cudaStream_t)stream);
}

extern "C" int nvfp4b_read_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return NVFP4B_ERR_CUDA;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));
    }
    return v;
}
