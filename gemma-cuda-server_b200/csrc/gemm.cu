// gemm.cu -- dense W4A4 NVFP4 GEMM entry points on the tcgen05 core (gemm_core.cuh).
//
// Replaces the reference's cuBLASLt call (kernels/fp4_gemm.cu:113-162): D = alpha * A[M,K] @ B[N,K]^T.
// Epilogues: bf16 row-major (the north-star output, alpha fused), fp32 column-major (the reference nvfp4_gemm
// contract, ld = M) and fp32 row-major.
// Tile configurations (one CTA per SM, persistent):
//   TILE_256: 128 x 256 tiles, 4 stages of 54 KB, one TMEM accumulator (256 columns) drained early by 8 epilogue
//             warps.  The MMA reads 12 KB of smem operands per 128-cycle instruction.
//   TILE_128: 128 x 128 tiles, 6 stages of 36 KB, two TMEM accumulators, 4 epilogue warps.  The MMA reads 8 KB
//             per 64-cycle instruction, i.e. it alone saturates shared-memory bandwidth.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gemm.cuh"
#include "gemm_core.cuh"
#include "sm100.cuh"

namespace nvfp4b {

namespace {

// STAGED (bf16 row-major only): each epilogue warp turns its 32-row x 32-column chunks around in a 2 KB
// shared-memory tile (16-byte segments XOR-swizzled by (row >> 1) & 3, conflict-free both ways) so every store
// instruction writes 8 rows x 64 contiguous bytes -- whole sectors -- instead of 32 rows x 16 bytes.
constexpr int kStoreTileBytes = 2048;   // per epilogue warp: one 32 x 32 bf16 tile

template <int OUT, bool STAGED = false>
struct DenseEpi {
    void* d;
    long long ldd;
    int M, N;
    float alpha, b_dequant;
    const float* d_a_amax;

    __device__ __forceinline__ void store_staged(int row0, int n0, int lane, const uint32_t (&r)[32], float a,
                                                 uint8_t* tile) const {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(a * __uint_as_float(r[8 * v + 2 * i]),
                                                               a * __uint_as_float(r[8 * v + 2 * i + 1]));
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
            *reinterpret_cast<uint4*>(tile + lane * 64 + ((v ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
        }
        __syncwarp();
        const int seg = lane & 3;
        const int col = n0 + 8 * seg;
        const bool vec = n0 + 32 <= N && (ldd & 7) == 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int rr = 8 * i + (lane >> 2);
            const uint4 val = *reinterpret_cast<const uint4*>(tile + rr * 64 + ((seg ^ ((rr >> 1) & 3)) << 4));
            const long long m = (long long)row0 + rr;
            if (m >= M) continue;
            __nv_bfloat16* D = static_cast<__nv_bfloat16*>(d) + m * ldd + col;
            if (vec) {
                *reinterpret_cast<uint4*>(D) = val;
            } else {
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&val);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (col + e < N) D[e] = h[e];
            }
        }
        __syncwarp();
    }

    __device__ __forceinline__ void store(long long m, int n0, const uint32_t (&r)[32], float a) const {
        if constexpr (OUT == NVFP4B_OUT_BF16_ROWMAJOR) {
            __nv_bfloat16* D = static_cast<__nv_bfloat16*>(d) + m * ldd + n0;
            if (n0 + 32 <= N && (ldd & 7) == 0) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __nv_bfloat162 h = __floats2bfloat162_rn(a * __uint_as_float(r[8 * v + 2 * i]),
                                                                       a * __uint_as_float(r[8 * v + 2 * i + 1]));
                        w[i] = *reinterpret_cast<const uint32_t*>(&h);
                    }
                    *reinterpret_cast<uint4*>(D + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (n0 + i < N) D[i] = __float2bfloat16_rn(a * __uint_as_float(r[i]));
            }
        } else if constexpr (OUT == NVFP4B_OUT_F32_COLMAJOR) {
            float* D = static_cast<float*>(d) + m;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n0 + i < N) D[(long long)(n0 + i) * ldd] = a * __uint_as_float(r[i]);
        } else {
            float* D = static_cast<float*>(d) + m * ldd + n0;
            if (n0 + 32 <= N && (ldd & 3) == 0) {
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    *reinterpret_cast<float4*>(D + 4 * v) =
                        make_float4(a * __uint_as_float(r[4 * v]), a * __uint_as_float(r[4 * v + 1]),
                                    a * __uint_as_float(r[4 * v + 2]), a * __uint_as_float(r[4 * v + 3]));
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (n0 + i < N) D[i] = a * __uint_as_float(r[i]);
            }
        }
    }

    __device__ __forceinline__ void finish() const {}
    __device__ __forceinline__ bool row_live(const TileInfo&, int) const { return true; }

    template <int CH>
    __device__ __forceinline__ void process(const TileInfo& ti, int row, int col_base, const uint32_t (&r)[CH][32],
                                            uint8_t* esm) const {
        const float a = d_a_amax ? __fdiv_rn(b_dequant, gscale_from_amax(__ldg(d_a_amax))) : alpha;
        if constexpr (STAGED && OUT == NVFP4B_OUT_BF16_ROWMAJOR) {
            const int lane = threadIdx.x & 31;
            uint8_t* tile = esm + ((threadIdx.x >> 5) - 4) * kStoreTileBytes;   // epilogue warps are 4..
            const int row0 = ti.a_row + row - lane;
            if (row0 >= M) return;                                            // warp-uniform
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int n0 = ti.n0 + col_base + 32 * c;                    // warp-uniform
                if (n0 < N) store_staged(row0, n0, lane, r[c], a, tile);
            }
            return;
        }
        const long long m = (long long)ti.a_row + row;
        if (m >= M) return;
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int n0 = ti.n0 + col_base + 32 * c;
            if (n0 < N) store(m, n0, r[c], a);
        }
    }
};

using Tile256 = KCfg<256, 4, 1, 8>;
using Tile128 = KCfg<128, 6, 2, 4>;
using TilePair = PairCfg<5, 8, 8 * kStoreTileBytes>;   // + bf16 store staging tiles

std::atomic<int> g_variant{0};   // 0 = automatic, 1 = TILE_256, 2 = TILE_128, 3 = TILE_PAIR

template <class C, int OUT>
int run_dense(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, const GemmParams& p,
              cudaStream_t stream) {
    CUtensorMap ma, mb;
    int st = make_kmajor_map(&ma, a, p.M, p.K / 2, C::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, b, p.N, p.K / 2, C::BN);
    if (st) return st;
    CoreParams cp;
    cp.err = device_error_ptr();
    if (!cp.err) return NVFP4B_ERR_CUDA;
    cp.sfa = a_sf;
    cp.sfb = b_sf;
    cp.tile_cols = (p.K / 16 + 3) / 4;
    cp.k_tiles = (cp.tile_cols + 3) / 4;
    DenseSched<C::BN> s;
    s.m_tiles = (p.M + C::BM - 1) / C::BM;
    s.n_tiles = (p.N + C::BN - 1) / C::BN;
    s.group_m = 16;
    s.N = p.N;
    s.b_row_tiles = (p.N + 127) / 128;
    s.k_tiles = cp.k_tiles;
    DenseEpi<OUT> e;
    e.d = p.d;
    e.ldd = p.ldd;
    e.M = p.M;
    e.N = p.N;
    e.alpha = p.alpha;
    e.b_dequant = p.b_dequant;
    e.d_a_amax = p.d_a_amax;
    const int tiles = s.m_tiles * s.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    return launch_core<C>(ma, mb, cp, s, e, grid, stream);
}

template <int OUT>
int run_dense_pair(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, const GemmParams& p,
                   cudaStream_t stream) {
    using C = TilePair;
    CUtensorMap ma, mb, msa, msb;
    int st = make_kmajor_map(&ma, a, p.M, p.K / 2, C::BM);
    if (st) return st;
    st = make_kmajor_map(&mb, b, p.N, p.K / 2, C::BN / 2);
    if (st) return st;
    st = make_scale_map(&msa, a_sf, (long long)scale_bytes(p.M, p.K));
    if (st) return st;
    st = make_scale_map(&msb, b_sf, (long long)scale_bytes(p.N, p.K));
    if (st) return st;
    CoreParams cp;
    cp.err = device_error_ptr();
    if (!cp.err) return NVFP4B_ERR_CUDA;
    cp.sfa = a_sf;
    cp.sfb = b_sf;
    cp.tile_cols = (p.K / 16 + 3) / 4;
    cp.k_tiles = (cp.tile_cols + 3) / 4;
    PairDenseSched s;
    s.m_tiles = (p.M + C::PAIR_M - 1) / C::PAIR_M;
    s.n_tiles = (p.N + C::BN - 1) / C::BN;
    s.group_m = 8;
    s.k_tiles = cp.k_tiles;
    DenseEpi<OUT, true> e;
    e.d = p.d;
    e.ldd = p.ldd;
    e.M = p.M;
    e.N = p.N;
    e.alpha = p.alpha;
    e.b_dequant = p.b_dequant;
    e.d_a_amax = p.d_a_amax;
    return launch_pair<C>(ma, mb, msa, msb, cp, s, e, s.m_tiles * s.n_tiles, stream);
}

int dispatch_pair(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, const GemmParams& p,
                  cudaStream_t stream) {
    switch (p.out_kind) {
        case NVFP4B_OUT_BF16_ROWMAJOR: return run_dense_pair<NVFP4B_OUT_BF16_ROWMAJOR>(a, a_sf, b, b_sf, p, stream);
        case NVFP4B_OUT_F32_COLMAJOR: return run_dense_pair<NVFP4B_OUT_F32_COLMAJOR>(a, a_sf, b, b_sf, p, stream);
        case NVFP4B_OUT_F32_ROWMAJOR: return run_dense_pair<NVFP4B_OUT_F32_ROWMAJOR>(a, a_sf, b, b_sf, p, stream);
        default: return NVFP4B_ERR_ARG;
    }
}

template <class C>
int dispatch_out(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, const GemmParams& p,
                 cudaStream_t stream) {
    switch (p.out_kind) {
        case NVFP4B_OUT_BF16_ROWMAJOR: return run_dense<C, NVFP4B_OUT_BF16_ROWMAJOR>(a, a_sf, b, b_sf, p, stream);
        case NVFP4B_OUT_F32_COLMAJOR: return run_dense<C, NVFP4B_OUT_F32_COLMAJOR>(a, a_sf, b, b_sf, p, stream);
        case NVFP4B_OUT_F32_ROWMAJOR: return run_dense<C, NVFP4B_OUT_F32_ROWMAJOR>(a, a_sf, b, b_sf, p, stream);
        default: return NVFP4B_ERR_ARG;
    }
}

}  // namespace

// 2-D K-major tensor map over `rows` rows of `row_bytes` bytes, box = 128 bytes x box_rows, 128-byte swizzle.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static std::atomic<EncodeTiledFn> cached{nullptr};   // host threads may race to fill it (same value)
    EncodeTiledFn enc = cached.load(std::memory_order_acquire);
    if (!enc) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        enc = reinterpret_cast<EncodeTiledFn>(ptr);
        cached.store(enc, std::memory_order_release);
    }
    return enc;
}

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

int make_rows_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes, int box_bytes,
                  int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return record_cuda_error(cudaErrorNotSupported);
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NVFP4B_OK : NVFP4B_ERR_ALIGN;
}

int make_scale_map(CUtensorMap* map, const void* base, long long bytes) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return record_cuda_error(cudaErrorNotSupported);
    cuuint64_t dims[2] = {256u, (cuuint64_t)(bytes / 256)};
    cuuint64_t strides[1] = {256u};
    cuuint32_t box[2] = {256u, 8u};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? NVFP4B_OK : NVFP4B_ERR_ALIGN;
}

int gemm_dense(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, GemmParams p,
               cudaStream_t stream) {
    // Automatic: the CTA-pair tiles whenever there are more rows than one 128-row block (they halve each SM's
    // operand traffic and stage the output through shared memory); 128 x 256 single-CTA tiles otherwise.
    const int sel = g_variant.load(std::memory_order_relaxed);
    const int v = sel != 0 ? sel : (p.M > 128 ? 3 : 1);
    if (v == 3) return dispatch_pair(a, a_sf, b, b_sf, p, stream);
    if (v == 2) return dispatch_out<Tile128>(a, a_sf, b, b_sf, p, stream);
    return dispatch_out<Tile256>(a, a_sf, b, b_sf, p, stream);
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

extern "C" int nvfp4b_gemm_set_tile_config(int config) {
    if (config < 0 || config > 3) return NVFP4B_ERR_ARG;
    g_variant = config;
    return NVFP4B_OK;
}
