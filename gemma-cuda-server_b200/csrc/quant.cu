// quant.cu -- NVFP4 activation quantiser for sm_100a (bf16 or fp32 in; e2m1 codes + tile-layout e4m3 scales out)
// and the global-amax reduction that feeds the dynamic global scale.
//
// Replaces the reference's quant_kernel / nvfp4_quantize_activations (kernels/nvfp4_quant.cu:15-57), which is one
// thread per 16-block with sixteen 4-byte loads and scattered single-byte scale stores.  Here:
//   * work unit = one warp-task: 32 blocks = rows {r, r+1} + 32q (q = 0..3) of one 128-row tile, times the 4
//     blocks of one 64-column scale-tile column.  Lane l handles (row 2*rp + l/16 + 32*((l/4)%4), block l%4).
//     With that mapping the 32 scale bytes a warp produces are 32 CONSECUTIVE bytes of the tile layout
//     (tile*512 + rp*32 + lane), so the scale store is one coalesced 32-byte write, and the 4 lanes of each row
//     read 128 contiguous input bytes (bf16) and write 32 contiguous code bytes.
//   * rounding is bit-exact against the reference's float64 numpy quantiser (see common.cuh).
//   * warp-tasks are ordered scale-tile-column fastest, so consecutive warps stream consecutive input columns.
//   * padding rows (m >= M) and padding blocks (b >= K/16) write zero scale bytes; codes only for real data.
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvfp4b {

template <typename T>
struct InputTraits;

template <>
struct InputTraits<uint16_t> {   // bf16 bit patterns: 16 values = 2 x 16-byte loads
    struct Raw { uint4 a, b; };
    static __device__ __forceinline__ void load(const uint16_t* p, Raw& r) {
        r.a = __ldg(reinterpret_cast<const uint4*>(p));
        r.b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    }
    static __device__ __forceinline__ void unpack(const Raw& r, float* v) {
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) { v[2 * i] = bf16lo(w[i]); v[2 * i + 1] = bf16hi(w[i]); }
    }
};

template <>
struct InputTraits<float> {      // fp32: 4 x 16-byte loads
    struct Raw { float4 q[4]; };
    static __device__ __forceinline__ void load(const float* p, Raw& r) {
#pragma unroll
        for (int i = 0; i < 4; ++i) r.q[i] = __ldg(reinterpret_cast<const float4*>(p) + i);
    }
    static __device__ __forceinline__ void unpack(const Raw& r, float* v) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[4 * i] = r.q[i].x; v[4 * i + 1] = r.q[i].y; v[4 * i + 2] = r.q[i].z; v[4 * i + 3] = r.q[i].w;
        }
    }
};

constexpr int kQuantCols = 4;   // scale-tile columns (64 values each) streamed by one warp

// One warp per work item = (row group, chunk of kQuantCols scale-tile columns).  A row group is rows
// {2*rp, 2*rp+1} + 32q (q = 0..3) of one 128-row tile; the warp streams along K, prefetching the next tile
// column's 32 bytes per lane while it encodes the current one.  All index arithmetic is 32-bit except the
// row offset, computed once per item.
template <typename T>
__global__ void __launch_bounds__(256, 4) quantize_kernel(const T* __restrict__ x, int M, int K, float gscale,
                                                          const float* __restrict__ d_amax,
                                                          uint8_t* __restrict__ packed,
                                                          uint8_t* __restrict__ scales, int tile_cols,
                                                          int n_chunks, int n_items) {
    using Tr = InputTraits<T>;
    const int item = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (item >= n_items) return;
    const float g = d_amax ? gscale_from_amax(__ldg(d_amax)) : gscale;
    const int lane = threadIdx.x & 31;
    const int rg = item / n_chunks;
    const int tc0 = (item - rg * n_chunks) * kQuantCols;
    const int tc1 = min(tc0 + kQuantCols, tile_cols);
    const int mt = rg >> 4, rp = rg & 15;
    const int m = mt * 128 + ((lane >> 2) & 3) * 32 + 2 * rp + (lane >> 4);
    const int kb_count = K >> 4;
    const bool row_ok = m < M;
    const T* xrow = x + (size_t)(row_ok ? m : 0) * K + (lane & 3) * 16;
    uint8_t* prow = packed + (size_t)(row_ok ? m : 0) * (K >> 1) + (lane & 3) * 8;
    uint8_t* sf = scales + ((size_t)mt * tile_cols) * 512 + rp * 32 + lane;
    typename Tr::Raw raw;
    bool ok = row_ok && tc0 * 4 + (lane & 3) < kb_count;
    if (ok) Tr::load(xrow + tc0 * 64, raw);
    for (int tc = tc0; tc < tc1; ++tc) {
        typename Tr::Raw nraw;
        const bool nok = tc + 1 < tc1 && row_ok && (tc + 1) * 4 + (lane & 3) < kb_count;
        if (nok) Tr::load(xrow + (tc + 1) * 64, nraw);
        uint32_t b = 0;
        if (ok) {
            float v[16];
            Tr::unpack(raw, v);
            uint32_t w0, w1;
            b = quantize16(v, g, w0, w1);
            *reinterpret_cast<uint2*>(prow + tc * 32) = make_uint2(w0, w1);
        }
        sf[tc * 512] = (uint8_t)b;
        raw = nraw;
        ok = nok;
    }
}

// max |x| over n bf16 values -> atomicMax on the fp32 bit pattern of d_amax (non-negative floats order like
// their bit patterns).  d_amax must hold 0 before the launch.
__global__ void __launch_bounds__(256) amax_bf16_kernel(const uint16_t* __restrict__ x, long long n,
                                                        float* __restrict__ d_amax) {
    uint32_t best = 0;   // max of |bf16| bit patterns, packed two per word
    const long long nvec = n >> 3;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < nvec; i += 4 * stride) {
        uint4 a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = __ldg(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            best = __vmaxu2(best, a[u].x & 0x7FFF7FFFu);
            best = __vmaxu2(best, a[u].y & 0x7FFF7FFFu);
            best = __vmaxu2(best, a[u].z & 0x7FFF7FFFu);
            best = __vmaxu2(best, a[u].w & 0x7FFF7FFFu);
        }
    }
    for (; i < nvec; i += stride) {
        const uint4 a = __ldg(xv + i);
        best = __vmaxu2(best, a.x & 0x7FFF7FFFu);
        best = __vmaxu2(best, a.y & 0x7FFF7FFFu);
        best = __vmaxu2(best, a.z & 0x7FFF7FFFu);
        best = __vmaxu2(best, a.w & 0x7FFF7FFFu);
    }
    for (long long i = (nvec << 3) + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        best = __vmaxu2(best, (uint32_t)(x[i] & 0x7FFFu));
    uint32_t m16 = max(best & 0xFFFFu, best >> 16);
    m16 = __reduce_max_sync(0xFFFFFFFFu, m16);
    if ((threadIdx.x & 31) == 0 && m16 != 0) atomicMax(reinterpret_cast<unsigned int*>(d_amax), m16 << 16);
}

// logical [outer, K/16] -> tile layout; one thread per output byte (padding written as zero).
__global__ void swizzle_kernel(const uint8_t* __restrict__ logical, uint8_t* __restrict__ out, int outer, int kb,
                               int tile_cols, long long total) {
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const long long tile = o >> 9;
        const int within = (int)(o & 511);
        const int tr = (int)(tile / tile_cols), tcol = (int)(tile % tile_cols);
        const int m = tr * 128 + ((within >> 2) & 3) * 32 + (within >> 4);
        const int b = tcol * 4 + (within & 3);
        out[o] = (m < outer && b < kb) ? logical[(long long)m * kb + b] : (uint8_t)0;
    }
}

template <typename T>
static int launch_quantize(const T* x, int M, int K, float gscale, const float* d_amax, uint8_t* packed,
                           uint8_t* scales, void* stream) {
    if (!x || !packed || !scales) return NVFP4B_ERR_NULL;
    if (M <= 0 || K <= 0 || (K & 15)) return NVFP4B_ERR_SHAPE;
    if (!aligned16(x) || !aligned16(packed) || !aligned16(scales)) return NVFP4B_ERR_ALIGN;
    const int tile_cols = (K / 16 + 3) / 4;
    const int n_chunks = (tile_cols + kQuantCols - 1) / kQuantCols;
    const long long n_items = (long long)((M + 127) / 128) * 16 * n_chunks;
    if (n_items > (1ll << 30)) return NVFP4B_ERR_SHAPE;
    const unsigned blocks = (unsigned)((n_items + 7) / 8);
    quantize_kernel<T><<<blocks, 256, 0, (cudaStream_t)stream>>>(x, M, K, gscale, d_amax, packed, scales, tile_cols,
                                                                 n_chunks, (int)n_items);
    return launch_status();
}

}  // namespace nvfp4b

using namespace nvfp4b;

extern "C" int nvfp4b_quantize_bf16(const void* x, int M, int K, float gscale, const float* d_amax, uint8_t* packed,
                                    uint8_t* scales, void* stream) {
    return launch_quantize<uint16_t>(static_cast<const uint16_t*>(x), M, K, gscale, d_amax, packed, scales, stream);
}

extern "C" int nvfp4b_quantize_f32(const float* x, int M, int K, float gscale, const float* d_amax, uint8_t* packed,
                                   uint8_t* scales, void* stream) {
    return launch_quantize<float>(x, M, K, gscale, d_amax, packed, scales, stream);
}

extern "C" int nvfp4b_amax_bf16(const void* x, long long n, float* d_amax, void* stream) {
    if (!x || !d_amax) return NVFP4B_ERR_NULL;
    if (n <= 0) return NVFP4B_ERR_SHAPE;
    if (!aligned16(x)) return NVFP4B_ERR_ALIGN;
    cudaError_t e = cudaMemsetAsync(d_amax, 0, sizeof(float), (cudaStream_t)stream);
    if (e != cudaSuccess) return record_cuda_error(e);
    long long blocks = ((n >> 3) + 255) / 256;
    const long long cap = (long long)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    amax_bf16_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint16_t*>(x), n, d_amax);
    return launch_status();
}

extern "C" int nvfp4b_swizzle_scales(const uint8_t* logical, uint8_t* swizzled, int outer, int K, void* stream) {
    if (!logical || !swizzled) return NVFP4B_ERR_NULL;
    if (outer <= 0 || K <= 0 || (K & 15)) return NVFP4B_ERR_SHAPE;
    const long long total = (long long)scale_bytes(outer, K);
    long long blocks = (total + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    swizzle_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(logical, swizzled, outer, K / 16,
                                                                       (K / 16 + 3) / 4, total);
    return launch_status();
}
