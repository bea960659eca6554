// quant.cu -- NVFP4 activation quantiser for sm_100a (bf16 or fp32 in; e2m1 codes + tile-layout e4m3 scales out)
// and the global-amax reduction that feeds the dynamic global scale.
//
// Replaces the reference's quant_kernel / nvfp4_quantize_activations (kernels/nvfp4_quant.cu:15-57), which is one
// thread per 16-block with sixteen 4-byte loads and scattered single-byte scale stores.  Here:
//   * bf16 input: one warp per row, each lane quantising two blocks per step from two pairs of 16-byte loads (a
//     warp reads 2 KB of contiguous row per step, writes 512 contiguous code bytes); fp32 input: work item = (row,
//     32 consecutive blocks), persistent warps prefetching the next item.  Scale bytes land in runs of 4
//     consecutive bytes of the 128x4-tile layout.
//   * rounding is bit-exact against the reference's float64 numpy quantiser (see common.cuh); the per-element
//     encode is straight-line with one exactness check per block.
//   * padding rows (m >= M, up to the 128-row tile) and padding blocks (b >= K/16, up to the 4-block tile column)
//     write zero scale bytes, so the whole scale buffer is written every call.
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvfp4b {

template <typename T>
struct InputTraits;

template <>
struct InputTraits<float> {      // fp32: 4 x 16-byte loads
    struct Raw { float4 q[4]; };
    static __device__ __forceinline__ void load(const float* p, Raw& r) {
#pragma unroll
        for (int i = 0; i < 4; ++i) r.q[i] = __ldg(reinterpret_cast<const float4*>(p) + i);
    }
    static __device__ __forceinline__ uint32_t quantize(const Raw& r, float g, uint32_t& w0, uint32_t& w1) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[4 * i] = r.q[i].x; v[4 * i + 1] = r.q[i].y; v[4 * i + 2] = r.q[i].z; v[4 * i + 3] = r.q[i].w;
        }
        return quantize16(v, g, w0, w1);
    }
};

// fp32 input.  Work item = (row, 32 consecutive 16-element blocks): a warp's loads are 2 KB of contiguous fp32.  Rows are padded
// to the 128-row tile and blocks to the 4-block tile column; padding lanes only write a zero scale byte.  Warps are
// persistent (grid = 8 blocks per SM) and walk items with a stride, loading the next item while encoding the current
// one, so every lane keeps 64 bytes in flight.  Scale bytes go to the tile layout (4 consecutive lanes -> 4
// consecutive bytes).
template <typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, int M, int K, float gscale,
                                                       const float* __restrict__ d_amax,
                                                       uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                                                       int tile_cols, int chunks_per_row, int n_items) {
    using Tr = InputTraits<T>;
    const int lane = threadIdx.x & 31;
    const int warps = (int)((gridDim.x * blockDim.x) >> 5);
    int item = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    if (item >= n_items) return;
    const float g = d_amax ? gscale_from_amax(__ldg(d_amax)) : gscale;
    const int kb = K >> 4, bmax = tile_cols * 4;
    int m = item / chunks_per_row;
    int b = (item - m * chunks_per_row) * 32 + lane;
    bool ok = m < M && b < kb;
    typename Tr::Raw raw;
    if (ok) Tr::load(x + (size_t)m * K + b * 16, raw);
    while (true) {
        const int nitem = item + warps;
        const bool more = nitem < n_items;
        int nm = 0, nb = 0;
        bool nok = false;
        typename Tr::Raw nraw;
        if (more) {
            nm = nitem / chunks_per_row;
            nb = (nitem - nm * chunks_per_row) * 32 + lane;
            nok = nm < M && nb < kb;
            if (nok) Tr::load(x + (size_t)nm * K + nb * 16, nraw);
        }
        if (b < bmax) {
            uint32_t sf = 0;
            if (ok) {
                uint32_t w0, w1;
                sf = Tr::quantize(raw, g, w0, w1);
                *reinterpret_cast<uint2*>(packed + (size_t)m * (K >> 1) + b * 8) = make_uint2(w0, w1);
            }
            scales[((size_t)(m >> 7) * tile_cols + (b >> 2)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (b & 3)] =
                (uint8_t)sf;
        }
        if (!more) break;
        item = nitem;
        m = nm;
        b = nb;
        ok = nok;
        raw = nraw;
    }
}

// bf16 input, one warp per row (grid-stride over the rows padded to the 128-row tile): lane l takes blocks l and
// l + 32 of each 64-block step, i.e. each step reads 2 KB of contiguous row as two 1 KB warp-wide runs, both loads
// issued before either block is encoded.  Codes go out as 8-byte stores (a warp writes 256 contiguous bytes per
// block set); scale bytes go to the tile layout (4 consecutive lanes -> 4 consecutive bytes).  Padding rows and
// padding blocks only write zero scale bytes.  No integer division: rows advance by the warp count.
// Each block is first encoded by the straight-line bracket path (quantize16_bf16_fast, no branches); a block it
// cannot prove (~1-3% of blocks: an element, or the block scale, within 2^-20 of a rounding boundary) is noted in the
// lane's mask and, after the row, the warp's noted blocks are redone by the exact path (quantize16_bf16) one per
// lane, in parallel, over a per-warp list in shared memory -- instead of the whole warp idling on the divergent exact
// path of one lane at every step.  The redo overwrites the block's codes and scale (the warp barrier orders the two
// stores).
constexpr int kQuantRowsBlock = 256;
constexpr int kQuantBPL = 2;                  // blocks per lane per step: a warp-step covers 32 * kQuantBPL blocks
constexpr int kFixSteps = 32 / kQuantBPL;     // steps whose flags one 32-bit lane mask holds

__global__ void __launch_bounds__(kQuantRowsBlock, 4) quantize_bf16_rows_kernel(const uint16_t* __restrict__ x, int M,
                                                                             int K, float gscale,
                                                                             const float* __restrict__ d_amax,
                                                                             uint8_t* __restrict__ packed,
                                                                             uint8_t* __restrict__ scales,
                                                                             int tile_cols, int rows_padded) {
    __shared__ int fix_list[kQuantRowsBlock / 32][32 * 32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int warps = (int)((gridDim.x * blockDim.x) >> 5);
    const float g = d_amax ? gscale_from_amax(__ldg(d_amax)) : gscale;
    const int kb = K >> 4, bmax = tile_cols * 4;
    constexpr int kStep = 32 * kQuantBPL;
    int* list = fix_list[wid];
    for (int m = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); m < rows_padded; m += warps) {
        const bool real = m < M;
        const uint16_t* xr = x + (size_t)(real ? m : 0) * K;
        uint8_t* pr = packed + (size_t)(real ? m : 0) * (K >> 1);
        uint8_t* sr = scales + (size_t)(m >> 7) * tile_cols * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4;
        for (int s0 = 0; s0 < bmax; s0 += kStep * kFixSteps) {
            uint32_t mask = 0;     // bit kQuantBPL * i + j: block j of step i needs the exact path
            const int s1 = min(bmax, s0 + kStep * kFixSteps);
            for (int b0 = s0; b0 < s1; b0 += kStep) {
                uint4 q[kQuantBPL][2];
#pragma unroll
                for (int j = 0; j < kQuantBPL; ++j) {       // every load of the step before any encode
                    const int b = b0 + lane + 32 * j;
                    q[j][0] = q[j][1] = make_uint4(0, 0, 0, 0);
                    if (real && b < kb) {
                        q[j][0] = __ldg(reinterpret_cast<const uint4*>(xr + b * 16));
                        q[j][1] = __ldg(reinterpret_cast<const uint4*>(xr + b * 16) + 1);
                    }
                }
                const int step = (b0 - s0) / kStep;
#pragma unroll
                for (int j = 0; j < kQuantBPL; ++j) {
                    const int b = b0 + lane + 32 * j;
                    if (b >= bmax) continue;
                    uint32_t sf = 0;
                    if (real && b < kb) {
                        const uint32_t w[8] = {q[j][0].x, q[j][0].y, q[j][0].z, q[j][0].w,
                                               q[j][1].x, q[j][1].y, q[j][1].z, q[j][1].w};
                        uint32_t k0, k1;
                        sf = quantize16_bf16_fast(w, g, k0, k1);
                        *reinterpret_cast<uint2*>(pr + b * 8) = make_uint2(k0, k1);
                        mask |= (sf >> 8) << (kQuantBPL * step + j);
                    }
                    sr[(b >> 2) * 512 + (b & 3)] = (uint8_t)sf;
                }
            }
            // cooperative exact redo of the noted blocks of these steps
            const int cnt = __popc(mask);
            int incl = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += u;
            }
            const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
            if (total == 0) continue;                 // warp-uniform
            int pos = incl - cnt;
            while (mask) {
                const int bit = __ffs(mask) - 1;
                mask &= mask - 1;
                list[pos++] = s0 + (bit / kQuantBPL) * kStep + lane + (bit % kQuantBPL) * 32;
            }
            __syncwarp();
            for (int i = lane; i < total; i += 32) {
                const int b = list[i];
                const uint4 q0 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16));
                const uint4 q1 = __ldg(reinterpret_cast<const uint4*>(xr + b * 16) + 1);
                const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                uint32_t k0, k1;
                const uint32_t sf = quantize16_bf16(w, g, k0, k1);
                *reinterpret_cast<uint2*>(pr + b * 8) = make_uint2(k0, k1);
                sr[(b >> 2) * 512 + (b & 3)] = (uint8_t)sf;
            }
            __syncwarp();
        }
    }
}

// max |x| over n bf16 values -> d_amax (fp32 bit pattern; non-negative floats order like their bit patterns).
// Each thread keeps 8 independent 16-byte loads in flight (default caching, so the quantiser that reads x next finds
// it in the L2); the block reduces in shared memory and issues ONE atomicMax
// (same-address atomics serialise at the L2, so per-warp atomics would dominate).  d_amax must hold 0.  A streaming
// read of this shape measured 5.4 TB/s with 4 blocks of 256 threads per SM and 8 loads in flight per thread.
constexpr int kAmaxUnroll = 8;
__global__ void __launch_bounds__(256) amax_bf16_kernel(const uint16_t* __restrict__ x, long long n,
                                                        float* __restrict__ d_amax) {
    __shared__ uint32_t red[8];
    uint32_t best = 0;   // max of |bf16| bit patterns, packed two per word
    const long long nvec = n >> 3;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (kAmaxUnroll - 1) * stride < nvec; i += kAmaxUnroll * stride) {
        uint4 a[kAmaxUnroll];
#pragma unroll
        for (int u = 0; u < kAmaxUnroll; ++u) a[u] = __ldg(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < kAmaxUnroll; ++u) {
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
    for (long long k = (nvec << 3) + (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride)
        best = __vmaxu2(best, (uint32_t)(x[k] & 0x7FFFu));
    uint32_t m16 = max(best & 0xFFFFu, best >> 16);
    m16 = __reduce_max_sync(0xFFFFFFFFu, m16);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m16;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
        v = __reduce_max_sync(0xFFFFFFFFu, v);
        if (threadIdx.x == 0 && v != 0) atomicMax(reinterpret_cast<unsigned int*>(d_amax), v << 16);
    }
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
    const int chunks_per_row = (tile_cols * 4 + 31) / 32;
    const int rows_padded = (M + 127) / 128 * 128;
    const long long n_items = (long long)rows_padded * chunks_per_row;
    if (n_items > (1ll << 30)) return NVFP4B_ERR_SHAPE;
    long long blocks = (n_items + 7) / 8;
    const long long cap = (long long)sm_count() * 8;
    if constexpr (sizeof(T) == 2) {
        long long rb = (rows_padded + 7) / 8;                      // 8 warps (rows) per block
        if (rb > cap) rb = cap;
        quantize_bf16_rows_kernel<<<(unsigned)rb, kQuantRowsBlock, 0, (cudaStream_t)stream>>>(
            x, M, K, gscale, d_amax, packed, scales, tile_cols, rows_padded);
    } else {
        if (blocks > cap) blocks = cap;
        quantize_kernel<T><<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(x, M, K, gscale, d_amax, packed,
                                                                               scales, tile_cols, chunks_per_row,
                                                                               (int)n_items);
    }
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
    long long blocks = ((n >> 3) + 256 * kAmaxUnroll - 1) / (256 * kAmaxUnroll);
    const long long cap = (long long)sm_count() * 4;
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
