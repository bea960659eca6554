// w4a16.cu -- W4A16 kernels behind the reference's fp4_gemv / w4a16_gemm entry points
// (kernels/fp4_gemm.cu:45-111): NVFP4 weights (raw, unswizzled codes [N, K/2] and e4m3 scales [N, K/16], dequant
// = code * e4m3 / w_gscale) times fp16 activations, fp32 out.  Memory-bound on the weight stream.
//
// One warp per output row n.  The fast path (K % 32 == 0, 16-byte aligned rows) streams 16 bytes of codes
// (32 values) per lane per step with an evict-first load, decodes two codes at a time with cvt.rn.f16x2.e2m1x2 and
// accumulates in fp32; the activation rows stay in L1/L2.  Unlike the reference (whose acc[16] limits M to 16,
// kernels/fp4_gemm.cu:86), any M is accepted: rows are processed 8 at a time, re-streaming the weight row per
// group (served from L2 for the small M these entry points are used at).  Other shapes/alignments take a
// byte-granular path with the same arithmetic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvfp4b {

__device__ __forceinline__ float2 e2m1x2_to_float2(uint32_t byte) {
    uint32_t h2;
    asm("{\n\t.reg .b8 q;\n\tmov.b32 {q, _, _, _}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, q;\n\t}" : "=r"(h2) : "r"(byte));
    const __half2 h = *reinterpret_cast<const __half2*>(&h2);
    return __half22float2(h);
}

constexpr int kW4A16Rows = 8;

__global__ void __launch_bounds__(256) w4a16_fast_kernel(float* __restrict__ out, const uint8_t* __restrict__ wp,
                                                         const uint8_t* __restrict__ ws, float inv_g,
                                                         const __half* __restrict__ x, int M, int N, int K) {
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (n >= N) return;
    const uint4* wrow = reinterpret_cast<const uint4*>(wp + (size_t)n * (K / 2));
    const uint16_t* srow = reinterpret_cast<const uint16_t*>(ws + (size_t)n * (K / 16));
    const int chunks = K / 32;
    for (int m0 = 0; m0 < M; m0 += kW4A16Rows) {
        const int mr = min(kW4A16Rows, M - m0);
        float acc[kW4A16Rows];
#pragma unroll
        for (int i = 0; i < kW4A16Rows; ++i) acc[i] = 0.f;
        for (int c = lane; c < chunks; c += 32) {
            const uint4 w = __ldcs(wrow + c);
            const uint32_t s2 = __ldcs(srow + c);
            const float sc0 = e4m3_to_float(s2 & 0xFF) * inv_g, sc1 = e4m3_to_float(s2 >> 8) * inv_g;
            float wv[32];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                    const float2 f = e2m1x2_to_float2((ww[q] >> (8 * bb)) & 0xFF);
                    const float s = (q < 2) ? sc0 : sc1;
                    wv[8 * q + 2 * bb] = f.x * s;
                    wv[8 * q + 2 * bb + 1] = f.y * s;
                }
#pragma unroll
            for (int i = 0; i < kW4A16Rows; ++i) {
                if (i < mr) {
                    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)(m0 + i) * K + (size_t)c * 32);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint4 xv = __ldg(xr + q);
                        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb) {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&xw[bb]));
                            acc[i] = fmaf(wv[8 * q + 2 * bb], f.x, acc[i]);
                            acc[i] = fmaf(wv[8 * q + 2 * bb + 1], f.y, acc[i]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kW4A16Rows; ++i) {
            float v = acc[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
            if (lane == 0 && i < mr) out[(size_t)(m0 + i) * N + n] = v;
        }
    }
}

// M == 1 (the decode GEMV, fp4_gemv): the same arithmetic and summation order as w4a16_fast_kernel at M = 1, with
// one accumulator, so each lane keeps up to four 16-byte weight loads in flight (issued before any is used) at 40
// registers: the weight stream needs several loads in flight per lane to cover DRAM latency, and one load at a time
// left this GEMV at ~1.2 TB/s.  (A persistent variant that also prefetches the warp's next row needs 77 registers
// and measured slower, 1.8 vs 2.05 TB/s.)
__global__ void __launch_bounds__(256) w4a16_gemv_kernel(float* __restrict__ out, const uint8_t* __restrict__ wp,
                                                         const uint8_t* __restrict__ ws, float inv_g,
                                                         const __half* __restrict__ x, int N, int K) {
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (n >= N) return;
    const uint4* wrow = reinterpret_cast<const uint4*>(wp + (size_t)n * (K / 2));
    const uint16_t* srow = reinterpret_cast<const uint16_t*>(ws + (size_t)n * (K / 16));
    const uint4* xv4 = reinterpret_cast<const uint4*>(x);
    const int chunks = K / 32;
    float acc = 0.f;
    for (int cg = lane; cg < chunks; cg += 128) {
        uint4 wq[4];
        uint32_t sq[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = cg + 32 * u;
            wq[u] = c < chunks ? __ldcs(wrow + c) : make_uint4(0, 0, 0, 0);
            sq[u] = c < chunks ? (uint32_t)__ldcs(srow + c) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = cg + 32 * u;
            if (c >= chunks) break;
            const float sc0 = e4m3_to_float(sq[u] & 0xFF) * inv_g, sc1 = e4m3_to_float(sq[u] >> 8) * inv_g;
            const uint32_t ww[4] = {wq[u].x, wq[u].y, wq[u].z, wq[u].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 xq = __ldg(xv4 + (size_t)c * 4 + q);
                const uint32_t xw[4] = {xq.x, xq.y, xq.z, xq.w};
                const float s = (q < 2) ? sc0 : sc1;
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                    const float2 f = e2m1x2_to_float2((ww[q] >> (8 * bb)) & 0xFF);
                    const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xw[bb]));
                    acc = fmaf(f.x * s, xf.x, acc);
                    acc = fmaf(f.y * s, xf.y, acc);
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) out[n] = acc;
}

// Value of one e2m1 code (sign in bit 3) by arithmetic, without the packed conversion instruction.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
    const float m = e2m1_magnitude(c & 7u);
    return (c & 8u) ? -m : m;
}

// Byte-granular path: any alignment of the codes and scales, 2-byte aligned activations, K % 16 == 0.  One
// 16-element block per lane step; codes decoded by arithmetic.
__global__ void __launch_bounds__(256) w4a16_bytes_kernel(float* __restrict__ out, const uint8_t* __restrict__ wp,
                                                          const uint8_t* __restrict__ ws, float inv_g,
                                                          const __half* __restrict__ x, int M, int N, int K) {
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (n >= N) return;
    const uint8_t* wrow = wp + (size_t)n * (K / 2);
    const uint8_t* srow = ws + (size_t)n * (K / 16);
    const int blocks = K / 16;
    for (int m = 0; m < M; ++m) {
        const __half* xr = x + (size_t)m * K;
        float acc = 0.f;
        for (int b = lane; b < blocks; b += 32) {
            const float s = e4m3_to_float(srow[b]) * inv_g;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t c = wrow[8 * b + j];
                acc = fmaf(e2m1_value(c & 0xFu) * s, __half2float(xr[16 * b + 2 * j]), acc);
                acc = fmaf(e2m1_value(c >> 4) * s, __half2float(xr[16 * b + 2 * j + 1]), acc);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (lane == 0) out[(size_t)m * N + n] = acc;
    }
}

int w4a16(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16, int M, int N, int K,
          cudaStream_t s) {
    if (!out || !wp || !ws || !x16) return NVFP4B_ERR_NULL;
    if (M <= 0 || N <= 0 || K <= 0 || (K & 15)) return NVFP4B_ERR_SHAPE;
    if (reinterpret_cast<uintptr_t>(x16) & 1u) return NVFP4B_ERR_ALIGN;
    const float inv_g = 1.0f / w_gscale;
    const dim3 grid((N + 7) / 8);
    const bool fast = (K % 32 == 0) && aligned16(wp) && aligned16(x16) && ((reinterpret_cast<uintptr_t>(ws) & 1) == 0);
    if (fast && M == 1)
        w4a16_gemv_kernel<<<grid, 256, 0, s>>>(out, wp, ws, inv_g, static_cast<const __half*>(x16), N, K);
    else if (fast)
        w4a16_fast_kernel<<<grid, 256, 0, s>>>(out, wp, ws, inv_g, static_cast<const __half*>(x16), M, N, K);
    else
        w4a16_bytes_kernel<<<grid, 256, 0, s>>>(out, wp, ws, inv_g, static_cast<const __half*>(x16), M, N, K);
    return launch_status();
}

}  // namespace nvfp4b

extern "C" int nvfp4b_w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16,
                                 int M, int N, int K, void* stream) {
    return nvfp4b::w4a16(out, wp, ws, w_gscale, x16, M, N, K, (cudaStream_t)stream);
}
