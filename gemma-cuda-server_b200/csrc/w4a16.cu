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

// ---- tensor-core form for M <= 8 (the decode GEMV and small batches) ---------------------------------------------
// out[m, n] = inv_g * sum_k (e2m1 * e4m3)[n, k] * x[m, k], on mma.sync m16n8k16 (fp16 x fp16 -> fp32): the weight
// rows are the MMA's M dimension (16 per warp), the activation rows its N dimension (8; rows >= M are zero).  A weight
// times its block scale is exact in fp16 (at most 2 x 4 significant bits, |value| <= 6 * 448, >= 2^-10), every fp16
// product is exact in fp32 and the sums are fp32, so the result has the fp32-accumulation accuracy of the FFMA
// kernels with ~3x fewer instructions per weight (the scalar forms are issue-bound at ~2 TB/s on the lm_head shape).
// Inside each 128-wide chunk of K, lane (g, q) = (lane / 4, lane % 4) owns codes [32q, 32q + 32) of weight rows g and
// g + 8: for the j-th MMA of the chunk its fragment slots k = {2q, 2q + 1, 2q + 8, 2q + 9} carry its codes
// {4j, 4j + 1, 4j + 2, 4j + 3}.  Every lane with the same q maps a slot to the same K index, so the activation
// fragment (lane (g, q) holds token g at those slots) uses the same permutation and the contraction is unchanged.

__device__ __forceinline__ uint32_t e2m1x2_to_half2(uint32_t byte) {
    uint32_t h2;
    asm("{\n\t.reg .b8 q;\n\tmov.b32 {q, _, _, _}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, q;\n\t}" : "=r"(h2) : "r"(byte));
    return h2;
}

// (s, s) as f16x2 for an e4m3 scale byte (exact: every e4m3 value is an f16).
__device__ __forceinline__ uint32_t e4m3_to_half2x(uint32_t b) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((unsigned short)((b & 0xFFu) | ((b & 0xFFu) << 8))));
    return h2;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct W4a16Piece {
    uint4 ca, cb;        // 16 bytes of codes of rows g and g + 8
    uint32_t sa, sb;     // their two scale bytes
    uint4 x[4];          // 32 fp16 activations of token g
};

__device__ __forceinline__ void w4a16_load_piece(W4a16Piece& p, const uint8_t* wa, const uint8_t* wb,
                                                 const uint8_t* sa, const uint8_t* sb, const __half* xr, int k0,
                                                 bool kv, bool va, bool vb, bool xm) {
    p.ca = p.cb = make_uint4(0, 0, 0, 0);
    p.sa = p.sb = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) p.x[i] = make_uint4(0, 0, 0, 0);
    if (!kv) return;
    if (va) {
        p.ca = __ldcs(reinterpret_cast<const uint4*>(wa + k0 / 2));
        p.sa = __ldcs(reinterpret_cast<const uint16_t*>(sa + k0 / 16));
    }
    if (vb) {
        p.cb = __ldcs(reinterpret_cast<const uint4*>(wb + k0 / 2));
        p.sb = __ldcs(reinterpret_cast<const uint16_t*>(sb + k0 / 16));
    }
    if (xm)
#pragma unroll
        for (int i = 0; i < 4; ++i) p.x[i] = __ldg(reinterpret_cast<const uint4*>(xr + k0) + i);
}

__device__ __forceinline__ void w4a16_mma_piece(float (&d)[4], const W4a16Piece& p) {
    const uint32_t ca[4] = {p.ca.x, p.ca.y, p.ca.z, p.ca.w}, cb[4] = {p.cb.x, p.cb.y, p.cb.z, p.cb.w};
    const uint32_t xw[16] = {p.x[0].x, p.x[0].y, p.x[0].z, p.x[0].w, p.x[1].x, p.x[1].y, p.x[1].z, p.x[1].w,
                             p.x[2].x, p.x[2].y, p.x[2].z, p.x[2].w, p.x[3].x, p.x[3].y, p.x[3].z, p.x[3].w};
    const uint32_t sa0 = e4m3_to_half2x(p.sa), sa1 = e4m3_to_half2x(p.sa >> 8);
    const uint32_t sb0 = e4m3_to_half2x(p.sb), sb1 = e4m3_to_half2x(p.sb >> 8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t wa = ca[j >> 1] >> (16 * (j & 1)), wb = cb[j >> 1] >> (16 * (j & 1));
        const uint32_t s_a = j < 4 ? sa0 : sa1, s_b = j < 4 ? sb0 : sb1;
        mma_16816(d, hmul2_u32(e2m1x2_to_half2(wa & 0xFFu), s_a), hmul2_u32(e2m1x2_to_half2(wb & 0xFFu), s_b),
                  hmul2_u32(e2m1x2_to_half2((wa >> 8) & 0xFFu), s_a), hmul2_u32(e2m1x2_to_half2((wb >> 8) & 0xFFu), s_b),
                  xw[2 * j], xw[2 * j + 1]);
    }
}

constexpr int kW4A16MmaMaxM = 8;

__global__ void __launch_bounds__(256) w4a16_mma_kernel(float* __restrict__ out, const uint8_t* __restrict__ wp,
                                                        const uint8_t* __restrict__ ws, float inv_g,
                                                        const __half* __restrict__ x, int M, int N, int K) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int n0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 16;
    if (n0 >= N) return;
    const int ra = n0 + g, rb = n0 + g + 8;
    const bool va = ra < N, vb = rb < N, xm = g < M;
    const uint8_t* wa = wp + (size_t)(va ? ra : 0) * (K / 2);
    const uint8_t* wb = wp + (size_t)(vb ? rb : 0) * (K / 2);
    const uint8_t* sa = ws + (size_t)(va ? ra : 0) * (K / 16);
    const uint8_t* sb = ws + (size_t)(vb ? rb : 0) * (K / 16);
    const __half* xr = x + (size_t)(xm ? g : 0) * K;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    const int chunks = (K + 127) / 128;
    W4a16Piece cur, nxt;
    w4a16_load_piece(cur, wa, wb, sa, sb, xr, q * 32, q * 32 < K, va, vb, xm);
    for (int c = 0; c < chunks; ++c) {         // the next chunk's loads are issued before this chunk's MMAs
        const int k1 = (c + 1) * 128 + q * 32;
        w4a16_load_piece(nxt, wa, wb, sa, sb, xr, k1, c + 1 < chunks && k1 < K, va, vb, xm);
        w4a16_mma_piece(d, cur);
        cur = nxt;
    }
    const int m0 = 2 * q, m1 = 2 * q + 1;
    if (va) {
        if (m0 < M) out[(size_t)m0 * N + ra] = d[0] * inv_g;
        if (m1 < M) out[(size_t)m1 * N + ra] = d[1] * inv_g;
    }
    if (vb) {
        if (m0 < M) out[(size_t)m0 * N + rb] = d[2] * inv_g;
        if (m1 < M) out[(size_t)m1 * N + rb] = d[3] * inv_g;
    }
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
    if (fast && M <= kW4A16MmaMaxM && ((reinterpret_cast<uintptr_t>(ws) & 1) == 0))
        w4a16_mma_kernel<<<(unsigned)((N + 127) / 128), 256, 0, s>>>(out, wp, ws, inv_g,
                                                                     static_cast<const __half*>(x16), M, N, K);
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
