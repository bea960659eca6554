// w4a16.cu -- W4A16 kernels behind the reference's fp4_gemv / w4a16_gemm entry points
// (kernels/fp4_gemm.cu:45-111): NVFP4 weights (raw, unswizzled codes [N, K/2] and e4m3 scales [N, K/16], dequant
// = code * e4m3 / w_gscale) times fp16 activations, fp32 out.  Memory-bound on the weight stream.
//
// The fast shapes (K % 32 == 0, 16-byte aligned codes and activations) run on the tensor cores: mma.sync m16n8k16
// over exact fp16 weight x scale products, 16 weight rows per warp, fp32 accumulation.  Three feeds of the weights:
// TMA into a shared-memory ring (M <= 2, K % 256 == 0: the decode GEMV), registers (M <= 8), and a per-lane cp.async
// ring in passes of 16 activation rows (larger M, K % 64 == 0; the reference's acc[16] limits M to 16,
// kernels/fp4_gemm.cu:86, here any M).  The remaining fast shapes take one warp per output row with FFMA
// accumulation, 8 activation rows per pass over the weight row; K % 32 != 0 or unaligned rows take a byte-granular
// path with the same arithmetic.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gemm_core.cuh"

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

// Streaming form of the same MMA tiling, for the weight-stream-bound shapes (K % 64 == 0, 4-byte aligned scales).
// The register double buffer above keeps one 128-wide chunk (1 KB of codes per warp) in flight, which covers DRAM
// latency for ~3.4 TB/s only.  Here every lane copies its pieces (16 codes bytes of rows g and g + 8, and the
// 4-byte scale word holding its two scale bytes of each row) with cp.async into a ring of kW4Stages chunks in shared
// memory, kW4Stages - 1 chunks ahead of the MMAs.  A lane reads back only what it copied itself, so the ring needs
// no barrier: cp.async.wait_group orders a lane's own copies.  The warps are persistent: warp w walks row groups
// w, w + W, w + 2W, ... (16 rows each) as one sequence of (group, chunk) items, so the copies of the next group
// start while the current one finishes.
constexpr int kW4Stages = 8;
constexpr int kW4Warps = 8;

struct W4Stage {
    uint4 codes[2][32];      // [row g / row g + 8][lane]: conflict-free 16-byte shared loads
    uint2 scales[32];        // [lane]: (scale word of row g, of row g + 8)
};
constexpr int kW4SmemBytes = kW4Warps * kW4Stages * (int)sizeof(W4Stage);

__device__ __forceinline__ void cp_async_16(void* dst, const void* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

__device__ __forceinline__ void cp_async_4(void* dst, const void* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(valid ? 4 : 0) : "memory");
}

// NT activation tiles of 8 tokens per pass (M <= 8 NT): the weight fragments are decoded once per chunk and used
// by NT MMAs, so M <= 16 streams the weights once.
template <int NT>
__global__ void __launch_bounds__(kW4Warps * 32, 2) w4a16_stream_kernel(float* __restrict__ out,
                                                                        const uint8_t* __restrict__ wp,
                                                                        const uint8_t* __restrict__ ws, float inv_g,
                                                                        const __half* __restrict__ x, int M, int N,
                                                                        int K) {
    extern __shared__ __align__(16) uint8_t w4_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, q = lane & 3;
    W4Stage* ring = reinterpret_cast<W4Stage*>(w4_smem) + warp * kW4Stages;
    const int groups = (N + 15) / 16, chunks = (K + 127) / 128;
    const int w0 = blockIdx.x * kW4Warps + warp, nw = gridDim.x * kW4Warps;
    const int items = w0 < groups ? ((groups - 1 - w0) / nw + 1) * chunks : 0;

    int ig = w0, ic = 0;                       // (group, chunk) of the next item to copy
    auto issue = [&](int i) {
        W4Stage& st = ring[i % kW4Stages];
        const int k0 = ic * 128 + q * 32;
        const bool live = i < items && k0 < K;
        const int ra = ig * 16 + g, rb = ra + 8;
        const bool va = live && ra < N, vb = live && rb < N;
        const size_t sw = (size_t)ic * 8 + 4 * (q >> 1);
        cp_async_16(&st.codes[0][lane], va ? wp + (size_t)ra * (K / 2) + k0 / 2 : wp, va);
        cp_async_16(&st.codes[1][lane], vb ? wp + (size_t)rb * (K / 2) + k0 / 2 : wp, vb);
        cp_async_4(&st.scales[lane].x, va ? ws + (size_t)ra * (K / 16) + sw : ws, va);
        cp_async_4(&st.scales[lane].y, vb ? ws + (size_t)rb * (K / 16) + sw : ws, vb);
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (++ic == chunks) { ic = 0; ig += nw; }
    };
    // token g + 8t's 32 activations of chunk c, as the B fragments of the chunk's 8 MMAs (zero past M or K)
    auto load_x = [&](uint4 (&xv)[NT][4], int c) {
        const int k0 = c * 128 + q * 32;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const bool ok = g + 8 * t < M && k0 < K;
            const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(ok ? g + 8 * t : 0) * K + (ok ? k0 : 0));
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[t][i] = ok ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
        }
    };

#pragma unroll 1
    for (int i = 0; i < kW4Stages - 1; ++i) issue(i);
    float d[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
    uint4 xc[NT][4], xn[NT][4];
    load_x(xc, 0);
    int grp = w0, c = 0;
#pragma unroll 1
    for (int i = 0; i < items; ++i) {
        issue(i + kW4Stages - 1);          // into the stage item i - 1 was read from
        asm volatile("cp.async.wait_group %0;" ::"n"(kW4Stages - 1) : "memory");
        const W4Stage& st = ring[i % kW4Stages];
        const uint4 pa = st.codes[0][lane], pb = st.codes[1][lane];
        const uint2 sw = st.scales[lane];
        const int cn = c + 1 == chunks ? 0 : c + 1;
        load_x(xn, cn);
        const uint32_t ca[4] = {pa.x, pa.y, pa.z, pa.w}, cb[4] = {pb.x, pb.y, pb.z, pb.w};
        const uint32_t sh = 16 * (q & 1);
        const uint32_t sa0 = e4m3_to_half2x(sw.x >> sh), sa1 = e4m3_to_half2x(sw.x >> (sh + 8));
        const uint32_t sb0 = e4m3_to_half2x(sw.y >> sh), sb1 = e4m3_to_half2x(sw.y >> (sh + 8));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t wa = ca[j >> 1] >> (16 * (j & 1)), wb = cb[j >> 1] >> (16 * (j & 1));
            const uint32_t s_a = j < 4 ? sa0 : sa1, s_b = j < 4 ? sb0 : sb1;
            const uint32_t a0 = hmul2_u32(e2m1x2_to_half2(wa & 0xFFu), s_a);
            const uint32_t a1 = hmul2_u32(e2m1x2_to_half2(wb & 0xFFu), s_b);
            const uint32_t a2 = hmul2_u32(e2m1x2_to_half2((wa >> 8) & 0xFFu), s_a);
            const uint32_t a3 = hmul2_u32(e2m1x2_to_half2((wb >> 8) & 0xFFu), s_b);
            const int xi = 2 * j;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint32_t b0 = (&xc[t][xi >> 2].x)[xi & 3], b1 = (&xc[t][(xi + 1) >> 2].x)[(xi + 1) & 3];
                mma_16816(d[t], a0, a1, a2, a3, b0, b1);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j = 0; j < 4; ++j) xc[t][j] = xn[t][j];
        if (cn == 0) {                     // the group's last chunk: write its 16 x M outputs
            const int ra = grp * 16 + g, rb = ra + 8;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int m0 = 8 * t + 2 * q, m1 = m0 + 1;
                if (ra < N) {
                    if (m0 < M) out[(size_t)m0 * N + ra] = d[t][0] * inv_g;
                    if (m1 < M) out[(size_t)m1 * N + ra] = d[t][1] * inv_g;
                }
                if (rb < N) {
                    if (m0 < M) out[(size_t)m0 * N + rb] = d[t][2] * inv_g;
                    if (m1 < M) out[(size_t)m1 * N + rb] = d[t][3] * inv_g;
                }
                d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
            }
            grp += nw;
        }
        c = cn;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <int NT>
int launch_w4a16_stream_nt(float* out, const uint8_t* wp, const uint8_t* ws, float inv_g, const __half* x, int M,
                           int N, int K, cudaStream_t s) {
    static std::atomic<int> per_sm[64];         // resident blocks per SM, per device (host threads may race: same value)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4B_ERR_CUDA;
    int r = per_sm[dev].load(std::memory_order_acquire);
    if (r == 0) {
        cudaError_t err = cudaFuncSetAttribute(w4a16_stream_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kW4SmemBytes);
        if (err == cudaSuccess)
            err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, w4a16_stream_kernel<NT>, kW4Warps * 32,
                                                                kW4SmemBytes);
        if (err != cudaSuccess) return record_cuda_error(err);
        if (r <= 0) return record_cuda_error(cudaErrorLaunchOutOfResources);
        per_sm[dev].store(r, std::memory_order_release);
    }
    const long long groups = (N + 15) / 16, need = (groups + kW4Warps - 1) / kW4Warps;
    const long long cap = (long long)r * sm_count();
    w4a16_stream_kernel<NT><<<(unsigned)(need < cap ? need : cap), kW4Warps * 32, kW4SmemBytes, s>>>(
        out, wp, ws, inv_g, x, M, N, K);
    return launch_status();
}

// Activation rows in passes of 16 (8 for a last pass of at most 8 rows); each pass streams the weights once.
int launch_w4a16_stream(float* out, const uint8_t* wp, const uint8_t* ws, float inv_g, const __half* x, int M, int N,
                        int K, cudaStream_t s) {
    for (int m0 = 0; m0 < M; m0 += 16) {
        const int mr = M - m0 < 16 ? M - m0 : 16;
        const int st = mr <= 8 ? launch_w4a16_stream_nt<1>(out + (size_t)m0 * N, wp, ws, inv_g, x + (size_t)m0 * K, mr,
                                                           N, K, s)
                               : launch_w4a16_stream_nt<2>(out + (size_t)m0 * N, wp, ws, inv_g, x + (size_t)m0 * K, mr,
                                                           N, K, s);
        if (st != NVFP4B_OK) return st;
    }
    return NVFP4B_OK;
}

// ---- TMA-fed form (K % 256 == 0): the weight-stream-bound lm_head / decode shapes ----------------------------------
// A persistent CTA per SM streams tasks of 16 CW weight rows: a producer warp loads, per slab of 256 K values, the
// rows' codes (16 CW x 128 bytes, 128-byte swizzle) and raw scales (16 CW x 16 bytes) with two TMA copies into a
// ring of slabs (~150 KB in flight per SM: register- and LSU-fed loads could not keep enough bytes in flight to cover
// DRAM latency).  CW consumer warps take 16 rows each and run the same mma.sync m16n8k16 arithmetic as above, with
// the even and odd MMAs of a half-slab on two accumulator chains (the MMA latency, not issue, bounds a chain).  In a
// slab, lane (g, q) owns K values [64q, 64q + 64) -- 16-byte units 2q and 2q + 1 of a 128-byte row, which the
// swizzle (unit ^ row % 8) spreads over all 32 banks -- and its four scale bytes 4q..4q + 3 of each row.  The weights
// are loaded with the L2 evict-first priority (read once); the activations stay in L1/L2.
template <int NT>
struct W4T {
    // launched for one activation tile (M <= 8; the dispatch takes it for M <= 2): 16 consumer warps, 5 stages
    static_assert(NT == 1, "one tile of 8 activation rows");
    static constexpr int CW = 16;                              // consumer warps
    static constexpr int ROWS = 16 * CW;
    static constexpr int CODES = ROWS * 128, SCALES = ROWS * 16;
    static constexpr int STAGES = 5;
    static constexpr int THREADS = (CW + 1) * 32;
    static constexpr int SMEM = STAGES * (CODES + SCALES) + 2 * STAGES * 8 + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory");
};

template <int NT>
__global__ void __launch_bounds__(W4T<NT>::THREADS, 1)
    w4a16_tma_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts,
                     float* __restrict__ out, const __half* __restrict__ x, float inv_g, int M, int N, int K,
                     int* err) {
    using namespace sm100;
    using C = W4T<NT>;
    extern __shared__ uint8_t w4t_raw[];
    uint8_t* sc = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(w4t_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ss = sc + C::STAGES * C::CODES;
    uint64_t* full = reinterpret_cast<uint64_t*>(ss + C::STAGES * C::SCALES);
    uint64_t* empty = full + C::STAGES;
    volatile int* sflag = reinterpret_cast<volatile int*>(empty + C::STAGES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], C::CW); }
        *sflag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const int tasks = (N + C::ROWS - 1) / C::ROWS, slabs = K / 256;
    if (warp == C::CW) {
        if (lane == 0) {                               // producer
            prefetch_tmap(&tw);
            prefetch_tmap(&ts);
            const uint64_t pol = l2_policy_evict_first();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tasks && ok; t += gridDim.x)
                for (int sl = 0; sl < slabs; ++sl) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, sflag, kErrTimeoutProducer)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[stage], C::CODES + C::SCALES);
                    tma_load_2d_hint(sc + stage * C::CODES, &tw, &full[stage], sl * 128, t * C::ROWS, pol);
                    tma_load_2d_hint(ss + stage * C::SCALES, &ts, &full[stage], sl * 16, t * C::ROWS, pol);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
        }
    } else {                                           // consumers
        const int g = lane >> 2, q = lane & 3;
        const int ra = warp * 16 + g, rb = ra + 8;     // rows within the task
        // token g + 8t's 32 activations of half-slab h of slab sl (K [256 sl + 64 q + 32 h, + 32)), zero past M
        auto load_x = [&](uint4 (&xv)[NT][4], int sl, int h) {
            const int k0 = sl * 256 + 64 * q + 32 * h;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const bool ok = g + 8 * t < M;
                const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(ok ? g + 8 * t : 0) * K + k0);
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[t][i] = ok ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
            }
        };
        // the 8 MMAs of one half-slab (codes of rows ra / rb, 16 bytes each, their two scale bytes), alternating
        // between the accumulator chains d[0] and d[1]
        auto mma_half = [&](float (&d)[2][NT][4], const uint4& pa, const uint4& pb, uint32_t sa2, uint32_t sb2,
                            const uint4 (&xv)[NT][4]) {
            const uint32_t ca[4] = {pa.x, pa.y, pa.z, pa.w}, cb[4] = {pb.x, pb.y, pb.z, pb.w};
            const uint32_t sa0 = e4m3_to_half2x(sa2), sa1 = e4m3_to_half2x(sa2 >> 8);
            const uint32_t sb0 = e4m3_to_half2x(sb2), sb1 = e4m3_to_half2x(sb2 >> 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t wa = ca[j >> 1] >> (16 * (j & 1)), wb = cb[j >> 1] >> (16 * (j & 1));
                const uint32_t s_a = j < 4 ? sa0 : sa1, s_b = j < 4 ? sb0 : sb1;
                const uint32_t a0 = hmul2_u32(e2m1x2_to_half2(wa & 0xFFu), s_a);
                const uint32_t a1 = hmul2_u32(e2m1x2_to_half2(wb & 0xFFu), s_b);
                const uint32_t a2 = hmul2_u32(e2m1x2_to_half2((wa >> 8) & 0xFFu), s_a);
                const uint32_t a3 = hmul2_u32(e2m1x2_to_half2((wb >> 8) & 0xFFu), s_b);
                const int xi = 2 * j;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    mma_16816(d[j & 1][t], a0, a1, a2, a3, (&xv[t][xi >> 2].x)[xi & 3],
                              (&xv[t][(xi + 1) >> 2].x)[(xi + 1) & 3]);
            }
        };
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        uint4 xc[NT][4], xn[NT][4];
        load_x(xc, 0, 0);
        for (int t = blockIdx.x; t < tasks && ok; t += gridDim.x) {
            float d[2][NT][4];
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
                for (int u = 0; u < NT; ++u) d[c][u][0] = d[c][u][1] = d[c][u][2] = d[c][u][3] = 0.f;
            for (int sl = 0; sl < slabs; ++sl) {
                if (!mbar_wait(&full[stage], phase, sflag, kErrTimeoutMma)) { ok = false; break; }
                const uint8_t* cs = sc + stage * C::CODES;
                const uint8_t* s16 = ss + stage * C::SCALES;
                const uint4 pa0 = *reinterpret_cast<const uint4*>(cs + ra * 128 + ((2 * q) ^ g) * 16);
                const uint4 pa1 = *reinterpret_cast<const uint4*>(cs + ra * 128 + ((2 * q + 1) ^ g) * 16);
                const uint4 pb0 = *reinterpret_cast<const uint4*>(cs + rb * 128 + ((2 * q) ^ g) * 16);
                const uint4 pb1 = *reinterpret_cast<const uint4*>(cs + rb * 128 + ((2 * q + 1) ^ g) * 16);
                const uint32_t swa = *reinterpret_cast<const uint32_t*>(s16 + ra * 16 + 4 * q);
                const uint32_t swb = *reinterpret_cast<const uint32_t*>(s16 + rb * 16 + 4 * q);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[stage]);        // the slab is in registers: release it
                if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                load_x(xn, sl, 1);
                mma_half(d, pa0, pb0, swa, swb, xc);
#pragma unroll
                for (int u = 0; u < NT; ++u)
#pragma unroll
                    for (int i = 0; i < 4; ++i) xc[u][i] = xn[u][i];
                load_x(xn, sl + 1 < slabs ? sl + 1 : 0, 0);        // the next task starts again at slab 0
                mma_half(d, pa1, pb1, swa >> 16, swb >> 16, xc);
#pragma unroll
                for (int u = 0; u < NT; ++u)
#pragma unroll
                    for (int i = 0; i < 4; ++i) xc[u][i] = xn[u][i];
            }
            if (!ok) break;
            const int na = t * C::ROWS + ra, nb = t * C::ROWS + rb;
#pragma unroll
            for (int u = 0; u < NT; ++u) {
                const int m0 = 8 * u + 2 * q, m1 = m0 + 1;
                if (na < N) {
                    if (m0 < M) out[(size_t)m0 * N + na] = (d[0][u][0] + d[1][u][0]) * inv_g;
                    if (m1 < M) out[(size_t)m1 * N + na] = (d[0][u][1] + d[1][u][1]) * inv_g;
                }
                if (nb < N) {
                    if (m0 < M) out[(size_t)m0 * N + nb] = (d[0][u][2] + d[1][u][2]) * inv_g;
                    if (m1 < M) out[(size_t)m1 * N + nb] = (d[0][u][3] + d[1][u][3]) * inv_g;
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && *sflag != 0) atomicCAS(err, 0, *sflag);
}

template <int NT>
int launch_w4a16_tma_nt(const uint8_t* wp, const uint8_t* ws, float* out, const __half* x, float inv_g, int M, int N,
                        int K, int* err, cudaStream_t s) {
    using C = W4T<NT>;
    static std::atomic<int> ready[64];          // per device: shared-memory limit raised (host threads may race)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4B_ERR_CUDA;
    if (!ready[dev].load(std::memory_order_acquire)) {
        const cudaError_t e = cudaFuncSetAttribute(w4a16_tma_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   C::SMEM);
        if (e != cudaSuccess) return record_cuda_error(e);
        ready[dev].store(1, std::memory_order_release);
    }
    CUtensorMap tw, ts;
    int st = make_kmajor_map(&tw, wp, N, K / 2, C::ROWS);
    if (st) return st;
    st = make_rows_map(&ts, ws, N, K / 16, 16, C::ROWS);
    if (st) return st;
    const int tasks = (N + C::ROWS - 1) / C::ROWS, sms = sm_count();
    w4a16_tma_kernel<NT><<<tasks < sms ? tasks : sms, C::THREADS, C::SMEM, s>>>(tw, ts, out, x, inv_g, M, N, K, err);
    return launch_status();
}

// M <= 8 activation rows, one weight pass.
int launch_w4a16_tma(float* out, const uint8_t* wp, const uint8_t* ws, float inv_g, const __half* x, int M, int N,
                     int K, cudaStream_t s) {
    int* err = device_error_ptr();
    if (!err) return NVFP4B_ERR_CUDA;
    return launch_w4a16_tma_nt<1>(wp, ws, out, x, inv_g, M, N, K, err, s);
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
    // M <= 2: TMA-fed tensor-core kernel (112.7 us on the lm_head shape N = 262144, K = 2816, against 120.8 us for
    // the register-fed one); up to 8 rows the register-fed kernel (its 24 warps per SM hide the activation loads
    // better: 149.5 against 200.7 us at M = 8); above, passes of 16 rows through the cp.async ring kernel (M = 16:
    // 238 us, one weight pass).
    if (fast && M <= 2 && K % 256 == 0 && aligned16(ws))
        return launch_w4a16_tma(out, wp, ws, inv_g, static_cast<const __half*>(x16), M, N, K, s);
    if (fast && M <= kW4A16MmaMaxM)
        w4a16_mma_kernel<<<(unsigned)((N + 127) / 128), 256, 0, s>>>(out, wp, ws, inv_g,
                                                                     static_cast<const __half*>(x16), M, N, K);
    else if (fast && K % 64 == 0 && (reinterpret_cast<uintptr_t>(ws) & 3) == 0)
        return launch_w4a16_stream(out, wp, ws, inv_g, static_cast<const __half*>(x16), M, N, K, s);
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
