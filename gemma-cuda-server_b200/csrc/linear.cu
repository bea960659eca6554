// linear.cu -- the dense Linear of the reference's forward pass (src/forward.cu:424-445) on this library:
// out_row[M, N] = in_row[M, K] @ W[N, K]^T, fp32 row-major in and out, NVFP4 weights.
//
// The reference runs every Linear as W4A16 (fp16 activations: fp4_gemv at M = 1, w4a16_gemm otherwise).  Here a
// prefill-sized call (M >= NVFP4B_LINEAR_W4A4_MIN_M) goes through the W4A4 path instead: the fp32 activations are
// quantised to NVFP4 (static global scale from the checkpoint, or dynamic from the device amax) and multiplied on
// the tcgen05 tensor cores with an fp32 row-major epilogue (no transpose kernel).  Smaller M keeps the reference's
// W4A16 arithmetic (fp16 activations, fp32 accumulation).  Everything is enqueued on the caller's stream inside a
// caller-owned workspace: no allocation, no synchronisation, capture-safe.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvfp4b {

// |x| max of fp32 data into d_amax (which the host entry zeroes first).  Non-negative floats order like their bit
// patterns, so the block result goes to memory with one integer atomicMax.
__global__ void __launch_bounds__(256) amax_f32_kernel(const float* __restrict__ x, long long n,
                                                       float* __restrict__ d_amax) {
    __shared__ uint32_t red[8];
    uint32_t best = 0;
    const long long nvec = n >> 2;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < nvec; i += 4 * stride) {
        uint4 a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = __ldg(xv + i + u * stride);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            best = max(best, max(max(a[u].x & 0x7FFFFFFFu, a[u].y & 0x7FFFFFFFu),
                                 max(a[u].z & 0x7FFFFFFFu, a[u].w & 0x7FFFFFFFu)));
    }
    for (; i < nvec; i += stride) {
        const uint4 a = __ldg(xv + i);
        best = max(best, max(max(a.x & 0x7FFFFFFFu, a.y & 0x7FFFFFFFu), max(a.z & 0x7FFFFFFFu, a.w & 0x7FFFFFFFu)));
    }
    for (long long k = (nvec << 2) + (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride)
        best = max(best, __float_as_uint(x[k]) & 0x7FFFFFFFu);
    best = __reduce_max_sync(0xFFFFFFFFu, best);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0u;
        v = __reduce_max_sync(0xFFFFFFFFu, v);
        if (threadIdx.x == 0 && v != 0) atomicMax(reinterpret_cast<unsigned int*>(d_amax), v);
    }
}

// fp32 -> fp16 (RNE), 4 elements per thread per step (the reference's k_f32_to_f16 before its W4A16 calls).
__global__ void __launch_bounds__(256) f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y,
                                                         long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long nvec = n >> 2;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
        __half2 h[2] = {__floats2half2_rn(v.x, v.y), __floats2half2_rn(v.z, v.w)};
        *reinterpret_cast<uint2*>(y + 4 * i) = *reinterpret_cast<const uint2*>(h);
    }
    for (long long k = (nvec << 2) + (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += stride)
        y[k] = __float2half_rn(x[k]);
}

static inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }

// Workspace: [0, 256) device amax; then either the NVFP4 activations (codes, tile-layout scales) or the fp16 copy.
static size_t linear_ws(int M, int K) {
    const size_t w4a4 = round256((size_t)M * K / 2) + round256(scale_bytes(M, K));
    const size_t w4a16 = round256((size_t)M * K * 2);
    return 256 + (w4a4 > w4a16 ? w4a4 : w4a16);
}

static int launch_amax_f32(const float* x, long long n, float* d_amax, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(d_amax, 0, sizeof(float), s);
    if (e != cudaSuccess) return record_cuda_error(e);
    long long blocks = ((n >> 2) + 1023) / 1024;
    const long long cap = (long long)sm_count() * 2;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    amax_f32_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, n, d_amax);
    return launch_status();
}

}  // namespace nvfp4b

using namespace nvfp4b;

extern "C" int nvfp4b_amax_f32(const float* x, long long n, float* d_amax, void* stream) {
    if (!x || !d_amax) return NVFP4B_ERR_NULL;
    if (n <= 0) return NVFP4B_ERR_SHAPE;
    if (!aligned16(x)) return NVFP4B_ERR_ALIGN;
    return launch_amax_f32(x, n, d_amax, (cudaStream_t)stream);
}

extern "C" size_t nvfp4b_linear_workspace_bytes(int M, int K) {
    if (M <= 0 || K <= 0) return 0;
    return linear_ws(M, K);
}

extern "C" int nvfp4b_linear(float* out, const float* in, int M, int N, int K, const uint8_t* w,
                             const uint8_t* w_scales, const uint8_t* w_scales_tiled, float w_gscale, float a_gscale,
                             int mode, void* workspace, size_t workspace_bytes, void* stream) {
    if (!out || !in || !w || !workspace) return NVFP4B_ERR_NULL;
    if (M <= 0 || N <= 0 || K <= 0 || (K & 15)) return NVFP4B_ERR_SHAPE;
    if (!(w_gscale > 0.0f)) return NVFP4B_ERR_SHAPE;
    if (mode < NVFP4B_LINEAR_AUTO || mode > NVFP4B_LINEAR_W4A4) return NVFP4B_ERR_ARG;
    if (workspace_bytes < linear_ws(M, K)) return NVFP4B_ERR_SHAPE;
    if (!aligned16(workspace) || !aligned16(in)) return NVFP4B_ERR_ALIGN;
    const cudaStream_t s = (cudaStream_t)stream;
    const bool w4a4 = mode == NVFP4B_LINEAR_W4A4 || (mode == NVFP4B_LINEAR_AUTO && M >= NVFP4B_LINEAR_W4A4_MIN_M);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* d_amax = reinterpret_cast<float*>(ws);
    if (w4a4) {
        if (!w_scales_tiled) return NVFP4B_ERR_NULL;
        if (K & 31) return NVFP4B_ERR_SHAPE;                       // 16-byte code rows for the GEMM's TMA
        uint8_t* codes = ws + 256;
        uint8_t* scales = codes + round256((size_t)M * K / 2);
        const bool dynamic = !(a_gscale > 0.0f);
        if (dynamic) {
            const int rc = launch_amax_f32(in, (long long)M * K, d_amax, s);
            if (rc) return rc;
        }
        int rc = nvfp4b_quantize_f32(in, M, K, dynamic ? 0.0f : a_gscale, dynamic ? d_amax : nullptr, codes, scales,
                                     stream);
        if (rc) return rc;
        return nvfp4b_gemm(codes, scales, dynamic ? 1.0f : 1.0f / a_gscale, dynamic ? d_amax : nullptr, w,
                           w_scales_tiled, 1.0f / w_gscale, M, N, K, out, NVFP4B_OUT_F32_ROWMAJOR, N, stream);
    }
    if (!w_scales) return NVFP4B_ERR_NULL;
    __half* x16 = reinterpret_cast<__half*>(ws + 256);
    const long long n = (long long)M * K;
    long long blocks = ((n >> 2) + 255) / 256;
    const long long cap = (long long)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    f32_to_f16_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, x16, n);
    const int rc = launch_status();
    if (rc) return rc;
    return nvfp4b_w4a16_gemm(out, w, w_scales, w_gscale, x16, M, N, K, stream);
}
