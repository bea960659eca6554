// compat.cu -- the reference's C++ operator API (include/nvfp4_quant.h, include/fp4_gemm.h of the reference),
// exported with the same C++ signatures so src/forward.cu, src/draft.cu and the reference's own tests link against
// libnvfp4_b200.so unchanged.  Each function forwards to the C ABI in nvfp4_b200.h.
#include <cstdio>
#include <cstring>

#include "fp4_gemm.h"
#include "nvfp4_b200.h"
#include "nvfp4_quant.h"

// The reference's void entry points report failure only through the CUDA error state, which its callers read with
// cudaGetLastError() / CU() (src/forward.cu:23).  An argument error (K not a multiple of 16, a null or misaligned
// pointer) is rejected by the C ABI before anything is launched, so on its own it would leave that state clean and
// the caller would go on with unwritten buffers.  compat_fail() therefore leaves a launch error behind: a launch
// with an empty grid, which the runtime rejects on the host with cudaErrorInvalidConfiguration -- nothing reaches
// the device, and the next cudaGetLastError() returns (and clears) it.
namespace {
__global__ void compat_failed_call_kernel() {}
}  // namespace

static void compat_fail(const char* fn, int status, cudaStream_t stream) {
    fprintf(stderr, "%s: nvfp4_b200 status %d\n", fn, status);
    compat_failed_call_kernel<<<0, 1, 0, stream>>>();
}

// include/nvfp4_quant.h:10-11 -- static global scale, fp32 input; void, errors via the CUDA error state.
void nvfp4_quantize_activations(const float* dX, uint8_t* dPacked, uint8_t* dScalesSwz, int M, int K, float gscale,
                                cudaStream_t stream) {
    const int st = nvfp4b_quantize_f32(dX, M, K, gscale, nullptr, dPacked, dScalesSwz, stream);
    if (st != NVFP4B_OK) compat_fail("nvfp4_quantize_activations", st, stream);
}

// include/fp4_gemm.h:13 (kernels/fp4_gemm.cu:14-19)
size_t nvfp4_scale_buffer_bytes(int outer, int K) { return nvfp4b_scale_buffer_bytes(outer, K); }

// include/fp4_gemm.h:17 (kernels/fp4_gemm.cu:21-33): host relayout, padding zeroed.
void nvfp4_swizzle_scales(const uint8_t* logical, uint8_t* swizzled, int outer, int K) {
    const int kb = K / 16, tile_cols = (kb + 3) / 4;
    memset(swizzled, 0, nvfp4b_scale_buffer_bytes(outer, K));
    for (int m = 0; m < outer; ++m) {
        const size_t row_base = (size_t)(m / 128) * tile_cols * 512 + (size_t)(m % 32) * 16 + ((m % 128) / 32) * 4;
        for (int b = 0; b < kb; ++b) swizzled[row_base + (size_t)(b / 4) * 512 + (b % 4)] = logical[(size_t)m * kb + b];
    }
}

extern "C" int nvfp4b_w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16,
                                 int M, int N, int K, void* stream);

// include/fp4_gemm.h:21-22
void w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16, int M, int N,
                int K, cudaStream_t s) {
    const int st = nvfp4b_w4a16_gemm(out, wp, ws, w_gscale, x16, M, N, K, s);
    if (st != NVFP4B_OK) compat_fail("w4a16_gemm", st, s);
}

// include/fp4_gemm.h:26-27
void fp4_gemv(float* y, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16, int N, int K,
              cudaStream_t s) {
    const int st = nvfp4b_w4a16_gemm(y, wp, ws, w_gscale, x16, 1, N, K, s);
    if (st != NVFP4B_OK) compat_fail("fp4_gemv", st, s);
}

// include/fp4_gemm.h:31-35 -- fp32 column-major D (ld = M); lt / workspace unused.  0 on success.
int nvfp4_gemm(float* dD, const uint8_t* dA_packed, const uint8_t* dA_scales_swz, float a_gscale,
               const uint8_t* dB_packed, const uint8_t* dB_scales_swz, float b_gscale, int M, int N, int K,
               cublasLtHandle_t lt, void* workspace, size_t ws_bytes, cudaStream_t stream) {
    (void)lt;
    (void)workspace;
    (void)ws_bytes;
    const int st = nvfp4b_gemm(dA_packed, dA_scales_swz, a_gscale, nullptr, dB_packed, dB_scales_swz, b_gscale, M, N,
                               K, dD, NVFP4B_OUT_F32_COLMAJOR, M, stream);
    if (st != NVFP4B_OK) fprintf(stderr, "nvfp4_gemm: error %d (M=%d N=%d K=%d)\n", st, M, N, K);
    return st;
}
