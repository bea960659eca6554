// C entry points forwarding to the reference's own C++ functions (compiled from its unmodified sources by
// oracle/build.py).  TEST INFRASTRUCTURE ONLY: lets the tests call the reference's host swizzle, its CUDA
// quantiser, its cuBLASLt NVFP4 GEMM and its W4A16 kernels through ctypes.
#include "fp4_gemm.h"
#include "nvfp4_quant.h"

extern "C" {

size_t ref_scale_buffer_bytes(int outer, int K) { return nvfp4_scale_buffer_bytes(outer, K); }

void ref_swizzle_scales(const uint8_t* logical, uint8_t* swizzled, int outer, int K) {
    nvfp4_swizzle_scales(logical, swizzled, outer, K);
}

void ref_quantize_activations(const float* dX, uint8_t* dPacked, uint8_t* dScalesSwz, int M, int K, float gscale,
                              void* stream) {
    nvfp4_quantize_activations(dX, dPacked, dScalesSwz, M, K, gscale, (cudaStream_t)stream);
}

// One cuBLASLt handle + workspace per process, created on first use (test helper only).
static cublasLtHandle_t g_lt = nullptr;
static void* g_ws = nullptr;
static const size_t kWsBytes = 64u << 20;

int ref_nvfp4_gemm(float* dD, const uint8_t* dA, const uint8_t* dAs, float ag, const uint8_t* dB,
                   const uint8_t* dBs, float bg, int M, int N, int K, void* stream) {
    if (!g_lt) {
        if (cublasLtCreate(&g_lt) != CUBLAS_STATUS_SUCCESS) return -200;
        if (cudaMalloc(&g_ws, kWsBytes) != cudaSuccess) return -201;
    }
    return nvfp4_gemm(dD, dA, dAs, ag, dB, dBs, bg, M, N, K, g_lt, g_ws, kWsBytes, (cudaStream_t)stream);
}

void ref_w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16, int M,
                    int N, int K, void* stream) {
    w4a16_gemm(out, wp, ws, w_gscale, x16, M, N, K, (cudaStream_t)stream);
}

void ref_fp4_gemv(float* y, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16, int N, int K,
                  void* stream) {
    fp4_gemv(y, wp, ws, w_gscale, x16, N, K, (cudaStream_t)stream);
}

}  // extern "C"
