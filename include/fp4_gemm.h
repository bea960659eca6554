// fp4_gemm.h -- drop-in declarations of the reference's NVFP4 GEMM module (include/fp4_gemm.h:13-35 of the
// reference), implemented by libnvfp4_b200.so with hand-written sm_100a kernels (no cuBLASLt on the path; the
// cuBLASLt handle type stays in the signature so existing callers compile unchanged).
//
// nvfp4_gemm: D[M,N] = a_gscale * b_gscale * A[M,K] @ B[N,K]^T, A and B NVFP4 (codes + scales in the 128x4-tile
// layout), D fp32 COLUMN-major with ld = M, beta = 0.  a_gscale / b_gscale are dequant multipliers (1 / the
// compressed-tensors global scale).  Returns 0 on success, non-zero otherwise.  `lt`, `workspace` and `ws_bytes`
// are accepted and ignored.
#pragma once
#include <cstdint>
#include <cstddef>
#include <cublasLt.h>
#include <cuda_runtime.h>

// Bytes of the tile-layout scale buffer for an [outer, K] operand: ceil(outer/128) * ceil(K/64) * 512.
size_t nvfp4_scale_buffer_bytes(int outer, int K);

// Host relayout of logical e4m3 scales [outer, K/16] into the tile layout; padding zeroed.
void nvfp4_swizzle_scales(const uint8_t* logical, uint8_t* swizzled, int outer, int K);

// W4A16: out[M,N] (fp32, row-major) = x16[M,K] (fp16) @ dequant(W[N,K])^T, raw (unswizzled) weight codes and
// scales, dequant = code * e4m3 / w_gscale.
void w4a16_gemm(float* out, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16,
                int M, int N, int K, cudaStream_t s);

// W4A16 GEMV for one token: y[N] = dequant(W[N,K]) @ x16[K] (fp16 activations).
void fp4_gemv(float* y, const uint8_t* wp, const uint8_t* ws, float w_gscale, const void* x16,
              int N, int K, cudaStream_t s);

int nvfp4_gemm(float* dD,
               const uint8_t* dA_packed, const uint8_t* dA_scales_swz, float a_gscale,
               const uint8_t* dB_packed, const uint8_t* dB_scales_swz, float b_gscale,
               int M, int N, int K,
               cublasLtHandle_t lt, void* workspace, size_t ws_bytes, cudaStream_t stream);
