// nvfp4_quant.h -- drop-in declaration of the reference's activation quantiser entry point
// (include/nvfp4_quant.h:10-11 of the reference), implemented by libnvfp4_b200.so on sm_100a.
//
// dX is row-major fp32 [M, K] on the device, K a multiple of 16.  dPacked receives the e2m1 codes [M, K/2]
// (even element in the low nibble); dScalesSwz receives the e4m3 block scales in the 128x4-tile layout and must
// hold nvfp4_scale_buffer_bytes(M, K) bytes -- every byte, padding included, is written.  gscale is the
// compressed-tensors global scale (2688 / amax).  Work is enqueued on `stream`; errors are reported through
// cudaGetLastError()-style status only (the function returns nothing, as in the reference).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

void nvfp4_quantize_activations(const float* dX, uint8_t* dPacked, uint8_t* dScalesSwz,
                                int M, int K, float gscale, cudaStream_t stream);
