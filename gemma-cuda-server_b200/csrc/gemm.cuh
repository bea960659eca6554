// gemm.cuh -- host-side parameters of the dense NVFP4 GEMM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4b {

struct GemmParams {
    int M, N, K;
    float alpha;             // a_dequant * b_dequant
    float b_dequant;
    const float* d_a_amax;   // if set: alpha = b_dequant / gscale(amax) on the device
    void* d;
    long long ldd;
    int out_kind;
};

int gemm_dense(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, GemmParams p,
               cudaStream_t stream);

}  // namespace nvfp4b
