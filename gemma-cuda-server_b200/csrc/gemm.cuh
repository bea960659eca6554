// gemm.cuh -- host-visible pieces of the NVFP4 tcgen05 GEMM shared by the dense and the grouped (MoE) paths.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nvfp4b {

struct GemmParams {
    const uint8_t* sfa;   // A scales, tile layout
    const uint8_t* sfb;   // B scales, tile layout
    int M, N, K;
    int m_tiles, n_tiles;
    int tile_cols;        // scale tiles along K = ceil(K/64) = number of 64-wide MMA K-steps
    int ksteps;
    int k_tiles;          // 256-wide pipeline stages along K
    int b_row_tiles;      // ceil(N/128): 128-row scale tiles that exist for B
    float alpha;          // a_dequant * b_dequant
    float b_dequant;
    const float* d_a_amax;   // if set: alpha = b_dequant / gscale(amax) on the device
    void* d;
    long long ldd;
    int out_kind;
};

int make_kmajor_map(CUtensorMap* map, const void* base, long long rows, long long row_bytes, int box_rows);
int gemm_dense(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf, GemmParams p,
               cudaStream_t stream);

}  // namespace nvfp4b
