// stream.cu -- a read-only HBM stream through the same TMA path the GEMMs use, for the roofline of the weight-stream
// bound kernels.  A [rows, row_bytes] byte matrix is read in boxes of 256 rows x 128 bytes (128-byte swizzle, as the
// GEMMs' B operand) by one persistent CTA per SM into a 4-stage shared-memory ring and discarded.  The measured rate
// depends on the size: a stream of a few hundred MB pays a fixed ramp and tail that a 1 GiB copy amortises, so the
// weight stream of a kernel is compared with this stream at the same byte count.
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemm_core.cuh"

namespace nvfp4b {
namespace {

constexpr int kStreamStages = 4, kStreamBox = 256 * 128;
constexpr int kStreamSmem = kStreamStages * kStreamBox + 2 * kStreamStages * 8 + 16 + 1024;

__global__ void __launch_bounds__(64, 1) read_stream_kernel(const __grid_constant__ CUtensorMap map, int tasks,
                                                            int ktiles, int* err) {
    using namespace sm100;
    extern __shared__ uint8_t rs_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rs_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStreamStages * kStreamBox);
    uint64_t* empty = full + kStreamStages;
    volatile int* flag = reinterpret_cast<volatile int*>(empty + kStreamStages);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStreamStages; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        *flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    int st = 0;
    uint32_t ph = 0;
    bool ok = true;
    if (threadIdx.x == 0) {                       // producer
        prefetch_tmap(&map);
        for (int t = blockIdx.x; t < tasks && ok; t += gridDim.x)
            for (int k = 0; k < ktiles; ++k) {
                if (!mbar_wait(&empty[st], ph ^ 1u, flag, kErrTimeoutProducer)) { ok = false; break; }
                mbar_arrive_expect_tx(&full[st], kStreamBox);
                tma_load_2d(sm + st * kStreamBox, &map, &full[st], k * 128, t * 256);
                if (++st == kStreamStages) { st = 0; ph ^= 1u; }
            }
    } else if (threadIdx.x == 32) {               // consumer: releases each stage once it landed
        for (int t = blockIdx.x; t < tasks && ok; t += gridDim.x)
            for (int k = 0; k < ktiles; ++k) {
                if (!mbar_wait(&full[st], ph, flag, kErrTimeoutMma)) { ok = false; break; }
                mbar_arrive(&empty[st]);
                if (++st == kStreamStages) { st = 0; ph ^= 1u; }
            }
    }
    __syncthreads();
    if (threadIdx.x == 0 && *flag != 0) atomicCAS(err, 0, *flag);
}

}  // namespace
}  // namespace nvfp4b

using namespace nvfp4b;

extern "C" int nvfp4b_hbm_read_stream(const void* p, long long rows, int row_bytes, void* stream) {
    if (!p) return NVFP4B_ERR_NULL;
    if (rows <= 0 || row_bytes <= 0 || (row_bytes % 128) || rows > (1LL << 30)) return NVFP4B_ERR_SHAPE;
    if (!aligned16(p)) return NVFP4B_ERR_ALIGN;
    static std::atomic<bool> ready[64];           // per device: shared-memory limit raised (host threads may race)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NVFP4B_ERR_CUDA;
    if (!ready[dev].load(std::memory_order_acquire)) {
        const cudaError_t e =
            cudaFuncSetAttribute(read_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStreamSmem);
        if (e != cudaSuccess) return record_cuda_error(e);
        ready[dev].store(true, std::memory_order_release);
    }
    CUtensorMap map;
    int st = make_kmajor_map(&map, p, rows, row_bytes, 256);
    if (st) return st;
    int* err = device_error_ptr();
    if (!err) return NVFP4B_ERR_CUDA;
    const int tasks = (int)((rows + 255) / 256), sms = sm_count();
    read_stream_kernel<<<tasks < sms ? tasks : sms, 64, kStreamSmem, (cudaStream_t)stream>>>(map, tasks,
                                                                                           row_bytes / 128, err);
    return launch_status();
}
