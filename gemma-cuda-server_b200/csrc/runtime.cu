// runtime.cu -- library-wide host helpers: error bookkeeping, device properties, sizes.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace nvfp4b {

static thread_local int t_last_cuda_error = 0;

// Kernels whose bounded waits expire record a code here (through the pointer they are given).
__device__ int g_device_error = 0;

// The per-device caches below may be filled by several host threads at once (each computes the same value), so
// their entries are atomics.
int* device_error_ptr() {
    static std::atomic<int*> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    int* p = cached[dev].load(std::memory_order_acquire);
    if (!p) {
        void* q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&q, g_device_error);
        if (e != cudaSuccess) { record_cuda_error(e); return nullptr; }
        p = static_cast<int*>(q);
        cached[dev].store(p, std::memory_order_release);
    }
    return p;
}

int record_cuda_error(cudaError_t e) {
    t_last_cuda_error = (int)e;
    return NVFP4B_ERR_CUDA;
}

int sm_count() {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace nvfp4b

extern "C" const char* nvfp4b_version(void) { return "nvfp4_b200 0.1 (sm_100a)"; }

extern "C" int nvfp4b_last_cuda_error(void) { return nvfp4b::t_last_cuda_error; }

extern "C" size_t nvfp4b_scale_buffer_bytes(int outer, int K) {
    if (outer <= 0 || K <= 0) return 0;
    return nvfp4b::scale_bytes(outer, K);
}

extern "C" int nvfp4b_read_device_error(int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, nvfp4b::g_device_error, sizeof(int));
    if (e != cudaSuccess) return nvfp4b::record_cuda_error(e);
    if (reset && v) {
        const int z = 0;
        e = cudaMemcpyToSymbol(nvfp4b::g_device_error, &z, sizeof(int));
        if (e != cudaSuccess) return nvfp4b::record_cuda_error(e);
    }
    return v;
}
