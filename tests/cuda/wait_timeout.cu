// Test kernel for the bounded copy wait of the conversion kernels (gq_device.cuh: mbar_wait).
// It waits on an mbarrier phase that nothing completes: no copy is issued and no thread
// arrives, so the wait must give up after its limit and report it; nothing else runs.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gq_device.cuh"

__global__ void wait_never(int* status, unsigned long long* waited_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        gq::mbar_init(&bar, 1);
        gq::mbar_init_fence();
    }
    __syncthreads();
    const uint64_t t0 = gq::global_ns();
    const bool ok = gq::mbar_wait(&bar, 0);
    const uint64_t t1 = gq::global_ns();
    if (threadIdx.x == 0) {
        *status = ok ? 1 : 0;
        *waited_ns = t1 - t0;
    }
}

extern "C" int run_wait_never(int* status, unsigned long long* waited_ns) {
    int* d_status = nullptr;
    unsigned long long* d_ns = nullptr;
    if (cudaMalloc(&d_status, sizeof(int)) != cudaSuccess) return -1;
    if (cudaMalloc(&d_ns, sizeof(unsigned long long)) != cudaSuccess) return -1;
    wait_never<<<1, 32>>>(d_status, d_ns);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(status, d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(waited_ns, d_ns, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d_status);
    cudaFree(d_ns);
    return static_cast<int>(e);
}
