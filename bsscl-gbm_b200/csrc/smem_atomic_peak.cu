// smem_atomic_peak.cu -- the ceiling of the histogram kernel's inner loop:
// 32-bit shared-memory atomic adds per second on this GPU, 2 CTAs of 512
// threads per SM (k_hist's shape), two access patterns:
//   (a) conflict-free: lane l of a warp adds to bank l;
//   (b) k_hist's pattern: 6 digit arrays of 16 features x 256 bins, bins
//       uniform random (bank and same-address conflicts as in real data);
//   (c) the same cell updates as 3 64-bit adds: each digit of g and of h
//       paired in one word (g_d + h_d * 2^32), 3 arrays of 16 x 256 words.
// Build and run: make -C bsscl-gbm_b200/csrc smem_atomic_peak && bsscl-gbm_b200/csrc/smem_atomic_peak
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdint>
__global__ void __launch_bounds__(512, 2) k_free(unsigned *out, int iters) {
    extern __shared__ unsigned acc[];
    for (int i = threadIdx.x; i < 6 * 4096; i += blockDim.x) acc[i] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int it = 0; it < iters; it++) {
#pragma unroll
        for (int d = 0; d < 6; d++) atomicAdd(&acc[d * 4096 + (w * 32 + ((it * 7) & 7) * 512 + lane) % 4096], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(out, acc[5]);
}
__global__ void __launch_bounds__(512, 2) k_rand(unsigned *out, int iters, unsigned seed) {
    extern __shared__ unsigned acc[];
    for (int i = threadIdx.x; i < 6 * 4096; i += blockDim.x) acc[i] = 0;
    __syncthreads();
    unsigned x = seed ^ (threadIdx.x * 2654435761u) ^ (blockIdx.x * 40503u);
    for (int it = 0; it < iters; it++) {
        x = x * 1664525u + 1013904223u;
        const int f = it & 15, b = (x >> 8) & 255;
#pragma unroll
        for (int d = 0; d < 6; d++) atomicAdd(&acc[d * 4096 + f * 256 + b], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(out, acc[5]);
}
__global__ void __launch_bounds__(512, 2) k_rand64(unsigned *out, int iters, unsigned seed) {
    extern __shared__ unsigned long long acc64[];
    for (int i = threadIdx.x; i < 3 * 4096; i += blockDim.x) acc64[i] = 0;
    __syncthreads();
    unsigned x = seed ^ (threadIdx.x * 2654435761u) ^ (blockIdx.x * 40503u);
    for (int it = 0; it < iters; it++) {
        x = x * 1664525u + 1013904223u;
        const int f = it & 15, b = (x >> 8) & 255;
#pragma unroll
        for (int d = 0; d < 3; d++) atomicAdd(&acc64[d * 4096 + f * 256 + b], 0x100000001ull);
    }
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(out, (unsigned)acc64[2]);
}
int main() {
    setvbuf(stdout, NULL, _IONBF, 0);
    int sms; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const int smem = 6 * 4096 * 4;
    cudaFuncSetAttribute(k_free, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_rand, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_rand64, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    unsigned *out; cudaMalloc(&out, 4);
    const int grid = 2 * sms, iters = 4096;
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    const char *names[] = {"conflict-free", "random bins (16 feat x 256)", "random bins, 64-bit pairs"};
    for (int mode = 0; mode < 3; mode++) {
        for (int rep = 0; rep < 3; rep++) {
            cudaEventRecord(a);
            if (mode == 0) k_free<<<grid, 512, smem>>>(out, iters);
            else if (mode == 1) k_rand<<<grid, 512, smem>>>(out, iters, rep);
            else k_rand64<<<grid, 512, smem>>>(out, iters, rep);
            cudaEventRecord(b); cudaEventSynchronize(b);
            float ms; cudaEventElapsedTime(&ms, a, b);
            const double cells = (double)grid * 512 * iters;   // (row, feature) cell updates
            const double ops = cells * (mode == 2 ? 3 : 6);
            printf("%s: %.3f ms, %.1f G lane-atomics/s, %.1f G cell updates/s\n", names[mode], ms, ops / ms / 1e6,
                   cells / ms / 1e6);
        }
    }
    cudaError_t e = cudaGetLastError();
    printf("status: %s\n", cudaGetErrorString(e));
    return e != cudaSuccess;
}
