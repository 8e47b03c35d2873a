// L2 -> SM read-bandwidth probe (test infrastructure: tests/test_probes_gpu.py
// builds and runs it).  Every thread streams 16-byte ld.global.cg loads over a
// buffer of a given size, several passes; a buffer that fits in L2 measures the
// L2 -> SM bandwidth, a 2 GiB one the DRAM read bandwidth.  It answers: how fast
// can the SMs re-read data that is still in L2 (the second read of x in a single
// pass), and up to what footprint does it stay there?
//   prints: blocks_per_sm threads_per_sm footprint_MB passes GB/s
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

__global__ void read_kernel(const uint4* __restrict__ p, size_t n16, int passes, unsigned* out) {
    unsigned acc = 0;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (int ps = 0; ps < passes; ++ps) {
        // rotate the starting offset per pass so no thread keeps the same lines
        const size_t i0 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x + static_cast<size_t>(ps) * 7919 * 32) % stride;
        for (size_t i = i0; i < n16; i += stride) {
            const uint4 v = __ldcg(p + i);
            acc ^= v.x ^ v.y ^ v.z ^ v.w;
        }
    }
    if (acc == 0x12345678u) out[0] = acc;  // keeps the loads
}

int main() {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const size_t maxBytes = static_cast<size_t>(2) << 30;
    uint4* buf = nullptr;
    unsigned* out = nullptr;
    if (cudaMalloc(&buf, maxBytes) != cudaSuccess || cudaMalloc(&out, 4) != cudaSuccess) return 1;
    cudaMemset(buf, 1, maxBytes);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    const size_t sizes[] = {static_cast<size_t>(16) << 20, static_cast<size_t>(32) << 20, static_cast<size_t>(48) << 20,
                            static_cast<size_t>(64) << 20, static_cast<size_t>(96) << 20, static_cast<size_t>(128) << 20,
                            maxBytes};
    for (int bpsm : {4, 8}) {
        for (size_t bytes : sizes) {
            const size_t n16 = bytes / 16;
            int passes = static_cast<int>((static_cast<size_t>(8) << 30) / bytes);
            if (passes < 2) passes = 2;
            const dim3 grid(sms * bpsm), block(256);
            read_kernel<<<grid, block>>>(buf, n16, 1, out);  // warm
            cudaEventRecord(a);
            read_kernel<<<grid, block>>>(buf, n16, passes, out);
            cudaEventRecord(b);
            cudaEventSynchronize(b);
            float ms = 0;
            cudaEventElapsedTime(&ms, a, b);
            printf("blocks_per_sm %d threads_per_sm %d footprint_MB %.1f passes %d GBps %.1f\n", bpsm, bpsm * 256,
                   bytes / 1e6, passes, static_cast<double>(bytes) * passes / (ms * 1e-3) / 1e9);
        }
    }
    const cudaError_t e = cudaGetLastError();
    printf("status %s\n", cudaGetErrorString(e));
    return e == cudaSuccess ? 0 : 1;
}
