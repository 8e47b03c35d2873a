// tcgen05.mma issue-rate probe (test infrastructure: tests/test_probes_gpu.py builds
// and runs it).  One CTA per SM; `issuers` warps each issue `iters` x 4 MMAs
// (kind::f16, bf16, K = 16 each, a 64-wide K chunk) of shape M x N from shared
// memory into their own TMEM accumulator, back to back, then one commit; the
// kernel reports the cycles from the first issue to the completion of the last.
// It answers: how many x bytes per cycle can one SM push through the tensor core
// when the token rows sit on the MMA's N dimension (N = rows, 8..32) rather than on
// M (M = 128 rows)?  Operands are zeros: the rate does not depend on the values.
//   usage: mma_rate <iters>    prints: M N issuers cycles_per_mma x_bytes_per_cycle
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "../../mhcpre_review_b200/csrc/ptx.cuh"

using namespace mhc;

constexpr int kMaxIssuers = 4;

__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int M, int N, int issuers, int iters,
                                                         unsigned long long* cycles, int* status) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* A = smem;                 // 128 rows x 128 B (SW128, K-major)
    uint8_t* B = smem + 128 * 128;     // 256 rows x 128 B
    uint64_t* done = reinterpret_cast<uint64_t*>(B + 256 * 128);  // [kMaxIssuers]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(done + kMaxIssuers);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < (128 + 256) * 128 / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (int k = 0; k < kMaxIssuers; ++k) mbar_init(&done[k], 1);
        fence_mbarrier_init();
    }
    fence_proxy_async();  // the zeroed operands are read by the tensor core (async proxy)
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;
    if (warp < issuers && lane == 0) {
        const uint32_t idesc = idesc_f16(1, static_cast<uint32_t>(M), static_cast<uint32_t>(N));
        const int stride = N <= 128 ? 128 : 256;                      // accumulator columns per issuer
        const uint32_t d = tbase + static_cast<uint32_t>(warp * stride);
        const uint32_t a0 = smem_u32(A), b0 = smem_u32(B);
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16)
                mma_f16_ss(d, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc, (it | k16) ? 1u : 0u);
        }
        mma_commit(&done[warp]);
        const bool ok = mbar_wait(&done[warp], 0u, nullptr, 1000000000ull);
        const long long t1 = clock64();
        cycles[blockIdx.x * kMaxIssuers + warp] = static_cast<unsigned long long>(t1 - t0);
        if (!ok) atomicExch(status, 1);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

int main(int argc, char** argv) {
    const int iters = argc > 1 ? atoi(argv[1]) : 256;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    unsigned long long* cyc;
    int* status;
    cudaMalloc(&cyc, sizeof(unsigned long long) * sms * kMaxIssuers);
    cudaMalloc(&status, sizeof(int));
    cudaMemset(status, 0, sizeof(int));
    // 120 KB of shared memory: one CTA per SM (each allocates all 512 TMEM columns)
    const size_t smem = 120 * 1024;
    cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    struct Shape { int M, N; } shapes[] = {{64, 8}, {64, 16}, {64, 32}, {64, 64}, {64, 128}, {64, 256},
                                           {128, 16}, {128, 48}, {128, 96}, {128, 160}, {128, 256}};
    unsigned long long* host = new unsigned long long[sms * kMaxIssuers];
    for (const Shape& s : shapes) {
        for (int issuers : {1, 2, 4}) {
            if (issuers * (s.N <= 128 ? 128 : 256) > 512) continue;  // accumulators must fit TMEM
            mma_rate_kernel<<<sms, 128, smem>>>(s.M, s.N, issuers, iters, cyc, status);
            cudaError_t e = cudaDeviceSynchronize();
            if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); return 1; }
            cudaMemcpy(host, cyc, sizeof(unsigned long long) * sms * kMaxIssuers, cudaMemcpyDeviceToHost);
            double worst = 0;  // the slowest issuer of the slowest SM
            for (int b = 0; b < sms; ++b)
                for (int w = 0; w < issuers; ++w) worst = host[b * kMaxIssuers + w] > worst ? host[b * kMaxIssuers + w] : worst;
            const double perMma = worst / (4.0 * iters);            // cycles per MMA per issuer
            // x bytes per MMA: rows on M -> M x 16 x 2; rows on N -> N x 16 x 2 (the other operand is the weights)
            const int rows = s.M == 128 ? 128 : s.N;
            const double xBytesPerCycle = issuers * rows * 16 * 2 / perMma;
            printf("M %3d N %3d issuers %d cycles_per_mma %8.1f x_bytes_per_cycle %7.1f (rows on %s)\n", s.M, s.N,
                   issuers, perMma, xBytesPerCycle, s.M == 128 ? "M" : "N");
        }
    }
    int st = 0;
    cudaMemcpy(&st, status, sizeof(int), cudaMemcpyDeviceToHost);
    printf("status %d\n", st);
    return st;
}
