// MhcPre kernels for B200 (sm_100a).
//
// Path 0 (every legal shape):
//   prepare   phi'[j,k] = gamma[k]*phi[j,k] split into hi + lo 16-bit halves of the x
//             dtype (fp16: scaled by a power of two into the normal range), stored
//             [2*mix][K] K-contiguous so TMA can stage it for the tensor cores.
//   gemm      persistent CTAs over (128-row tile, K split) items: TMA streams 64-wide K chunks of x
//             and phi' through a shared-memory ring; one thread issues tcgen05.mma
//             (M=128 token rows, N=2*mix, fp32 accumulators in TMEM); four warps
//             square-sum the same x chunks from shared memory and add finished
//             accumulator segments into fp32 registers; the epilogue writes fp32
//             partial records [split][row][mix partials, sum of squares].
//   epilogue  one CTA per row: sums the partial records over splits in a fixed
//             order, computes invRms, hPre/hPost/hRes, then hIn from x.
//
// Reference: code/op_kernel/mhc_pre.cpp (the AscendC kernel this replaces).
#include <algorithm>
#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "mhc_pre_internal.h"
#include "ptx.cuh"
#include "trace.cuh"

namespace mhc {

__device__ int g_device_status = 0;

__device__ __forceinline__ void set_device_status(int code) { atomicCAS(&g_device_status, 0, code); }

// Debug build (compile flag MHC_DEBUG; libmhcpre_b200_debug.so): MHC_CHECK(cond) guards
// an access -- the caller performs it only when the check passes; a failed check
// skips it, sets the device status word to MHC_STATUS_INTERNAL_CHECK and records the
// source line (mhcPreDebugLastCheckLine).  In the default build it is the constant
// true and costs nothing.
#ifdef MHC_DEBUG
__device__ int g_debug_line = 0;
__device__ __noinline__ bool debug_check_failed(int line) {
    set_device_status(MHC_STATUS_INTERNAL_CHECK);
    atomicCAS(&g_debug_line, 0, line);
    return false;
}
#define MHC_CHECK(cond) ((cond) ? true : ::mhc::debug_check_failed(__LINE__))
#else
#define MHC_CHECK(cond) true
#endif

// ---------------------------------------------------------------------------
// 16-bit helpers
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ uint16_t f32_to_x(float v) {
    if constexpr (DT == MHC_DTYPE_BF16) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    } else {
        return __half_as_ushort(__float2half_rn(v));
    }
}

// Unpacks the two 16-bit values of a 32-bit word to fp32 (exact).
template <int DT>
__device__ __forceinline__ float2 x2_to_f32(uint32_t w) {
    if constexpr (DT == MHC_DTYPE_BF16) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    } else {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        return __half22float2(h);
    }
}

template <int DT>
__device__ __forceinline__ uint32_t f32x2_to_x2(float a, float b) {
    return static_cast<uint32_t>(f32_to_x<DT>(a)) | (static_cast<uint32_t>(f32_to_x<DT>(b)) << 16);
}

// ---------------------------------------------------------------------------
// Weight preparation
// ---------------------------------------------------------------------------
__global__ void prep_maxabs_kernel(const float* __restrict__ phi, const float* __restrict__ gamma, int64_t K,
                                   int mix, uint32_t* __restrict__ maxbits) {
    const int64_t total = static_cast<int64_t>(mix) * K;
    float m = 0.0f;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v = phi[i];
        if (gamma != nullptr) v = __fmul_rn(v, gamma[i % K]);
        v = fabsf(v);
        if (v > m && v <= 3.0e38f) m = v;
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(maxbits, __float_as_uint(m));
}

template <int DT>
__global__ void prep_split_kernel(const float* __restrict__ phi, const float* __restrict__ gamma, int64_t K, int mix,
                                  WorkspaceHeader* __restrict__ hdr, uint16_t* __restrict__ out, uint32_t signature) {
    int e = 0;
    if constexpr (DT == MHC_DTYPE_F16) {
        // Scale so that max|phi'| * 2^e < 2^15: hi and lo then stay normal fp16.
        const float mx = __uint_as_float(hdr->maxAbsBits);
        if (mx > 0.0f) {
            int ex = 0;
            frexpf(mx, &ex);
            e = 15 - ex;
            e = max(-100, min(100, e));
        }
    }
    const float scale = ldexpf(1.0f, e);
    const int64_t total = static_cast<int64_t>(mix) * K;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = i / K;
        const int64_t k = i - j * K;
        float v = phi[i];
        if (gamma != nullptr) v = __fmul_rn(v, gamma[k]);
        v = __fmul_rn(v, scale);
        const uint16_t hb = f32_to_x<DT>(v);
        float hf;
        if constexpr (DT == MHC_DTYPE_BF16) {
            hf = __bfloat162float(__ushort_as_bfloat16(hb));
        } else {
            hf = __half2float(__ushort_as_half(hb));
        }
        const uint16_t lb = f32_to_x<DT>(__fsub_rn(v, hf));
        out[j * K + k] = hb;
        out[(mix + j) * K + k] = lb;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        hdr->phiScaleExp = e;
        hdr->signature = signature;
        hdr->magic = kPreparedMagic;
    }
}

// ---------------------------------------------------------------------------
// Path 0, kernel 1: split-K GEMM (tcgen05) + square-sum
// ---------------------------------------------------------------------------
struct GemmParams {
    int64_t M;
    int tilesM;
    int batch;      // chunks issued together by the producer
    int mix;
    int W;
    int chunks;
    int splits;
    int stages;
    uint32_t signature;  // of the description: the workspace must hold weights prepared for it
    float* partials;
    int64_t partFloats;  // floats of the records buffer (bounds checks of the debug build)
    const WorkspaceHeader* hdr;
};



// Adds one finished TMEM accumulator segment (hi columns [0,MIX), lo columns
// [MIX,2*MIX) at column `col`, this warp's lane quadrant in `lane_base`) into the
// fp32 running sums.  The loads of a group are all issued before one wait, so a
// flush costs about one TMEM round trip per group instead of one per 8 columns.
template <int MIX>
__device__ __forceinline__ void add_segment(uint32_t lane_base, uint32_t col, float (&run)[MIX]) {
    constexpr int G = (MIX % 24 == 0) ? 24 : 40;  // columns per group: 24 (mix 24, 48) or 40 (mix 80)
    static_assert(MIX % G == 0 && G % 8 == 0, "group must tile the mix columns");
#pragma unroll
    for (int j0 = 0; j0 < MIX; j0 += G) {
        uint32_t hi[G], lo[G];
#pragma unroll
        for (int k = 0; k < G; k += 8) {
            tmem_ld_x8(lane_base + col + j0 + k, *reinterpret_cast<uint32_t(*)[8]>(hi + k));
            tmem_ld_x8(lane_base + col + MIX + j0 + k, *reinterpret_cast<uint32_t(*)[8]>(lo + k));
        }
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < G; ++t)
            run[j0 + t] = __fadd_rn(run[j0 + t], __fadd_rn(__uint_as_float(hi[t]), __uint_as_float(lo[t])));
    }
}

constexpr int kGemmThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 square-sum + epilogue

// The tensor core accumulates in fp32 but does not round like an IEEE fp32 adder:
// over thousands of K steps the accumulator drifts (measured ~1e-4 relative at
// K = 32768).  Each TMEM accumulation therefore covers only kSegChunks 64-wide
// K chunks; finished segments are added into IEEE fp32 registers by the epilogue
// warps while the MMA fills the other accumulator buffer.
constexpr int kSegChunks = 4;
// CTAs per SM the GEMM is compiled for (their registers must fit that share of the
// SM's): four for n=4, two for n=8, one for n=6 (which runs two within that budget).
template <int N>
constexpr int gemm_min_ctas() { return N <= 48 ? 4 : N > 128 ? 2 : 1; }

template <int N>
struct GemmCfg {
    static constexpr int kXBytes = kRowsPerTile * kChunk * 2;  // 16 KB
    static constexpr int kPhiBytes = N * kChunk * 2;          // N rows x 128 B
    static constexpr int kStageBytes = kXBytes + kPhiBytes;
    // Accumulator buffers: with two, the square-sum warps add segment s-1 into
    // registers while the MMA fills segment s; two buffers keep a CTA's TMEM at 128
    // columns for n=4 (four CTAs per SM) and 256 for n=6 (two).  n=8 (N=160) keeps
    // one, so that two CTAs fit the SM's 512 columns: the MMA then waits for each
    // flush, which the other CTA covers.
    static constexpr int kAccBufs = N > 128 ? 1 : 2;
    static constexpr int kFlushLag = kAccBufs - 1;
    // kAccBufs accumulator buffers of N fp32 columns each
    static constexpr uint32_t kTmemCols = kAccBufs * N <= 64    ? 64
                                          : kAccBufs * N <= 128 ? 128
                                          : kAccBufs * N <= 256 ? 256
                                                                : 512;
    static_assert(kAccBufs * N <= 512, "accumulator buffers must fit in TMEM");
    static_assert(N % 16 == 0 && N <= 256, "MMA N for M=128 must be a multiple of 16, at most 256");
};

template <int DT, int N>
__global__ void __launch_bounds__(kGemmThreads, gemm_min_ctas<N>())
    gemm_sumsq_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiMap,
                      const GemmParams p) {
    // Persistent: CTA b processes the work items (row tile, K split) b, b+G, b+2G, ...
    // with one continuous TMA/MMA pipeline, so the SM never drains between items.
    using Cfg = GemmCfg<N>;
    constexpr int MIX = N / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * Cfg::kStageBytes);  // [S]
    uint64_t* empty = full + S;
    constexpr int kAccBufs = Cfg::kAccBufs;
    constexpr int kFlushLag = Cfg::kFlushLag;
    uint64_t* accFull = empty + S;            // [kAccBufs]
    uint64_t* accEmpty = accFull + kAccBufs;  // [kAccBufs]
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(accEmpty + kAccBufs);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int numItems = p.tilesM * p.splits;
    const int G = gridDim.x;
    auto item_range = [&](int w, int& tile, int& split, int& cBegin, int& nChunks) {
        tile = w / p.splits;
        split = w - tile * p.splits;
        cBegin = static_cast<int>((static_cast<int64_t>(split) * p.chunks) / p.splits);
        nChunks = static_cast<int>((static_cast<int64_t>(split + 1) * p.chunks) / p.splits) - cBegin;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + 4);
        }
        for (int b = 0; b < kAccBufs; ++b) {
            mbar_init(&accFull[b], 1);
            mbar_init(&accEmpty[b], 4);
        }
        *abortFlag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmemSlot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&xMap);
        tma_prefetch_desc(&phiMap);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // This grid is launched as a programmatic dependent of the kernel before it in the
    // stream: the launch and the set-up above overlap that kernel's tail, and every
    // thread waits here, before its first read of global memory, for that kernel to
    // complete (its writes, x or the prepared weights among them, are then visible).
    grid_dependency_wait();
    // the epilogue grid may start launching now; it waits for this grid in-kernel
    grid_launch_dependents();
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelBegin, 0, 0);
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);

    auto stage_x = [&](int s) { return smem + static_cast<size_t>(s) * Cfg::kStageBytes; };
    auto stage_phi = [&](int s) { return smem + static_cast<size_t>(s) * Cfg::kStageBytes + Cfg::kXBytes; };
    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
    };

    if (prepared) {
        if (warp == 0) {
            if (lane == 0) {
                int g = 0;
                const int batch = p.batch;
                for (int w = blockIdx.x; w < numItems && !*abortFlag; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    MHC_TRACE_EV(kTrGemmItemBegin, tile, split);
                    // Chunks are issued in batches of consecutive K ranges, so that each
                    // row's neighbouring 128-byte segments reach DRAM close together.
                    for (int i0 = 0; i0 < nChunks && !*abortFlag; i0 += batch) {
                        const int nb = min(batch, nChunks - i0);
                        bool okb = true;
                        for (int u = 0; u < nb; ++u) {
                            const int gg = g + u;
                            if (gg >= S && !mbar_wait(&empty[gg % S], (static_cast<uint32_t>(gg / S) & 1u) ^ 1u, abortFlag)) {
                                fail();
                                okb = false;
                                break;
                            }
                        }
                        if (!okb) break;
                        for (int u = 0; u < nb; ++u, ++g) {
                            const int s = g % S;
                            mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
                            const int kc = (cBegin + i0 + u) * kChunk;
                            tma_load_2d(stage_x(s), &xMap, &full[s], kc, tile * kRowsPerTile);
                            tma_load_2d(stage_phi(s), &phiMap, &full[s], kc, 0);
                        }
                    }
                }
                if (*abortFlag != 0) {
                    // Let copies already in flight land before the CTA exits (bounded).
                    for (int k = (g > S ? g - S : 0); k < g; ++k)
                        mbar_wait(&full[k % S], static_cast<uint32_t>(k / S) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp == 1) {
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_f16(DT, kRowsPerTile, N);
                int g = 0, segBase = 0;
                bool ok = true;
                for (int w = blockIdx.x; w < numItems && ok; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    for (int i = 0; i < nChunks; ++i, ++g) {
                        const int s = g % S;
                        const int seg = segBase + i / kSegChunks;
                        const int b = seg % kAccBufs;
                        if (i % kSegChunks == 0 && seg >= kAccBufs &&
                            !mbar_wait(&accEmpty[b], static_cast<uint32_t>(seg / kAccBufs - 1) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&full[s], static_cast<uint32_t>(g / S) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(stage_x(s));
                        const uint32_t b0 = smem_u32(stage_phi(s));
                        const uint32_t d = tacc + static_cast<uint32_t>(b * N);
#pragma unroll
                        for (int k16 = 0; k16 < kChunk / 16; ++k16) {
                            mma_f16_ss(d, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                       (i % kSegChunks != 0 || k16 > 0) ? 1u : 0u);
                        }
                        mma_commit(&empty[s]);
                        if (i % kSegChunks == kSegChunks - 1 || i == nChunks - 1) mma_commit(&accFull[b]);
                    }
                    segBase += (nChunks + kSegChunks - 1) / kSegChunks;
                }
            }
        } else {
            // warps 2..5: one token row per thread; TMEM lane quadrant = warp % 4
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(q * 32) << 16);
            float run[MIX];
            // Adds finished accumulator segment `seg` into run[] and frees its buffer.
            auto flush = [&](int seg) -> bool {
                const int b = seg % kAccBufs;
                // warp-uniform outcome: the TMEM loads below are warp-collective
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&accFull[b], static_cast<uint32_t>(seg / kAccBufs) & 1u, abortFlag)))
                    return false;
                tc_fence_after();
                add_segment<MIX>(lane_base, static_cast<uint32_t>(b * N), run);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&accEmpty[b]);
                return true;
            };
            const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
            int g = 0, segBase = 0;
            bool ok = true;
            for (int w = blockIdx.x; w < numItems && ok; w += G) {
                int tile, split, cBegin, nChunks;
                item_range(w, tile, split, cBegin, nChunks);
#pragma unroll
                for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
                float ss = 0.0f;
                for (int i = 0; i < nChunks; ++i, ++g) {
                    const int s = g % S;
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>(g / S) & 1u, abortFlag))) {
                        ok = false;
                        break;
                    }
                    const uint32_t base = smem_u32(stage_x(s)) + row * 128;
                    float part = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint4 v = lds128(base + ((j ^ (row & 7)) << 4));
                        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float2 f = x2_to_f32<DT>(wv[t]);
                            part = fmaf(f.x, f.x, part);
                            part = fmaf(f.y, f.y, part);
                        }
                    }
                    ss += part;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                    const int segL = i / kSegChunks;
                    if ((i % kSegChunks == kSegChunks - 1 || i == nChunks - 1) && segL >= kFlushLag) {
                        if (!flush(segBase + segL - kFlushLag)) {
                            ok = false;
                            break;
                        }
                    }
                }
                {
                    // the item's remaining segments (the last kFlushLag, or fewer)
                    const int nSeg = (nChunks + kSegChunks - 1) / kSegChunks;
                    for (int sg = max(0, nSeg - kFlushLag); sg < nSeg && ok; ++sg) ok = flush(segBase + sg);
                }
                segBase += (nChunks + kSegChunks - 1) / kSegChunks;
                if (!ok) break;
                const int64_t grow = static_cast<int64_t>(tile) * kRowsPerTile + row;
                const int64_t recAt = (static_cast<int64_t>(split) * p.M + grow) * p.W;
                if (grow < p.M && MHC_CHECK(split < p.splits && recAt + MIX < p.partFloats)) {
                    float* out = p.partials + recAt;
#pragma unroll
                    for (int j0 = 0; j0 < MIX; j0 += 4) {
                        float4 a;
                        a.x = __fmul_rn(run[j0 + 0], unscale);
                        a.y = __fmul_rn(run[j0 + 1], unscale);
                        a.z = __fmul_rn(run[j0 + 2], unscale);
                        a.w = __fmul_rn(run[j0 + 3], unscale);
                        *reinterpret_cast<float4*>(out + j0) = a;
                    }
                    out[MIX] = ss;
                }
                if (warp == 2 && lane == 0) MHC_TRACE_EV(kTrGemmRecord, tile, split);
            }
            if (!ok && lane == 0) fail();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tacc, Cfg::kTmemCols);
    }
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelEnd, 0, 0);
}

// ---------------------------------------------------------------------------
// Path 0, kernel 2: split reduction, epilogue, hIn
// ---------------------------------------------------------------------------
struct EpiParams {
    int64_t M;
    int64_t D;
    int64_t K;
    int mix;
    int W;
    int splits;
    float invK;
    float normEps;
    float hcEps;
    const float* partials;
    int64_t partFloats;  // floats of the records buffer (bounds checks of the debug build)
    const uint16_t* x;
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    int blocksPerSm;  // 12 or 16: the epilogue variant
};

constexpr int kEpiThreads = 128;
// Splits whose partial records the epilogue stages in shared memory at a time: the
// loads of a block are all in flight together instead of one split after another.
constexpr int kEpiSplitBlock = 48;

// sigmoid(v) = 1 / (1 + exp(-v)), in the operation order of the reference's
// Sigmoid helper (code/op_kernel/mhc_pre.cpp:542-555).
__device__ __forceinline__ float sigmoid_ref(float v) {
    float t = __fmul_rn(v, -1.0f);
    t = expf(t);
    t = __fadd_rn(t, 1.0f);
    return __fdiv_rn(1.0f, t);
}

// Launched as a programmatic dependent of the GEMM: it waits for the GEMM's
// completion (and memory) before reading the partial records.  Dynamic shared
// memory: min(splits, kEpiSplitBlock) * (mix + 1) floats.
// BLOCKS: resident blocks per SM it is compiled for (12: 40 registers a thread; 16:
// at most 32).  The arithmetic does not depend on it.
template <int DT, int NS, int BLOCKS>
__global__ void __launch_bounds__(kEpiThreads, BLOCKS) epilogue_hin_kernel(const EpiParams p) {
    constexpr int mix = NS * NS + 2 * NS;
    constexpr int cols = mix + 1;
    extern __shared__ float sPart[];  // [block split][cols]
    __shared__ float sMix[mix];
    __shared__ float sPre[NS];
    __shared__ float sSum;
    // Rows in reverse: the GEMM's last items read the last tiles, whose x is still
    // partly in L2 when this grid's first CTAs start.
    const int64_t r = p.M - 1 - blockIdx.x;
    const int tid = threadIdx.x;
    grid_dependency_wait();
    // a following split-K GEMM may start launching (it waits for this grid before it
    // reads or writes global memory)
    grid_launch_dependents();
    if (tid == 0) MHC_TRACE_EV(kTrEpiRowBegin, static_cast<uint64_t>(r) & 0xffffffffu, static_cast<uint64_t>(r) >> 32);
    // sum over splits in split order, staged kEpiSplitBlock splits at a time
    float acc = 0.0f;
    for (int sp0 = 0; sp0 < p.splits; sp0 += kEpiSplitBlock) {
        const int nb = min(kEpiSplitBlock, p.splits - sp0);
        const int vals = nb * cols;
#pragma unroll 8
        for (int i = tid; i < vals; i += kEpiThreads) {
            const int sp = i / cols;
            const int j = i - sp * cols;
            const int64_t at = (static_cast<int64_t>(sp0 + sp) * p.M + r) * p.W + j;
            sPart[i] = MHC_CHECK(at < p.partFloats && i < kEpiSplitBlock * cols) ? __ldcg(p.partials + at) : 0.0f;
        }
        __syncthreads();
        if (tid < cols)
            for (int sp = 0; sp < nb; ++sp) acc = __fadd_rn(acc, sPart[sp * cols + tid]);
        __syncthreads();
    }
    if (tid < mix) sMix[tid] = acc;
    else if (tid == mix) sSum = acc;
    __syncthreads();
    // invRms = 1 / Sqrt(sum * invFlatDim + normEps)   (mhc_pre.cpp:504-519)
    float v = __fmul_rn(sSum, p.invK);
    v = __fadd_rn(v, p.normEps);
    const float invRms = __fdiv_rn(1.0f, __fsqrt_rn(v));
    const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
    if (tid < NS) {
        const float sPreScale = __fmul_rn(invRms, a0);
        const float sPostScale = __fmul_rn(invRms, a1);
        float t = __fadd_rn(__fmul_rn(sMix[tid], sPreScale), __ldg(p.bias + tid));
        sPre[tid] = __fadd_rn(sigmoid_ref(t), p.hcEps);
        float u = __fadd_rn(__fmul_rn(sMix[NS + tid], sPostScale), __ldg(p.bias + NS + tid));
        p.hPost[r * NS + tid] = __fmul_rn(sigmoid_ref(u), 2.0f);
    }
    if (tid < NS * NS) {
        const float sResScale = __fmul_rn(invRms, a2);
        p.hRes[r * NS * NS + tid] =
            __fadd_rn(__fmul_rn(sMix[2 * NS + tid], sResScale), __ldg(p.bias + 2 * NS + tid));
    }
    __syncthreads();
    float pre[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) pre[s] = sPre[s];
    const uint4* xr = reinterpret_cast<const uint4*>(p.x + r * p.K);
    uint4* hr = reinterpret_cast<uint4*>(p.hIn + r * p.D);
    const int64_t vecPerStream = p.D / 8;
    for (int64_t vi = tid; vi < vecPerStream; vi += kEpiThreads) {
        float acc[8];
        {
            const uint4 w = __ldg(xr + vi);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = x2_to_f32<DT>(ws[t]);
                acc[2 * t] = __fmul_rn(f.x, pre[0]);
                acc[2 * t + 1] = __fmul_rn(f.y, pre[0]);
            }
        }
#pragma unroll
        for (int s = 1; s < NS; ++s) {
            const uint4 w = __ldg(xr + s * vecPerStream + vi);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = x2_to_f32<DT>(ws[t]);
                acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(f.x, pre[s]));
                acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(f.y, pre[s]));
            }
        }
        uint4 o;
        o.x = f32x2_to_x2<DT>(acc[0], acc[1]);
        o.y = f32x2_to_x2<DT>(acc[2], acc[3]);
        o.z = f32x2_to_x2<DT>(acc[4], acc[5]);
        o.w = f32x2_to_x2<DT>(acc[6], acc[7]);
        hr[vi] = o;
    }
    if (tid == 0) MHC_TRACE_EV(kTrEpiRowDone, static_cast<uint64_t>(r) & 0xffffffffu, static_cast<uint64_t>(r) >> 32);
}

#include "mhc_pre_fused.cuh"
#include "mhc_pre_cluster.cuh"
#include "mhc_pre_pair.cuh"
#include "mhc_pre_decode.cuh"
#include "mhc_pre_small.cuh"
#include "mhc_pre_onepass.cuh"
#include "mhc_post.cuh"
#include "mhc_post_pre.cuh"

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
#ifdef MHC_DEBUG
// Debug build: a cap on the records-buffer size the kernels are told (0: none), so
// a test can make their bounds checks fail on purpose without any access outside a
// buffer (a failed check skips the access).
static std::atomic<int64_t> g_debug_record_cap{0};
void debug_set_record_cap(int64_t floats) { g_debug_record_cap.store(floats); }
int debug_last_check_line(int* line) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(line, g_debug_line, sizeof(int));
    const int zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_debug_line, &zero, sizeof(int));
    return e;
}
static int64_t debug_record_limit(int64_t floats) {
    const int64_t cap = g_debug_record_cap.load();
    return cap > 0 && cap < floats ? cap : floats;
}
#else
static int64_t debug_record_limit(int64_t floats) { return floats; }
#endif
int launch_prepare(const Problem& p, const Plan& plan, const float* phi, const float* gamma, void* workspace,
                   cudaStream_t stream) {
    auto* hdr = reinterpret_cast<WorkspaceHeader*>(workspace);
    auto* out = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(workspace) + plan.phiOffset);
    cudaError_t e = cudaMemsetAsync(hdr, 0, sizeof(WorkspaceHeader), stream);
    if (e != cudaSuccess) return e;
    const float* g = p.hasGamma ? gamma : nullptr;
    const int64_t total = static_cast<int64_t>(p.mix) * p.K;
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 8));
    if (p.dtype == MHC_DTYPE_F16) {
        prep_maxabs_kernel<<<blocks, threads, 0, stream>>>(phi, g, p.K, p.mix, &hdr->maxAbsBits);
        prep_split_kernel<MHC_DTYPE_F16><<<blocks, threads, 0, stream>>>(phi, g, p.K, p.mix, hdr, out, p.signature);
    } else {
        prep_split_kernel<MHC_DTYPE_BF16><<<blocks, threads, 0, stream>>>(phi, g, p.K, p.mix, hdr, out, p.signature);
    }
    return cudaGetLastError();
}

// Raises a kernel's dynamic shared memory limit on the current device when the
// launch needs more than was already set there (the attribute call costs host time,
// so each kernel remembers the largest value set per device).
constexpr int kMaxDevices = 64;
template <typename Kern>
static cudaError_t ensure_smem(Kern kern, std::atomic<int> (&setBytes)[kMaxDevices], size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int want = static_cast<int>(bytes);
    if (dev >= 0 && dev < kMaxDevices && setBytes[dev].load(std::memory_order_acquire) >= want) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
        int cur = setBytes[dev].load(std::memory_order_relaxed);
        while (cur < want && !setBytes[dev].compare_exchange_weak(cur, want, std::memory_order_release)) {
        }
    }
    return e;
}

template <int DT, int N>
static int launch_gemm(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap, const GemmParams& gp,
                       cudaStream_t stream) {
    auto kern = gemm_sumsq_kernel<DT, N>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: see the wait at the top of the kernel
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.gemmGrid), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, xMap, phiMap, gp);
}

template <int DT>
static int launch_gemm_pair(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiHalfMap,
                            const GemmParams& gp, cudaStream_t stream) {
    auto kern = gemm_pair_kernel<DT>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    // clusters of two CTAs (the pair), launched as a programmatic dependent like the
    // one-CTA GEMM.  Pairs never wait on other pairs: they need not all be resident.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.gemmGrid), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, xMap, phiHalfMap, gp);
}

template <int DT, int NS>
static int launch_epi(const Problem& p, const EpiParams& ep, cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(std::min(ep.splits, kEpiSplitBlock)) * (p.mix + 1) * sizeof(float);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.M), 1, 1);
    cfg.blockDim = dim3(kEpiThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // programmatic dependent launch: starts while the GEMM drains, waits in-kernel
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, ep.blocksPerSm == 16 ? epilogue_hin_kernel<DT, NS, 16> : epilogue_hin_kernel<DT, NS, 12>,
                              ep);
}

template <int DT, int NS>
static int launch_fused_t(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap, const FusedParams& fp,
                          cudaStream_t stream) {
    auto kern = mhc_pre_fused_kernel<DT, NS>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.teams * plan.teamS), 1, 1);
    cfg.blockDim = dim3(kFusedThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: teams wait on each other
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, xMap, phiMap, fp);
}

static int launch_fused(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                        const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes, void* workspace,
                        cudaStream_t stream, cudaEvent_t evBegin, cudaEvent_t evEnd) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + plan.cntOffset, 0, plan.cntBytes, stream);
    if (e != cudaSuccess) return e;
    FusedParams fp;
    fp.M = p.M;
    fp.D = p.D;
    fp.J = plan.J;
    fp.S = plan.teamS;
    fp.T = plan.teams;
    fp.tilesM = plan.tilesM;
    fp.W = p.W;
    fp.gStages = plan.gStages;
    fp.hStages = plan.hStages;
    fp.l2mode = plan.l2mode;
    fp.invK = 1.0f / static_cast<float>(p.K);
    fp.normEps = p.normEps;
    fp.hcEps = p.hcEps;
    fp.alpha = alpha;
    fp.bias = bias;
    fp.hIn = static_cast<uint16_t*>(hIn);
    fp.hPost = hPost;
    fp.hRes = hRes;
    fp.part = reinterpret_cast<float*>(ws + plan.partOffset);
    fp.hpre = reinterpret_cast<float*>(ws + plan.hpreOffset);
    fp.cnt = reinterpret_cast<unsigned*>(ws + plan.cntOffset);
    fp.hdr = reinterpret_cast<const WorkspaceHeader*>(workspace);
    fp.signature = p.signature;
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc;
    switch (p.n) {
        case 4: rc = bf ? launch_fused_t<MHC_DTYPE_BF16, 4>(plan, xMap, phiMap, fp, stream)
                        : launch_fused_t<MHC_DTYPE_F16, 4>(plan, xMap, phiMap, fp, stream); break;
        case 6: rc = bf ? launch_fused_t<MHC_DTYPE_BF16, 6>(plan, xMap, phiMap, fp, stream)
                        : launch_fused_t<MHC_DTYPE_F16, 6>(plan, xMap, phiMap, fp, stream); break;
        default: rc = bf ? launch_fused_t<MHC_DTYPE_BF16, 8>(plan, xMap, phiMap, fp, stream)
                         : launch_fused_t<MHC_DTYPE_F16, 8>(plan, xMap, phiMap, fp, stream); break;
    }
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    return 0;
}

template <int DT, int NS>
static int launch_decode_t(const Plan& plan, const DecodeParams& dp, cudaStream_t stream) {
    auto kern = mhc_pre_decode_kernel<DT, NS>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.gemmGrid), 1, 1);
    cfg.blockDim = dim3(kDecodeThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // the grid barrier needs every CTA resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, dp);
}

static int launch_decode(const Problem& p, const Plan& plan, const void* x, const float* alpha, const float* bias,
                         void* hIn, float* hPost, float* hRes, void* workspace, cudaStream_t stream,
                         cudaEvent_t evBegin, cudaEvent_t evEnd) {
    auto* hdr = reinterpret_cast<WorkspaceHeader*>(workspace);
    DecodeParams dp;
    dp.M = static_cast<int>(p.M);
    dp.chunks = plan.chunks;
    dp.W = p.W;
    dp.K = p.K;
    dp.D = p.D;
    dp.invK = 1.0f / static_cast<float>(p.K);
    dp.normEps = p.normEps;
    dp.hcEps = p.hcEps;
    dp.x = static_cast<const uint16_t*>(x);
    dp.phi = reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(workspace) + plan.phiOffset);
    dp.alpha = alpha;
    dp.bias = bias;
    dp.hIn = static_cast<uint16_t*>(hIn);
    dp.hPost = hPost;
    dp.hRes = hRes;
    dp.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.partOffset);
    dp.partFloats = debug_record_limit(static_cast<int64_t>(plan.partBytes / 4));
    dp.barrier = &hdr->gridBarrier;
    dp.hdr = hdr;
    dp.signature = p.signature;
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc;
    switch (p.n) {
        case 4: rc = bf ? launch_decode_t<MHC_DTYPE_BF16, 4>(plan, dp, stream)
                        : launch_decode_t<MHC_DTYPE_F16, 4>(plan, dp, stream); break;
        case 6: rc = bf ? launch_decode_t<MHC_DTYPE_BF16, 6>(plan, dp, stream)
                        : launch_decode_t<MHC_DTYPE_F16, 6>(plan, dp, stream); break;
        default: rc = bf ? launch_decode_t<MHC_DTYPE_BF16, 8>(plan, dp, stream)
                         : launch_decode_t<MHC_DTYPE_F16, 8>(plan, dp, stream); break;
    }
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    return 0;
}

size_t decode_smem(const Problem& p) { return decode_smem_bytes(static_cast<int>(p.M), p.mix); }

int launch_post(const Problem& p, const void* x, const void* y, const float* hPost, const float* hRes, void* xNext,
                cudaStream_t stream) {
    PostParams pp;
    pp.M = p.M;
    pp.D = p.D;
    pp.x = static_cast<const uint16_t*>(x);
    pp.y = static_cast<const uint16_t*>(y);
    pp.hPost = hPost;
    pp.hRes = hRes;
    pp.xNext = static_cast<uint16_t*>(xNext);
    const dim3 grid(static_cast<unsigned>(p.M)), block(kPostThreads);
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    switch (p.n) {
        case 4:
            if (bf) mhc_post_kernel<MHC_DTYPE_BF16, 4><<<grid, block, 0, stream>>>(pp);
            else mhc_post_kernel<MHC_DTYPE_F16, 4><<<grid, block, 0, stream>>>(pp);
            break;
        case 6:
            if (bf) mhc_post_kernel<MHC_DTYPE_BF16, 6><<<grid, block, 0, stream>>>(pp);
            else mhc_post_kernel<MHC_DTYPE_F16, 6><<<grid, block, 0, stream>>>(pp);
            break;
        default:
            if (bf) mhc_post_kernel<MHC_DTYPE_BF16, 8><<<grid, block, 0, stream>>>(pp);
            else mhc_post_kernel<MHC_DTYPE_F16, 8><<<grid, block, 0, stream>>>(pp);
            break;
    }
    return cudaGetLastError();
}

template <int DT, int NS>
static int launch_small_t(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap, const SmallParams& sp,
                          cudaStream_t stream) {
    auto kern = mhc_pre_small_kernel<DT, NS>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.gemmGrid), 1, 1);
    cfg.blockDim = dim3(kSmallThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // the grid barriers need every CTA resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, xMap, phiMap, sp);
}

static int launch_small(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                        const void* x, const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes,
                        void* workspace, cudaStream_t stream, cudaEvent_t evBegin, cudaEvent_t evEnd) {
    auto* hdr = reinterpret_cast<WorkspaceHeader*>(workspace);
    SmallParams sp;
    sp.M = static_cast<int>(p.M);
    sp.tiles = plan.tilesM;
    sp.chunks = plan.chunks;
    sp.stages = plan.stages;
    sp.segChunks = kSegChunks;
    sp.W = p.W;
    sp.K = p.K;
    sp.D = p.D;
    sp.invK = 1.0f / static_cast<float>(p.K);
    sp.normEps = p.normEps;
    sp.hcEps = p.hcEps;
    sp.signature = p.signature;
    sp.x = static_cast<const uint16_t*>(x);
    sp.alpha = alpha;
    sp.bias = bias;
    sp.hIn = static_cast<uint16_t*>(hIn);
    sp.hPost = hPost;
    sp.hRes = hRes;
    sp.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.partOffset);
    sp.partFloats = debug_record_limit(static_cast<int64_t>(plan.partBytes / 4));
    sp.barrier = &hdr->gridBarrier;
    sp.hdr = hdr;
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc;
    switch (p.n) {
        case 4: rc = bf ? launch_small_t<MHC_DTYPE_BF16, 4>(plan, xMap, phiMap, sp, stream)
                        : launch_small_t<MHC_DTYPE_F16, 4>(plan, xMap, phiMap, sp, stream); break;
        case 6: rc = bf ? launch_small_t<MHC_DTYPE_BF16, 6>(plan, xMap, phiMap, sp, stream)
                        : launch_small_t<MHC_DTYPE_F16, 6>(plan, xMap, phiMap, sp, stream); break;
        default: rc = bf ? launch_small_t<MHC_DTYPE_BF16, 8>(plan, xMap, phiMap, sp, stream)
                         : launch_small_t<MHC_DTYPE_F16, 8>(plan, xMap, phiMap, sp, stream); break;
    }
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    return 0;
}

size_t cluster_extra(const Problem& p) { return cluster_extra_smem(p.W); }

template <int DT, int NS>
static cudaError_t cluster_prepare_attrs(const Plan& plan) {
    auto kern = mhc_pre_cluster_kernel<DT, NS>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    if (plan.teamS > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
}

template <int DT, int NS>
static int cluster_teams_t(const Plan& plan, int* teams) {
    cudaError_t e = cluster_prepare_attrs<DT, NS>(plan);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.teamS), 1, 1);
    cfg.blockDim = dim3(kClusterThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(plan.teamS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, mhc_pre_cluster_kernel<DT, NS>, &cfg);
    if (e != cudaSuccess) return e;
    *teams = n;
    return 0;
}

// Clusters of plan.teamS CTAs that fit on the device at once (the persistent teams).
int cluster_max_teams(const Problem& p, const Plan& plan, int* teams) {
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    switch (p.n) {
        case 4: return bf ? cluster_teams_t<MHC_DTYPE_BF16, 4>(plan, teams) : cluster_teams_t<MHC_DTYPE_F16, 4>(plan, teams);
        case 6: return bf ? cluster_teams_t<MHC_DTYPE_BF16, 6>(plan, teams) : cluster_teams_t<MHC_DTYPE_F16, 6>(plan, teams);
        default: return bf ? cluster_teams_t<MHC_DTYPE_BF16, 8>(plan, teams) : cluster_teams_t<MHC_DTYPE_F16, 8>(plan, teams);
    }
}

template <int DT, int NS>
static int launch_cluster_t(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                            const ClusterParams& cp, cudaStream_t stream) {
    cudaError_t e = cluster_prepare_attrs<DT, NS>(plan);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(plan.teams * plan.teamS), 1, 1);
    cfg.blockDim = dim3(kClusterThreads, 1, 1);
    cfg.dynamicSmemBytes = plan.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(plan.teamS);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mhc_pre_cluster_kernel<DT, NS>, xMap, phiMap, cp);
}

static int launch_cluster(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                          const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes, void* workspace,
                          cudaStream_t stream, cudaEvent_t evBegin, cudaEvent_t evEnd) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + plan.cntOffset, 0, plan.cntBytes, stream);
    if (e != cudaSuccess) return e;
    ClusterParams cp;
    cp.M = p.M;
    cp.D = p.D;
    cp.J = plan.J;
    cp.S = plan.teamS;
    cp.T = plan.teams;
    cp.tilesM = plan.tilesM;
    cp.W = p.W;
    cp.gStages = plan.gStages;
    cp.hStages = plan.hStages;
    cp.l2mode = plan.l2mode;
    cp.lead = plan.lead;
    cp.invK = 1.0f / static_cast<float>(p.K);
    cp.normEps = p.normEps;
    cp.hcEps = p.hcEps;
    cp.alpha = alpha;
    cp.bias = bias;
    cp.hIn = static_cast<uint16_t*>(hIn);
    cp.hPost = hPost;
    cp.hRes = hRes;
    cp.gAbort = reinterpret_cast<unsigned*>(ws + plan.cntOffset);
    cp.hdr = reinterpret_cast<const WorkspaceHeader*>(workspace);
    cp.signature = p.signature;
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc;
    switch (p.n) {
        case 4: rc = bf ? launch_cluster_t<MHC_DTYPE_BF16, 4>(plan, xMap, phiMap, cp, stream)
                        : launch_cluster_t<MHC_DTYPE_F16, 4>(plan, xMap, phiMap, cp, stream); break;
        case 6: rc = bf ? launch_cluster_t<MHC_DTYPE_BF16, 6>(plan, xMap, phiMap, cp, stream)
                        : launch_cluster_t<MHC_DTYPE_F16, 6>(plan, xMap, phiMap, cp, stream); break;
        default: rc = bf ? launch_cluster_t<MHC_DTYPE_BF16, 8>(plan, xMap, phiMap, cp, stream)
                         : launch_cluster_t<MHC_DTYPE_F16, 8>(plan, xMap, phiMap, cp, stream); break;
    }
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    return 0;
}

template <int DT, int EW, int MINB>
static int launch_onepass_t(const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                            const OnePassParams& op, cudaStream_t stream) {
    auto kern = mhc_pre_onepass_kernel<DT, 4, EW, MINB>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, plan.smemBytes);
    if (e != cudaSuccess) return e;
    // The hIn warps wait for other CTAs' items, so every CTA must be resident: the
    // grid is the CTAs per SM that the plan sized shared memory, registers and TMEM
    // for (two or three) times the SMs.  It is an ordinary launch: the runtime's
    // occupancy calculator reports one CTA per SM for kernels of this kind (the
    // split-K GEMM included, which runs four), so a cooperative launch would be
    // refused.  Should a CTA not be resident, the waits give up (bounded) and the
    // call reports MHC_STATUS_DEVICE_TIMEOUT.
    kern<<<plan.gemmGrid, onepass_threads<EW>(), plan.smemBytes, stream>>>(xMap, phiMap, op);
    return cudaGetLastError();
}

static int launch_onepass(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
                          const void* x, const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes,
                          void* workspace, cudaStream_t stream, cudaEvent_t evBegin, cudaEvent_t evEnd) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + plan.cntOffset, 0, plan.cntBytes, stream);
    if (e != cudaSuccess) return e;
    OnePassParams op;
    op.M = p.M;
    op.D = p.D;
    op.K = p.K;
    op.tilesM = plan.tilesM;
    op.chunks = plan.chunks;
    op.splits = plan.splits;
    op.stages = plan.stages;
    op.batch = std::max(1, plan.tmaBatch);
    op.W = p.W;
    op.RT = plan.ringTiles;
    op.invK = 1.0f / static_cast<float>(p.K);
    op.normEps = p.normEps;
    op.hcEps = p.hcEps;
    op.signature = p.signature;
    op.x = static_cast<const uint16_t*>(x);
    op.alpha = alpha;
    op.bias = bias;
    op.hIn = static_cast<uint16_t*>(hIn);
    op.hPost = hPost;
    op.hRes = hRes;
    op.rec = reinterpret_cast<float*>(ws + plan.partOffset);
    op.recFloats = debug_record_limit(static_cast<int64_t>(plan.partBytes / 4));
    op.cnt = reinterpret_cast<unsigned*>(ws + plan.cntOffset);
    op.hdr = reinterpret_cast<const WorkspaceHeader*>(workspace);
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc;
    if (plan.opCtasPerSm == 2)
        rc = bf ? launch_onepass_t<MHC_DTYPE_BF16, 8, 2>(plan, xMap, phiMap, op, stream)
                : launch_onepass_t<MHC_DTYPE_F16, 8, 2>(plan, xMap, phiMap, op, stream);
    else
        rc = bf ? launch_onepass_t<MHC_DTYPE_BF16, 4, 3>(plan, xMap, phiMap, op, stream)
                : launch_onepass_t<MHC_DTYPE_F16, 4, 3>(plan, xMap, phiMap, op, stream);
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    return 0;
}

int launch_run(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
               const void* x, const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes,
               void* workspace, cudaStream_t stream, cudaEvent_t evBegin, cudaEvent_t evEnd) {
    if (plan.path == 5)
        return launch_onepass(p, plan, xMap, phiMap, x, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin,
                              evEnd);
    if (plan.path == 1)
        return launch_fused(p, plan, xMap, phiMap, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin, evEnd);
    if (plan.path == 2)
        return launch_decode(p, plan, x, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin, evEnd);
    if (plan.path == 3)
        return launch_cluster(p, plan, xMap, phiMap, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin, evEnd);
    if (plan.path == 4)
        return launch_small(p, plan, xMap, phiMap, x, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin, evEnd);
    GemmParams gp;
    gp.M = p.M;
    gp.tilesM = plan.tilesM;
    gp.batch = std::max(1, plan.tmaBatch);
    gp.mix = p.mix;
    gp.W = p.W;
    gp.chunks = plan.chunks;
    gp.splits = plan.splits;
    gp.stages = plan.stages;
    gp.signature = p.signature;
    gp.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.partOffset);
    gp.partFloats = debug_record_limit(static_cast<int64_t>(plan.partBytes / 4));
    gp.hdr = reinterpret_cast<const WorkspaceHeader*>(workspace);
    int rc;
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    if (evBegin != nullptr && cudaEventRecord(evBegin, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    switch (p.n) {
        case 4: rc = bf ? launch_gemm<MHC_DTYPE_BF16, 48>(plan, xMap, phiMap, gp, stream)
                        : launch_gemm<MHC_DTYPE_F16, 48>(plan, xMap, phiMap, gp, stream); break;
        case 6: rc = bf ? launch_gemm<MHC_DTYPE_BF16, 96>(plan, xMap, phiMap, gp, stream)
                        : launch_gemm<MHC_DTYPE_F16, 96>(plan, xMap, phiMap, gp, stream); break;
        default:
            if (plan.pairGemm)
                rc = bf ? launch_gemm_pair<MHC_DTYPE_BF16>(plan, xMap, phiMap, gp, stream)
                        : launch_gemm_pair<MHC_DTYPE_F16>(plan, xMap, phiMap, gp, stream);
            else
                rc = bf ? launch_gemm<MHC_DTYPE_BF16, 160>(plan, xMap, phiMap, gp, stream)
                        : launch_gemm<MHC_DTYPE_F16, 160>(plan, xMap, phiMap, gp, stream);
            break;
    }
    if (rc != 0) return rc;
    if (evEnd != nullptr && cudaEventRecord(evEnd, stream) != cudaSuccess) return cudaErrorInvalidResourceHandle;
    EpiParams ep;
    ep.M = p.M;
    ep.D = p.D;
    ep.K = p.K;
    ep.mix = p.mix;
    ep.W = p.W;
    ep.splits = plan.splits;
    ep.invK = 1.0f / static_cast<float>(p.K);
    ep.normEps = p.normEps;
    ep.hcEps = p.hcEps;
    ep.partials = gp.partials;
    ep.partFloats = gp.partFloats;
    ep.blocksPerSm = plan.epiBlocks;
    ep.x = static_cast<const uint16_t*>(x);
    ep.alpha = alpha;
    ep.bias = bias;
    ep.hIn = static_cast<uint16_t*>(hIn);
    ep.hPost = hPost;
    ep.hRes = hRes;
    switch (p.n) {
        case 4: return bf ? launch_epi<MHC_DTYPE_BF16, 4>(p, ep, stream) : launch_epi<MHC_DTYPE_F16, 4>(p, ep, stream);
        case 6: return bf ? launch_epi<MHC_DTYPE_BF16, 6>(p, ep, stream) : launch_epi<MHC_DTYPE_F16, 6>(p, ep, stream);
        default: return bf ? launch_epi<MHC_DTYPE_BF16, 8>(p, ep, stream) : launch_epi<MHC_DTYPE_F16, 8>(p, ep, stream);
    }
}

// ---------------------------------------------------------------------------
// The post step fused with the next MhcPre's contraction, then the split-K epilogue
// ---------------------------------------------------------------------------
bool post_pre_applies(const Problem& p, const Plan& defaultPlan) {
    return p.n == kPostPreNS && p.D % kChunk == 0 && defaultPlan.path == 0;
}

PostPrePlan make_post_pre_plan(const Problem& p, const Plan& defaultPlan, int smCount) {
    PostPrePlan pp{};
    pp.tilesM = defaultPlan.tilesM;
    pp.dChunks = static_cast<int>(p.D / kChunk);
    // as many splits as the split-K plan (so the same workspace holds the records),
    // at most one per d-chunk
    pp.splits = std::max(1, std::min(defaultPlan.splits, pp.dChunks));
    pp.stages = kPostPreStages;
    pp.grid = std::min(pp.tilesM * pp.splits, smCount);  // one CTA per SM
    pp.smemBytes = post_pre_smem_bytes(pp.stages);
    return pp;
}

template <int DT>
static int launch_post_pre_kernel(const PostPrePlan& pp, const CUtensorMap& xMap, const CUtensorMap& yMap,
                                  const CUtensorMap& xNextMap, const CUtensorMap& phiMap, const PostPreParams& prm,
                                  cudaStream_t stream) {
    auto kern = post_pre_kernel<DT>;
    static std::atomic<int> setBytes[kMaxDevices];
    cudaError_t e = ensure_smem(kern, setBytes, pp.smemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pp.grid), 1, 1);
    cfg.blockDim = dim3(kPostPreThreads, 1, 1);
    cfg.dynamicSmemBytes = pp.smemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, xMap, yMap, xNextMap, phiMap, prm);
}

int launch_post_pre(const Problem& p, const PostPrePlan& pp, const Plan& plan, const CUtensorMap& xMap,
                    const CUtensorMap& yMap, const CUtensorMap& xNextMap, const CUtensorMap& phiMap,
                    const float* hPost, const float* hRes, const void* xNext, const float* alpha, const float* bias,
                    void* hIn, float* hPostNext, float* hResNext, void* workspace, cudaStream_t stream) {
    PostPreParams prm;
    prm.M = p.M;
    prm.D = p.D;
    prm.tilesM = pp.tilesM;
    prm.dChunks = pp.dChunks;
    prm.splits = pp.splits;
    prm.stages = pp.stages;
    prm.W = p.W;
    prm.signature = p.signature;
    prm.hPost = hPost;
    prm.hRes = hRes;
    prm.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.partOffset);
    prm.partFloats = debug_record_limit(static_cast<int64_t>(plan.partBytes / 4));
    prm.hdr = reinterpret_cast<const WorkspaceHeader*>(workspace);
    const bool bf = p.dtype == MHC_DTYPE_BF16;
    int rc = bf ? launch_post_pre_kernel<MHC_DTYPE_BF16>(pp, xMap, yMap, xNextMap, phiMap, prm, stream)
                : launch_post_pre_kernel<MHC_DTYPE_F16>(pp, xMap, yMap, xNextMap, phiMap, prm, stream);
    if (rc != 0) return rc;
    EpiParams ep;
    ep.M = p.M;
    ep.D = p.D;
    ep.K = p.K;
    ep.mix = p.mix;
    ep.W = p.W;
    ep.splits = pp.splits;
    ep.invK = 1.0f / static_cast<float>(p.K);
    ep.normEps = p.normEps;
    ep.hcEps = p.hcEps;
    ep.partials = prm.partials;
    ep.partFloats = prm.partFloats;
    ep.blocksPerSm = plan.epiBlocks;
    ep.x = static_cast<const uint16_t*>(xNext);
    ep.alpha = alpha;
    ep.bias = bias;
    ep.hIn = static_cast<uint16_t*>(hIn);
    ep.hPost = hPostNext;
    ep.hRes = hResNext;
    return bf ? launch_epi<MHC_DTYPE_BF16, kPostPreNS>(p, ep, stream) : launch_epi<MHC_DTYPE_F16, kPostPreNS>(p, ep, stream);
}

// ---------------------------------------------------------------------------
// Diagnostics: the bounded waits give up as designed
// ---------------------------------------------------------------------------
// A counter that nothing ever sets.
__device__ unsigned g_diag_never_set = 0;

// Waits, with the given limit, on the two kinds of wait the kernels use: a global
// counter (cross-CTA handshakes) that nothing increments, and an mbarrier (TMA and
// MMA rings) that nothing arrives on.  Both must give up; the kernel then reports
// MHC_STATUS_DEVICE_TIMEOUT through the device status word and returns normally,
// so the context stays usable.  result[0..1] = 1 where a wait gave up.
__global__ void diag_wait_timeout_kernel(uint64_t limit_ns, int* result) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool counterDone = wait_counter(&g_diag_never_set, 1u, nullptr, limit_ns);
        const bool barrierDone = mbar_wait(&bar, 0u, nullptr, limit_ns);
        result[0] = counterDone ? 0 : 1;
        result[1] = barrierDone ? 0 : 1;
        if (!counterDone || !barrierDone) set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
    }
}

int diag_wait_timeout(uint64_t limit_ns, int* result_host, cudaStream_t stream) {
    int* d = nullptr;
    cudaError_t e = cudaMalloc(&d, 2 * sizeof(int));
    if (e != cudaSuccess) return e;
    diag_wait_timeout_kernel<<<1, 32, 0, stream>>>(limit_ns, d);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(result_host, d, 2 * sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    cudaFree(d);
    return e;
}

#ifdef MHC_TRACE
// Copies the recorded stage stamps to the host and clears the trace (trace build).
int trace_read(void* dst, size_t maxRecords, size_t* recorded) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    unsigned n = 0;
    if ((e = cudaMemcpyFromSymbol(&n, g_trace_count, sizeof(n))) != cudaSuccess) return e;
    const size_t avail = std::min<size_t>(n, kTraceCapacity);
    const size_t take = std::min(avail, maxRecords);
    if (take > 0 && dst != nullptr &&
        (e = cudaMemcpyFromSymbol(dst, g_trace, take * sizeof(TraceRecord))) != cudaSuccess)
        return e;
    const unsigned zero = 0;
    if ((e = cudaMemcpyToSymbol(g_trace_count, &zero, sizeof(zero))) != cudaSuccess) return e;
    *recorded = n;
    return 0;
}
#endif

int read_and_clear_device_status(int32_t* status) {
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
    if (e != cudaSuccess) return e;
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return e;
    *status = v;
    return 0;
}

}  // namespace mhc
