// Path 4: the single-launch small-batch kernel for up to kSmallMaxRows rows, by
// default for kDecodeDefaultRows < M <= kSmallDefaultRows (included by mhc_pre_kernels.cu inside namespace mhc, after the decode kernel whose
// helpers it uses).
//
// Between the decode kernel's few rows and the split-K path's large batches, the
// operator is latency-bound: at M = 128 (config 5) x is 7.3 MB and the prepared
// weights 2.75 MB, a few microseconds of HBM time, while two launches and their
// dependent memory round trips cost more.  So one cooperative launch of G CTAs (one
// per SM, at most one per 64-wide chunk) does everything:
//   phase 1   CTA g takes the K-slice of chunks [g*C/G, (g+1)*C/G) for ALL T = M/128
//             row tiles.  Each ring stage holds the T x tiles of one chunk and the
//             chunk of the prepared weights, which all T tiles' tcgen05 MMAs share
//             (M=128, N=2*mix, K=16, one TMEM accumulator of N columns per tile,
//             flushed into fp32 registers every kSegChunks chunks as in the split-K
//             GEMM).  Four warps per tile form the rows' square sums from the same
//             stages and write the partial records [g][row][W].  Warp 1 issues tile
//             0's MMAs and each further tile's first warp its own, in parallel.
//   barrier   a grid barrier on the workspace header's arrival counter (bounded);
//   phase 2   row m belongs to CTA m % G, which finishes it alone: four warps each
//             sum a quarter of the row's G records in record (split) order (lanes
//             over the columns: coalesced), the quarters are added in order through
//             shared memory, one warp forms invRms, hPre, hPost and hRes, and all
//             threads stream the row's hIn with hPre from shared memory.
// A row's arithmetic depends on G and K only (not on timing or M): deterministic.
// The per-row formulas and their operation order are those of the split-K path's
// epilogue (reference code/op_kernel/mhc_pre.cpp:504-519, :736-758, :793-812).
#pragma once

constexpr int kSmallMaxTiles = kSmallMaxRows / kRowsPerTile;  // 4
constexpr int kSmallThreads = 576;  // 18 warps: TMA, TMEM allocation, 4 per tile (up to 4 tiles)
static_assert(2 + 4 * kSmallMaxTiles <= kSmallThreads / 32, "a warp quad per row tile");

struct SmallParams {
    int M;
    int tiles;      // ceil(M / 128)
    int chunks;     // ceil(K / 64)
    int stages;     // ring depth
    int segChunks;  // K chunks per TMEM accumulation segment
    int W;          // floats per partial record
    int64_t K;
    int64_t D;
    float invK;
    float normEps;
    float hcEps;
    uint32_t signature;
    const uint16_t* x;  // [M][K]
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    float* part;                  // [G][M][W]
    int64_t partFloats;           // floats of part (bounds checks of the debug build)
    unsigned long long* barrier;  // WorkspaceHeader::gridBarrier
    const WorkspaceHeader* hdr;
};

// TMEM columns the small kernel allocates: one accumulator of N columns per tile,
// rounded up to a power of two (at least 32).
__host__ __device__ constexpr uint32_t small_tmem_cols(int tiles, int N) {
    return tiles * N <= 32 ? 32 : tiles * N <= 64 ? 64 : tiles * N <= 128 ? 128 : tiles * N <= 256 ? 256 : 512;
}

// Grid barrier on the 64-bit arrival counter: each of the G CTAs adds 1, and the
// target is the next multiple of G above the value it found, so consecutive barriers
// (and launches) need no reset.  Thread 0 waits (bounded); returns false on timeout.
__device__ __forceinline__ bool small_grid_barrier(unsigned long long* counter, int G, volatile int* sFlag) {
    __syncthreads();  // the CTA's writes are done (CTA scope) ...
    if (threadIdx.x == 0) {
        __threadfence();  // ... and released at GPU scope with the arrival
        const unsigned long long old = atomicAdd(counter, 1ull);
        const unsigned long long target = (old / static_cast<unsigned long long>(G) + 1) * G;
        bool ok = false;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t i = 0; i < kMaxPolls; ++i) {
            if (ld_acquire_u64(counter) >= target) {
                ok = true;
                break;
            }
            if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) break;
            __nanosleep(32);
        }
        if (!ok) {
            *sFlag = 1;
            set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        }
    }
    __syncthreads();
    return *sFlag == 0;
}

template <int DT, int NS>
__global__ void __launch_bounds__(kSmallThreads, 1)
    mhc_pre_small_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiMap,
                         const SmallParams p) {
    constexpr int MIX = NS * NS + 2 * NS;
    constexpr int N = 2 * MIX;
    constexpr int kXBytes = kRowsPerTile * kChunk * 2;
    constexpr int kPhiBytes = N * kChunk * 2;
    const int T = p.tiles;
    const int S = p.stages;
    const int SC = p.segChunks;
    const size_t stageBytes = static_cast<size_t>(T) * kXBytes + kPhiBytes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * stageBytes);  // [S]
    uint64_t* empty = full + S;                                                                 // [S]
    uint64_t* accFull = empty + S;                   // [kSmallMaxTiles]
    uint64_t* accEmpty = accFull + kSmallMaxTiles;  // [kSmallMaxTiles]
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(accEmpty + kSmallMaxTiles);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);
    volatile int* sFlag = abortFlag + 1;

    const int G = gridDim.x;
    const int g = blockIdx.x;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int M = p.M;
    const uint32_t tmemCols = small_tmem_cols(T, N);
    const int c0 = static_cast<int>(static_cast<int64_t>(g) * p.chunks / G);
    const int nq = static_cast<int>(static_cast<int64_t>(g + 1) * p.chunks / G) - c0;  // >= 1 (G <= chunks)
    const int nSeg = (nq + SC - 1) / SC;
    // Without weights prepared for this description the launch returns before any
    // grid barrier (every CTA reads the same header), so the arrival counter only
    // ever sees launches of the description it was zeroed for, all with the same G.
    if (!(p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature)) {
        if (g == 0 && tid == 0) set_device_status(MHC_STATUS_NOT_PREPARED);
        return;
    }

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], T + 4 * T);  // each tile's MMA commit and its four warps
        }
        for (int t = 0; t < T; ++t) {
            mbar_init(&accFull[t], 1);
            mbar_init(&accEmpty[t], 4);
        }
        *abortFlag = 0;
        *sFlag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmemSlot, tmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&xMap);
        tma_prefetch_desc(&phiMap);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tacc = *tmemSlot;
    auto stage_x = [&](int s, int t) { return smem + static_cast<size_t>(s) * stageBytes + static_cast<size_t>(t) * kXBytes; };
    auto stage_phi = [&](int s) { return smem + static_cast<size_t>(s) * stageBytes + static_cast<size_t>(T) * kXBytes; };
    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
    };

    // ---------------- phase 1: partial records of this CTA's K-slice ----------------
    {
        if (warp == 0) {
            if (lane == 0) {
                int q = 0;
                for (; q < nq && !*abortFlag; ++q) {
                    const int s = q % S;
                    if (q >= S && !mbar_wait(&empty[s], (static_cast<uint32_t>(q / S) & 1u) ^ 1u, abortFlag)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(stageBytes));
                    const int kc = (c0 + q) * kChunk;
                    // rows past M (the last tile's tail) are filled with zeros by the copy
                    for (int t = 0; t < T; ++t) tma_load_2d(stage_x(s, t), &xMap, &full[s], kc, t * kRowsPerTile);
                    tma_load_2d(stage_phi(s), &phiMap, &full[s], kc, 0);
                }
                if (*abortFlag != 0) {
                    // let copies already in flight land before the CTA moves on (bounded)
                    for (int k = (q > S ? q - S : 0); k < q; ++k)
                        mbar_wait(&full[k % S], static_cast<uint32_t>(k / S) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp == 1) {
            // MMA issuer of tile 0 (the other tiles issue from their first square-sum
            // warp: one issuing thread retires a tcgen05.mma only about every 145
            // cycles, so the tiles issue in parallel)
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_f16(DT, kRowsPerTile, N);
                for (int q = 0; q < nq; ++q) {
                    const int s = q % S;
                    const int seg = q / SC;
                    if (q % SC == 0 && seg >= 1 &&
                        !mbar_wait(&accEmpty[0], static_cast<uint32_t>(seg - 1) & 1u, abortFlag)) {
                        fail();
                        break;
                    }
                    if (!mbar_wait(&full[s], static_cast<uint32_t>(q / S) & 1u, abortFlag)) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(stage_x(s, 0));
                    const uint32_t b0 = smem_u32(stage_phi(s));
#pragma unroll
                    for (int k16 = 0; k16 < kChunk / 16; ++k16)
                        mma_f16_ss(tacc, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                   (q % SC != 0 || k16 > 0) ? 1u : 0u);
                    mma_commit(&empty[s]);
                    if (q % SC == SC - 1 || q == nq - 1) mma_commit(&accFull[0]);
                }
            }
        } else if (warp < 2 + 4 * T) {
            // tile tw = (warp - 2) / 4, one token row per thread; TMEM lane quadrant =
            // warp % 4 (four consecutive warps cover all four).  For tiles 1.. lane 0
            // of the tile's first warp also issues the tile's MMAs.
            const int tw = (warp - 2) >> 2;
            const bool issuer = tw > 0 && ((warp - 2) & 3) == 0;
            constexpr uint32_t idesc = idesc_f16(DT, kRowsPerTile, N);
            const int q4 = warp & 3;
            const int row = q4 * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(q4 * 32) << 16);
            float run[MIX];
#pragma unroll
            for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
            float ss = 0.0f;
            bool ok = true;
            for (int q = 0; q < nq && ok; ++q) {
                const int s = q % S;
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>(q / S) & 1u, abortFlag))) {
                    ok = false;
                    break;
                }
                if (issuer) {
                    bool issued = true;
                    if (lane == 0) {
                        const int seg = q / SC;
                        // the tile's accumulator is free once its four warps flushed the
                        // previous segment (this warp did so at the end of chunk q-1)
                        if (q % SC == 0 && seg >= 1 &&
                            !mbar_wait(&accEmpty[tw], static_cast<uint32_t>(seg - 1) & 1u, abortFlag)) {
                            issued = false;
                        } else {
                            tc_fence_after();
                            const uint32_t a0 = smem_u32(stage_x(s, tw));
                            const uint32_t b0 = smem_u32(stage_phi(s));
                            const uint32_t d = tacc + static_cast<uint32_t>(tw * N);
#pragma unroll
                            for (int k16 = 0; k16 < kChunk / 16; ++k16)
                                mma_f16_ss(d, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                           (q % SC != 0 || k16 > 0) ? 1u : 0u);
                            mma_commit(&empty[s]);
                            if (q % SC == SC - 1 || q == nq - 1) mma_commit(&accFull[tw]);
                        }
                    }
                    if (!__all_sync(0xffffffffu, __shfl_sync(0xffffffffu, issued, 0))) {
                        ok = false;
                        break;
                    }
                }
                const uint32_t base = smem_u32(stage_x(s, tw)) + row * 128;
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
                if (q % SC == SC - 1 || q == nq - 1) {
                    // add the finished segment into run[] and free the accumulator
                    const int seg = q / SC;
                    if (!__all_sync(0xffffffffu,
                                    mbar_wait(&accFull[tw], static_cast<uint32_t>(seg) & 1u, abortFlag))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    add_segment<MIX>(lane_base, static_cast<uint32_t>(tw * N), run);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0 && seg + 1 < nSeg) mbar_arrive(&accEmpty[tw]);
                }
            }
            if (!ok) {
                if (lane == 0) fail();
            } else {
                const int m = tw * kRowsPerTile + row;
                const int64_t recAt = (static_cast<int64_t>(g) * M + m) * p.W;
                if (m < M && MHC_CHECK(recAt + MIX < p.partFloats)) {
                    const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
                    float* out = p.part + recAt;
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
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tacc, tmemCols);
    }

    // ---------------- grid barrier ----------------
    // Every CTA arrives, also one whose phase 1 gave up (its status is set), so that
    // the others do not wait for it until their limit; it then skips phase 2.
    if (!small_grid_barrier(p.barrier, G, sFlag)) return;
    const bool work = *abortFlag == 0;

    // ---------------- phase 2: rows of this CTA ----------------
    // Row m belongs to CTA m % G, up to four rows per round:
    //   (a) four warps share a row: warp k sums records [k*Q, (k+1)*Q) (Q = ceil(G/4))
    //       in record order, lane j taking columns j, j+32, ... (a record's columns
    //       are contiguous, so every load instruction is coalesced and a quarter's
    //       loads are in flight together); the quarters meet in shared memory;
    //   (b) one warp per row adds the quarters in order, forms invRms, writes hPost
    //       and hRes and leaves hPre in shared memory;
    //   (c) all threads stream the round's hIn (x of every stream, 8 elements per
    //       task, two tasks per iteration with their loads issued first).
    constexpr int COLS = MIX + 1;
    constexpr int CPL = (COLS + 31) / 32;  // columns per lane
    constexpr int kRecBatch = 40 / CPL;    // records whose loads are in flight together
    const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
    float* sq4 = reinterpret_cast<float*>(smem);  // [4 rows][4 quarters][COLS] (the ring is idle now)
    float* sPre = sq4 + 16 * COLS;                // [4 rows][NS]
    const int rowsHere = (g < M && work) ? (M - g + G - 1) / G : 0;  // rows g, g+G, ...
    const int recQ = (G + 3) / 4;
    const int64_t vecPerStream = p.D / 8;
    for (int j0 = 0; j0 < rowsHere; j0 += 4) {  // the same trip count for the whole CTA
        const int nr = min(4, rowsHere - j0);
        // (a) quarter sums
        if (warp < 4 * nr) {
            const int rsl = warp >> 2, k = warp & 3;
            const int m = g + G * (j0 + rsl);
            const int rb = k * recQ, re = min(G, rb + recQ);
            float tot[CPL];
#pragma unroll
            for (int c = 0; c < CPL; ++c) tot[c] = 0.0f;
            const float* rp = p.part + static_cast<int64_t>(m) * p.W + lane;
            const int64_t recStride = static_cast<int64_t>(M) * p.W;
            for (int r0 = rb; r0 < re; r0 += kRecBatch) {
                float v[kRecBatch][CPL];
#pragma unroll
                for (int i = 0; i < kRecBatch; ++i)
#pragma unroll
                    for (int c = 0; c < CPL; ++c)
                        v[i][c] = (r0 + i < re && lane + 32 * c < COLS &&
                                   MHC_CHECK(static_cast<int64_t>(m) * p.W + lane + (r0 + i) * recStride + 32 * c <
                                             p.partFloats))
                                      ? __ldcg(rp + (r0 + i) * recStride + 32 * c)
                                      : 0.0f;
#pragma unroll
                for (int i = 0; i < kRecBatch; ++i)
                    if (r0 + i < re)
#pragma unroll
                        for (int c = 0; c < CPL; ++c) tot[c] = __fadd_rn(tot[c], v[i][c]);
            }
#pragma unroll
            for (int c = 0; c < CPL; ++c)
                if (lane + 32 * c < COLS) sq4[(rsl * 4 + k) * COLS + lane + 32 * c] = tot[c];
        }
        __syncthreads();
        // (b) row totals and the small outputs
        if (warp < nr) {
            const int rsl = warp;
            const int m = g + G * (j0 + rsl);
            float tot[CPL];
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const int col = min(lane + 32 * c, COLS - 1);
                float t = sq4[(rsl * 4 + 0) * COLS + col];
#pragma unroll
                for (int k = 1; k < 4; ++k) t = __fadd_rn(t, sq4[(rsl * 4 + k) * COLS + col]);
                tot[c] = t;
            }
            // the square sum is column MIX: slot MIX / 32 of lane MIX % 32
            float sq = tot[0];
#pragma unroll
            for (int c = 1; c < CPL; ++c)
                if (c == MIX / 32) sq = tot[c];
            sq = __shfl_sync(0xffffffffu, sq, MIX % 32);
            // invRms = 1 / Sqrt(sum * invFlatDim + normEps)   (mhc_pre.cpp:504-519)
            float v = __fmul_rn(sq, p.invK);
            v = __fadd_rn(v, p.normEps);
            const float invRms = __fdiv_rn(1.0f, __fsqrt_rn(v));
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                const int col = lane + 32 * c;
                if (col < NS) {
                    const float t1 = __fadd_rn(__fmul_rn(tot[c], __fmul_rn(invRms, a0)), __ldg(p.bias + col));
                    sPre[rsl * NS + col] = __fadd_rn(sigmoid_ref(t1), p.hcEps);
                } else if (col < 2 * NS) {
                    const float t1 = __fadd_rn(__fmul_rn(tot[c], __fmul_rn(invRms, a1)), __ldg(p.bias + col));
                    p.hPost[static_cast<int64_t>(m) * NS + (col - NS)] = __fmul_rn(sigmoid_ref(t1), 2.0f);
                } else if (col < MIX) {
                    p.hRes[static_cast<int64_t>(m) * NS * NS + (col - 2 * NS)] =
                        __fadd_rn(__fmul_rn(tot[c], __fmul_rn(invRms, a2)), __ldg(p.bias + col));
                }
            }
        }
        __syncthreads();
        // (c) hIn = sum over streams s (in order from 0) of x_s * hPre_s, fp32, rounded RN
        const int64_t tasks = static_cast<int64_t>(nr) * vecPerStream;
        for (int64_t i0 = tid; i0 < tasks; i0 += 2 * kSmallThreads) {
            uint4 w[2][NS];
            int rs[2];
            int64_t vv[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t i = i0 + h * kSmallThreads;
                rs[h] = static_cast<int>(i / vecPerStream);
                vv[h] = i - rs[h] * vecPerStream;
                if (i < tasks) {
                    const int64_t m = g + static_cast<int64_t>(G) * (j0 + rs[h]);
                    const uint4* xr = reinterpret_cast<const uint4*>(p.x + m * p.K) + vv[h];
#pragma unroll
                    for (int s2 = 0; s2 < NS; ++s2) w[h][s2] = __ldg(xr + s2 * vecPerStream);
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (i0 + h * kSmallThreads >= tasks) break;
                const int64_t m = g + static_cast<int64_t>(G) * (j0 + rs[h]);
                float acc[8];
#pragma unroll
                for (int s2 = 0; s2 < NS; ++s2) {
                    const float pr = sPre[rs[h] * NS + s2];
                    const uint32_t ws[4] = {w[h][s2].x, w[h][s2].y, w[h][s2].z, w[h][s2].w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float2 f = x2_to_f32<DT>(ws[t]);
                        if (s2 == 0) {
                            acc[2 * t] = __fmul_rn(f.x, pr);
                            acc[2 * t + 1] = __fmul_rn(f.y, pr);
                        } else {
                            acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(f.x, pr));
                            acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(f.y, pr));
                        }
                    }
                }
                uint4 o;
                o.x = f32x2_to_x2<DT>(acc[0], acc[1]);
                o.y = f32x2_to_x2<DT>(acc[2], acc[3]);
                o.z = f32x2_to_x2<DT>(acc[4], acc[5]);
                o.w = f32x2_to_x2<DT>(acc[6], acc[7]);
                reinterpret_cast<uint4*>(p.hIn + m * p.D)[vv[h]] = o;
            }
        }
        // the next round's (a) writes sq4 only; its (b) writes sPre after a barrier
    }
}
