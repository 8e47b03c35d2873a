// Split-K GEMM on CTA pairs for n = 8 (included by mhc_pre_kernels.cu after the
// cluster kernel, whose cluster helpers it uses).
//
// At n = 8 the prepared weights of one 64-wide chunk are N = 160 rows (20 KB),
// larger than the chunk's 128-row x tile (16 KB): a stage of the one-CTA GEMM
// carries 16 of 36 KB as x, so the two CTAs an SM holds keep only about 96 KB of x
// in flight.  Here the two CTAs of a 2-CTA cluster share one tcgen05.mma of
// M = 256 rows (cta_group::2): each CTA stages its own 128-row x tile and HALF of
// the weight chunk (rows 0-79, the hi part, in the first CTA; rows 80-159, the lo
// part, in the second), the first CTA issues the MMA for both, and each CTA's TMEM
// receives its own rows' 160 accumulator columns.  A stage is then 16 + 10 KB, and
// four stages per CTA give about 128 KB of x in flight per SM, as at n = 4.
//
// Signalling within the pair (every wait bounded):
//   full[s]     in the first CTA: both CTAs' TMA loads of stage s complete on it
//               (the second CTA's loads address it across the pair); the first
//               CTA's producer sets the expected bytes of both.
//   xready[s]   in the second CTA: the first CTA's MMA thread arrives on it once
//               full[s] completed, so the second CTA's square-sum warps know their
//               x stage has landed.
//   empty[s]    in each CTA: the MMA's completion (a commit multicast to both
//               CTAs) plus that CTA's four square-sum warps free its stage s.
//   accFull     in each CTA: the MMA's commit (multicast) at a segment's end.
//   accEmpty    in the first CTA: all eight square-sum warps (four of them across
//               the pair) after adding the segment into their registers.
// The arithmetic of a row is the same as in the one-CTA GEMM (the same K = 16 MMA
// steps into a 4-chunk TMEM segment, the same fp32 flush order), so both give the
// same bits.
// No TMA load here uses multicast: each CTA loads its own x tile and weight half.
#pragma once

// tcgen05 and TMA forms for a CTA pair (cta_group::2).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on the mbarrier at this shared-memory offset in both CTAs of the
// pair when all tcgen05.mma this thread issued have completed.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (bar_cluster: a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t c0,
                                                 int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}

// Waits (acquire, cluster scope) for a phase of a local mbarrier that the partner
// CTA or a multicast commit arrives on.  Bounded; also gives up when the CTA's
// abort flag (may be null) is raised.
__device__ __forceinline__ bool mbar_wait_pair(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait_cluster(addr, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait_cluster(addr, parity)) return true;
        if ((i & 255u) == 255u) {
            if (abort != nullptr && *abort != 0) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) return false;
        }
    }
    return false;
}

constexpr int kPairN = 160;             // n = 8: 2 * mix
constexpr int kPairHalfN = kPairN / 2;  // weight rows each CTA stages
constexpr int kPairXBytes = kRowsPerTile * kChunk * 2;
constexpr int kPairPhiBytes = kPairHalfN * kChunk * 2;
constexpr int kPairStageBytes = kPairXBytes + kPairPhiBytes;  // 26 KB
constexpr uint32_t kPairTmemCols = 256;                       // 160 accumulator columns, rounded up

static_assert(pair_smem_bytes(0) == 1024 + 512, "host and device agree on the layout");

// GemmParams as for the one-CTA GEMM; tilesM counts 128-row tiles, items are
// (256-row pair tile, K split), CTA pair q takes items q, q + P, ... (P = grid / 2).
template <int DT>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiHalfMap,
                     const GemmParams p) {
    constexpr int MIX = kPairN / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * kPairStageBytes);  // [S]
    uint64_t* empty = full + S;     // [S]
    uint64_t* xready = empty + S;   // [S]
    uint64_t* accFull = xready + S;
    uint64_t* accEmpty = accFull + 1;
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(accEmpty + 1);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: issues the MMA; 1: its partner
    const int pair = blockIdx.x >> 1;
    const int P = gridDim.x >> 1;
    const int pairTiles = (p.tilesM + 1) / 2;
    const int numItems = pairTiles * p.splits;
    auto item_range = [&](int w, int& ptile, int& split, int& cBegin, int& nChunks) {
        ptile = w / p.splits;
        split = w - ptile * p.splits;
        cBegin = static_cast<int>((static_cast<int64_t>(split) * p.chunks) / p.splits);
        nChunks = static_cast<int>((static_cast<int64_t>(split + 1) * p.chunks) / p.splits) - cBegin;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);        // the first CTA's producer (plus both CTAs' bytes)
            mbar_init(&empty[s], 1 + 4);   // the MMA commit + this CTA's square-sum warps
            mbar_init(&xready[s], 1);      // the first CTA's MMA thread
        }
        mbar_init(accFull, 1);
        mbar_init(accEmpty, 8);  // the pair's eight square-sum warps
        *abortFlag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmemSlot, kPairTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&xMap);
        tma_prefetch_desc(&phiHalfMap);
    }
    tc_fence_before();
    // both CTAs' barriers are initialised before either addresses the other's
    cluster_barrier();
    tc_fence_after();
    grid_dependency_wait();   // as in the one-CTA GEMM: the kernel before this one is complete
    grid_launch_dependents();
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelBegin, 0, rank);
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);
    const uint32_t fullLead0 = cluster_map(smem_u32(&full[0]), 0);     // full[] of the first CTA
    const uint32_t accEmptyLead = cluster_map(smem_u32(accEmpty), 0);
    const uint32_t xreadyPeer0 = cluster_map(smem_u32(&xready[0]), 1);  // xready[] of the second CTA

    auto stage_x = [&](int s) { return smem + static_cast<size_t>(s) * kPairStageBytes; };
    auto stage_phi = [&](int s) { return smem + static_cast<size_t>(s) * kPairStageBytes + kPairXBytes; };
    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
    };

    if (prepared) {
        if (warp == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            if (lane == 0) {
                int g = 0;
                const int batch = p.batch;
                for (int w = pair; w < numItems && !*abortFlag; w += P) {
                    int ptile, split, cBegin, nChunks;
                    item_range(w, ptile, split, cBegin, nChunks);
                    const int rowBase = ptile * 2 * kRowsPerTile + static_cast<int>(rank) * kRowsPerTile;
                    MHC_TRACE_EV(kTrGemmItemBegin, ptile, split);
                    for (int i0 = 0; i0 < nChunks && !*abortFlag; i0 += batch) {
                        const int nb = min(batch, nChunks - i0);
                        bool okb = true;
                        for (int u = 0; u < nb; ++u) {
                            const int gg = g + u;
                            if (gg >= S &&
                                !mbar_wait(&empty[gg % S], (static_cast<uint32_t>(gg / S) & 1u) ^ 1u, abortFlag)) {
                                fail();
                                okb = false;
                                break;
                            }
                        }
                        if (!okb) break;
                        for (int u = 0; u < nb; ++u, ++g) {
                            const int s = g % S;
                            const int kc = (cBegin + i0 + u) * kChunk;
                            const uint32_t bar = fullLead0 + static_cast<uint32_t>(s) * 8u;
                            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
                            tma_load_2d_pair(stage_x(s), &xMap, bar, kc, rowBase);
                            tma_load_2d_pair(stage_phi(s), &phiHalfMap, bar, kc, static_cast<int>(rank) * kPairHalfN);
                        }
                    }
                }
                if (*abortFlag != 0) {
                    // Let this CTA's copies in flight land before it leaves: they
                    // land in its own stages; stage s of chunk k is free again once
                    // empty[s] passed phase k / S (bounded).
                    for (int k = (g > S ? g - S : 0); k < g; ++k)
                        mbar_wait(&empty[k % S], static_cast<uint32_t>(k / S) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp == 1) {
            // ---------------- MMA issuer (the first CTA) ----------------
            if (lane == 0 && rank == 0) {
                constexpr uint32_t idesc = idesc_f16(DT, 2 * kRowsPerTile, kPairN);
                int g = 0, segBase = 0;
                bool ok = true;
                for (int w = pair; w < numItems && ok; w += P) {
                    int ptile, split, cBegin, nChunks;
                    item_range(w, ptile, split, cBegin, nChunks);
                    for (int i = 0; i < nChunks; ++i, ++g) {
                        const int s = g % S;
                        const int seg = segBase + i / kSegChunks;
                        if (i % kSegChunks == 0 && seg >= 1 &&
                            !mbar_wait_pair(accEmpty, static_cast<uint32_t>(seg - 1) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&full[s], static_cast<uint32_t>(g / S) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        // the partner's x stage has landed too: its square-sum may start
                        mbar_remote_arrive(xreadyPeer0 + static_cast<uint32_t>(s) * 8u);
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(stage_x(s));
                        const uint32_t b0 = smem_u32(stage_phi(s));
#pragma unroll
                        for (int k16 = 0; k16 < kChunk / 16; ++k16) {
                            mma_f16_ss_pair(tacc, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                            (i % kSegChunks != 0 || k16 > 0) ? 1u : 0u);
                        }
                        mma_commit_pair_both(&empty[s]);
                        if (i % kSegChunks == kSegChunks - 1 || i == nChunks - 1) mma_commit_pair_both(accFull);
                    }
                    segBase += (nChunks + kSegChunks - 1) / kSegChunks;
                }
            }
        } else {
            // ---------------- square-sum + flush (both CTAs; one row per thread) ----------------
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(q * 32) << 16);
            float run[MIX];
            auto flush = [&](int seg) -> bool {
                if (!__all_sync(0xffffffffu, mbar_wait_pair(accFull, static_cast<uint32_t>(seg) & 1u, abortFlag)))
                    return false;
                tc_fence_after();
                add_segment<MIX>(lane_base, 0u, run);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(accEmpty);
                    else mbar_remote_arrive(accEmptyLead);
                }
                return true;
            };
            const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
            int g = 0, segBase = 0;
            bool ok = true;
            for (int w = pair; w < numItems && ok; w += P) {
                int ptile, split, cBegin, nChunks;
                item_range(w, ptile, split, cBegin, nChunks);
#pragma unroll
                for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
                float ss = 0.0f;
                for (int i = 0; i < nChunks; ++i, ++g) {
                    const int s = g % S;
                    const uint32_t par = static_cast<uint32_t>(g / S) & 1u;
                    // the first CTA's x is ready with full[s]; the second's with xready[s]
                    const bool ready = rank == 0 ? mbar_wait(&full[s], par, abortFlag)
                                                 : mbar_wait_pair(&xready[s], par, abortFlag);
                    if (!__all_sync(0xffffffffu, ready)) {
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
                    if (i % kSegChunks == kSegChunks - 1 || i == nChunks - 1) {
                        if (!flush(segBase + i / kSegChunks)) {
                            ok = false;
                            break;
                        }
                    }
                }
                segBase += (nChunks + kSegChunks - 1) / kSegChunks;
                if (!ok) break;
                const int64_t grow = static_cast<int64_t>(ptile) * 2 * kRowsPerTile + rank * kRowsPerTile + row;
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
                if (warp == 2 && lane == 0) MHC_TRACE_EV(kTrGemmRecord, ptile, split);
            }
            if (!ok && lane == 0) fail();
        }
    }

    // Neither CTA may leave while the pair's MMA can still read its stages or arrive
    // on its barriers: every role above has finished (all its waits are bounded),
    // then the pair meets once more before TMEM is freed.
    tc_fence_before();
    __syncthreads();
    cluster_barrier();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tacc, kPairTmemCols);
    }
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelEnd, 0, rank);
}
