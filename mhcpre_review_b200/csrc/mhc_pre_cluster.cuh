// Path 3: the single-pass MhcPre with cluster teams (included by mhc_pre_kernels.cu
// inside namespace mhc, after the fused kernel, whose FusedCfg and ring sizes it
// shares).
//
// A team is a thread-block cluster of S CTAs (S = 16 or 8, one CTA per SM).  Team t
// processes the 128-row tiles t, t+T, ...; member c owns the D-slice
// [c*J*64, (c+1)*J*64) of every stream.  Per tile, each member:
//   1. streams its chunks of x and of the prepared weights through a TMA ring into
//      tcgen05.mma (M=128 rows, N=2*mix), accumulating in 4-chunk segments that
//      warps 4-7 add into fp32 registers, which also square-sum x;
//   2. writes each row's partial record straight into the shared memory of the
//      row's owner (member r / (128/S)) over DSMEM, then arrives on the owner's
//      mbarrier (release, cluster scope);
//   3. as an owner (warp 3), waits for its S records per row, sums them in member
//      order (the result does not depend on timing), computes invRms, hPre, hPost
//      and hRes, writes hPost/hRes, and writes hPre into every member's shared
//      memory, arriving on each member's mbarrier;
//   4. re-reads its chunks of the tile through a second TMA ring (an L2 hit: the
//      team read them a tile ago) and forms hIn for its slice.
// Step 4 of tile i overlaps steps 1-3 of tile i+1.  The handshake of steps 2-3
// stays inside the cluster (about a microsecond, measured), and the GEMM producer
// may run at most one tile plus `lead` chunks ahead of the hIn warps' consumption,
// so the data all CTAs stream between a chunk's read and its re-read stays near one
// tile per CTA (about 60 MB at config 4), which L2 holds.
// Every wait is bounded; a timeout sets the device status word and a global abort
// word, and all roles wind down.  A cluster barrier at the end keeps every CTA's
// shared memory alive until its peers are done with it.
#pragma once

struct ClusterParams {
    int64_t M;
    int64_t D;
    int J;        // 64-wide chunks per stream per member
    int S;        // cluster (team) size
    int T;        // teams (clusters resident together)
    int tilesM;   // ceil(M / 128)
    int W;        // floats per partial record
    int gStages;  // GEMM ring depth
    int hStages;  // hIn ring depth
    int l2mode;   // as FusedParams::l2mode
    int lead;     // chunks the first read may run ahead of the re-read beyond one tile
    float invK;
    float normEps;
    float hcEps;
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    unsigned* gAbort;  // global abort word (zeroed per run)
    const WorkspaceHeader* hdr;
    uint32_t signature;
};

constexpr int kClusterThreads = 384;  // 12 warps, the roles of the fused kernel

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

// Arrives on an mbarrier of another CTA of the cluster, releasing this thread's
// earlier writes at cluster scope.
__device__ __forceinline__ void mbar_remote_arrive(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits (acquire, cluster scope) for a phase of a local mbarrier that CTAs of the
// cluster arrive on.  Bounded; also gives up when the global abort word is set.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, const unsigned* gabort) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try_wait_cluster(addr, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0; i < kMaxPolls; ++i) {
        if (mbar_try_wait_cluster(addr, parity)) return true;
        if ((i & 255u) == 255u) {
            if (*reinterpret_cast<const volatile unsigned*>(gabort) != 0) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) return false;
        }
    }
    return false;
}

__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// Every thread of every CTA of the cluster.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile(
        "barrier.cluster.arrive.release.aligned;\n"
        "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Shared memory of the cluster kernel beyond the two rings, in bytes.
__host__ __device__ constexpr size_t cluster_extra_smem(int W) {
    return static_cast<size_t>(2) * kRowsPerTile * W * 4   // records of the owned rows: [2][S][128/S][W]
           + static_cast<size_t>(2) * kRowsPerTile * 8 * 4  // hPre of the tile's rows: [2][128][8]
           + static_cast<size_t>(16) * W * 4                // owner's sums: [128/S <= 16][W]
           + 64 * 8 + 64;                                   // mbarriers, TMEM slot, flags
}

template <int DT, int NS>
__global__ void __launch_bounds__(kClusterThreads, 1)
    mhc_pre_cluster_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiMap,
                           const ClusterParams p) {
    constexpr int MIX = NS * NS + 2 * NS;
    constexpr int N = 2 * MIX;
    using Cfg = FusedCfg<N>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int GS = p.gStages, HS = p.hStages;
    const int S = p.S;
    const int ownRows = kRowsPerTile / S;  // 8 or 16: rows this member owns in every tile
    uint8_t* gRing = smem;
    uint8_t* hRing = gRing + static_cast<size_t>(GS) * Cfg::kGStageBytes;
    float* recBuf = reinterpret_cast<float*>(hRing + static_cast<size_t>(HS) * kHinStageBytes);  // [2][S][ownRows][W]
    float* hpreBuf = recBuf + 2 * kRowsPerTile * p.W;                                             // [2][128][8]
    float* sTot = hpreBuf + 2 * kRowsPerTile * 8;                                                 // [ownRows][W]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sTot + 16 * p.W);
    uint64_t* gFull = bars;
    uint64_t* gEmpty = gFull + GS;
    uint64_t* hFull = gEmpty + GS;
    uint64_t* hEmpty = hFull + HS;
    uint64_t* accFull = hEmpty + HS;       // [2]
    uint64_t* accEmpty = accFull + 2;      // [2]
    uint64_t* hpreTaken = accEmpty + 2;    // [2]: this CTA's hIn warps have read hPre of the slot
    uint64_t* recFull = hpreTaken + 2;     // [2]: S members' records of the owned rows arrived
    uint64_t* hpreFull = recFull + 2;      // [2]: S owners' hPre arrived
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(hpreFull + 2);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);  // [0]: abort, [1]: hIn agreement
    unsigned* hinDone = reinterpret_cast<unsigned*>(tmemSlot + 3);             // 4 x chunks the hIn warps consumed

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int team = blockIdx.x / S;
    const int member = static_cast<int>(cluster_ctarank());
    const int nLocal = team < p.tilesM ? (p.tilesM - 1 - team) / p.T + 1 : 0;
    const int nq = p.J * NS;  // chunks per tile
    const int segPerTile = (nq + kSegChunks - 1) / kSegChunks;
    const unsigned* gabort = p.gAbort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GS; ++s) {
            mbar_init(&gFull[s], 1);
            mbar_init(&gEmpty[s], 1 + 4);
        }
        for (int s = 0; s < HS; ++s) {
            mbar_init(&hFull[s], 1);
            mbar_init(&hEmpty[s], 4);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accFull[b], 1);
            mbar_init(&accEmpty[b], 4);
            mbar_init(&hpreTaken[b], 4);
            mbar_init(&recFull[b], S);   // one arrival per member (the warp holding the rows)
            mbar_init(&hpreFull[b], S);  // one arrival per owner
        }
        *abortFlag = 0;
        *hinDone = 0;
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
    cluster_barrier();  // every CTA's mbarriers are initialised before any remote arrival
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);

    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
        atomicExch(p.gAbort, 1u);
    };
    // K coordinate of local chunk q (stream-inner order: q = j*NS + s)
    auto chunk_k = [&](int q) -> int {
        const int j = q / NS, s = q - (q / NS) * NS;
        return static_cast<int>(s * p.D + (static_cast<int64_t>(member) * p.J + j) * kChunk);
    };

    if (prepared && nLocal > 0) {
        if (warp == 0) {
            // ---------------- GEMM producer ----------------
            if (lane == 0) {
                const uint64_t polX = p.l2mode == 1 ? l2_policy_evict_last() : l2_policy_evict_normal();
                int g = 0;
                for (int i = 0; i < nLocal && !*abortFlag; ++i) {
                    const int tile = team + i * p.T;
                    for (int q = 0; q < nq; ++q, ++g) {
                        const int s = g % GS;
                        if (g >= GS && !mbar_wait(&gEmpty[s], (static_cast<uint32_t>(g / GS) & 1u) ^ 1u, abortFlag)) {
                            fail();
                            break;
                        }
                        // stay at most one tile + lead chunks ahead of the re-read
                        const int need = g - nq - p.lead + 1;
                        if (need > 0) {
                            const unsigned target = 4u * static_cast<unsigned>(need);
                            bool ok = *reinterpret_cast<volatile unsigned*>(hinDone) >= target;
                            if (!ok) {
                                const uint64_t t0 = global_timer_ns();
                                for (uint32_t it = 0; it < kMaxPolls && !*abortFlag; ++it) {
                                    if (*reinterpret_cast<volatile unsigned*>(hinDone) >= target) {
                                        ok = true;
                                        break;
                                    }
                                    if ((it & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) break;
                                    __nanosleep(32);
                                }
                            }
                            if (!ok) {
                                fail();
                                break;
                            }
                        }
                        mbar_arrive_expect_tx(&gFull[s], Cfg::kGStageBytes);
                        uint8_t* st = gRing + static_cast<size_t>(s) * Cfg::kGStageBytes;
                        const int kc = chunk_k(q);
                        tma_load_2d_hint(st, &xMap, &gFull[s], kc, tile * kRowsPerTile, polX);
                        tma_load_2d_hint(st + Cfg::kXBytes, &phiMap, &gFull[s], kc, 0, polX);
                    }
                }
                if (*abortFlag) {
                    for (int k = (g > GS ? g - GS : 0); k < g; ++k)
                        mbar_wait(&gFull[k % GS], static_cast<uint32_t>(k / GS) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp == 1) {
            // ---------------- MMA issuer ----------------
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_f16(DT, kRowsPerTile, N);
                int g = 0;
                bool ok = true;
                for (int i = 0; i < nLocal && ok; ++i) {
                    for (int q = 0; q < nq; ++q, ++g) {
                        const int s = g % GS;
                        const int seg = i * segPerTile + q / kSegChunks;
                        const int b = seg & 1;
                        if (q % kSegChunks == 0 && seg >= 2 &&
                            !mbar_wait(&accEmpty[b], static_cast<uint32_t>((seg >> 1) - 1) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        if (!mbar_wait(&gFull[s], static_cast<uint32_t>(g / GS) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(gRing + static_cast<size_t>(s) * Cfg::kGStageBytes);
                        const uint32_t b0 = a0 + Cfg::kXBytes;
                        const uint32_t d = tacc + static_cast<uint32_t>(b * N);
#pragma unroll
                        for (int k16 = 0; k16 < kChunk / 16; ++k16) {
                            mma_f16_ss(d, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                       (q % kSegChunks != 0 || k16 > 0) ? 1u : 0u);
                        }
                        mma_commit(&gEmpty[s]);
                        if (q % kSegChunks == kSegChunks - 1 || q == nq - 1) mma_commit(&accFull[b]);
                    }
                }
            }
        } else if (warp == 2) {
            // ---------------- hIn producer (re-reads the tile's x from L2) ----------------
            if (lane == 0) {
                const uint64_t polX = p.l2mode == 0 ? l2_policy_evict_normal() : l2_policy_evict_first();
                int h = 0;
                for (int i = 0; i < nLocal && !*abortFlag; ++i) {
                    const int tile = team + i * p.T;
                    for (int q = 0; q < nq; ++q, ++h) {
                        const int s = h % HS;
                        if (h >= HS && !mbar_wait(&hEmpty[s], (static_cast<uint32_t>(h / HS) & 1u) ^ 1u, abortFlag)) {
                            fail();
                            break;
                        }
                        mbar_arrive_expect_tx(&hFull[s], kHinStageBytes);
                        tma_load_2d_hint(hRing + static_cast<size_t>(s) * kHinStageBytes, &xMap, &hFull[s],
                                         chunk_k(q), tile * kRowsPerTile, polX);
                    }
                }
                if (*abortFlag) {
                    for (int k = (h > HS ? h - HS : 0); k < h; ++k)
                        mbar_wait(&hFull[k % HS], static_cast<uint32_t>(k / HS) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp >= 4 && warp < 8) {
            // ---------------- square-sum + accumulator flushes + records to the owners ----------------
            const int qd = warp & 3;
            const int row = qd * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(qd * 32) << 16);
            const int owner = row / ownRows;
            const int ownerRow = row - owner * ownRows;
            const int ownersPerWarp = 32 / ownRows;
            float run[MIX];
            auto flush = [&](int seg) -> bool {
                const int b = seg & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&accFull[b], static_cast<uint32_t>(seg >> 1) & 1u, abortFlag)))
                    return false;
                tc_fence_after();
                add_segment<MIX>(lane_base, static_cast<uint32_t>(b * N), run);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&accEmpty[b]);
                return true;
            };
            const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
            int g = 0;
            for (int i = 0; i < nLocal; ++i) {
                const int slot = i & 1;
                bool ok = true;
#pragma unroll
                for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
                float ss = 0.0f;
                for (int q = 0; q < nq; ++q, ++g) {
                    const int s = g % GS;
                    if (!__all_sync(0xffffffffu, mbar_wait(&gFull[s], static_cast<uint32_t>(g / GS) & 1u, abortFlag))) {
                        ok = false;
                        break;
                    }
                    const uint32_t base = smem_u32(gRing + static_cast<size_t>(s) * Cfg::kGStageBytes) + row * 128;
                    float part = 0.0f;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const uint4 v = lds128(base + ((jj ^ (row & 7)) << 4));
                        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float2 f = x2_to_f32<DT>(w[t]);
                            part = fmaf(f.x, f.x, part);
                            part = fmaf(f.y, f.y, part);
                        }
                    }
                    ss += part;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&gEmpty[s]);
                    const int segL = q / kSegChunks;
                    if ((q % kSegChunks == kSegChunks - 1 || q == nq - 1) && segL >= 1) {
                        if (!flush(i * segPerTile + segL - 1)) {
                            ok = false;
                            break;
                        }
                    }
                }
                if (ok) ok = flush(i * segPerTile + segPerTile - 1);
                // The owners' record slot of tile i was last used by tile i-2: every
                // owner has read it once this CTA's hIn warps have taken hPre of i-2.
                if (ok && i >= 2)
                    ok = __all_sync(0xffffffffu, mbar_wait(&hpreTaken[slot],
                                                           static_cast<uint32_t>(i / 2 - 1) & 1u, abortFlag));
                if (!ok) {
                    if (lane == 0) fail();
                    break;
                }
                // this row's record -> recBuf[slot][member][ownerRow] of the owner
                const uint32_t local = smem_u32(recBuf) +
                                       static_cast<uint32_t>(((slot * S + member) * ownRows + ownerRow) * p.W) * 4u;
                const uint32_t dst = cluster_map(local, static_cast<uint32_t>(owner));
#pragma unroll
                for (int j0 = 0; j0 < MIX; j0 += 4) {
                    float4 a;
                    a.x = __fmul_rn(run[j0 + 0], unscale);
                    a.y = __fmul_rn(run[j0 + 1], unscale);
                    a.z = __fmul_rn(run[j0 + 2], unscale);
                    a.w = __fmul_rn(run[j0 + 3], unscale);
                    st_cluster_v4(dst + j0 * 4, a);
                }
                st_cluster_v4(dst + MIX * 4, make_float4(ss, 0.f, 0.f, 0.f));  // W >= MIX + 4 rounded
                fence_acq_rel_cluster();
                __syncwarp();
                // one arrival per owner whose rows this warp holds
                if (lane < ownersPerWarp) {
                    const int o = (qd * 32) / ownRows + lane;
                    mbar_remote_arrive(cluster_map(smem_u32(&recFull[slot]), static_cast<uint32_t>(o)));
                }
            }
        } else if (warp == 3) {
            // ---------------- owner: the team reduction of this member's rows ----------------
            const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
            const int w4 = p.W / 4;
            for (int i = 0; i < nLocal; ++i) {
                const int tile = team + i * p.T;
                const int slot = i & 1;
                if (!__all_sync(0xffffffffu, mbar_wait_cluster(&recFull[slot], static_cast<uint32_t>(i / 2) & 1u,
                                                               gabort))) {
                    if (lane == 0) fail();
                    break;
                }
                // sum over members in member order; each lane takes 4 columns of a row
                const float* recs = recBuf + static_cast<size_t>(slot) * S * ownRows * p.W;
                for (int idx = lane; idx < ownRows * w4; idx += 32) {
                    const int r = idx / w4;
                    const int j = (idx - r * w4) * 4;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int m = 0; m < S; ++m) {
                        const float4 v = *reinterpret_cast<const float4*>(recs + (m * ownRows + r) * p.W + j);
                        acc.x = __fadd_rn(acc.x, v.x);
                        acc.y = __fadd_rn(acc.y, v.y);
                        acc.z = __fadd_rn(acc.z, v.z);
                        acc.w = __fadd_rn(acc.w, v.w);
                    }
                    *reinterpret_cast<float4*>(sTot + r * p.W + j) = acc;
                }
                __syncwarp();
                // epilogue of the owned rows: hPost/hRes out; hPre staged in sTot's row
                float pre[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if (lane < ownRows) {
                    const int r = member * ownRows + lane;
                    const int64_t grow = static_cast<int64_t>(tile) * kRowsPerTile + r;
                    const float* tot = sTot + lane * p.W;
                    float v = __fmul_rn(tot[MIX], p.invK);
                    v = __fadd_rn(v, p.normEps);
                    const float invRms = __fdiv_rn(1.0f, __fsqrt_rn(v));
                    const float sPre = __fmul_rn(invRms, a0), sPost = __fmul_rn(invRms, a1),
                                sRes = __fmul_rn(invRms, a2);
#pragma unroll
                    for (int s2 = 0; s2 < NS; ++s2) {
                        const float t1 = __fadd_rn(__fmul_rn(tot[s2], sPre), __ldg(p.bias + s2));
                        pre[s2] = __fadd_rn(sigmoid_ref(t1), p.hcEps);
                        if (grow < p.M) {
                            const float u = __fadd_rn(__fmul_rn(tot[NS + s2], sPost), __ldg(p.bias + NS + s2));
                            p.hPost[grow * NS + s2] = __fmul_rn(sigmoid_ref(u), 2.0f);
                        }
                    }
                    if (grow < p.M) {
#pragma unroll 4
                        for (int k = 0; k < NS * NS; ++k)
                            p.hRes[grow * NS * NS + k] =
                                __fadd_rn(__fmul_rn(tot[2 * NS + k], sRes), __ldg(p.bias + 2 * NS + k));
                    }
                }
                __syncwarp();
                // hPre of the owned rows -> hpreBuf[slot][member*ownRows + r] of every member:
                // lane m writes member m's copy, then arrives on member m's barrier
                float* stage = sTot;  // [ownRows][8], reusing the sums (already consumed)
                if (lane < ownRows) {
                    *reinterpret_cast<float4*>(stage + lane * 8) = make_float4(pre[0], pre[1], pre[2], pre[3]);
                    *reinterpret_cast<float4*>(stage + lane * 8 + 4) = make_float4(pre[4], pre[5], pre[6], pre[7]);
                }
                __syncwarp();
                if (lane < S) {
                    const uint32_t local =
                        smem_u32(hpreBuf) + static_cast<uint32_t>((slot * kRowsPerTile + member * ownRows) * 8) * 4u;
                    const uint32_t dst = cluster_map(local, static_cast<uint32_t>(lane));
                    for (int r = 0; r < ownRows; ++r) {
                        st_cluster_v4(dst + r * 32, *reinterpret_cast<const float4*>(stage + r * 8));
                        st_cluster_v4(dst + r * 32 + 16, *reinterpret_cast<const float4*>(stage + r * 8 + 4));
                    }
                    mbar_remote_arrive(cluster_map(smem_u32(&hpreFull[slot]), static_cast<uint32_t>(lane)));
                }
                __syncwarp();
            }
        } else if (warp >= 8) {
            // ---------------- hIn: x re-read from L2 + hPre of the whole tile ----------------
            const int bt = threadIdx.x - 256;  // 0..127: the tile row
            volatile int* bflag = abortFlag + 1;
            float pre[NS];
            int h = 0;
            for (int i = 0; i < nLocal; ++i) {
                const int tile = team + i * p.T;
                const int slot = i & 1;
                if (bt == 0) *bflag = mbar_wait_cluster(&hpreFull[slot], static_cast<uint32_t>(i / 2) & 1u, gabort) ? 0 : 1;
                if (bar_red_or(2, 128, bt == 0 && *bflag != 0)) {
                    if (bt == 0) fail();
                    break;
                }
                {
                    const float* hp = hpreBuf + (slot * kRowsPerTile + bt) * 8;
                    const float4 h0 = *reinterpret_cast<const float4*>(hp);
                    pre[0] = h0.x; pre[1] = h0.y; pre[2] = h0.z; pre[3] = h0.w;
                    if constexpr (NS > 4) {
                        const float4 h1 = *reinterpret_cast<const float4*>(hp + 4);
                        pre[4] = h1.x; pre[5] = h1.y;
                        if constexpr (NS > 6) { pre[6] = h1.z; pre[7] = h1.w; }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&hpreTaken[slot]);
                const int64_t grow = static_cast<int64_t>(tile) * kRowsPerTile + bt;
                uint16_t* hrow = p.hIn + grow * p.D + static_cast<int64_t>(member) * p.J * kChunk;
                float acc[kChunk];
                bool ok = true;
                for (int q = 0; q < nq; ++q, ++h) {
                    const int s = h % HS;
                    const int str = q % NS;
                    if (!__all_sync(0xffffffffu, mbar_wait(&hFull[s], static_cast<uint32_t>(h / HS) & 1u, abortFlag))) {
                        ok = false;
                        h += nq - q;
                        break;
                    }
                    const uint32_t base = smem_u32(hRing + static_cast<size_t>(s) * kHinStageBytes) + bt * 128;
                    const float ps = pre[str];
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const uint4 v = lds128(base + ((jj ^ (bt & 7)) << 4));
                        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float2 f = x2_to_f32<DT>(w[t]);
                            const int e = jj * 8 + 2 * t;
                            if (str == 0) {
                                acc[e] = __fmul_rn(f.x, ps);
                                acc[e + 1] = __fmul_rn(f.y, ps);
                            } else {
                                acc[e] = __fadd_rn(acc[e], __fmul_rn(f.x, ps));
                                acc[e + 1] = __fadd_rn(acc[e + 1], __fmul_rn(f.y, ps));
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&hEmpty[s]);
                        atomicAdd(hinDone, 1u);
                    }
                    if (str == NS - 1 && grow < p.M) {
                        uint4* dst = reinterpret_cast<uint4*>(hrow + (q / NS) * kChunk);
#pragma unroll
                        for (int v8 = 0; v8 < 8; ++v8) {
                            uint4 o;
                            o.x = f32x2_to_x2<DT>(acc[v8 * 8 + 0], acc[v8 * 8 + 1]);
                            o.y = f32x2_to_x2<DT>(acc[v8 * 8 + 2], acc[v8 * 8 + 3]);
                            o.z = f32x2_to_x2<DT>(acc[v8 * 8 + 4], acc[v8 * 8 + 5]);
                            o.w = f32x2_to_x2<DT>(acc[v8 * 8 + 6], acc[v8 * 8 + 7]);
                            __stcs(dst + v8, o);
                        }
                    }
                }
                if (bar_red_or(2, 128, !ok)) {
                    if (bt == 0) fail();
                    break;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tacc, Cfg::kTmemCols);
    }
    cluster_barrier();  // no CTA leaves while a peer may still write its shared memory
}
