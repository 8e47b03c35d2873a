// Path 1: the fused single-kernel MhcPre (included by mhc_pre_kernels.cu).
//
// Persistent CTAs form teams of S members (one CTA per SM, co-resident through a
// cooperative launch).  Team t processes the 128-row tiles t, t+T, t+2T, ...; member
// c owns the D-slice [c*J*64, (c+1)*J*64) of every stream, i.e. J*n chunks of 64 K
// elements per tile.  Per tile, each member:
//   1. streams its chunks of x and of the prepared weights through a TMA ring; one
//      thread issues tcgen05.mma (M=128 rows, N=2*mix) into TMEM, accumulating in
//      segments that warps 4-7 add into fp32 registers, which also square-sum x;
//   2. publishes its partial records (mix sums + sum of squares per row) in a global
//      buffer and bumps the team's counter (release);
//   3. as the owner of R/S rows (warp 3), fetches those rows' records of all S
//      members with one bulk copy per row (records are stored row-major, members
//      inner), sums them in member order (so the result does not depend on timing),
//      computes invRms, hPre, hPost, hRes, writes hPost/hRes and publishes hPre
//      (release);
//   4. re-reads its chunks of the tile through a second TMA ring (an L2 hit: the
//      first read was moments ago) and forms hIn for its slice from hPre.
// Step 4 of tile i (warps 8-11) overlaps steps 1-2 of tile i+1 (warps 0-1, 4-7) and
// step 3 of tile i+1 (warp 3).  The re-read can hit L2 only while the data that all
// teams stream between a tile's first read and its re-read fits in L2; the host
// picks a team size for which one round of tiles stays under 40 MB.  Measured on
// B200, the handshake of steps 2-3 takes tens of microseconds while every SM
// streams, so most re-reads still miss and this path is opt-in.
// Every wait is bounded; a timeout sets the device status word and a team-wide
// abort word, and all roles wind down.
// It is included inside namespace mhc after the path-0 kernels, whose helpers
// (16-bit conversions, sigmoid_ref, set_device_status, kSegChunks) it uses.
#pragma once

struct FusedParams {
    int64_t M;
    int64_t D;
    int J;          // 64-wide chunks per stream per member (D-slice = J*64)
    int S;          // team size
    int T;          // teams
    int tilesM;     // ceil(M / 128)
    int W;          // floats per partial record
    int gStages;    // GEMM ring depth
    int hStages;    // hIn ring depth
    int l2mode;     // L2 hints: 0 none; 1 first read evict_last, re-read evict_first; 2 re-read evict_first only
    float invK;
    float normEps;
    float hcEps;
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    float* part;     // [T][kSlots][128][S][W]
    float* hpre;     // [T][2][128][8]
    unsigned* cnt;   // [T][2*kSlots]: record arrivals per slot, then hPre arrivals per slot; [2*kSlots*T]: abort word
    const WorkspaceHeader* hdr;
    uint32_t signature;  // of the description (checked against the prepared weights)
};

constexpr int kFusedThreads = 384;  // 12 warps
// Record/hPre slots per team: the GEMM warps may run up to kSlots tiles ahead of
// the team reduction, which hides its cross-CTA latency.
constexpr int kSlots = kFusedSlots;
constexpr int kHinStageBytes = kRowsPerTile * kChunk * 2;  // 16 KB

template <int N>
struct FusedCfg {
    static constexpr int kXBytes = kRowsPerTile * kChunk * 2;
    static constexpr int kPhiBytes = N * kChunk * 2;
    static constexpr int kGStageBytes = kXBytes + kPhiBytes;
    static constexpr uint32_t kTmemCols = 2 * N <= 64 ? 64 : 2 * N <= 128 ? 128 : 2 * N <= 256 ? 256 : 512;
};

template <int DT, int NS>
__global__ void __launch_bounds__(kFusedThreads, 1)
    mhc_pre_fused_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiMap,
                         const FusedParams p) {
    constexpr int MIX = NS * NS + 2 * NS;
    constexpr int N = 2 * MIX;
    using Cfg = FusedCfg<N>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int GS = p.gStages, HS = p.hStages;
    uint8_t* gRing = smem;
    uint8_t* hRing = gRing + static_cast<size_t>(GS) * Cfg::kGStageBytes;
    float* sTot = reinterpret_cast<float*>(hRing + static_cast<size_t>(HS) * kHinStageBytes);  // [16][W]
    const int ownRows = (kRowsPerTile + p.S - 1) / p.S;
    float* ownBuf = sTot + 16 * p.W;  // [ownRows][S][W]: the owned rows' records of all members
    uint64_t* bars = reinterpret_cast<uint64_t*>(ownBuf + static_cast<size_t>(ownRows) * p.S * p.W);
    uint64_t* gFull = bars;
    uint64_t* gEmpty = gFull + GS;
    uint64_t* hFull = gEmpty + GS;
    uint64_t* hEmpty = hFull + HS;
    uint64_t* accFull = hEmpty + HS;   // [2]
    uint64_t* accEmpty = accFull + 2;  // [2]
    uint64_t* hpreTaken = accEmpty + 2;  // [kSlots]
    uint64_t* ownBar = hpreTaken + kSlots;
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(ownBar + 1);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int team = blockIdx.x / p.S;
    const int member = blockIdx.x % p.S;
    const int nLocal = team < p.tilesM ? (p.tilesM - 1 - team) / p.T + 1 : 0;
    const int nq = p.J * NS;  // chunks per tile
    const int segPerTile = (nq + kSegChunks - 1) / kSegChunks;
    const int ownBase = member * ownRows;
    const int ownCount = max(0, min(ownRows, kRowsPerTile - ownBase));
    unsigned* cntT = p.cnt + 2 * kSlots * team;
    const unsigned* gabort = p.cnt + 2 * kSlots * p.T;

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
        }
        for (int b = 0; b < kSlots; ++b) mbar_init(&hpreTaken[b], 4);
        mbar_init(ownBar, 1);
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
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);

    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
        atomicExch(const_cast<unsigned*>(gabort), 1u);
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
            // ---------------- square-sum + accumulator flushes + partial records ----------------
            const int qd = warp & 3;
            const int row = qd * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(qd * 32) << 16);
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
                // The record slot of tile i was last used by tile i-kSlots: wait until
                // this CTA has taken that tile's hPre (then every owner has consumed it).
                if (ok && i >= kSlots)
                    ok = __all_sync(0xffffffffu, mbar_wait(&hpreTaken[i % kSlots],
                                                           static_cast<uint32_t>(i / kSlots - 1) & 1u, abortFlag));
                if (ok) {
                    float* rec = p.part + ((((static_cast<int64_t>(team) * kSlots + (i % kSlots)) * kRowsPerTile + row) *
                                                p.S + member) * p.W);
#pragma unroll
                    for (int j0 = 0; j0 < MIX; j0 += 4) {
                        float4 a;
                        a.x = __fmul_rn(run[j0 + 0], unscale);
                        a.y = __fmul_rn(run[j0 + 1], unscale);
                        a.z = __fmul_rn(run[j0 + 2], unscale);
                        a.w = __fmul_rn(run[j0 + 3], unscale);
                        *reinterpret_cast<float4*>(rec + j0) = a;
                    }
                    rec[MIX] = ss;
                    fence_proxy_async();  // the owners read the records with bulk copies
                    __threadfence();
                }
                // all four warps agree before the release (no warp may be left waiting)
                if (bar_red_or(1, 128, !ok)) {
                    if (threadIdx.x == 128) fail();
                    break;
                }
                if (threadIdx.x == 128) red_release_add(&cntT[i % kSlots], 1u);
            }
        } else if (warp == 3) {
            // ---------------- owner: team reduction of the rows this member owns ----------------
            // Runs ahead of the hIn warps, so the cross-CTA handshakes overlap the
            // hIn streaming of the previous tile.
            const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
            const int w4 = p.W / 4;
            for (int i = 0; i < nLocal; ++i) {
                const int tile = team + i * p.T;
                const int slot = i % kSlots;
                const unsigned target = static_cast<unsigned>(p.S) * static_cast<unsigned>(i / kSlots + 1);
                // (a) every member's records of tile i
                const bool got = __all_sync(0xffffffffu, lane == 0 ? wait_counter(&cntT[slot], target, gabort) : true);
                if (!got) {
                    if (lane == 0) fail();
                    break;
                }
                // (b) the owned rows' records of every member, one bulk copy per row, then
                // the sum over members in member order; each lane takes 4 columns of a row
                if (ownCount > 0) {
                    const int64_t rowFloats = static_cast<int64_t>(p.S) * p.W;
                    const float* recs =
                        p.part + ((static_cast<int64_t>(team) * kSlots + slot) * kRowsPerTile + ownBase) * rowFloats;
                    fence_proxy_async();  // acquired records, and last tile's reads of ownBuf, before the copies
                    if (lane == 0) mbar_arrive_expect_tx(ownBar, static_cast<uint32_t>(rowFloats * 4 * ownCount));
                    __syncwarp();
                    if (lane < ownCount)
                        bulk_load(ownBuf + lane * rowFloats, recs + lane * rowFloats, static_cast<uint32_t>(rowFloats * 4),
                                  ownBar);
                    if (!__all_sync(0xffffffffu, mbar_wait(ownBar, static_cast<uint32_t>(i) & 1u, abortFlag))) {
                        if (lane == 0) {
                            fail();
                            // let the copies in flight land before the CTA can exit (bounded)
                            mbar_wait(ownBar, static_cast<uint32_t>(i) & 1u, nullptr, 100000000ull);
                        }
                        __syncwarp();
                        break;
                    }
                    for (int idx = lane; idx < ownCount * w4; idx += 32) {
                        const int r = idx / w4;
                        const int j = (idx - r * w4) * 4;
                        const float* src = ownBuf + r * rowFloats + j;
                        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int m = 0; m < p.S; ++m) {
                            const float4 v = *reinterpret_cast<const float4*>(src + m * p.W);
                            acc.x = __fadd_rn(acc.x, v.x);
                            acc.y = __fadd_rn(acc.y, v.y);
                            acc.z = __fadd_rn(acc.z, v.z);
                            acc.w = __fadd_rn(acc.w, v.w);
                        }
                        *reinterpret_cast<float4*>(sTot + r * p.W + j) = acc;
                    }
                }
                __syncwarp();
                // (c) epilogue of the owned rows: hPost/hRes out, hPre published
                if (lane < ownCount) {
                    const int r = ownBase + lane;
                    const int64_t grow = static_cast<int64_t>(tile) * kRowsPerTile + r;
                    const float* tot = sTot + lane * p.W;
                    float v = __fmul_rn(tot[MIX], p.invK);
                    v = __fadd_rn(v, p.normEps);
                    const float invRms = __fdiv_rn(1.0f, __fsqrt_rn(v));
                    const float sPre = __fmul_rn(invRms, a0), sPost = __fmul_rn(invRms, a1), sRes = __fmul_rn(invRms, a2);
                    float* hp = p.hpre + ((static_cast<int64_t>(team) * kSlots + slot) * kRowsPerTile + r) * 8;
#pragma unroll
                    for (int s2 = 0; s2 < NS; ++s2) {
                        const float t1 = __fadd_rn(__fmul_rn(tot[s2], sPre), __ldg(p.bias + s2));
                        hp[s2] = __fadd_rn(sigmoid_ref(t1), p.hcEps);
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
                    __threadfence();
                }
                __syncwarp();
                if (lane == 0) red_release_add(&cntT[kSlots + slot], 1u);
            }
        } else if (warp >= 8) {
            // ---------------- hIn: x re-read from L2 + hPre of the whole tile ----------------
            const int bt = threadIdx.x - 256;  // 0..127: the tile row
            volatile int* bflag = abortFlag + 1;
            float pre[NS];
            int h = 0;
            for (int i = 0; i < nLocal; ++i) {
                const int tile = team + i * p.T;
                const int slot = i % kSlots;
                const unsigned target = static_cast<unsigned>(p.S) * static_cast<unsigned>(i / kSlots + 1);
                // hPre of all rows of tile i (published by all owners)
                if (bt == 0) *bflag = wait_counter(&cntT[kSlots + slot], target, gabort) ? 0 : 1;
                if (bar_red_or(2, 128, bt == 0 && *bflag != 0)) {
                    if (bt == 0) fail();
                    break;
                }
                {
                    const float* hpr = p.hpre + ((static_cast<int64_t>(team) * kSlots + slot) * kRowsPerTile + bt) * 8;
                    const float4 h0 = __ldcg(reinterpret_cast<const float4*>(hpr));
                    pre[0] = h0.x; pre[1] = h0.y; pre[2] = h0.z; pre[3] = h0.w;
                    if constexpr (NS > 4) {
                        const float4 h1 = __ldcg(reinterpret_cast<const float4*>(hpr + 4));
                        pre[4] = h1.x; pre[5] = h1.y;
                        if constexpr (NS > 6) { pre[6] = h1.z; pre[7] = h1.w; }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&hpreTaken[slot]);
                // hIn for this member's D-slice of row bt, stream order 0..n-1
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
                    if (lane == 0) mbar_arrive(&hEmpty[s]);
                    if (str == NS - 1 && grow < p.M) {
                        uint4* dst = reinterpret_cast<uint4*>(hrow + (q / NS) * kChunk);
#pragma unroll
                        for (int v8 = 0; v8 < 8; ++v8) {
                            uint4 o;
                            o.x = f32x2_to_x2<DT>(acc[v8 * 8 + 0], acc[v8 * 8 + 1]);
                            o.y = f32x2_to_x2<DT>(acc[v8 * 8 + 2], acc[v8 * 8 + 3]);
                            o.z = f32x2_to_x2<DT>(acc[v8 * 8 + 4], acc[v8 * 8 + 5]);
                            o.w = f32x2_to_x2<DT>(acc[v8 * 8 + 6], acc[v8 * 8 + 7]);
                            __stcs(dst + v8, o);  // streaming store: hIn is not read again
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
}
