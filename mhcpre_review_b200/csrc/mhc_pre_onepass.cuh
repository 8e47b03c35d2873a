// Path 5: the one-pass kernel (included by mhc_pre_kernels.cu).
//
// x crosses HBM once.  Persistent CTAs (P per SM, all co-resident through a
// cooperative launch) each run two independent roles:
//   GEMM warps 0-5  the split-K contraction of path 0 -- a TMA ring of 64-wide K
//                   chunks of x and of the prepared weights, tcgen05.mma (M = 128 token
//                   rows, N = 2*mix) into TMEM, the square-sum read from the same
//                   stages -- over small work items (128-row tile, K split of a few
//                   chunks) in tile-major order, item w on CTA w mod G.  An item's
//                   partial records go into a ring of RT tile slots [slot][row][split][W]
//                   and add one arrival per warp to the slot's counter.
//   hIn warps 6..   one row per warp at a time (warp e of CTA b takes rows b + G*e,
//                   b + G*(e + EW), ...).  For each row: wait for its tile's arrivals;
//                   sum its records over the splits in split order (lane j, column j);
//                   mark the row's records consumed; compute invRms, hPre, hPost, hRes
//                   in the reference's operation order; then re-read the row's x and
//                   write hIn.  Rows are independent, so the warps of an SM overlap one
//                   row's records with another's x stream.
// Items are small (a few chunks), so every tile's items run at about the same time
// on many CTAs and a tile completes a few microseconds after its first chunk was
// read: its re-read then finds x in L2, and DRAM sees x once.  The TMA producer does
// not start an item of tile t before the hIn warps have consumed every record of
// tile t - RT (the previous occupant of the ring slot), which bounds both the record
// ring and the x footprint between first read and re-read.
//
// Results depend on K and the split count only (never on M, the grid or timing):
// each split's MMA segments are added in order, the splits in a fixed order.
// Every wait is bounded; a timeout sets the device status word and a global abort
// word that every role polls, and all roles wind down.
//
// Reference: the single-round protocol this replaces serialises preprocess, GEMM
// and postprocess and reads x twice (code/op_kernel/mhc_pre.cpp:266-286; the
// re-read is LoadHInBlock, :622-639).
#pragma once

struct OnePassParams {
    int64_t M;
    int64_t D;
    int64_t K;
    int tilesM;
    int chunks;
    int splits;      // K splits (items per tile)
    int stages;      // TMA ring depth
    int batch;       // chunks the producer issues per batch
    int W;           // floats per partial record
    int RT;          // record ring: tile slots
    float invK;
    float normEps;
    float hcEps;
    uint32_t signature;
    const uint16_t* x;
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    float* rec;      // [RT][128][splits][W]
    int64_t recFloats;  // floats of rec (bounds checks of the debug build)
    unsigned* cnt;   // [RT] record arrivals (4 per item), [RT] rows consumed, [1] abort word
    const WorkspaceHeader* hdr;
};

constexpr int kOpGemmWarps = 6;
template <int EW>
constexpr int onepass_threads() { return (kOpGemmWarps + EW) * 32; }

// Adds one finished TMEM accumulator segment into the fp32 running sums, G columns
// of hi and of lo per TMEM round trip (smaller G keeps fewer registers live).
template <int MIX, int G>
__device__ __forceinline__ void add_segment_g(uint32_t lane_base, uint32_t col, float (&run)[MIX]) {
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


template <int DT, int NS, int EW, int MINB>
__global__ void __launch_bounds__(onepass_threads<EW>(), MINB)
    mhc_pre_onepass_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap phiMap,
                           const OnePassParams p) {
    constexpr int MIX = NS * NS + 2 * NS;
    constexpr int N = 2 * MIX;
    static_assert(EW >= 1, "at least one hIn warp");
    static_assert(MIX + 1 <= 32, "one lane per record column");
    using Cfg = GemmCfg<N>;
    constexpr int kAccBufs = Cfg::kAccBufs;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * Cfg::kStageBytes);  // [S]
    uint64_t* empty = full + S;
    uint64_t* accFull = empty + S;            // [kAccBufs]
    uint64_t* accEmpty = accFull + kAccBufs;  // [kAccBufs]
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(accEmpty + kAccBufs);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int numItems = p.tilesM * p.splits;
    unsigned* cntRec = p.cnt;
    unsigned* cntDone = p.cnt + p.RT;
    unsigned* gAbort = p.cnt + 2 * p.RT;
    auto item_range = [&](int w, int& tile, int& split, int& cBegin, int& nChunks) {
        tile = w / p.splits;
        split = w - tile * p.splits;
        cBegin = static_cast<int>((static_cast<int64_t>(split) * p.chunks) / p.splits);
        nChunks = static_cast<int>((static_cast<int64_t>(split + 1) * p.chunks) / p.splits) - cBegin;
    };
    // rows of earlier occupants of tile t's ring slot, all of which must have been
    // consumed before tile t's records go there (earlier tiles are full: 128 rows)
    auto slot_free_target = [&](int t) { return static_cast<unsigned>(kRowsPerTile) * static_cast<unsigned>(t / p.RT); };

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
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelBegin, 5, 0);
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);

    auto stage_x = [&](int s) { return smem + static_cast<size_t>(s) * Cfg::kStageBytes; };
    auto stage_phi = [&](int s) { return smem + static_cast<size_t>(s) * Cfg::kStageBytes + Cfg::kXBytes; };
    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
        atomicExch(gAbort, 1u);
    };

    if (prepared) {
        if (warp == 0) {
            // ---------------- TMA producer ----------------
            if (lane == 0) {
                int g = 0;
                const int batch = p.batch;
                for (int w = blockIdx.x; w < numItems && !*abortFlag; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    MHC_TRACE_EV(kTrGemmItemBegin, tile, split);
                    // the ring slot's previous tile must be consumed (bounds the footprint)
                    if (tile >= p.RT && !wait_counter(&cntDone[tile % p.RT], slot_free_target(tile), gAbort)) {
                        fail();
                        break;
                    }
                    MHC_TRACE_EV(kTrGemmItemIssue, tile, split);
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
            // ---------------- MMA issuer ----------------
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
        } else if (warp < kOpGemmWarps) {
            // ---------------- square-sum, accumulator flush, records ----------------
            // one token row per thread; TMEM lane quadrant = warp % 4
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(q * 32) << 16);
            float run[MIX];
            auto flush = [&](int seg) -> bool {
                const int b = seg % kAccBufs;
                // warp-uniform outcome: the TMEM loads below are warp-collective
                if (!__all_sync(0xffffffffu,
                                mbar_wait(&accFull[b], static_cast<uint32_t>(seg / kAccBufs) & 1u, abortFlag)))
                    return false;
                tc_fence_after();
                add_segment_g<MIX, 8>(lane_base, static_cast<uint32_t>(b * N), run);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&accEmpty[b]);
                return true;
            };
            const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
            // Each finished accumulator segment is added into run[] one segment later
            // (when the next one ends, by then long complete), also across items; the
            // item's record is written when its last segment has been added.
            int g = 0, gseg = 0;
            bool ok = true, havePrev = false, prevLast = false;
            int prevSeg = 0, prevTile = 0, prevSplit = 0;
            float prevSs = 0.0f;
#pragma unroll
            for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
            auto retire_prev = [&]() -> bool {
                if (!flush(prevSeg)) return false;
                if (!prevLast) return true;
                const int slot = prevTile % p.RT;
                // the slot's previous tile was consumed before the producer started
                // this item; checked again where the records are written (bounded)
                if (prevTile >= p.RT) {
                    bool freed = true;
                    if (lane == 0) freed = wait_counter(&cntDone[slot], slot_free_target(prevTile), gAbort);
                    if (!__shfl_sync(0xffffffffu, freed ? 1 : 0, 0)) return false;
                }
                const int64_t grow = static_cast<int64_t>(prevTile) * kRowsPerTile + row;
                const int64_t recAt = ((static_cast<int64_t>(slot) * kRowsPerTile + row) * p.splits + prevSplit) * p.W;
                if (grow < p.M && MHC_CHECK(slot < p.RT && prevSplit < p.splits && recAt + MIX < p.recFloats)) {
                    float* out = p.rec + recAt;
#pragma unroll
                    for (int j0 = 0; j0 < MIX; j0 += 4) {
                        float4 a;
                        a.x = __fmul_rn(run[j0 + 0], unscale);
                        a.y = __fmul_rn(run[j0 + 1], unscale);
                        a.z = __fmul_rn(run[j0 + 2], unscale);
                        a.w = __fmul_rn(run[j0 + 3], unscale);
                        *reinterpret_cast<float4*>(out + j0) = a;
                    }
                    out[MIX] = prevSs;
                }
#pragma unroll
                for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
                // publish: the warp's stores, then one release (cumulative over them)
                __syncwarp();
                if (lane == 0) red_release_add(&cntRec[slot], 1u);
                if (warp == 2 && lane == 0) MHC_TRACE_EV(kTrGemmRecord, prevTile, prevSplit);
                return true;
            };
            for (int w = blockIdx.x; w < numItems && ok; w += G) {
                int tile, split, cBegin, nChunks;
                item_range(w, tile, split, cBegin, nChunks);
                float ss = 0.0f;
                for (int i = 0; i < nChunks; ++i, ++g) {
                    const int s = g % S;
                    const uint32_t parity = static_cast<uint32_t>(g / S) & 1u;
                    if (havePrev && prevLast &&
                        !__all_sync(0xffffffffu, mbar_try_wait(smem_u32(&full[s]), parity))) {
                        // A finished item's record is still pending (records are written
                        // one segment late).  The next stage is not loaded yet: write the
                        // record now, because the producer may be waiting for hIn warps
                        // that wait for this very record.
                        if (!retire_prev()) {
                            ok = false;
                            break;
                        }
                        havePrev = false;
                    }
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], parity, abortFlag))) {
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
                        if (havePrev && !retire_prev()) {
                            ok = false;
                            break;
                        }
                        havePrev = true;
                        prevSeg = gseg++;
                        prevLast = i == nChunks - 1;
                        prevTile = tile;
                        prevSplit = split;
                        prevSs = ss;
                    }
                }
            }
            if (ok && havePrev) ok = retire_prev();
            if (!ok && lane == 0) fail();
        } else {
            // ---------------- hIn warps: one row per warp ----------------
            const int ew = warp - kOpGemmWarps;
            const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
            const float biasL = lane < MIX ? __ldg(p.bias + lane) : 0.0f;
            const unsigned arrivalsPerTile = 4u * static_cast<unsigned>(p.splits);
            const int64_t vecPerStream = p.D / 8;
            const int64_t rowStep = static_cast<int64_t>(G) * EW;
            for (int64_t r = blockIdx.x + static_cast<int64_t>(ew) * G; r < p.M; r += rowStep) {
                const int tile = static_cast<int>(r / kRowsPerTile);
                const int lrow = static_cast<int>(r - static_cast<int64_t>(tile) * kRowsPerTile);
                const int slot = tile % p.RT;
                const uint32_t rlo = static_cast<uint32_t>(static_cast<uint64_t>(r) & 0xffffffffu);
                const uint32_t rhi = static_cast<uint32_t>(static_cast<uint64_t>(r) >> 32);
                (void)rlo;  // trace arguments (used in the MHC_TRACE build only)
                (void)rhi;
                bool ok = true;
                if (lane == 0) {
                    MHC_TRACE_EV(kTrRowWait, rlo, rhi);
                    ok = wait_counter(&cntRec[slot], arrivalsPerTile * static_cast<unsigned>(tile / p.RT + 1), gAbort);
                    MHC_TRACE_EV(kTrRowReady, rlo, rhi);
                }
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
                    if (lane == 0) fail();
                    break;
                }
                // lane j sums record column j over the splits, in split order
                float acc = 0.0f;
                const int64_t rowAt = (static_cast<int64_t>(slot) * kRowsPerTile + lrow) * p.splits * p.W;
                if (lane <= MIX && MHC_CHECK(rowAt + static_cast<int64_t>(p.splits) * p.W <= p.recFloats)) {
                    const float* col = p.rec + rowAt + lane;
                    constexpr int kB = 28;  // loads in flight per lane
                    int sp = 0;
                    for (; sp + kB <= p.splits; sp += kB) {
                        float v[kB];
#pragma unroll
                        for (int u = 0; u < kB; ++u) v[u] = __ldcg(col + (sp + u) * p.W);
#pragma unroll
                        for (int u = 0; u < kB; ++u) acc = __fadd_rn(acc, v[u]);
                    }
                    for (; sp < p.splits; ++sp) acc = __fadd_rn(acc, __ldcg(col + sp * p.W));
                }
                // every lane's loads have returned (their values are summed): the row's
                // records are consumed and the slot may be reused
                __syncwarp();
                if (lane == 0) {
                    red_release_add(&cntDone[slot], 1u);
                    MHC_TRACE_EV(kTrRowReduced, rlo, rhi);
                }
                const float ssum = __shfl_sync(0xffffffffu, acc, MIX);
                // invRms = 1 / Sqrt(sum * invFlatDim + normEps)   (mhc_pre.cpp:504-519)
                float tv = __fmul_rn(ssum, p.invK);
                tv = __fadd_rn(tv, p.normEps);
                const float invRms = __fdiv_rn(1.0f, __fsqrt_rn(tv));
                float hpre = 0.0f;
                if (lane < NS) {
                    const float u = __fadd_rn(__fmul_rn(acc, __fmul_rn(invRms, a0)), biasL);
                    hpre = __fadd_rn(sigmoid_ref(u), p.hcEps);
                } else if (lane < 2 * NS) {
                    const float u = __fadd_rn(__fmul_rn(acc, __fmul_rn(invRms, a1)), biasL);
                    p.hPost[r * NS + (lane - NS)] = __fmul_rn(sigmoid_ref(u), 2.0f);
                } else if (lane < MIX) {
                    p.hRes[r * NS * NS + (lane - 2 * NS)] = __fadd_rn(__fmul_rn(acc, __fmul_rn(invRms, a2)), biasL);
                }
                float pre[NS];
#pragma unroll
                for (int s = 0; s < NS; ++s) pre[s] = __shfl_sync(0xffffffffu, hpre, s);
                // hIn = sum_s hPre[s] * x[s, :], streams in order, separate multiply and
                // add (mhc_pre.cpp:91-222), rounded to the x dtype (:811-812)
                const uint4* xr = reinterpret_cast<const uint4*>(p.x + r * p.K);
                uint4* hr = reinterpret_cast<uint4*>(p.hIn + r * p.D);
                for (int64_t vi = lane; vi < vecPerStream; vi += 64) {
                    const bool two = vi + 32 < vecPerStream;
                    uint4 wa[NS], wb[NS];
#pragma unroll
                    for (int s = 0; s < NS; ++s) wa[s] = __ldcs(xr + s * vecPerStream + vi);
                    if (two) {
#pragma unroll
                        for (int s = 0; s < NS; ++s) wb[s] = __ldcs(xr + s * vecPerStream + vi + 32);
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (h == 1 && !two) break;
                        const uint4* wv = h == 0 ? wa : wb;
                        float o8[8];
#pragma unroll
                        for (int s = 0; s < NS; ++s) {
                            const uint32_t ws[4] = {wv[s].x, wv[s].y, wv[s].z, wv[s].w};
#pragma unroll
                            for (int t = 0; t < 4; ++t) {
                                const float2 f = x2_to_f32<DT>(ws[t]);
                                if (s == 0) {
                                    o8[2 * t] = __fmul_rn(f.x, pre[0]);
                                    o8[2 * t + 1] = __fmul_rn(f.y, pre[0]);
                                } else {
                                    o8[2 * t] = __fadd_rn(o8[2 * t], __fmul_rn(f.x, pre[s]));
                                    o8[2 * t + 1] = __fadd_rn(o8[2 * t + 1], __fmul_rn(f.y, pre[s]));
                                }
                            }
                        }
                        uint4 o;
                        o.x = f32x2_to_x2<DT>(o8[0], o8[1]);
                        o.y = f32x2_to_x2<DT>(o8[2], o8[3]);
                        o.z = f32x2_to_x2<DT>(o8[4], o8[5]);
                        o.w = f32x2_to_x2<DT>(o8[6], o8[7]);
                        __stcs(hr + vi + h * 32, o);
                    }
                }
                if (lane == 0) MHC_TRACE_EV(kTrRowDone, rlo, rhi);
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
    if (threadIdx.x == 0) MHC_TRACE_EV(kTrKernelEnd, 5, 0);
}
