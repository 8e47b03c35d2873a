// The mHC post step fused with the next layer's MhcPre contraction (included by
// mhc_pre_kernels.cu after the split-K GEMM, the post step and their helpers).
//
// A layer ends with the post step, xNext[m,s,:] = sum_t hRes[m,s,t]*x[m,t,:] +
// hPost[m,s]*y[m,:], and the next layer starts with MhcPre on xNext, whose first pass
// reads xNext again.  This kernel forms xNext and that first pass together, so the
// pass never reads xNext from memory:
//   producer warp   TMA: for one 64-wide d-chunk of a 128-row tile, the x tiles of
//                   all n streams, the y tile, and the n chunks of the next layer's
//                   prepared weights that meet those K positions (k = s*D + d).
//   post warps 4-19 each thread owns a quarter of a row's 16-byte pieces: it reads the n
//                   x pieces and the y piece, forms the n xNext pieces in the post
//                   step's operation order (mhc_post.cuh), writes them back over the
//                   x pieces (the stage then holds xNext in the TMA layout), and adds
//                   their squares into the row's sum of squares.
//   MMA warp        tcgen05.mma of the n xNext tiles against their weight chunks into
//                   a TMEM segment (one segment per d-chunk, as in the split-K GEMM).
//   store warp      TMA stores of the n xNext tiles to memory.
//   warps 4-7       add each finished segment into fp32 registers one segment late
//                   and write the item's partial records [split][row][W].
// The split-K epilogue kernel then reads the records and xNext and writes the next
// layer's hIn, hPost and hRes.  Work items are (128-row tile, split of the d-chunks);
// a split covers every stream of its d-chunks.  D must be a multiple of 64 (a d-chunk
// never crosses into the next stream) and n = 4 (a stage of n+1 tiles and n weight
// chunks, 104 KB, fits twice in shared memory).  xNext may be x itself: each CTA
// loads a region before it stores over it, and regions of different items are
// disjoint.  Every wait is bounded.
#pragma once

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t c0, int32_t c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the shared-memory reads of every committed bulk group are done.
__device__ __forceinline__ void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until every committed bulk group is complete (its writes performed).
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

struct PostPreParams {
    int64_t M;
    int64_t D;
    int tilesM;
    int dChunks;     // D / 64
    int splits;      // splits of the d-chunks (records per row)
    int stages;
    int W;
    uint32_t signature;
    const float* hPost;   // [M][n] of the layer that ends
    const float* hRes;    // [M][n][n]
    float* partials;      // [split][M][W]
    int64_t partFloats;   // floats of partials (bounds checks of the debug build)
    const WorkspaceHeader* hdr;
};

constexpr int kPostPreThreads = 640;  // 20 warps: producer, MMA, stores, spare, 16 post warps
constexpr int kPostPreWarps = 16;     // post warps: four per row quarter, each two of a row's eight 16-byte pieces

// Rounds two fp32 values to the 16-bit dtype (nearest even) in one conversion; the
// same bits as f32x2_to_x2.
template <int DT>
__device__ __forceinline__ uint32_t f32x2_to_x2_packed(float a, float b) {
    if constexpr (DT == MHC_DTYPE_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&h);
    } else {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
}
constexpr int kPostPreNS = 4;
constexpr int kPostPreN = 2 * (kPostPreNS * kPostPreNS + 2 * kPostPreNS);  // 48
constexpr int kPostPreTile = kRowsPerTile * kChunk * 2;                        // 16 KB
constexpr int kPostPrePhi = kPostPreN * kChunk * 2;                           // 6 KB
constexpr int kPostPreStage = (kPostPreNS + 1) * kPostPreTile + kPostPreNS * kPostPrePhi;  // 104 KB
static_assert(kPostPreStage == static_cast<int>(kPostPreStageBytesHost), "host and device agree on the stage");

template <int DT>
__global__ void __launch_bounds__(kPostPreThreads, 1)
    post_pre_kernel(const __grid_constant__ CUtensorMap xMap, const __grid_constant__ CUtensorMap yMap,
                    const __grid_constant__ CUtensorMap xNextMap, const __grid_constant__ CUtensorMap phiMap,
                    const PostPreParams p) {
    constexpr int NS = kPostPreNS;
    constexpr int N = kPostPreN;
    constexpr int MIX = N / 2;
    constexpr int kAccBufs = 2;  // TMEM: 2 x 48 columns
    constexpr uint32_t kTmemCols = 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * kPostPreStage);  // [S]
    uint64_t* empty = full + S;        // [S] MMA commit + store thread
    uint64_t* postDone = empty + S;    // [S] the post warps
    uint64_t* accFull = postDone + S;  // [2]
    uint64_t* accEmpty = accFull + 2;  // [2] the four flush warps
    uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(accEmpty + 2);
    volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);
    float* sSumsq = reinterpret_cast<float*>(smem + static_cast<size_t>(S) * kPostPreStage + 256);  // [3][128]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int numItems = p.tilesM * p.splits;
    auto item_range = [&](int w, int& tile, int& split, int& cBegin, int& nChunks) {
        tile = w / p.splits;
        split = w - tile * p.splits;
        cBegin = static_cast<int>((static_cast<int64_t>(split) * p.dChunks) / p.splits);
        nChunks = static_cast<int>((static_cast<int64_t>(split + 1) * p.dChunks) / p.splits) - cBegin;
    };
    auto tile_x = [&](int s, int t) { return smem + static_cast<size_t>(s) * kPostPreStage + t * kPostPreTile; };
    auto tile_y = [&](int s) { return smem + static_cast<size_t>(s) * kPostPreStage + NS * kPostPreTile; };
    auto chunk_phi = [&](int s, int t) {
        return smem + static_cast<size_t>(s) * kPostPreStage + (NS + 1) * kPostPreTile + t * kPostPrePhi;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);
            mbar_init(&postDone[s], kPostPreWarps);
        }
        for (int b = 0; b < kAccBufs; ++b) {
            mbar_init(&accFull[b], 1);
            mbar_init(&accEmpty[b], 4);
        }
        *abortFlag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmemSlot, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&xMap);
        tma_prefetch_desc(&yMap);
        tma_prefetch_desc(&xNextMap);
        tma_prefetch_desc(&phiMap);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dependency_wait();  // programmatic dependent: the kernel before this one is complete
    grid_launch_dependents();
    const uint32_t tacc = *tmemSlot;
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared && threadIdx.x == 0) set_device_status(MHC_STATUS_NOT_PREPARED);
    auto fail = [&]() {
        set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
        *abortFlag = 1;
    };

    if (prepared) {
        if (warp == 0) {
            // ---------------- TMA producer ----------------
            if (lane == 0) {
                int g = 0;
                for (int w = blockIdx.x; w < numItems && !*abortFlag; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    for (int i = 0; i < nChunks; ++i, ++g) {
                        const int s = g % S;
                        if (g >= S && !mbar_wait(&empty[s], (static_cast<uint32_t>(g / S) & 1u) ^ 1u, abortFlag)) {
                            fail();
                            break;
                        }
                        const int d0 = (cBegin + i) * kChunk;
                        MHC_TRACE_EV(kTrGemmItemIssue, g, tile);
                        mbar_arrive_expect_tx(&full[s], kPostPreStage);
                        for (int t = 0; t < NS; ++t) {
                            const int k0 = static_cast<int>(t * p.D) + d0;
                            tma_load_2d(tile_x(s, t), &xMap, &full[s], k0, tile * kRowsPerTile);
                            tma_load_2d(chunk_phi(s, t), &phiMap, &full[s], k0, 0);
                        }
                        tma_load_2d(tile_y(s), &yMap, &full[s], d0, tile * kRowsPerTile);
                    }
                }
                if (*abortFlag != 0) {
                    for (int k = (g > S ? g - S : 0); k < g; ++k)
                        mbar_wait(&full[k % S], static_cast<uint32_t>(k / S) & 1u, nullptr, 100000000ull);
                }
            }
        } else if (warp == 1) {
            // ---------------- MMA issuer: one TMEM segment per d-chunk ----------------
            if (lane == 0) {
                constexpr uint32_t idesc = idesc_f16(DT, kRowsPerTile, N);
                int g = 0;
                bool ok = true;
                for (int w = blockIdx.x; w < numItems && ok; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    for (int i = 0; i < nChunks; ++i, ++g) {
                        const int s = g % S;
                        const int b = g % kAccBufs;
                        if (g >= kAccBufs &&
                            !mbar_wait(&accEmpty[b], static_cast<uint32_t>(g / kAccBufs - 1) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        // the stage holds xNext once the post warps are done with it
                        if (!mbar_wait(&postDone[s], static_cast<uint32_t>(g / S) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tacc + static_cast<uint32_t>(b * N);
#pragma unroll
                        for (int t = 0; t < NS; ++t) {
                            const uint32_t a0 = smem_u32(tile_x(s, t));
                            const uint32_t b0 = smem_u32(chunk_phi(s, t));
#pragma unroll
                            for (int k16 = 0; k16 < kChunk / 16; ++k16)
                                mma_f16_ss(d, sdesc_sw128(a0 + k16 * 32), sdesc_sw128(b0 + k16 * 32), idesc,
                                           (t > 0 || k16 > 0) ? 1u : 0u);
                        }
                        mma_commit(&empty[s]);
                        mma_commit(&accFull[b]);
                    }
                }
            }
        } else if (warp == 2) {
            // ---------------- xNext stores ----------------
            if (lane == 0) {
                int g = 0;
                bool ok = true;
                for (int w = blockIdx.x; w < numItems && ok; w += G) {
                    int tile, split, cBegin, nChunks;
                    item_range(w, tile, split, cBegin, nChunks);
                    for (int i = 0; i < nChunks; ++i, ++g) {
                        const int s = g % S;
                        if (!mbar_wait(&postDone[s], static_cast<uint32_t>(g / S) & 1u, abortFlag)) {
                            fail();
                            ok = false;
                            break;
                        }
                        const int d0 = (cBegin + i) * kChunk;
                        for (int t = 0; t < NS; ++t)
                            tma_store_2d(&xNextMap, tile_x(s, t), static_cast<int>(t * p.D) + d0, tile * kRowsPerTile);
                        bulk_commit_group();
                        bulk_wait_group_read0();  // the stage may be refilled once the stores have read it
                        mbar_arrive(&empty[s]);
                        MHC_TRACE_EV(kTrRowDone, g, tile);
                    }
                }
                bulk_wait_group0();  // every xNext store is complete before the CTA ends
            }
        } else if (warp >= 4) {
            // ---------------- post step, square-sum, flush, records ----------------
            const int pw = warp - 4;         // 0..15
            const int q = pw & 3;            // row quarter = TMEM lane quadrant
            const int part = pw >> 2;        // pieces [2*part, 2*part + 2) of a row
            const int row = q * 32 + lane;
            const bool flusher = part == 0;  // warps 4-7 hold run[] and write records
            const uint32_t lane_base = tacc + (static_cast<uint32_t>(q * 32) << 16);
            const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
            float run[MIX];
            float res[NS * NS], post[NS];
            int g = 0;
            bool ok = true;
            auto flush = [&](int seg) -> bool {
                const int b = seg % kAccBufs;
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
            for (int w = blockIdx.x; w < numItems && ok; w += G) {
                int tile, split, cBegin, nChunks;
                item_range(w, tile, split, cBegin, nChunks);
                const int64_t grow = static_cast<int64_t>(tile) * kRowsPerTile + row;
                // this row's coefficients of the layer that ends (rows past M: zero)
#pragma unroll
                for (int k = 0; k < NS * NS; ++k) res[k] = grow < p.M ? __ldg(p.hRes + grow * NS * NS + k) : 0.0f;
#pragma unroll
                for (int k = 0; k < NS; ++k) post[k] = grow < p.M ? __ldg(p.hPost + grow * NS + k) : 0.0f;
#pragma unroll
                for (int j = 0; j < MIX; ++j) run[j] = 0.0f;
                float ss = 0.0f;
                bool itemOk = true;
                for (int i = 0; i < nChunks; ++i, ++g) {
                    const int s = g % S;
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>(g / S) & 1u, abortFlag))) {
                        itemOk = false;
                        break;
                    }
                    if (pw == 0 && lane == 0) MHC_TRACE_EV(kTrRowReady, g, tile);
                    const uint32_t yBase = smem_u32(tile_y(s)) + row * 128;
                    uint32_t xBase[NS];
#pragma unroll
                    for (int t = 0; t < NS; ++t) xBase[t] = smem_u32(tile_x(s, t)) + row * 128;
#pragma unroll
                    for (int jj = 0; jj < 2; ++jj) {
                        const int j = part * 2 + jj;                 // 16-byte piece of the 128-byte row
                        const uint32_t off = static_cast<uint32_t>((j ^ (row & 7)) << 4);  // 128-byte swizzle
                        uint4 xv[NS];
#pragma unroll
                        for (int t = 0; t < NS; ++t) xv[t] = lds128(xBase[t] + off);
                        const uint4 yv = lds128(yBase + off);
                        uint32_t ow[NS][4];
                        const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
                        for (int qq = 0; qq < 4; ++qq) {
                            float2 xf[NS];
#pragma unroll
                            for (int t = 0; t < NS; ++t) {
                                const uint32_t wv = qq == 0 ? xv[t].x : qq == 1 ? xv[t].y : qq == 2 ? xv[t].z : xv[t].w;
                                xf[t] = x2_to_f32<DT>(wv);
                            }
                            const float2 yf = x2_to_f32<DT>(yw[qq]);
                            // the post step's operation order (mhc_post.cuh)
#pragma unroll
                            for (int o = 0; o < NS; ++o) {
                                float a = __fmul_rn(res[o * NS], xf[0].x);
                                float c = __fmul_rn(res[o * NS], xf[0].y);
#pragma unroll
                                for (int t = 1; t < NS; ++t) {
                                    a = __fmaf_rn(res[o * NS + t], xf[t].x, a);
                                    c = __fmaf_rn(res[o * NS + t], xf[t].y, c);
                                }
                                a = __fmaf_rn(post[o], yf.x, a);
                                c = __fmaf_rn(post[o], yf.y, c);
                                const uint32_t packed = f32x2_to_x2_packed<DT>(a, c);
                                ow[o][qq] = packed;
                                // the next MhcPre's square-sum, of the rounded xNext
                                const float2 r = x2_to_f32<DT>(packed);
                                ss = fmaf(r.x, r.x, ss);
                                ss = fmaf(r.y, r.y, ss);
                            }
                        }
                        // every input piece of this row position is read: write xNext over x
#pragma unroll
                        for (int o = 0; o < NS; ++o)
                            sts128(xBase[o] + off, make_uint4(ow[o][0], ow[o][1], ow[o][2], ow[o][3]));
                    }
                    fence_proxy_async_shared();  // the MMA and the TMA stores read these shared-memory writes
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&postDone[s]);
                    if (pw == 0 && lane == 0) MHC_TRACE_EV(kTrRowReduced, g, tile);
                    // the previous d-chunk's segment (its MMA finished while this one's
                    // post step ran) into registers
                    if (flusher && i >= 1 && !flush(g - 1)) {
                        itemOk = false;
                        break;
                    }
                }
                // the item's last segment; the four parts of each row's sum of squares.
                // Every post warp takes both barriers once per item, also after a wait
                // gave up (the abort flag then ends every other wait promptly), so the
                // barriers always match.
                if (flusher && itemOk) itemOk = flush(g - 1);
                if (!flusher) sSumsq[(part - 1) * kRowsPerTile + row] = ss;
                named_bar_sync(1, kPostPreWarps * 32);
                const bool anyFailed = bar_red_or(2, kPostPreWarps * 32, !itemOk);
                if (!anyFailed && flusher) {
                    const float ssRow =
                        ((ss + sSumsq[row]) + sSumsq[kRowsPerTile + row]) + sSumsq[2 * kRowsPerTile + row];
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
                        out[MIX] = ssRow;
                    }
                }
                named_bar_sync(1, kPostPreWarps * 32);  // sSumsq is free for the next item
                if (anyFailed) ok = false;
            }
            if (!ok && lane == 0) fail();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tacc, kTmemCols);
    }
}
