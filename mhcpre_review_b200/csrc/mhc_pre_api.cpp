// C ABI of the MhcPre operator (declared in include/mhc_pre.h).
//
// This layer mirrors the reference host op (code/op_host/mhc_pre.cpp):
//   - the same shape rejects as TilingFunc (:57-79, :126-129),
//   - the InferShape output shapes (:217-249) are implied by the description,
//   - a workspace sized on the host, owned by the caller (:183-190),
// and replaces the Ascend tiling (core split, M64 matmul tiling, tiling cache)
// with a B200 launch plan.  It keeps no mutable global state.
#include <algorithm>
#include <cstring>

#include "mhc_pre_internal.h"
#ifdef MHC_TRACE
#include "../../include/mhc_pre_trace.h"
#endif
#ifdef MHC_DEBUG
#include "../../include/mhc_pre_debug.h"
#endif

namespace mhc {

static uint32_t fnv1a(const void* data, size_t n, uint32_t h = 2166136261u) {
    const auto* b = static_cast<const uint8_t*>(data);
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 16777619u;
    }
    return h;
}

int make_problem(const mhcPreDesc_t* desc, Problem* p) {
    if (desc == nullptr || p == nullptr) return MHC_STATUS_NULL_POINTER;
    if (desc->batch <= 0 || desc->seq <= 0 || desc->headDim <= 0) return MHC_STATUS_BAD_SHAPE;
    if (desc->streams != 4 && desc->streams != 6 && desc->streams != 8) return MHC_STATUS_BAD_STREAM_COUNT;
    if (desc->dtype != MHC_DTYPE_F16 && desc->dtype != MHC_DTYPE_BF16) return MHC_STATUS_BAD_DTYPE;
    const int64_t n = desc->streams;
    const int64_t mix = n * n + 2 * n;
    if (mix > kMaxMix) return MHC_STATUS_MIX_TOO_LARGE;
    if (desc->headDim % 16 != 0 || (n * desc->headDim) % 8 != 0) return MHC_STATUS_BAD_HEAD_DIM;
    // TMA coordinates and the row index of the tile grid are 32-bit.
    if (desc->batch > (int64_t(1) << 31) / desc->seq) return MHC_STATUS_TOO_LARGE;
    const int64_t M = desc->batch * desc->seq;
    const int64_t K = n * desc->headDim;
    if (K >= (int64_t(1) << 31) || M >= (int64_t(1) << 31)) return MHC_STATUS_TOO_LARGE;
    p->M = M;
    p->n = static_cast<int>(n);
    p->D = desc->headDim;
    p->K = K;
    p->mix = static_cast<int>(mix);
    p->N = static_cast<int>(2 * mix);
    p->W = static_cast<int>((mix + 1 + 3) / 4 * 4);
    p->dtype = desc->dtype;
    p->hasGamma = desc->hasGamma != 0;
    p->normEps = desc->normEps;
    p->hcEps = desc->hcEps;
    const int64_t sig[4] = {n, desc->headDim, desc->dtype, desc->hasGamma != 0};
    p->signature = fnv1a(sig, sizeof(sig));
    return MHC_STATUS_SUCCESS;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// At most this many 64-wide chunks per K split for large M (3200 K elements).  At
// config 4 (448 chunks) that makes 9 splits: 512 tiles x 9 = 4608 items fill 7.8
// waves of the GEMM's 592 CTA slots on one GPU, and the 8-GPU shard's 576 items
// fill 97% of one wave (7 splits left the last wave almost empty and the shard's
// only wave 76% full: 1.5% and 1.4% slower, measured).
constexpr int kGroupChunks = 50;
constexpr int64_t kShardRows = 8192;  // from this M up, splits depend on K only
constexpr int kMinSplitChunks = 6;    // smallest split below kShardRows rows

int make_plan(const Problem& p, int smCount, const mhcPrePlanOptions_t* opt, Plan* plan) {
    static const mhcPrePlanOptions_t kDefaults = {MHC_PRE_PATH_AUTO, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, {0, 0, 0, 0, 0}};
    const mhcPrePlanOptions_t& o = opt != nullptr ? *opt : kDefaults;
    const bool autoPath = o.path == MHC_PRE_PATH_AUTO;
    Plan pl{};
    pl.path = 0;
    pl.tilesM = static_cast<int>((p.M + kRowsPerTile - 1) / kRowsPerTile);
    pl.chunks = static_cast<int>((p.K + kChunk - 1) / kChunk);
    // GEMM CTAs per SM.  One CTA's MMA issue stream retires a tcgen05.mma about every
    // 145 cycles whatever N is, and a CTA's ring streams about stages x 16 KB per TMA
    // round trip (~2.5 us), so more CTAs per SM stream faster and split the work into
    // more, smaller shares (the last round of items costs less), as far as TMEM
    // (the kernel's accumulator buffers of N columns, rounded to a power of two),
    // registers and shared memory allow: four for n=4 (2 stages each), two for n=6
    // (two buffers) and for n=8 (one buffer).
    const int accBufs = p.N > 128 ? 1 : 2;  // GemmCfg<N>::kAccBufs
    const int accNeed = accBufs * p.N;
    const int accCols = accNeed <= 64 ? 64 : accNeed <= 128 ? 128 : accNeed <= 256 ? 256 : 512;
    const int maxCtas = std::min(512 / accCols, p.N <= 48 ? 4 : 2);
    int ctasPerSm = maxCtas;
    if (o.gemmCtasPerSm > 0) ctasPerSm = std::min(o.gemmCtasPerSm, maxCtas);
    const int slots = ctasPerSm * smCount;
    // K splits.  From kShardRows rows up, the split count depends on K only (groups
    // of at most kGroupChunks chunks), so a row's arithmetic, and therefore its
    // result bits, do not depend on M: token shards of that size reproduce the
    // unsharded run exactly.  Smaller problems split further to fill the GEMM's CTA
    // slots, down to kMinSplitChunks chunks per split: below that the epilogue's
    // reduction over splits costs more than the GEMM CTAs save.
    const int groups = (pl.chunks + kGroupChunks - 1) / kGroupChunks;
    int splits = groups;
    if (p.M < kShardRows && pl.tilesM < slots)
        splits = std::max(groups, std::min(slots / pl.tilesM, std::max(1, pl.chunks / kMinSplitChunks)));
    if (o.splits > 0) splits = o.splits;
    splits = std::min(splits, pl.chunks);
    pl.splits = splits;
    const size_t stageBytes = static_cast<size_t>(kRowsPerTile) * kChunk * 2 + static_cast<size_t>(p.N) * kChunk * 2;
    const size_t smemLimit = 232448;  // sm_100 per-block opt-in maximum
    const size_t fixed = 1024 /*alignment slack*/ + 256 /*barriers*/;
    const size_t budget = ctasPerSm == 1 ? smemLimit : ctasPerSm == 2 ? 110 * 1024 : ctasPerSm == 3 ? 74 * 1024
                                                                                                        : 55 * 1024;
    int stages = static_cast<int>((budget - fixed) / stageBytes);
    stages = std::max(2, std::min(stages, 8));
    if (o.gemmStages > 0) stages = std::max(2, std::min(o.gemmStages, stages));
    pl.stages = stages;
    pl.tmaBatch = o.tmaBatch > 0 ? std::min(o.tmaBatch, stages) : std::min(4, stages / 2);
    pl.l2mode = o.l2Hint > 0 ? std::min(o.l2Hint - 1, 2) : 1;
    pl.lead = 0;
    pl.gemmGrid = std::min(pl.tilesM * splits, smCount * ctasPerSm);
    pl.smemBytes = fixed + static_cast<size_t>(stages) * stageBytes;
    // n = 8: the GEMM on CTA pairs when plan options ask for it (the same splits,
    // so the same result bits): items are (256-row pair tile, split), one pair per
    // SM's worth of CTA slots, four 26 KB stages per CTA.
    pl.pairGemm = p.N == 160 && o.pairedGemm == 2;
    pl.epiBlocks = o.epiBlocks != 0 ? o.epiBlocks : p.M <= kEpiWideMaxRows ? 16 : 12;
    if (pl.pairGemm) {
        const int pairTiles = (pl.tilesM + 1) / 2;
        pl.stages = std::max(2, std::min(o.gemmStages > 0 ? o.gemmStages : 4, 4));
        pl.tmaBatch = o.tmaBatch > 0 ? std::min(o.tmaBatch, pl.stages) : std::min(4, pl.stages / 2);
        pl.gemmGrid = 2 * std::min(pairTiles * splits, smCount);
        pl.smemBytes = pair_smem_bytes(pl.stages);
    }
    pl.phiOffset = sizeof(WorkspaceHeader);
    pl.phiBytes = static_cast<size_t>(p.N) * static_cast<size_t>(p.K) * 2;
    pl.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
    pl.partBytes = static_cast<size_t>(splits) * static_cast<size_t>(p.M) * static_cast<size_t>(p.W) * 4;
    pl.totalBytes = align_up(pl.partOffset + pl.partBytes, 256);

    // Path 2, the decode kernel, by default for M up to kDecodeDefaultRows: one
    // cooperative launch of one CTA per SM (at most one per 64-wide chunk), CUDA-core
    // partial sums per K-slice, a grid barrier, then the per-row reduction, epilogue
    // and hIn.  Plan options select it up to kDecodeMaxRows (tests); forcing any
    // other path turns it off.
    {
        if ((autoPath && p.M <= kDecodeDefaultRows) || (o.path == 2 && p.M <= kDecodeMaxRows)) {
            pl.path = 2;
            pl.splits = std::min(smCount, pl.chunks);
            pl.gemmGrid = pl.splits;
            pl.stages = 0;
            pl.smemBytes = decode_smem(p);
            pl.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
            pl.partBytes = static_cast<size_t>(pl.splits) * static_cast<size_t>(p.M) * static_cast<size_t>(p.W) * 4;
            pl.totalBytes = align_up(pl.partOffset + pl.partBytes, 256);
            *plan = pl;
            return MHC_STATUS_SUCCESS;
        }
    }

    // Path 4, the small-batch kernel, by default for kDecodeDefaultRows < M <=
    // kSmallDefaultRows: one
    // cooperative launch of one CTA per SM (at most one per 64-wide chunk).  Each CTA
    // runs the tcgen05 contraction of all T = ceil(M/128) row tiles over its K-slice
    // (every tile's MMA reads the same weight chunk); after one grid barrier each CTA
    // reduces the records of its rows (m % G == CTA) and streams their hIn.  It needs
    // T accumulators of N columns in TMEM.  Plan options select it for any M up to
    // kSmallMaxRows (tests); forcing any other path turns it off.  Above
    // kSmallDefaultRows rows the split-K path is faster: its epilogue spreads the hIn
    // stream over one CTA per row, while here each SM streams several rows.
    {
        const bool forced = o.path == 4;
        const int tiles = pl.tilesM;
        if (((autoPath && p.M > kDecodeDefaultRows && p.M <= kSmallDefaultRows) ||
             (forced && p.M <= kSmallMaxRows)) &&
            tiles * p.N <= 512) {
            pl.path = 4;
            pl.splits = std::min(smCount, pl.chunks);
            pl.gemmGrid = pl.splits;
            const size_t stage = small_stage_bytes(tiles, p.N);
            const int maxChunks = (pl.chunks + pl.splits - 1) / pl.splits;  // per CTA
            int stages = static_cast<int>((232448 - small_smem_bytes(tiles, p.N, 0)) / stage);
            stages = std::max(1, std::min(std::min(stages, 8), maxChunks));
            pl.stages = stages;
            pl.smemBytes = small_smem_bytes(tiles, p.N, stages);
            pl.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
            pl.partBytes = static_cast<size_t>(pl.splits) * static_cast<size_t>(p.M) * static_cast<size_t>(p.W) * 4;
            pl.totalBytes = align_up(pl.partOffset + pl.partBytes, 256);
            *plan = pl;
            return MHC_STATUS_SUCCESS;
        }
    }

    // Path 5, the one-pass kernel (n = 4; opt-in through plan options): x is read from
    // HBM once.  Work items of kOnePassItemChunks chunks (a K-split count that depends
    // on K only, so results never depend on M), three CTAs per SM with four hIn warps
    // each, or two with eight; the ring depth fills each CTA's share of shared memory.
    if (o.path == 5 && p.n == 4) {
        Plan c = pl;
        c.path = 5;
        c.opCtasPerSm = o.gemmCtasPerSm == 2 ? 2 : 3;
        c.splits = o.splits > 0 ? std::min(o.splits, pl.chunks) : std::max(1, pl.chunks / kOnePassItemChunks);
        const size_t ctaBudget = c.opCtasPerSm == 2 ? 113 * 1024 : 75 * 1024;
        int st = static_cast<int>((ctaBudget - onepass_host_smem(stageBytes, 0)) / stageBytes);
        st = std::max(2, std::min(st, 8));
        if (o.gemmStages > 0) st = std::max(2, std::min(o.gemmStages, st));
        c.stages = st;
        c.tmaBatch = o.tmaBatch > 0 ? std::min(o.tmaBatch, st) : std::max(1, std::min(4, st / 2));
        c.ringTiles = std::min(o.ringTiles > 0 ? o.ringTiles : kOnePassRingTiles, pl.tilesM);
        c.gemmGrid = c.opCtasPerSm * smCount;
        c.smemBytes = onepass_host_smem(stageBytes, st);
        c.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
        c.partBytes = static_cast<size_t>(c.ringTiles) * kRowsPerTile * static_cast<size_t>(c.splits) *
                      static_cast<size_t>(p.W) * 4;
        c.cntOffset = align_up(c.partOffset + c.partBytes, 256);
        c.cntBytes = align_up((2 * static_cast<size_t>(c.ringTiles) + 1) * 4, 256);
        c.totalBytes = c.cntOffset + c.cntBytes;
        *plan = c;
        return MHC_STATUS_SUCCESS;
    }

    // Path 3, the cluster-team kernel (opt-in through plan options), when D splits into
    // 64-wide chunks evenly over a cluster of S = 16 (or 8) CTAs.  The teams are as
    // many clusters as fit on the device at once.
    {
        if (o.path == 3 && p.D % kChunk == 0) {
            const int dc = static_cast<int>(p.D / kChunk);
            const int S = dc % 16 == 0 ? 16 : dc % 8 == 0 ? 8 : 0;
            if (S > 0) {
                Plan c = pl;
                c.path = 3;
                c.teamS = S;
                c.J = dc / S;
                c.splits = 1;
                const size_t gStage = static_cast<size_t>(kRowsPerTile) * kChunk * 2 + static_cast<size_t>(p.N) * kChunk * 2;
                const size_t hStage = static_cast<size_t>(kRowsPerTile) * kChunk * 2;
                // ring depths: the hIn ring shrinks (4 -> 2) until a GEMM ring of >= 2 fits
                const size_t fixed = 1024 + cluster_extra(p);
                c.hStages = 0;
                for (int hs = 4; hs >= 2; --hs) {
                    if (fixed + hs * hStage + 2 * gStage > 232448) continue;
                    c.hStages = hs;
                    c.gStages = std::min(6, static_cast<int>((232448 - fixed - hs * hStage) / gStage));
                    break;
                }
                c.smemBytes = fixed + c.gStages * gStage + c.hStages * hStage;
                c.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
                c.partBytes = 0;
                c.hpreOffset = c.partOffset;
                c.cntOffset = c.partOffset;
                c.cntBytes = 256;  // the global abort word
                c.lead = o.clusterLead > 0 ? o.clusterLead : c.gStages + 2;
                c.totalBytes = c.cntOffset + c.cntBytes;
                int teams = 0;
                if (c.hStages > 0 && cluster_max_teams(p, c, &teams) == 0 && teams > 0) {
                    c.teams = std::min(teams, c.tilesM);
                    *plan = c;
                    return MHC_STATUS_SUCCESS;
                }
            }
        }
    }

    // Path 1, the fused kernel, when D splits into 64-wide chunks evenly over a team
    // (a row's arithmetic depends on the team size S only, not on M).  S divides
    // D/64.  Its hIn pass re-reads x from L2, which can hit only while the tiles the
    // teams have in flight fit in L2; S is the smallest divisor that keeps one round
    // of tiles (one per team) under kFusedFootprint among those using the most SMs,
    // else the largest divisor.
    // It is opt-in (through plan options): on B200 one team handshake
    // (records, owner reduction, hPre) takes tens of microseconds while every SM
    // streams, because each step queues behind the SM's TMA traffic; a byte of x then
    // waits ~80 us for its re-read, far more than L2 holds at full bandwidth, so the
    // re-read mostly misses and the kernel runs slower than the split-K path.
    if (o.path == 1 && p.D % kChunk == 0) {
        const int dc = static_cast<int>(p.D / kChunk);
        const double tileBytes = static_cast<double>(kRowsPerTile) * static_cast<double>(p.K) * 2.0;
        constexpr double kFusedFootprint = 40.0e6;
        int bestS = 0, bestUse = -1;
        for (int S = 8; S <= 64 && S <= smCount; ++S) {
            if (dc % S != 0) continue;
            const int teams = std::min<int64_t>(smCount / S, pl.tilesM);
            if (teams * tileBytes > kFusedFootprint) continue;
            const int use = teams * S;
            if (use > bestUse) {
                bestS = S;
                bestUse = use;
            }
        }
        if (bestS == 0)
            for (int S = 8; S <= 64 && S <= smCount; ++S)
                if (dc % S == 0) bestS = S;
        if (bestS == 0 && dc >= 8 && dc <= 32 && dc <= smCount) bestS = dc;  // owners hold <= 16 rows
        // A team size from the plan options must divide D/64, 8 <= S <= 64.
        if (o.teamSize > 0) {
            const int fs = o.teamSize;
            if (fs >= 8 && fs <= 64 && fs <= smCount && dc % fs == 0) bestS = fs;
        }
        if (bestS > 0) {
            const int T = std::min(smCount / bestS, pl.tilesM);
            if (T >= 1) {
                pl.path = 1;
                pl.teamS = bestS;
                pl.teams = T;
                pl.J = dc / bestS;
                const size_t gStage = static_cast<size_t>(kRowsPerTile) * kChunk * 2 + static_cast<size_t>(p.N) * kChunk * 2;
                const size_t hStage = static_cast<size_t>(kRowsPerTile) * kChunk * 2;
                pl.hStages = p.N <= 48 ? 5 : 4;
                const size_t ownBytes = static_cast<size_t>((kRowsPerTile + bestS - 1) / bestS) * bestS * p.W * 4;
                const size_t fixed = 1024 + 16 * static_cast<size_t>(p.W) * 4 + ownBytes + 512;
                int gs = static_cast<int>((smemLimit - fixed - pl.hStages * hStage) / gStage);
                pl.gStages = std::max(2, std::min(gs, 8));
                pl.smemBytes = fixed + pl.gStages * gStage + pl.hStages * hStage;
                pl.splits = 1;
                pl.partOffset = align_up(pl.phiOffset + pl.phiBytes, 256);
                pl.partBytes = static_cast<size_t>(T) * kFusedSlots * bestS * kRowsPerTile * p.W * 4;
                pl.hpreOffset = align_up(pl.partOffset + pl.partBytes, 256);
                pl.cntOffset = align_up(pl.hpreOffset + static_cast<size_t>(T) * kFusedSlots * kRowsPerTile * 8 * 4, 256);
                pl.cntBytes = align_up((2 * kFusedSlots * static_cast<size_t>(T) + 1) * 4, 256);
                pl.totalBytes = pl.cntOffset + pl.cntBytes;
            }
        }
    }
    *plan = pl;
    return MHC_STATUS_SUCCESS;
}

static int device_sm_count(int* sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MHC_STATUS_CUDA_ERROR;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return MHC_STATUS_CUDA_ERROR;
    if (major != 10) return MHC_STATUS_UNSUPPORTED_DEVICE;
    if (cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return MHC_STATUS_CUDA_ERROR;
    return MHC_STATUS_SUCCESS;
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }
static bool aligned4(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn lookup_encode_fn() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
        return nullptr;
    return reinterpret_cast<EncodeTiledFn>(fn);
}

// The driver entry point, looked up once per process (the lookup costs microseconds
// per call otherwise).
static EncodeTiledFn get_encode_fn() {
    static const EncodeTiledFn fn = lookup_encode_fn();
    return fn;
}

// 2-D K-contiguous matrix [rows][K] of 16-bit elements, 64 x boxRows boxes,
// 128-byte swizzle (the layout the tensor-core descriptors expect).
static int encode_2d(EncodeTiledFn enc, CUtensorMap* map, const void* base, int dtype, uint64_t K, uint64_t rows,
                     uint32_t boxRows) {
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {K * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunk), boxRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        dtype == MHC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

static int options_ok(const mhcPrePlanOptions_t* opt) {
    if (opt == nullptr) return MHC_STATUS_SUCCESS;
    if (opt->path < MHC_PRE_PATH_AUTO || opt->path > 5) return MHC_STATUS_BAD_SHAPE;
    if (opt->pairedGemm < 0 || opt->pairedGemm > 2) return MHC_STATUS_BAD_SHAPE;
    if (opt->epiBlocks != 0 && opt->epiBlocks != 12 && opt->epiBlocks != 16) return MHC_STATUS_BAD_SHAPE;
    for (int r : opt->reserved)
        if (r != 0) return MHC_STATUS_BAD_SHAPE;
    return MHC_STATUS_SUCCESS;
}

// Validation and plan for the current device under the given options (may be null).
static int plan_with(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* opt, Problem* p, Plan* plan) {
    int rc = options_ok(opt);
    if (rc != 0) return rc;
    rc = make_problem(desc, p);
    if (rc != 0) return rc;
    int sms = 0;
    rc = device_sm_count(&sms);
    if (rc != 0) return rc;
    return make_plan(*p, sms, opt, plan);
}

static int prepare_common(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* opt, Problem* p, Plan* plan,
                          size_t wsBytes, const void* ws) {
    int rc = plan_with(desc, opt, p, plan);
    if (rc != 0) return rc;
    if (ws == nullptr) return MHC_STATUS_NULL_POINTER;
    if (!aligned16(ws)) return MHC_STATUS_MISALIGNED;
    if (wsBytes < plan->totalBytes) return MHC_STATUS_WORKSPACE_TOO_SMALL;
    return MHC_STATUS_SUCCESS;
}

static int run_prepared(const Problem& p, const Plan& plan, const void* x, const float* alpha, const float* bias,
                        void* hIn, float* hPost, float* hRes, void* workspace, cudaStream_t stream,
                        cudaEvent_t evBegin = nullptr, cudaEvent_t evEnd = nullptr) {
    if (x == nullptr || alpha == nullptr || bias == nullptr || hIn == nullptr || hPost == nullptr ||
        hRes == nullptr)
        return MHC_STATUS_NULL_POINTER;
    if (!aligned16(x) || !aligned16(hIn) || !aligned4(hPost) || !aligned4(hRes) || !aligned4(alpha) ||
        !aligned4(bias))
        return MHC_STATUS_MISALIGNED;
    CUtensorMap xMap{}, phiMap{};
    if (plan.path == 2) {  // the decode kernel reads with plain loads: no tensor maps
        const int e = launch_run(p, plan, xMap, phiMap, x, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin,
                                 evEnd);
        return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
    }
    EncodeTiledFn enc = get_encode_fn();
    if (enc == nullptr) return MHC_STATUS_CUDA_ERROR;
    int rc = encode_2d(enc, &xMap, x, p.dtype, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.M), kRowsPerTile);
    if (rc != 0) return rc;
    const void* phiPrep = static_cast<const uint8_t*>(workspace) + plan.phiOffset;
    // the CTA-pair GEMM stages half of the weight rows in each CTA
    rc = encode_2d(enc, &phiMap, phiPrep, p.dtype, static_cast<uint64_t>(p.K), static_cast<uint64_t>(p.N),
                   static_cast<uint32_t>(plan.path == 0 && plan.pairGemm ? p.N / 2 : p.N));
    if (rc != 0) return rc;
    const int e =
        launch_run(p, plan, xMap, phiMap, x, alpha, bias, hIn, hPost, hRes, workspace, stream, evBegin, evEnd);
    return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

// Helpers for the no-allocation entry point (mhc_pre_noalloc.cu): the same
// validation, plan, weight preparation and launch as the entry points below,
// with the workspace supplied by the caller of these helpers.
int plan_for(const mhcPreDesc_t* desc, Problem* p, Plan* plan) { return plan_with(desc, nullptr, p, plan); }

int prepare_and_run(const Problem& p, const Plan& plan, const void* x, const float* phi, const float* alpha,
                    const float* bias, const float* gamma, void* hIn, float* hPost, float* hRes, void* workspace,
                    cudaStream_t stream) {
    if (phi == nullptr || (p.hasGamma && gamma == nullptr)) return MHC_STATUS_NULL_POINTER;
    if (!aligned4(phi) || (p.hasGamma && !aligned4(gamma))) return MHC_STATUS_MISALIGNED;
    if (launch_prepare(p, plan, phi, gamma, workspace, stream) != 0) return MHC_STATUS_CUDA_ERROR;
    return run_prepared(p, plan, x, alpha, bias, hIn, hPost, hRes, workspace, stream);
}

}  // namespace mhc

using namespace mhc;

extern "C" {

int mhcPreAbiVersion(void) { return MHC_PRE_ABI_VERSION; }

const char* mhcPreStatusString(int status) {
    switch (status) {
        case MHC_STATUS_SUCCESS: return "success";
        case MHC_STATUS_NULL_POINTER: return "null pointer";
        case MHC_STATUS_BAD_SHAPE: return "batch, seq and headDim must be positive";
        case MHC_STATUS_BAD_STREAM_COUNT: return "streams must be 4, 6 or 8";
        case MHC_STATUS_BAD_HEAD_DIM: return "headDim must be a multiple of 16";
        case MHC_STATUS_MIX_TOO_LARGE: return "streams*streams + 2*streams exceeds 80";
        case MHC_STATUS_BAD_DTYPE: return "dtype must be F16 or BF16";
        case MHC_STATUS_MISALIGNED: return "x, hIn, workspace need 16-byte and fp32 tensors 4-byte alignment";
        case MHC_STATUS_WORKSPACE_TOO_SMALL: return "workspace smaller than mhcPreGetWorkspaceSize";
        case MHC_STATUS_CUDA_ERROR: return "CUDA error";
        case MHC_STATUS_UNSUPPORTED_DEVICE: return "current device is not a B200 (sm_100)";
        case MHC_STATUS_DEVICE_TIMEOUT: return "a kernel gave up a bounded wait";
        case MHC_STATUS_NOT_PREPARED: return "workspace holds no prepared weights";
        case MHC_STATUS_TOO_LARGE: return "problem exceeds a size limit";
        case MHC_STATUS_INTERNAL_CHECK: return "a kernel's bounds check failed (debug build)";
        default: return "unknown status";
    }
}

int mhcPreGetWorkspaceSizeEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options,
                             size_t* workspaceBytes) {
    if (workspaceBytes == nullptr) return MHC_STATUS_NULL_POINTER;
    Problem p;
    Plan plan;
    const int rc = plan_with(desc, options, &p, &plan);
    if (rc != 0) return rc;
    *workspaceBytes = plan.totalBytes;
    return MHC_STATUS_SUCCESS;
}

int mhcPreGetWorkspaceSize(const mhcPreDesc_t* desc, size_t* workspaceBytes) {
    return mhcPreGetWorkspaceSizeEx(desc, nullptr, workspaceBytes);
}

int mhcPreQueryPlanEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, mhcPrePlan_t* out) {
    if (out == nullptr) return MHC_STATUS_NULL_POINTER;
    Problem p;
    Plan plan;
    const int rc = plan_with(desc, options, &p, &plan);
    if (rc != 0) return rc;
    std::memset(out, 0, sizeof(*out));
    out->path = plan.path;
    out->kernelsPerRun = plan.path == 0 ? 2 : 1;  // (the one-pass path also clears its counters: a memset)
    const bool teamPath = plan.path == 1 || plan.path == 3;
    out->gridCtas = teamPath ? plan.teams * plan.teamS : plan.gemmGrid;
    out->splits = teamPath ? plan.teamS : plan.splits;
    out->rowsPerTile = kRowsPerTile;
    out->reserved[0] = teamPath ? plan.teams : 0;
    return MHC_STATUS_SUCCESS;
}

int mhcPreQueryPlan(const mhcPreDesc_t* desc, mhcPrePlan_t* out) { return mhcPreQueryPlanEx(desc, nullptr, out); }

int mhcPrePrepareWeightsEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, const float* phi,
                           const float* gamma, void* workspace, size_t workspaceBytes, void* stream) {
    Problem p;
    Plan plan;
    int rc = prepare_common(desc, options, &p, &plan, workspaceBytes, workspace);
    if (rc != 0) return rc;
    if (phi == nullptr || (p.hasGamma && gamma == nullptr)) return MHC_STATUS_NULL_POINTER;
    if (!aligned4(phi) || (p.hasGamma && !aligned4(gamma))) return MHC_STATUS_MISALIGNED;
    const int e = launch_prepare(p, plan, phi, gamma, workspace, static_cast<cudaStream_t>(stream));
    return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

int mhcPrePrepareWeights(const mhcPreDesc_t* desc, const float* phi, const float* gamma, void* workspace,
                         size_t workspaceBytes, void* stream) {
    return mhcPrePrepareWeightsEx(desc, nullptr, phi, gamma, workspace, workspaceBytes, stream);
}

int mhcPreRunPreparedEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, const void* x,
                        const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes, void* workspace,
                        size_t workspaceBytes, void* stream, void* mainKernelBegin, void* mainKernelEnd) {
    Problem p;
    Plan plan;
    int rc = prepare_common(desc, options, &p, &plan, workspaceBytes, workspace);
    if (rc != 0) return rc;
    return run_prepared(p, plan, x, alpha, bias, hIn, hPost, hRes, workspace, static_cast<cudaStream_t>(stream),
                        static_cast<cudaEvent_t>(mainKernelBegin), static_cast<cudaEvent_t>(mainKernelEnd));
}

int mhcPreRunPrepared(const mhcPreDesc_t* desc, const void* x, const float* alpha, const float* bias, void* hIn,
                      float* hPost, float* hRes, void* workspace, size_t workspaceBytes, void* stream) {
    return mhcPreRunPreparedEx(desc, nullptr, x, alpha, bias, hIn, hPost, hRes, workspace, workspaceBytes, stream,
                               nullptr, nullptr);
}

int mhcPreRunPreparedProfiled(const mhcPreDesc_t* desc, const void* x, const float* alpha, const float* bias,
                              void* hIn, float* hPost, float* hRes, void* workspace, size_t workspaceBytes,
                              void* stream, void* mainKernelBegin, void* mainKernelEnd) {
    return mhcPreRunPreparedEx(desc, nullptr, x, alpha, bias, hIn, hPost, hRes, workspace, workspaceBytes, stream,
                               mainKernelBegin, mainKernelEnd);
}

int mhcPreRun(const mhcPreDesc_t* desc, const void* x, const float* phi, const float* alpha, const float* bias,
              const float* gamma, void* hIn, float* hPost, float* hRes, void* workspace, size_t workspaceBytes,
              void* stream) {
    int rc = mhcPrePrepareWeights(desc, phi, gamma, workspace, workspaceBytes, stream);
    if (rc != 0) return rc;
    return mhcPreRunPrepared(desc, x, alpha, bias, hIn, hPost, hRes, workspace, workspaceBytes, stream);
}

int mhcPostRun(const mhcPreDesc_t* desc, const void* x, const void* y, const float* hPost, const float* hRes,
               void* xNext, void* stream) {
    Problem p;
    int rc = make_problem(desc, &p);
    if (rc != 0) return rc;
    int sms = 0;
    rc = device_sm_count(&sms);
    if (rc != 0) return rc;
    if (x == nullptr || y == nullptr || hPost == nullptr || hRes == nullptr || xNext == nullptr)
        return MHC_STATUS_NULL_POINTER;
    if (!aligned16(x) || !aligned16(y) || !aligned16(xNext) || !aligned4(hPost) || !aligned4(hRes))
        return MHC_STATUS_MISALIGNED;
    if (p.M > 0x7fffffff) return MHC_STATUS_TOO_LARGE;  // one block per row
    const int e = launch_post(p, x, y, hPost, hRes, xNext, static_cast<cudaStream_t>(stream));
    return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

int mhcPostPreRun(const mhcPreDesc_t* desc, const void* x, const void* y, const float* hPost, const float* hRes,
                  void* xNext, const float* alpha, const float* bias, void* hIn, float* hPostNext, float* hResNext,
                  void* workspace, size_t workspaceBytes, void* stream) {
    Problem p;
    Plan plan;
    int rc = prepare_common(desc, nullptr, &p, &plan, workspaceBytes, workspace);
    if (rc != 0) return rc;
    if (x == nullptr || y == nullptr || hPost == nullptr || hRes == nullptr || xNext == nullptr ||
        alpha == nullptr || bias == nullptr || hIn == nullptr || hPostNext == nullptr || hResNext == nullptr)
        return MHC_STATUS_NULL_POINTER;
    if (!aligned16(x) || !aligned16(y) || !aligned16(xNext) || !aligned4(hPost) || !aligned4(hRes))
        return MHC_STATUS_MISALIGNED;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!post_pre_applies(p, plan)) {
        // the two steps one after the other
        if (launch_post(p, x, y, hPost, hRes, xNext, st) != 0) return MHC_STATUS_CUDA_ERROR;
        return run_prepared(p, plan, xNext, alpha, bias, hIn, hPostNext, hResNext, workspace, st);
    }
    if (!aligned16(hIn) || !aligned4(hPostNext) || !aligned4(hResNext) || !aligned4(alpha) || !aligned4(bias))
        return MHC_STATUS_MISALIGNED;
    int sms = 0;
    rc = device_sm_count(&sms);
    if (rc != 0) return rc;
    const PostPrePlan pp = make_post_pre_plan(p, plan, sms);
    EncodeTiledFn enc = get_encode_fn();
    if (enc == nullptr) return MHC_STATUS_CUDA_ERROR;
    CUtensorMap xMap{}, yMap{}, xNextMap{}, phiMap{};
    const uint64_t K = static_cast<uint64_t>(p.K), M = static_cast<uint64_t>(p.M), D = static_cast<uint64_t>(p.D);
    if ((rc = encode_2d(enc, &xMap, x, p.dtype, K, M, kRowsPerTile)) != 0) return rc;
    if ((rc = encode_2d(enc, &yMap, y, p.dtype, D, M, kRowsPerTile)) != 0) return rc;
    if ((rc = encode_2d(enc, &xNextMap, xNext, p.dtype, K, M, kRowsPerTile)) != 0) return rc;
    const void* phiPrep = static_cast<const uint8_t*>(workspace) + plan.phiOffset;
    if ((rc = encode_2d(enc, &phiMap, phiPrep, p.dtype, K, static_cast<uint64_t>(p.N), static_cast<uint32_t>(p.N))) != 0)
        return rc;
    const int e = launch_post_pre(p, pp, plan, xMap, yMap, xNextMap, phiMap, hPost, hRes, xNext, alpha, bias, hIn,
                                  hPostNext, hResNext, workspace, st);
    return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

int mhcPreDiagWaitTimeout(uint32_t limitMicroseconds, int32_t* countersGaveUp, int32_t* barriersGaveUp,
                          void* stream) {
    if (countersGaveUp == nullptr || barriersGaveUp == nullptr) return MHC_STATUS_NULL_POINTER;
    if (limitMicroseconds == 0 || limitMicroseconds > 1000000u) return MHC_STATUS_BAD_SHAPE;
    int major = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return MHC_STATUS_CUDA_ERROR;
    if (major != 10) return MHC_STATUS_UNSUPPORTED_DEVICE;
    int r[2] = {0, 0};
    if (diag_wait_timeout(static_cast<uint64_t>(limitMicroseconds) * 1000u, r, static_cast<cudaStream_t>(stream)) != 0)
        return MHC_STATUS_CUDA_ERROR;
    *countersGaveUp = r[0];
    *barriersGaveUp = r[1];
    return MHC_STATUS_SUCCESS;
}

#ifdef MHC_TRACE
MHC_API int mhcPreTraceRead(void* dst, size_t maxRecords, size_t* recorded) {
    if (recorded == nullptr) return MHC_STATUS_NULL_POINTER;
    return trace_read(dst, maxRecords, recorded) == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}
#endif

#ifdef MHC_DEBUG
MHC_API int mhcPreDebugSetRecordCap(int64_t maxFloats) {
    if (maxFloats < 0) return MHC_STATUS_BAD_SHAPE;
    debug_set_record_cap(maxFloats);
    return MHC_STATUS_SUCCESS;
}

MHC_API int mhcPreDebugLastCheckLine(int32_t* line) {
    if (line == nullptr) return MHC_STATUS_NULL_POINTER;
    int v = 0;
    if (debug_last_check_line(&v) != 0) return MHC_STATUS_CUDA_ERROR;
    *line = v;
    return MHC_STATUS_SUCCESS;
}
#endif

int mhcPreGetDeviceStatus(int32_t* deviceStatus) {
    if (deviceStatus == nullptr) return MHC_STATUS_NULL_POINTER;
    const int e = read_and_clear_device_status(deviceStatus);
    return e == 0 ? MHC_STATUS_SUCCESS : MHC_STATUS_CUDA_ERROR;
}

}  // extern "C"
