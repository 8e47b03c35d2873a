// Internal interface between the C-ABI layer (mhc_pre_api.cpp) and the kernels
// (mhc_pre_kernels.cu).  Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/mhc_pre.h"

namespace mhc {

// Workspace header written by the weight-preparation kernel.
struct WorkspaceHeader {
    uint32_t magic;       // kPreparedMagic once weights are prepared
    int32_t phiScaleExp;  // fp16: prepared phi' = phi * 2^exp (bf16: 0)
    uint32_t signature;   // hash of the description the weights were prepared for
    uint32_t maxAbsBits;  // max |phi'| (float bits) during preparation
    // Arrivals at the grid barrier of the decode and small-batch kernels, summed
    // over all their launches on this workspace (zeroed with the header when weights
    // are prepared).  Each launch of either kernel adds its grid size G, and a launch
    // without prepared weights returns before arriving, so the count stays a
    // multiple of G.  A launch that gave up the barrier (MHC_STATUS_DEVICE_TIMEOUT)
    // can leave it off: prepare the weights again before the next launch.
    unsigned long long gridBarrier;
    uint32_t pad[58];
};
static_assert(sizeof(WorkspaceHeader) == 256, "header is 256 bytes");
constexpr uint32_t kPreparedMagic = 0x5048434Du;  // "MCHP"

constexpr int kRowsPerTile = 128;  // token rows per tensor-core tile (MMA M)
constexpr int kChunk = 64;         // K elements per TMA box / pipeline stage (128 bytes)
constexpr int kMaxMix = 80;
constexpr int kFusedSlots = 2;     // record/hPre slots per team in the fused kernel
// Row ranges of the single-launch kernels.  The decode kernel (path 2) handles up to
// kDecodeMaxRows rows and the small-batch kernel (path 4) up to kSmallMaxRows; by
// default the plan takes the decode kernel up to kDecodeDefaultRows, the small-batch
// kernel up to kSmallDefaultRows and the split-K path beyond, where each was the
// fastest in a CUDA-graph latency sweep on B200 (n=4, D=7168).
constexpr int kDecodeMaxRows = 32;
constexpr int kDecodeDefaultRows = 16;
constexpr int kSmallMaxRows = 512;
constexpr int kSmallDefaultRows = 384;

// Shared memory of the small-batch kernel (path 4): a ring of stages, each holding
// the row tiles of one K chunk and that chunk of the prepared weights.
constexpr size_t small_stage_bytes(int tiles, int N) {
    return static_cast<size_t>(tiles) * kRowsPerTile * kChunk * 2 + static_cast<size_t>(N) * kChunk * 2;
}
constexpr size_t small_smem_bytes(int tiles, int N, int stages) {
    return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * small_stage_bytes(tiles, N) + 256 /*barriers*/;
}

// Everything a launch needs, derived once from the description.
struct Problem {
    int64_t M;      // batch * seq
    int n;          // streams
    int64_t D;      // head dim
    int64_t K;      // n * D
    int mix;        // n*n + 2n
    int N;          // 2 * mix (hi and lo halves of the prepared weights)
    int W;          // floats per partial record: mix + 1 rounded up to 4
    int dtype;      // mhcDtype_t
    bool hasGamma;
    float normEps;
    float hcEps;
    uint32_t signature;
};

struct Plan {
    int path;        // 0: split-K GEMM + epilogue kernels, 1: fused team kernel, 2: decode kernel,
                     // 3: cluster-team kernel, 4: small-batch kernel
    int tilesM;      // ceil(M / 128)
    int chunks;      // ceil(K / 64)
    int splits;      // K splits (path 0)
    int stages;      // pipeline depth of the GEMM kernel (path 0)
    int gemmGrid;    // persistent CTAs of the GEMM kernel (path 0)
    size_t smemBytes;
    size_t phiOffset, phiBytes;
    size_t partOffset, partBytes;
    // path 1 (fused): teams of S members, J chunks per stream per member
    int teamS, teams, J, gStages, hStages;
    size_t hpreOffset, cntOffset, cntBytes;
    size_t totalBytes;
    // launch tuning (defaults unless plan options override them)
    int tmaBatch;    // path 0: chunks per TMA producer batch
    int l2mode;      // paths 1 and 3: L2 hint mode
    int lead;        // path 3: chunks the first read may run ahead of the re-read
    // path 5 (one pass): record ring slots and CTAs per SM
    int ringTiles;
    int opCtasPerSm;
    // path 0 at n = 8: the GEMM runs on CTA pairs (one M = 256 MMA, cta_group::2)
    bool pairGemm;
    // path 0: epilogue blocks (rows) resident per SM the epilogue is compiled for, 12
    // or 16; 16 takes fewer registers per thread and keeps more rows in flight, which
    // pays where the epilogue is latency-bound (up to kEpiWideMaxRows rows)
    int epiBlocks;
};
constexpr int64_t kEpiWideMaxRows = 16384;

// The post step fused with the next MhcPre's contraction (n = 4, D % 64 == 0): a stage
// holds the x tiles of the 4 streams and the y tile of one 64-wide d-chunk (16 KB
// each) and the 4 weight chunks of N = 48 rows (6 KB each).
constexpr size_t kPostPreStageBytesHost = 5 * static_cast<size_t>(kRowsPerTile) * kChunk * 2 + 4 * 48 * kChunk * 2;
constexpr int kPostPreStages = 2;
constexpr size_t post_pre_smem_bytes(int stages) {
    return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * kPostPreStageBytesHost + 256 /*barriers*/ +
           3 * 128 * 4 /*partial sums of squares*/;
}
struct PostPrePlan {
    int tilesM, dChunks, splits, stages, grid;
    size_t smemBytes;
};
// The fused path applies (n = 4, D % 64 == 0, and the default MhcPre plan is the
// split-K path); its splits never exceed the split-K plan's, so the workspace of
// mhcPreGetWorkspaceSize suffices.
bool post_pre_applies(const Problem& p, const Plan& defaultPlan);
PostPrePlan make_post_pre_plan(const Problem& p, const Plan& defaultPlan, int smCount);
int launch_post_pre(const Problem& p, const PostPrePlan& pp, const Plan& plan, const CUtensorMap& xMap,
                    const CUtensorMap& yMap, const CUtensorMap& xNextMap, const CUtensorMap& phiMap,
                    const float* hPost, const float* hRes, const void* xNext, const float* alpha, const float* bias,
                    void* hIn, float* hPostNext, float* hResNext, void* workspace, cudaStream_t stream);

// Shared memory of the CTA-pair GEMM (n = 8): stages of a 128-row x tile and half of
// the 160 weight rows of one 64-wide chunk.
constexpr size_t kPairStageBytesHost = static_cast<size_t>(kRowsPerTile) * kChunk * 2 + 80 * kChunk * 2;
constexpr size_t pair_smem_bytes(int stages) {
    return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * kPairStageBytesHost + 512 /*barriers*/;
}

// One-pass kernel (path 5) layout constants, shared by the plan and the launcher.
constexpr int kOnePassItemChunks = 4;  // default 64-wide chunks per work item
constexpr int kOnePassRingTiles = 16;  // default record ring slots
constexpr size_t onepass_host_smem(size_t stageBytes, int stages) {
    return 1024 /*alignment slack*/ + static_cast<size_t>(stages) * stageBytes + 256 /*barriers*/;
}

int make_problem(const mhcPreDesc_t* desc, Problem* p);
// opt may be null (the default plan, which depends on the description and the
// device only).
int make_plan(const Problem& p, int smCount, const mhcPrePlanOptions_t* opt, Plan* plan);

// Kernel launchers (return cudaError_t as int).
int launch_prepare(const Problem& p, const Plan& plan, const float* phi, const float* gamma, void* workspace,
                   cudaStream_t stream);
int launch_run(const Problem& p, const Plan& plan, const CUtensorMap& xMap, const CUtensorMap& phiMap,
               const void* x, const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes,
               void* workspace, cudaStream_t stream, cudaEvent_t evBegin = nullptr, cudaEvent_t evEnd = nullptr);
int read_and_clear_device_status(int32_t* status);
int trace_read(void* dst, size_t maxRecords, size_t* recorded);  // trace build only (MHC_TRACE)
void debug_set_record_cap(int64_t floats);                        // debug build only (MHC_DEBUG)
int debug_last_check_line(int* line);                             // debug build only (MHC_DEBUG)
int launch_post(const Problem& p, const void* x, const void* y, const float* hPost, const float* hRes, void* xNext,
                cudaStream_t stream);
size_t decode_smem(const Problem& p);  // dynamic shared memory of the decode kernel
int diag_wait_timeout(uint64_t limit_ns, int* result_host, cudaStream_t stream);
size_t cluster_extra(const Problem& p);  // cluster kernel's shared memory beyond its rings
int cluster_max_teams(const Problem& p, const Plan& plan, int* teams);

// Validation + plan for the current device, and prepare-then-run into a given
// workspace (used by the no-allocation entry point).
int plan_for(const mhcPreDesc_t* desc, Problem* p, Plan* plan);  // default plan
int prepare_and_run(const Problem& p, const Plan& plan, const void* x, const float* phi, const float* alpha,
                    const float* bias, const float* gamma, void* hIn, float* hPost, float* hRes, void* workspace,
                    cudaStream_t stream);

}  // namespace mhc
