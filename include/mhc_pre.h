/*
 * mhc_pre.h -- C ABI of the B200-native MhcPre operator (libmhcpre_b200.so).
 *
 * MhcPre is the "pre" half of a manifold-constrained hyper-connection block.
 * For every token row r of x [B, S, n, D] (n in {4, 6, 8}, K = n*D,
 * mix = n*n + 2n):
 *
 *   invRms[r] = 1 / sqrt(sum_k x[r,k]^2 / K + normEps)      raw x, before gamma
 *   mix[r,j]  = sum_k x[r,k] * gamma[k] * phi[j,k]           phi stored [mix][K]
 *   hPre[r,s] = sigmoid(mix[r,s] * invRms * alpha[0] + bias[s]) + hcEps
 *   hPost     = 2 * sigmoid(mix[r,n+s] * invRms * alpha[1] + bias[n+s])   -> output
 *   hRes      = mix[r,2n+i] * invRms * alpha[2] + bias[2n+i]             -> output
 *   hIn[r,d]  = round_to_x_dtype(((hPre0*x0[d] + hPre1*x1[d]) + hPre2*x2[d]) + ...)
 *
 * It replaces the reference's generated two-phase aclnn API
 * (ZXY-0508/MhcPre-review, OpDef at code/op_host/mhc_pre.cpp:261-304, called at
 * cloud_runner/runner.cpp:443-472):
 *
 *   aclnnMhcPreGetWorkspaceSize(x, phi, alpha, bias, gamma, normEps, hcEps,
 *                               hIn, hPost, hRes, &workspaceSize, &executor)
 *   aclnnMhcPre(workspace, workspaceSize, executor, stream)
 *
 * Conventions (same as the reference):
 *   - the caller allocates every device buffer and the workspace; the operator
 *     writes only hIn, hPost, hRes and the workspace;
 *   - calls are asynchronous on the given CUDA stream (a cudaStream_t passed as
 *     void*; NULL is the legacy default stream) and never synchronize;
 *   - 0 means success, negative values are errors (see mhcStatus_t);
 *   - there is no global mutable host state: calls are reentrant and thread-safe
 *     (the reference keeps an unlocked 4-slot tiling cache, mhc_pre.cpp:51).
 * x, hIn and the workspace must be 16-byte aligned, the fp32 tensors 4-byte
 * aligned; all tensors are dense row-major.
 */
#ifndef MHC_PRE_H
#define MHC_PRE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MHC_PRE_ABI_VERSION 1

/* Exported entry points keep default visibility even when the library is
 * built with -fvisibility=hidden. */
#if defined(__GNUC__)
#define MHC_API __attribute__((visibility("default")))
#else
#define MHC_API
#endif

/* Data type of x and hIn (the reference's template key DT_X,
 * code/op_kernel/tiling_key_mhc_pre.h:6-13). */
typedef enum {
    MHC_DTYPE_F16 = 0,
    MHC_DTYPE_BF16 = 1
} mhcDtype_t;

typedef enum {
    MHC_STATUS_SUCCESS = 0,
    MHC_STATUS_NULL_POINTER = -1,        /* a required pointer is NULL */
    MHC_STATUS_BAD_SHAPE = -2,           /* B, S or D <= 0 (TilingFunc, mhc_pre.cpp:76-78) */
    MHC_STATUS_BAD_STREAM_COUNT = -3,    /* n not in {4, 6, 8} (mhc_pre.cpp:77) */
    MHC_STATUS_BAD_HEAD_DIM = -4,        /* D % 16 != 0 or n*D % 8 != 0 (mhc_pre.cpp:127-128) */
    MHC_STATUS_MIX_TOO_LARGE = -5,       /* n*n + 2n > 80 (mhc_pre.cpp:127) */
    MHC_STATUS_BAD_DTYPE = -6,           /* dtype not F16/BF16 (OpDef, mhc_pre.cpp:265-268) */
    MHC_STATUS_MISALIGNED = -7,          /* a device pointer violates the alignment rule above */
    MHC_STATUS_WORKSPACE_TOO_SMALL = -8, /* workspace smaller than mhcPreGetWorkspaceSize */
    MHC_STATUS_CUDA_ERROR = -9,          /* a CUDA runtime/driver call failed */
    MHC_STATUS_UNSUPPORTED_DEVICE = -10, /* current device is not sm_100 */
    MHC_STATUS_DEVICE_TIMEOUT = -11,     /* a kernel gave up a bounded wait (see mhcPreGetDeviceStatus) */
    MHC_STATUS_NOT_PREPARED = -12,       /* mhcPreRunPrepared on a workspace without prepared weights */
    MHC_STATUS_TOO_LARGE = -13,          /* problem exceeds a documented size limit */
    MHC_STATUS_INTERNAL_CHECK = -14      /* debug build only: a kernel's bounds check failed
                                            (see include/mhc_pre_debug.h) */
} mhcStatus_t;

/* Problem description: the shape/attribute part of the aclnn executor.
 * x is [batch, seq, streams, headDim]; gamma is optional ([streams, headDim]).
 * normEps/hcEps are the OpDef attributes (default 1e-6, mhc_pre.cpp:297-298). */
typedef struct {
    int64_t batch;
    int64_t seq;
    int64_t streams;
    int64_t headDim;
    int32_t dtype;    /* mhcDtype_t */
    int32_t hasGamma; /* 0 or 1 */
    float normEps;
    float hcEps;
} mhcPreDesc_t;

/* Validates the description (same rejects as the reference TilingFunc,
 * mhc_pre.cpp:57-79, :126-129) and returns the workspace size in bytes for the
 * current CUDA device.  Replaces aclnnMhcPreGetWorkspaceSize. */
MHC_API int mhcPreGetWorkspaceSize(const mhcPreDesc_t* desc, size_t* workspaceBytes);

/* Prepares the weights into the workspace: phi'[j,k] = gamma[k]*phi[j,k] split
 * into a high and a low 16-bit part of the x dtype, laid out for the tensor
 * cores.  phi is fp32 [mix][K] (the reference's phi layout, K-contiguous; see
 * cloud_runner/runner.cpp:157); gamma is fp32 [K] or NULL when hasGamma == 0.
 * After this call, mhcPreRunPrepared may be called any number of times with the
 * same workspace.  No reference counterpart: the reference re-reads fp32 phi on
 * every launch (mhc_pre.cpp:535). */
MHC_API int mhcPrePrepareWeights(const mhcPreDesc_t* desc, const float* phi, const float* gamma, void* workspace,
                                 size_t workspaceBytes, void* stream);

/* One-shot operator call: prepares the weights and runs the operator.
 * x: [B,S,n,D] f16/bf16; phi: fp32 [mix][K]; alpha: fp32 [3] (pre, post, res);
 * bias: fp32 [mix]; gamma: fp32 [K] or NULL; hIn: [B,S,D] x dtype;
 * hPost: fp32 [B,S,n]; hRes: fp32 [B,S,n,n].
 * Replaces aclnnMhcPreGetWorkspaceSize + aclnnMhcPre (runner.cpp:443-472). */
MHC_API int mhcPreRun(const mhcPreDesc_t* desc, const void* x, const float* phi, const float* alpha,
                      const float* bias, const float* gamma, void* hIn, float* hPost, float* hRes, void* workspace,
                      size_t workspaceBytes, void* stream);

/* Runs the operator with weights prepared earlier by mhcPrePrepareWeights into
 * the same workspace (relaunching the same executor, probe_e1e2.cpp:312-318). */
MHC_API int mhcPreRunPrepared(const mhcPreDesc_t* desc, const void* x, const float* alpha, const float* bias,
                              void* hIn, float* hPost, float* hRes, void* workspace, size_t workspaceBytes,
                              void* stream);

/* mhcPreRunPrepared that also records two caller-created CUDA events (cudaEvent_t
 * passed as void*, either may be NULL) on the stream immediately before and after
 * the operator's main kernel, so a caller can time that kernel alone inside a
 * longer loop.  Profiling aid; no reference counterpart. */
MHC_API int mhcPreRunPreparedProfiled(const mhcPreDesc_t* desc, const void* x, const float* alpha, const float* bias,
                                      void* hIn, float* hPost, float* hRes, void* workspace, size_t workspaceBytes,
                                      void* stream, void* mainKernelBegin, void* mainKernelEnd);

/* Size of the library's fixed device scratch area used by mhcPreRunNoAlloc. */
#define MHC_PRE_NOALLOC_SCRATCH_BYTES (96u * 1024u * 1024u)

/* mhcPreRun for callers that cannot allocate device memory while they run: a
 * plugin handed only its tensors' device pointers and no allocator, a serving
 * runtime whose device memory is planned and locked before traffic starts, or a
 * latency-critical loop that must not call cudaMalloc (it can synchronize the
 * device).  Same inputs, outputs and results as mhcPreRun, but no workspace
 * argument: the prepared weights and the split-K partial records live in one
 * 96 MiB array (MHC_PRE_NOALLOC_SCRATCH_BYTES) compiled into the library, which
 * every GPU that loads the library keeps until the process exits.  A problem
 * whose mhcPreGetWorkspaceSize exceeds that size is rejected with
 * MHC_STATUS_TOO_LARGE before anything runs (config 4, M = 65536, n = 4,
 * D = 7168, needs 65.6 MiB and fits).  The call itself allocates nothing: no
 * cudaMalloc, no cudaFree, no allocating library routine.  The first call on a
 * device looks up that device's copy of the array (cudaGetSymbolAddress, which
 * may load the library's device code); make that first call before any stream
 * capture.  The address is kept for the rest of the process: after
 * cudaDeviceReset (or any other teardown of the device's primary context) the
 * library's device code is loaded anew and the kept address is stale, so do not
 * call this entry point again in that process after a reset.  All calls on a device share the one array and it keeps the last
 * call's contents, so calls that can overlap on the GPU (different streams or
 * host threads without ordering between them) race and corrupt each other:
 * issue them in order, for example on one stream.  No counterpart in the
 * reference. */
MHC_API int mhcPreRunNoAlloc(const mhcPreDesc_t* desc, const void* x, const float* phi, const float* alpha,
                             const float* bias, const float* gamma, void* hIn, float* hPost, float* hRes,
                             void* stream);

/* Execution plan chosen for a description on the current device (for tests,
 * benchmarks and profiling; no reference counterpart). */
typedef struct {
    int32_t path;           /* 0 = split-K GEMM + epilogue kernels, 1 = fused team kernel
                               (opt-in), 2 = single-launch decode kernel (M <= 16),
                               3 = cluster-team kernel (opt-in), 4 = single-launch
                               small-batch kernel (16 < M <= 384), 5 = one-pass
                               kernel (x read from HBM once) */
    int32_t kernelsPerRun;  /* kernels launched by mhcPreRunPrepared */
    int32_t gridCtas;       /* CTAs of the main kernel */
    int32_t splits;         /* K splits (paths 0, 2 and 4) or team size (paths 1 and 3) */
    int32_t rowsPerTile;    /* token rows per tensor-core tile */
    int32_t reserved[3];
} mhcPrePlan_t;

MHC_API int mhcPreQueryPlan(const mhcPreDesc_t* desc, mhcPrePlan_t* plan);

/* Plan options: an explicit override of the launch plan, for tests, benchmarks
 * and profiling.  The entry points above never take options, and the library
 * reads no environment variables, so their plan depends only on the description
 * and the device.  In the struct, every field at 0 keeps the library's own choice,
 * except path, whose default is MHC_PRE_PATH_AUTO.  Options that change the K
 * splits change the order of the fp32 sums and so the last bits of the results;
 * the default plan's results are the ones the parity tests pin.  No reference
 * counterpart (the reference's tiling is fixed by TilingFunc,
 * code/op_host/mhc_pre.cpp:123-190). */
#define MHC_PRE_PATH_AUTO (-1)
typedef struct {
    int32_t path;          /* MHC_PRE_PATH_AUTO, or a path number of mhcPrePlan_t to use
                              where it applies: 0 split-K (any shape); 1 fused team
                              (D % 64 == 0); 2 decode (M <= 32); 3 cluster team
                              (D/64 a multiple of 8); 4 small batch (M <= 512); 5 one
                              pass (n = 4).  A path that does not apply falls back to
                              split-K. */
    int32_t splits;        /* split-K and one-pass paths: K splits */
    int32_t gemmCtasPerSm; /* split-K and one-pass paths: GEMM CTAs per SM (capped by
                              TMEM, registers and shared memory; one pass: 2 or 3) */
    int32_t gemmStages;    /* split-K and one-pass paths: pipeline depth (2 or more) */
    int32_t tmaBatch;      /* split-K and one-pass paths: chunks the TMA producer issues per batch */
    int32_t teamSize;      /* fused team path: CTAs per team (divides D/64, 8..64) */
    int32_t clusterLead;   /* cluster path: chunks the first read may run ahead of the re-read */
    int32_t l2Hint;        /* fused and cluster paths: 1 + L2 hint mode (mode 0: none;
                              1: first read evict_last, re-read evict_first, the default;
                              2: re-read evict_first only) */
    int32_t ringTiles;     /* one-pass path: tile slots of the partial-record ring */
    int32_t pairedGemm;    /* split-K path at n = 8: 0 the library's choice, 1 one-CTA GEMM,
                              2 GEMM on CTA pairs (one M = 256 tcgen05 MMA per pair) */
    int32_t epiBlocks;     /* split-K path: epilogue rows resident per SM, 0 the library's
                              choice (16 up to 16384 rows, else 12), 12 or 16 */
    int32_t reserved[5];   /* must be 0 */
} mhcPrePlanOptions_t;

/* mhcPreGetWorkspaceSize / mhcPreQueryPlan / mhcPrePrepareWeights /
 * mhcPreRunPreparedProfiled under plan options (options may be NULL: the default
 * plan).  A workspace prepared under one set of options may be run under another
 * as long as it is large enough for both. */
MHC_API int mhcPreGetWorkspaceSizeEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options,
                                     size_t* workspaceBytes);
MHC_API int mhcPreQueryPlanEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, mhcPrePlan_t* plan);
MHC_API int mhcPrePrepareWeightsEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, const float* phi,
                                   const float* gamma, void* workspace, size_t workspaceBytes, void* stream);
MHC_API int mhcPreRunPreparedEx(const mhcPreDesc_t* desc, const mhcPrePlanOptions_t* options, const void* x,
                                const float* alpha, const float* bias, void* hIn, float* hPost, float* hRes,
                                void* workspace, size_t workspaceBytes, void* stream, void* mainKernelBegin,
                                void* mainKernelEnd);

/* Reads and clears the device-side error word of the current device (set when
 * a kernel gave up a bounded wait).  Synchronizes the current device.
 * *deviceStatus receives 0 or a negative mhcStatus_t.  After
 * MHC_STATUS_DEVICE_TIMEOUT the outputs of the calls since the last read are
 * invalid, and the workspace's weights must be prepared again
 * (mhcPrePrepareWeights) before the next call on it. */
MHC_API int mhcPreGetDeviceStatus(int32_t* deviceStatus);

/* Diagnostics for failure detection: launches one kernel that waits, with a limit
 * of limitMicroseconds (1 .. 1e6), on a global counter that nothing increments and
 * on an mbarrier that nothing arrives on -- the two kinds of bounded wait the
 * kernels use.  Both waits give up; the kernel sets the device status word to
 * MHC_STATUS_DEVICE_TIMEOUT (read it with mhcPreGetDeviceStatus) and returns
 * normally, leaving the context usable.  *countersGaveUp / *barriersGaveUp receive
 * 1 where the wait gave up.  Synchronizes the stream.  No reference counterpart. */
MHC_API int mhcPreDiagWaitTimeout(uint32_t limitMicroseconds, int32_t* countersGaveUp, int32_t* barriersGaveUp,
                                  void* stream);

/* The mHC post step that follows MhcPre in a layer: once the layer has turned
 * hIn into its output y, the residual streams advance as
 *     xNext[m][s][:] = sum_t hRes[m][s][t] * x[m][t][:] + hPost[m][s] * y[m][:]
 * with x [B,S,n,D] and y [B,S,D] in the description's 16-bit dtype, hPost [B,S,n]
 * and hRes [B,S,n,n] fp32 (as mhcPreRun writes them) and xNext [B,S,n,D] in the x
 * dtype.  Arithmetic: fp32, the first stream's term a rounded product, each
 * further term (streams in order, then y) one fused multiply-add, one
 * round-to-nearest-even at the end.  xNext may be x itself (in place); y must not
 * overlap xNext.  The description's gamma flag and eps values are ignored.  Needs
 * no workspace and allocates nothing; asynchronous on the stream.  The reference
 * has no code for this step (it stops at hIn/hPost/hRes), so there is no
 * counterpart to cite and its results are checked against this library's own C
 * restatement. */
MHC_API int mhcPostRun(const mhcPreDesc_t* desc, const void* x, const void* y, const float* hPost,
                       const float* hRes, void* xNext, void* stream);

/* The post step of one layer fused with the next layer's MhcPre.  A layer ends
 * with mhcPostRun (xNext from x, the layer output y, hPost and hRes) and the next
 * layer begins with MhcPre on xNext, whose first pass reads xNext back from
 * memory.  This call forms xNext and that pass together, so xNext is written once
 * and read once (by the pass that forms hIn) instead of written once and read
 * twice: 22% less memory traffic for the pair of steps at n = 4.
 * desc describes the next MhcPre (its shape is the post step's too; its hasGamma
 * and eps values are the next layer's).  x, y, hPost, hRes and xNext are as for
 * mhcPostRun (xNext may be x; y must not overlap xNext); alpha, bias, hIn,
 * hPostNext, hResNext and the workspace are as for mhcPreRunPrepared, with the next
 * layer's weights prepared in the workspace (mhcPrePrepareWeights), which must be
 * at least mhcPreGetWorkspaceSize(desc) bytes.  Results: xNext bit for bit as
 * mhcPostRun; hIn, hPostNext and hResNext as mhcPreRunPrepared on that xNext,
 * within the parity tolerances (the fused pass splits K differently).  The fused
 * kernel applies for n = 4, headDim a multiple of 64, and more rows than the
 * single-launch paths take (M > 384); otherwise the call runs mhcPostRun and then
 * mhcPreRunPrepared.  No reference counterpart (the reference has no post step). */
MHC_API int mhcPostPreRun(const mhcPreDesc_t* desc, const void* x, const void* y, const float* hPost,
                          const float* hRes, void* xNext, const float* alpha, const float* bias, void* hIn,
                          float* hPostNext, float* hResNext, void* workspace, size_t workspaceBytes, void* stream);

/* Human-readable name of a status code (static string). */
MHC_API const char* mhcPreStatusString(int status);

/* MHC_PRE_ABI_VERSION of the loaded library. */
MHC_API int mhcPreAbiVersion(void);

#ifdef __cplusplus
}
#endif
#endif /* MHC_PRE_H */
