/* A plain C99 consumer of the MhcPre C ABI (include/mhc_pre.h), the way a host
 * program that called the reference's aclnnMhcPreGetWorkspaceSize / aclnnMhcPre
 * pair would call this library.  Test program: it links the CPU oracle
 * (oracle/mhc_pre_oracle.h) only to check the results.
 *
 *   consumer --no-gpu   ABI version, status strings and the shape rejects, which
 *                       need no device
 *   consumer            on a B200: one-shot and prepared runs of a split-K, a
 *                       small-batch and a decode shape, and the post step fused with
 *                       the next MhcPre (mhcPostPreRun) on each, compared with the
 *                       oracle on the same inputs
 * Exit status 0 when every check passes. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "mhc_pre.h"
#include "mhc_pre_oracle.h"

static int failures = 0;
#define CHECK(cond, ...)                           \
    do {                                           \
        if (!(cond)) {                             \
            fprintf(stderr, "FAIL: " __VA_ARGS__); \
            fprintf(stderr, "\n");                 \
            ++failures;                            \
        }                                          \
    } while (0)

static mhcPreDesc_t desc(int64_t B, int64_t S, int64_t n, int64_t D, int32_t dtype, int32_t gamma) {
    mhcPreDesc_t d;
    memset(&d, 0, sizeof(d));
    d.batch = B;
    d.seq = S;
    d.streams = n;
    d.headDim = D;
    d.dtype = dtype;
    d.hasGamma = gamma;
    d.normEps = 1e-6f;
    d.hcEps = 1e-6f;
    return d;
}

static void no_gpu_checks(void) {
    size_t ws = 0;
    CHECK(mhcPreAbiVersion() == MHC_PRE_ABI_VERSION, "ABI version");
    CHECK(mhcPreStatusString(MHC_STATUS_SUCCESS) != NULL, "status string");
    mhcPreDesc_t d = desc(1, 8, 5, 256, MHC_DTYPE_BF16, 1);
    CHECK(mhcPreGetWorkspaceSize(&d, &ws) == MHC_STATUS_BAD_STREAM_COUNT, "n=5 rejected");
    d = desc(1, 8, 4, 20, MHC_DTYPE_BF16, 1);
    CHECK(mhcPreGetWorkspaceSize(&d, &ws) == MHC_STATUS_BAD_HEAD_DIM, "D=20 rejected");
    d = desc(0, 8, 4, 256, MHC_DTYPE_BF16, 1);
    CHECK(mhcPreGetWorkspaceSize(&d, &ws) == MHC_STATUS_BAD_SHAPE, "B=0 rejected");
    d = desc(1, 8, 4, 256, 7, 1);
    CHECK(mhcPreGetWorkspaceSize(&d, &ws) == MHC_STATUS_BAD_DTYPE, "dtype rejected");
    CHECK(mhcPreGetWorkspaceSize(NULL, &ws) == MHC_STATUS_NULL_POINTER, "null desc rejected");
}

/* deterministic inputs: a 64-bit LCG and Box-Muller */
static uint64_t lcg_state = 12345;
static double uniform01(void) {
    lcg_state = lcg_state * 6364136223846793005ull + 1442695040888963407ull;
    return ((lcg_state >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
static float normal(void) {
    const double u = uniform01(), v = uniform01();
    return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

static int ulp_distance(uint16_t a, uint16_t b) {
    const int ma = a & 0x7FFF, mb = b & 0x7FFF;
    const int oa = (a & 0x8000) ? -ma : ma, ob = (b & 0x8000) ? -mb : mb;
    return abs(oa - ob);
}

static void check_outputs(int64_t M, int64_t n, int64_t D, const uint16_t* hin, const float* post, const float* res,
                          const uint16_t* rin, const float* rpost, const float* rres, const char* what, int path) {
    double err = 0.0;
    for (int64_t i = 0; i < M * n; ++i) err = fmax(err, fabs(post[i] - rpost[i]) / fmax(1.0, fabs(rpost[i])));
    for (int64_t i = 0; i < M * n * n; ++i) err = fmax(err, fabs(res[i] - rres[i]) / fmax(1.0, fabs(rres[i])));
    int64_t within1 = 0;
    for (int64_t i = 0; i < M * D; ++i) within1 += ulp_distance(hin[i], rin[i]) <= 1;
    const double frac = (double)within1 / (double)(M * D);
    printf("%s M=%lld n=%lld D=%lld path %d: hPost/hRes max rel err %.2e, hIn within 1 ulp %.5f\n", what,
           (long long)M, (long long)n, (long long)D, path, err, frac);
    CHECK(err <= 1e-4, "%s: hPost/hRes error %.3e", what, err);
    CHECK(frac >= 0.999, "%s: hIn within 1 ulp %.5f", what, frac);
}

static void run_case(int64_t S, int64_t n, int64_t D, int32_t dtype, int32_t gamma) {
    const int64_t M = S, K = n * D, mix = n * n + 2 * n;
    uint16_t* x = malloc(sizeof(uint16_t) * M * K);
    float* phi = malloc(sizeof(float) * mix * K);
    float* g = malloc(sizeof(float) * K);
    float alpha[3], bias[80];
    for (int64_t i = 0; i < M * K; ++i)
        x[i] = dtype == MHC_DTYPE_BF16 ? mhc_oracle_f32_to_bf16(normal()) : mhc_oracle_f32_to_f16(normal());
    for (int64_t i = 0; i < mix * K; ++i) phi[i] = 0.02f * normal();
    for (int64_t i = 0; i < K; ++i) g[i] = 1.0f + 0.05f * normal();
    for (int i = 0; i < 3; ++i) alpha[i] = 0.5f + (float)uniform01();
    for (int64_t i = 0; i < mix; ++i) bias[i] = 0.1f * normal();

    mhcPreDesc_t d = desc(1, S, n, D, dtype, gamma);
    size_t wsBytes = 0;
    CHECK(mhcPreGetWorkspaceSize(&d, &wsBytes) == MHC_STATUS_SUCCESS, "workspace size");
    void *dx, *dphi, *dg, *dalpha, *dbias, *dhin, *dpost, *dres, *dws;
    cudaMalloc(&dx, sizeof(uint16_t) * M * K);
    cudaMalloc(&dphi, sizeof(float) * mix * K);
    cudaMalloc(&dg, sizeof(float) * K);
    cudaMalloc(&dalpha, sizeof(alpha));
    cudaMalloc(&dbias, sizeof(float) * mix);
    cudaMalloc(&dhin, sizeof(uint16_t) * M * D);
    cudaMalloc(&dpost, sizeof(float) * M * n);
    cudaMalloc(&dres, sizeof(float) * M * n * n);
    cudaMalloc(&dws, wsBytes);
    cudaMemcpy(dx, x, sizeof(uint16_t) * M * K, cudaMemcpyHostToDevice);
    cudaMemcpy(dphi, phi, sizeof(float) * mix * K, cudaMemcpyHostToDevice);
    cudaMemcpy(dg, g, sizeof(float) * K, cudaMemcpyHostToDevice);
    cudaMemcpy(dalpha, alpha, sizeof(alpha), cudaMemcpyHostToDevice);
    cudaMemcpy(dbias, bias, sizeof(float) * mix, cudaMemcpyHostToDevice);

    /* one shot: prepare + run on the default stream */
    int rc = mhcPreRun(&d, dx, dphi, dalpha, dbias, gamma ? dg : NULL, dhin, dpost, dres, dws, wsBytes, NULL);
    CHECK(rc == MHC_STATUS_SUCCESS, "mhcPreRun: %s", mhcPreStatusString(rc));
    cudaDeviceSynchronize();
    uint16_t* hin = malloc(sizeof(uint16_t) * M * D);
    float* post = malloc(sizeof(float) * M * n);
    float* res = malloc(sizeof(float) * M * n * n);
    cudaMemcpy(hin, dhin, sizeof(uint16_t) * M * D, cudaMemcpyDeviceToHost);
    cudaMemcpy(post, dpost, sizeof(float) * M * n, cudaMemcpyDeviceToHost);
    cudaMemcpy(res, dres, sizeof(float) * M * n * n, cudaMemcpyDeviceToHost);

    /* prepared executor, relaunched: bitwise equal to the one-shot call */
    CHECK(mhcPreRunPrepared(&d, dx, dalpha, dbias, dhin, dpost, dres, dws, wsBytes, NULL) == MHC_STATUS_SUCCESS,
          "mhcPreRunPrepared");
    cudaDeviceSynchronize();
    uint16_t* hin2 = malloc(sizeof(uint16_t) * M * D);
    cudaMemcpy(hin2, dhin, sizeof(uint16_t) * M * D, cudaMemcpyDeviceToHost);
    CHECK(memcmp(hin, hin2, sizeof(uint16_t) * M * D) == 0, "relaunch bitwise equal");
    int32_t devStatus = -1;
    CHECK(mhcPreGetDeviceStatus(&devStatus) == MHC_STATUS_SUCCESS && devStatus == 0, "device status %d", devStatus);
    mhcPrePlan_t plan;
    CHECK(mhcPreQueryPlan(&d, &plan) == MHC_STATUS_SUCCESS, "plan");

    /* the CPU oracle on the same inputs */
    uint16_t* rin = malloc(sizeof(uint16_t) * M * D);
    float* rpost = malloc(sizeof(float) * M * n);
    float* rres = malloc(sizeof(float) * M * n * n);
    CHECK(mhc_pre_oracle(M, (int)n, D, dtype == MHC_DTYPE_BF16 ? MHC_ORACLE_BF16 : MHC_ORACLE_F16,
                         MHC_ORACLE_ORDER_KERNEL, x, phi, alpha, bias, gamma ? g : NULL, 1e-6f, 1e-6f, rin, rpost,
                         rres, 0, M, 0) == 0,
          "oracle");
    check_outputs(M, n, D, hin, post, res, rin, rpost, rres, "mhcPreRun", plan.path);

    /* a layer boundary: the post step with this call's hPost/hRes and a layer output y,
       fused with the next MhcPre on the same prepared weights (mhcPostPreRun); the
       oracle runs the post step (bit for bit) and then MhcPre on its xNext */
    const int odt = dtype == MHC_DTYPE_BF16 ? MHC_ORACLE_BF16 : MHC_ORACLE_F16;
    uint16_t* y = malloc(sizeof(uint16_t) * M * D);
    for (int64_t i = 0; i < M * D; ++i)
        y[i] = dtype == MHC_DTYPE_BF16 ? mhc_oracle_f32_to_bf16(normal()) : mhc_oracle_f32_to_f16(normal());
    void *dy, *dxn, *dhin2, *dpost2, *dres2;
    cudaMalloc(&dy, sizeof(uint16_t) * M * D);
    cudaMalloc(&dxn, sizeof(uint16_t) * M * K);
    cudaMalloc(&dhin2, sizeof(uint16_t) * M * D);
    cudaMalloc(&dpost2, sizeof(float) * M * n);
    cudaMalloc(&dres2, sizeof(float) * M * n * n);
    cudaMemcpy(dy, y, sizeof(uint16_t) * M * D, cudaMemcpyHostToDevice);
    rc = mhcPostPreRun(&d, dx, dy, dpost, dres, dxn, dalpha, dbias, dhin2, dpost2, dres2, dws, wsBytes, NULL);
    CHECK(rc == MHC_STATUS_SUCCESS, "mhcPostPreRun: %s", mhcPreStatusString(rc));
    cudaDeviceSynchronize();
    CHECK(mhcPreGetDeviceStatus(&devStatus) == MHC_STATUS_SUCCESS && devStatus == 0, "device status %d", devStatus);
    uint16_t* xn = malloc(sizeof(uint16_t) * M * K);
    uint16_t* rxn = malloc(sizeof(uint16_t) * M * K);
    cudaMemcpy(xn, dxn, sizeof(uint16_t) * M * K, cudaMemcpyDeviceToHost);
    cudaMemcpy(hin2, dhin2, sizeof(uint16_t) * M * D, cudaMemcpyDeviceToHost);
    float* post2 = malloc(sizeof(float) * M * n);
    float* res2 = malloc(sizeof(float) * M * n * n);
    cudaMemcpy(post2, dpost2, sizeof(float) * M * n, cudaMemcpyDeviceToHost);
    cudaMemcpy(res2, dres2, sizeof(float) * M * n * n, cudaMemcpyDeviceToHost);
    CHECK(mhc_post_oracle(M, (int)n, D, odt, x, y, post, res, rxn, 0) == 0, "post oracle");
    CHECK(memcmp(xn, rxn, sizeof(uint16_t) * M * K) == 0, "mhcPostPreRun: xNext equals the post oracle bit for bit");
    CHECK(mhc_pre_oracle(M, (int)n, D, odt, MHC_ORACLE_ORDER_KERNEL, rxn, phi, alpha, bias, gamma ? g : NULL, 1e-6f,
                         1e-6f, rin, rpost, rres, 0, M, 0) == 0,
          "oracle on xNext");
    check_outputs(M, n, D, hin2, post2, res2, rin, rpost, rres, "mhcPostPreRun", plan.path);
    free(y); free(xn); free(rxn); free(post2); free(res2);
    cudaFree(dy); cudaFree(dxn); cudaFree(dhin2); cudaFree(dpost2); cudaFree(dres2);

    cudaFree(dx); cudaFree(dphi); cudaFree(dg); cudaFree(dalpha); cudaFree(dbias);
    cudaFree(dhin); cudaFree(dpost); cudaFree(dres); cudaFree(dws);
    free(x); free(phi); free(g); free(hin); free(hin2); free(post); free(res); free(rin); free(rpost); free(rres);
}

int main(int argc, char** argv) {
    no_gpu_checks();
    if (!(argc > 1 && strcmp(argv[1], "--no-gpu") == 0)) {
        run_case(700, 4, 256, MHC_DTYPE_BF16, 1);  /* split-K path, ragged last tile */
        run_case(300, 4, 256, MHC_DTYPE_BF16, 1);  /* small-batch path, ragged last tile */
        run_case(5, 8, 512, MHC_DTYPE_F16, 0);     /* decode path */
    }
    printf("%s (%d failures)\n", failures ? "FAILED" : "OK", failures);
    return failures ? 1 : 0;
}
