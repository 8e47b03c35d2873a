/*
 * CPU oracle for the mHC post step -- TEST INFRASTRUCTURE ONLY (parity unpinned).
 *
 * Like the MhcPre oracle in this directory, only tests/ and bench.py's CPU leg may
 * load it; the product path never calls it.  The reference repository stops at
 * hIn/hPost/hRes and has no code, tests or vectors for the step after the layer,
 * so nothing pins this restatement to it: it states the arithmetic the library
 * defines for mhcPostRun, operation for operation, so that the GPU kernel can be
 * checked bit for bit against it:
 *
 *   xNext[m,s,d] = RN_dtype( fma(hPost[m,s], y[m,d],
 *                      fma(hRes[m,s,n-1], x[m,n-1,d], ...
 *                        fma(hRes[m,s,1], x[m,1,d], hRes[m,s,0]*x[m,0,d]) ...)) )
 *
 * in fp32 (the first term a rounded product, each further term one fused
 * multiply-add, C's fmaf), then one round-to-nearest-even to the x dtype.
 * xNext must not overlap x or y here (the GPU step may run in place; the
 * checker writes a separate buffer).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "mhc_pre_oracle.h"

static inline float post_load(uint16_t b, int dtype)
{
    return dtype == MHC_ORACLE_BF16 ? mhc_oracle_bf16_to_f32(b) : mhc_oracle_f16_to_f32(b);
}

static inline uint16_t post_store(float v, int dtype)
{
    return dtype == MHC_ORACLE_BF16 ? mhc_oracle_f32_to_bf16(v) : mhc_oracle_f32_to_f16(v);
}

int mhc_post_oracle(int64_t M, int n, int64_t D, int dtype, const uint16_t *x, const uint16_t *y,
                    const float *hPost, const float *hRes, uint16_t *xNext, int threads)
{
    if (M < 0 || n <= 0 || D <= 0 || x == NULL || y == NULL || hPost == NULL || hRes == NULL || xNext == NULL) {
        return -1;
    }
    if (dtype != MHC_ORACLE_F16 && dtype != MHC_ORACLE_BF16) {
        return -1;
    }
#ifdef _OPENMP
    if (threads > 0) {
        omp_set_num_threads(threads);
    }
#pragma omp parallel for schedule(static)
#else
    (void)threads;
#endif
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t *xr = x + m * n * D;
        const uint16_t *yr = y + m * D;
        const float *res = hRes + m * n * n;
        const float *post = hPost + m * n;
        uint16_t *out = xNext + m * n * D;
        for (int s = 0; s < n; ++s) {
            for (int64_t d = 0; d < D; ++d) {
                float a = res[s * n] * post_load(xr[d], dtype);
                for (int t = 1; t < n; ++t) {
                    a = fmaf(res[s * n + t], post_load(xr[t * D + d], dtype), a);
                }
                a = fmaf(post[s], post_load(yr[d], dtype), a);
                out[s * D + d] = post_store(a, dtype);
            }
        }
    }
    return 0;
}
