/*
 * CPU oracle for the MhcPre operator -- TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker for the CUDA path: only tests/, the smoke()
 * entry and bench.py's CPU-baseline leg may load it.  The product path never
 * calls it and has no CPU fallback.
 *
 * It restates the reference operator (ZXY-0508/MhcPre-review) in plain C with
 * fp32 arithmetic and no FMA contraction (built with -ffp-contract=off):
 *
 *   invRms[r] = 1 / sqrt(sum_k x[r,k]^2 * (1/K) + normEps)      (raw x, before gamma)
 *   mix[r,j]  = sum_k (x[r,k]*gamma[k]) * phi[j,k]              (phi stored [mix][K])
 *   hPre      = sigmoid(mix*invRms*alpha[0] + bias[s]) + hcEps  (internal only)
 *   hPost     = 2*sigmoid(mix*invRms*alpha[1] + bias[n+s])
 *   hRes      = mix*invRms*alpha[2] + bias[2n+i]                (linear, no sigmoid)
 *   hIn[r,d]  = RN_dtype(((hPre0*x0 + hPre1*x1) + hPre2*x2) + ...)
 *
 * Two rounding orders are provided, both taken from the reference:
 *   MHC_ORACLE_ORDER_KERNEL  follows code/op_kernel/mhc_pre.cpp:
 *       sum of squares per 512-element tile then across tiles (:458-497),
 *       invRms = 1/Sqrt(sum*invFlatDim + normEps) in fp32 (:504-519),
 *       scale = invRms*alpha then mix*scale (:736-747), sigmoid as
 *       Muls/Add/Muls(-1)/Exp/Adds(1)/Div/Adds(eps) (:542-555),
 *       hIn = Brcb mul then (x0+x1)+x2... (:91-222, :793-812).
 *   MHC_ORACLE_ORDER_AUDIT   follows audit_group_vec.py:279-324 exactly
 *       (sequential fp32 square-sum, double sqrt/exp/eps adds, (mix*invRms)*alpha,
 *       the helper's fp16 subnormal-carry quirk); it reproduces the audit's
 *       outputs bit for bit.
 * The GEMM accumulates sequentially over k in fp32 in both orders
 * (audit_group_vec.py:243-252; cloud_runner/runner.cpp:155-158).
 */
#ifndef MHC_PRE_ORACLE_H
#define MHC_PRE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { MHC_ORACLE_F16 = 0, MHC_ORACLE_BF16 = 1 };
enum { MHC_ORACLE_ORDER_KERNEL = 0, MHC_ORACLE_ORDER_AUDIT = 1 };

/* Runs rows [row_begin, row_end) of an [M, n, D] problem.  x, hIn are 16-bit
 * patterns of the given dtype; phi is [mix][n*D]; gamma may be NULL.
 * Returns 0 on success, negative on bad arguments. threads<=0 uses OpenMP's default. */
int mhc_pre_oracle(int64_t M, int n, int64_t D, int dtype, int order,
                   const uint16_t *x, const float *phi, const float *alpha,
                   const float *bias, const float *gamma, float norm_eps, float hc_eps,
                   uint16_t *hIn, float *hPost, float *hRes,
                   int64_t row_begin, int64_t row_end, int threads);

/* Bit-level conversion helpers (IEEE round to nearest even), the conversions of
 * audit_group_vec.py:162-213 and cloud_runner/runner.cpp:45-116.  The _audit
 * variant keeps the reference helper's subnormal-carry quirk (it maps values
 * that round up to the smallest normal, 2^-14, to zero); the audit order uses
 * it for hIn so that the oracle reproduces the audit bit for bit. */
uint16_t mhc_oracle_f32_to_f16(float v);
uint16_t mhc_oracle_f32_to_f16_audit(float v);
uint16_t mhc_oracle_f32_to_bf16(float v);
float mhc_oracle_f16_to_f32(uint16_t h);
float mhc_oracle_bf16_to_f32(uint16_t b);

/* Inputs of the reference's E3 runner (cloud_runner/runner.cpp:370-382). */
void mhc_oracle_runner_inputs(unsigned seed, int64_t nx, int64_t nphi, int64_t nbias, int64_t ngamma,
                              float *x, float *phi, float *bias, float *gamma);

/* Number of OpenMP threads the oracle would use (for reporting). */
int mhc_oracle_max_threads(void);

/* The mHC post step (mhc_post_oracle.c): xNext[m,s,:] = sum_t hRes[m,s,t]*x[m,t,:]
 * + hPost[m,s]*y[m,:] in the library's operation order (parity unpinned: the
 * reference has no such step).  x, y, xNext are 16-bit patterns of the dtype;
 * xNext must not overlap x or y.  Returns 0, or negative on bad arguments. */
int mhc_post_oracle(int64_t M, int n, int64_t D, int dtype, const uint16_t *x, const uint16_t *y,
                    const float *hPost, const float *hRes, uint16_t *xNext, int threads);

#ifdef __cplusplus
}
#endif
#endif
