/*
 * CPU oracle for MhcPre -- TEST INFRASTRUCTURE ONLY (see mhc_pre_oracle.h).
 *
 * Built with -O3 -ffp-contract=off -fopenmp: every multiply and add below is a
 * separately rounded IEEE fp32 operation unless a double is named explicitly.
 */
#include "mhc_pre_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f32_bits(float v) { uint32_t b; memcpy(&b, &v, 4); return b; }
static inline float bits_f32(uint32_t b) { float v; memcpy(&v, &b, 4); return v; }

/* fp32 -> fp16 bits, IEEE round to nearest even (subnormals, overflow to inf;
 * NaN keeps a quiet payload bit of 1).  `audit_carry` reproduces a quirk of the
 * reference's helper (audit_group_vec.py:181, cloud_runner/runner.cpp:85): it
 * masks the rounded subnormal with 0x3FF, so a value just below the smallest
 * normal (2^-14) that rounds up to it becomes 0 instead of 2^-14. */
static uint16_t f32_to_f16_impl(float value, int audit_carry)
{
    const uint32_t v = f32_bits(value);
    const uint32_t sign = (v >> 16) & 0x8000u;
    const uint32_t exp = (v >> 23) & 0xFFu;
    const uint32_t mant = v & 0x7FFFFFu;
    if (exp == 0xFFu) {
        return (uint16_t)(sign | 0x7C00u | (mant ? 1u : 0u));
    }
    int32_t e16 = (int32_t)exp - 127 + 15;
    if (e16 >= 0x1F) {
        return (uint16_t)(sign | 0x7C00u);
    }
    if (e16 <= 0) {
        const int shift = 14 - e16;
        if (shift >= 25) {
            return (uint16_t)sign;
        }
        const uint32_t m = mant | 0x800000u;
        uint32_t half = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t tie = 1u << (shift - 1);
        if (rem > tie || (rem == tie && (half & 1u))) {
            half++;
        }
        return (uint16_t)(sign | (audit_carry ? (half & 0x3FFu) : half));
    }
    uint32_t m16 = mant >> 13;
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (m16 & 1u))) {
        m16++;
        if (m16 == 0x400u) {
            m16 = 0;
            e16++;
        }
    }
    if (e16 >= 0x1F) {
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | ((uint32_t)e16 << 10) | m16);
}

uint16_t mhc_oracle_f32_to_f16(float value) { return f32_to_f16_impl(value, 0); }
uint16_t mhc_oracle_f32_to_f16_audit(float value) { return f32_to_f16_impl(value, 1); }

/* fp32 -> bf16 bits: add 0x7FFF plus the kept LSB, truncate
 * (audit_group_vec.py:209-213, cloud_runner/runner.cpp:102-108). */
uint16_t mhc_oracle_f32_to_bf16(float value)
{
    const uint32_t v = f32_bits(value);
    const uint32_t lsb = (v >> 16) & 1u;
    return (uint16_t)(((v + 0x7FFFu + lsb) & 0xFFFF0000u) >> 16);
}

float mhc_oracle_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (h >> 15) & 1u;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    uint32_t out;
    if (exp == 0x1Fu) {
        out = (sign << 31) | 0x7F800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            out = sign << 31;
        } else {
            /* subnormal: value = mant * 2^-24, exact in fp32 */
            const float f = (float)mant * 5.9604644775390625e-8f;
            return sign ? -f : f;
        }
    } else {
        out = (sign << 31) | ((exp - 15u + 127u) << 23) | (mant << 13);
    }
    return bits_f32(out);
}

float mhc_oracle_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

int mhc_oracle_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static inline float load_x(const uint16_t *p, int dtype)
{
    return dtype == MHC_ORACLE_BF16 ? mhc_oracle_bf16_to_f32(*p) : mhc_oracle_f16_to_f32(*p);
}

static inline uint16_t store_x(float v, int dtype, int order)
{
    if (dtype == MHC_ORACLE_BF16) {
        return mhc_oracle_f32_to_bf16(v);
    }
    return order == MHC_ORACLE_ORDER_AUDIT ? mhc_oracle_f32_to_f16_audit(v) : mhc_oracle_f32_to_f16(v);
}

/* The Ascend kernel's vector tile for the square-sum (code/op_host/mhc_pre.cpp:11). */
#define ORACLE_SUM_TILE 512

int mhc_pre_oracle(int64_t M, int n, int64_t D, int dtype, int order,
                   const uint16_t *x, const float *phi, const float *alpha,
                   const float *bias, const float *gamma, float norm_eps, float hc_eps,
                   uint16_t *hIn, float *hPost, float *hRes,
                   int64_t row_begin, int64_t row_end, int threads)
{
    if (M <= 0 || D <= 0 || (n != 4 && n != 6 && n != 8) || x == NULL || phi == NULL ||
        alpha == NULL || bias == NULL || hIn == NULL || hPost == NULL || hRes == NULL ||
        row_begin < 0 || row_end > M || row_begin > row_end ||
        (dtype != MHC_ORACLE_F16 && dtype != MHC_ORACLE_BF16) ||
        (order != MHC_ORACLE_ORDER_KERNEL && order != MHC_ORACLE_ORDER_AUDIT)) {
        return -1;
    }
    const int64_t K = (int64_t)n * D;
    const int mix = n * n + 2 * n;

    /* phi transposed to [K][mix] so the inner loop runs over the mix outputs; the
     * per-output accumulation order over k stays sequential. */
    float *phiT = (float *)malloc(sizeof(float) * (size_t)K * (size_t)mix);
    if (phiT == NULL) {
        return -2;
    }
    for (int j = 0; j < mix; ++j) {
        for (int64_t k = 0; k < K; ++k) {
            phiT[k * mix + j] = phi[(int64_t)j * K + k];
        }
    }
    const float inv_flat = 1.0f / (float)K; /* host invFlatDim, code/op_host/mhc_pre.cpp:154 */
    int failed = 0;

#ifdef _OPENMP
    if (threads > 0) {
        omp_set_num_threads(threads);
    }
#else
    (void)threads;
#endif

#pragma omp parallel
    {
        float *xf = (float *)malloc(sizeof(float) * (size_t)K);
        float *xg = (float *)malloc(sizeof(float) * (size_t)K);
        if (xf == NULL || xg == NULL) {
#pragma omp atomic write
            failed = 1;
        }
#pragma omp for schedule(dynamic, 4)
        for (int64_t r = row_begin; r < row_end; ++r) {
            if (xf == NULL || xg == NULL) {
                continue;
            }
            const uint16_t *xr = x + r * K;
            for (int64_t k = 0; k < K; ++k) {
                xf[k] = load_x(xr + k, dtype);
            }

            /* 1. inverse RMS over the raw x (before gamma). */
            float inv_rms;
            if (order == MHC_ORACLE_ORDER_KERNEL) {
                float row_sum = 0.0f;
                for (int64_t t0 = 0; t0 < K; t0 += ORACLE_SUM_TILE) {
                    const int64_t t1 = (t0 + ORACLE_SUM_TILE < K) ? t0 + ORACLE_SUM_TILE : K;
                    float tile = 0.0f;
                    for (int64_t k = t0; k < t1; ++k) {
                        const float sq = xf[k] * xf[k];
                        tile = tile + sq;
                    }
                    row_sum = row_sum + tile;
                }
                float v = row_sum * inv_flat;
                v = v + norm_eps;
                v = sqrtf(v);
                inv_rms = 1.0f / v;
            } else {
                float row_sum = 0.0f;
                for (int64_t k = 0; k < K; ++k) {
                    const float sq = xf[k] * xf[k];
                    row_sum = row_sum + sq;
                }
                const float t = row_sum * inv_flat;
                const float u = (float)((double)t + 1.0e-6); /* audit adds the double norm_eps */
                inv_rms = (float)(1.0 / sqrt((double)u));
                (void)norm_eps;
            }

            /* 2. gamma */
            for (int64_t k = 0; k < K; ++k) {
                xg[k] = gamma ? xf[k] * gamma[k] : xf[k];
            }

            /* 3. mix = xg . phi^T, sequential fp32 accumulation over k */
            float acc[80];
            for (int j = 0; j < mix; ++j) {
                acc[j] = 0.0f;
            }
            for (int64_t k = 0; k < K; ++k) {
                const float a = xg[k];
                const float *prow = phiT + k * mix;
                for (int j = 0; j < mix; ++j) {
                    const float p = a * prow[j];
                    acc[j] = acc[j] + p;
                }
            }

            /* 4-6. epilogue */
            float pre[8];
            if (order == MHC_ORACLE_ORDER_KERNEL) {
                const float s_pre = inv_rms * alpha[0];
                const float s_post = inv_rms * alpha[1];
                const float s_res = inv_rms * alpha[2];
                for (int s = 0; s < n; ++s) {
                    float v = acc[s] * s_pre;
                    v = v + bias[s];
                    v = v * -1.0f;
                    v = expf(v);
                    v = v + 1.0f;
                    v = 1.0f / v;
                    pre[s] = v + hc_eps;

                    float w = acc[n + s] * s_post;
                    w = w + bias[n + s];
                    w = w * -1.0f;
                    w = expf(w);
                    w = w + 1.0f;
                    w = 1.0f / w;
                    hPost[r * n + s] = w * 2.0f;
                }
                for (int i = 0; i < n * n; ++i) {
                    const float v = acc[2 * n + i] * s_res;
                    hRes[r * n * n + i] = v + bias[2 * n + i];
                }
            } else {
                for (int j = 0; j < mix; ++j) {
                    acc[j] = acc[j] * inv_rms;
                }
                for (int s = 0; s < n; ++s) {
                    const float wp = acc[s] * alpha[0];
                    const float w_pre = wp + bias[s];
                    const double sig = 1.0 / (1.0 + exp(-(double)w_pre));
                    pre[s] = (float)(sig + 1.0e-6); /* audit adds the double hc_eps */
                    const float wq = acc[n + s] * alpha[1];
                    const float w_post = wq + bias[n + s];
                    const double sig2 = 1.0 / (1.0 + exp(-(double)w_post));
                    hPost[r * n + s] = (float)(2.0 * sig2);
                }
                for (int i = 0; i < n * n; ++i) {
                    const float v = acc[2 * n + i] * alpha[2];
                    hRes[r * n * n + i] = v + bias[2 * n + i];
                }
                (void)hc_eps;
            }

            /* 7. hIn from the raw x, stream order 0..n-1, separate mul and add */
            for (int64_t d = 0; d < D; ++d) {
                float a;
                if (order == MHC_ORACLE_ORDER_KERNEL) {
                    a = xf[d] * pre[0];
                    for (int s = 1; s < n; ++s) {
                        const float p = xf[(int64_t)s * D + d] * pre[s];
                        a = a + p;
                    }
                } else {
                    a = 0.0f;
                    for (int s = 0; s < n; ++s) {
                        const float p = pre[s] * xf[(int64_t)s * D + d];
                        a = a + p;
                    }
                }
                hIn[r * D + d] = store_x(a, dtype, order);
            }
        }
        free(xf);
        free(xg);
    }
    free(phiT);
    return failed ? -2 : 0;
}

/* Inputs of the reference's E3 shape-matrix runner, drawn with the C library's
 * rand() exactly as cloud_runner/runner.cpp:370-382 does after srand(seed):
 * x, then phi ([mix][K] order), then bias, then gamma (always drawn). */
void mhc_oracle_runner_inputs(unsigned seed, int64_t nx, int64_t nphi, int64_t nbias, int64_t ngamma,
                              float *x, float *phi, float *bias, float *gamma)
{
    srand(seed);
    for (int64_t i = 0; i < nx; ++i) {
        x[i] = (float)(rand() % 2000) / 10000.0f - 0.1f;
    }
    for (int64_t i = 0; i < nphi; ++i) {
        phi[i] = (float)(rand() % 200) / 10000.0f - 0.01f;
    }
    for (int64_t i = 0; i < nbias; ++i) {
        bias[i] = (float)(rand() % 200) / 10000.0f - 0.01f;
    }
    for (int64_t i = 0; i < ngamma; ++i) {
        gamma[i] = 1.0f + (float)(rand() % 200) / 10000.0f;
    }
}
