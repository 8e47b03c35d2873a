// The mHC post step (included by mhc_pre_kernels.cu inside namespace mhc, after the
// 16-bit conversion helpers it uses).
//
// After MhcPre has produced hIn, hPost and hRes and the layer has turned hIn into
// its output y, the residual streams advance as
//     xNext[m, s, :] = sum_t hRes[m, s, t] * x[m, t, :] + hPost[m, s] * y[m, :]
// (hRes applied as an n x n mix of the streams, hPost scattering the layer output
// back onto them).  The reference has no code for this step; its arithmetic here is
// fixed as: fp32, the first term a rounded product, every further term (streams in
// order t = 0, 1, ..., then the layer output) one fused multiply-add, and one
// round-to-nearest-even to the x dtype at the end.
//
// The step is a pure stream: per row it reads n*D + D 16-bit values and writes n*D,
// against n*(n+1) multiply-adds per output, so HBM bounds it.  One 128-thread block
// per row stages the row's n*n + n coefficients in shared memory; each thread then
// takes 8-element vectors of the row, loads that vector of all n streams and of y
// (16-byte loads), and writes the vector of all n output streams.  A thread reads
// every input it overwrites before writing, so xNext may be x itself (y must not
// overlap xNext).
#pragma once

constexpr int kPostThreads = 128;

struct PostParams {
    int64_t M;
    int64_t D;
    const uint16_t* x;      // [M][n][D]
    const uint16_t* y;      // [M][D]
    const float* hPost;     // [M][n]
    const float* hRes;      // [M][n][n]
    uint16_t* xNext;        // [M][n][D]
};

template <int DT, int NS>
__global__ void __launch_bounds__(kPostThreads) mhc_post_kernel(const PostParams p) {
    __shared__ float sRes[NS * NS];
    __shared__ float sPost[NS];
    const int64_t m = blockIdx.x;
    const int tid = threadIdx.x;
    if (tid < NS * NS) sRes[tid] = __ldg(p.hRes + m * NS * NS + tid);
    else if (tid < NS * NS + NS) sPost[tid - NS * NS] = __ldg(p.hPost + m * NS + (tid - NS * NS));
    __syncthreads();
    const int64_t vecPerStream = p.D / 8;
    const uint4* xr = reinterpret_cast<const uint4*>(p.x + m * NS * p.D);
    const uint4* yr = reinterpret_cast<const uint4*>(p.y + m * p.D);
    uint4* outr = reinterpret_cast<uint4*>(p.xNext + m * NS * p.D);
    for (int64_t vi = tid; vi < vecPerStream; vi += kPostThreads) {
        // the packed 16-bit words of this vector of every stream and of y; element
        // pairs are unpacked one word at a time, which keeps registers (and so rows in
        // flight per SM) close to the epilogue kernel's
        uint32_t xw[NS][4];
        uint32_t yw[4];
#pragma unroll
        for (int t = 0; t < NS; ++t) {
            const uint4 w = xr[t * vecPerStream + vi];  // plain load: xNext may be x
            xw[t][0] = w.x;
            xw[t][1] = w.y;
            xw[t][2] = w.z;
            xw[t][3] = w.w;
        }
        {
            const uint4 w = __ldg(yr + vi);
            yw[0] = w.x;
            yw[1] = w.y;
            yw[2] = w.z;
            yw[3] = w.w;
        }
        uint32_t ow[NS][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float2 xf[NS];
#pragma unroll
            for (int t = 0; t < NS; ++t) xf[t] = x2_to_f32<DT>(xw[t][q]);
            const float2 yf = x2_to_f32<DT>(yw[q]);
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                float a = __fmul_rn(sRes[s * NS], xf[0].x);
                float b = __fmul_rn(sRes[s * NS], xf[0].y);
#pragma unroll
                for (int t = 1; t < NS; ++t) {
                    a = __fmaf_rn(sRes[s * NS + t], xf[t].x, a);
                    b = __fmaf_rn(sRes[s * NS + t], xf[t].y, b);
                }
                a = __fmaf_rn(sPost[s], yf.x, a);
                b = __fmaf_rn(sPost[s], yf.y, b);
                ow[s][q] = f32x2_to_x2<DT>(a, b);
            }
        }
#pragma unroll
        for (int s = 0; s < NS; ++s) outr[s * vecPerStream + vi] = make_uint4(ow[s][0], ow[s][1], ow[s][2], ow[s][3]);
    }
}
