// Path 2: the single-launch decode kernel for small M (included by mhc_pre_kernels.cu
// inside namespace mhc, after the path-0 kernels whose helpers it uses).
//
// At M <= kDecodeMaxRows rows (the plan's default takes it up to kDecodeDefaultRows)
// the x . phi' product is about 0.7 M multiply-adds per row: CUDA cores finish it in
// well under a microsecond, and what costs time is
// reading phi' once (2.75 MB at n=4, D=7168) and the launches.  So one cooperative
// launch of G CTAs (one per SM) does everything:
//   phase 1  CTA g takes the K-slice [g*C/G, (g+1)*C/G) of the C 64-wide chunks,
//            stages x[:, slice] and w = hi + lo of the prepared weights (exact in
//            fp32) in shared memory, 256 K elements at a time, and forms the partial
//            mix sums and the partial sum of squares of every row with register
//            tiles of 4 rows x 8 columns (lanes split K; a butterfly reduce-scatter
//            of the 32 tile values then leaves lane l with value l's sum in 31
//            shuffles), written to a partial record [g][row][W];
//   barrier  a grid barrier on a 64-bit arrival counter in the workspace header
//            (each launch adds G; the target is the next multiple of G), bounded;
//   phase 2  independent warp units spread over all warps of the grid: an hIn unit
//            (row m, 256-wide slice of D) sums the G partial records of hPre's
//            columns and the square sum (lanes over the records, in order, then a
//            fixed xor tree), computes invRms and hPre and forms hIn for its slice;
//            an output unit (row m, mix column c >= n) sums column c and the square
//            sum the same way and writes hPost[m][c-n] or hRes[m][c-2n].  Each unit
//            costs two dependent memory round trips, and all run concurrently.
// The arithmetic of a row depends on G and K only, not on timing: results are
// deterministic.
#pragma once

constexpr int kDecodeThreads = 512;
constexpr int kDecodePiece = 256;    // K elements staged in shared memory at a time
constexpr int kDecodeRowTile = 4;    // register tile rows
constexpr int kDecodeColTile = 8;    // register tile columns (mix sums + the square sum)
static_assert(kDecodeRowTile * kDecodeColTile == 32, "one tile value per lane after the reduce-scatter");
constexpr int kDecodeDRange = 256;   // hIn elements per phase-2 unit (one warp, 8 per lane)

struct DecodeParams {
    int M;
    int chunks;  // ceil(K / 64)
    int W;       // floats per partial record
    int64_t K;
    int64_t D;
    float invK;
    float normEps;
    float hcEps;
    const uint16_t* x;    // [M][K]
    const uint16_t* phi;  // prepared [2*mix][K]: hi rows, then lo rows
    const float* alpha;
    const float* bias;
    uint16_t* hIn;
    float* hPost;
    float* hRes;
    float* part;                     // [G][M][W]
    int64_t partFloats;              // floats of part (bounds checks of the debug build)
    unsigned long long* barrier;     // WorkspaceHeader::gridBarrier
    const WorkspaceHeader* hdr;
    uint32_t signature;              // of the description (checked against the prepared weights)
};

// Shared memory of the decode kernel, in bytes (host and device agree on it).
__host__ __device__ constexpr size_t decode_smem_bytes(int M, int mix) {
    return static_cast<size_t>(M) * kDecodePiece * 2          // x piece
           + static_cast<size_t>(mix) * kDecodePiece * 4      // w piece
           + static_cast<size_t>(M) * (mix + 1) * 4           // running sums
           + 16;                                              // flag
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float warp_sum_tree(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int DT>
__device__ __forceinline__ float x16_to_f32(uint16_t b) {
    if constexpr (DT == MHC_DTYPE_BF16) {
        return __bfloat162float(__ushort_as_bfloat16(b));
    } else {
        return __half2float(__ushort_as_half(b));
    }
}

template <int DT, int NS>
__global__ void __launch_bounds__(kDecodeThreads, 1) mhc_pre_decode_kernel(const DecodeParams p) {
    constexpr int MIX = NS * NS + 2 * NS;
    constexpr int COLS = MIX + 1;
    constexpr int CT = (COLS + kDecodeColTile - 1) / kDecodeColTile;
    extern __shared__ __align__(16) uint8_t smem[];
    uint16_t* sx = reinterpret_cast<uint16_t*>(smem);                                       // [M][piece]
    float* sw = reinterpret_cast<float*>(smem + static_cast<size_t>(p.M) * kDecodePiece * 2);  // [MIX][piece]
    float* sacc = sw + MIX * kDecodePiece;                                                   // [M][COLS]
    volatile int* sFlag = reinterpret_cast<volatile int*>(sacc + p.M * COLS);

    const int G = gridDim.x;
    const int g = blockIdx.x;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int M = p.M;
    // Without weights prepared for this description the launch returns before the
    // grid barrier (every CTA reads the same header), so the arrival counter only
    // ever sees launches of the description it was zeroed for, all with the same G.
    const bool prepared = p.hdr->magic == kPreparedMagic && p.hdr->signature == p.signature;
    if (!prepared) {
        if (g == 0 && tid == 0) set_device_status(MHC_STATUS_NOT_PREPARED);
        return;
    }

    // ---------------- phase 1: partial records of this CTA's K-slice ----------------
    const int c0 = static_cast<int>(static_cast<int64_t>(g) * p.chunks / G);
    const int c1 = static_cast<int>(static_cast<int64_t>(g + 1) * p.chunks / G);
    const int64_t kBegin = static_cast<int64_t>(c0) * kChunk;
    const int64_t kEnd = min(static_cast<int64_t>(c1) * kChunk, p.K);
    for (int i = tid; i < M * COLS; i += kDecodeThreads) sacc[i] = 0.0f;
    const int rowTiles = (M + kDecodeRowTile - 1) / kDecodeRowTile;
    const int tiles = rowTiles * CT;
    for (int64_t k0 = kBegin; k0 < kEnd; k0 += kDecodePiece) {
        const int kp = static_cast<int>(min(static_cast<int64_t>(kDecodePiece), kEnd - k0));  // multiple of 16
        const int v8 = kp / 8;
        __syncthreads();  // the previous piece is consumed
        if (prepared) {
            // all loads of a batch are issued before any is used
            constexpr int kB = 4;
            for (int i0 = tid; i0 < M * v8; i0 += kDecodeThreads * kB) {
                uint4 v[kB];
#pragma unroll
                for (int b = 0; b < kB; ++b) {
                    const int i = i0 + b * kDecodeThreads;
                    if (i < M * v8) {
                        const int m = i / v8, c = i - (i / v8) * v8;
                        v[b] = __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(m) * p.K + k0) + c);
                    }
                }
#pragma unroll
                for (int b = 0; b < kB; ++b) {
                    const int i = i0 + b * kDecodeThreads;
                    if (i < M * v8) {
                        const int m = i / v8, c = i - (i / v8) * v8;
                        *reinterpret_cast<uint4*>(sx + m * kDecodePiece + c * 8) = v[b];
                    }
                }
            }
            for (int i0 = tid; i0 < MIX * v8; i0 += kDecodeThreads * kB) {
                uint4 h[kB], l[kB];
#pragma unroll
                for (int b = 0; b < kB; ++b) {
                    const int i = i0 + b * kDecodeThreads;
                    if (i < MIX * v8) {
                        const int j = i / v8, c = i - (i / v8) * v8;
                        h[b] = __ldg(reinterpret_cast<const uint4*>(p.phi + static_cast<int64_t>(j) * p.K + k0) + c);
                        l[b] = __ldg(reinterpret_cast<const uint4*>(p.phi + static_cast<int64_t>(MIX + j) * p.K + k0) +
                                     c);
                    }
                }
#pragma unroll
                for (int b = 0; b < kB; ++b) {
                    const int i = i0 + b * kDecodeThreads;
                    if (i < MIX * v8) {
                        const int j = i / v8, c = i - (i / v8) * v8;
                        const uint32_t hw[4] = {h[b].x, h[b].y, h[b].z, h[b].w};
                        const uint32_t lw[4] = {l[b].x, l[b].y, l[b].z, l[b].w};
                        float w[8];
#pragma unroll
                        for (int t = 0; t < 4; ++t) {
                            const float2 hf = x2_to_f32<DT>(hw[t]);
                            const float2 lf = x2_to_f32<DT>(lw[t]);
                            w[2 * t] = __fadd_rn(hf.x, lf.x);
                            w[2 * t + 1] = __fadd_rn(hf.y, lf.y);
                        }
                        float4* dst = reinterpret_cast<float4*>(sw + j * kDecodePiece + c * 8);
                        dst[0] = make_float4(w[0], w[1], w[2], w[3]);
                        dst[1] = make_float4(w[4], w[5], w[6], w[7]);
                    }
                }
            }
        }
        __syncthreads();
        for (int t = warp; t < tiles; t += kDecodeThreads / 32) {
            const int rt = t / CT, ct = t - (t / CT) * CT;
            const int m0 = rt * kDecodeRowTile, j0 = ct * kDecodeColTile;
            float acc[kDecodeRowTile][kDecodeColTile];
#pragma unroll
            for (int a = 0; a < kDecodeRowTile; ++a)
#pragma unroll
                for (int b = 0; b < kDecodeColTile; ++b) acc[a][b] = 0.0f;
            for (int kk = lane; kk < kp; kk += 32) {
                float xv[kDecodeRowTile], wv[kDecodeColTile];
#pragma unroll
                for (int a = 0; a < kDecodeRowTile; ++a)
                    xv[a] = x16_to_f32<DT>(sx[min(m0 + a, M - 1) * kDecodePiece + kk]);
#pragma unroll
                for (int b = 0; b < kDecodeColTile; ++b) wv[b] = sw[min(j0 + b, MIX - 1) * kDecodePiece + kk];
#pragma unroll
                for (int a = 0; a < kDecodeRowTile; ++a)
#pragma unroll
                    for (int b = 0; b < kDecodeColTile; ++b)
                        acc[a][b] = fmaf(xv[a], j0 + b == MIX ? xv[a] : wv[b], acc[a][b]);
            }
            // butterfly reduce-scatter: after the step of width w, a lane keeps the half
            // of the remaining values selected by its lane bit w; at the end lane l
            // holds the warp sum of tile value l (row l / 8, column l % 8)
            float v[32];
#pragma unroll
            for (int a = 0; a < kDecodeRowTile; ++a)
#pragma unroll
                for (int b = 0; b < kDecodeColTile; ++b) v[a * kDecodeColTile + b] = acc[a][b];
#pragma unroll
            for (int w = 16; w >= 1; w >>= 1) {
                const bool upper = (lane & w) != 0;
#pragma unroll
                for (int i = 0; i < w; ++i) {
                    const float send = upper ? v[i] : v[i + w];
                    const float keep = upper ? v[i + w] : v[i];
                    v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, w));
                }
            }
            {
                const int m = m0 + lane / kDecodeColTile, j = j0 + lane % kDecodeColTile;
                if (m < M && j < COLS) sacc[m * COLS + j] = __fadd_rn(sacc[m * COLS + j], v[0]);
            }
        }
    }
    __syncthreads();
    {
        const float unscale = ldexpf(1.0f, -p.hdr->phiScaleExp);
        float* rec = p.part + static_cast<int64_t>(g) * M * p.W;
        for (int i = tid; i < M * COLS; i += kDecodeThreads) {
            const int m = i / COLS, j = i - (i / COLS) * COLS;
            if (MHC_CHECK((static_cast<int64_t>(g) * M + m) * p.W + j < p.partFloats))
                rec[m * p.W + j] = j < MIX ? __fmul_rn(sacc[i], unscale) : sacc[i];
        }
    }

    // ---------------- grid barrier ----------------
    __syncthreads();  // the CTA's records are written (CTA scope) ...
    if (tid == 0) {
        __threadfence();  // ... and released at GPU scope with the arrival
        const unsigned long long old = atomicAdd(p.barrier, 1ull);
        const unsigned long long target = (old / static_cast<unsigned long long>(G) + 1) * G;
        bool ok = false;
        const uint64_t t0 = global_timer_ns();
        for (uint32_t i = 0; i < kMaxPolls; ++i) {
            if (ld_acquire_u64(p.barrier) >= target) {
                ok = true;
                break;
            }
            if ((i & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) break;
            __nanosleep(32);
        }
        *sFlag = ok ? 0 : 1;
        if (!ok) set_device_status(MHC_STATUS_DEVICE_TIMEOUT);
    }
    __syncthreads();
    if (*sFlag != 0) return;

    // ---------------- phase 2: warp units ----------------
    const int nd = static_cast<int>((p.D + kDecodeDRange - 1) / kDecodeDRange);
    const int hinUnits = M * nd;
    const int units = hinUnits + M * (MIX - NS);
    const float a0 = __ldg(p.alpha + 0), a1 = __ldg(p.alpha + 1), a2 = __ldg(p.alpha + 2);
    // Sums over the G records of columns cols[0..NC) of row m: lane r takes records
    // r, r+32, ... in order, then the fixed xor tree (every lane gets the totals).
    // The loads of all columns are issued together.
    auto column_totals = [&](int m, const int (&cols)[NS + 1], int nc, float (&tot)[NS + 1]) {
#pragma unroll
        for (int q = 0; q <= NS; ++q) tot[q] = 0.0f;
        for (int r0 = 0; r0 < G; r0 += 160) {
            float vals[NS + 1][5];
#pragma unroll
            for (int q = 0; q <= NS; ++q)
#pragma unroll
                for (int i = 0; i < 5; ++i) {
                    const int r = r0 + lane + 32 * i;
                    const int64_t at = (static_cast<int64_t>(r) * M + m) * p.W + cols[q];
                    vals[q][i] = (q < nc && r < G && MHC_CHECK(at < p.partFloats)) ? __ldcg(p.part + at) : 0.0f;
                }
#pragma unroll
            for (int q = 0; q <= NS; ++q)
#pragma unroll
                for (int i = 0; i < 5; ++i) tot[q] = __fadd_rn(tot[q], vals[q][i]);
        }
#pragma unroll
        for (int q = 0; q <= NS; ++q)
            if (q < nc) tot[q] = warp_sum_tree(tot[q]);
    };
    auto inv_rms = [&](float sumsq) -> float {
        float v = __fmul_rn(sumsq, p.invK);
        v = __fadd_rn(v, p.normEps);
        return __fdiv_rn(1.0f, __fsqrt_rn(v));
    };
    // warp-major numbering spreads the units over all CTAs (SMs) before doubling up
    const int warps = G * (kDecodeThreads / 32);
    for (int u = warp * G + g; u < units; u += warps) {
        if (u < hinUnits) {
            const int m = u / nd, dr = u - (u / nd) * nd;
            // the x loads do not depend on hPre: issue them with the record loads
            const int64_t d = static_cast<int64_t>(dr) * kDecodeDRange + lane * 8;
            const bool active = d < p.D;
            const uint16_t* xr = p.x + static_cast<int64_t>(m) * p.K + d;
            uint4 w[NS];
#pragma unroll
            for (int s2 = 0; s2 < NS; ++s2)
                w[s2] = active ? __ldg(reinterpret_cast<const uint4*>(xr + s2 * p.D)) : make_uint4(0, 0, 0, 0);
            int cols[NS + 1];
#pragma unroll
            for (int q = 0; q <= NS; ++q) cols[q] = q < NS ? q : MIX;
            float tot[NS + 1];
            column_totals(m, cols, NS + 1, tot);
            const float sPreScale = __fmul_rn(inv_rms(tot[NS]), a0);
            float pre[NS];
#pragma unroll
            for (int s2 = 0; s2 < NS; ++s2) {
                const float t1 = __fadd_rn(__fmul_rn(tot[s2], sPreScale), __ldg(p.bias + s2));
                pre[s2] = __fadd_rn(sigmoid_ref(t1), p.hcEps);
            }
            if (active) {
                float acc[8];
#pragma unroll
                for (int s2 = 0; s2 < NS; ++s2) {
                    const uint32_t ws[4] = {w[s2].x, w[s2].y, w[s2].z, w[s2].w};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const float2 f = x2_to_f32<DT>(ws[t]);
                        if (s2 == 0) {
                            acc[2 * t] = __fmul_rn(f.x, pre[0]);
                            acc[2 * t + 1] = __fmul_rn(f.y, pre[0]);
                        } else {
                            acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(f.x, pre[s2]));
                            acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(f.y, pre[s2]));
                        }
                    }
                }
                uint4 o;
                o.x = f32x2_to_x2<DT>(acc[0], acc[1]);
                o.y = f32x2_to_x2<DT>(acc[2], acc[3]);
                o.z = f32x2_to_x2<DT>(acc[4], acc[5]);
                o.w = f32x2_to_x2<DT>(acc[6], acc[7]);
                *reinterpret_cast<uint4*>(p.hIn + static_cast<int64_t>(m) * p.D + d) = o;
            }
        } else {
            const int v = u - hinUnits;
            const int m = v / (MIX - NS);
            const int c = NS + (v - m * (MIX - NS));
            int cols[NS + 1];
#pragma unroll
            for (int q = 0; q <= NS; ++q) cols[q] = q == 0 ? c : MIX;
            float tot[NS + 1];
            column_totals(m, cols, 2, tot);
            const float tc = tot[0];
            const float invRms = inv_rms(tot[1]);
            if (lane == 0) {
                if (c < 2 * NS) {
                    const float t2 = __fadd_rn(__fmul_rn(tc, __fmul_rn(invRms, a1)), __ldg(p.bias + c));
                    p.hPost[static_cast<int64_t>(m) * NS + (c - NS)] = __fmul_rn(sigmoid_ref(t2), 2.0f);
                } else {
                    p.hRes[static_cast<int64_t>(m) * NS * NS + (c - 2 * NS)] =
                        __fadd_rn(__fmul_rn(tc, __fmul_rn(invRms, a2)), __ldg(p.bias + c));
                }
            }
        }
    }
}
