// int8 weights with float32 activations: the reference's matmul_i8 (nanoinfer's int8 engine,
// nanocompile/lower.py:320-356 int8_dots, scaled by lower.py:398-412 / fusion.py:677-711), bit for bit.
//
// For output (t, n) there are 32 float accumulators; accumulator j takes element j of every
// 32-element block of the row in order, acc = fmaf(float(w), x, acc); 8-element groups past the
// last whole block go into accumulators 0..7 group after group; _combine; each element past the
// last group is then added as sum = sum + float(w) * x; the result is sum * scale[n]. This kernel
// takes widths that are multiples of 16 (whole 16-byte loads), so that last step never occurs:
// the model's widths are whole 32-element blocks, and the groups are covered by widths of 32b + 16.
//
// Two lanes per weight row: lane h of a row owns accumulators 16h..16h+15, so for every block
// it needs exactly the 16 bytes at 32 k0 + 16 h -- one 16-byte load, the two lanes of a row
// covering its 32-byte sector -- kept four blocks ahead in registers. A warp holds 16 rows; the
// bytes become floats exactly (value + 128 stored as a byte: float(u) is the bits 0x4B000000 | u
// minus 2^23, then minus 128), once for all the tokens of a pass. The activations come through
// the read-only cache (the same addresses for every row of the warp). The two halves of _combine
// meet by shuffles; the epilogue is the fp32 path's: bias, residual, or SiLU(gate) * up with the
// gate and up rows of one output in the same lanes.
#pragma once

#include "nc_kernels.cuh"

namespace nc {

constexpr int I8F_WARPS = 4;
constexpr int I8F_ROWS = I8F_WARPS * 16;     // output rows per CTA

struct GemvI8fArgs {
    float *out;                 // [m, n]
    const float *x;             // [m, k]
    const uint8_t *w, *w2;      // [n, k] int8 + 128 (w2: EPI_SWIGLU's up weights)
    const float *scales, *scales2;
    const float *bias, *residual;
    int m, n, k;
};

// float(int8 value) of byte i of a word of (value + 128) bytes, exactly
__device__ __forceinline__ float i8f_byte(uint32_t word, int i) {
    return fsub(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650u | (uint32_t)i)), 8388736.0f);
}

template <int T, int EPI>
__global__ void __launch_bounds__(I8F_WARPS * 32) gemv_i8f_kernel(const GemvI8fArgs a) {
    constexpr bool TWO = EPI == EPI_SWIGLU;
    constexpr int NM = TWO ? 2 : 1, D = 4;
    __shared__ uint64_t tab[32];
    if (TWO && threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, h = lane & 1;
    const int row = blockIdx.x * I8F_ROWS + warp * 16 + (lane >> 1);
    const int rowc = min(row, a.n - 1);
    const int K = a.k, blocks = K / 32, wide = blocks * 32, groups = (K % 32) / 8;
    const uint8_t *wr[NM];
    wr[0] = a.w + (int64_t)rowc * K;
    if (TWO) wr[NM - 1] = a.w2 + (int64_t)rowc * K;
    if (TWO) __syncthreads();

    release_dependents();
    // the first blocks' weights do not depend on the previous kernel
    uint4 ring[D][NM];
#pragma unroll
    for (int s = 0; s < D; ++s)
#pragma unroll
        for (int m = 0; m < NM; ++m)
            if (s < blocks) ring[s][m] = __ldg(reinterpret_cast<const uint4 *>(wr[m] + 32 * s + 16 * h));
    wait_for_producer();

    for (int t0 = 0; t0 < a.m; t0 += T) {
        float acc[NM][T][16];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int t = 0; t < T; ++t)
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[m][t][i] = 0.0f;
        const float *xr[T];
#pragma unroll
        for (int t = 0; t < T; ++t) xr[t] = a.x + (int64_t)min(t0 + t, a.m - 1) * K;
        if (t0 > 0) {                                     // refill the ring for this pass
#pragma unroll
            for (int s = 0; s < D; ++s)
#pragma unroll
                for (int m = 0; m < NM; ++m)
                    if (s < blocks) ring[s][m] = __ldg(reinterpret_cast<const uint4 *>(wr[m] + 32 * s + 16 * h));
        }
        for (int b0 = 0; b0 < blocks; b0 += D) {
#pragma unroll
            for (int s = 0; s < D; ++s) {
                const int b = b0 + s;
                if (b < blocks) {
                    uint4 cur[NM];
#pragma unroll
                    for (int m = 0; m < NM; ++m) cur[m] = ring[s][m];
                    if (b + D < blocks) {
#pragma unroll
                        for (int m = 0; m < NM; ++m)
                            ring[s][m] = __ldg(reinterpret_cast<const uint4 *>(wr[m] + 32 * (b + D) + 16 * h));
                    }
                    float wf[NM][16];
#pragma unroll
                    for (int m = 0; m < NM; ++m) {
                        const uint32_t words[4] = {cur[m].x, cur[m].y, cur[m].z, cur[m].w};
#pragma unroll
                        for (int i = 0; i < 16; ++i) wf[m][i] = i8f_byte(words[i >> 2], i & 3);
                    }
#pragma unroll
                    for (int t = 0; t < T; ++t) {
                        const float4 *xp = reinterpret_cast<const float4 *>(xr[t] + 32 * b + 16 * h);
                        float xv[16];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 v = __ldg(xp + q);
                            xv[4 * q] = v.x;
                            xv[4 * q + 1] = v.y;
                            xv[4 * q + 2] = v.z;
                            xv[4 * q + 3] = v.w;
                        }
#pragma unroll
                        for (int m = 0; m < NM; ++m)
#pragma unroll
                            for (int i = 0; i < 16; ++i) acc[m][t][i] = __fmaf_rn(wf[m][i], xv[i], acc[m][t][i]);
                    }
                }
            }
        }
        // 8-element groups past the last whole block: accumulators 0..7 (lane h = 0's)
        for (int k1 = 0; k1 < groups; ++k1) {
            if (h == 0) {
                const int at = wide + 8 * k1;
#pragma unroll
                for (int m = 0; m < NM; ++m) {
                    const uint2 wv = *reinterpret_cast<const uint2 *>(wr[m] + at);
#pragma unroll
                    for (int t = 0; t < T; ++t)
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            acc[m][t][i] = __fmaf_rn(i8f_byte(i < 4 ? wv.x : wv.y, i & 3), xr[t][at + i], acc[m][t][i]);
                }
            }
        }
        // _combine: lane 1 of the row sends (a[16+l] + a[24+l]); lane 0 finishes the tree
        float y[NM][T];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int t = 0; t < T; ++t) {
                float hv[8];
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    const float pair = fadd(acc[m][t][l], acc[m][t][8 + l]);    // h = 0: a[l] + a[8+l]; h = 1: a[16+l] + a[24+l]
                    const float other = __shfl_xor_sync(0xffffffffu, pair, 1);
                    hv[l] = fadd(pair, other);                                  // used on lane h = 0 only
                }
                const float sum = fadd(fadd(fadd(hv[0], hv[4]), fadd(hv[1], hv[5])), fadd(fadd(hv[2], hv[6]), fadd(hv[3], hv[7])));
                y[m][t] = fmul(sum, (m ? a.scales2 : a.scales)[rowc]);
            }
        if (h == 0 && row < a.n) {
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int tok = t0 + t;
                if (tok >= a.m) break;
                float out = y[0][t];
                if (EPI == EPI_BIAS) out = fadd(out, a.bias[row]);
                if (EPI == EPI_RESIDUAL) out = fadd(a.residual[(int64_t)tok * a.n + row], out);
                if (TWO) out = swiglu(y[0][t], y[NM - 1][t], tab);
                a.out[(int64_t)tok * a.n + row] = out;
            }
        }
    }
}

}  // namespace nc
