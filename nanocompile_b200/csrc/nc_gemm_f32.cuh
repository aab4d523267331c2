// Float32 projections over many rows at once -- above all the tied LM head of a batched decode
// step -- with the reference's in-order sums (nanocompile/lower.py:255-274: acc = acc + x[k] * w[n, k],
// k = 0, 1, 2, ...), bit for bit.
//
// gemv_f32_kernel walks the weights once per 16 tokens; here one pass serves up to 2*T tokens:
// a CTA owns 128 weight rows and 2*T tokens, thread (row, token group) keeps T independent
// chains, so the weight tile a thread reads from shared memory feeds 8*T multiply-adds and the
// 545 MB LM-head matrix crosses HBM once per step for a 64-row batch. Tiles of 32 columns of
// the weights (XOR-swizzled so a thread reading its own row is conflict-free) and of the
// activations stream through a cp.async ring. With ARGMAX each CTA reduces its rows to a
// (value, index) winner per token; the last CTA to finish reduces the winners in CTA order
// (np.argmax's first maximum, NaN the largest).
#pragma once

#include "nc_kernels.cuh"

namespace nc {

constexpr int GF_THREADS = 2 * F32_ROWS;   // (row, token group) for 128 rows and two groups

__host__ __device__ inline size_t gemm_f32_smem(int T) {
    return sizeof(float4) * F32_STAGES * (F32_ROWS * (F32_TILE / 4) + 2 * T * (F32_TILE / 4));
}

template <int T, int EPI, bool ARGMAX>
__global__ void __launch_bounds__(GF_THREADS, 2) gemm_f32_kernel(GemvF32Args a) {
    static_assert(EPI != EPI_SWIGLU, "one weight matrix");
    constexpr int W_PIECES = F32_ROWS * (F32_TILE / 4);
    constexpr int X_PIECES = 2 * T * (F32_TILE / 4);
    constexpr int STAGE_F4 = W_PIECES + X_PIECES;
    static_assert(W_PIECES % GF_THREADS == 0 && X_PIECES % GF_THREADS == 0, "piece layout");
    extern __shared__ float4 smem4[];
    __shared__ float wv[GF_THREADS / 32][T];
    __shared__ int wi[GF_THREADS / 32][T];
    const int t = threadIdx.x, rl = t % F32_ROWS, tg = t / F32_ROWS, warp = t / 32, lane = t % 32;
    const int row0 = blockIdx.x * F32_ROWS, row = row0 + rl;
    const int m0 = blockIdx.y * 2 * T;
    const int K = a.k, tiles = K / F32_TILE;

    auto load_w = [&](int stage, int kt) {
        float4 *st = smem4 + stage * STAGE_F4;
#pragma unroll
        for (int p = 0; p < W_PIECES / GF_THREADS; ++p) {
            const int id = t + p * GF_THREADS, r = id / 8, s = id % 8;
            const float *src = a.w + (int64_t)min(row0 + r, a.n - 1) * K + kt * F32_TILE + s * 4;
            cp_async16(st + r * 8 + (s ^ (r & 7)), src);
        }
    };
    auto load_x = [&](int stage, int kt) {
        float4 *st = smem4 + stage * STAGE_F4 + W_PIECES;
#pragma unroll
        for (int p = 0; p < X_PIECES / GF_THREADS; ++p) {
            const int id = t + p * GF_THREADS, mm = id / 8, s = id % 8;
            const int m = min(m0 + mm, a.m - 1);
            const int64_t xr = a.row_map ? a.row_map[m] : m;
            cp_async16(st + mm * 8 + s, a.x + xr * K + kt * F32_TILE + s * 4);
        }
    };

    // the weights of the first tiles do not depend on the previous kernel: issue them first
    release_dependents();
#pragma unroll
    for (int s = 0; s < F32_STAGES - 1; ++s)
        if (s < tiles) load_w(s, s);
    wait_for_producer();
#pragma unroll
    for (int s = 0; s < F32_STAGES - 1; ++s) {
        if (s < tiles) load_x(s, s);
        cp_async_commit();
    }

    float acc[T];
#pragma unroll
    for (int i = 0; i < T; ++i) acc[i] = 0.0f;
    for (int kt = 0; kt < tiles; ++kt) {
        cp_async_wait<F32_STAGES - 2>();
        __syncthreads();
        const int nxt = kt + F32_STAGES - 1;
        if (nxt < tiles) {
            load_w(nxt % F32_STAGES, nxt);
            load_x(nxt % F32_STAGES, nxt);
        }
        cp_async_commit();
        const float4 *st = smem4 + (kt % F32_STAGES) * STAGE_F4;
        const float4 *xt = st + W_PIECES + tg * T * 8;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const float4 w4 = st[rl * 8 + (s ^ (rl & 7))];
#pragma unroll
            for (int i = 0; i < T; ++i) {
                const float4 xv = xt[i * 8 + s];
                acc[i] = fadd(acc[i], fmul(xv.x, w4.x));
                acc[i] = fadd(acc[i], fmul(xv.y, w4.y));
                acc[i] = fadd(acc[i], fmul(xv.z, w4.z));
                acc[i] = fadd(acc[i], fmul(xv.w, w4.w));
            }
        }
    }
    cp_async_wait<0>();

    // epilogue: outputs, then (ARGMAX) each token's winner among the CTA's rows
#pragma unroll
    for (int i = 0; i < T; ++i) {
        const int m = m0 + tg * T + i;
        if (m < a.m && row < a.n) {
            float y = acc[i];
            if (EPI == EPI_BIAS) y = fadd(y, a.bias[row]);
            if (EPI == EPI_RESIDUAL) y = fadd(a.residual[(int64_t)m * a.n + row], y);
            if (a.out) a.out[(int64_t)m * a.n + row] = y;
        }
    }
    if constexpr (ARGMAX) {
#pragma unroll
        for (int i = 0; i < T; ++i) {
            float v = row < a.n ? acc[i] : -__uint_as_float(0x7f800000u);
            int idx = row < a.n ? row : 0x7fffffff;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (argmax_better(ov, oi, v, idx)) { v = ov; idx = oi; }
            }
            if (lane == 0) { wv[warp][i] = v; wi[warp][i] = idx; }
        }
        __syncthreads();
        constexpr int WPG = F32_ROWS / 32;              // warps per token group
        if (t < 2 * T) {
            const int g = t / T, i = t % T, m = m0 + t;
            float v = wv[g * WPG][i];
            int idx = wi[g * WPG][i];
            for (int w = 1; w < WPG; ++w)
                if (argmax_better(wv[g * WPG + w][i], wi[g * WPG + w][i], v, idx)) { v = wv[g * WPG + w][i]; idx = wi[g * WPG + w][i]; }
            if (m < a.m) {
                a.part_val[(int64_t)m * gridDim.x + blockIdx.x] = v;
                a.part_idx[(int64_t)m * gridDim.x + blockIdx.x] = idx;
            }
        }
        // the last CTA to finish reduces the per-CTA winners, in CTA order
        __shared__ bool last;
        __threadfence();
        __syncthreads();
        if (t == 0) last = atomicAdd(a.counter, 1u) == gridDim.x * gridDim.y - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            for (int m = warp; m < a.m; m += GF_THREADS / 32) {
                float v = -__uint_as_float(0x7f800000u);
                int idx = 0x7fffffff;
                for (int c = lane; c < (int)gridDim.x; c += 32) {
                    const float cv = __ldcg(a.part_val + (int64_t)m * gridDim.x + c);
                    const int ci = __ldcg(a.part_idx + (int64_t)m * gridDim.x + c);
                    if (argmax_better(cv, ci, v, idx)) { v = cv; idx = ci; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                    if (argmax_better(ov, oi, v, idx)) { v = ov; idx = oi; }
                }
                if (lane == 0) a.tokens[m] = idx;
            }
            if (t == 0) *a.counter = 0u;
        }
    }
}

}  // namespace nc
