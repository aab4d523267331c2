// The tied LM head + greedy argmax of a decode step with a few rows, from int8 copies of the
// embedding, with the reference's tokens.
//
// The reference's logits are in-order float32 dot products (nanocompile/lower.py:255-274) and its
// token is np.argmax of them (nanocompile/models/qwen2.py:364). With one to sixteen rows the
// float32 embedding (vocab x hidden x 4 bytes) is the whole cost of the step's head, so the
// prefilter reads a quarter of it:
//
//  1. lm_q8_kernel (once, when the embedding is uploaded): per vocabulary row n, the scale
//     s_n = max_i |w_ni| / 127 and q_ni = rint(w_ni / s_n), so |w_ni - s_n q_ni| <= s_n (1/2 + 2^-16).
//  2. lm_head_q8_kernel: per token, the activations as two int8 digits per value,
//     x ~ sx (x0 + x1 / 128) with sx = max|x| / 127 and |x - sx (x0 + x1/128)| <= sx / 200; the
//     digit dot products with q_n are exact int32 sums (dp4a), and
//     approx_n = s_n sx (sum q x0 + sum q x1 / 128). Its distance to the reference's logit is at
//     most s_n B with
//        B = (1 + 2^-8) [ S (1/2 + 2^-10) + 127 K sx / 200 + 127 S (1.01 K + 16) 2^-24 ],
//     S = sum_k |x_k|: the weights' rounding, the digits' rounding, and the reference's own
//     float32 chain plus the few roundings of approx. A CTA writes approx for its 128 rows and
//     the largest lower bound approx_n - s_n B among them.
//  3. lm_head_q8_pick_kernel: L = the largest lower bound over all rows; every row whose upper
//     bound approx_n + s_n B is not below L is a candidate (the reference's first maximum always
//     is: its logit is at least every other row's, hence at least L), and each candidate's exact
//     in-order logit decides, np.argmax's way (first maximum, NaN largest). The CTAs' winners meet
//     in the last CTA to finish.
//
// Non-finite activations make B infinite: every row is then a candidate and the pick is the
// reference's full computation. A row whose bound s_n B is 2^90 or more (its exact sum could come
// near float32's range) is always a candidate and never sets the lower bound L; so is a row with a
// non-finite weight, whose scale, approx and bound are not finite. The digit
// sums are exact in float32 while 127 * 127 * K < 2^24 (K <= 1024). Both bounds carry an absolute
// 2^-100 for roundings in the subnormal range, and max|x| below 2^-100 also makes B infinite.
#pragma once

#include "nc_lm_head_tc.cuh"

namespace nc {

constexpr int LMQ_ROWS = 128;       // vocabulary rows per prefilter CTA
constexpr int LMQ_THREADS = 256;    // 8 warps; 8 lanes per row, 4 rows per warp per pass
constexpr int LMQ_MAXK = 1024;
constexpr int LMQ_PIECES = LMQ_MAXK / 128;   // 16-byte pieces per lane per row
constexpr int LMQ_MAXT = 8;         // tokens per prefilter pass
constexpr int LMQ_MAXM = 16;        // rows of a step the int8 head serves
constexpr int LMQ_PICK_THREADS = 256;
constexpr int LMQ_PICK_CTAS = 148;     // one wave of the pick kernel
constexpr int LMQ_PREFILTER_CTAS = 3 * 148;   // persistent prefilter: three CTAs per SM
constexpr float LMQ_ABS = 0x1p-100f;   // absolute slack: roundings in the subnormal range
constexpr float LMQ_BIG = 0x1p90f;     // a larger bound s_n B: the row is a candidate, not a lower bound

struct LmHeadQ8Args {
    int m, n, k;                    // tokens, vocabulary rows, hidden
    const int8_t *q;                // [n][k]
    const float *s;                 // [n]
    const float *x;                 // [m][k] the normed rows
    const float *w;                 // [n][k] the float32 weights (exact logits)
    float *approx;                  // [m][n]
    float *cta_low;                 // [m][ctas]
    float *bound;                   // [m]
    float *pick_val;                // [m][pick ctas]
    int32_t *pick_idx;
    unsigned int *counter;          // pick CTAs finished (the last one resets it)
    int64_t *tokens;                // [m]
};

// One warp per vocabulary row.
__global__ void __launch_bounds__(256) lm_q8_kernel(int8_t *__restrict__ q, float *__restrict__ s,
                                                    const float *__restrict__ w, int n, int k) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= n) return;
    const float *wr = w + (int64_t)row * k;
    float mx = 0.0f;
    bool nan = false;
    for (int i = lane; i < k; i += 32) {
        const float v = fabsf(wr[i]);
        nan |= v != v;
        mx = fmaxf(mx, v);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    nan = __any_sync(0xffffffffu, nan);
    const float sc = nan ? __uint_as_float(0x7fc00000u) : mx / 127.0f;
    const bool usable = sc > 0.0f && sc <= 3.0e38f;
    for (int i = lane; i < k; i += 32) {
        float v = usable ? rintf(wr[i] / sc) : 0.0f;
        v = fminf(127.0f, fmaxf(-127.0f, v));
        q[(int64_t)row * k + i] = (int8_t)(int)v;
    }
    if (lane == 0) s[row] = sc;
}

__device__ __forceinline__ void lmq_load(uint4 *wv, const int8_t *q, int row, int n, int k, int j, int pieces) {
#pragma unroll
    for (int p = 0; p < LMQ_PIECES; ++p) {
        wv[p] = make_uint4(0u, 0u, 0u, 0u);
        if (p < pieces && row < n) wv[p] = __ldcs(reinterpret_cast<const uint4 *>(q + (int64_t)row * k + (p * 8 + j) * 16));
    }
}

template <int T>
__global__ void __launch_bounds__(LMQ_THREADS) lm_head_q8_kernel(const LmHeadQ8Args a) {
    __shared__ __align__(16) int8_t xd[T][2][LMQ_MAXK];   // the digits x0 | x1 per token
    __shared__ float s_sx[T], s_bnd[T];
    __shared__ float r_max[LMQ_THREADS / 32][T], r_sum[LMQ_THREADS / 32][T];
    __shared__ int r_bad[LMQ_THREADS / 32][T];
    __shared__ float s_low[LMQ_THREADS / 32][T];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, grp = lane >> 3, j = lane & 7;
    const int K = a.k, pieces = K / 128;
    // persistent: this CTA takes 128-row blocks blockIdx.x, blockIdx.x + gridDim.x, ... (4 passes of
    // 32 rows each), the digits prepared once
    const int ctas = (a.n + LMQ_ROWS - 1) / LMQ_ROWS, t0 = blockIdx.y * T, tn = min(T, a.m - t0);
    constexpr int PASSES = LMQ_ROWS / 32;
    const int my_blocks = blockIdx.x < ctas ? (ctas - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    auto pass_row = [&](int p) { return (blockIdx.x + (p / PASSES) * gridDim.x) * LMQ_ROWS + (p % PASSES) * 32 + warp * 4 + grp; };

    // the first pass's weights do not depend on the previous kernel
    release_dependents();
    uint4 wv[LMQ_PIECES], wn[LMQ_PIECES];
    if (my_blocks) lmq_load(wv, a.q, pass_row(0), a.n, K, j, pieces);
    wait_for_producer();

    // per token: max |x|, sum |x|, any non-finite value
    float mx[T], sm[T];
    int bad[T];
#pragma unroll
    for (int u = 0; u < T; ++u) { mx[u] = 0.0f; sm[u] = 0.0f; bad[u] = 0; }
    for (int i = t; i < K; i += LMQ_THREADS)
#pragma unroll
        for (int u = 0; u < T; ++u)
            if (u < tn) {
                const float v = fabsf(a.x[(int64_t)(t0 + u) * K + i]);
                bad[u] |= !(v <= 3.0e38f);
                mx[u] = fmaxf(mx[u], v);
                sm[u] += v;
            }
#pragma unroll
    for (int u = 0; u < T; ++u) {
        for (int o = 16; o > 0; o >>= 1) {
            mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
            sm[u] += __shfl_xor_sync(0xffffffffu, sm[u], o);
            bad[u] |= __shfl_xor_sync(0xffffffffu, bad[u], o);
        }
        if (lane == 0) { r_max[warp][u] = mx[u]; r_sum[warp][u] = sm[u]; r_bad[warp][u] = bad[u]; }
    }
    __syncthreads();
    if (t < T) {
        float M = 0.0f, S = 0.0f;
        int B = 0;
        for (int w = 0; w < LMQ_THREADS / 32; ++w) { M = fmaxf(M, r_max[w][t]); S += r_sum[w][t]; B |= r_bad[w][t]; }
        S *= 1.0f + 0x1p-10f;                    // an upper bound on the exact sum of K terms
        const float sx = M / 127.0f;
        s_sx[t] = sx;
        float bnd = S * (0.5f + 0x1p-10f) + 127.0f * (float)K * sx / 200.0f +
                    127.0f * S * (1.01f * (float)K + 16.0f) * 0x1p-24f;
        bnd *= 1.0f + 0x1p-8f;
        if (B || M < 0x1p-100f) bnd = __uint_as_float(0x7f800000u);
        s_bnd[t] = bnd;
        if (blockIdx.x == 0 && t < tn) a.bound[t0 + t] = bnd;
    }
    __syncthreads();
    // the digits
    for (int i = t; i < T * K; i += LMQ_THREADS) {
        const int u = i / K, kk = i % K;
        int d0 = 0, d1 = 0;
        if (u < tn && s_sx[u] > 0.0f) {
            const float v = a.x[(int64_t)(t0 + u) * K + kk] / s_sx[u];
            const float r0 = fminf(127.0f, fmaxf(-127.0f, rintf(v)));
            const float r1 = fminf(127.0f, fmaxf(-127.0f, rintf((v - r0) * 128.0f)));
            d0 = (int)r0;
            d1 = (int)r1;
        }
        xd[u][0][kk] = (int8_t)d0;
        xd[u][1][kk] = (int8_t)d1;
    }
    __syncthreads();

    const float sx_j = j < tn ? s_sx[j] : 0.0f, bnd_j = j < tn ? s_bnd[j] : 0.0f;
    float low = -__uint_as_float(0x7f800000u);      // lane j: token j's largest lower bound in the block
    for (int p = 0; p < my_blocks * PASSES; ++p) {
        const int row = pass_row(p);
        if (p + 1 < my_blocks * PASSES) lmq_load(wn, a.q, pass_row(p + 1), a.n, K, j, pieces);
        int hi[T], lo[T];
#pragma unroll
        for (int u = 0; u < T; ++u) { hi[u] = 0; lo[u] = 0; }
#pragma unroll
        for (int q = 0; q < LMQ_PIECES; ++q) {
            if (q < pieces) {
                const int off = (q * 8 + j) * 16;
#pragma unroll
                for (int u = 0; u < T; ++u) {
                    const uint4 d0 = *reinterpret_cast<const uint4 *>(&xd[u][0][off]);
                    const uint4 d1 = *reinterpret_cast<const uint4 *>(&xd[u][1][off]);
                    hi[u] = __dp4a((int)wv[q].x, (int)d0.x, hi[u]);
                    hi[u] = __dp4a((int)wv[q].y, (int)d0.y, hi[u]);
                    hi[u] = __dp4a((int)wv[q].z, (int)d0.z, hi[u]);
                    hi[u] = __dp4a((int)wv[q].w, (int)d0.w, hi[u]);
                    lo[u] = __dp4a((int)wv[q].x, (int)d1.x, lo[u]);
                    lo[u] = __dp4a((int)wv[q].y, (int)d1.y, lo[u]);
                    lo[u] = __dp4a((int)wv[q].z, (int)d1.z, lo[u]);
                    lo[u] = __dp4a((int)wv[q].w, (int)d1.w, lo[u]);
                }
            }
        }
        // sums over the row's 8 lanes; lane j keeps token j
        int myhi = 0, mylo = 0;
#pragma unroll
        for (int u = 0; u < T; ++u) {
            int h = hi[u], l = lo[u];
            h += __shfl_xor_sync(0xffffffffu, h, 1);
            l += __shfl_xor_sync(0xffffffffu, l, 1);
            h += __shfl_xor_sync(0xffffffffu, h, 2);
            l += __shfl_xor_sync(0xffffffffu, l, 2);
            h += __shfl_xor_sync(0xffffffffu, h, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            if (j == u) { myhi = h; mylo = l; }
        }
        if (j < tn && row < a.n) {
            const float sn = a.s[row];
            const float ap = sn * sx_j * ((float)myhi + (float)mylo * 0.0078125f);
            a.approx[(int64_t)(t0 + j) * a.n + row] = ap;
            const float e = sn * bnd_j;
            if (e < LMQ_BIG) low = fmaxf(low, ap - fadd(e, LMQ_ABS));
        }
        if (p + 1 < my_blocks * PASSES) {
#pragma unroll
            for (int q = 0; q < LMQ_PIECES; ++q) wv[q] = wn[q];
        }
        if (p % PASSES == PASSES - 1) {
            // the block's largest lower bound per token
            low = fmaxf(low, __shfl_xor_sync(0xffffffffu, low, 8));
            low = fmaxf(low, __shfl_xor_sync(0xffffffffu, low, 16));
            if (lane < T) s_low[warp][lane] = low;
            __syncthreads();
            if (t < tn) {
                float v = s_low[0][t];
                for (int w = 1; w < LMQ_THREADS / 32; ++w) v = fmaxf(v, s_low[w][t]);
                a.cta_low[(int64_t)(t0 + t) * ctas + blockIdx.x + (p / PASSES) * gridDim.x] = v;
            }
            __syncthreads();
            low = -__uint_as_float(0x7f800000u);
        }
    }
}

// Per token: L, this CTA's share of the rows (strided over the grid) tested against it, the
// survivors listed in shared memory, then rechecked exactly one per warp. grid = any number of
// CTAs; shared memory = K floats (x) + 16 x K floats (two staged rows per warp) + the list.
constexpr int LMQ_SCAN = 8;        // rows a pick thread tests per round (151,936 rows take one round)
constexpr int LMQ_LIST = 4096;     // candidate slots per CTA (more than its rows per token at 148 CTAs)

__host__ __device__ inline size_t lmq_pick_smem(int k) { return sizeof(float) * (size_t)(17 * k) + sizeof(int) * LMQ_LIST; }

__global__ void __launch_bounds__(LMQ_PICK_THREADS)
lm_head_q8_pick_kernel(const LmHeadQ8Args a, int ctas) {
    extern __shared__ __align__(16) float pxs[];       // [K] x | [8][K] staged rows | list
    __shared__ float rv[LMQ_PICK_THREADS / 32];
    __shared__ int ri[LMQ_PICK_THREADS / 32];
    __shared__ float s_low;
    __shared__ int s_count;
    __shared__ bool s_last;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int K = a.k;
    float *rowbuf = pxs + K + warp * 2 * K;            // two staged rows per warp
    int *list = reinterpret_cast<int *>(pxs + 17 * K);
    const int64_t gt = (int64_t)blockIdx.x * LMQ_PICK_THREADS + t, stride = (int64_t)gridDim.x * LMQ_PICK_THREADS;
    release_dependents();
    wait_for_producer();
    for (int m = 0; m < a.m; ++m) {
        __syncthreads();
        // the first round of this thread's approximations and scales, requested before L is known
        float ap[LMQ_SCAN], sv[LMQ_SCAN];
        auto fetch = [&](int64_t n0) {
#pragma unroll
            for (int u = 0; u < LMQ_SCAN; ++u) {
                const int64_t n = n0 + u * stride;
                ap[u] = n < a.n ? a.approx[(int64_t)m * a.n + n] : 0.0f;
                sv[u] = n < a.n ? a.s[n] : 0.0f;
            }
        };
        fetch(gt);
        for (int k = t; k < K; k += LMQ_PICK_THREADS) pxs[k] = a.x[(int64_t)m * K + k];
        float g = -__uint_as_float(0x7f800000u);
        for (int c = t; c < ctas; c += LMQ_PICK_THREADS) g = fmaxf(g, a.cta_low[(int64_t)m * ctas + c]);
        for (int o = 16; o > 0; o >>= 1) g = fmaxf(g, __shfl_xor_sync(0xffffffffu, g, o));
        if (lane == 0) rv[warp] = g;
        if (t == 0) s_count = 0;
        __syncthreads();
        if (t == 0) {
            float b = rv[0];
            for (int i = 1; i < LMQ_PICK_THREADS / 32; ++i) b = fmaxf(b, rv[i]);
            s_low = b;
        }
        __syncthreads();
        const float L = s_low, B = a.bound[m];
        // this thread's rows, LMQ_SCAN at a time with all their loads in flight together
        for (int64_t n0 = gt; n0 < a.n; n0 += LMQ_SCAN * stride) {
            if (n0 != gt) fetch(n0);
#pragma unroll
            for (int u = 0; u < LMQ_SCAN; ++u) {
                const int64_t n = n0 + u * stride;
                if (n >= a.n) break;
                const float e = sv[u] * B;
                if (e < LMQ_BIG && ap[u] + fadd(e, LMQ_ABS) < L) continue;   // NaN: a candidate
                const int at = atomicAdd(&s_count, 1);
                if (at < LMQ_LIST) list[at] = (int)n;
            }
        }
        __syncthreads();
        const int count = min(s_count, LMQ_LIST);
        float bv = -__uint_as_float(0x7f800000u);
        int bi = 0x7fffffff;
        // the list; or, when it overflowed, every row of this CTA's share, a list at a time
        const bool overflow = s_count > LMQ_LIST;
        for (int64_t base = (int64_t)blockIdx.x * LMQ_PICK_THREADS;; base += stride) {
            int cnt = count;
            if (overflow) {
                if (base >= a.n) break;
                __syncthreads();
                if (base + t < a.n) list[t] = (int)(base + t);
                __syncthreads();
                cnt = (int)(a.n - base < LMQ_PICK_THREADS ? a.n - base : LMQ_PICK_THREADS);
            }
            best_of_list_warp(a.w, list, warp, LMQ_PICK_THREADS / 32, cnt, pxs, rowbuf, K, bv, bi);
            if (!overflow) break;
        }
        __syncthreads();
        if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
        __syncthreads();
        if (t == 0) {
            for (int i = 1; i < LMQ_PICK_THREADS / 32; ++i)
                if (argmax_better(rv[i], ri[i], bv, bi)) { bv = rv[i]; bi = ri[i]; }
            a.pick_val[(int64_t)m * gridDim.x + blockIdx.x] = bv;
            a.pick_idx[(int64_t)m * gridDim.x + blockIdx.x] = bi;
        }
    }
    // the last CTA to finish reduces every CTA's winner
    if (t == 0) {
        __threadfence();
        s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int m = warp; m < a.m; m += LMQ_PICK_THREADS / 32) {
        float bv = -__uint_as_float(0x7f800000u);
        int bi = 0x7fffffff;
        for (int c = lane; c < (int)gridDim.x; c += 32) {
            const float v = __ldcg(a.pick_val + (int64_t)m * gridDim.x + c);
            const int i = __ldcg(a.pick_idx + (int64_t)m * gridDim.x + c);
            if (argmax_better(v, i, bv, bi)) { bv = v; bi = i; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) a.tokens[m] = bi;
    }
    if (t == 0) *a.counter = 0u;
}

}  // namespace nc
