// Batched int8-vnni projection: more than four rows (prefill chunks, batched decode).
//
// The arithmetic is the reference's matmul_i8_vnni kernel (nanocompile/lower.py:363-397), the
// same as gemv_i8_fused_kernel's: for output (m, n) there are 32 float accumulators, accumulator
// i takes word i (bytes 4i..4i+3) of every 128-byte chunk of the row,
//     acc_i = fma(dot4(w[n, word], x[m, word]), xs[m, block of the word], acc_i)
// chunk after chunk (then the 32-byte tail groups into accumulators 0..7), and the 32 are summed
// by the pairing tree of _combine (index bits 3, 4, 2, 0, 1).
//
// The layout is built for many rows at once. Lane = accumulator, so a warp's 32 lanes cover one
// chunk and every lane runs its own accumulator's chains; a warp owns R rows (of each of the NM
// weights) x T tokens, NM*R*T independent chains per lane. Weight words come straight from
// global memory -- a warp reads whole 128-byte lines -- D chunks ahead in a register ring; the
// CTA's T tokens of activations are staged in shared memory once and read as one conflict-free
// word per lane. After the chunks a transposing butterfly finishes the tree: at each pairing
// level a lane keeps half of its outputs and trades the other half with its partner, so 31
// shuffles (not 5 per output) leave every lane with NM*R*T/32 finished outputs.
#pragma once

#include "nc_kernels.cuh"

namespace nc {

constexpr int GEMM_WARPS = 8;

// The output a lane holds after the transposing butterfly (P outputs per lane, k < P):
// o = k + P * sel(lane), sel = 16*l3 + 8*l4 + 4*l2 + 2*l0 + l1 (the pairing order 3,4,2,0,1).
__device__ __forceinline__ int butterfly_sel(int lane) {
    return ((lane >> 3) & 1) * 16 + ((lane >> 4) & 1) * 8 + ((lane >> 2) & 1) * 4 + (lane & 1) * 2 + ((lane >> 1) & 1);
}

template <int N>
__device__ __forceinline__ void butterfly_reduce(float *v, int lane) {
    constexpr int bits[5] = {3, 4, 2, 0, 1};
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int half = N >> (s + 1);
        const bool hi = (lane >> bits[s]) & 1;
#pragma unroll
        for (int k = 0; k < half; ++k) {
            const float mine = hi ? v[k + half] : v[k];
            const float other = hi ? v[k] : v[k + half];
            v[k] = fadd(mine, __shfl_xor_sync(0xffffffffu, other, 1 << bits[s]));
        }
    }
}

// Dynamic shared memory of one CTA: [xq: T*k bytes][xs: T*bpad][offsets: T (padded)]
// [PRO_OFFSET terms: T*bpad][EPI_SWIGLU_QUANT outputs: T*ROWS].
__host__ __device__ inline size_t gemm_i8_smem(int T, int rows, int k, bool offset_terms, bool quant_out) {
    const int bpad = (k / QBLOCK + 3) & ~3;
    size_t s = (size_t)T * k + sizeof(float) * ((size_t)T * bpad + ((T + 3) & ~3));
    if (offset_terms) s += sizeof(float) * (size_t)T * bpad;
    if (quant_out) s += sizeof(float) * (size_t)T * rows;
    return s;
}

template <int R, int T, int MAXG, int PRO, int EPI>
__global__ void __launch_bounds__(GEMM_WARPS * 32, 2) gemm_i8_kernel(FusedI8Args f) {
    constexpr bool TWO = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_QUANT;
    constexpr int NM = TWO ? 2 : 1, ROWS = GEMM_WARPS * R;
    constexpr int NACC = NM * R * T, P = NACC / 32;
    constexpr int D = NM * R >= 8 ? 3 : 8;             // weight chunks in flight per warp
    static_assert(NACC % 32 == 0, "the butterfly needs a multiple of 32 chains per lane");
    static_assert(EPI != EPI_SWIGLU_QUANT || ROWS % QBLOCK == 0, "quantized outputs need whole 32-row blocks");
    static_assert(PRO != PRO_NORM, "the norm prologue is the few-row kernel's");
    const GemvI8Args &a = f.g;
    extern __shared__ __align__(16) float dsm[];
    __shared__ uint64_t tab[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.k, blocks = K / QBLOCK, bpad = (blocks + 3) & ~3, kw = K / 4;
    const int chunks = K / CHUNK, stride = chunks * CHUNK, groups = (K % CHUNK) / QBLOCK;
    const int cta_row0 = blockIdx.x * ROWS, row0 = cta_row0 + warp * R;
    const int t0 = blockIdx.y * T, tn = min(T, a.m - t0);
    if (TWO && threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];

    // ---- independent of the previous kernel: the first D chunks of this warp's weight rows ----
    release_dependents();
    const uint32_t *w0 = reinterpret_cast<const uint32_t *>(a.w) + lane;
    const uint32_t *w1 = TWO ? reinterpret_cast<const uint32_t *>(a.w2) + lane : nullptr;
    int roff[R];
#pragma unroll
    for (int r = 0; r < R; ++r) roff[r] = min(row0 + r, a.n - 1) * kw;
    uint32_t ring[D][NM][R];
#pragma unroll
    for (int s = 0; s < D; ++s)
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (s < chunks) {
                ring[s][0][r] = __ldg(w0 + roff[r] + s * 32);
                if (TWO) ring[s][NM - 1][r] = __ldg(w1 + roff[r] + s * 32);
            }

    // ---- stage the CTA's tokens: xq rows (cp.async), block scales, offsets ----
    int8_t *xq_s = reinterpret_cast<int8_t *>(dsm);
    float *xs_s = reinterpret_cast<float *>(xq_s + (size_t)T * K);
    float *offs_s = xs_s + T * bpad;
    float *term_s = offs_s + ((T + 3) & ~3);
    float *hq_s = term_s + (PRO == PRO_OFFSET ? T * bpad : 0);
    wait_for_producer();
    {
        const int per = K / 16;
        for (int i = threadIdx.x; i < T * per; i += blockDim.x) {
            const int t = i / per, p = i - t * per;
            const int src = min(t0 + t, a.m - 1);
            cp_async16(xq_s + t * K + p * 16, a.xq + (int64_t)src * K + p * 16);
        }
        cp_async_commit();
        for (int i = threadIdx.x; i < T * blocks; i += blockDim.x) {
            const int t = i / blocks, b = i - t * blocks;
            const int64_t src = (int64_t)min(t0 + t, a.m - 1) * blocks + b;
            const float s = a.xs[src];
            xs_s[t * bpad + b] = s;
            if (PRO == PRO_OFFSET) term_s[t * bpad + b] = fmul((float)f.bsums_in[src], s);
        }
        if (PRO == PRO_NONE)
            for (int t = threadIdx.x; t < T; t += blockDim.x) offs_s[t] = a.offset[min(t0 + t, a.m - 1)];
    }
    // the residuals of this lane's outputs, requested early
    float res[P];
    const int sel = butterfly_sel(lane);
#pragma unroll
    for (int k = 0; k < P; ++k) {
        const int o = k + P * sel, t = o % T, r = (o / T) % R;
        res[k] = (EPI == EPI_RESIDUAL && t < tn && row0 + r < a.n)
                     ? a.residual[(int64_t)(t0 + t) * a.n + row0 + r] : 0.0f;
    }
    cp_async_wait<0>();
    __syncthreads();
    if (PRO == PRO_OFFSET)   // the offset: 128 * in-order sum over blocks of bsum * scale
        for (int t = warp; t < T; t += GEMM_WARPS)
            if (lane == 0) offs_s[t] = fmul(chain_sum(term_s + t * bpad, blocks), 128.0f);

    // ---- the chains: chunk after chunk, D weight chunks in flight ----
    // accumulator pairs of rows (2p, 2p + 1): the exact conversion and the fmaf of both run as one
    // packed float2 add and one packed fma (each lane rounded as the scalar operation)
    static_assert(R % 2 == 0, "rows are paired");
    float2 acc[NM][R / 2][T];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int r = 0; r < R / 2; ++r)
#pragma unroll
            for (int t = 0; t < T; ++t) acc[m][r][t] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    const uint32_t *xw_s = reinterpret_cast<const uint32_t *>(xq_s) + lane;
    const float *sc_s = xs_s + (lane >> 3);
    for (int c0 = 0; c0 < chunks; c0 += D) {
#pragma unroll
        for (int s = 0; s < D; ++s) {
            const int c = c0 + s;
            if (c < chunks) {
                uint32_t cur[NM][R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    cur[0][r] = ring[s][0][r];
                    if (TWO) cur[NM - 1][r] = ring[s][NM - 1][r];
                }
                if (c + D < chunks) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        ring[s][0][r] = __ldg(w0 + roff[r] + (c + D) * 32);
                        if (TWO) ring[s][NM - 1][r] = __ldg(w1 + roff[r] + (c + D) * 32);
                    }
                }
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const uint32_t xw = xw_s[t * kw + c * 32];
                    const float sc = sc_s[t * bpad + 4 * c];
                    const float2 scv = make_float2(sc, sc);
#pragma unroll
                    for (int m = 0; m < NM; ++m)
#pragma unroll
                        for (int r = 0; r < R / 2; ++r) {
                            const float2 v = __fadd2_rn(make_float2(dp4_biased(cur[m][2 * r], xw),
                                                                    dp4_biased(cur[m][2 * r + 1], xw)), neg_magic);
                            acc[m][r][t] = __ffma2_rn(v, scv, acc[m][r][t]);
                        }
                }
            }
        }
    }
    // 32-byte groups past the last whole chunk: accumulators 0..7 (lanes 0..7)
#pragma unroll
    for (int k1 = 0; k1 < MAXG; ++k1) {
        if (k1 < groups && lane < 8) {
            const int wo = (stride + k1 * QBLOCK) / 4;
            uint32_t tw[NM][R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                tw[0][r] = __ldg(w0 + roff[r] + wo);
                if (TWO) tw[NM - 1][r] = __ldg(w1 + roff[r] + wo);
            }
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const uint32_t xw = xw_s[t * kw + wo];
                const float sc = xs_s[t * bpad + (stride / QBLOCK) + k1];
                const float2 scv = make_float2(sc, sc);
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int r = 0; r < R / 2; ++r) {
                        const float2 v = __fadd2_rn(make_float2(dp4_biased(tw[m][2 * r], xw),
                                                                dp4_biased(tw[m][2 * r + 1], xw)), neg_magic);
                        acc[m][r][t] = __ffma2_rn(v, scv, acc[m][r][t]);
                    }
            }
        }
    }

    // ---- the pairing tree, transposed across the lanes ----
    float v[NACC];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < T; ++t) v[(m * R + r) * T + t] = (r & 1) ? acc[m][r / 2][t].y : acc[m][r / 2][t].x;
    butterfly_reduce<NACC>(v, lane);
    __syncthreads();   // offsets (PRO_OFFSET) are visible from here

    // ---- epilogue: lane holds outputs o = k + P*sel, o = (m*R + r)*T + t ----
#pragma unroll
    for (int k = 0; k < P; ++k) {
        const int o = k + P * sel, t = o % T, r = (o / T) % R;
        const int row = row0 + r;
        float out = 0.0f;
        if (TWO) {
            // gate (m = 0) and up (m = 1) of the same (r, t) sit in lanes l and l ^ 8
            const float other = __shfl_xor_sync(0xffffffffu, v[k], 8);
            const bool up_lane = (lane >> 3) & 1;
            if (!up_lane && t < tn) {
                const float off = offs_s[t];
                const int rowc = min(row, a.n - 1);
                const float yg = fmul(fsub(v[k], off), a.scales[rowc]);
                const float yu = fmul(fsub(other, off), a.scales2[rowc]);
                out = swiglu(yg, yu, tab);
                if (EPI == EPI_SWIGLU && row < a.n) a.out[(int64_t)(t0 + t) * a.n + row] = out;
                if (EPI == EPI_SWIGLU_QUANT) hq_s[t * ROWS + warp * R + r] = out;
            }
        } else if (t < tn && row < a.n) {
            const float y = fmul(fsub(v[k], offs_s[t]), a.scales[row]);
            if (EPI == EPI_BIAS) out = fadd(y, a.bias[row]);
            else if (EPI == EPI_RESIDUAL) out = fadd(res[k], y);
            else out = y;
            a.out[(int64_t)(t0 + t) * a.n + row] = out;
        }
    }
    if (EPI == EPI_SWIGLU_QUANT) {
        // silu(gate) * up of whole 32-row blocks: one warp per (token, block)
        constexpr int CB = ROWS / QBLOCK;
        __syncthreads();
        for (int task = warp; task < T * CB; task += GEMM_WARPS) {
            const int t = task / CB, blk = task % CB;
            const int gb = cta_row0 / QBLOCK + blk, m = t0 + t;
            if (t < tn && gb < a.n / QBLOCK) {
                int8_t qv;
                int bs;
                const float sc = quantize_block_warp(hq_s[t * ROWS + blk * QBLOCK + lane], &qv, &bs);
                f.q_out[(int64_t)m * a.n + gb * QBLOCK + lane] = qv;
                if (lane == 0) {
                    f.xs_out[(int64_t)m * (a.n / QBLOCK) + gb] = sc;
                    f.bsums_out[(int64_t)m * (a.n / QBLOCK) + gb] = bs;
                }
            }
        }
    }
}

}  // namespace nc
