// nc_kernels.cuh -- the fused-group kernels of a Qwen2 step on sm_100a.
//
// Each kernel computes one kind of fused group of nanocompile's int8-vnni (or float32) Qwen2
// step, bit for bit: the same float32 operations in the same order as the C that
// nanocompile/fusion.py + codegen_c.py generate.  Parallelism only ever runs across
// independent results (rows, tokens, heads, accumulator lanes); every sum the reference
// forms sequentially is formed sequentially here, by one thread.
#pragma once

#include "nc_common.cuh"

namespace nc {

// ---- gather (nanocompile/fusion.py:713-731) --------------------------------------------
// One CTA per row.  An id outside 0..vocab-1 records its row in *err (atomicMin; all-ones =
// none) and leaves the row zero, where the reference returns status 1 before writing.
__global__ void gather_kernel(float *__restrict__ out, const int64_t *__restrict__ ids,
                              const float *__restrict__ table, unsigned long long *err,
                              int64_t vocab, int hidden) {
    release_dependents();
    wait_for_producer();
    const int r = blockIdx.x;
    const int64_t id = ids[r];
    float *dst = out + (int64_t)r * hidden;
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) atomicMin(err, (unsigned long long)r);
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = 0.0f;
        return;
    }
    const float *src = table + id * (int64_t)hidden;
    if ((hidden & 3) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
    }
}

// ---- block quantization of a row held in shared memory --------------------------------------
// Warp w quantizes blocks w, w + nwarps, ... (nanocompile/quantize.py:102-124), up to N of
// them at once so their divisions overlap; writes xq / xs / block sums and leaves each block's
// offset term float(sum_b) * scale_b in term[b].  With gain set, the row is first normalized on
// the way in, x * inv * gain (nanocompile/nn.py:34-38, the same two rounded products as a separate
// pass), and the normalized values also go to normed (nullable).
template <int N = 8>
__device__ __forceinline__ void quantize_row_smem(const float *row, int n, int8_t *xq, float *xs, int32_t *bsums,
                                                  float *term, int warp, int nwarps, int lane,
                                                  const float *gain = nullptr, float inv = 1.0f, float *normed = nullptr) {
    const int blocks = n / QBLOCK;
#pragma unroll 1
    for (int b0 = warp; b0 < blocks; b0 += N * nwarps) {
        float v[N], scale[N];
        int8_t q[N];
        int bs[N];
#pragma unroll
        for (int u = 0; u < N; ++u) {
            const int b = b0 + u * nwarps, i = b * QBLOCK + lane;
            v[u] = b < blocks ? row[i] : 0.0f;
            if (gain && b < blocks) {
                v[u] = fmul(fmul(v[u], inv), gain[i]);
                if (normed) normed[i] = v[u];
            }
        }
        quantize_blocks_warp<N>(v, q, scale, bs);
#pragma unroll
        for (int u = 0; u < N; ++u) {
            const int b = b0 + u * nwarps;
            if (b < blocks) {
                xq[b * QBLOCK + lane] = q[u];
                if (lane == 0) {
                    xs[b] = scale[u];
                    if (bsums) bsums[b] = bs[u];
                    term[b] = fmul((float)bs[u], scale[u]);
                }
            }
        }
    }
}

// ---- rms_norm row kernel + block quantization --------------------------------------------
// nanocompile/nn.py:34-38 as one row kernel (fusion.py:631-650): acc = acc + x*x over the row
// in order, then x * (1 / sqrtf(acc / n + eps)) * w; fused with nanocompile/quantize.py:102-124
// (block absmax, scale, xq, int32 block sums, offset = 128 * in-order sum of sum_b * scale_b).
// One CTA per output row; row_map (nullable) picks the input row.
constexpr int NORM_THREADS = 256;

// The norm of one row held in shared memory: x -> normalized, in place (squares in sq).
__device__ __forceinline__ void rms_norm_smem(float *x, float *sq, const float *w, int n, float eps, float *s_inv) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) sq[i] = fmul(x[i], x[i]);
    __syncthreads();
    if (threadIdx.x == 0) *s_inv = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(chain_sum(sq, n), (float)n), eps)));
    __syncthreads();
    const float inv = *s_inv;
    for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = fmul(fmul(x[i], inv), w[i]);
    __syncthreads();
}

__global__ void __launch_bounds__(NORM_THREADS)
norm_quant_kernel(float *__restrict__ normed, const float *__restrict__ x, const float *__restrict__ w,
                  int8_t *__restrict__ xq, float *__restrict__ xs, float *__restrict__ offset,
                  int32_t *__restrict__ bsums, const int32_t *__restrict__ row_map, int n, float eps) {
    extern __shared__ __align__(16) float smem[];
    const int n4 = (n + 3) & ~3;
    float *sq = smem;                          // [n]: squares
    float *row = smem + n4;                    // [n]: the row, then its normalized values
    float *ws = row + n4;                      // [n]: the gains
    __shared__ float s_inv;
    __shared__ __align__(16) float s_term[256];
    const int b = blockIdx.x;
    // a thread requests four values of a row at once (one round trip per 1024 values)
    // (and, with squares set, their squares x*x)
    auto stage = [&](float *dst, const float *src, float *squares) {
        for (int i0 = threadIdx.x; i0 < n; i0 += 4 * NORM_THREADS) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = i0 + u * NORM_THREADS < n ? src[i0 + u * NORM_THREADS] : 0.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (i0 + u * NORM_THREADS < n) {
                    dst[i0 + u * NORM_THREADS] = v[u];
                    if (squares) squares[i0 + u * NORM_THREADS] = fmul(v[u], v[u]);
                }
        }
    };
    release_dependents();
    stage(ws, w, nullptr);
    wait_for_producer();
    const int64_t in_row = row_map ? row_map[b] : b;
    stage(row, x + in_row * n, sq);
    __syncthreads();
    if (threadIdx.x == 0) s_inv = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(chain_sum(sq, n), (float)n), eps)));
    __syncthreads();
    const float inv = s_inv;
    float *nrow = normed ? normed + (int64_t)b * n : nullptr;
    if (!xq) {
        for (int i = threadIdx.x; i < n; i += NORM_THREADS) nrow[i] = fmul(fmul(row[i], inv), ws[i]);
        return;
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, blocks = n / QBLOCK;
    quantize_row_smem<4>(row, n, xq + (int64_t)b * n, xs + (int64_t)b * blocks, bsums ? bsums + (int64_t)b * blocks : nullptr,
                         s_term, warp, NORM_THREADS / 32, lane, ws, inv, nrow);
    __syncthreads();
    if (threadIdx.x == 0) offset[b] = fmul(chain_sum(s_term, blocks), 128.0f);
}

// Block quantization alone, one CTA (8 warps) per row; up to 256 blocks (k <= 8192).
__global__ void __launch_bounds__(NORM_THREADS)
quantize_kernel(int8_t *__restrict__ xq, const float *__restrict__ x, float *__restrict__ xs,
                float *__restrict__ offset, int32_t *__restrict__ bsums, int k) {
    extern __shared__ __align__(16) float qrow[];
    __shared__ __align__(16) float s_term[256];
    const int b = blockIdx.x;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, blocks = k / QBLOCK;
    release_dependents();
    wait_for_producer();
    for (int i = threadIdx.x; i < k; i += NORM_THREADS) qrow[i] = x[(int64_t)b * k + i];
    __syncthreads();
    quantize_row_smem(qrow, k, xq + (int64_t)b * k, xs + (int64_t)b * blocks, bsums ? bsums + (int64_t)b * blocks : nullptr,
                      s_term, warp, NORM_THREADS / 32, lane);
    __syncthreads();
    if (threadIdx.x == 0) offset[b] = fmul(chain_sum(s_term, blocks), 128.0f);
}

// ---- int8-vnni GEMV / skinny GEMM -----------------------------------------------------------
// nanocompile/lower.py:363-397: per output (token m, row n) 32 float32 accumulators; the
// 128-byte chunk k0 of the row feeds accumulator a = byte/4 with
//   acc[a] = fmaf(float(Dp4(w[4a..4a+3] + 128, x[..])), xs[block], acc[a])
// chunks in order; 32-byte groups past the last whole chunk feed accumulators 0..7; then
// _combine and (sum - offset) * scale, then the epilogue (fusion.py:699-711).
//
// LPR lanes cooperate on one row; lane j owns accumulators j*APL .. j*APL+APL-1 and reads
// the matching BPL bytes of every chunk, so each accumulator's chain stays in one lane, in
// order.  The combine is a butterfly that pairs exactly the accumulators _combine pairs.
struct GemvI8Args {
    float *out;               // [m, n]
    const int8_t *xq;         // [m, k]
    const float *xs;          // [m, k/32]
    const float *offset;      // [m]
    const uint8_t *w;         // [n, k], int8 + 128
    const float *scales;      // [n]
    const float *bias;        // EPI_BIAS: [n]
    const float *residual;    // EPI_RESIDUAL: [m, n] (may alias out)
    const uint8_t *w2;        // EPI_SWIGLU: second weight
    const float *scales2;
    int m, n, k;
};

template <int BPL>
struct Seg;
template <>
struct Seg<16> {
    using T = uint4;
    __device__ static void split(const T &v, uint32_t *o) { o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w; }
};
template <>
struct Seg<8> {
    using T = uint2;
    __device__ static void split(const T &v, uint32_t *o) { o[0] = v.x; o[1] = v.y; }
};
template <>
struct Seg<4> {
    using T = uint32_t;
    __device__ static void split(const T &v, uint32_t *o) { o[0] = v; }
};
struct alignas(16) U32x8 {
    uint4 lo, hi;
};
template <>
struct Seg<32> {
    using T = U32x8;
    __device__ static void split(const T &v, uint32_t *o) {
        o[0] = v.lo.x; o[1] = v.lo.y; o[2] = v.lo.z; o[3] = v.lo.w;
        o[4] = v.hi.x; o[5] = v.hi.y; o[6] = v.hi.z; o[7] = v.hi.w;
    }
};

// Butterfly over the accumulator index bits in _combine's pairing order: a^8, a^16, a^4,
// a^1, a^2.  Bits below log2(APL) are inside a lane, the rest across lanes (xor shuffle).
template <int APL>
__device__ __forceinline__ float combine_lanes(float *v) {
    constexpr int LG = APL == 8 ? 3 : (APL == 4 ? 2 : (APL == 2 ? 1 : 0));
    const int order[5] = {3, 4, 2, 0, 1};
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int bit = order[s];
        if (bit < LG) {
#pragma unroll
            for (int i = 0; i < APL; ++i)
                if (!(i & (1 << bit))) v[i] = fadd(v[i], v[i | (1 << bit)]);
        } else {
            const int lane_bit = 1 << (bit - LG);
#pragma unroll
            for (int i = 0; i < APL; ++i) v[i] = fadd(v[i], __shfl_xor_sync(0xffffffffu, v[i], lane_bit));
        }
    }
    return v[0];
}

template <int LPR, int TOK, int UNROLL, int EPI>
__global__ void __launch_bounds__(128)
gemv_i8_kernel(GemvI8Args a) {
    constexpr int RPW = 32 / LPR;     // rows per warp
    constexpr int BPL = 128 / LPR;    // bytes of a chunk per lane
    constexpr int APL = BPL / 4;      // accumulators per lane
    constexpr bool TWO = EPI == EPI_SWIGLU;
    using SegT = typename Seg<BPL>::T;
    __shared__ uint64_t tab[32];
    release_dependents();
    wait_for_producer();
    if (EPI == EPI_SWIGLU) {
        if (threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];
        __syncthreads();
    }
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int grp = lane / LPR, j = lane % LPR;
    const int row = (blockIdx.x * (blockDim.x / 32) + warp) * RPW + grp;
    const bool row_ok = row < a.n;
    const int rowc = row_ok ? row : a.n - 1;
    const int K = a.k, blocks = K / QBLOCK;
    const int chunks = K / CHUNK, stride = chunks * CHUNK, groups = (K % CHUNK) / 32;
    const uint8_t *wrow = a.w + (int64_t)rowc * K;
    const uint8_t *wrow2 = TWO ? a.w2 + (int64_t)rowc * K : nullptr;

    for (int m0 = 0; m0 < a.m; m0 += TOK) {
        float acc[TOK][APL], acc2[TWO ? TOK : 1][APL];
#pragma unroll
        for (int t = 0; t < TOK; ++t)
#pragma unroll
            for (int i = 0; i < APL; ++i) {
                acc[t][i] = 0.0f;
                if (TWO) acc2[t][i] = 0.0f;
            }
        // whole 128-byte chunks, UNROLL at a time so the weight loads are in flight together
        for (int c0 = 0; c0 < chunks; c0 += UNROLL) {
            uint32_t wv[UNROLL][APL], wv2[TWO ? UNROLL : 1][APL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                if (c0 + u < chunks) {
                    const int off = (c0 + u) * CHUNK + j * BPL;
                    Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow + off)), wv[u]);
                    if (TWO) Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow2 + off)), wv2[u]);
                }
            }
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
                const int m = m0 + t;
                if (m >= a.m) break;
                const int8_t *xrow = a.xq + (int64_t)m * K;
                const float *xsr = a.xs + (int64_t)m * blocks;
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    if (c0 + u < chunks) {
                        const int off = (c0 + u) * CHUNK + j * BPL;
                        uint32_t xv[APL];
                        Seg<BPL>::split(*reinterpret_cast<const SegT *>(xrow + off), xv);
                        const float s = xsr[off / QBLOCK];
#pragma unroll
                        for (int i = 0; i < APL; ++i) {
                            acc[t][i] = __fmaf_rn(dp4_lane(wv[u][i], xv[i]), s, acc[t][i]);
                            if (TWO) acc2[t][i] = __fmaf_rn(dp4_lane(wv2[u][i], xv[i]), s, acc2[t][i]);
                        }
                    }
                }
            }
        }
        // leftover 32-byte groups: into accumulators 0..7, group after group
        if (groups && j * BPL < 32) {
            for (int k1 = 0; k1 < groups; ++k1) {
                const int off = stride + k1 * 32 + j * BPL;
                uint32_t wv[APL], wv2[APL];
                Seg<BPL>::split(*reinterpret_cast<const SegT *>(wrow + off), wv);
                if (TWO) Seg<BPL>::split(*reinterpret_cast<const SegT *>(wrow2 + off), wv2);
#pragma unroll
                for (int t = 0; t < TOK; ++t) {
                    const int m = m0 + t;
                    if (m >= a.m) break;
                    uint32_t xv[APL];
                    Seg<BPL>::split(*reinterpret_cast<const SegT *>(a.xq + (int64_t)m * K + off), xv);
                    const float s = a.xs[(int64_t)m * blocks + off / QBLOCK];
#pragma unroll
                    for (int i = 0; i < APL; ++i) {
                        acc[t][i] = __fmaf_rn(dp4_lane(wv[i], xv[i]), s, acc[t][i]);
                        if (TWO) acc2[t][i] = __fmaf_rn(dp4_lane(wv2[i], xv[i]), s, acc2[t][i]);
                    }
                }
            }
        }
        // combine, scale, epilogue
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
            const int m = m0 + t;
            if (m >= a.m) break;
            const float sum = combine_lanes<APL>(acc[t]);
            float sum2 = 0.0f;
            if (TWO) sum2 = combine_lanes<APL>(acc2[t]);
            if (j == 0 && row_ok) {
                const float off = a.offset[m];
                const float y = fmul(fsub(sum, off), a.scales[row]);
                float out;
                if (EPI == EPI_BIAS) {
                    out = fadd(y, a.bias[row]);
                } else if (EPI == EPI_RESIDUAL) {
                    out = fadd(a.residual[(int64_t)m * a.n + row], y);
                } else if (EPI == EPI_SWIGLU) {
                    const float y1 = fmul(fsub(sum2, off), a.scales2[row]);
                    out = swiglu(y, y1, tab);
                } else {
                    out = y;
                }
                a.out[(int64_t)m * a.n + row] = out;
            }
        }
    }
}

// Weights-stationary fused projection.  Each lane loads its BPL-byte slice of every chunk of
// its row into registers first (NCH chunks at most) -- the weights cross HBM once per step,
// and their latency overlaps the prologue.  Then per token: the Dp4 chains, the combine, the
// epilogue.  The activations come from one of three prologues:
//   PRO_NONE   xq / xs / offset in global memory (written by an earlier kernel);
//   PRO_NORM   the CTA computes rms_norm + block quantization of x itself (rows <= 4): the
//              input-norm / post-attention-norm row kernel and calls 2-7, fused in front;
//   PRO_OFFSET xq / xs / block sums in global memory, the offset (128 * in-order sum over
//              blocks of sum_b * scale_b) formed here.
// EPI_SWIGLU_QUANT is silu(gate) * up followed by the block quantization of that output
// (calls 33-38): the CTA owns whole 32-row blocks and writes xq / xs / block sums.
enum Prologue : int { PRO_NONE = 0, PRO_NORM = 1, PRO_OFFSET = 2 };
constexpr int EPI_SWIGLU_QUANT = 4;
constexpr int PRO_NORM_ROWS = 4;

struct FusedI8Args {
    GemvI8Args g;
    const float *x;            // PRO_NORM: the residual stream [m, k]
    const float *norm_w;       // PRO_NORM: gains [k]
    float eps;
    const int32_t *bsums_in;   // PRO_OFFSET: block sums [m, k/32]
    int8_t *q_out;             // EPI_SWIGLU_QUANT: xq / xs / block sums of the output [m, n]
    float *xs_out;
    int32_t *bsums_out;
};

// Shared-memory budget for the activations of one token tile (xq rows + their block scales).
constexpr int ACT_TILE_BYTES = 64 * 1024;

__host__ __device__ inline int act_tile_tokens(int k) { return ACT_TILE_BYTES / (k + 4 * (k / QBLOCK)); }

template <int LPR, int NCH, int MAXG, int PRO, int EPI, int TB>
__global__ void __launch_bounds__(256, (EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_QUANT) ? 2 : 1)
gemv_i8_fused_kernel(FusedI8Args f) {
    // MAXG: 32-byte groups past the last whole chunk (0 when the width is whole chunks).
    // TB: tokens advanced together (independent chains in flight; 1 for a single token).
    constexpr int BPL = 128 / LPR;
    constexpr int APL = BPL / 4;
    constexpr bool TWO = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_QUANT;
    constexpr bool XPRE = !TWO && TB == 1;  // activations of all chunks into registers first
    using SegT = typename Seg<BPL>::T;
    const GemvI8Args &a = f.g;
    extern __shared__ __align__(16) float dsm[];
    __shared__ uint64_t tab[32];
    __shared__ float s_inv;
    __shared__ float hq[TB][32 * 8];
    const int nwarps = blockDim.x / 32;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int grp = lane / LPR, j = lane % LPR;
    const int row0 = blockIdx.x * nwarps * (32 / LPR);
    const int row = row0 + warp * (32 / LPR) + grp;
    const bool row_ok = row < a.n;
    const int rowc = row_ok ? row : a.n - 1;
    const int K = a.k, blocks = K / QBLOCK, bl4 = (blocks + 3) & ~3;
    const int chunks = K / CHUNK, stride = chunks * CHUNK, groups = (K % CHUNK) / 32;
    const bool tail_lane = j * BPL < 32;
    const uint8_t *wrow = a.w + (int64_t)rowc * K;
    const uint8_t *wrow2 = TWO ? a.w2 + (int64_t)rowc * K : nullptr;
    if (TWO && threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];

    // ---- what does not depend on the previous kernel: this row's weights and constants ----
    release_dependents();
    uint32_t wv[NCH][APL], wv2[TWO ? NCH : 1][APL], tw[MAXG ? MAXG : 1][APL], tw2[TWO && MAXG ? MAXG : 1][APL];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        if (c < chunks) {
            Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow + c * CHUNK + j * BPL)), wv[c]);
            if (TWO) Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow2 + c * CHUNK + j * BPL)), wv2[c]);
        }
    }
#pragma unroll
    for (int k1 = 0; k1 < MAXG; ++k1) {
        if (k1 < groups && tail_lane) {
            Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow + stride + k1 * 32 + j * BPL)), tw[k1]);
            if (TWO) Seg<BPL>::split(__ldcs(reinterpret_cast<const SegT *>(wrow2 + stride + k1 * 32 + j * BPL)), tw2[k1]);
        }
    }
    const float scale = a.scales[rowc];
    const float scale2 = TWO ? a.scales2[rowc] : 0.0f;
    const float bias = EPI == EPI_BIAS ? a.bias[rowc] : 0.0f;

    // dsm layout: [activation tile: xq rows | xs rows] [prologue scratch]
    const int tile_tokens = PRO == PRO_NORM ? PRO_NORM_ROWS : min(a.m, act_tile_tokens(K));
    int8_t *xq_t = reinterpret_cast<int8_t *>(dsm);
    float *xs_t = dsm + tile_tokens * K / 4;
    float *scratch = xs_t + tile_tokens * bl4;
    float *offs = scratch;                       // [m]
    float *term = offs + ((a.m + 3) & ~3);       // PRO_OFFSET: [m][bl4]; PRO_NORM: [bl4]
    float *xrow = term + bl4, *sq = xrow + K, *gains = sq + K;   // PRO_NORM only
    if (PRO == PRO_NORM)
        for (int i = threadIdx.x; i < K; i += blockDim.x) gains[i] = f.norm_w[i];

    wait_for_producer();

    // ---- prologue: the offsets (and for PRO_NORM the whole quantized activations) ----
    if (PRO == PRO_NORM) {
        for (int m = 0; m < a.m; ++m) {
            for (int i = threadIdx.x; i < K; i += blockDim.x) xrow[i] = f.x[(int64_t)m * K + i];
            __syncthreads();
            rms_norm_smem(xrow, sq, gains, K, f.eps, &s_inv);
            quantize_row_smem(xrow, K, xq_t + m * K, xs_t + m * bl4, nullptr, term, warp, nwarps, lane);
            __syncthreads();
            if (threadIdx.x == 0) offs[m] = fmul(chain_sum(term, blocks), 128.0f);
            __syncthreads();
        }
    } else if (PRO == PRO_OFFSET) {
        for (int i = threadIdx.x; i < a.m * blocks; i += blockDim.x) {
            const int m = i / blocks, b = i % blocks;
            term[m * bl4 + b] = fmul((float)f.bsums_in[i], a.xs[i]);
        }
        __syncthreads();
        for (int m = threadIdx.x; m < a.m; m += blockDim.x) offs[m] = fmul(chain_sum(term + m * bl4, blocks), 128.0f);
    } else {
        for (int m = threadIdx.x; m < a.m; m += blockDim.x) offs[m] = a.offset[m];
    }

    for (int t0 = 0; t0 < a.m; t0 += tile_tokens) {
        const int tn = min(tile_tokens, a.m - t0);
        if (PRO != PRO_NORM) {
            // stage this tile's activations: xq rows (16-byte pieces) and block scales
            __syncthreads();
            const int pieces = tn * K / 16;
            for (int i = threadIdx.x; i < pieces; i += blockDim.x)
                reinterpret_cast<uint4 *>(xq_t)[i] = reinterpret_cast<const uint4 *>(a.xq + (int64_t)t0 * K)[i];
            for (int i = threadIdx.x; i < tn * blocks; i += blockDim.x)
                xs_t[(i / blocks) * bl4 + i % blocks] = a.xs[(int64_t)t0 * blocks + i];
        }
        __syncthreads();
        for (int tm = 0; tm < tn; tm += TB) {
            float acc[TB][APL], acc2[TB][APL];
#pragma unroll
            for (int b = 0; b < TB; ++b)
#pragma unroll
                for (int i = 0; i < APL; ++i) { acc[b][i] = 0.0f; acc2[b][i] = 0.0f; }
            uint32_t xv[XPRE ? NCH : 1][APL];
            float sv[XPRE ? NCH : 1];
            if (XPRE) {
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    if (c < chunks) {
                        const int off = c * CHUNK + j * BPL;
                        Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq_t + tm * K + off), xv[c]);
                        sv[c] = xs_t[tm * bl4 + off / QBLOCK];
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                if (c < chunks) {
                    const int off = c * CHUNK + j * BPL;
#pragma unroll
                    for (int b = 0; b < TB; ++b) {
                        if (tm + b < tn) {
                            uint32_t xc[APL];
                            float sc;
                            if (XPRE) {
#pragma unroll
                                for (int i = 0; i < APL; ++i) xc[i] = xv[XPRE ? c : 0][i];
                                sc = sv[XPRE ? c : 0];
                            } else {
                                Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq_t + (tm + b) * K + off), xc);
                                sc = xs_t[(tm + b) * bl4 + off / QBLOCK];
                            }
#pragma unroll
                            for (int i = 0; i < APL; ++i) {
                                acc[b][i] = __fmaf_rn(dp4_lane(wv[c][i], xc[i]), sc, acc[b][i]);
                                if (TWO) acc2[b][i] = __fmaf_rn(dp4_lane(wv2[c][i], xc[i]), sc, acc2[b][i]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int k1 = 0; k1 < MAXG; ++k1) {
                if (k1 < groups && tail_lane) {
                    const int off = stride + k1 * 32 + j * BPL;
#pragma unroll
                    for (int b = 0; b < TB; ++b) {
                        if (tm + b < tn) {
                            uint32_t tx[APL];
                            Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq_t + (tm + b) * K + off), tx);
                            const float s = xs_t[(tm + b) * bl4 + off / QBLOCK];
#pragma unroll
                            for (int i = 0; i < APL; ++i) {
                                acc[b][i] = __fmaf_rn(dp4_lane(tw[MAXG ? k1 : 0][i], tx[i]), s, acc[b][i]);
                                if (TWO) acc2[b][i] = __fmaf_rn(dp4_lane(tw2[TWO && MAXG ? k1 : 0][i], tx[i]), s, acc2[b][i]);
                            }
                        }
                    }
                }
            }
            // the residuals of these tokens, requested before the combine
            float res[TB];
#pragma unroll
            for (int b = 0; b < TB; ++b) {
                const int m = t0 + tm + b;
                res[b] = (EPI == EPI_RESIDUAL && j == 0 && tm + b < tn) ? a.residual[(int64_t)m * a.n + rowc] : 0.0f;
            }
            float sum[TB], sum2[TB];
#pragma unroll
            for (int b = 0; b < TB; ++b) {
                sum[b] = combine_lanes<APL>(acc[b]);
                sum2[b] = TWO ? combine_lanes<APL>(acc2[b]) : 0.0f;
            }
#pragma unroll
            for (int b = 0; b < TB; ++b) {
                const int m = t0 + tm + b;
                float out = 0.0f;
                if (j == 0 && tm + b < tn) {
                    const float off = offs[m];
                    const float y = fmul(fsub(sum[b], off), scale);
                    if (EPI == EPI_BIAS) out = fadd(y, bias);
                    else if (EPI == EPI_RESIDUAL) out = fadd(res[b], y);
                    else if (TWO) out = swiglu(y, fmul(fsub(sum2[b], off), scale2), tab);
                    else out = y;
                    if (EPI != EPI_SWIGLU_QUANT && row_ok) a.out[(int64_t)m * a.n + row] = out;
                }
                if (EPI == EPI_SWIGLU_QUANT && j == 0) hq[b][row - row0] = out;
            }
            if (EPI == EPI_SWIGLU_QUANT) {
                // the CTA's rows are whole blocks: one warp per (token, block)
                const int rows_cta = nwarps * (32 / LPR), cblocks = rows_cta / QBLOCK;
                __syncthreads();
                for (int wb = warp; wb < TB * cblocks; wb += nwarps) {
                    const int b = wb / cblocks, blk = wb % cblocks;
                    const int gb = row0 / QBLOCK + blk, m = t0 + tm + b;
                    if (tm + b < tn && gb < a.n / QBLOCK) {
                        int8_t qv;
                        int bs;
                        const float sc = quantize_block_warp(hq[b][blk * QBLOCK + lane], &qv, &bs);
                        f.q_out[(int64_t)m * a.n + gb * QBLOCK + lane] = qv;
                        if (lane == 0) {
                            f.xs_out[(int64_t)m * (a.n / QBLOCK) + gb] = sc;
                            f.bsums_out[(int64_t)m * (a.n / QBLOCK) + gb] = bs;
                        }
                    }
                }
                __syncthreads();
            }
        }
    }
}

// ---- float32 GEMV with in-order sums (projections of float32 models, and the LM head) -------
// nanocompile/lower.py:255-274: acc = acc + x[k] * w[n, k], k = 0, 1, 2, ... -- one thread owns
// one row n and walks k in order.  Rows are staged through shared memory in 32-column tiles
// by cp.async (16-byte pieces, XOR-swizzled so a thread reading its own row is conflict-free),
// STAGES tiles in flight.  With ARGMAX the kernel also reduces each token's logits to the
// index of the first maximum (np.argmax, nanocompile/models/qwen2.py:364).
constexpr int F32_ROWS = 128;
constexpr int F32_TILE = 32;
constexpr int F32_STAGES = 4;

struct GemvF32Args {
    float *out;               // [m, n] (nullable with ARGMAX)
    const float *x;           // [m, k] (row_map picks rows)
    const float *w;           // [n, k]
    const float *bias, *residual, *w2;
    const int32_t *row_map;   // nullable
    float *part_val;          // ARGMAX scratch [m, gridDim.x]
    int32_t *part_idx;
    unsigned int *counter;    // ARGMAX: CTAs finished (reset by the last one)
    int64_t *tokens;          // ARGMAX: [m]
    int m, n, k;
};

__device__ __forceinline__ bool argmax_better(float va, int ia, float vb, int ib) {
    const bool na = va != va, nb = vb != vb;
    if (na || nb) return na && (!nb || ia < ib);
    if (va != vb) return va > vb;
    return ia < ib;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

template <int TOK, int EPI, bool ARGMAX>
__global__ void __launch_bounds__(F32_ROWS)
gemv_f32_kernel(GemvF32Args a) {
    constexpr bool TWO = EPI == EPI_SWIGLU;
    constexpr int NW = TWO ? 2 : 1;
    extern __shared__ float4 smem4[];
    // per stage: NW weight tiles [128 rows][8 pieces of 4 floats], then the x tile [TOK][32]
    constexpr int W_PIECES = F32_ROWS * (F32_TILE / 4);
    constexpr int STAGE_F4 = NW * W_PIECES + TOK * (F32_TILE / 4);
    __shared__ uint64_t tab[32];
    if (TWO) {
        if (threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];
    }
    const int t = threadIdx.x;
    const int row0 = blockIdx.x * F32_ROWS;
    const int row = row0 + t;
    const int K = a.k, tiles = K / F32_TILE;

    auto load_w = [&](int stage, int kt) {
        float4 *st = smem4 + stage * STAGE_F4;
#pragma unroll
        for (int p = 0; p < NW * W_PIECES / F32_ROWS; ++p) {
            const int id = t + p * F32_ROWS;             // piece id within the NW tiles
            const int which = id / W_PIECES, rem = id % W_PIECES;
            const int r = rem / 8, s = rem % 8;
            const int gr = min(row0 + r, a.n - 1);
            const float *src = (which ? a.w2 : a.w) + (int64_t)gr * K + kt * F32_TILE + s * 4;
            cp_async16(st + which * W_PIECES + r * 8 + (s ^ (r & 7)), src);
        }
    };
    auto load_x = [&](int stage, int kt, int m0) {
        float4 *st = smem4 + stage * STAGE_F4;
        if (t < TOK * 8) {
            const int mm = t / 8, s = t % 8;
            const int m = min(m0 + mm, a.m - 1);
            const int64_t xr = a.row_map ? a.row_map[m] : m;
            cp_async16(st + NW * W_PIECES + mm * 8 + s, a.x + xr * K + kt * F32_TILE + s * 4);
        }
    };
    auto load_tile = [&](int stage, int kt, int m0) {
        load_w(stage, kt);
        load_x(stage, kt, m0);
    };

    // the weights of the first tiles do not depend on the previous kernel: issue them first
    release_dependents();
#pragma unroll
    for (int s = 0; s < F32_STAGES - 1; ++s)
        if (s < tiles) load_w(s, s);
    wait_for_producer();
    bool prefetched = true;

    for (int m0 = 0; m0 < a.m; m0 += TOK) {
        float acc[TOK], acc2[TWO ? TOK : 1];
#pragma unroll
        for (int i = 0; i < TOK; ++i) {
            acc[i] = 0.0f;
            if (TWO) acc2[i] = 0.0f;
        }
#pragma unroll
        for (int s = 0; s < F32_STAGES - 1; ++s) {
            if (s < tiles) {
                if (!prefetched) load_w(s, s);
                load_x(s, s, m0);
            }
            cp_async_commit();
        }
        prefetched = false;
        for (int kt = 0; kt < tiles; ++kt) {
            cp_async_wait<F32_STAGES - 2>();
            __syncthreads();
            const int nxt = kt + F32_STAGES - 1;
            if (nxt < tiles) load_tile(nxt % F32_STAGES, nxt, m0);
            cp_async_commit();
            const float4 *st = smem4 + (kt % F32_STAGES) * STAGE_F4;
            const float4 *xt = st + NW * W_PIECES;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                const float4 wv = st[t * 8 + (s ^ (t & 7))];
                float4 wv2 = wv;
                if (TWO) wv2 = st[W_PIECES + t * 8 + (s ^ (t & 7))];
#pragma unroll
                for (int i = 0; i < TOK; ++i) {
                    const float4 xv = xt[i * 8 + s];
                    acc[i] = fadd(acc[i], fmul(xv.x, wv.x));
                    acc[i] = fadd(acc[i], fmul(xv.y, wv.y));
                    acc[i] = fadd(acc[i], fmul(xv.z, wv.z));
                    acc[i] = fadd(acc[i], fmul(xv.w, wv.w));
                    if (TWO) {
                        acc2[i] = fadd(acc2[i], fmul(xv.x, wv2.x));
                        acc2[i] = fadd(acc2[i], fmul(xv.y, wv2.y));
                        acc2[i] = fadd(acc2[i], fmul(xv.z, wv2.z));
                        acc2[i] = fadd(acc2[i], fmul(xv.w, wv2.w));
                    }
                }
            }
        }
        cp_async_wait<0>();
        __syncthreads();
        // epilogue
#pragma unroll
        for (int i = 0; i < TOK; ++i) {
            const int m = m0 + i;
            if (m >= a.m) break;
            if (row < a.n) {
                float y = acc[i];
                if (EPI == EPI_BIAS) y = fadd(y, a.bias[row]);
                if (EPI == EPI_RESIDUAL) y = fadd(a.residual[(int64_t)m * a.n + row], y);
                if (EPI == EPI_SWIGLU) y = swiglu(y, acc2[i], tab);
                if (a.out) a.out[(int64_t)m * a.n + row] = y;
            }
            if (ARGMAX) {
                float v = row < a.n ? acc[i] : __uint_as_float(0xff800000u);
                int idx = row < a.n ? row : 0x7fffffff;
                if (row >= a.n) v = -__uint_as_float(0x7f800000u);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
                    if (argmax_better(ov, oi, v, idx)) { v = ov; idx = oi; }
                }
                __shared__ float wv[F32_ROWS / 32];
                __shared__ int wi[F32_ROWS / 32];
                if ((t & 31) == 0) { wv[t / 32] = v; wi[t / 32] = idx; }
                __syncthreads();
                if (t == 0) {
                    for (int q = 1; q < F32_ROWS / 32; ++q)
                        if (argmax_better(wv[q], wi[q], v, idx)) { v = wv[q]; idx = wi[q]; }
                    a.part_val[(int64_t)m * gridDim.x + blockIdx.x] = v;
                    a.part_idx[(int64_t)m * gridDim.x + blockIdx.x] = idx;
                }
                __syncthreads();
            }
        }
    }
    if (ARGMAX) {
        // the last CTA to finish reduces the per-CTA winners, in CTA order
        __shared__ bool last;
        __threadfence();
        __syncthreads();
        if (t == 0) last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            for (int m = t / 32; m < a.m; m += F32_ROWS / 32) {
                float v = -__uint_as_float(0x7f800000u);
                int idx = 0x7fffffff;
                for (int c = t % 32; c < (int)gridDim.x; c += 32) {
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
                if ((t & 31) == 0) a.tokens[m] = idx;
            }
            if (t == 0) *a.counter = 0u;
        }
    }
}

// ---- RoPE + KV append + decode attention ----------------------------------------------------
// One CTA per (row, query head).  q and k get RoPE exactly as the fused elementwise kernel does
// it (nanocompile/nn.py:97-106: t1 = y + b, t1*cos + rot(t1)*sin; the bias is already in qkv);
// the first head of each KV group writes the new k and v to the cache; then
// (nanocompile/models/qwen2.py:143-150, nn.py:57-66): scores acc = acc + q*k over d in order,
// t = score * scale + 0, NaN-propagating max, in-order sum of expf(t - max),
// p = expf(t - max) / sum, ctx = in-order sum over positions of p * v.  The two position-long
// sums are single-thread chains (chain_sum); V is staged through shared memory in chunks by
// cp.async, several chunks ahead of the chain that consumes them.
// Positions after the row's own are masked in the reference (-inf, so exp = 0 and they add
// exact zeros); they are skipped here, which is the same result for finite inputs.
struct AttnArgs {
    float *ctx;                // [rows, heads*d]
    const float *qkv;          // [rows, (heads + 2*kv)*d]
    float *cache;              // this layer, slot 0: [{K,V}][kv][cap][d]; slot stride below
    const float *cos_tab, *sin_tab;   // [cap, d/2]
    const int32_t *slot, *pos;
    int64_t slot_stride;
    int heads, kv, d, cap;
    float scale;
    int mode;                  // 0: rope + append + attend (decode); 1: rope + append only; 2: attend only
    int8_t *q_out;             // nullable: block-quantize ctx (d % 32 == 0) into xq / xs / block sums
    float *xs_out;
    int32_t *bsums_out;
    int64_t cache_row0;        // grouped kernel with a tensor map: the map's row of cache[0]
};

constexpr int ATTN_CHUNK = 128;      // positions per staged K or V chunk
constexpr int ATTN_STAGES = 3;
constexpr int ATTN_MAX_GROUP = 8;    // query heads per KV head

__host__ __device__ constexpr int attention_threads(int heads_per_cta) { return 64 * (heads_per_cta < 2 ? 2 : heads_per_cta); }

template <int D>
__host__ __device__ constexpr size_t attention_smem_floats(int heads_per_cta, int cap) {
    return (size_t)ATTN_STAGES * ATTN_CHUNK * D + (size_t)heads_per_cta * (((size_t)cap + 3) & ~(size_t)3) +
           (size_t)(heads_per_cta + 2) * D;
}

// One CTA per (row, G query heads that share one KV head; repeat_kv, nanocompile/nn.py:109-120).
// G = 1 spreads a decode step's heads over as many SMs as there are heads; G = the group size
// reads each KV head's rows once for all its query heads (large batches).  K chunks, then V
// chunks, stream through a ring of shared-memory stages by cp.async, XOR-swizzled by 16-byte
// piece so a thread reading one position's row does not bank-conflict with its neighbours.
template <int D, int G>
__global__ void __launch_bounds__(attention_threads(G))
attention_kernel(AttnArgs a) {
    constexpr int T = attention_threads(G);
    constexpr int PPR = D / 4;                       // 16-byte pieces per row
    constexpr int HALF = D / 2;
    extern __shared__ __align__(16) float sm[];
    release_dependents();
    wait_for_producer();
    const int group = a.heads / a.kv;
    const int ctas_per_row = a.heads / G;
    const int r = blockIdx.x / ctas_per_row, h0 = (blockIdx.x % ctas_per_row) * G, g = h0 / group;
    const bool owner = h0 % group == 0;              // the CTA that writes this KV head's new row
    const int pos = a.pos[r], len = pos + 1;
    const int cap4 = (a.cap + 3) & ~3;
    float4 *ring = reinterpret_cast<float4 *>(sm);                 // [STAGES][CHUNK][PPR]
    float *e = sm + ATTN_STAGES * ATTN_CHUNK * D;                  // [G][cap4]
    float *q = e + G * cap4;                                       // [G][D]
    float *kn = q + G * D, *vn = kn + D;                           // [D] each
    __shared__ uint64_t tab[32];
    __shared__ float s_max[G], s_sum[G];
    __shared__ float wmax[T / 32][1];
    const int t = threadIdx.x;
    if (t < 32) tab[t] = kExpTab[t];

    float *base = a.cache + (int64_t)a.slot[r] * a.slot_stride;
    float *K = base + (int64_t)g * a.cap * D;
    float *V = base + ((int64_t)a.kv + g) * a.cap * D;
    const float *qkv = a.qkv + (int64_t)r * (a.heads + 2 * a.kv) * D;
    const float *cs = a.cos_tab + (int64_t)pos * HALF, *sn = a.sin_tab + (int64_t)pos * HALF;

    // RoPE of the CTA's q heads and of the new k; the new v
    for (int i = t; i < (G + 2) * D; i += T) {
        const int h = i / D, c = i % D;
        const float *src = h < G ? qkv + (h0 + h) * D : (h == G ? qkv + (a.heads + g) * D : qkv + (a.heads + a.kv + g) * D);
        if (h == G + 1) {
            vn[c] = src[c];
            continue;
        }
        const float t1 = src[c];
        const float rot = c < HALF ? -src[c + HALF] : src[c - HALF];
        const float v = fadd(fmul(t1, cs[c % HALF]), fmul(rot, sn[c % HALF]));
        if (h < G) q[h * D + c] = v;
        else kn[c] = v;
    }
    __syncthreads();
    if (a.mode != 2) {
        if (owner)
            for (int c = t; c < D; c += T) {
                K[(int64_t)pos * D + c] = kn[c];
                V[(int64_t)pos * D + c] = vn[c];
            }
        if (a.mode == 1) return;
    }
    const bool own_new = a.mode == 0;       // position pos comes from kn / vn, not the cache

    const int nk = (len + ATTN_CHUNK - 1) / ATTN_CHUNK;
    // K chunks are XOR-swizzled by piece (a scoring thread reads a whole row); V chunks are plain
    // (a warp reads consecutive dimensions of one row).
    auto stage = [&](int idx) {             // chunk idx < nk: K chunk idx; else V chunk idx - nk
        if (idx < 2 * nk) {
            const bool is_k = idx < nk;
            const float *src = is_k ? K : V;
            const int j0 = (is_k ? idx : idx - nk) * ATTN_CHUNK;
            float4 *dst = ring + (idx % ATTN_STAGES) * ATTN_CHUNK * PPR;
            for (int pc = t; pc < ATTN_CHUNK * PPR; pc += T) {
                const int row = pc / PPR, col = pc % PPR;
                if (j0 + row < len)
                    cp_async16(dst + row * PPR + (is_k ? (col ^ (row % PPR)) : col), src + (int64_t)(j0 + row) * D + col * 4);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int i = 0; i < ATTN_STAGES - 1; ++i) stage(i);

    // scores: thread t scores head t / SPH's positions t % SPH, t % SPH + SPH, ... of each chunk,
    // with its head's q in registers
    constexpr int SPH = (T / G) / 32 * 32 >= ATTN_CHUNK ? ATTN_CHUNK : (T / G) / 32 * 32;   // whole warps per head
    const int hh = t / SPH, pl = t % SPH;
    const bool scorer = hh < G;
    float4 qr[PPR];
#pragma unroll
    for (int c = 0; c < PPR; ++c) qr[c] = reinterpret_cast<const float4 *>(q + (scorer ? hh : 0) * D)[c];
    float mx = __uint_as_float(0xff800000u);
    for (int ci = 0; ci < nk; ++ci) {
        cp_async_wait<ATTN_STAGES - 2>();
        __syncthreads();
        stage(ci + ATTN_STAGES - 1);
        const float4 *ck = ring + (ci % ATTN_STAGES) * ATTN_CHUNK * PPR;
        if (scorer) {
            for (int row = pl; row < ATTN_CHUNK; row += SPH) {
                const int j = ci * ATTN_CHUNK + row;
                if (j >= len) break;
                const bool fresh = own_new && j == pos;
                float acc = 0.0f;
#pragma unroll
                for (int c = 0; c < PPR; ++c) {
                    const float4 kv4 = fresh ? reinterpret_cast<const float4 *>(kn)[c] : ck[row * PPR + (c ^ (row % PPR))];
                    acc = fadd(acc, fmul(qr[c].x, kv4.x));
                    acc = fadd(acc, fmul(qr[c].y, kv4.y));
                    acc = fadd(acc, fmul(qr[c].z, kv4.z));
                    acc = fadd(acc, fmul(qr[c].w, kv4.w));
                }
                const float sc = fadd(fmul(acc, a.scale), 0.0f);
                e[hh * cap4 + j] = sc;
                mx = nan_max(mx, sc);
            }
        }
    }
    // per-head maxima: the warps of each head's scoring threads
    mx = warp_nan_max(mx);
    if ((t & 31) == 0) wmax[t / 32][0] = mx;
    __syncthreads();
    if (t < G) {
        constexpr int WPH = SPH / 32 > 0 ? SPH / 32 : 1;
        float m = wmax[t * WPH][0];
        for (int w = 1; w < WPH; ++w) m = nan_max(m, wmax[t * WPH + w][0]);
        s_max[t] = m;
    }
    __syncthreads();
    for (int i = t; i < G * len; i += T) {
        const int h = i / len, j = i % len;
        e[h * cap4 + j] = expf_exact(fsub(e[h * cap4 + j], s_max[h]), tab);
    }
    __syncthreads();
    if (t < G) s_sum[t] = chain_sum(e + t * cap4, len);           // the in-order sums
    __syncthreads();
    for (int i = t; i < G * len; i += T) {
        const int h = i / len, j = i % len;
        e[h * cap4 + j] = fdiv(e[h * cap4 + j], s_sum[h]);
    }

    // probabilities @ V: thread t owns (head t / D, dimension t % D), positions in order
    const int ph = t / D, dim = t % D;
    const bool pv = ph < G;
    float acc = 0.0f;
    for (int ci = 0; ci < nk; ++ci) {
        const int idx = nk + ci;
        cp_async_wait<ATTN_STAGES - 2>();
        __syncthreads();
        stage(idx + ATTN_STAGES - 1);
        if (pv) {
            const float *cv = reinterpret_cast<const float *>(ring + (idx % ATTN_STAGES) * ATTN_CHUNK * PPR) + dim;
            const float *p = e + ph * cap4 + ci * ATTN_CHUNK;
            const int n = min(ATTN_CHUNK, len - ci * ATTN_CHUNK);
            const bool last = ci == nk - 1;
            const int stop = (own_new && last) ? n - 1 : n;           // the new row comes from vn
            int jj = 0;
            for (; jj + 8 <= stop; jj += 8) {
                const float4 p0 = *reinterpret_cast<const float4 *>(p + jj);
                const float4 p1 = *reinterpret_cast<const float4 *>(p + jj + 4);
                float vw[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) vw[u] = cv[(jj + u) * D];
                acc = fadd(acc, fmul(p0.x, vw[0]));
                acc = fadd(acc, fmul(p0.y, vw[1]));
                acc = fadd(acc, fmul(p0.z, vw[2]));
                acc = fadd(acc, fmul(p0.w, vw[3]));
                acc = fadd(acc, fmul(p1.x, vw[4]));
                acc = fadd(acc, fmul(p1.y, vw[5]));
                acc = fadd(acc, fmul(p1.z, vw[6]));
                acc = fadd(acc, fmul(p1.w, vw[7]));
            }
            for (; jj < stop; ++jj) acc = fadd(acc, fmul(p[jj], cv[jj * D]));
            if (stop != n) acc = fadd(acc, fmul(p[n - 1], vn[dim]));
        }
    }
    cp_async_wait<0>();
    const int width = a.heads * D;
    if (pv && a.ctx) a.ctx[(int64_t)r * width + (h0 + ph) * D + dim] = acc;
    if (a.q_out) {
        // the CTA's outputs are whole quantization blocks of o_proj's input (calls 18-23)
        __syncthreads();
        if (pv) q[ph * D + dim] = acc;
        __syncthreads();
        const int w = t / 32, lane = t % 32;
        if (w < G * D / QBLOCK) {
            int8_t qv;
            int bs;
            const float sc = quantize_block_warp(q[w * QBLOCK + lane], &qv, &bs);
            const int col = h0 * D + w * QBLOCK;
            a.q_out[(int64_t)r * width + col + lane] = qv;
            if (lane == 0) {
                a.xs_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = sc;
                a.bsums_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = bs;
            }
        }
    }
}

// ---- small helpers ---------------------------------------------------------------------------
__global__ void xor80_kernel(uint8_t *p, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] ^= 0x80;
}

// Per-row int8 weights on the device (nanocompile/quantize.py:55-70), one CTA per row:
// scale = max|w| / 127 (a NaN-propagating maximum: |w| bit patterns order as unsigned
// integers, NaN above inf; a zero scale becomes 1), then for each value v = w / scale the
// rounding sign(v) * floor(|v| + 0.5) and the clip to +-127 -- every step the single float32
// rounding NumPy takes.  packed != 0 stores value + 128 as a byte, the layout the projection
// kernels read; otherwise the int8 value.  A NaN or infinite weight gives a NaN or infinite
// scale and zero values where the quotient is NaN (NumPy's cast of NaN to int8 is
// platform-defined; on x86-64 it is 0 as well).
constexpr int QI8_THREADS = 256;
__global__ void __launch_bounds__(QI8_THREADS) quantize_int8_rows_kernel(void *out, float *scales, const float *w,
                                                                         int64_t cols, int packed) {
    __shared__ unsigned s_max[QI8_THREADS / 32];
    const int64_t row = blockIdx.x;
    const float *src = w + row * cols;
    unsigned mx = 0;
    for (int64_t i = threadIdx.x; i < cols; i += QI8_THREADS) mx = max(mx, __float_as_uint(src[i]) & 0x7fffffffu);
    mx = __reduce_max_sync(0xffffffffu, mx);
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
    __syncthreads();
    unsigned top = 0;
#pragma unroll
    for (int i = 0; i < QI8_THREADS / 32; ++i) top = max(top, s_max[i]);
    float scale = __fdiv_rn(__uint_as_float(top), 127.0f);
    if (scale == 0.0f) scale = 1.0f;
    if (threadIdx.x == 0) scales[row] = scale;
    for (int64_t i = threadIdx.x; i < cols; i += QI8_THREADS) {
        const float v = __fdiv_rn(src[i], scale);
        const float mag = floorf(__fadd_rn(fabsf(v), 0.5f));
        float r = v > 0.0f ? mag : (v < 0.0f ? -mag : 0.0f);
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        const int q = (int)r;
        if (packed) static_cast<uint8_t *>(out)[row * cols + i] = (uint8_t)(q + 128);
        else static_cast<int8_t *>(out)[row * cols + i] = (int8_t)q;
    }
}

// Every non-negative float through div127 and through the IEEE divide; counts differences.
__global__ void selfcheck_div127_kernel(unsigned long long *mismatches) {
    unsigned long long bad = 0;
    for (uint64_t u = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; u < 0x80000000ull;
         u += (uint64_t)gridDim.x * blockDim.x) {
        const float x = __uint_as_float((uint32_t)u);
        const float a = div127(x), b = fdiv(x, 127.0f);
        if (__float_as_uint(a) != __float_as_uint(b) && !(a != a && b != b)) ++bad;
    }
    if (bad) atomicAdd(mismatches, bad);
}

__global__ void expf_kernel(float *out, const float *x, int64_t n) {
    __shared__ uint64_t tab[32];
    if (threadIdx.x < 32) tab[threadIdx.x] = kExpTab[threadIdx.x];
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = expf_exact(x[i], tab);
}

// After a decode step: the argmax becomes the next input, positions advance, and the token
// is appended to the device-side history.
__global__ void advance_kernel(int64_t *ids, int32_t *pos, const int64_t *tokens, int64_t *history,
                               int32_t *step, int rows) {
    release_dependents();
    wait_for_producer();
    const int r = threadIdx.x;
    const int s = *step;
    if (r < rows) {
        ids[r] = tokens[r];
        pos[r] += 1;
        history[(int64_t)s * rows + r] = tokens[r];
    }
    __syncthreads();
    if (r == 0) *step = s + 1;
}

}  // namespace nc
