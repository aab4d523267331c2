// The tied LM head + greedy argmax of a batched decode step on the 5th-generation tensor cores,
// with the reference's tokens.
//
// The reference's logits are in-order float32 dot products (nanocompile/lower.py:255-274) and its
// token is np.argmax of them (nanocompile/models/qwen2.py:364). A tensor-core product cannot
// reproduce those bits, but the argmax only needs the largest exact logit, so three kernels:
//
//  1. lm_prep_kernel: each token's normed activations split into x_hi (the float with its 13 low
//     mantissa bits cleared, a tf32 value) and x_lo = x - x_hi, written as 64-row x 32-float tiles
//     in the 128-byte-swizzled layout of a K-major tcgen05 operand; and the token's candidate
//     margin delta.
//  2. lm_head_tc_kernel: logits approximated with tcgen05.mma kind::tf32 as w*x_hi + w*x_lo,
//     accumulated in TMEM (w enters as tf32: its low mantissa bits are not used). A CTA owns 128
//     vocabulary rows x 64 tokens; per K tile of 32 floats one bulk copy brings the weights (kept
//     as pre-swizzled 16 KB tiles, lm_tiles_kernel) and two bring x_hi / x_lo into a 3-stage ring (two CTAs per SM);
//     one thread issues 8 MMAs per tile and another the copies, handing stages over on mbarriers
//     (tcgen05.commit for the MMAs' completion), every wait bounded. The epilogue reads the
//     accumulator tile from TMEM (tcgen05.ld) and keeps, per token, the CTA's best value and every
//     row within delta of it.
//  3. lm_head_pick_kernel: per token, the global best approximation, the candidates within delta
//     of it, their exact in-order logits, and np.argmax over those (first maximum, NaN largest).
//
// delta bounds twice the distance between the tensor-core value and the reference's exact value:
// per product |w x - approx| <= (2^-10 + 2^-21) |w||x| (w's dropped bits, x_lo's), and the two
// float32 sums (the reference's in order, the tensor core's) add at most 2 K 2^-24 sum_k |w_k||x_k|;
// with sum_k |w_k||x_k| <= max|w| sum_k |x_k|, delta = 2^-8 max(1, K/2048) max|w| sum_k |x_k|
// covers twice the total. By Cauchy-Schwarz sum_k |w_k||x_k| <= ||w_row||_2 ||x||_2 as well, so
// the margin takes the smaller of max|w| sum|x| and max_row ||w_row||_2 ||x||_2 (the latter with
// a factor 1 + 2^-10 for the float32 sum of squares; the row norms come from the host in double,
// rounded up): for weights without outliers the second is several times tighter, and every row it
// leaves out needs no exact recheck. The best exact row is then within delta of the best approximation, so
// it is always a candidate. A CTA whose candidates overflow its list, or that saw a NaN or +inf,
// hands all of its rows to the pick kernel, which recomputes them exactly. A bounded wait that
// gives up records a fault in g_attention_fault (the host turns it into an error) and also hands
// all rows over.
#pragma once

#include <cuda.h>

#include "nc_attention.cuh"

namespace nc {

constexpr int LMT_ROWS = 128;       // vocabulary rows per CTA (MMA M)
constexpr int LMT_TOK = 64;         // tokens per CTA (MMA N)
constexpr int LMT_KT = 32;          // K floats per tile: one 128-byte swizzled row
constexpr int LMT_STAGES = 3;               // two CTAs per SM: one's epilogue overlaps the other's stream
constexpr int LMT_THREADS = 128;
constexpr int LMT_CAND = 16;        // candidates kept per (CTA, token)
constexpr int LMT_TMEM_COLS = 64;   // the fp32 accumulator tile: 128 lanes x 64 columns

// per stage: w | x_hi | x_lo
constexpr int LMT_W_BYTES = LMT_ROWS * LMT_KT * 4;   // 16 KB
constexpr int LMT_X_BYTES = LMT_TOK * LMT_KT * 4;    // 8 KB
constexpr int LMT_STAGE_BYTES = LMT_W_BYTES + 2 * LMT_X_BYTES;
constexpr int LMT_TS = LMT_TOK + 1;     // accumulator tile row stride in shared memory (floats)
constexpr size_t LMT_SMEM = 1024 + (size_t)LMT_STAGES * LMT_STAGE_BYTES;   // the epilogue tile reuses the stages
static_assert(LMT_ROWS * LMT_TS * 4 <= LMT_STAGES * LMT_STAGE_BYTES, "epilogue tile fits the stages");

struct LmHeadTcArgs {
    int m, n, k;                    // tokens, vocabulary rows, hidden
    float wmax;                     // max |w| over the weights
    const float *tiles;             // the weights as swizzled 128 x 32 tiles (lm_tiles_kernel)
    const float *xhi, *xlo;         // the activations as swizzled 64 x 32 tiles (lm_prep_kernel)
    float *cand_val;                // [m][ctas][CAND]
    int32_t *cand_idx;              // [m][ctas][CAND]
    int32_t *cand_cnt;              // [m][ctas]: count (> CAND: all rows of the CTA)
    float *cta_best;                // [m][ctas]: the CTA's best approximation
    const float *delta;             // [m] (lm_prep_kernel)
};

// K-major operand in the 128-byte swizzled layout: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address, 16-byte units
    d |= (uint64_t)1 << 16;                             // leading byte offset (unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset: 8 rows x 128 bytes
    d |= (uint64_t)1 << 46;                             // descriptor version
    d |= (uint64_t)2 << 61;                             // 128-byte swizzle
    return d;
}

// kind::tf32, fp32 accumulator, A = M x K and B = N x K both K-major, M = 128, N = 64.
constexpr uint32_t LMT_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(LMT_TOK >> 3) << 17) |
                               ((uint32_t)(LMT_ROWS >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(LMT_IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// hi = x with the 13 low mantissa bits cleared (a tf32 value), lo = x - hi (exact)
__device__ __forceinline__ void split_tf32(float4 *hi, float4 *lo) {
    float4 v = *hi, h, l;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    l.x = fsub(v.x, h.x);
    l.y = fsub(v.y, h.y);
    l.z = fsub(v.z, h.z);
    l.w = fsub(v.w, h.w);
    *hi = h;
    *lo = l;
}

// The weights re-laid for the tensor cores, once at upload: tile (row block rb, column tile kt)
// is 16 KB at ((rb * K/32 + kt) * 128) * 32 floats, holding rows rb*128.. and columns kt*32.. in
// exactly the 128-byte-swizzled image a TMA tensor copy would make (16-byte unit u of row r at
// u ^ (r % 8)), so one contiguous bulk copy per tile streams the matrix at full DRAM efficiency.
// Rows past n are zero.
__global__ void lm_tiles_kernel(float *__restrict__ dst, const float *__restrict__ src, int n, int k) {
    const int kt_n = k / LMT_KT;
    const int64_t units = (int64_t)((n + LMT_ROWS - 1) / LMT_ROWS) * kt_n * LMT_ROWS * 8;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < units; i += (int64_t)gridDim.x * blockDim.x) {
        const int u = (int)(i & 7), r = (int)((i >> 3) % LMT_ROWS);
        const int64_t tile = i / (8 * LMT_ROWS);
        const int kt = (int)(tile % kt_n);
        const int64_t rb = tile / kt_n;
        const int64_t row = rb * LMT_ROWS + r;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (row < n) v = *reinterpret_cast<const float4 *>(src + row * k + kt * LMT_KT + u * 4);
        *reinterpret_cast<float4 *>(dst + (tile * LMT_ROWS + r) * LMT_KT + ((u ^ (r & 7)) * 4)) = v;
    }
}

// Token m's activations -> x_hi / x_lo tiles (token block m / 64, row m % 64, each K tile of 32
// floats one 8 KB swizzled image) and its margin delta[m].
__global__ void __launch_bounds__(256) lm_prep_kernel(float *__restrict__ xhi, float *__restrict__ xlo,
                                                      float *__restrict__ delta, const float *__restrict__ x, int k,
                                                      float wmax, float wnorm) {
    __shared__ float part[8], part2[8];
    const int m = blockIdx.x, t = threadIdx.x, tb = m / LMT_TOK, r = m % LMT_TOK, kt_n = k / LMT_KT;
    release_dependents();
    wait_for_producer();
    float acc = 0.0f, acc2 = 0.0f;
    for (int c = t; c < k / 4; c += 256) {
        float4 v = *reinterpret_cast<const float4 *>(x + (int64_t)m * k + 4 * c);
        acc += fabsf(v.x) + fabsf(v.y) + fabsf(v.z) + fabsf(v.w);
        acc2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        float4 lo = v;
        split_tf32(&v, &lo);
        const int kt = c / 8, u = c % 8;
        const int64_t at = ((int64_t)(tb * kt_n + kt) * LMT_TOK + r) * LMT_KT + ((u ^ (r & 7)) * 4);
        *reinterpret_cast<float4 *>(xhi + at) = v;
        *reinterpret_cast<float4 *>(xlo + at) = lo;
    }
    for (int o = 16; o > 0; o >>= 1) {
        acc += __shfl_xor_sync(0xffffffffu, acc, o);
        acc2 += __shfl_xor_sync(0xffffffffu, acc2, o);
    }
    if ((t & 31) == 0) {
        part[t / 32] = acc;
        part2[t / 32] = acc2;
    }
    __syncthreads();
    if (t == 0) {
        float sum = 0.0f, sq = 0.0f;
        for (int i = 0; i < 8; ++i) {
            sum += part[i];
            sq += part2[i];
        }
        const float l1 = wmax * sum, l2 = wnorm * sqrtf(sq) * (1.0f + 0x1p-10f);
        // fminf passes a NaN on only when both are NaN: keep the NaN (every row rechecked) when
        // either bound is not a number
        const float bound = (l1 != l1 || l2 != l2) ? l1 + l2 : fminf(l1, l2);
        delta[m] = 0x1p-8f * fmaxf(1.0f, (float)k / 2048.0f) * bound;
    }
}

__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Warp roles: warp 1 lane 0 issues the bulk copies, warp 0 lane 0 the MMAs; stages are handed
// over on mbarriers (full: copies landed -> MMA, empty: MMA completion -> copies). All four warps
// then read the accumulator tile (TMEM lanes 32w..32w+31) and pick the candidates.
__global__ void __launch_bounds__(LMT_THREADS, 2)
lm_head_tc_kernel(const LmHeadTcArgs a) {
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ uint64_t full[LMT_STAGES], empty[LMT_STAGES], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    unsigned char *base = smraw + ((1024 - (smem_addr(smraw) & 1023)) & 1023);
    const int row0 = blockIdx.x * LMT_ROWS, tok0 = blockIdx.y * LMT_TOK;
    const int tiles = a.k / LMT_KT;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                     "r"(LMT_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        for (int s = 0; s < LMT_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        s_fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    auto stage_ptr = [&](int s) { return base + s * LMT_STAGE_BYTES; };

    if (warp == 1) {
        // ---- copies: the weight tiles do not depend on the previous kernels ----
        if (lane == 0) {
            const float *wt = a.tiles + (int64_t)blockIdx.x * tiles * LMT_ROWS * LMT_KT;
            const float *xh = a.xhi + (int64_t)blockIdx.y * tiles * LMT_TOK * LMT_KT;
            const float *xl = a.xlo + (int64_t)blockIdx.y * tiles * LMT_TOK * LMT_KT;
            for (int kt = 0; kt < tiles; ++kt) {
                const int s = kt % LMT_STAGES;
                if (kt >= LMT_STAGES && !mbar_wait_bounded(&empty[s], (unsigned)((kt / LMT_STAGES - 1) & 1))) {
                    s_fail = 1;
                    break;
                }
                if (s_fail) break;
                unsigned char *st = stage_ptr(s);
                mbar_expect_tx(&full[s], (unsigned)LMT_STAGE_BYTES);
                bulk_copy_g2s(st, wt + (int64_t)kt * LMT_ROWS * LMT_KT, LMT_W_BYTES, &full[s]);
                if (kt == 0) wait_for_producer();      // the activations are the previous kernel's
                bulk_copy_g2s(st + LMT_W_BYTES, xh + (int64_t)kt * LMT_TOK * LMT_KT, LMT_X_BYTES, &full[s]);
                bulk_copy_g2s(st + LMT_W_BYTES + LMT_X_BYTES, xl + (int64_t)kt * LMT_TOK * LMT_KT, LMT_X_BYTES, &full[s]);
            }
        }
    } else if (warp == 0) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int kt = 0; kt < tiles; ++kt) {
                const int s = kt % LMT_STAGES;
                if (s_fail || !mbar_wait_bounded(&full[s], (unsigned)((kt / LMT_STAGES) & 1))) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t wa = smem_addr(stage_ptr(s)), xa = wa + LMT_W_BYTES, xl = xa + LMT_X_BYTES;
#pragma unroll
                for (int ks = 0; ks < LMT_KT / 8; ++ks) {       // 8 tf32 (32 bytes) of K per MMA
                    const uint32_t off = ks * 32;
                    umma_tf32(tmem, umma_desc_sw128(wa + off), umma_desc_sw128(xa + off), (kt | ks) != 0);
                    umma_tf32(tmem, umma_desc_sw128(wa + off), umma_desc_sw128(xl + off), 1);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(&done);   // after every MMA issued (also on a failure: nothing is left in flight)
        }
    }
    wait_for_producer();
    release_dependents();
    __syncwarp();
    const bool ok_done = mbar_wait_bounded(&done, 0);
    bool failed = false;
    if (__syncthreads_or(!ok_done || s_fail)) {
        failed = true;
        if (t == 0) atomicOr(&g_attention_fault, 1u);
    }
    tc_fence_after();

    // the accumulator tile: warp w reads TMEM lanes 32w..32w+31 = rows, 64 columns = tokens;
    // the stage memory is free now and holds it
    float *tile = reinterpret_cast<float *>(base);      // [128 rows][LMT_TS]
    if (!failed) {
        const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll
        for (int c = 0; c < LMT_TOK; c += 16) {
            uint32_t r[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                : "r"(taddr + c));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 16; ++j) tile[(32 * warp + lane) * LMT_TS + c + j] = __uint_as_float(r[j]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(LMT_TMEM_COLS) : "memory");
    }

    // per token (4 warps x 16 tokens): the CTA's best approximation and the rows within delta of it
    const int ctas = gridDim.x;
    for (int j = warp; j < LMT_TOK; j += LMT_THREADS / 32) {
        const int m = tok0 + j;
        if (m >= a.m) continue;
        const float delta = a.delta[m];
        float v[LMT_ROWS / 32];
        float best = -__uint_as_float(0x7f800000u);
        bool finite = !failed && delta == delta && delta < __uint_as_float(0x7f800000u);
#pragma unroll
        for (int q = 0; q < LMT_ROWS / 32; ++q) {
            const int rl = lane + 32 * q;
            v[q] = row0 + rl < a.n ? tile[rl * LMT_TS + j] : -__uint_as_float(0x7f800000u);
            if (row0 + rl < a.n && !(v[q] < __uint_as_float(0x7f800000u))) finite = false;   // NaN or +inf
            best = fmaxf(best, v[q]);
        }
        best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 16));
        best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 8));
        best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 4));
        best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 2));
        best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 1));
        finite = __all_sync(0xffffffffu, finite);
        const int64_t slot = (int64_t)m * ctas + blockIdx.x;
        int cnt = 0;
        if (finite) {
#pragma unroll
            for (int q = 0; q < LMT_ROWS / 32; ++q) {
                const bool c = v[q] >= best - delta;
                const unsigned bal = __ballot_sync(0xffffffffu, c);
                if (c) {
                    const int at = cnt + __popc(bal & ((1u << lane) - 1));
                    if (at < LMT_CAND) {
                        a.cand_val[slot * LMT_CAND + at] = v[q];
                        a.cand_idx[slot * LMT_CAND + at] = row0 + lane + 32 * q;
                    }
                }
                cnt += __popc(bal);
            }
        } else {
            cnt = LMT_CAND + 1;                // hand every row of the CTA to the exact recheck
        }
        if (lane == 0) {
            a.cand_cnt[slot] = cnt;
            a.cta_best[slot] = finite ? best : __uint_as_float(0x7f800000u);
        }
    }
}

// np.argmax over the exact logits of the candidates of token blockIdx.x. The candidate rows are
// listed first; then every thread takes one candidate and forms the reference's in-order dot
// product, its row streamed from memory eight 16-byte pieces ahead of the chain, the activations
// broadcast from shared memory.
constexpr int LMP_THREADS = 512;   // 16 warps: 16 candidate rows' in-order chains at a time
constexpr int LMP_LIST = 4096;

// x, two staged rows per warp, the candidate list
__host__ __device__ inline size_t lm_pick_smem(int k) {
    return sizeof(float) * (size_t)((1 + 2 * LMP_THREADS / 32) * k) + sizeof(int) * LMP_LIST;
}

// The reference's in-order dot product of x and w (both in shared memory, 16-byte aligned,
// n a multiple of 16), one thread: the next 16 products' operands are loaded while the current
// 16 are added.
__device__ __forceinline__ float chain_dot(const float *x, const float *w, int n) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x), *w4 = reinterpret_cast<const float4 *>(w);
    float acc = 0.0f;
    float4 xa[4], wa[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) { xa[u] = x4[u]; wa[u] = w4[u]; }
    for (int i = 0; i < n / 4; i += 4) {
        float4 xb[4], wb[4];
        const bool more = i + 4 < n / 4;
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (more) { xb[u] = x4[i + 4 + u]; wb[u] = w4[i + 4 + u]; }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            acc = fadd(acc, fmul(xa[u].x, wa[u].x));
            acc = fadd(acc, fmul(xa[u].y, wa[u].y));
            acc = fadd(acc, fmul(xa[u].z, wa[u].z));
            acc = fadd(acc, fmul(xa[u].w, wa[u].w));
        }
        if (more) {
#pragma unroll
            for (int u = 0; u < 4; ++u) { xa[u] = xb[u]; wa[u] = wb[u]; }
        }
    }
    return acc;
}

// One warp: the best (np.argmax order) exact logit among list[first], list[first + step], ...
// (count entries): each row comes into shared memory (buf, two k-float halves) by coalesced loads,
// the next row's loads in flight while lane 0 forms the current row's in-order dot with xs.
// k <= 1024. Updates (bv, bi) in lane 0.
__device__ __forceinline__ void best_of_list_warp(const float *w, const int *list, int first, int step, int count,
                                                  const float *xs, float *buf, int k, float &bv, int &bi) {
    const int lane = threadIdx.x & 31, k4 = k / 4;
    float4 r[8];
    auto fetch = [&](int i) {
        const float4 *src = reinterpret_cast<const float4 *>(w + (int64_t)list[i] * k);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (lane + 32 * u < k4) r[u] = src[lane + 32 * u];
    };
    if (first < count) fetch(first);
    int slot = 0;
    for (int i = first; i < count; i += step) {
        float *b = buf + slot * k;
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (lane + 32 * u < k4) reinterpret_cast<float4 *>(b)[lane + 32 * u] = r[u];
        __syncwarp();
        if (i + step < count) fetch(i + step);
        if (lane == 0) {
            const float v = chain_dot(xs, b, k);
            if (argmax_better(v, list[i], bv, bi)) { bv = v; bi = list[i]; }
        }
        slot ^= 1;
    }
    __syncwarp();
}

__global__ void __launch_bounds__(LMP_THREADS)
lm_head_pick_kernel(const LmHeadTcArgs a, const float *x, const float *w, int ctas, int64_t *tokens) {
    extern __shared__ __align__(16) float psm[];
    __shared__ float s_gbest;
    __shared__ int s_count;
    __shared__ float rv[LMP_THREADS / 32];
    __shared__ int ri[LMP_THREADS / 32];
    const int m = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int K = a.k;
    float *xs = psm;                                   // [K]
    float *rowbuf = psm + K;                           // [warps][2][K] staged candidate rows
    int *list = reinterpret_cast<int *>(psm + (1 + 2 * LMP_THREADS / 32) * K);
    release_dependents();
    wait_for_producer();
    const float delta = a.delta[m];
    for (int k = t; k < K; k += LMP_THREADS) xs[k] = x[(int64_t)m * K + k];
    // the best approximation over all CTAs
    float g = -__uint_as_float(0x7f800000u);
    for (int c = t; c < ctas; c += LMP_THREADS) g = fmaxf(g, a.cta_best[(int64_t)m * ctas + c]);
    for (int o = 16; o > 0; o >>= 1) g = fmaxf(g, __shfl_xor_sync(0xffffffffu, g, o));
    if (lane == 0) rv[warp] = g;
    if (t == 0) s_count = 0;
    __syncthreads();
    if (t == 0) {
        float b = rv[0];
        for (int i = 1; i < LMP_THREADS / 32; ++i) b = fmaxf(b, rv[i]);
        s_gbest = b;
    }
    __syncthreads();
    const float thr = s_gbest - delta;
    // the candidate list: rows within delta of the best, or every row of a CTA that handed its
    // rows over; past LMP_LIST entries the rest are checked in the list's place, row by row
    for (int c = t; c < ctas; c += LMP_THREADS) {
        const int64_t slot = (int64_t)m * ctas + c;
        if (!(a.cta_best[slot] >= thr)) continue;
        const int cnt = a.cand_cnt[slot];
        if (cnt > LMT_CAND) {
            for (int i = 0; i < LMT_ROWS; ++i) {
                const int row = c * LMT_ROWS + i;
                if (row >= a.n) break;
                const int at = atomicAdd(&s_count, 1);
                if (at < LMP_LIST) list[at] = row;
            }
        } else {
            for (int i = 0; i < cnt; ++i)
                if (a.cand_val[slot * LMT_CAND + i] >= thr) {
                    const int at = atomicAdd(&s_count, 1);
                    if (at < LMP_LIST) list[at] = a.cand_idx[slot * LMT_CAND + i];
                }
        }
    }
    __syncthreads();
    const int count = min(s_count, LMP_LIST);
    float bv = -__uint_as_float(0x7f800000u);
    int bi = 0x7fffffff;
    best_of_list_warp(w, list, warp, LMP_THREADS / 32, count, xs, rowbuf + warp * 2 * K, K, bv, bi);
    if (s_count > LMP_LIST && warp == 0) {
        // more candidates than the list holds (non-finite inputs): every row, straight from memory
        for (int row = lane; row < a.n; row += 32) {
            if (!(a.cta_best[(int64_t)m * ctas + row / LMT_ROWS] >= thr)) continue;
            const float *wr = w + (int64_t)row * K;
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc = fadd(acc, fmul(xs[k], wr[k]));
            if (argmax_better(acc, row, bv, bi)) { bv = acc; bi = row; }
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
    __syncthreads();
    if (t == 0) {
        for (int i = 1; i < LMP_THREADS / 32; ++i)
            if (argmax_better(rv[i], ri[i], bv, bi)) { bv = rv[i]; bi = ri[i]; }
        tokens[m] = bi;
    }
}

}  // namespace nc
