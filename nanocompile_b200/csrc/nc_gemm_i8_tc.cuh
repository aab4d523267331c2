// Batched int8-vnni projection on the 5th-generation tensor cores (tcgen05.mma kind::i8), with
// the reference's bits.
//
// The reference (nanocompile/lower.py:363-397, int8_vnni_dots) converts every 4-byte Dp4 lane to
// float on its own and chains it into one of 32 accumulators: for output (t, n),
//     acc[8g + l] = fma(float(Dp4(w[n, 128c + 32g + 4l ..+3] + 128, x[t, same])), xs[t, 4c + g], acc)
// chunk c after chunk c, then _combine (lower.py:298-317).  A tensor-core product sums over K, so
// the lanes must stay apart: the B operand is block-diagonal.  For one 32-byte group the MMA's N
// columns are the pairs (token t, lane l), and column (t, l) holds token t's four bytes of lane l
// with zeros in the other 28 bytes.  D[n, (t, l)] is then exactly the int32 Dp4 of (n, t, l), one
// MMA (M = 128 weight rows, K = 32 bytes) per group, at 1/8 of the int8 peak -- far above what
// the CUDA cores can consume.  The CUDA cores keep only the reference's float work: the exact
// int-to-float conversion (TMEM slots are pre-filled with the bits of 1.5 * 2^23, so the MMA's
// accumulate leaves 1.5 * 2^23 + Dp4 as a float and one subtraction recovers Dp4 exactly), the
// in-order fmaf chains, _combine and the epilogue.
//
// Roles (18 warps, one CTA per SM, persistent over work items = 128 weight rows x 4 tokens):
//  - warp 16 (producer): per 128-byte chunk one TMA tensor copy of the weight tile (128-byte
//    swizzle, K-major) and the block-diagonal activation tile: the stages are zeroed once, and
//    each chunk only its T * 32 nonzero words are stored, from quantized activations loaded
//    four chunks ahead into registers; a proxy fence, then one arrive on the stage's mbarrier;
//  - warp 17 lane 0 (MMA issuer): per chunk one MMA per group into a TMEM slot, tcgen05.commit to
//    the stage's and the slot's barriers;
//  - warps 0-15 (epilogue): warp w reads TMEM lanes 32 (w % 4).. (its rows) and the 8 columns
//    (lanes) of token w / 4 of every group of a chunk, all four groups before one wait; it re-arms
//    the slot with the 1.5 * 2^23 bits, releases it, and runs the chains two accumulators at a time
//    (packed float2 add and fma, each lane rounded as the scalar operation); after the item's last
//    chunk _combine, (sum - offset) * scale and the epilogue (bias / residual / SwiGLU + quantize).
//    The next item's block scales are loaded into registers while the current one runs.
// Gate/up items hold 64 gate rows and the 64 up rows of the same outputs (TMEM lanes 0-63 and
// 64-127), so SiLU(gate) * up and its block quantization stay in the CTA.  Every wait is bounded
// (g_wait_cycles); a wait that gives up records a fault in g_attention_fault, stops the pipeline,
// drains the copies and MMAs in flight (bounded by NC_DRAIN_CYCLES) and frees the TMEM.
#pragma once

#include <cuda.h>

#include "nc_gemm_i8.cuh"
#include "nc_lm_head_tc.cuh"

namespace nc {

constexpr int I8TC_ROWS = 128;                         // MMA M: weight rows per item = TMEM lanes
constexpr int I8TC_EPI_WARPS = 16;                     // four per TMEM sub-partition
constexpr int I8TC_THREADS = (I8TC_EPI_WARPS + 2) * 32;
constexpr int I8TC_STAGES = 4;
constexpr int I8TC_A_BYTES = I8TC_ROWS * CHUNK;        // 16 KB: 128 rows x one 128-byte chunk
constexpr uint32_t I8TC_MAGIC = 0x4B400000u;           // the bits of 1.5 * 2^23
constexpr float I8TC_MAGIC_F = 12582912.0f;

template <int T>
struct I8Tc {
    static_assert(T == 4, "tokens per item: one per epilogue warp of a sub-partition");
    static constexpr int N = 8 * T;                    // MMA N: (token, lane) columns of one group
    static constexpr int B_BYTES = N * CHUNK;          // one chunk of block-diagonal activations
    static constexpr int SLOT_COLS = 4 * N;            // one chunk's four groups
    static constexpr int SLOTS = 512 / SLOT_COLS;
    static constexpr int TPW = T / 4;                  // tokens per epilogue thread
    static constexpr int COLS = 8 * TPW;               // TMEM columns per thread and group
    // kind::i8: D s32, A u8 (the weights + 128), B s8 (the activations), both K-major
    static constexpr uint32_t IDESC = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
                                      ((uint32_t)(I8TC_ROWS >> 4) << 24);
};

struct I8TcLayout {
    int bpad;          // block scales per token, padded to 4
    size_t a_off, b_off, xs_off, offs_off, term_off, ex_off, hq_off, bytes;
};

__host__ __device__ inline I8TcLayout i8tc_layout(int T, int k) {
    I8TcLayout L{};
    L.bpad = (k / QBLOCK + 3) & ~3;
    const size_t b_bytes = (size_t)8 * T * CHUNK;
    L.a_off = 0;
    L.b_off = L.a_off + (size_t)I8TC_STAGES * I8TC_A_BYTES;
    L.xs_off = L.b_off + (size_t)I8TC_STAGES * b_bytes;
    L.offs_off = L.xs_off + sizeof(float) * (size_t)T * L.bpad;
    L.term_off = L.offs_off + sizeof(float) * 8;
    L.ex_off = L.term_off + sizeof(float) * (size_t)T * L.bpad;
    L.hq_off = L.ex_off + sizeof(float) * (size_t)T * 64;
    L.bytes = 1024 + L.hq_off + sizeof(float) * (size_t)T * 64;       // + alignment of the base to 1 KB
    return L;
}


__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, 1, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%4, %5, %6, %7}, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_only(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[C]);
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
template <int C>
__device__ __forceinline__ void tmem_st_magic(uint32_t taddr);
template <>
__device__ __forceinline__ void tmem_st_magic<16>(uint32_t taddr) {
    const uint32_t m = I8TC_MAGIC;
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
                     taddr),
                 "r"(m)
                 : "memory");
}
template <>
__device__ __forceinline__ void tmem_st_magic<8>(uint32_t taddr) {
    const uint32_t m = I8TC_MAGIC;
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(m)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(I8TC_EPI_WARPS * 32) : "memory"); }

template <int T, int PRO, int EPI>
// 18 warps: the busiest sub-partition holds five, so 16384 / (5 * 32) caps a thread at 96 registers.
__global__ void __launch_bounds__(I8TC_THREADS, 1)
gemm_i8_tc_kernel(const FusedI8Args f, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap wmap2) {
    using S = I8Tc<T>;
    constexpr bool TWO = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_QUANT;
    static_assert(PRO != PRO_NORM, "the norm prologue is the few-row kernel's");
    const GemvI8Args &a = f.g;
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ uint64_t full[I8TC_STAGES], sempty[I8TC_STAGES], tfull[S::SLOTS], tempty[S::SLOTS], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_fail;
    __shared__ uint64_t tab[32];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    unsigned char *base = smraw + ((1024 - (smem_addr(smraw) & 1023)) & 1023);
    const int K = a.k, blocks = K / QBLOCK, whole = K / CHUNK, chunks = (K + CHUNK - 1) / CHUNK;
    const I8TcLayout L = i8tc_layout(T, K);
    const int bpad = L.bpad;
    const int row_tiles = TWO ? (a.n + 63) / 64 : (a.n + I8TC_ROWS - 1) / I8TC_ROWS;
    const int items = row_tiles * ((a.m + T - 1) / T);
    float *xs_s = reinterpret_cast<float *>(base + L.xs_off);
    float *offs_s = reinterpret_cast<float *>(base + L.offs_off);
    float *term_s = reinterpret_cast<float *>(base + L.term_off);
    float *ex_s = reinterpret_cast<float *>(base + L.ex_off);
    float *hq_s = reinterpret_cast<float *>(base + L.hq_off);
    const long long limit = g_wait_cycles;

    // ---- set-up: TMEM, barriers, zeroed activation stages ----
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (t == 0) {
        for (int s = 0; s < I8TC_STAGES; ++s) {
            mbar_init(&full[s], 1);                 // the producer's arrive (+ the weight tile's bytes)
            mbar_init(&sempty[s], 1);
        }
        for (int s = 0; s < S::SLOTS; ++s) {
            mbar_init(&tfull[s], 1);
            mbar_init(&tempty[s], I8TC_EPI_WARPS);
        }
        mbar_init(&done, 1);
        s_fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (TWO && t < 32) tab[t] = kExpTab[t];
    {
        uint4 *b4 = reinterpret_cast<uint4 *>(base + L.b_off);
        for (int i = t; i < I8TC_STAGES * S::B_BYTES / 16; i += I8TC_THREADS) b4[i] = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    release_dependents();
    wait_for_producer();

    if (warp == I8TC_EPI_WARPS) {
        // ---- producer: weight tiles by TMA, block-diagonal activations by plain stores ----
        constexpr int PF = 4;                           // chunks of activations loaded ahead
        const int mine = blockIdx.x < items ? (items - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int total = mine * chunks;
        const int w = lane, g = w >> 3, l = w & 7;      // this lane's word of a chunk: segment g, lane l
        // word w of a chunk goes to row tt * 8 + l, 16-byte unit (2g + l / 4) ^ l, word l % 4
        const uint32_t at = (uint32_t)((((2 * g + (l >> 2)) ^ l) << 4) + ((l & 3) << 2));
        auto load = [&](int kk, uint32_t (&v)[T]) {
            if (kk >= total) return;
            const int it = blockIdx.x + (kk / chunks) * gridDim.x, c = kk % chunks;
            const int t0 = (it / row_tiles) * T;
            if (c * CHUNK + g * QBLOCK >= K) return;
#pragma unroll
            for (int tt = 0; tt < T; ++tt)
                v[tt] = __ldg(reinterpret_cast<const uint32_t *>(a.xq + (int64_t)min(t0 + tt, a.m - 1) * K + c * CHUNK) + w);
        };
        uint32_t pre[PF][T];
#pragma unroll
        for (int u = 0; u < PF; ++u) load(u, pre[u]);
        int last_issue[I8TC_STAGES];
#pragma unroll
        for (int s = 0; s < I8TC_STAGES; ++s) last_issue[s] = -1;
        bool ok = true;
        for (int k0 = 0; k0 < total && ok; k0 += PF) {
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int k = k0 + u;
                if (k >= total || !ok) break;
                const int it = blockIdx.x + (k / chunks) * gridDim.x, c = k % chunks, rt = it % row_tiles;
                const int s = k % I8TC_STAGES;
                if (k >= I8TC_STAGES) ok = mbar_wait_for(&sempty[s], (unsigned)((k / I8TC_STAGES - 1) & 1), limit);
                ok = __all_sync(0xffffffffu, ok && !s_fail);
                if (!ok) {
                    s_fail = 1;
                    break;
                }
                unsigned char *as = base + L.a_off + (size_t)s * I8TC_A_BYTES;
                uint32_t *bs = reinterpret_cast<uint32_t *>(base + L.b_off + (size_t)s * S::B_BYTES);
                if (lane == 0) {
                    mbar_expect_tx_only(&full[s], (unsigned)I8TC_A_BYTES);
                    if (TWO) {
                        tma_load_2d(as, &wmap, c * CHUNK, rt * 64, &full[s]);
                        tma_load_2d(as + I8TC_A_BYTES / 2, &wmap2, c * CHUNK, rt * 64, &full[s]);
                    } else {
                        tma_load_2d(as, &wmap, c * CHUNK, rt * I8TC_ROWS, &full[s]);
                    }
                }
                last_issue[s] = k;
                if (c * CHUNK + g * QBLOCK < K) {
#pragma unroll
                    for (int tt = 0; tt < T; ++tt) bs[((tt * 8 + l) * CHUNK + at) / 4] = pre[u][tt];
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the stores, to the tensor cores
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                load(k + PF, pre[u]);
            }
        }
        // drain: every weight tile this warp requested has landed before the CTA can leave
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < I8TC_STAGES; ++s)
                if (last_issue[s] >= 0) mbar_wait_for(&full[s], (unsigned)((last_issue[s] / I8TC_STAGES) & 1),
                                                      NC_DRAIN_CYCLES);
        }
    } else if (warp == I8TC_EPI_WARPS + 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            int k = 0, q = 0;
            for (int it = blockIdx.x; it < items && !s_fail; it += gridDim.x) {
                for (int c = 0; c < chunks; ++c, ++k, ++q) {
                    const int s = k % I8TC_STAGES, slot = q % S::SLOTS;
                    if (s_fail || !mbar_wait_for(&full[s], (unsigned)((k / I8TC_STAGES) & 1), limit) ||
                        !mbar_wait_for(&tempty[slot], (unsigned)((q / S::SLOTS) & 1), limit)) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t as = smem_addr(base + L.a_off + (size_t)s * I8TC_A_BYTES);
                    const uint32_t bs = smem_addr(base + L.b_off + (size_t)s * S::B_BYTES);
                    const int groups = min(4, (K - c * CHUNK) / QBLOCK);
                    for (int g = 0; g < groups; ++g)
                        umma_i8(tmem + (uint32_t)(slot * S::SLOT_COLS + g * S::N), umma_desc_sw128(as + 32 * g),
                                umma_desc_sw128(bs + 32 * g), S::IDESC);
                    umma_commit(&sempty[s]);
                    umma_commit(&tfull[slot]);
                }
            }
            umma_commit(&done);           // after every MMA issued, also on a failure
        }
    } else {
        // ---- epilogue ----
        static_assert(S::TPW == 1, "one token per epilogue thread");
        const int sp = warp & 3, wq = warp >> 2;          // TMEM lanes 32 sp.., the item's token wq
        const uint32_t lane_base = tmem + ((uint32_t)(32 * sp) << 16) + (uint32_t)(wq * S::COLS);
        // every slot starts armed with the 1.5 * 2^23 bits
        for (int slot = 0; slot < S::SLOTS; ++slot) {
#pragma unroll
            for (int g = 0; g < 4; ++g) tmem_st_magic<S::COLS>(lane_base + slot * S::SLOT_COLS + g * S::N);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0)
            for (int slot = 0; slot < S::SLOTS; ++slot) mbar_arrive(&tempty[slot]);
        const int et = t;                               // 0..511
        constexpr int PFN = 2;                          // block scales per thread and item (T * blocks <= 1024)
        float pf_xs[PFN], pf_off = 0.0f;
        int pf_bs[PFN];
        auto prefetch = [&](int it) {
            if (it >= items) return;
            const int t0 = (it / row_tiles) * T;
#pragma unroll
            for (int u = 0; u < PFN; ++u) {
                const int i = et + u * I8TC_EPI_WARPS * 32;
                if (i < T * blocks) {
                    const int tt = i / blocks, b = i - tt * blocks;
                    const int64_t src = (int64_t)min(t0 + tt, a.m - 1) * blocks + b;
                    pf_xs[u] = __ldg(a.xs + src);
                    if (PRO == PRO_OFFSET) pf_bs[u] = __ldg(f.bsums_in + src);
                }
            }
            if (PRO == PRO_NONE && et < T) pf_off = __ldg(a.offset + min(t0 + et, a.m - 1));
        };
        prefetch(blockIdx.x);
        const float2 neg_magic = make_float2(-I8TC_MAGIC_F, -I8TC_MAGIC_F);
        int q = 0;
        for (int it = blockIdx.x; it < items; it += gridDim.x) {
            const int rt = it % row_tiles, t0 = (it / row_tiles) * T;
            // the item's block scales and offsets (loaded during the previous item)
#pragma unroll
            for (int u = 0; u < PFN; ++u) {
                const int i = et + u * I8TC_EPI_WARPS * 32;
                if (i < T * blocks) {
                    const int tt = i / blocks, b = i - tt * blocks;
                    xs_s[tt * bpad + b] = pf_xs[u];
                    if (PRO == PRO_OFFSET) term_s[tt * bpad + b] = fmul((float)pf_bs[u], pf_xs[u]);
                }
            }
            if (PRO == PRO_NONE && et < T) offs_s[et] = pf_off;
            epi_bar();
            // the offset: 128 * in-order sum over blocks of block sum * scale (read after the chunks)
            if (PRO == PRO_OFFSET && warp < T && lane == 0) offs_s[warp] = fmul(chain_sum(term_s + warp * bpad, blocks), 128.0f);
            prefetch(it + gridDim.x);

            // accumulator pairs (8g + l, 8g + l + 1), l even
            float2 acc2[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc2[i] = make_float2(0.0f, 0.0f);
            const float *xs_t = xs_s + wq * bpad;
            for (int c = 0; c < chunks; ++c, ++q) {
                const int slot = q % S::SLOTS;
                bool ok = mbar_wait_for(&tfull[slot], (unsigned)((q / S::SLOTS) & 1), limit) && !s_fail;
                if (!__all_sync(0xffffffffu, ok)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = lane_base + slot * S::SLOT_COLS;
                const int groups = c < whole ? 4 : (K - c * CHUNK) / QBLOCK;
                uint32_t d[4][8];
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    if (g < groups) tmem_ld<8>(sa + g * S::N, d[g]);
                tmem_wait_ld();
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    if (g < groups) tmem_st_magic<8>(sa + g * S::N);
                if (c < whole) {
                    const float4 sc4 = *reinterpret_cast<const float4 *>(xs_t + 4 * c);
                    const float scg[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const float2 sc = make_float2(scg[g], scg[g]);
#pragma unroll
                        for (int l = 0; l < 8; l += 2) {
                            const float2 v = __fadd2_rn(make_float2(__uint_as_float(d[g][l]), __uint_as_float(d[g][l + 1])),
                                                        neg_magic);
                            acc2[4 * g + l / 2] = __ffma2_rn(v, sc, acc2[4 * g + l / 2]);
                        }
                    }
                } else {
                    // 32-byte groups past the last whole chunk: accumulators 0..7, group after group
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        if (g < groups) {
                            const float s1 = xs_t[4 * c + g];
                            const float2 sc = make_float2(s1, s1);
#pragma unroll
                            for (int l = 0; l < 8; l += 2) {
                                const float2 v = __fadd2_rn(make_float2(__uint_as_float(d[g][l]), __uint_as_float(d[g][l + 1])),
                                                            neg_magic);
                                acc2[l / 2] = __ffma2_rn(v, sc, acc2[l / 2]);
                            }
                        }
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[slot]);
            }
            // every epilogue warp must take the same barriers: agree on failure first (this barrier
            // also publishes the offsets)
            epi_bar();
            if (s_fail) break;

            // ---- _combine, dequantize, epilogue ----
            float acc[32];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                acc[2 * i] = acc2[i].x;
                acc[2 * i + 1] = acc2[i].y;
            }
            const int lrow = 32 * sp + lane;                 // TMEM lane = row of the item
            const int tl = wq, tok = t0 + tl;
            const float sum = combine32(acc);
            if (!TWO) {
                const int row = rt * I8TC_ROWS + lrow;
                if (tok < a.m && row < a.n) {
                    const float y = fmul(fsub(sum, offs_s[tl]), a.scales[row]);
                    float out = y;
                    if (EPI == EPI_BIAS) out = fadd(y, a.bias[row]);
                    if (EPI == EPI_RESIDUAL) out = fadd(a.residual[(int64_t)tok * a.n + row], y);
                    a.out[(int64_t)tok * a.n + row] = out;
                }
            } else {
                const int i = rt * 64 + (lrow & 63);
                const bool up = lrow >= 64;
                const int ic = min(i, a.n - 1);
                const float y = fmul(fsub(sum, offs_s[tl]), up ? a.scales2[ic] : a.scales[ic]);
                if (up) ex_s[tl * 64 + (lrow - 64)] = y;
                else hq_s[tl * 64 + lrow] = y;
                epi_bar();
                for (int i2 = et; i2 < T * 64; i2 += I8TC_EPI_WARPS * 32) {
                    const int tl2 = i2 / 64, r = i2 % 64, col = rt * 64 + r, tok2 = t0 + tl2;
                    const float out = swiglu(hq_s[i2], ex_s[i2], tab);
                    if (EPI == EPI_SWIGLU && tok2 < a.m && col < a.n) a.out[(int64_t)tok2 * a.n + col] = out;
                    hq_s[i2] = out;
                }
                if (EPI == EPI_SWIGLU_QUANT) {
                    epi_bar();
                    // one warp per (token, 32-row block)
                    for (int task = warp; task < T * 2; task += I8TC_EPI_WARPS) {
                        const int tl2 = task >> 1, blk = task & 1, tok2 = t0 + tl2, gb = rt * 2 + blk;
                        if (tok2 < a.m && gb < a.n / QBLOCK) {
                            int8_t qv;
                            int bsv;
                            const float sc = quantize_block_warp(hq_s[tl2 * 64 + blk * QBLOCK + lane], &qv, &bsv);
                            f.q_out[(int64_t)tok2 * a.n + gb * QBLOCK + lane] = qv;
                            if (lane == 0) {
                                f.xs_out[(int64_t)tok2 * (a.n / QBLOCK) + gb] = sc;
                                f.bsums_out[(int64_t)tok2 * (a.n / QBLOCK) + gb] = bsv;
                            }
                        }
                    }
                }
                epi_bar();                              // ex_s / hq_s are free for the next item
            }
        }
    }

    // ---- leave: every MMA done, then free the TMEM ----
    __syncwarp();
    if (!mbar_wait_for(&done, 0, NC_DRAIN_CYCLES)) s_fail = 1;
    tc_fence_after();
    __syncthreads();
    if (s_fail && t == 0) atomicOr(&g_attention_fault, 1u);
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

}  // namespace nc
