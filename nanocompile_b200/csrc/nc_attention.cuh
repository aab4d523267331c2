// Grouped decode attention for batches (more than eight rows): one CTA per (row, KV head) with
// all G query heads of its group (repeat_kv, nanocompile/nn.py:109-120).
//
// The arithmetic is attention_kernel's, which follows nanocompile/models/qwen2.py:143-150 and
// nanocompile/nn.py:57-66 step for step: RoPE of q and the new k, scores acc = acc + q*k over d in
// order, t = score * scale + 0, NaN-propagating max, in-order sum of expf(t - max),
// p = expf(t - max) / sum, ctx = in-order sum over positions of p * v.
//
// What changes is the data movement, built for many rows sharing the GPU:
//  * K and V chunks stream through a ring of shared-memory stages by TMA: a chunk is D/32 tensor
//    copies of 256 rows x 128 bytes from one 2-D tensor map over the whole KV arena, with 128-byte
//    swizzling, completion counted in bytes on an mbarrier. Many chunks are in flight per SM at no
//    instruction cost, and the swizzle lets a thread read one whole K row without bank conflicts.
//    Where no tensor map can describe the cache (its extent is not known, or the head dimension is
//    not a multiple of 32) the same kernel stages by cp.async: per thread eight 16-byte copies per
//    chunk at offsets computed once, K pieces XOR-swizzled by row.
//  * 512 threads (16 warps) per CTA; each phase takes the threads its shared-memory traffic can
//    feed. A 16-byte load costs four shared-memory wavefronts even as a broadcast, so the phases
//    are laid out for few loads per product rather than for many threads.
//  * Scores: a thread takes two positions of a 256-row chunk and four heads (K pieces of two
//    rows and q pieces of four heads per step of four dimensions: eight chains).
//  * The exps of chunk c + 1 are made by fifteen warps while warp 0 adds chunk c to the in-order
//    sums of its G heads.
//  * Probabilities are kept head-major ([8][cap]); a P.V warp takes two heads, a thread two
//    adjacent dimensions of both (four chains): one 8-byte V load, read once for the two heads,
//    and two broadcast probabilities per position. K and V are read through offsets precomputed
//    for the eight swizzle phases.
//  * The chunk holding the new position gets the new k / v row written into its stage, so the
//    scores and P.V read one layout.
//  * Decode streams the K history (cached by earlier steps) from before the wait on the previous
//    kernel.
//  * The division by the softmax sum is a reciprocal multiply with a residual check that proves
//    the correctly rounded quotient (fdiv_recip), the IEEE divide where it cannot.
#pragma once

#include <cuda.h>

#include "nc_kernels.cuh"

namespace nc {

__device__ unsigned int g_attention_fault;     // set when a TMA stage never completed (bounded wait)

constexpr int ATB_THREADS = 512;
constexpr int ATB_CHUNK = 256;     // positions per stage
constexpr int ATB_STAGES = 2;
constexpr int ATB_HEADS = 8;       // query heads per CTA at most

constexpr int ATB_BOX = 32;        // floats per 128-byte swizzled TMA box row

__host__ __device__ constexpr int atb_cap4(int cap) { return (cap + 3) & ~3; }

// Dynamic shared memory: 1 KB of alignment slack (128-byte swizzled TMA boxes start on 1 KB
// boundaries), the ring, probabilities [8][cap4], q [8][D], new k and v.
__host__ __device__ inline size_t attention_batched_smem(int d, int cap) {
    return 1024 + sizeof(float) * ((size_t)ATB_STAGES * ATB_CHUNK * d + (size_t)ATB_HEADS * atb_cap4(cap) +
                                   (size_t)(ATB_HEADS + 2) * d);
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Asks L2 for bytes from p (16-byte aligned start and size), in requests of at most 1 MB.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, int64_t bytes) {
    const char *c = (const char *)p;
    while (bytes > 0) {
        const int n = (int)(bytes < (1 << 20) ? bytes : (1 << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
// Bounded: gives up after 2^31 SM cycles (about a second).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - start > NC_DRAIN_CYCLES) return false;
    return true;
}
// Bounded by `limit` cycles (g_wait_cycles for the waits a kernel can abandon and drain after).
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, unsigned parity, long long limit) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - start > limit) return false;
    return true;
}
// One 2-D tile of the tensor map (x = column, y = row) into shared memory, counted on bar.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// In-order sum of p[0], p[stride], p[2*stride], ... (n terms), one thread; the next eight loads
// are issued before the current eight dependent adds.
__device__ __forceinline__ float chain_sum_strided(const float *p, int n, int stride) {
    float acc = 0.0f, a[8], b[8];
    int j = 0;
    const int n8 = n & ~7;
    if (n8) {
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = p[u * stride];
        for (; j < n8; j += 8) {
            if (j + 8 < n8) {
#pragma unroll
                for (int u = 0; u < 8; ++u) b[u] = p[(j + 8 + u) * stride];
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = fadd(acc, a[u]);
#pragma unroll
            for (int u = 0; u < 8; ++u) a[u] = b[u];
        }
    }
    for (; j < n; ++j) acc = fadd(acc, p[j * stride]);
    return acc;
}

// acc + p[0]*v(0) + p[1]*v(1) + ... + p[n-1]*v(n-1), strictly in order, one thread; the next
// eight probabilities and values are loaded while the current eight are added. p is 16-byte aligned.
__device__ __forceinline__ float pv_add8(float acc, const float4 &p0, const float4 &p1, const float *v) {
    acc = fadd(acc, fmul(p0.x, v[0]));
    acc = fadd(acc, fmul(p0.y, v[1]));
    acc = fadd(acc, fmul(p0.z, v[2]));
    acc = fadd(acc, fmul(p0.w, v[3]));
    acc = fadd(acc, fmul(p1.x, v[4]));
    acc = fadd(acc, fmul(p1.y, v[5]));
    acc = fadd(acc, fmul(p1.z, v[6]));
    acc = fadd(acc, fmul(p1.w, v[7]));
    return acc;
}
template <typename V>
__device__ __forceinline__ float pv_chain(float acc, const float *p, int n, V &&vat) {
    int j = 0;
    if (n >= 8) {
        float4 a0 = *reinterpret_cast<const float4 *>(p), a1 = *reinterpret_cast<const float4 *>(p + 4);
        float va[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) va[u] = vat(u);
#pragma unroll 1
        for (; j + 16 <= n; j += 8) {
            const float4 b0 = *reinterpret_cast<const float4 *>(p + j + 8), b1 = *reinterpret_cast<const float4 *>(p + j + 12);
            float vb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) vb[u] = vat(j + 8 + u);
            acc = pv_add8(acc, a0, a1, va);
            a0 = b0;
            a1 = b1;
#pragma unroll
            for (int u = 0; u < 8; ++u) va[u] = vb[u];
        }
        acc = pv_add8(acc, a0, a1, va);
        j += 8;
    }
#pragma unroll 1
    for (; j < n; ++j) acc = fadd(acc, fmul(p[j], vat(j)));
    return acc;
}

// Logical piece c (16 bytes) of row `row` of a staged K chunk.
template <int D, bool TMA>
__device__ __forceinline__ float4 staged_piece(const float *stage, int row, int c) {
    if constexpr (TMA) {
        const int b = c / (ATB_BOX / 4), u = c % (ATB_BOX / 4);
        return *reinterpret_cast<const float4 *>(stage + b * ATB_CHUNK * ATB_BOX + row * ATB_BOX + ((u ^ (row & 7)) << 2));
    } else {
        return reinterpret_cast<const float4 *>(stage)[row * (D / 4) + (c ^ (row % (D / 4)))];
    }
}
// Where element `dim` of row `row` of a staged V chunk sits (TMA: of a K chunk as well).
template <int D, bool TMA>
__device__ __forceinline__ int staged_index(int row, int dim) {
    if constexpr (TMA) {
        const int b = dim / ATB_BOX, col = dim % ATB_BOX;
        return b * ATB_CHUNK * ATB_BOX + row * ATB_BOX + ((((col >> 2) ^ (row & 7)) << 2) | (col & 3));
    } else {
        return row * D + dim;
    }
}
// The same for a staged K chunk: cp.async chunks swizzle K's 16-byte pieces by row (staged_piece).
template <int D, bool TMA>
__device__ __forceinline__ int staged_k_index(int row, int dim) {
    if constexpr (TMA) return staged_index<D, TMA>(row, dim);
    else return row * D + ((((dim >> 2) ^ (row % (D / 4))) << 2) | (dim & 3));
}

template <int D, int G, bool TMA>
__global__ void __launch_bounds__(ATB_THREADS, 1)
attention_batched_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap kvmap) {
    static_assert(G >= 2 && G <= ATB_HEADS, "group of 2..8 query heads");
    static_assert(D % 4 == 0 && D <= 128, "head dim");
    static_assert(!TMA || D % ATB_BOX == 0, "TMA staging takes 32-float boxes");
    constexpr int PPR = D / 4, HALF = D / 2;
    constexpr int NP = ATB_CHUNK * PPR / ATB_THREADS; // cp.async: 16-byte pieces a thread copies per chunk
    static_assert(ATB_THREADS % PPR == 0 && NP >= 1, "piece layout");
    constexpr int STAGE = ATB_CHUNK * D;              // floats per stage
    constexpr int SP = 2, SH = 4;                     // scores: positions x heads per thread
    constexpr int SROWS = ATB_CHUNK / SP;             // position groups of a chunk
    constexpr int S_THREADS = SROWS * ((G + SH - 1) / SH);
    constexpr int DP = D / 2, PV_THREADS = DP * ((G + 1) / 2);   // P.V: (dimension pair, two heads)
    constexpr int QUADS = ATB_CHUNK / 4;              // exps: four positions of one head per item
    static_assert(S_THREADS % 32 == 0 && S_THREADS <= ATB_THREADS && SROWS % 8 == 0, "scoring warps");
    static_assert(ATB_THREADS - PV_THREADS >= 32, "threads left for the divisions");
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ uint64_t bars[ATB_STAGES];
    __shared__ uint64_t tab[32];
    __shared__ float s_max[ATB_HEADS], s_sum[ATB_HEADS], s_rcp[ATB_HEADS];
    __shared__ float wmax[ATB_THREADS / 32][SH];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

    const int r = blockIdx.x / a.kv, g = blockIdx.x % a.kv, h0 = g * G;
    const int pos = a.pos[r], len = pos + 1, slot = a.slot[r], cap4 = atb_cap4(a.cap);
    float *ring = reinterpret_cast<float *>(smraw + ((1024 - (smem_addr(smraw) & 1023)) & 1023));   // [STAGES][STAGE]
    float *e = ring + ATB_STAGES * STAGE;                         // [8][cap4]
    float *q = e + ATB_HEADS * cap4;                              // [8][D], heads past G zero
    float *kn = q + ATB_HEADS * D, *vn = kn + D;
    if (t < 32) tab[t] = kExpTab[t];
    if (TMA && t == 0) {
        for (int s = 0; s < ATB_STAGES; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kvmap)) : "memory");
    }

    float *base = a.cache + (int64_t)slot * a.slot_stride;
    float *K = base + (int64_t)g * a.cap * D;
    float *V = base + ((int64_t)a.kv + g) * a.cap * D;

    // The ring sequence: K chunks 0..nk-1, then V chunks 0..nk-1.
    const int nk = (len + ATB_CHUNK - 1) / ATB_CHUNK;
    const int64_t krow0 = a.cache_row0 + (int64_t)slot * (a.slot_stride / D) + (int64_t)g * a.cap;
    const int64_t vrow0 = krow0 + (int64_t)a.kv * a.cap;
    // cp.async: thread t copies column t % PPR of rows t / PPR + i * (THREADS / PPR); K pieces go
    // to column col ^ (row % PPR) (the rows of one thread agree modulo PPR).
    const int pcol = t % PPR, prow0 = t / PPR;
    const int kcol = pcol ^ (prow0 % PPR);
    int next = 0;                                   // next ring index to issue
    auto issue = [&](int idx) {
        if constexpr (TMA) {
            if (t == 0 && idx < 2 * nk) {
                const bool is_k = idx < nk;
                const int j0 = (is_k ? idx : idx - nk) * ATB_CHUNK;
                float *dst = ring + (idx % ATB_STAGES) * STAGE;
                uint64_t *bar = &bars[idx % ATB_STAGES];
                mbar_expect_tx(bar, (unsigned)(STAGE * sizeof(float)));
#pragma unroll
                for (int b = 0; b < D / ATB_BOX; ++b)
                    tma_load_2d(dst + b * ATB_CHUNK * ATB_BOX, &kvmap, b * ATB_BOX, (int)((is_k ? krow0 : vrow0) + j0), bar);
            }
        } else {
            if (idx < 2 * nk) {
                const bool is_k = idx < nk;
                const int j0 = (is_k ? idx : idx - nk) * ATB_CHUNK;
                const float *src = (is_k ? K : V) + (int64_t)(j0 + prow0) * D + pcol * 4;
                float4 *dst = reinterpret_cast<float4 *>(ring + (idx % ATB_STAGES) * STAGE) + prow0 * PPR + (is_k ? kcol : pcol);
#pragma unroll
                for (int i = 0; i < NP; ++i) {
                    const int row = prow0 + i * (ATB_THREADS / PPR);
                    if (j0 + row < len) cp_async16(dst + i * (ATB_THREADS / PPR) * PPR, src + (int64_t)i * (ATB_THREADS / PPR) * D);
                }
            }
            cp_async_commit();
        }
        next = idx + 1;
    };
    auto ready = [&](int idx) -> bool {
        if constexpr (TMA) return mbar_wait_bounded(&bars[idx % ATB_STAGES], (unsigned)((idx / ATB_STAGES) & 1));
        cp_async_wait<ATB_STAGES - 2>();
        return true;
    };
    // Decode (mode 0): the cached rows come from earlier steps, not from the previous kernel, so
    // the K history starts towards L2 and the first chunk towards shared memory before the wait.
    // The whole K history goes into L2 (its chunks stream through the two stages while the scores
    // are formed), the V history when the last K chunk is in (it arrives during the softmax).
    const bool early = a.mode == 0;
    if (early) {
        if (t == 0) prefetch_l2_bulk(K, (int64_t)len * D * sizeof(float));
        for (int i = 0; i < ATB_STAGES - 1; ++i) issue(i);
    }
    release_dependents();
    wait_for_producer();

    const float *qkv = a.qkv + (int64_t)r * (a.heads + 2 * a.kv) * D;
    const float *cs = a.cos_tab + (int64_t)pos * HALF, *sn = a.sin_tab + (int64_t)pos * HALF;
    // RoPE of the group's q heads (rows past G zero) and of the new k; the new v
    for (int i = t; i < (ATB_HEADS + 2) * D; i += ATB_THREADS) {
        const int h = i / D, c = i % D;
        if (h < ATB_HEADS && h >= G) {
            q[h * D + c] = 0.0f;
            continue;
        }
        const float *src = h < ATB_HEADS ? qkv + (h0 + h) * D
                                         : (h == ATB_HEADS ? qkv + (a.heads + g) * D : qkv + (a.heads + a.kv + g) * D);
        if (h == ATB_HEADS + 1) {
            vn[c] = src[c];
            continue;
        }
        const float t1 = src[c];
        const float rot = c < HALF ? -src[c + HALF] : src[c - HALF];
        const float v = fadd(fmul(t1, cs[c % HALF]), fmul(rot, sn[c % HALF]));
        if (h < ATB_HEADS) q[h * D + c] = v;
        else kn[c] = v;
    }
    __syncthreads();
    if (a.mode != 2) {
        for (int c = t; c < D; c += ATB_THREADS) {
            K[(int64_t)pos * D + c] = kn[c];
            V[(int64_t)pos * D + c] = vn[c];
        }
        if (a.mode == 1) return;
    }
    const bool own_new = a.mode == 0;    // position pos comes from kn / vn, not the cache
    if (!early) {
        if (t == 0) prefetch_l2_bulk(K, (int64_t)len * D * sizeof(float));
        for (int i = 0; i < ATB_STAGES - 1; ++i) issue(i);
    }
    // Decode: the staged chunk that holds position pos gets the new row from kn / vn, so every
    // phase reads one layout. Rows written by the threads go to the async proxy (the ring stage
    // is loaded by TMA again later) behind a proxy fence.
    auto own_row = [&](float *st, int row, const float *src, bool is_k) {
        for (int c = t; c < D; c += ATB_THREADS)
            st[is_k ? staged_k_index<D, TMA>(row, c) : staged_index<D, TMA>(row, c)] = src[c];
        if (TMA) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
    };

    // ---- scores: thread (two positions of the chunk, four heads), eight chains ----
    // Per step of four dimensions a thread loads two K pieces and four q pieces (broadcast) for
    // 32 products: fewer 16-byte loads per product than one position per thread, and eight warps
    // (two per scheduler) to hide the chains' latency.
    const int pq = t % SROWS, hb = (t / SROWS) * SH;
    const bool scorer = t < S_THREADS;
    float mx[SH];
#pragma unroll
    for (int h = 0; h < SH; ++h) mx[h] = __uint_as_float(0xff800000u);
    // TMA stages: piece c of row pq + i * SROWS sits at (c / 8) * CHUNK * BOX + i * SROWS * BOX +
    // koff[c % 8] (the rows agree modulo 8), so the K loads take no index arithmetic
    int koff[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) koff[u] = pq * ATB_BOX + ((u ^ (pq & 7)) << 2);
    int failed_at = -1;
    for (int ci = 0; ci < nk; ++ci) {
        const bool ok = ready(ci);
        if (__syncthreads_or(!ok)) { failed_at = ci; break; }
        issue(ci + ATB_STAGES - 1);
        const int j0 = ci * ATB_CHUNK;
        float *st = ring + (ci % ATB_STAGES) * STAGE;
        if (own_new && ci == nk - 1) own_row(st, pos - j0, kn, true);
        if (scorer) {
            float acc[SP][SH];
#pragma unroll
            for (int i = 0; i < SP; ++i)
#pragma unroll
                for (int h = 0; h < SH; ++h) acc[i][h] = 0.0f;
#pragma unroll
            for (int c = 0; c < PPR; ++c) {
                float4 kr[SP];
#pragma unroll
                for (int i = 0; i < SP; ++i) {
                    if constexpr (TMA)
                        kr[i] = *reinterpret_cast<const float4 *>(st + (c >> 3) * ATB_CHUNK * ATB_BOX + i * SROWS * ATB_BOX + koff[c & 7]);
                    else
                        kr[i] = staged_piece<D, TMA>(st, pq + i * SROWS, c);
                }
                // the eight chains advance component by component (x, y, z, w of the piece),
                // so consecutive adds belong to different chains
                float4 qx[SH];
#pragma unroll
                for (int h = 0; h < SH; ++h) qx[h] = reinterpret_cast<const float4 *>(q + (hb + h) * D)[c];
#pragma unroll
                for (int h = 0; h < SH; ++h)
#pragma unroll
                    for (int i = 0; i < SP; ++i) acc[i][h] = fadd(acc[i][h], fmul(qx[h].x, kr[i].x));
#pragma unroll
                for (int h = 0; h < SH; ++h)
#pragma unroll
                    for (int i = 0; i < SP; ++i) acc[i][h] = fadd(acc[i][h], fmul(qx[h].y, kr[i].y));
#pragma unroll
                for (int h = 0; h < SH; ++h)
#pragma unroll
                    for (int i = 0; i < SP; ++i) acc[i][h] = fadd(acc[i][h], fmul(qx[h].z, kr[i].z));
#pragma unroll
                for (int h = 0; h < SH; ++h)
#pragma unroll
                    for (int i = 0; i < SP; ++i) acc[i][h] = fadd(acc[i][h], fmul(qx[h].w, kr[i].w));
            }
#pragma unroll
            for (int i = 0; i < SP; ++i) {
                const int j = j0 + pq + i * SROWS;
                if (j < len) {
#pragma unroll
                    for (int h = 0; h < SH; ++h) {
                        const float sc = fadd(fmul(acc[i][h], a.scale), 0.0f);
                        e[(hb + h) * cap4 + j] = sc;
                        mx[h] = nan_max(mx[h], sc);
                    }
                }
            }
        }
    }
    if (failed_at >= 0) goto fault;
    if (t == 0) prefetch_l2_bulk(V, (int64_t)len * D * sizeof(float));
    {
        // per-head maxima: head quad hq is scored by warps hq * SROWS / 32 ... (hq + 1) * SROWS / 32 - 1
        if (scorer) {
#pragma unroll
            for (int h = 0; h < SH; ++h) {
                const float m = warp_nan_max(mx[h]);
                if (lane == 0) wmax[warp][h] = m;
            }
        }
        __syncthreads();
        constexpr int WPH = SROWS / 32;
        if (t < G) {
            const int w0 = (t / SH) * WPH, h = t % SH;
            float m = wmax[w0][h];
            for (int w = 1; w < WPH; ++w) m = nan_max(m, wmax[w0 + w][h]);
            s_max[t] = m;
        }
        __syncthreads();
        // The exps of chunk ci + 1 (warps 1..15, a quad of one head per item) are made while
        // lanes 0..G-1 of warp 0 add chunk ci to the in-order sums; chunk 0 by all first.
        auto exps_chunk = [&](int ci, int u, int n) {
            if (ci >= nk) return;
            const int j0 = ci * ATB_CHUNK;
            for (int i = u; i < G * QUADS; i += n) {
                const int h = i / QUADS, j = j0 + 4 * (i % QUADS);
                if (j < len) {
                    float4 *p = reinterpret_cast<float4 *>(e + h * cap4 + j);   // positions past len are never read
                    const float mh = s_max[h];
                    float4 v = *p;
                    v.x = expf_exact(fsub(v.x, mh), tab);
                    v.y = expf_exact(fsub(v.y, mh), tab);
                    v.z = expf_exact(fsub(v.z, mh), tab);
                    v.w = expf_exact(fsub(v.w, mh), tab);
                    *p = v;
                }
            }
        };
        exps_chunk(0, t, ATB_THREADS);
        __syncthreads();
        float sum = 0.0f;
        for (int ci = 0; ci < nk; ++ci) {
            if (warp == 0) {
                if (lane < G) {
                    const int j0 = ci * ATB_CHUNK;
                    sum = chain_sum(e + lane * cap4 + j0, min(ATB_CHUNK, len - j0), sum);
                }
            } else {
                exps_chunk(ci + 1, t - 32, ATB_THREADS - 32);
            }
            __syncthreads();
        }
        if (t < G) {
            s_sum[t] = sum;
            s_rcp[t] = __frcp_rn(sum);
        }
        __syncthreads();
    }
    {
        // ---- probabilities @ V: thread (dimension pair, two heads), positions in order ----
        // A warp takes the 32 dimension pairs of two heads: per position one 8-byte V load per
        // thread (the row read once for both heads: with one head per warp, shared-memory
        // wavefronts bounded this loop) and the two heads' probabilities (broadcasts, four at a
        // time); eight positions per step, the next step's loads issued before the current
        // step's chains (two register sets in turn). Row u (mod 8) of a staged chunk keeps the
        // thread's pair at voff[u] (the 128-byte swizzle), so the loads take no index arithmetic. The divisions e / sum of a
        // chunk are made by the threads without P.V work while the P.V threads consume the chunk
        // before it (chunk 0 before the loop); the barrier that opens each chunk orders the two.
        const bool pv = t < PV_THREADS;
        auto divide_chunk = [&](int ci) {
            if (pv || ci >= nk) return;
            const int u = t - PV_THREADS, j0 = ci * ATB_CHUNK;
            for (int i = u; i < G * ATB_CHUNK; i += ATB_THREADS - PV_THREADS) {
                const int h = i / ATB_CHUNK, j = j0 + i % ATB_CHUNK;
                if (j < len) e[h * cap4 + j] = fdiv_recip(e[h * cap4 + j], s_sum[h], s_rcp[h]);
            }
        };
        divide_chunk(0);
        const int dim = 2 * (t % DP), hq = 2 * (t / DP);            // heads hq, hq + 1 (if < G)
        const float *pr0 = e + min(hq, G - 1) * cap4, *pr1 = e + min(hq + 1, G - 1) * cap4;
        int voff[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) voff[k] = staged_index<D, TMA>(k, dim);
        constexpr int VROW8 = TMA ? 8 * ATB_BOX : 8 * D;  // floats from row j to row j + 8 (same box)
        float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        struct Step {
            float4 p[2][2];
            float2 v[8];
        };
        for (int ci = 0; ci < nk; ++ci) {
            const int idx = nk + ci;
            const bool ok = ready(idx);
            if (__syncthreads_or(!ok)) { failed_at = idx; break; }
            issue(idx + ATB_STAGES - 1);
            const int j0 = ci * ATB_CHUNK;
            const float *st = ring + (idx % ATB_STAGES) * STAGE;
            if (own_new && ci == nk - 1) own_row(ring + (idx % ATB_STAGES) * STAGE, pos - j0, vn, false);
            divide_chunk(ci + 1);
            if (pv) {
                const int n = min(ATB_CHUNK, len - j0), n8 = n & ~7;
                auto load = [&](int j, Step &x) {
                    x.p[0][0] = *reinterpret_cast<const float4 *>(pr0 + j0 + j);
                    x.p[0][1] = *reinterpret_cast<const float4 *>(pr0 + j0 + j + 4);
                    x.p[1][0] = *reinterpret_cast<const float4 *>(pr1 + j0 + j);
                    x.p[1][1] = *reinterpret_cast<const float4 *>(pr1 + j0 + j + 4);
                    const float *vr = st + (j / 8) * VROW8;
#pragma unroll
                    for (int k = 0; k < 8; ++k) x.v[k] = *reinterpret_cast<const float2 *>(vr + voff[k]);
                };
                // the four chains (two heads x two dimensions) advance together, position by
                // position, so each add has three others to hide its latency behind
                auto step = [&](const Step &x) {
                    const float pk[2][8] = {{x.p[0][0].x, x.p[0][0].y, x.p[0][0].z, x.p[0][0].w,
                                             x.p[0][1].x, x.p[0][1].y, x.p[0][1].z, x.p[0][1].w},
                                            {x.p[1][0].x, x.p[1][0].y, x.p[1][0].z, x.p[1][0].w,
                                             x.p[1][1].x, x.p[1][1].y, x.p[1][1].z, x.p[1][1].w}};
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float m00 = fmul(pk[0][k], x.v[k].x), m01 = fmul(pk[0][k], x.v[k].y);
                        const float m10 = fmul(pk[1][k], x.v[k].x), m11 = fmul(pk[1][k], x.v[k].y);
                        acc[0][0] = fadd(acc[0][0], m00);
                        acc[0][1] = fadd(acc[0][1], m01);
                        acc[1][0] = fadd(acc[1][0], m10);
                        acc[1][1] = fadd(acc[1][1], m11);
                    }
                };
                int jj = 0;
                if (n8) {
                    Step A, B;
                    load(0, A);
#pragma unroll 1
                    for (; jj + 16 <= n8; jj += 16) {
                        load(jj + 8, B);
                        step(A);
                        load(min(jj + 16, n8 - 8), A);     // past the last step: a reload, unused
                        step(B);
                    }
                    if (jj < n8) {
                        step(A);
                        jj += 8;
                    }
                }
#pragma unroll 1
                for (; jj < n; ++jj) {
                    const float2 v = *reinterpret_cast<const float2 *>(st + staged_index<D, TMA>(jj, dim));
                    const float p0 = pr0[j0 + jj], p1 = pr1[j0 + jj];
                    acc[0][0] = fadd(acc[0][0], fmul(p0, v.x));
                    acc[0][1] = fadd(acc[0][1], fmul(p0, v.y));
                    acc[1][0] = fadd(acc[1][0], fmul(p1, v.x));
                    acc[1][1] = fadd(acc[1][1], fmul(p1, v.y));
                }
            }
        }
        if (failed_at >= 0) goto fault;
        if (!TMA) cp_async_wait<0>();
        // ---- outputs: ctx, or the block quantization of o_proj's input ----
        const int width = a.heads * D;
        __syncthreads();
        if (pv) {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (hq + i < G) {
                    const float2 o = make_float2(acc[i][0], acc[i][1]);
                    if (a.ctx) *reinterpret_cast<float2 *>(a.ctx + (int64_t)r * width + (h0 + hq + i) * D + dim) = o;
                    *reinterpret_cast<float2 *>(q + (hq + i) * D + dim) = o;
                }
            }
        }
        if (a.q_out) {
            __syncthreads();
            for (int w = warp; w < G * D / QBLOCK; w += ATB_THREADS / 32) {
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
        return;
    }
fault:
    // a TMA stage never completed: record it, let the copies in flight land (bounded), leave
    if (t == 0) {
        atomicOr(&g_attention_fault, 1u);
        for (int idx = failed_at; idx < min(next, 2 * nk); ++idx) ready(idx);
    }
}

}  // namespace nc

namespace nc {

// ---- few-row decode attention: a CTA per (row, query head, 32-dimension slice) -------------------
// Decode with a handful of rows has too few (row, head) pairs to fill the GPU, and each pair's
// work is dominated by in-order chains. Splitting the output dimensions over CTAs multiplies the
// CTAs by D/32: every CTA recomputes its head's scores and softmax (a few microseconds of
// independent work over the K rows, which L2 serves to the other slices), then owns 32 P.V
// chains over its slice of V -- streamed through a cp.async ring from the start of the kernel --
// and the quantization of exactly one 32-value block of o_proj's input. Same arithmetic and
// order as attention_kernel.
constexpr int ATS_THREADS = 256;
constexpr int ATS_CHUNK = 256;      // positions per staged V chunk
constexpr int ATS_STAGES = 4;       // chunks in flight: a 1024-position slice is requested at once
constexpr int ATS_SLICE = 32;       // output dimensions per CTA

__host__ __device__ inline size_t attention_split_smem(int d, int cap) {
    return sizeof(float) * ((size_t)atb_cap4(cap) + (size_t)ATS_STAGES * ATS_CHUNK * ATS_SLICE + 3 * (size_t)d);
}

template <int D>
__global__ void __launch_bounds__(ATS_THREADS) attention_split_kernel(const AttnArgs a) {
    static_assert(D % ATS_SLICE == 0 && D % 4 == 0, "head dim");
    constexpr int PPR = D / 4, HALF = D / 2, SLICES = D / ATS_SLICE;
    extern __shared__ __align__(16) float sms[];
    __shared__ uint64_t tab[32];
    __shared__ float s_red[ATS_THREADS / 32];
    __shared__ float s_max, s_sum, s_rcp;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    release_dependents();
    wait_for_producer();
    const int ds = blockIdx.x % SLICES, rh = blockIdx.x / SLICES;
    const int h = rh % a.heads, r = rh / a.heads, group = a.heads / a.kv, g = h / group;
    const int pos = a.pos[r], len = pos + 1, slot = a.slot[r], cap4 = atb_cap4(a.cap);
    float *e = sms;                                        // [cap4]
    float *vring = e + cap4;                               // [STAGES][CHUNK][SLICE]
    float *q = vring + ATS_STAGES * ATS_CHUNK * ATS_SLICE; // [D]
    float *kn = q + D, *vn = kn + D;
    if (t < 32) tab[t] = kExpTab[t];
    float *base = a.cache + (int64_t)slot * a.slot_stride;
    float *K = base + (int64_t)g * a.cap * D;
    float *V = base + ((int64_t)a.kv + g) * a.cap * D;
    const float *qkv = a.qkv + (int64_t)r * (a.heads + 2 * a.kv) * D;
    const float *cs = a.cos_tab + (int64_t)pos * HALF, *sn = a.sin_tab + (int64_t)pos * HALF;
    for (int i = t; i < 3 * D; i += ATS_THREADS) {
        const int which = i / D, c = i % D;
        const float *src = which == 0 ? qkv + h * D : (which == 1 ? qkv + (a.heads + g) * D : qkv + (a.heads + a.kv + g) * D);
        if (which == 2) {
            vn[c] = src[c];
            continue;
        }
        const float t1 = src[c];
        const float rot = c < HALF ? -src[c + HALF] : src[c - HALF];
        const float v = fadd(fmul(t1, cs[c % HALF]), fmul(rot, sn[c % HALF]));
        if (which == 0) q[c] = v;
        else kn[c] = v;
    }
    __syncthreads();
    if (a.mode != 2) {
        if (h % group == 0 && ds == 0)
            for (int c = t; c < D; c += ATS_THREADS) {
                K[(int64_t)pos * D + c] = kn[c];
                V[(int64_t)pos * D + c] = vn[c];
            }
        if (a.mode == 1) return;
    }
    const bool own_new = a.mode == 0;

    // V slice chunks: position rows of 128 bytes, 8 pieces each, 8 pieces per thread per chunk
    const int nv = (len + ATS_CHUNK - 1) / ATS_CHUNK;
    auto stage_v = [&](int ci) {
        if (ci < nv) {
            float4 *dst = reinterpret_cast<float4 *>(vring + (ci % ATS_STAGES) * ATS_CHUNK * ATS_SLICE);
            for (int i = t; i < ATS_CHUNK * (ATS_SLICE / 4); i += ATS_THREADS) {
                const int row = i / (ATS_SLICE / 4), pc = i % (ATS_SLICE / 4), j = ci * ATS_CHUNK + row;
                if (j < len) cp_async16(dst + i, V + (int64_t)j * D + ds * ATS_SLICE + pc * 4);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < ATS_STAGES; ++s) stage_v(s);

    // scores: a thread per position, its head's q in registers, K rows from memory; the next
    // row's K is requested before the current row's chain (head dims up to 64)
    constexpr bool PREFETCH = D <= 64;
    float4 qr[PPR];
#pragma unroll
    for (int c = 0; c < PPR; ++c) qr[c] = reinterpret_cast<const float4 *>(q)[c];
    auto krow = [&](int j) {
        return (own_new && j == pos) ? reinterpret_cast<const float4 *>(kn) : reinterpret_cast<const float4 *>(K + (int64_t)j * D);
    };
    float mx = __uint_as_float(0xff800000u);
    float4 kv[PPR], kx[PREFETCH ? PPR : 1];
    if (PREFETCH && t < len) {
        const float4 *kr = krow(t);
#pragma unroll
        for (int c = 0; c < PPR; ++c) kx[c] = kr[c];
    }
    for (int j = t; j < len; j += ATS_THREADS) {
        if (PREFETCH) {
#pragma unroll
            for (int c = 0; c < PPR; ++c) kv[c] = kx[PREFETCH ? c : 0];
            if (j + ATS_THREADS < len) {
                const float4 *kr = krow(j + ATS_THREADS);
#pragma unroll
                for (int c = 0; c < PPR; ++c) kx[PREFETCH ? c : 0] = kr[c];
            }
        } else {
            const float4 *kr = krow(j);
#pragma unroll
            for (int c = 0; c < PPR; ++c) kv[c] = kr[c];
        }
        float acc = 0.0f;
#pragma unroll
        for (int c = 0; c < PPR; ++c) {
            acc = fadd(acc, fmul(qr[c].x, kv[c].x));
            acc = fadd(acc, fmul(qr[c].y, kv[c].y));
            acc = fadd(acc, fmul(qr[c].z, kv[c].z));
            acc = fadd(acc, fmul(qr[c].w, kv[c].w));
        }
        const float sc = fadd(fmul(acc, a.scale), 0.0f);
        e[j] = sc;
        mx = nan_max(mx, sc);
    }
    mx = warp_nan_max(mx);
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    if (t == 0) {
        float m = s_red[0];
        for (int w = 1; w < ATS_THREADS / 32; ++w) m = nan_max(m, s_red[w]);
        s_max = m;
    }
    __syncthreads();
    const float mh = s_max;
    for (int j = t; j < len; j += ATS_THREADS) e[j] = expf_exact(fsub(e[j], mh), tab);
    __syncthreads();
    if (t == 0) {
        const float sum = chain_sum(e, len);        // the in-order sum
        s_sum = sum;
        s_rcp = __frcp_rn(sum);
    }
    __syncthreads();
    const float sh = s_sum, rh2 = s_rcp;
    for (int j = t; j < len; j += ATS_THREADS) e[j] = fdiv_recip(e[j], sh, rh2);

    // P.V: warp 0's lanes own the slice's 32 dimensions, positions in order
    float acc = 0.0f;
    for (int ci = 0; ci < nv; ++ci) {
        cp_async_wait<ATS_STAGES - 1>();             // chunk ci has landed
        __syncthreads();
        if (warp == 0) {
            const float *cv = vring + (ci % ATS_STAGES) * ATS_CHUNK * ATS_SLICE + lane;
            const float *pp = e + ci * ATS_CHUNK;
            const int n = min(ATS_CHUNK, len - ci * ATS_CHUNK);
            const int stop = (own_new && ci == nv - 1) ? n - 1 : n;    // the new row comes from vn
            acc = pv_chain(acc, pp, stop, [&](int j) { return cv[j * ATS_SLICE]; });
            if (stop != n) acc = fadd(acc, fmul(pp[n - 1], vn[ds * ATS_SLICE + lane]));
        }
        __syncthreads();                             // the chunk is consumed before it is refilled
        stage_v(ci + ATS_STAGES);
    }
    cp_async_wait<0>();
    if (warp == 0) {
        const int width = a.heads * D, col = h * D + ds * ATS_SLICE;
        if (a.ctx) a.ctx[(int64_t)r * width + col + lane] = acc;
        if (a.q_out) {
            int8_t qv;
            int bs;
            const float sc = quantize_block_warp(acc, &qv, &bs);
            a.q_out[(int64_t)r * width + col + lane] = qv;
            if (lane == 0) {
                a.xs_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = sc;
                a.bsums_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = bs;
            }
        }
    }
}


// ---- one decode-attention item, head dim 64, K and V by TMA ------------------------------------
// The (row, query head, 32-dimension slice) item of attention_split_kernel with the cache read by
// the tensor map of rows of 64 floats (32 x 256 boxes, 128-byte swizzle): 256-position K chunks
// (two boxes, 64 KB) through a 2-stage ring, one position per thread -- each thread reads its
// row's 16-byte pieces from the swizzled stage without bank conflicts, where reading K rows from
// global memory one row per thread touched 32 lines per warp load -- then, in the same 128 KB,
// 4 stages of the V slice (one box each), requested while the softmax runs. Same arithmetic and
// order as attention_split_kernel.
constexpr int ATT_THREADS = 256;
constexpr int ATT_KSTAGE = ATB_CHUNK * 64;          // floats: 256 rows x 64
constexpr int ATT_VSTAGE = ATB_CHUNK * ATB_BOX;     // floats: 256 rows x 32
constexpr int ATT_RING_BYTES = 2 * ATT_KSTAGE * 4;  // = 4 V stages
static_assert(ATT_RING_BYTES == 4 * ATT_VSTAGE * 4, "K and V stages share the ring");

struct AttnItem {
    const CUtensorMap *map;
    int64_t krow0, vrow0;          // tensor-map rows of K[0] / V[0] of the item's (slot, layer, KV head)
    int ds, pos, len;              // slice, the row's position, positions attended
    bool own_new;                  // position pos from kn / vn (decode), not the cache
    float scale;
};

// Thread 0 requests K chunk ci (stage ci % 2).
__device__ __forceinline__ void att_issue_k(const AttnItem &it, float *ring, uint64_t *kbar, int ci) {
    uint64_t *bar = &kbar[ci & 1];
    float *dst = ring + (ci & 1) * ATT_KSTAGE;
    mbar_expect_tx(bar, (unsigned)(ATT_KSTAGE * sizeof(float)));
    tma_load_2d(dst, it.map, 0, (int)(it.krow0 + (int64_t)ci * ATB_CHUNK), bar);
    tma_load_2d(dst + ATB_CHUNK * ATB_BOX, it.map, ATB_BOX, (int)(it.krow0 + (int64_t)ci * ATB_CHUNK), bar);
}
__device__ __forceinline__ void att_issue_v(const AttnItem &it, float *ring, uint64_t *vbar, int ci) {
    uint64_t *bar = &vbar[ci & 3];
    mbar_expect_tx(bar, (unsigned)(ATT_VSTAGE * sizeof(float)));
    tma_load_2d(ring + (ci & 3) * ATT_VSTAGE, it.map, it.ds * ATB_BOX, (int)(it.vrow0 + (int64_t)ci * ATB_CHUNK), bar);
}

// Thread 0, before the item (its K rows do not depend on this step's q/k/v): the first two chunks.
__device__ __forceinline__ void att_prefetch_k(const AttnItem &it, float *ring, uint64_t *kbar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const int nk = (it.len + ATB_CHUNK - 1) / ATB_CHUNK;
    att_issue_k(it, ring, kbar, 0);
    if (nk > 1) att_issue_k(it, ring, kbar, 1);
}

// Runs the item with ATT_THREADS threads; q, kn, vn (RoPE applied) in shared memory, e a [len]
// scratch, ring 1024-byte aligned, kbar[2] / vbar[4] initialized mbarriers whose phases kpar /
// vpar track (bit per stage), K chunks 0 and 1 already requested (att_prefetch_k). Warp 0's
// lane c gets dimension ds*32 + c of the context in *acc. False when a wait gave up (then every
// thread returns false). With st set, thread 0 writes globaltimer stamps there: st[0] when the
// scores are done, st[1] when the probabilities are.
__device__ __forceinline__ bool att_item_tma(const AttnItem &it, const float *q, const float *kn, const float *vn, float *e,
                                             float *ring, uint64_t *kbar, uint64_t *vbar, unsigned &kpar, unsigned &vpar,
                                             const uint64_t *tab, float *s_red, float *s_scal, float *acc_out,
                                             unsigned long long *st = nullptr) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int len = it.len, nk = (len + ATB_CHUNK - 1) / ATB_CHUNK;
    float mx = __uint_as_float(0xff800000u);
    float4 qr[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) qr[c] = reinterpret_cast<const float4 *>(q)[c];
    // thread t reads row t of a staged K chunk: its 16-byte piece u of box b sits at
    // b * 256 * 32 + t * 32 + ((u ^ (t % 8)) * 4) floats, one register per u
    int koff[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) koff[u] = t * ATB_BOX + ((u ^ (t & 7)) << 2);
#pragma unroll 1
    for (int ci = 0; ci < nk; ++ci) {
        const int s = ci & 1;
        const bool ok = mbar_wait_bounded(&kbar[s], (kpar >> s) & 1u);
        kpar ^= 1u << s;
        if (__syncthreads_or(!ok)) return false;
        float *stage = ring + s * ATT_KSTAGE;
        if (it.own_new && ci == nk - 1) {                 // the new key replaces row pos of the chunk
            const int row = it.pos - ci * ATB_CHUNK;
            for (int c = t; c < 64; c += ATT_THREADS) stage[staged_index<64, true>(row, c)] = kn[c];
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        const int j = ci * ATB_CHUNK + t;
        if (j < len) {
            float acc = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const float4 kv = *reinterpret_cast<const float4 *>(stage + (c >> 3) * ATB_CHUNK * ATB_BOX + koff[c & 7]);
                acc = fadd(acc, fmul(qr[c].x, kv.x));
                acc = fadd(acc, fmul(qr[c].y, kv.y));
                acc = fadd(acc, fmul(qr[c].z, kv.z));
                acc = fadd(acc, fmul(qr[c].w, kv.w));
            }
            const float sc = fadd(fmul(acc, it.scale), 0.0f);
            e[j] = sc;
            mx = nan_max(mx, sc);
        }
        __syncthreads();                                    // stage s read
        if (t == 0 && ci + 2 < nk) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            att_issue_k(it, ring, kbar, ci + 2);
        }
    }
    // the ring now takes the V slice: four chunks in flight while the softmax runs
    if (st && t == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(st[0]));
    if (t == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int ci = 0; ci < nk && ci < 4; ++ci) att_issue_v(it, ring, vbar, ci);
    }
    mx = warp_nan_max(mx);
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    if (t == 0) {
        float v = s_red[0];
        for (int w = 1; w < ATT_THREADS / 32; ++w) v = nan_max(v, s_red[w]);
        s_scal[0] = v;
    }
    __syncthreads();
    const float mh = s_scal[0];
#pragma unroll 1
    for (int j = t; j < len; j += ATT_THREADS) e[j] = expf_exact(fsub(e[j], mh), tab);
    __syncthreads();
    if (t == 0) {
        const float sum = chain_sum(e, len);                // the in-order sum
        s_scal[1] = sum;
        s_scal[2] = __frcp_rn(sum);
    }
    __syncthreads();
    const float shs = s_scal[1], rcp = s_scal[2];
#pragma unroll 1
    for (int j = t; j < len; j += ATT_THREADS) e[j] = fdiv_recip(e[j], shs, rcp);
    __syncthreads();
    if (st && t == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(st[1]));
    // P.V: warp 0's lanes own the slice's 32 dimensions, positions in order; element (row j,
    // column c) of a swizzled stage sits at j*32 + ((c/4) ^ (j%8))*4 + c%4, so row 8k + u of
    // lane c is voff[u] + 256 k: eight registers, then immediate offsets over 32 positions
    float acc = 0.0f;
    bool vok = true;
    if (warp == 0) {
        const int cl = lane & 3, cu = lane >> 2;
        int voff[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) voff[u] = u * ATB_BOX + ((cu ^ u) << 2) + cl;
#pragma unroll 1
        for (int ci = 0; ci < nk; ++ci) {
            const int s = ci & 3;
            vok = __all_sync(0xffffffffu, mbar_wait_bounded(&vbar[s], (vpar >> s) & 1u));
            vpar ^= 1u << s;
            if (!vok) break;
            const float *cv = ring + s * ATT_VSTAGE;
            const float *pp = e + ci * ATB_CHUNK;
            const int n = min(ATB_CHUNK, len - ci * ATB_CHUNK);
            const int stop = (it.own_new && ci == nk - 1) ? n - 1 : n;    // the new row comes from vn
            int j = 0;
#pragma unroll 2
            for (; j + 32 <= stop; j += 32) {
                float v[32];
                float4 pv[8];
#pragma unroll
                for (int k = 0; k < 4; ++k)
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[8 * k + u] = cv[j * ATB_BOX + k * 8 * ATB_BOX + voff[u]];
#pragma unroll
                for (int k = 0; k < 8; ++k) pv[k] = *reinterpret_cast<const float4 *>(pp + j + 4 * k);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    acc = fadd(acc, fmul(pv[k].x, v[4 * k]));
                    acc = fadd(acc, fmul(pv[k].y, v[4 * k + 1]));
                    acc = fadd(acc, fmul(pv[k].z, v[4 * k + 2]));
                    acc = fadd(acc, fmul(pv[k].w, v[4 * k + 3]));
                }
            }
#pragma unroll 1
            for (; j < stop; ++j) acc = fadd(acc, fmul(pp[j], cv[j * ATB_BOX + (((cu ^ (j & 7)) << 2) | cl)]));
            if (stop != n) acc = fadd(acc, fmul(pp[n - 1], vn[it.ds * ATB_BOX + lane]));
            __syncwarp();
            if (lane == 0 && ci + 4 < nk) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                att_issue_v(it, ring, vbar, ci + 4);
            }
        }
    }
    *acc_out = acc;
    return !__syncthreads_or(!vok);
}

__host__ __device__ inline size_t attention_tma_smem(int cap) {
    return 1024 + (size_t)ATT_RING_BYTES + sizeof(float) * ((size_t)atb_cap4(cap) + 3 * 64);
}

// attention_split_kernel for head dim 64 with the cache read through the tensor map.
__global__ void __launch_bounds__(ATT_THREADS) attention_split_tma_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap kvmap) {
    extern __shared__ __align__(16) unsigned char att_sm[];
    __shared__ uint64_t tab[32];
    __shared__ __align__(8) uint64_t kbar[2], vbar[4];
    __shared__ float s_red[ATT_THREADS / 32], s_scal[3];
    constexpr int D = 64, HALF = 32, SLICES = 2;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    float *ring = reinterpret_cast<float *>(att_sm + ((1024 - (smem_addr(att_sm) & 1023)) & 1023));
    float *e = ring + ATT_RING_BYTES / 4;
    float *q = e + atb_cap4(a.cap), *kn = q + D, *vn = kn + D;
    const int ds = blockIdx.x % SLICES, rh = blockIdx.x / SLICES;
    const int h = rh % a.heads, r = rh / a.heads, group = a.heads / a.kv, g = h / group;
    const int pos = a.pos[r], len = pos + 1;
    const int64_t slot = a.slot[r];
    if (t < 32) tab[t] = kExpTab[t];
    AttnItem it;
    it.map = &kvmap;
    it.krow0 = a.cache_row0 + slot * (a.slot_stride / D) + (int64_t)g * a.cap;
    it.vrow0 = a.cache_row0 + slot * (a.slot_stride / D) + (int64_t)(a.kv + g) * a.cap;
    it.ds = ds; it.pos = pos; it.len = len; it.own_new = a.mode == 0; it.scale = a.scale;
    if (t == 0) {
        for (int i = 0; i < 2; ++i) mbar_init(&kbar[i], 1);
        for (int i = 0; i < 4; ++i) mbar_init(&vbar[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // decode: the cached rows come from earlier steps, not from the previous kernel
        if (a.mode == 0) att_prefetch_k(it, ring, kbar);
    }
    release_dependents();
    wait_for_producer();
    if (t == 0 && a.mode == 2) att_prefetch_k(it, ring, kbar);   // the prompt's rows: just appended
    float *base = a.cache + slot * a.slot_stride;
    float *K = base + (int64_t)g * a.cap * D;
    float *V = base + ((int64_t)a.kv + g) * a.cap * D;
    const float *qkv = a.qkv + (int64_t)r * (a.heads + 2 * a.kv) * D;
    const float *cs = a.cos_tab + (int64_t)pos * HALF, *sn = a.sin_tab + (int64_t)pos * HALF;
    for (int i = t; i < 3 * D; i += ATT_THREADS) {
        const int which = i / D, c = i % D;
        const float *src = which == 0 ? qkv + h * D : (which == 1 ? qkv + (a.heads + g) * D : qkv + (a.heads + a.kv + g) * D);
        if (which == 2) {
            vn[c] = src[c];
            continue;
        }
        const float t1 = src[c];
        const float rot = c < HALF ? -src[c + HALF] : src[c - HALF];
        const float v = fadd(fmul(t1, cs[c % HALF]), fmul(rot, sn[c % HALF]));
        if (which == 0) q[c] = v;
        else kn[c] = v;
    }
    __syncthreads();
    if (a.mode != 2) {
        if (h % group == 0 && ds == 0)
            for (int c = t; c < D; c += ATT_THREADS) {
                K[(int64_t)pos * D + c] = kn[c];
                V[(int64_t)pos * D + c] = vn[c];
            }
        if (a.mode == 1) return;
    }
    unsigned kpar = 0, vpar = 0;
    float acc;
    if (!att_item_tma(it, q, kn, vn, e, ring, kbar, vbar, kpar, vpar, tab, s_red, s_scal, &acc)) {
        if (t == 0) atomicExch(&g_attention_fault, 1u);
        return;
    }
    if (warp == 0) {
        const int width = a.heads * D, col = h * D + ds * ATB_BOX;
        if (a.ctx) a.ctx[(int64_t)r * width + col + lane] = acc;
        if (a.q_out) {
            int8_t qv;
            int bs;
            const float sc = quantize_block_warp(acc, &qv, &bs);
            a.q_out[(int64_t)r * width + col + lane] = qv;
            if (lane == 0) {
                a.xs_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = sc;
                a.bsums_out[(int64_t)r * (width / QBLOCK) + col / QBLOCK] = bs;
            }
        }
    }
}
}  // namespace nc
