// A whole int8-vnni decode step of up to MK_ROWS rows as one persistent kernel.
//
// With a handful of rows a decode step is a chain of small dependent pieces: per layer the
// input norm (an in-order sum over the hidden width), 1152 q/k/v rows, attention, 896 o rows,
// the post-attention norm, 2 x 4864 gate/up rows, 896 down rows. As separate kernels each piece
// pays a launch, a ramp and a drain, and no piece has the weights of the next one in flight. Here
// one CTA per SM (cooperative launch: every CTA is resident) runs every layer as five phases,
//   A  input norm + quantization (every CTA, redundantly) -> its q/k/v rows with the bias
//   B  RoPE, cache append and attention: a CTA per (row, query head, 32-dimension slice) -> the
//      quantized attention output (o_proj's input blocks)
//   C  its o rows with the residual add
//   D  post-attention norm + quantization (every CTA) -> its whole 32-row blocks of gate/up, SiLU
//      times up, and their quantization (down's input blocks)
//   E  its down rows with the residual add
// A phase's outputs cross to the CTAs that need them as tagged 8-byte words: the low half is the
// value (or four int8), the high half names the launch and the (layer, phase) that wrote it. A
// consumer reads the words it needs until every one carries the expected tag, so the hand-over
// costs one trip through L2 and there is no grid-wide barrier. A CTA's own o/down rows keep the
// residual stream in registers. Every CTA loads the weights (and scales) of its next phase into
// registers (gate/up and down rows: shared memory, by bulk copies) before it starts waiting for
// that phase's inputs, and asks L2 for its weights of the next layer at the start of each layer;
// an attention CTA requests its first two K chunks (TMA) and asks L2 for the rest of the K and V
// history there too.
//
// Every value is computed with the same float32 operations in the same order as the separate
// kernels (norm_quant_kernel, gemv_i8_fused_kernel, attention_split_kernel), which follow
// nanocompile/nn.py:34-38, nanocompile/quantize.py:102-124, nanocompile/lower.py:363-397,
// nanocompile/fusion.py:699-711 and nanocompile/models/qwen2.py:143-150.
//
// Buffer reuse is safe without barriers: a buffer is rewritten only by a phase whose inputs
// depend, through the chain of hand-overs, on every CTA having read the buffer's previous
// contents. A wait that does not see its tags within 2^31 cycles sets g_mk_fault and every CTA
// returns; the host reports the fault and clears the tagged buffers. The last CTA to leave
// advances the launch number.
#pragma once

#include "nc_lm_head_tc.cuh"

namespace nc {

constexpr int MK_THREADS = 256;
constexpr int MK_WARPS = MK_THREADS / 32;
constexpr int MK_ROWS = 4;              // rows (sequences) of a step
constexpr int MK_NCH = 8;               // 128-byte chunks of a hidden-wide weight row (<= 1024)
constexpr int MK_GU_LPR = 8;            // lanes per gate/up row: 4 rows per warp, 32 per pass
constexpr int MK_NCH_DOWN = 40;         // chunks of an MLP-wide weight row (<= 5120)
constexpr int MK_MAX_LAYERS = 48;       // (layer, phase) fits the tag's low byte
constexpr int MK_BLOCK_WORDS = 10;      // a quantized block: 8 words of int8, its scale, its sum
// Phase stamps (globaltimer, ns) a CTA writes per layer when MkArgs::stamps is set:
//   0 layer start        1 input words in      2 input norm + quantization done   3 q/k/v rows out
//   4 q/k/v words in (attention CTAs)          5 scores done      6 softmax done   7 attention out
//   8 attention blocks in 9 o rows out         10 residual words in 11 post norm done
//   12 gate/up rows staged 13 SwiGLU blocks out 14 SwiGLU blocks in 15 down rows out
constexpr int MK_EVENTS = 16;

__device__ unsigned int g_mk_fault;

struct MkLayer {
    const uint8_t *wqkv, *wo, *wg, *wu, *wd;            // int8 + 128, [n][k]
    const float *sqkv, *so, *sg, *su, *sd, *bqkv, *in_norm, *post_norm;
    float *cache;                                         // this layer's KV, slot 0
    int64_t row0;                                         // cache[0] as a row of the KV tensor map
};

struct MkArgs {
    const MkLayer *layers;
    int nl, m, H, I, heads, kv, d, cap;
    float eps, scale;
    int64_t slot_stride, slot_rows, vocab;     // slot_rows = slot_stride / d
    const float *embed;
    const int64_t *ids;
    unsigned long long *err;
    const int32_t *slot, *pos;
    const float *cos_tab, *sin_tab, *final_norm;
    float *normed;                            // [m][H] the final norm (the LM head's input)
    unsigned long long *xt;                   // tagged residual stream [MK_ROWS][H]
    unsigned long long *qkvt;                 // tagged q/k/v [MK_ROWS][Nqkv]
    unsigned long long *aqt;                  // tagged attention output blocks [MK_ROWS][Hq/32][10]
    unsigned long long *hqt;                  // tagged SwiGLU output blocks [MK_ROWS][I/32][10]
    unsigned int *sync;                       // [0] CTAs finished, [1] launch number
    unsigned long long *stamps;               // [G][nl][MK_EVENTS] phase stamps, or null
};

// dynamic shared memory: the layer table | gains [2][H] | rows / squares [m][H] | quantized
// activations [m][max(H, Hq, I)] | block scales, terms, sums [m][blocks] | attention
// probabilities [cap4] | K / V stages, then the gate/up rows, then the down rows | q/k/v [3][d] |
// cos/sin [d]
struct MkSmem {
    int layers, gain, xrow, sq, xq, xs, term, bsum, e, vring, qkn, cs;
    int bytes;
};

__host__ __device__ inline MkSmem mk_smem(int nl, int m, int H, int K, int d, int cap) {
    MkSmem s{};
    int off = 0;
    auto take = [&](int bytes) { const int at = off; off += (bytes + 15) & ~15; return at; };
    s.layers = take(nl * (int)sizeof(MkLayer));
    s.gain = take(4 * 2 * H);
    s.xrow = take(4 * m * H);
    s.sq = take(4 * m * H);
    s.xq = take(m * K);
    s.xs = take(4 * m * (K / QBLOCK));
    s.term = take(4 * m * (K / QBLOCK));
    s.bsum = take(4 * m * (K / QBLOCK));
    s.e = take(4 * ((cap + 3) & ~3));
    // attention's K / V ring (1024-byte aligned for the 128-byte swizzle: up to 1008 bytes of
    // padding in front), and after attention this CTA's gate/up rows [2][2*32][H]
    s.vring = take(1024 + max(ATT_RING_BYTES, 2 * 2 * QBLOCK * H));
    s.qkn = take(4 * 3 * d);
    s.cs = take(4 * d);
    s.bytes = off;
    return s;
}

__host__ __device__ inline void mk_split(int n, int parts, int b, int *lo, int *hi) {
    *lo = (int)((int64_t)n * b / parts);
    *hi = (int)((int64_t)n * (b + 1) / parts);
}

__device__ __forceinline__ void mk_st(unsigned long long *p, uint32_t value, uint32_t tag) {
    const unsigned long long v = ((unsigned long long)tag << 32) | value;
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long mk_ld(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mk_prefetch_l2(const void *p, int64_t bytes) {
    // 16-byte aligned start and size (rows of a multiple of 128 bytes)
    const char *c = (const char *)p;
#pragma unroll 1
    while (bytes > 0) {
        const int n = (int)(bytes < (1 << 20) ? bytes : (1 << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c), "r"(n) : "memory");
        c += n;
        bytes -= n;
    }
}

__device__ __forceinline__ unsigned long long mk_now() {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    return v;
}

constexpr int MK_POLL_WORDS = 4;

// Reads words addr(0) .. addr(n-1) until each carries tag, handing (index, value) to store; up to
// MK_POLL_WORDS words per thread are in flight together (a hand-over of up to
// MK_POLL_WORDS * MK_THREADS words takes one round trip once the words are there). False (and
// g_mk_fault set) when the wait gave up.
template <typename A, typename F>
__device__ __forceinline__ bool mk_poll(int n, uint32_t tag, A &&addr, F &&store, long long limit = NC_DRAIN_CYCLES) {
    const long long t0 = clock64();
#pragma unroll 1
    for (int base = threadIdx.x; base < n; base += MK_POLL_WORDS * MK_THREADS) {
        bool pend[MK_POLL_WORDS];
#pragma unroll
        for (int u = 0; u < MK_POLL_WORDS; ++u) pend[u] = base + u * MK_THREADS < n;
        for (;;) {
            unsigned long long v[MK_POLL_WORDS];
#pragma unroll
            for (int u = 0; u < MK_POLL_WORDS; ++u)
                if (pend[u]) v[u] = mk_ld(addr(base + u * MK_THREADS));
            bool any = false;
#pragma unroll
            for (int u = 0; u < MK_POLL_WORDS; ++u)
                if (pend[u]) {
                    if ((uint32_t)(v[u] >> 32) == tag) {
                        store(base + u * MK_THREADS, (uint32_t)v[u]);
                        pend[u] = false;
                    } else {
                        any = true;
                    }
                }
            if (!any) break;
            if (*(volatile unsigned *)&g_mk_fault || clock64() - t0 > limit) {
                atomicExch(&g_mk_fault, 1u);
                return false;
            }
        }
    }
    return true;
}

// mk_poll over the contiguous words src[0..n), for the hand-overs of whole rows and of quantized
// blocks. MK_TO_ROWS: word i is float x[i] -> rows[i] = x, squares[i] = x * x;
// MK_TO_BLOCKS: ten words per quantized block rb -> four int8 each to q[rb * 32 ..], the scale to
// scales[rb], the block sum to sums[rb].
enum MkPollTo : int { MK_TO_ROWS = 0, MK_TO_BLOCKS = 1 };
__device__ __forceinline__ bool mk_poll_into(const unsigned long long *src, int n, uint32_t tag, int to, float *rows,
                                          float *squares, int8_t *q, float *scales, int *sums) {
    return mk_poll(n, tag, [&](int i) { return src + i; }, [&](int i, uint32_t v) {
        if (to == MK_TO_ROWS) {
            const float f = __uint_as_float(v);
            rows[i] = f;
            squares[i] = fmul(f, f);
        } else {
            const int w = i % MK_BLOCK_WORDS, rb = i / MK_BLOCK_WORDS;
            if (w < 8) reinterpret_cast<uint32_t *>(q)[(rb * QBLOCK) / 4 + w] = v;
            else if (w == 8) scales[rb] = __uint_as_float(v);
            else sums[rb] = (int)v;
        }
    });
}

// One warp's quantized block (lane = position) as ten tagged words: four int8 per word, the
// scale, the block sum.
__device__ __forceinline__ void mk_put_block(unsigned long long *dst, int8_t qv, float scale, int bsum, uint32_t tag) {
    const int lane = threadIdx.x & 31;
    uint32_t w = (uint32_t)(uint8_t)qv << (8 * (lane & 3));
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    if ((lane & 3) == 0) mk_st(dst + lane / 4, w, tag);
    if (lane == 1) mk_st(dst + 8, __float_as_uint(scale), tag);
    if (lane == 2) mk_st(dst + 9, (uint32_t)bsum, tag);
}

// Loads that stay where they are written: volatile, so the compiler cannot sink them to their
// first use (after a wait they are meant to overlap). Streaming (evict-first) for weights.
__device__ __forceinline__ uint32_t mk_ldw(const void *p) {
    uint32_t v;
    asm volatile("ld.global.cs.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 mk_ldw4(const void *p) {
    uint4 v;
    asm volatile("ld.global.cs.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float mk_ldf(const float *p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// One lane's bytes of one weight row: BPL of each 128-byte chunk (the reference's accumulators
// j*APL .. j*APL+APL-1 of every chunk).
template <int LPR, int NCH>
struct MkSlice {
    static constexpr int BPL = 128 / LPR, APL = BPL / 4;
    using SegT = typename Seg<BPL>::T;
    uint32_t w[NCH][APL];
    __device__ __forceinline__ void load(const uint8_t *row, int chunks, int j, bool ok) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            if (ok && c < chunks) {
                const uint8_t *p = row + c * CHUNK + j * BPL;
                if constexpr (BPL == 4) {
                    w[c][0] = mk_ldw(p);
                } else if constexpr (BPL == 16) {
                    Seg<16>::split(mk_ldw4(p), w[c]);
                } else {
                    static_assert(BPL == 4 || BPL == 16, "register slices of 4 or 16 bytes");
                }
            }
            else {
#pragma unroll
                for (int i = 0; i < APL; ++i) w[c][i] = 0x80808080u;
            }
        }
    }
    // the row's 32 accumulators over the chunks, combined (every lane of the warp calls it)
    __device__ __forceinline__ float dot(const int8_t *xq, const float *xs, int chunks, int j) const {
        float acc[APL];
#pragma unroll
        for (int i = 0; i < APL; ++i) acc[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            if (c < chunks) {
                const int off = c * CHUNK + j * BPL;
                uint32_t xv[APL];
                Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq + off), xv);
                const float sc = xs[off / QBLOCK];
#pragma unroll
                for (int i = 0; i < APL; ++i) acc[i] = __fmaf_rn(dp4_lane(w[c][i], xv[i]), sc, acc[i]);
            }
        }
        return combine_lanes<APL>(acc);
    }
};

// The same combined sum for a weight row staged in shared memory (int8 + 128), LPR lanes per row.
template <int LPR>
__device__ __forceinline__ float mk_dot_smem(const uint8_t *wrow, const int8_t *xq, const float *xs, int chunks, int j) {
    constexpr int BPL = 128 / LPR, APL = BPL / 4;
    using SegT = typename Seg<BPL>::T;
    float acc[APL];
#pragma unroll
    for (int i = 0; i < APL; ++i) acc[i] = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        const int off = c * CHUNK + j * BPL;
        uint32_t wv[APL], xv[APL];
        Seg<BPL>::split(*reinterpret_cast<const SegT *>(wrow + off), wv);
        Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq + off), xv);
        const float sc = xs[off / QBLOCK];
#pragma unroll
        for (int i = 0; i < APL; ++i) acc[i] = __fmaf_rn(dp4_lane(wv[i], xv[i]), sc, acc[i]);
    }
    return combine_lanes<APL>(acc);
}

// The gate and up rows of one SwiGLU output together (the same activations): both combined sums.
template <int LPR>
__device__ __forceinline__ void mk_dot2_smem(const uint8_t *grow, const uint8_t *urow, const int8_t *xq, const float *xs,
                                             int chunks, int j, float *g, float *u) {
    constexpr int BPL = 128 / LPR, APL = BPL / 4;
    using SegT = typename Seg<BPL>::T;
    float ag[APL], au[APL];
#pragma unroll
    for (int i = 0; i < APL; ++i) ag[i] = au[i] = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        const int off = c * CHUNK + j * BPL;
        uint32_t gv[APL], uv[APL], xv[APL];
        Seg<BPL>::split(*reinterpret_cast<const SegT *>(grow + off), gv);
        Seg<BPL>::split(*reinterpret_cast<const SegT *>(urow + off), uv);
        Seg<BPL>::split(*reinterpret_cast<const SegT *>(xq + off), xv);
        const float sc = xs[off / QBLOCK];
#pragma unroll
        for (int i = 0; i < APL; ++i) {
            ag[i] = __fmaf_rn(dp4_lane(gv[i], xv[i]), sc, ag[i]);
            au[i] = __fmaf_rn(dp4_lane(uv[i], xv[i]), sc, au[i]);
        }
    }
    *g = combine_lanes<APL>(ag);
    *u = combine_lanes<APL>(au);
}

// rms_norm (nanocompile/nn.py:34-38) of the m rows in xrow (squares in sq) with gain, then block
// quantization (nanocompile/quantize.py:102-124) into xq / xs and the offsets. Out of line: one
// copy serves both norms of a layer, which keeps the per-layer loop's code near 110 KB (measured
// 1.3% faster per token than two inlined copies).
__device__ __noinline__ void mk_norm_quant(int m, int H, float eps, const float *gain, float *xrow, const float *sq,
                                              int8_t *xq, float *xs, float *term, float *offs, float *s_inv) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, blocks = H / QBLOCK;
    if (lane == 0 && warp < m)
        s_inv[warp] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(chain_sum(sq + warp * H, H), (float)H), eps)));
    __syncthreads();
    for (int r = 0; r < m; ++r)
        quantize_row_smem<4>(xrow + r * H, H, xq + r * H, xs + r * blocks, nullptr, term + r * blocks, warp, MK_WARPS, lane,
                             gain, s_inv[r]);
    __syncthreads();
    if (lane == 0 && warp < m) offs[warp] = fmul(chain_sum(term + warp * blocks, blocks), 128.0f);
    __syncthreads();
}

// Tagged quantized blocks (k wide per row) into xq / xs, and each block's offset term
// float(sum_b) * scale_b. False when the wait gave up.
__device__ __forceinline__ bool mk_take_blocks(const unsigned long long *src, uint32_t tag, int m, int k, int8_t *xq, float *xs,
                                               float *term, int *bsum) {
    const int t = threadIdx.x, blocks = k / QBLOCK;
    const bool ok = mk_poll_into(src, m * blocks * MK_BLOCK_WORDS, tag, MK_TO_BLOCKS, nullptr, nullptr, xq, xs, bsum);
    if (__syncthreads_or(!ok)) return false;
#pragma unroll 1
    for (int i = t; i < m * blocks; i += MK_THREADS) term[i] = fmul((float)bsum[i], xs[i]);
    __syncthreads();
    return true;
}

// The offsets 128 * in-order sum of the terms, one row per lane of the last warp (which has no
// o / down row: the CTA's rows are fewer than its warps), while the other warps run their dots.
__device__ __forceinline__ void mk_offsets(const float *term, int m, int blocks, float *offs) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == MK_WARPS - 1 && lane < m) offs[lane] = fmul(chain_sum(term + lane * blocks, blocks), 128.0f);
}

// NCH: the chunks of a hidden-wide weight row that a lane's registers hold (q/k/v and o rows);
// NCHD bounds an MLP-wide row (the down rows come through shared memory).
// kvmap: the KV arena as rows of d floats, 32 x 256 boxes with the 128-byte swizzle.
template <int NCH, int NCHD>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_mk_kernel(const MkArgs a, const __grid_constant__ CUtensorMap kvmap) {
    extern __shared__ __align__(16) unsigned char mk_sm[];
    __shared__ uint64_t tab[32];
    __shared__ float s_inv[MK_ROWS], s_offs[MK_ROWS], s_red[MK_WARPS];
    __shared__ float s_hout[MK_ROWS][2 * QBLOCK];
    __shared__ float s_dot[MK_ROWS][MK_WARPS];
    __shared__ __align__(8) uint64_t s_kbar[2], s_vbar[4], s_gbar, s_dbar;
    __shared__ float s_scal[3];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31, b = blockIdx.x, G = gridDim.x;
    const int H = a.H, I = a.I, m = a.m, d = a.d, Hq = a.heads * a.d, Nqkv = (a.heads + 2 * a.kv) * a.d;
    const MkSmem L = mk_smem(a.nl, m, H, max(H, max(Hq, I)), d, a.cap);
    MkLayer *layers = reinterpret_cast<MkLayer *>(mk_sm + L.layers);
    float *gain_in = reinterpret_cast<float *>(mk_sm + L.gain), *gain_post = gain_in + H;
    float *xrow = reinterpret_cast<float *>(mk_sm + L.xrow), *sq = reinterpret_cast<float *>(mk_sm + L.sq);
    int8_t *xq = reinterpret_cast<int8_t *>(mk_sm + L.xq);
    float *xs = reinterpret_cast<float *>(mk_sm + L.xs), *term = reinterpret_cast<float *>(mk_sm + L.term);
    int *bsum = reinterpret_cast<int *>(mk_sm + L.bsum);
    float *e = reinterpret_cast<float *>(mk_sm + L.e);
    float *vring = reinterpret_cast<float *>(mk_sm + L.vring + ((1024 - (smem_addr(mk_sm + L.vring) & 1023)) & 1023));
    float *q = reinterpret_cast<float *>(mk_sm + L.qkn), *kn = q + d, *vn = kn + d;
    float *cs = reinterpret_cast<float *>(mk_sm + L.cs), *sn = cs + d / 2;
    if (t < 32) tab[t] = kExpTab[t];
    if (t == 0) {
        for (int s = 0; s < 2; ++s) mbar_init(&s_kbar[s], 1);
        for (int s = 0; s < 4; ++s) mbar_init(&s_vbar[s], 1);
        mbar_init(&s_gbar, 1);
        mbar_init(&s_dbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    unsigned kpar = 0, vpar = 0, gpar = 0, dpar = 0;    // mbarrier phases: K, V (warp 0), gate/up, down
    for (int i = t; i < a.nl * (int)sizeof(MkLayer) / 8; i += MK_THREADS)
        reinterpret_cast<uint64_t *>(layers)[i] = reinterpret_cast<const uint64_t *>(a.layers)[i];
    const uint32_t launch = (a.sync[1] + 1u) & 0xffffffu;
    auto tag = [&](int l, int k) { return (launch << 8) | (uint32_t)(l * 5 + k); };   // k: 0 x after o, 1 x after down,
                                                                                   // 2 q/k/v, 3 attention, 4 SwiGLU
    auto stamp = [&](int l, int ev) {
        if (a.stamps && t == 0) a.stamps[((int64_t)b * a.nl + l) * MK_EVENTS + ev] = mk_now();
    };

    // this CTA's rows of every projection
    int q0, q1, o0, o1, u0, u1;
    mk_split(Nqkv, G, b, &q0, &q1);
    mk_split(H, G, b, &o0, &o1);                        // o and down rows alike
    mk_split(I / QBLOCK, G, b, &u0, &u1);
    const int gu0 = u0 * QBLOCK, gun = (u1 - u0) * QBLOCK;
    // this CTA's attention item: (row, query head, 32-dimension slice)
    const int slices = d / ATS_SLICE, items = m * a.heads * slices;
    const bool attn = b < items;
    const int ads = b % slices, ah = (b / slices) % a.heads, ar = attn ? b / (slices * a.heads) : 0;
    const int group = a.heads / a.kv, ag = ah / group;
    const int apos = attn ? a.pos[ar] : 0, alen = apos + 1, HALF = d / 2;
    const int64_t aslot = attn ? a.slot[ar] : 0;
    for (int i = t; i < HALF; i += MK_THREADS) {
        cs[i] = a.cos_tab[(int64_t)apos * HALF + i];
        sn[i] = a.sin_tab[(int64_t)apos * HALF + i];
    }
    __syncthreads();

    // the residual stream of this CTA's o / down rows, held by lane 0 of warp (row - o0)
    const int orow = o0 + warp;
    const bool orow_ok = orow < o1;
    float res[MK_ROWS];
#pragma unroll
    for (int r = 0; r < MK_ROWS; ++r) {
        res[r] = 0.0f;
        if (r < m && orow_ok && lane == 0) {
            const int64_t id = a.ids[r];
            if (id >= 0 && id < a.vocab) res[r] = a.embed[id * H + orow];
        }
    }
    if (b == 0 && t < m) {
        const int64_t id = a.ids[t];
        if (id < 0 || id >= a.vocab) atomicMin(a.err, (unsigned long long)t);
    }

    auto prefetch_layer = [&](int l) {
        if (t != 0 || l >= a.nl) return;
        const MkLayer &W = layers[l];
        mk_prefetch_l2(W.wqkv + (int64_t)q0 * H, (int64_t)(q1 - q0) * H);
        mk_prefetch_l2(W.wo + (int64_t)o0 * Hq, (int64_t)(o1 - o0) * Hq);
        mk_prefetch_l2(W.wg + (int64_t)gu0 * H, (int64_t)gun * H);
        mk_prefetch_l2(W.wu + (int64_t)gu0 * H, (int64_t)gun * H);
        mk_prefetch_l2(W.wd + (int64_t)o0 * I, (int64_t)(o1 - o0) * I);
    };
    MkSlice<32, NCH> wq, wo;
    uint8_t *gus = reinterpret_cast<uint8_t *>(vring);           // gate rows [64][H], then up rows
    auto stage_gu = [&](const MkLayer &W) {       // this CTA's gate/up rows: one bulk copy per matrix
        if (t != 0) return;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&s_gbar, (unsigned)(2 * gun * H));
        if (gun) {
            bulk_copy_g2s(gus, W.wg + (int64_t)gu0 * H, (unsigned)(gun * H), &s_gbar);
            bulk_copy_g2s(gus + 2 * QBLOCK * H, W.wu + (int64_t)gu0 * H, (unsigned)(gun * H), &s_gbar);
        }
    };
    float sc_q = 0.0f, bias_q = 0.0f;

    prefetch_layer(0);
    {
        const int row = q0 + warp;
        const bool ok = row < q1;
        wq.load(layers[0].wqkv + (int64_t)row * H, H / CHUNK, lane, ok);
        sc_q = ok ? mk_ldf(layers[0].sqkv + row) : 0.0f;
        bias_q = ok ? mk_ldf(layers[0].bqkv + row) : 0.0f;
    }

    for (int l = 0; l < a.nl; ++l) {
        const MkLayer &W = layers[l];
        stamp(l, 0);
        float *base = W.cache + aslot * a.slot_stride;
        float *Kc = base + (int64_t)ag * a.cap * d;
        float *Vc = base + ((int64_t)a.kv + ag) * a.cap * d;
        AttnItem it;
        it.map = &kvmap;
        it.krow0 = W.row0 + aslot * a.slot_rows + (int64_t)ag * a.cap;
        it.vrow0 = W.row0 + aslot * a.slot_rows + (int64_t)(a.kv + ag) * a.cap;
        it.ds = ads; it.pos = apos; it.len = alen; it.own_new = true; it.scale = a.scale;
        if (attn && t == 0) {                                    // cached rows: earlier steps'
            att_prefetch_k(it, vring, s_kbar);
            // the rest of the history towards L2, once per (row, KV head): K past the two staged
            // chunks, and V, which is requested only when the scores are done
            if (ah % group == 0 && ads == 0) {
                if (alen > 2 * ATB_CHUNK) mk_prefetch_l2(Kc + (int64_t)2 * ATB_CHUNK * d, (int64_t)(alen - 2 * ATB_CHUNK) * d * 4);
                mk_prefetch_l2(Vc, (int64_t)alen * d * 4);
            }
        }
        prefetch_layer(l + 1);
        if (!attn) stage_gu(W);
#pragma unroll 1
        for (int i = t; i < H / 4; i += MK_THREADS) {        // the norms' gains, waited for before use
            cp_async16(gain_in + 4 * i, W.in_norm + 4 * i);
            cp_async16(gain_post + 4 * i, W.post_norm + 4 * i);
        }
        cp_async_commit();

        // ---- A: input norm + quantization, q/k/v rows with the bias ----
        if (l == 0) {
#pragma unroll 1
            for (int i = t; i < m * H; i += MK_THREADS) {
                const int64_t id = a.ids[i / H];
                const float v = (id >= 0 && id < a.vocab) ? a.embed[id * H + i % H] : 0.0f;
                xrow[i] = v;
                sq[i] = fmul(v, v);
            }
            __syncthreads();
        } else {
            const bool ok = mk_poll_into(a.xt, m * H, tag(l - 1, 1), MK_TO_ROWS, xrow, sq, nullptr, nullptr, nullptr);
            if (__syncthreads_or(!ok)) return;
        }
        stamp(l, 1);
        cp_async_wait<0>();                                  // the gains (made visible by the norm's barriers)
        mk_norm_quant(m, H, a.eps, gain_in, xrow, sq, xq, xs, term, s_offs, s_inv);
        stamp(l, 2);
        {
            const int row = q0 + warp;
            const bool ok = row < q1;
#pragma unroll 1
            for (int r = 0; r < m; ++r) {
                const float sum = wq.dot(xq + r * H, xs + r * (H / QBLOCK), H / CHUNK, lane);
                if (ok && lane == 0)
                    mk_st(a.qkvt + (int64_t)r * Nqkv + row, __float_as_uint(fadd(fmul(fsub(sum, s_offs[r]), sc_q), bias_q)),
                          tag(l, 2));
            }
        }
        stamp(l, 3);
        wo.load(W.wo + (int64_t)orow * Hq, Hq / CHUNK, lane, orow_ok);
        const float sc_o = orow_ok ? mk_ldf(W.so + orow) : 0.0f;

        // ---- B: RoPE, cache append, attention over the row's positions ----
        if (attn) {
            const unsigned long long *src = a.qkvt + (int64_t)ar * Nqkv;
            const bool ok = mk_poll(3 * d, tag(l, 2), [&](int i) {
                const int which = i / d, c = i % d;
                return src + (which == 0 ? ah * d : (which == 1 ? (a.heads + ag) * d : (a.heads + a.kv + ag) * d)) + c;
            }, [&](int i, uint32_t v) { e[i] = __uint_as_float(v); });   // q | k | v as written, RoPE below
            if (__syncthreads_or(!ok)) return;
            stamp(l, 4);
#pragma unroll 1
            for (int i = t; i < 3 * d; i += MK_THREADS) {
                const int which = i / d, c = i % d;
                if (which == 2) {
                    vn[c] = e[i];
                    continue;
                }
                const float t1 = e[i];
                const float rot = c < HALF ? -e[i + HALF] : e[i - HALF];
                const float v = fadd(fmul(t1, cs[c % HALF]), fmul(rot, sn[c % HALF]));
                if (which == 0) q[c] = v;
                else kn[c] = v;
            }
            __syncthreads();
            if (ah % group == 0 && ads == 0)
#pragma unroll 1
                for (int c = t; c < d; c += MK_THREADS) {
                    Kc[(int64_t)apos * d + c] = kn[c];
                    Vc[(int64_t)apos * d + c] = vn[c];
                }
            float acc;
            unsigned long long *ast = a.stamps ? a.stamps + ((int64_t)b * a.nl + l) * MK_EVENTS + 5 : nullptr;
            if (!att_item_tma(it, q, kn, vn, e, vring, s_kbar, s_vbar, kpar, vpar, tab, s_red, s_scal, &acc, ast)) {
                if (t == 0) atomicExch(&g_mk_fault, 1u);
                return;
            }
            stage_gu(W);                                 // the ring is free again
            if (warp == 0) {
                const int blk = (ah * d + ads * ATS_SLICE) / QBLOCK;
                int8_t qv;
                int bs;
                const float sc = quantize_block_warp(acc, &qv, &bs);
                mk_put_block(a.aqt + ((int64_t)ar * (Hq / QBLOCK) + blk) * MK_BLOCK_WORDS, qv, sc, bs, tag(l, 3));
            }
            stamp(l, 7);
        }
        const int lr = warp * (32 / MK_GU_LPR) + lane / MK_GU_LPR;     // this lane's gate/up row in a pass

        // ---- C: o rows with the residual add ----
        if (!mk_take_blocks(a.aqt, tag(l, 3), m, Hq, xq, xs, term, bsum)) return;
        stamp(l, 8);
        {
            mk_offsets(term, m, Hq / QBLOCK, s_offs);
            if (orow_ok) {                              // one copy of the dot: rows in a loop
#pragma unroll 1
                for (int r = 0; r < m; ++r) {
                    const float v = wo.dot(xq + r * Hq, xs + r * (Hq / QBLOCK), Hq / CHUNK, lane);
                    if (lane == 0) s_dot[r][warp] = v;
                }
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < MK_ROWS; ++r) {
                if (r < m && orow_ok && lane == 0) {
                    res[r] = fadd(res[r], fmul(fsub(s_dot[r][warp], s_offs[r]), sc_o));
                    mk_st(a.xt + (int64_t)r * H + orow, __float_as_uint(res[r]), tag(l, 0));
                }
            }
        }
        stamp(l, 9);
        float sg[2], su[2];                                           // rows lr, lr + 32
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            sg[p] = lr + 32 * p < gun ? mk_ldf(W.sg + gu0 + lr + 32 * p) : 0.0f;
            su[p] = lr + 32 * p < gun ? mk_ldf(W.su + gu0 + lr + 32 * p) : 0.0f;
        }

        // ---- D: post-attention norm + quantization, gate/up blocks, SiLU * up, quantization ----
        {
            const bool ok = mk_poll_into(a.xt, m * H, tag(l, 0), MK_TO_ROWS, xrow, sq, nullptr, nullptr, nullptr);
            if (__syncthreads_or(!ok)) return;
        }
        stamp(l, 10);
        mk_norm_quant(m, H, a.eps, gain_post, xrow, sq, xq, xs, term, s_offs, s_inv);
        stamp(l, 11);
        {
            const bool ok = mbar_wait_bounded(&s_gbar, gpar);
            gpar ^= 1u;
            if (__syncthreads_or(!ok)) {
                if (t == 0) atomicExch(&g_mk_fault, 1u);
                return;
            }
        }
        stamp(l, 12);
        {
            const int j = lane % MK_GU_LPR;
            const int passes = gun > QBLOCK ? 2 : (gun > 0 ? 1 : 0);    // the same in every lane
#pragma unroll 1
            for (int pr = 0; pr < passes * m; ++pr) {                    // (pass, row) pairs
                const int p = pr / m, r = pr % m, row = lr + 32 * p;
                const uint8_t *grow = gus + (row < gun ? row : 0) * H, *urow = grow + 2 * QBLOCK * H;
                float g, u;
                mk_dot2_smem<MK_GU_LPR>(grow, urow, xq + r * H, xs + r * (H / QBLOCK), H / CHUNK, j, &g, &u);
                if (row < gun && j == 0) {
                    const float off = s_offs[r];
                    s_hout[r][row] = swiglu(fmul(fsub(g, off), p ? sg[1] : sg[0]), fmul(fsub(u, off), p ? su[1] : su[0]), tab);
                }
            }
            __syncthreads();
            // the gate/up rows are read: this CTA's down rows take their place, one bulk copy
            // that lands while the SwiGLU blocks are handed over
            if (t == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(&s_dbar, (unsigned)((o1 - o0) * I));
                if (o1 > o0) bulk_copy_g2s(gus, W.wd + (int64_t)o0 * I, (unsigned)((o1 - o0) * I), &s_dbar);
            }
            const int ub = gun / QBLOCK;
#pragma unroll 1
            for (int wb = warp; wb < m * ub; wb += MK_WARPS) {
                const int r = wb / ub, blk = wb % ub;
                int8_t qv;
                int bs;
                const float sc = quantize_block_warp(s_hout[r][blk * QBLOCK + lane], &qv, &bs);
                mk_put_block(a.hqt + ((int64_t)r * (I / QBLOCK) + u0 + blk) * MK_BLOCK_WORDS, qv, sc, bs, tag(l, 4));
            }
        }
        stamp(l, 13);
        const float sc_d = orow_ok ? mk_ldf(W.sd + orow) : 0.0f;

        // ---- E: down rows with the residual add ----
        if (!mk_take_blocks(a.hqt, tag(l, 4), m, I, xq, xs, term, bsum)) return;
        stamp(l, 14);
        {
            {
                const bool ok = mbar_wait_bounded(&s_dbar, dpar);
                dpar ^= 1u;
                if (__syncthreads_or(!ok)) {
                    if (t == 0) atomicExch(&g_mk_fault, 1u);
                    return;
                }
            }
            mk_offsets(term, m, I / QBLOCK, s_offs);
            if (orow_ok) {                              // one copy of the dot: rows in a loop
#pragma unroll 1
                for (int r = 0; r < m; ++r) {
                    const float v = mk_dot_smem<32>(gus + (int64_t)warp * I, xq + r * I, xs + r * (I / QBLOCK), I / CHUNK, lane);
                    if (lane == 0) s_dot[r][warp] = v;
                }
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < MK_ROWS; ++r) {
                if (r < m && orow_ok && lane == 0) {
                    res[r] = fadd(res[r], fmul(fsub(s_dot[r][warp], s_offs[r]), sc_d));
                    mk_st(a.xt + (int64_t)r * H + orow, __float_as_uint(res[r]), tag(l, 1));
                }
            }
        }
        stamp(l, 15);
        if (l + 1 < a.nl) {
            const MkLayer &N = layers[l + 1];
            const int row = q0 + warp;
            const bool ok = row < q1;
            wq.load(N.wqkv + (int64_t)row * H, H / CHUNK, lane, ok);
            sc_q = ok ? mk_ldf(N.sqkv + row) : 0.0f;
            bias_q = ok ? mk_ldf(N.bqkv + row) : 0.0f;
        }
    }

    // the final norm of row b (nanocompile/nn.py:34-38) for the LM head
    if (b < m) {
        const bool ok = mk_poll_into(a.xt + (int64_t)b * H, H, tag(a.nl - 1, 1), MK_TO_ROWS, xrow, sq, nullptr, nullptr, nullptr);
        if (__syncthreads_or(!ok)) return;
        if (t == 0) s_inv[0] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(chain_sum(sq, H), (float)H), a.eps)));
        __syncthreads();
#pragma unroll 1
        for (int i = t; i < H; i += MK_THREADS) a.normed[(int64_t)b * H + i] = fmul(fmul(xrow[i], s_inv[0]), a.final_norm[i]);
    }
    // the last CTA out advances the launch number
    __syncthreads();
    if (t == 0) {
        __threadfence();
        if (atomicAdd(a.sync, 1u) == (unsigned)G - 1) {
            a.sync[0] = 0u;
            a.sync[1] = a.sync[1] + 1u;
            __threadfence();
        }
    }
}

// The library's two bounded waits run out on purpose, with nothing in flight: kind 0 polls
// tagged hand-over words (mk_poll) that carry no tag, kind 1 waits on an mbarrier expecting bytes
// that no copy will bring.  Both give up after g_wait_cycles and set their fault word, which the
// host reports as NC_ERR_KERNEL (nc_selftest_wait).
__global__ void __launch_bounds__(MK_THREADS) wait_selftest_kernel(const unsigned long long *words, int n, int kind) {
    __shared__ uint64_t bar;
    const long long limit = g_wait_cycles;
    if (kind == 0) {
        const bool ok = mk_poll(n, 0x5eedu, [&](int i) { return words + i; }, [&](int, uint32_t) {}, limit);
        if (!ok && threadIdx.x == 0) atomicExch(&g_mk_fault, 1u);
        return;
    }
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(&bar, 1024);                  // the arrival comes, the bytes never do
        if (!mbar_wait_for(&bar, 0, limit)) atomicOr(&g_attention_fault, 1u);
    }
}

}  // namespace nc
