// nc_common.cuh -- device helpers shared by the kernels.
//
// Everything here computes exactly what nanocompile's generated C computes (that code is
// compiled with -ffp-contract=off, nanocompile/codegen_c.py:50).  This file is compiled with
// -fmad=false, and the order-sensitive arithmetic is spelled with explicit round-to-nearest
// intrinsics so no contraction or reassociation can change a bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nc {

constexpr int QBLOCK = 32;     // nanocompile/quantize.py:43, activation scale block
constexpr int CHUNK = 128;     // nanocompile/lower.py:360 VNNI_STRIDE: four 32-byte groups

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// ---- glibc's expf ------------------------------------------------------------------------
// The softmax and SiLU of the reference call the C library's expf.  glibc (2.28+) computes it
// with the table-driven method of ARM's optimized-routines: x * 32/ln2 = k + r, then
// exp(x) = 2^(k/32) * p(r) with a cubic p, all in double, rounded once to float.  This is a
// restatement of that method (the table is 2^(i/32) from its definition, with the exponent
// bits of i/32 folded out); the remainder is a fused multiply-subtract as in glibc's FMA
// build.  Every float input in (-103.9, 88.7) gives glibc's bits (checked on the CPU for all
// 2.24e9 of them, and on the device by the tests).
__device__ __constant__ uint64_t kExpTab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

__device__ __forceinline__ float expf_exact(float x, const uint64_t *tab) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) {                          // |x| >= 88, inf or nan
        if (ux == 0xff800000u) return 0.0f;          // exp(-inf)
        if (abstop >= 0x7f8) return x + x;           // +inf, nan
        if (x > 0x1.62e42ep6f) return __uint_as_float(0x7f800000u);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_32 = 0x1.71547652b82fep+0 * 32;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double xd = (double)x;
    const double z = __dmul_rn(inv_ln2_32, xd);
    double kd = __dadd_rn(z, shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2_32, xd, -kd);
    const uint64_t t = tab[ki & 31] + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double p = __fma_rn(c0, r, c1);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(p, __dmul_rn(r, r), y);
    return __double2float_rn(__dmul_rn(y, s));
}

// ---- int8 lanes ---------------------------------------------------------------------------
// nanocompile/codegen_c.py:85-89 nc_dp4: sum over 4 bytes of (w + 128) * x.  The weights are
// stored already offset (u8 = w ^ 0x80), so one dp4a.u32.s32 gives the lane.  Seeding the
// accumulator with the bits of 1.5 * 2^23 makes the result the float 12582912 + v exactly
// (|v| <= 4 * 255 * 127 < 2^22), so int -> float is one exact subtraction, not a conversion.
// The Dp4 lane as the float 1.5 * 2^23 + Dp4 (exact: |Dp4| < 2^22); subtracting 1.5 * 2^23 gives it.
__device__ __forceinline__ float dp4_biased(uint32_t w_u8x4, uint32_t x_s8x4) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_u8x4), "r"(x_s8x4), "r"(0x4B400000));
    return __int_as_float(d);
}

__device__ __forceinline__ float dp4_lane(uint32_t w_u8x4, uint32_t x_s8x4) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_u8x4), "r"(x_s8x4), "r"(0x4B400000));
    return __fsub_rn(__int_as_float(d), 12582912.0f);
}

// ---- reductions -------------------------------------------------------------------------
// The reference's max: acc = (acc < v || v != v) ? v : acc (nanocompile/fusion.py:603-610).
// Any NaN wins; otherwise the maximum, independent of order (only +-0 compare equal with
// different bits, and both give the same downstream result).
__device__ __forceinline__ float nan_max(float acc, float v) { return (acc < v || v != v) ? v : acc; }

__device__ __forceinline__ float warp_nan_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// nanocompile/lower.py:298-317 _combine: (acc0+acc1)+(acc2+acc3) lane by lane, then lanes j
// and j+4, then two hadds.
__device__ __forceinline__ float combine32(const float *acc) {
    float h[8];
#pragma unroll
    for (int kh = 0; kh < 8; ++kh) h[kh] = fadd(fadd(acc[kh], acc[8 + kh]), fadd(acc[16 + kh], acc[24 + kh]));
    return fadd(fadd(fadd(h[0], h[4]), fadd(h[1], h[5])), fadd(fadd(h[2], h[6]), fadd(h[3], h[7])));
}

// nanocompile/nn.py:41-55: silu(g) * u with e = expf(-|g|), sigma = (g >= 0 ? 1 : e) / (1 + e).
__device__ __forceinline__ float swiglu(float g, float u, const uint64_t *tab) {
    const bool nonneg = 0.0f <= g;
    const float e = expf_exact(nonneg ? -g : g, tab);
    const float sig = fdiv(nonneg ? 1.0f : e, fadd(e, 1.0f));
    return fmul(fmul(g, sig), u);
}

// One 32-value block of block-32 quantization by one warp, lane = position in the block
// (nanocompile/quantize.py:102-124): returns the scale; *q the lane's int8 and *bsum the
// block's int32 sum.  |v| >= 0 orders like its bit pattern, so the block maximum is one
// integer max-reduction; a NaN anywhere makes the maximum a NaN, as the reference's
// NaN-propagating max does (only the NaN payload may differ).  A -0 magnitude becomes +0,
// which gives the same scale (mag <= 0 -> 1).
__device__ __forceinline__ float block_magnitude(float v) {
    return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v) & 0x7fffffffu));
}
// The IEEE divide for rare fallbacks, as a call: inlined, the compiler may evaluate it on every
// path before the branch that needs it.
__device__ __noinline__ float fdiv_slow(float a, float b) { return __fdiv_rn(a, b); }

// mag / 127 correctly rounded, without the IEEE divide's branchy slow path: q0 = mag * y with
// y = RN(1/127), then one remainder correction r = mag - q0 * 127 (exact, by FMA), q = q0 + r * y
// (the correction step of Markstein's FMA division).  Checked equal to IEEE division for every
// non-negative float by nc_selfcheck_div127; non-finite and tiny magnitudes take the IEEE divide.
__device__ __forceinline__ float div127(float mag) {
    const float y = 0x1.020408p-7f;                      // RN(1/127)
    if (!(mag < 0x1p+120f) || mag < 0x1p-100f) return fdiv_slow(mag, 127.0f);
    const float q0 = fmul(mag, y);
    const float r = __fmaf_rn(-q0, 127.0f, mag);
    return __fmaf_rn(r, y, q0);
}
__device__ __forceinline__ float block_scale(float mag) { return (mag <= 0.0f) ? 1.0f : div127(mag); }

// a / b, correctly rounded, for many a over one b > 0 (softmax's division by the sum), given
// y = RN(1/b): q = RN(a*y) corrected once by its residual (Markstein), and accepted only when
// the residual a - b*q -- exact, because q is within an ulp of a/b -- proves q nearest:
// |a - b*q| < b * ulp(q)/2 (ulp(q)/4 at a power of two, where the spacing below halves).
// Anything else (huge or tiny quotients, NaN, an undecided residual) takes the IEEE divide.
// The fallback is a call (fdiv_slow) so the compiler cannot hoist the IEEE divide into the common path.

__device__ __forceinline__ float fdiv_recip(float a, float b, float y) {
    const float q0 = fmul(a, y);
    const float q = __fmaf_rn(__fmaf_rn(-b, q0, a), y, q0);
    const uint32_t uq = __float_as_uint(q) & 0x7fffffffu;
    if (uq >= 0x0d800000u && uq < 0x71800000u) {            // 2^-100 <= |q| < 2^100
        const float r = __fmaf_rn(-b, q, a);
        const float half_ulp = __uint_as_float((uq & 0x7f800000u) - (24u << 23));
        const float lim = fmul(b, (uq & 0x7fffffu) ? half_ulp : fmul(half_ulp, 0.5f));
        if (fabsf(r) < lim) return q;
    }
    return fdiv_slow(a, b);
}
// xq = (int8)clamp(roundf(v / scale), -127, 127).  Only the rounded integer is kept, so the
// quotient may come from the fast approximate divide (error <= 2 ulp, |v / scale| <= 128): the
// rounding can only differ from IEEE division's when the quotient is within 2 ulp of a
// half-integer, and every quotient within 1/512 of one is recomputed with the IEEE divide.
__device__ __forceinline__ int8_t quantize_value(float v, float scale) {
    float t = __fdividef(v, scale);
    const float a = fabsf(t);
    if (!(a < 256.0f) || !(scale >= 0x1p-100f) || fabsf(a - floorf(a) - 0.5f) < (1.0f / 512)) t = fdiv_slow(v, scale);
    t = roundf(t);
    t = (t <= 127.0f) ? t : 127.0f;
    t = (-127.0f <= t) ? t : -127.0f;
    return (int8_t)t;
}
// N blocks at once by one warp (lane = position in each block): the same scales, int8 values and
// block sums as N calls of quantize_block_warp, with the rare IEEE-divide fallbacks taken after
// every block's fast path, so the N blocks' dependent chains overlap.
template <int N>
__device__ __forceinline__ void quantize_blocks_warp(const float *v, int8_t *q, float *scale, int *bsum) {
    const float y = 0x1.020408p-7f;                      // RN(1/127), as in div127
    float mag[N], t[N];
    bool slow_scale = false, slow_q = false, sl[N];
#pragma unroll
    for (int u = 0; u < N; ++u) mag[u] = block_magnitude(v[u]);
#pragma unroll
    for (int u = 0; u < N; ++u) {
        const float q0 = fmul(mag[u], y);
        scale[u] = (mag[u] <= 0.0f) ? 1.0f : __fmaf_rn(__fmaf_rn(-q0, 127.0f, mag[u]), y, q0);
        slow_scale |= !(mag[u] <= 0.0f) && (!(mag[u] < 0x1p+120f) || mag[u] < 0x1p-100f);
    }
    if (slow_scale) {                                    // the same in every lane: mag is the block's
#pragma unroll
        for (int u = 0; u < N; ++u)
            if (!(mag[u] <= 0.0f) && (!(mag[u] < 0x1p+120f) || mag[u] < 0x1p-100f)) scale[u] = fdiv_slow(mag[u], 127.0f);
    }
#pragma unroll
    for (int u = 0; u < N; ++u) {
        t[u] = __fdividef(v[u], scale[u]);
        const float a = fabsf(t[u]);
        sl[u] = !(a < 256.0f) || !(scale[u] >= 0x1p-100f) || fabsf(a - floorf(a) - 0.5f) < (1.0f / 512);
        slow_q |= sl[u];
    }
    if (__any_sync(0xffffffffu, slow_q)) {
#pragma unroll
        for (int u = 0; u < N; ++u)
            if (sl[u]) t[u] = fdiv_slow(v[u], scale[u]);
    }
#pragma unroll
    for (int u = 0; u < N; ++u) {
        float r = roundf(t[u]);
        r = (r <= 127.0f) ? r : 127.0f;
        r = (-127.0f <= r) ? r : -127.0f;
        q[u] = (int8_t)r;
    }
#pragma unroll
    for (int u = 0; u < N; ++u) bsum[u] = __reduce_add_sync(0xffffffffu, (int)q[u]);
}

// Out of line: the persistent decode kernel calls it from two places every layer.
__device__ __noinline__ float quantize_block_warp(float v, int8_t *q, int *bsum) {
    float scale;
    quantize_blocks_warp<1>(&v, q, &scale, bsum);
    return scale;
}

// ---- in-order sums -------------------------------------------------------------------------
// acc = acc + p[0] + p[1] + ... strictly left to right, by one thread.  Two 32-value register
// buffers alternate: the next block's shared-memory loads are issued before the current
// block's 32 dependent adds (unconditionally: past the last block they reload it), so the chain
// runs at the add latency.  p must be 16-byte aligned and readable up to the next multiple of 4
// elements; the last n % 32 come as 16-byte loads, then their adds in order.
__device__ __forceinline__ void add32(float &acc, const float4 *v) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        acc = fadd(acc, v[u].x);
        acc = fadd(acc, v[u].y);
        acc = fadd(acc, v[u].z);
        acc = fadd(acc, v[u].w);
    }
}

__device__ __forceinline__ float chain_sum(const float *p, int n, float acc = 0.0f) {
    const int n32 = n & ~31;
    const float4 *p4 = reinterpret_cast<const float4 *>(p);
    float4 a[8], b[8];
    int i = 0;
    if (n32) {
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = p4[u];
#pragma unroll 1
        for (; i + 64 <= n32; i += 64) {
#pragma unroll
            for (int u = 0; u < 8; ++u) b[u] = p4[(i + 32) / 4 + u];
            add32(acc, a);
            const int na = min(i + 64, n32 - 32);
#pragma unroll
            for (int u = 0; u < 8; ++u) a[u] = p4[na / 4 + u];
            add32(acc, b);
        }
        if (i < n32) {
            add32(acc, a);
            i += 32;
        }
    }
    if (i < n) {
        const int nt = n - i;
#pragma unroll
        for (int u = 0; u < 8; ++u) b[u] = 4 * u < nt ? p4[i / 4 + u] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (4 * u < nt) acc = fadd(acc, b[u].x);
            if (4 * u + 1 < nt) acc = fadd(acc, b[u].y);
            if (4 * u + 2 < nt) acc = fadd(acc, b[u].z);
            if (4 * u + 3 < nt) acc = fadd(acc, b[u].w);
        }
    }
    return acc;
}

// ---- bounded waits ------------------------------------------------------------------------------
// Every spin on a flag or an mbarrier gives up after a number of SM cycles.  Waits after which a
// kernel can stop, drain what it has in flight and return use g_wait_cycles (default 2^31, about a
// second; nc_set_wait_limit changes it per device, for tests that make a wait run out); the waits
// that drain work already in flight, and the waits of kernels that cannot stop early, use the
// fixed NC_DRAIN_CYCLES.
__device__ long long g_wait_cycles = 1ll << 31;
constexpr long long NC_DRAIN_CYCLES = 1ll << 31;

// ---- programmatic dependent launch -----------------------------------------------------------
// Every kernel of a step is launched with programmatic stream serialization: it may start while
// the previous kernel still runs, loads what does not depend on it (weights, scales, the KV
// history), and waits here before touching the previous kernel's outputs -- or writing anything.
// Launched without the attribute, both instructions are no-ops.
__device__ __forceinline__ void wait_for_producer() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void release_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- epilogues ----------------------------------------------------------------------------
enum Epilogue : int { EPI_NONE = 0, EPI_BIAS = 1, EPI_RESIDUAL = 2, EPI_SWIGLU = 3 };

}  // namespace nc
