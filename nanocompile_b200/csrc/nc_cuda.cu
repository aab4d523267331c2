// nc_cuda.cu -- libnc_cuda.so: the C ABI of include/nc_cuda.h.
//
// The model runtime is the CUDA twin of nanocompile/runtime.py's CompiledGraph
// (nanocompile/runtime.py:167-318): built once per model, then called per step.  The
// reference plans an arena per call and crosses the FFI once per fused kernel
// (runtime.py:281-299); here one device arena is laid out at creation, every step is the
// same fixed sequence of fused kernels reading its sizes from device memory, and decode
// steps replay one captured CUDA graph.
#include "../../include/nc_cuda.h"
#include "nc_attention.cuh"
#include "nc_gemm_f32.cuh"
#include "nc_lm_head_tc.cuh"
#include "nc_lm_head_q8.cuh"
#include "nc_decode_mk.cuh"
#include "nc_gemm_i8.cuh"
#include "nc_gemm_i8_tc.cuh"
#include "nc_gemm_i8f.cuh"

#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

using namespace nc;

// ---- errors ---------------------------------------------------------------------------------
static thread_local std::string g_error;

static int32_t fail(int32_t code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                       \
    do {                                                                                     \
        cudaError_t e_ = (expr);                                                             \
        if (e_ != cudaSuccess)                                                               \
            return fail(NC_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                                 \
    } while (0)

#define NC_TRY(expr)                  \
    do {                              \
        int32_t s_ = (expr);          \
        if (s_ != NC_OK) return s_;   \
    } while (0)

extern "C" int32_t nc_last_error(char *buf, int64_t size) {
    if (buf && size > 0) {
        std::snprintf(buf, (size_t)size, "%s", g_error.c_str());
    }
    return (int32_t)g_error.size();
}

extern "C" int32_t nc_device_count(int32_t *count) {
    int n = 0;
    CUDA_TRY(cudaGetDeviceCount(&n));
    *count = n;
    return NC_OK;
}
extern "C" int32_t nc_set_device(int32_t device) {
    CUDA_TRY(cudaSetDevice(device));
    return NC_OK;
}
extern "C" int32_t nc_device_alloc(int64_t bytes, void **ptr) {
    CUDA_TRY(cudaMalloc(ptr, (size_t)(bytes > 0 ? bytes : 1)));
    return NC_OK;
}
extern "C" int32_t nc_device_free(void *ptr) {
    CUDA_TRY(cudaFree(ptr));
    return NC_OK;
}
extern "C" int32_t nc_copy_to_device(void *dst, const void *src, int64_t bytes) {
    CUDA_TRY(cudaMemcpy(dst, src, (size_t)bytes, cudaMemcpyHostToDevice));
    return NC_OK;
}
extern "C" int32_t nc_copy_to_host(void *dst, const void *src, int64_t bytes) {
    CUDA_TRY(cudaMemcpy(dst, src, (size_t)bytes, cudaMemcpyDeviceToHost));
    return NC_OK;
}
extern "C" int32_t nc_device_synchronize(void) {
    CUDA_TRY(cudaDeviceSynchronize());
    return NC_OK;
}

// ---- kernel launchers (shared by the fused-group ABI and the model) -------------------------
namespace {

// Every kernel of the step is launched with programmatic stream serialization (PDL): it may
// begin while its predecessor runs, prefetch immutable data (weights), and wait in-kernel for
// the predecessor's results.  NC_PDL=0 in the environment turns it off (for A/B timing).
bool pdl_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NC_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// NC_SPLIT_ATTENTION=0 keeps few-row attention at one CTA per query head.
bool split_attention_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NC_SPLIT_ATTENTION");
        return !(v && v[0] == '0');
    }();
    return on;
}

// NC_MK=0 keeps small int8 decode steps on the separate kernels.
bool mk_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NC_MK");
        return !(v && v[0] == '0');
    }();
    return on;
}

// NC_Q8_HEAD=0 turns the int8-prefiltered LM head of small decode steps off.
bool q8_head_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NC_Q8_HEAD");
        return !(v && v[0] == '0');
    }();
    return on;
}

// NC_TC_HEAD=0 keeps every LM head on the CUDA cores.
bool tc_head_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("NC_TC_HEAD");
        return !(v && v[0] == '0');
    }();
    return on;
}

// The tensor-core (tcgen05 kind::i8) batched projection is opt-in (NC_TC_I8=1): measured on a
// B200 it is slower than the dp4a kernel at 64 and 512 rows (gate/up 63 vs 41 us at 64 rows; 432
// vs 288 us at 512): one MMA per 32-byte group of N = 32 (token, lane) columns costs ~240 cycles
// to issue and complete, and only 1/8 of each block-diagonal operand is useful.
// Read at every launch decision (a captured decode graph keeps the choice it was captured with).
bool tc_i8_enabled() {
    const char *v = std::getenv("NC_TC_I8");
    return v && v[0] == '1';
}

int sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return sms > 0 ? sms : 148;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename K>
cudaError_t allow_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

int32_t check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(NC_ERR_CUDA, "launching %s: %s", what, cudaGetErrorString(e));
    return NC_OK;
}

int32_t launch_norm(cudaStream_t st, float *normed, const float *x, const float *w, int8_t *xq, float *xs,
                    float *off, int32_t *bsums, const int32_t *row_map, int rows, int n, float eps) {
    if (rows <= 0) return NC_OK;
    if (n > 8192 || (xq && n % QBLOCK)) return fail(NC_ERR_ARGUMENT, "rms_norm width %d unsupported", n);
    const size_t smem = sizeof(float) * 3 * (((size_t)n + 3) / 4 * 4);
    CUDA_TRY(allow_smem(norm_quant_kernel, smem));
    CUDA_TRY(launch_k(norm_quant_kernel, rows, NORM_THREADS, smem, st, normed, x, w, xq, xs, off, bsums, row_map, n, eps));
    return check_launch("norm_quant_kernel");
}

int32_t launch_quant(cudaStream_t st, int8_t *xq, const float *x, float *xs, float *off, int32_t *bsums,
                     int rows, int k) {
    if (rows <= 0) return NC_OK;
    if (k % QBLOCK || k > 8192) return fail(NC_ERR_ARGUMENT, "quantize width %d unsupported", k);
    CUDA_TRY(allow_smem(quantize_kernel, sizeof(float) * k));
    CUDA_TRY(launch_k(quantize_kernel, rows, NORM_THREADS, sizeof(float) * k, st, xq, x, xs, off, bsums, k));
    return check_launch("quantize_kernel");
}

template <int LPR, int TOK, int UNROLL>
int32_t launch_i8_epi(cudaStream_t st, const GemvI8Args &a, int epi) {
    constexpr int WARPS = 4, RPW = 32 / LPR;
    const int grid = (a.n + WARPS * RPW - 1) / (WARPS * RPW);
    switch (epi) {
        case EPI_NONE: CUDA_TRY(launch_k(gemv_i8_kernel<LPR, TOK, UNROLL, EPI_NONE>, grid, 32 * WARPS, 0, st, a)); break;
        case EPI_BIAS: CUDA_TRY(launch_k(gemv_i8_kernel<LPR, TOK, UNROLL, EPI_BIAS>, grid, 32 * WARPS, 0, st, a)); break;
        case EPI_RESIDUAL: CUDA_TRY(launch_k(gemv_i8_kernel<LPR, TOK, UNROLL, EPI_RESIDUAL>, grid, 32 * WARPS, 0, st, a)); break;
        case EPI_SWIGLU: CUDA_TRY(launch_k(gemv_i8_kernel<LPR, TOK, UNROLL, EPI_SWIGLU>, grid, 32 * WARPS, 0, st, a)); break;
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
    return check_launch("gemv_i8_kernel");
}

template <int LPR, int NCH, int MAXG, int PRO, int EPI, int TB>
int32_t launch_fused_t(cudaStream_t st, const FusedI8Args &f, size_t smem) {
    constexpr int THREADS = 256, ROWS = (THREADS / 32) * (32 / LPR);
    auto kernel = gemv_i8_fused_kernel<LPR, NCH, MAXG, PRO, EPI, TB>;
    CUDA_TRY(allow_smem(kernel, smem));
    CUDA_TRY(launch_k(kernel, (f.g.n + ROWS - 1) / ROWS, THREADS, smem, st, f));
    return check_launch("gemv_i8_fused_kernel");
}

// Several tokens are advanced together only in the batched model path's combinations.
template <int PRO, int EPI>
constexpr bool batched_combo() {
    return (PRO == PRO_NONE && (EPI == EPI_BIAS || EPI == EPI_RESIDUAL || EPI == EPI_SWIGLU_QUANT)) ||
           (PRO == PRO_OFFSET && EPI == EPI_RESIDUAL);
}

template <int LPR, int NCH, int MAXG, int PRO, int EPI>
int32_t launch_fused_tb(cudaStream_t st, const FusedI8Args &f, size_t smem) {
    if constexpr (batched_combo<PRO, EPI>()) {
        if (f.g.m >= 4) return launch_fused_t<LPR, NCH, MAXG, PRO, EPI, 4>(st, f, smem);
    }
    return launch_fused_t<LPR, NCH, MAXG, PRO, EPI, 1>(st, f, smem);
}

template <int LPR, int NCH, int MAXG, int PRO>
int32_t launch_fused_epi(cudaStream_t st, const FusedI8Args &f, int epi, size_t smem) {
    switch (epi) {
        case EPI_NONE: return launch_fused_tb<LPR, NCH, MAXG, PRO, EPI_NONE>(st, f, smem);
        case EPI_BIAS: return launch_fused_tb<LPR, NCH, MAXG, PRO, EPI_BIAS>(st, f, smem);
        case EPI_RESIDUAL: return launch_fused_tb<LPR, NCH, MAXG, PRO, EPI_RESIDUAL>(st, f, smem);
        case EPI_SWIGLU: return launch_fused_tb<LPR, NCH, MAXG, PRO, EPI_SWIGLU>(st, f, smem);
        case EPI_SWIGLU_QUANT: return launch_fused_tb<LPR, NCH, MAXG, PRO, EPI_SWIGLU_QUANT>(st, f, smem);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

template <int LPR, int NCH, int MAXG>
int32_t launch_fused_pro_g(cudaStream_t st, const FusedI8Args &f, int pro, int epi, size_t smem) {
    switch (pro) {
        case PRO_NONE: return launch_fused_epi<LPR, NCH, MAXG, PRO_NONE>(st, f, epi, smem);
        case PRO_OFFSET: return launch_fused_epi<LPR, NCH, MAXG, PRO_OFFSET>(st, f, epi, smem);
        case PRO_NORM:
            if constexpr (NCH <= 8) return launch_fused_epi<LPR, NCH, MAXG, PRO_NORM>(st, f, epi, smem);
            return fail(NC_ERR_ARGUMENT, "the norm prologue takes widths up to 1024");
        default: return fail(NC_ERR_ARGUMENT, "unknown prologue %d", pro);
    }
}

// Widths that are whole 128-byte chunks (the model's) use the variant without tail registers.
template <int LPR, int NCH>
int32_t launch_fused_pro(cudaStream_t st, const FusedI8Args &f, int pro, int epi, size_t smem) {
    if (f.g.k % CHUNK == 0) return launch_fused_pro_g<LPR, NCH, 0>(st, f, pro, epi, smem);
    return launch_fused_pro_g<LPR, NCH, 3>(st, f, pro, epi, smem);
}

// Batched projection (more than four rows): R rows x T tokens per warp, 8 warps per CTA.
template <int R, int T, int MAXG, int PRO, int EPI>
int32_t launch_gemm_t(cudaStream_t st, const FusedI8Args &f) {
    constexpr int ROWS = GEMM_WARPS * R;
    auto kernel = gemm_i8_kernel<R, T, MAXG, PRO, EPI>;
    const size_t smem = gemm_i8_smem(T, ROWS, f.g.k, PRO == PRO_OFFSET, EPI == EPI_SWIGLU_QUANT);
    if (smem > 200 * 1024) return fail(NC_ERR_ARGUMENT, "int8 width %d too wide for the batched projection", f.g.k);
    CUDA_TRY(allow_smem(kernel, smem));
    const dim3 grid((f.g.n + ROWS - 1) / ROWS, (f.g.m + T - 1) / T);
    CUDA_TRY(launch_k(kernel, grid, GEMM_WARPS * 32, smem, st, f));
    return check_launch("gemm_i8_kernel");
}

template <int MAXG, int PRO>
int32_t launch_gemm_epi(cudaStream_t st, const FusedI8Args &f, int epi) {
    switch (epi) {
        case EPI_NONE: return launch_gemm_t<4, 8, MAXG, PRO, EPI_NONE>(st, f);
        case EPI_BIAS: return launch_gemm_t<4, 8, MAXG, PRO, EPI_BIAS>(st, f);
        case EPI_RESIDUAL: return launch_gemm_t<4, 8, MAXG, PRO, EPI_RESIDUAL>(st, f);
        case EPI_SWIGLU: return launch_gemm_t<4, 8, MAXG, PRO, EPI_SWIGLU>(st, f);
        case EPI_SWIGLU_QUANT: return launch_gemm_t<4, 8, MAXG, PRO, EPI_SWIGLU_QUANT>(st, f);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

template <int MAXG>
int32_t launch_gemm_pro(cudaStream_t st, const FusedI8Args &f, int pro, int epi) {
    switch (pro) {
        case PRO_NONE: return launch_gemm_epi<MAXG, PRO_NONE>(st, f, epi);
        case PRO_OFFSET: return launch_gemm_epi<MAXG, PRO_OFFSET>(st, f, epi);
        default: return fail(NC_ERR_ARGUMENT, "prologue %d is not a batched one", pro);
    }
}

// The int8-vnni projection. More than four rows: the batched kernel. Otherwise
// weights-stationary, lanes per row chosen by shape (a row's slices must fit in registers: up
// to 8 chunks of 16 or 8 bytes per lane, or 40 chunks of 4 bytes).
int32_t launch_i8_fused(cudaStream_t st, const FusedI8Args &f, int pro, int epi) {
    const GemvI8Args &a = f.g;
    if (a.m <= 0 || a.n <= 0) return NC_OK;
    if (a.k % QBLOCK) return fail(NC_ERR_ARGUMENT, "int8 width %d is not a whole number of 32-blocks", a.k);
    if (pro == PRO_NORM && a.m > PRO_NORM_ROWS) return fail(NC_ERR_ARGUMENT, "the norm prologue takes up to 4 rows");
    if (epi == EPI_SWIGLU_QUANT && a.n % QBLOCK) return fail(NC_ERR_ARGUMENT, "quantized output width %d", a.n);
    if (pro != PRO_NORM && a.m > PRO_NORM_ROWS) {
        if (a.k % CHUNK == 0) return launch_gemm_pro<0>(st, f, pro, epi);
        return launch_gemm_pro<3>(st, f, pro, epi);
    }
    const int blocks = a.k / QBLOCK, bl4 = (blocks + 3) & ~3, chunks = a.k / CHUNK;
    if (a.k % 16) return fail(NC_ERR_ARGUMENT, "int8 width %d is not a multiple of 16", a.k);
    const int tile = pro == PRO_NORM ? PRO_NORM_ROWS : std::min(a.m, act_tile_tokens(a.k));
    if (tile < 1) return fail(NC_ERR_ARGUMENT, "int8 width %d too wide for the activation tile", a.k);
    size_t smem = (size_t)tile * a.k + sizeof(float) * ((size_t)tile * bl4 + ((a.m + 3) & ~3));
    if (pro == PRO_NORM) smem += sizeof(float) * ((size_t)bl4 + 3 * (size_t)a.k);
    if (pro == PRO_OFFSET) smem += sizeof(float) * (size_t)a.m * bl4;
    if (smem > 200 * 1024) return fail(NC_ERR_ARGUMENT, "projection needs too much shared memory");
    if (chunks <= 8) {
        if (a.n <= 2048 && epi != EPI_SWIGLU_QUANT) return launch_fused_pro<16, 8>(st, f, pro, epi, smem);
        return launch_fused_pro<8, 8>(st, f, pro, epi, smem);
    }
    if (chunks <= 40 && epi != EPI_SWIGLU_QUANT) return launch_fused_pro<32, 40>(st, f, pro, epi, smem);
    if (pro != PRO_NONE || epi == EPI_SWIGLU_QUANT)
        return fail(NC_ERR_ARGUMENT, "int8 width %d too wide for the fused projection", a.k);
    return a.m == 1 ? launch_i8_epi<32, 1, 16>(st, a, epi) : launch_i8_epi<32, 4, 16>(st, a, epi);
}

int32_t launch_i8(cudaStream_t st, const GemvI8Args &a, int epi) {
    FusedI8Args f{};
    f.g = a;
    return launch_i8_fused(st, f, PRO_NONE, epi);
}

template <int TOK, int EPI, bool ARGMAX>
int32_t launch_f32_t(cudaStream_t st, const GemvF32Args &a) {
    constexpr int NW = EPI == EPI_SWIGLU ? 2 : 1;
    const size_t smem = sizeof(float4) * F32_STAGES * (NW * F32_ROWS * (F32_TILE / 4) + TOK * (F32_TILE / 4));
    auto kernel = gemv_f32_kernel<TOK, EPI, ARGMAX>;
    CUDA_TRY(allow_smem(kernel, smem));
    const int grid = (a.n + F32_ROWS - 1) / F32_ROWS;
    CUDA_TRY(launch_k(kernel, grid, F32_ROWS, smem, st, a));
    return check_launch("gemv_f32_kernel");
}

template <int TOK>
int32_t launch_f32_tok(cudaStream_t st, const GemvF32Args &a, int epi, bool argmax) {
    if (argmax) return launch_f32_t<TOK, EPI_NONE, true>(st, a);
    switch (epi) {
        case EPI_NONE: return launch_f32_t<TOK, EPI_NONE, false>(st, a);
        case EPI_BIAS: return launch_f32_t<TOK, EPI_BIAS, false>(st, a);
        case EPI_RESIDUAL: return launch_f32_t<TOK, EPI_RESIDUAL, false>(st, a);
        case EPI_SWIGLU: return launch_f32_t<TOK, EPI_SWIGLU, false>(st, a);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

// Many rows: one pass over the weights for up to 2*T rows (T = 16 or 32).
template <int T, int EPI, bool ARGMAX>
int32_t launch_gemm_f32_t(cudaStream_t st, const GemvF32Args &a) {
    auto kernel = gemm_f32_kernel<T, EPI, ARGMAX>;
    const size_t smem = gemm_f32_smem(T);
    CUDA_TRY(allow_smem(kernel, smem));
    const dim3 grid((a.n + F32_ROWS - 1) / F32_ROWS, (a.m + 2 * T - 1) / (2 * T));
    CUDA_TRY(launch_k(kernel, grid, GF_THREADS, smem, st, a));
    return check_launch("gemm_f32_kernel");
}

template <int T>
int32_t launch_gemm_f32(cudaStream_t st, const GemvF32Args &a, int epi, bool argmax) {
    if (argmax) return launch_gemm_f32_t<T, EPI_NONE, true>(st, a);
    switch (epi) {
        case EPI_NONE: return launch_gemm_f32_t<T, EPI_NONE, false>(st, a);
        case EPI_BIAS: return launch_gemm_f32_t<T, EPI_BIAS, false>(st, a);
        case EPI_RESIDUAL: return launch_gemm_f32_t<T, EPI_RESIDUAL, false>(st, a);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

int32_t launch_f32(cudaStream_t st, const GemvF32Args &a, int epi, bool argmax) {
    if (a.m <= 0 || a.n <= 0) return NC_OK;
    if (a.k % F32_TILE) return fail(NC_ERR_ARGUMENT, "float32 width %d is not a multiple of %d", a.k, F32_TILE);
    if (argmax && epi != EPI_NONE) return fail(NC_ERR_ARGUMENT, "argmax takes no epilogue");
    if (a.m > 16 && epi != EPI_SWIGLU)
        return a.m <= 32 ? launch_gemm_f32<16>(st, a, epi, argmax) : launch_gemm_f32<32>(st, a, epi, argmax);
    return a.m == 1 ? launch_f32_tok<1>(st, a, epi, argmax) : launch_f32_tok<16>(st, a, epi, argmax);
}

// int8 weights with float32 activations (matmul_i8): 64 output rows per CTA, tokens in passes
// of four (two with the SwiGLU pair of weights).
template <int T, int EPI>
int32_t launch_i8f_t(cudaStream_t st, const GemvI8fArgs &a) {
    CUDA_TRY(launch_k(gemv_i8f_kernel<T, EPI>, (a.n + I8F_ROWS - 1) / I8F_ROWS, I8F_WARPS * 32, 0, st, a));
    return check_launch("gemv_i8f_kernel");
}

int32_t launch_i8f(cudaStream_t st, const GemvI8fArgs &a, int epi) {
    if (a.m <= 0 || a.n <= 0) return NC_OK;
    if (a.k % 16 || a.k <= 0) return fail(NC_ERR_ARGUMENT, "int8 width %d is not a multiple of 16", a.k);
    switch (epi) {
        case EPI_NONE: return a.m == 1 ? launch_i8f_t<1, EPI_NONE>(st, a) : launch_i8f_t<4, EPI_NONE>(st, a);
        case EPI_BIAS: return a.m == 1 ? launch_i8f_t<1, EPI_BIAS>(st, a) : launch_i8f_t<4, EPI_BIAS>(st, a);
        case EPI_RESIDUAL: return a.m == 1 ? launch_i8f_t<1, EPI_RESIDUAL>(st, a) : launch_i8f_t<4, EPI_RESIDUAL>(st, a);
        case EPI_SWIGLU: return a.m == 1 ? launch_i8f_t<1, EPI_SWIGLU>(st, a) : launch_i8f_t<2, EPI_SWIGLU>(st, a);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

size_t attention_smem(int heads_per_cta, int d, int cap) {
    switch (d) {
        case 16: return sizeof(float) * attention_smem_floats<16>(heads_per_cta, cap);
        case 64: return sizeof(float) * attention_smem_floats<64>(heads_per_cta, cap);
        case 128: return sizeof(float) * attention_smem_floats<128>(heads_per_cta, cap);
        default: return (size_t)1 << 40;
    }
}

template <int D, int G>
int32_t launch_attention_g(cudaStream_t st, const AttnArgs &a, int rows) {
    const size_t smem = sizeof(float) * attention_smem_floats<D>(G, a.cap);
    if (smem > 220 * 1024) return fail(NC_ERR_ARGUMENT, "attention over %d positions exceeds shared memory", a.cap);
    CUDA_TRY(allow_smem(attention_kernel<D, G>, smem));
    CUDA_TRY(launch_k(attention_kernel<D, G>, rows * (a.heads / G), attention_threads(G), smem, st, a));
    return check_launch("attention_kernel");
}

// A 2-D tensor map over a KV arena seen as rows of d floats (rows < 2^31): 256-row x 32-float
// boxes, 128-byte swizzle. cuTensorMapEncodeTiled comes from the driver through the runtime.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int32_t make_kv_map(CUtensorMap *map, float *base, int64_t rows, int d) {
    static EncodeTiledFn encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<EncodeTiledFn>(fn);
    }();
    if (!encode) return fail(NC_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    if (rows <= 0 || rows >= (int64_t(1) << 31) || d % ATB_BOX || ((uintptr_t)base & 15))
        return fail(NC_ERR_ARGUMENT, "no tensor map for %lld rows of %d floats", (long long)rows, d);
    const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)d * sizeof(float)};
    const cuuint32_t box[2] = {ATB_BOX, ATB_CHUNK};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, elem,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NC_OK;
}

// A 2-D tensor map over int8 weights [n, k] (u8, k bytes per row): 128-byte x box_rows boxes,
// 128-byte swizzle, the K-major operand layout of tcgen05.mma; rows past n read as zeros.
int32_t make_i8_map(CUtensorMap *map, const uint8_t *w, int64_t n, int64_t k, int box_rows) {
    static EncodeTiledFn encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<EncodeTiledFn>(fn);
    }();
    if (!encode) return fail(NC_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    if (n <= 0 || n >= (int64_t(1) << 31) || k <= 0 || k % QBLOCK || ((uintptr_t)w & 15))
        return fail(NC_ERR_ARGUMENT, "no tensor map for int8 weights %lld x %lld", (long long)n, (long long)k);
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)k};
    const cuuint32_t box[2] = {(cuuint32_t)CHUNK, (cuuint32_t)box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)w, dims, strides, box, elem,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NC_ERR_CUDA, "cuTensorMapEncodeTiled (int8 weights) failed (%d)", (int)r);
    return NC_OK;
}

// The tensor-core int8 projection (more than four rows): persistent CTAs over items of 128 weight
// rows x 4 tokens.
template <int T, int PRO, int EPI>
int32_t launch_i8_tc_t(cudaStream_t st, const FusedI8Args &f, const CUtensorMap &m1, const CUtensorMap &m2) {
    constexpr bool TWO = EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_QUANT;
    auto kernel = gemm_i8_tc_kernel<T, PRO, EPI>;
    const I8TcLayout L = i8tc_layout(T, f.g.k);
    if (L.bytes > 227 * 1024) return fail(NC_ERR_ARGUMENT, "int8 width %d too wide for the tensor-core projection", f.g.k);
    CUDA_TRY(allow_smem(kernel, L.bytes));
    const int row_tiles = TWO ? (f.g.n + 63) / 64 : (f.g.n + I8TC_ROWS - 1) / I8TC_ROWS;
    const int items = row_tiles * ((f.g.m + T - 1) / T);
    CUDA_TRY(launch_k(kernel, std::min(items, sm_count()), I8TC_THREADS, L.bytes, st, f, m1, m2));
    return check_launch("gemm_i8_tc_kernel");
}

template <int T, int PRO>
int32_t launch_i8_tc_epi(cudaStream_t st, const FusedI8Args &f, int epi, const CUtensorMap &m1, const CUtensorMap &m2) {
    switch (epi) {
        case EPI_NONE: return launch_i8_tc_t<T, PRO, EPI_NONE>(st, f, m1, m2);
        case EPI_BIAS: return launch_i8_tc_t<T, PRO, EPI_BIAS>(st, f, m1, m2);
        case EPI_RESIDUAL: return launch_i8_tc_t<T, PRO, EPI_RESIDUAL>(st, f, m1, m2);
        case EPI_SWIGLU: return launch_i8_tc_t<T, PRO, EPI_SWIGLU>(st, f, m1, m2);
        case EPI_SWIGLU_QUANT: return launch_i8_tc_t<T, PRO, EPI_SWIGLU_QUANT>(st, f, m1, m2);
        default: return fail(NC_ERR_ARGUMENT, "unknown epilogue %d", epi);
    }
}

// tokens: 0 or 4 (items of four tokens, one per epilogue warp of a TMEM sub-partition).
int32_t launch_i8_tc(cudaStream_t st, const FusedI8Args &f, int pro, int epi, const CUtensorMap &m1,
                     const CUtensorMap &m2, int tokens = 0) {
    const GemvI8Args &a = f.g;
    if (a.m <= 0 || a.n <= 0) return NC_OK;
    if (a.k % QBLOCK) return fail(NC_ERR_ARGUMENT, "int8 width %d is not a whole number of 32-blocks", a.k);
    if (epi == EPI_SWIGLU_QUANT && a.n % QBLOCK) return fail(NC_ERR_ARGUMENT, "quantized output width %d", a.n);
    if (tokens != 0 && tokens != 4) return fail(NC_ERR_ARGUMENT, "tokens per item %d: 4", tokens);
    if (4 * (a.k / QBLOCK) > 2 * I8TC_EPI_WARPS * 32)
        return fail(NC_ERR_ARGUMENT, "int8 width %d too wide for the tensor-core projection", a.k);
    if (pro != PRO_NONE && pro != PRO_OFFSET) return fail(NC_ERR_ARGUMENT, "prologue %d is not a batched one", pro);
    return pro == PRO_NONE ? launch_i8_tc_epi<4, PRO_NONE>(st, f, epi, m1, m2)
                           : launch_i8_tc_epi<4, PRO_OFFSET>(st, f, epi, m1, m2);
}

template <int D, int G, bool TMA>
int32_t launch_attention_batched(cudaStream_t st, const AttnArgs &a, int rows, const CUtensorMap &map) {
    auto kernel = attention_batched_kernel<D, G, TMA>;
    const size_t smem = attention_batched_smem(D, a.cap);
    CUDA_TRY(allow_smem(kernel, smem));
    CUDA_TRY(launch_k(kernel, rows * a.kv, ATB_THREADS, smem, st, a, map));
    return check_launch("attention_batched_kernel");
}

template <int D, bool TMA>
int32_t launch_attention_group(cudaStream_t st, const AttnArgs &a, int rows, const CUtensorMap &map, bool *done) {
    *done = true;
    switch (a.heads / a.kv) {
        case 2: return launch_attention_batched<D, 2, TMA>(st, a, rows, map);
        case 4: return launch_attention_batched<D, 4, TMA>(st, a, rows, map);
        case 7: return launch_attention_batched<D, 7, TMA>(st, a, rows, map);
        case 8: return launch_attention_batched<D, 8, TMA>(st, a, rows, map);
        default: *done = false; return NC_OK;
    }
}

// Many rows: one CTA per (row, KV head) with its whole group, while its shared memory (a
// probability per cached position and head) fits; K/V by TMA when a tensor map describes the
// cache, by cp.async otherwise.
template <int D>
int32_t launch_attention_grouped(cudaStream_t st, const AttnArgs &a, int rows, const CUtensorMap *map, bool *done) {
    *done = false;
    if constexpr (D == 16 || D == 64) {
        if (attention_batched_smem(D, a.cap) > 225 * 1024) return NC_OK;
        if constexpr (D % ATB_BOX == 0) {
            if (map) return launch_attention_group<D, true>(st, a, rows, *map, done);
        }
        CUtensorMap none;
        std::memset(&none, 0, sizeof(none));
        return launch_attention_group<D, false>(st, a, rows, none, done);
    }
    return NC_OK;
}

// Few rows (decode of a handful of sequences): one CTA per query head, for parallelism.  Many
// rows: one CTA per KV head, reading each KV row once for its group of query heads.
template <int D>
int32_t launch_attention_split(cudaStream_t st, const AttnArgs &a, int rows) {
    const size_t smem = attention_split_smem(D, a.cap);
    CUDA_TRY(allow_smem(attention_split_kernel<D>, smem));
    CUDA_TRY(launch_k(attention_split_kernel<D>, rows * a.heads * (D / ATS_SLICE), ATS_THREADS, smem, st, a));
    return check_launch("attention_split_kernel");
}

template <int D>
int32_t launch_attention_d(cudaStream_t st, const AttnArgs &a, int rows, const CUtensorMap *map) {
    const int group = a.heads / a.kv;
    if constexpr (D == 64) {
        // few rows, the cache behind a tensor map: the split items with K and V by TMA
        if (rows <= 8 && map && attention_tma_smem(a.cap) <= 220 * 1024 && split_attention_enabled()) {
            const size_t smem = attention_tma_smem(a.cap);
            CUDA_TRY(allow_smem(attention_split_tma_kernel, smem));
            CUDA_TRY(launch_k(attention_split_tma_kernel, rows * a.heads * (D / ATS_SLICE), ATT_THREADS, smem, st, a, *map));
            return check_launch("attention_split_tma_kernel");
        }
    }
    if constexpr (D % ATS_SLICE == 0) {
        // few rows: (row, head, 32-dimension slice) CTAs, while a probability per position fits
        if (rows <= 8 && attention_split_smem(D, a.cap) <= 200 * 1024 && split_attention_enabled())
            return launch_attention_split<D>(st, a, rows);
    }
    if (rows <= 8 || group == 1) return launch_attention_g<D, 1>(st, a, rows);
    bool done;
    const int32_t s = launch_attention_grouped<D>(st, a, rows, map, &done);
    if (done || s != NC_OK) return s;
    switch (group) {
        case 2: return launch_attention_g<D, 2>(st, a, rows);
        case 4: return launch_attention_g<D, 4>(st, a, rows);
        case 7: return launch_attention_g<D, 7>(st, a, rows);
        case 8: return launch_attention_g<D, 8>(st, a, rows);
        default: return launch_attention_g<D, 1>(st, a, rows);
    }
}

// map: a tensor map over the KV arena that holds a.cache (a.cache_row0 its row), or null.
int32_t launch_attention(cudaStream_t st, const AttnArgs &a, int rows, const CUtensorMap *map = nullptr) {
    if (rows <= 0) return NC_OK;
    const int group = a.heads / a.kv;
    if (a.heads % a.kv || group > ATTN_MAX_GROUP || group * a.d > attention_threads(group))
        return fail(NC_ERR_ARGUMENT, "attention with %d heads over %d KV heads of dim %d is unsupported", a.heads,
                    a.kv, a.d);
    if (a.q_out && a.d % QBLOCK) return fail(NC_ERR_ARGUMENT, "quantized attention output needs whole blocks");
    switch (a.d) {
        case 16: return launch_attention_d<16>(st, a, rows, map);
        case 64: return launch_attention_d<64>(st, a, rows, map);
        case 128: return launch_attention_d<128>(st, a, rows, map);
        default: return fail(NC_ERR_ARGUMENT, "head dim %d unsupported (16, 64, 128)", a.d);
    }
}

// A grouped-attention CTA whose TMA stage never completed (bounded wait) records it in
// g_attention_fault; the host reads and clears the flag after a step.
int32_t check_device_faults() {
    unsigned int fault = 0;
    CUDA_TRY(cudaMemcpyFromSymbol(&fault, g_attention_fault, sizeof(fault)));
    if (fault) {
        const unsigned int zero = 0;
        CUDA_TRY(cudaMemcpyToSymbol(g_attention_fault, &zero, sizeof(zero)));
        return fail(NC_ERR_KERNEL, "a pipeline stage (K/V, weight tile or tensor-core result) did not arrive within "
                                   "its wait limit");
    }
    CUDA_TRY(cudaMemcpyFromSymbol(&fault, g_mk_fault, sizeof(fault)));
    if (fault) {
        const unsigned int zero = 0;
        CUDA_TRY(cudaMemcpyToSymbol(g_mk_fault, &zero, sizeof(zero)));
        return fail(NC_ERR_KERNEL, "persistent decode step: a hand-over word did not arrive within its wait limit");
    }
    return NC_OK;
}

float f32_from_bits(int64_t bits) {
    uint32_t u = (uint32_t)bits;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

}  // namespace

// ---- 1. fused-group entry points -------------------------------------------------------------

extern "C" int32_t nc_gather_rows(void **p, const int64_t *s, void *stream) {
    const int rows = (int)s[0];
    if (rows <= 0) return NC_OK;
    CUDA_TRY(launch_k(gather_kernel, rows, 256, 0, (cudaStream_t)stream, (float *)p[0], (const int64_t *)p[1],
                      (const float *)p[2], (unsigned long long *)p[3], s[1], (int)s[2]));
    return check_launch("gather_kernel");
}

extern "C" int32_t nc_rms_norm_quantize(void **p, const int64_t *s, void *stream) {
    return launch_norm((cudaStream_t)stream, (float *)p[0], (const float *)p[1], (const float *)p[2], (int8_t *)p[3],
                       (float *)p[4], (float *)p[5], (int32_t *)p[6], nullptr, (int)s[0], (int)s[1],
                       f32_from_bits(s[2]));
}

extern "C" int32_t nc_quantize_blocks(void **p, const int64_t *s, void *stream) {
    return launch_quant((cudaStream_t)stream, (int8_t *)p[0], (const float *)p[1], (float *)p[2], (float *)p[3],
                        (int32_t *)p[4], (int)s[0], (int)s[1]);
}

extern "C" int32_t nc_matmul_i8_vnni(void **p, const int64_t *s, void *stream) {
    GemvI8Args a{};
    a.out = (float *)p[0];
    a.xq = (const int8_t *)p[1];
    a.xs = (const float *)p[2];
    a.offset = (const float *)p[3];
    a.w = (const uint8_t *)p[4];
    a.scales = (const float *)p[5];
    a.m = (int)s[0];
    a.n = (int)s[1];
    a.k = (int)s[2];
    const int epi = (int)s[3];
    if (epi == EPI_BIAS) a.bias = (const float *)p[6];
    if (epi == EPI_RESIDUAL) a.residual = (const float *)p[6];
    if (epi == EPI_SWIGLU) {
        a.w2 = (const uint8_t *)p[6];
        a.scales2 = (const float *)p[7];
    }
    return launch_i8((cudaStream_t)stream, a, epi);
}

extern "C" int32_t nc_matmul_i8_tc(void **p, const int64_t *s, void *stream) {
    FusedI8Args f{};
    GemvI8Args &a = f.g;
    a.out = (float *)p[0];
    a.xq = (const int8_t *)p[1];
    a.xs = (const float *)p[2];
    a.offset = (const float *)p[3];
    a.w = (const uint8_t *)p[4];
    a.scales = (const float *)p[5];
    a.m = (int)s[0];
    a.n = (int)s[1];
    a.k = (int)s[2];
    const int epi = (int)s[3], pro = (int)s[4], tokens = (int)s[5];
    if (epi == EPI_BIAS) a.bias = (const float *)p[6];
    if (epi == EPI_RESIDUAL) a.residual = (const float *)p[6];
    if (epi == EPI_SWIGLU || epi == EPI_SWIGLU_QUANT) {
        a.w2 = (const uint8_t *)p[6];
        a.scales2 = (const float *)p[7];
    }
    if (pro == PRO_OFFSET) f.bsums_in = (const int32_t *)p[8];
    if (epi == EPI_SWIGLU_QUANT) {
        f.q_out = (int8_t *)p[9];
        f.xs_out = (float *)p[10];
        f.bsums_out = (int32_t *)p[11];
    }
    if (a.m <= 0 || a.n <= 0) return NC_OK;
    const bool two = epi == EPI_SWIGLU || epi == EPI_SWIGLU_QUANT;
    CUtensorMap m1, m2;
    NC_TRY(make_i8_map(&m1, a.w, a.n, a.k, two ? 64 : I8TC_ROWS));
    m2 = m1;
    if (two) NC_TRY(make_i8_map(&m2, a.w2, a.n, a.k, 64));
    return launch_i8_tc((cudaStream_t)stream, f, pro, epi, m1, m2, tokens);
}

extern "C" int32_t nc_matmul_i8_f32(void **p, const int64_t *s, void *stream) {
    GemvI8fArgs a{};
    a.out = (float *)p[0];
    a.x = (const float *)p[1];
    a.w = (const uint8_t *)p[2];
    a.scales = (const float *)p[3];
    a.m = (int)s[0];
    a.n = (int)s[1];
    a.k = (int)s[2];
    const int epi = (int)s[3];
    if (epi == EPI_BIAS) a.bias = (const float *)p[4];
    if (epi == EPI_RESIDUAL) a.residual = (const float *)p[4];
    if (epi == EPI_SWIGLU) {
        a.w2 = (const uint8_t *)p[4];
        a.scales2 = (const float *)p[5];
    }
    return launch_i8f((cudaStream_t)stream, a, epi);
}

extern "C" int32_t nc_matmul_f32(void **p, const int64_t *s, void *stream) {
    GemvF32Args a{};
    a.out = (float *)p[0];
    a.x = (const float *)p[1];
    a.w = (const float *)p[2];
    a.m = (int)s[0];
    a.n = (int)s[1];
    a.k = (int)s[2];
    const int epi = (int)s[3];
    if (epi == EPI_BIAS) a.bias = (const float *)p[3];
    if (epi == EPI_RESIDUAL) a.residual = (const float *)p[3];
    if (epi == EPI_SWIGLU) a.w2 = (const float *)p[3];
    return launch_f32((cudaStream_t)stream, a, epi, false);
}

namespace {

// The int8-prefiltered LM head + argmax of up to LMQ_MAXM rows: prefilter, then pick.
int32_t launch_lm_head_q8(cudaStream_t st, const LmHeadQ8Args &a) {
    const int ctas = (a.n + LMQ_ROWS - 1) / LMQ_ROWS;   // 128-row blocks
    const int T = a.m <= 1 ? 1 : a.m <= 2 ? 2 : a.m <= 4 ? 4 : 8;
    const dim3 grid(std::min(ctas, LMQ_PREFILTER_CTAS), (a.m + T - 1) / T);
    if (T == 1) CUDA_TRY(launch_k(lm_head_q8_kernel<1>, grid, LMQ_THREADS, 0, st, a));
    else if (T == 2) CUDA_TRY(launch_k(lm_head_q8_kernel<2>, grid, LMQ_THREADS, 0, st, a));
    else if (T == 4) CUDA_TRY(launch_k(lm_head_q8_kernel<4>, grid, LMQ_THREADS, 0, st, a));
    else CUDA_TRY(launch_k(lm_head_q8_kernel<8>, grid, LMQ_THREADS, 0, st, a));
    NC_TRY(check_launch("lm_head_q8_kernel"));
    const size_t psmem = lmq_pick_smem(a.k);
    CUDA_TRY(allow_smem(lm_head_q8_pick_kernel, psmem));
    CUDA_TRY(launch_k(lm_head_q8_pick_kernel, LMQ_PICK_CTAS, LMQ_PICK_THREADS, psmem, st, a, ctas));
    return check_launch("lm_head_q8_pick_kernel");
}

}  // namespace

extern "C" int64_t nc_lm_head_scratch_bytes(int64_t rows, int64_t vocab) {
    const int64_t ctas = (vocab + F32_ROWS - 1) / F32_ROWS;
    return 256 + rows * ctas * (int64_t)(sizeof(float) + sizeof(int32_t));
}

extern "C" int32_t nc_lm_head_argmax(void **p, const int64_t *s, void *stream) {
    GemvF32Args a{};
    a.out = (float *)p[0];
    a.x = (const float *)p[1];
    a.w = (const float *)p[2];
    a.tokens = (int64_t *)p[3];
    a.m = (int)s[0];
    a.n = (int)s[1];
    a.k = (int)s[2];
    const int64_t ctas = (a.n + F32_ROWS - 1) / F32_ROWS;
    char *scratch = (char *)p[4];
    a.counter = (unsigned int *)scratch;
    a.part_val = (float *)(scratch + 256);
    a.part_idx = (int32_t *)(scratch + 256 + a.m * ctas * sizeof(float));
    if (!a.tokens) return launch_f32((cudaStream_t)stream, a, EPI_NONE, false);
    return launch_f32((cudaStream_t)stream, a, EPI_NONE, true);
}

extern "C" int32_t nc_lm_head_q8_prepare(void **p, const int64_t *s, void *stream) {
    const int64_t vocab = s[0], hidden = s[1];
    if (vocab <= 0 || hidden <= 0 || vocab > INT32_MAX || hidden > INT32_MAX) return fail(NC_ERR_ARGUMENT, "bad shape");
    lm_q8_kernel<<<(unsigned)((vocab + 7) / 8), 256, 0, (cudaStream_t)stream>>>((int8_t *)p[1], (float *)p[2],
                                                                              (const float *)p[0], (int)vocab, (int)hidden);
    return check_launch("lm_q8_kernel");
}

extern "C" int64_t nc_lm_head_q8_scratch_bytes(int64_t rows, int64_t vocab) {
    const int64_t ctas = (vocab + LMQ_ROWS - 1) / LMQ_ROWS;
    return 256 + 4 * (rows * vocab + rows * ctas + rows + 2 * rows * LMQ_PICK_CTAS);
}

extern "C" int32_t nc_lm_head_q8_argmax(void **p, const int64_t *s, void *stream) {
    LmHeadQ8Args a{};
    a.m = (int)s[0]; a.n = (int)s[1]; a.k = (int)s[2];
    if (a.m <= 0 || a.m > LMQ_MAXM || a.k % 128 || a.k > LMQ_MAXK || a.n <= 0)
        return fail(NC_ERR_ARGUMENT, "the int8 LM head takes 1..%d rows and a width that is a multiple of 128 up to %d",
                    LMQ_MAXM, LMQ_MAXK);
    a.x = (const float *)p[0]; a.w = (const float *)p[1]; a.q = (const int8_t *)p[2]; a.s = (const float *)p[3];
    a.tokens = (int64_t *)p[4];
    char *scratch = (char *)p[5];
    const int64_t ctas = (a.n + LMQ_ROWS - 1) / LMQ_ROWS;
    a.counter = (unsigned int *)scratch;
    a.approx = (float *)(scratch + 256);
    a.cta_low = a.approx + (int64_t)a.m * a.n;
    a.bound = a.cta_low + a.m * ctas;
    a.pick_val = a.bound + a.m;
    a.pick_idx = (int32_t *)(a.pick_val + a.m * LMQ_PICK_CTAS);
    return launch_lm_head_q8((cudaStream_t)stream, a);
}

extern "C" int32_t nc_attention(void **p, const int64_t *s, void *stream) {
    AttnArgs a{};
    a.ctx = (float *)p[0];
    a.qkv = (const float *)p[1];
    a.cache = (float *)p[2];
    a.cos_tab = (const float *)p[3];
    a.sin_tab = (const float *)p[4];
    a.slot = (const int32_t *)p[5];
    a.pos = (const int32_t *)p[6];
    const int rows = (int)s[0];
    a.heads = (int)s[1];
    a.kv = (int)s[2];
    a.d = (int)s[3];
    a.cap = (int)s[4];
    a.slot_stride = s[5];
    a.mode = s[6] ? 0 : 2;
    a.scale = f32_from_bits(s[7]);
    return launch_attention((cudaStream_t)stream, a, rows);
}

extern "C" int32_t nc_attention_cache(void **p, const int64_t *s, void *stream) {
    AttnArgs a{};
    a.ctx = (float *)p[0];
    a.qkv = (const float *)p[1];
    a.cache = (float *)p[2];
    a.cos_tab = (const float *)p[3];
    a.sin_tab = (const float *)p[4];
    a.slot = (const int32_t *)p[5];
    a.pos = (const int32_t *)p[6];
    const int rows = (int)s[0];
    a.heads = (int)s[1];
    a.kv = (int)s[2];
    a.d = (int)s[3];
    a.cap = (int)s[4];
    a.slot_stride = s[5];
    a.mode = s[6] ? 0 : 2;
    a.scale = f32_from_bits(s[7]);
    const int64_t slots = s[8];
    if (slots <= 0 || a.d <= 0 || a.slot_stride % a.d) return fail(NC_ERR_ARGUMENT, "bad cache extent");
    CUtensorMap map;
    if (a.d % ATB_BOX == 0 && slots * (a.slot_stride / a.d) < (int64_t(1) << 31)) {
        NC_TRY(make_kv_map(&map, a.cache, slots * (a.slot_stride / a.d), a.d));
        a.cache_row0 = 0;
        return launch_attention((cudaStream_t)stream, a, rows, &map);
    }
    return launch_attention((cudaStream_t)stream, a, rows);
}

extern "C" int32_t nc_device_faults(void) { return check_device_faults(); }

extern "C" int32_t nc_set_wait_limit(int64_t cycles) {
    const long long v = cycles > 0 ? (long long)cycles : (1ll << 31);
    CUDA_TRY(cudaMemcpyToSymbol(g_wait_cycles, &v, sizeof(v)));
    return NC_OK;
}

extern "C" int32_t nc_selftest_wait(int32_t kind) {
    if (kind != 0 && kind != 1) return fail(NC_ERR_ARGUMENT, "wait kind %d: 0 hand-over word, 1 pipeline stage", kind);
    unsigned long long *words = nullptr;
    CUDA_TRY(cudaMalloc(&words, 64 * sizeof(unsigned long long)));
    cudaError_t e = cudaMemset(words, 0, 64 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        wait_selftest_kernel<<<1, MK_THREADS>>>(words, 64, kind);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(words);
    if (e != cudaSuccess) return fail(NC_ERR_CUDA, "wait self-test: %s", cudaGetErrorString(e));
    return check_device_faults();
}

extern "C" int32_t nc_pack_int8_weights(void *dst_device, const int8_t *src_host, int64_t bytes) {
    CUDA_TRY(cudaMemcpy(dst_device, src_host, (size_t)bytes, cudaMemcpyHostToDevice));
    xor80_kernel<<<1024, 256>>>((uint8_t *)dst_device, bytes);
    NC_TRY(check_launch("xor80_kernel"));
    CUDA_TRY(cudaDeviceSynchronize());
    return NC_OK;
}

extern "C" int32_t nc_quantize_int8_rows(void **p, const int64_t *s, void *stream) {
    const int64_t rows = s[0], cols = s[1], packed = s[2];
    if (rows < 0 || cols <= 0 || rows > INT32_MAX) return fail(NC_ERR_ARGUMENT, "bad sizes %lld x %lld", (long long)rows,
                                                              (long long)cols);
    if (rows == 0) return NC_OK;
    quantize_int8_rows_kernel<<<(unsigned)rows, QI8_THREADS, 0, (cudaStream_t)stream>>>(
        p[0], (float *)p[1], (const float *)p[2], cols, packed ? 1 : 0);
    return check_launch("quantize_int8_rows_kernel");
}

extern "C" int32_t nc_selfcheck_div127(int64_t *mismatches) {
    unsigned long long *d = nullptr;
    CUDA_TRY(cudaMalloc(&d, sizeof *d));
    CUDA_TRY(cudaMemset(d, 0, sizeof *d));
    selfcheck_div127_kernel<<<1184, 256>>>(d);
    NC_TRY(check_launch("selfcheck_div127_kernel"));
    unsigned long long h = 0;
    CUDA_TRY(cudaMemcpy(&h, d, sizeof h, cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaFree(d));
    *mismatches = (int64_t)h;
    return NC_OK;
}

extern "C" int32_t nc_expf_exact(void **p, const int64_t *s, void *stream) {
    if (s[0] <= 0) return NC_OK;
    expf_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>((float *)p[0], (const float *)p[1], s[0]);
    return check_launch("expf_kernel");
}

// ---- 2. the model runtime ----------------------------------------------------------------------

struct WeightSlot {
    char *dst;
    int64_t bytes;
    bool int8;      // stored as int8 + 128
};

struct nc_model {
    nc_qwen2_config c{};
    int dev = 0;
    cudaStream_t stream = nullptr;
    char *arena = nullptr;
    int64_t arena_bytes = 0;
    std::map<std::string, WeightSlot> weights;
    std::set<std::string> uploaded;

    // weights
    float *embed = nullptr, *final_norm = nullptr, *cos_tab = nullptr, *sin_tab = nullptr;
    struct Layer {
        float *in_norm, *post_norm, *bqkv;
        uint8_t *wqkv, *wo, *wg, *wu, *wd;    // int8 mode
        float *sqkv, *so, *sg, *su, *sd;
        float *fqkv, *fo, *fg, *fu, *fd;      // float32 mode
        CUtensorMap mqkv, mo, mg, mu, md;     // int8 mode: the weights as tensor-core operand tiles
    };
    bool tc_i8 = false;                       // the tensor maps above are valid
    std::vector<Layer> layers;
    float *kv = nullptr;            // [slot][layer][2][kv][cap][d]
    int64_t slot_stride = 0, layer_stride = 0;
    CUtensorMap kv_map;             // the whole KV arena as rows of d floats (has_kv_map)
    bool has_kv_map = false;
    // the tensor-core LM head (batched decode steps that need only the tokens)
    float *lm_tiles = nullptr;      // the embedding as pre-swizzled 128 x 32 tiles (lm_tiles_kernel)
    float *lm_xhi = nullptr, *lm_xlo = nullptr;   // the normed rows as pre-swizzled 64 x 32 tiles
    bool tc_head = false;
    float wmax = 0.0f;              // max |w| of the embedding (set when it is uploaded)
    float wnorm = 0.0f;             // max over its rows of the row's 2-norm, rounded up (likewise)
    float *cand_val = nullptr, *cta_best = nullptr, *lm_delta = nullptr;
    int32_t *cand_idx = nullptr, *cand_cnt = nullptr;
    // the int8-prefiltered LM head (decode steps of up to LMQ_MAXM rows that need only the tokens)
    int8_t *lmq_q = nullptr;        // the embedding's rows quantized to int8 (lm_q8_kernel)
    float *lmq_s = nullptr, *lmq_approx = nullptr, *lmq_low = nullptr, *lmq_bound = nullptr, *lmq_pval = nullptr;
    int32_t *lmq_pidx = nullptr;
    unsigned int *lmq_counter = nullptr;
    bool q8_head = false;
    // the persistent decode kernel (steps of up to MK_ROWS rows)
    MkLayer *mk_layers = nullptr;   // per-layer weight pointers, on the device
    unsigned int *mk_sync = nullptr;   // CTAs finished, launch number
    unsigned long long *mk_xt = nullptr, *mk_qkvt = nullptr, *mk_aqt = nullptr, *mk_hqt = nullptr;   // tagged words
    int64_t mk_tagged_bytes = 0;    // the four tagged buffers, contiguous from mk_xt
    int mk_ctas = 0;                // one CTA per SM; 0: the kernel cannot serve this model
    unsigned long long *mk_stamps = nullptr;   // phase stamps of the next launches, or null
    bool logit_identity = false;    // the step's logit rows are its rows 0..rows-1 (set per step)

    // activations and step state
    float *x = nullptr, *normed = nullptr, *xs = nullptr, *off = nullptr, *qkv = nullptr, *ctx = nullptr,
          *hbuf = nullptr, *logits = nullptr, *part_val = nullptr;
    int8_t *xq = nullptr, *hq = nullptr;      // quantized activations: hidden-wide, and of the SwiGLU output
    float *hxs = nullptr;
    int32_t *bsums = nullptr;
    int32_t *part_idx = nullptr, *slot = nullptr, *pos = nullptr, *logit_row = nullptr, *step = nullptr;
    int64_t *ids = nullptr, *tokens = nullptr, *history = nullptr;
    unsigned long long *err = nullptr;
    unsigned int *counter = nullptr;
    int history_steps = 0;
    int64_t *pinned = nullptr;      // host staging [2][max_rows] for the per-step decode mode

    std::map<int, cudaGraphExec_t> decode_graphs;   // by 2 * batch size + tokens_only

    // kernel-time probe: CUDA events around every launch of an eager step, by fused-group kind
    bool probing = false;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> probe_marks;
    std::vector<cudaEvent_t> event_pool;
    size_t event_next = 0;
};

enum ProbeKind : int {
    K_GATHER = 0, K_QKV = 1, K_ATTENTION = 2, K_O = 3, K_GATE_UP = 4, K_DOWN = 5, K_NORM = 6, K_QUANT = 7,
    K_LM_HEAD = 8, K_LAYERS = 9, K_KINDS = 10
};

namespace {

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

cudaEvent_t probe_event(nc_model *m) {
    if (m->event_next == m->event_pool.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        m->event_pool.push_back(e);
    }
    return m->event_pool[m->event_next++];
}

// Brackets one launch with events when the model is probing (eager steps only).
struct Probe {
    nc_model *m;
    int kind;
    cudaEvent_t end = nullptr;
    Probe(nc_model *model, int k) : m(model), kind(k) {
        if (!m->probing) return;
        cudaEvent_t begin = probe_event(m);
        end = probe_event(m);
        cudaEventRecord(begin, m->stream);
        m->probe_marks.push_back({kind, {begin, end}});
    }
    ~Probe() {
        if (end) cudaEventRecord(end, m->stream);
    }
};

// Arena layout: a bump allocator over one cudaMalloc, 256-byte aligned pieces.
struct Layout {
    int64_t top = 0;
    std::vector<std::pair<void **, int64_t>> pieces;
    template <typename T>
    void add(T **ptr, int64_t bytes) {
        pieces.push_back({(void **)ptr, top});
        top = align_up(top + std::max<int64_t>(bytes, 1), 256);
    }
};

// One step: the fused groups of every layer, then the final norm and the LM head.  For int8
// with few rows (decode, short prompts) five kernels per layer:
//   q/k/v projection (rms_norm + quantize prologue, bias epilogue)
//   RoPE + cache append + attention (quantizing epilogue)
//   o projection (offset prologue, residual epilogue)
//   gate/up projection (rms_norm + quantize prologue, silu*up + quantize epilogue)
//   down projection (offset prologue, residual epilogue)
// With more rows the norms run as their own row kernels (one CTA per row, in parallel).
// The persistent decode kernel's instance for a model's widths: exact register slices for the
// 896 / 4864 widths of Qwen2.5-0.5B, the largest ones otherwise.
using MkKernel = void (*)(MkArgs, CUtensorMap);
MkKernel mk_kernel(int H, int I) {
    if (H / CHUNK == 7 && I / CHUNK == 38) return decode_mk_kernel<7, 38>;
    return decode_mk_kernel<MK_NCH, MK_NCH_DOWN>;
}

// The persistent decode kernel serves an int8 model whose widths fit its register slices, with
// one CTA per SM, when every CTA can be resident; returns the CTA count (0: not served).
int mk_capacity(const nc_qwen2_config &c, int dev) {
    if (!mk_enabled()) return 0;
    const int H = (int)c.hidden, I = (int)c.inter, d = (int)c.head_dim, Hq = (int)(c.heads * c.head_dim);
    const int Nqkv = (int)((c.heads + 2 * c.kv_heads) * c.head_dim);
    if (H % CHUNK || Hq % CHUNK || I % CHUNK || H > MK_NCH * CHUNK || Hq > MK_NCH * CHUNK || I > MK_NCH_DOWN * CHUNK)
        return 0;
    if (d != 64 || c.layers > MK_MAX_LAYERS) return 0;            // attention items of head dim 64
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 0;
    const int G = sms;
    if ((Nqkv + G - 1) / G > MK_WARPS || (H + G - 1) / G > MK_WARPS - 1 || (I / QBLOCK + G - 1) / G > 2 ||
        QBLOCK != MK_WARPS * (32 / MK_GU_LPR))
        return 0;
    if (MK_ROWS * c.heads * (d / ATS_SLICE) > G) return 0;
    const MkSmem L = mk_smem((int)c.layers, MK_ROWS, H, std::max(H, std::max(Hq, I)), d, (int)c.capacity);
    if (L.bytes > 224 * 1024) return 0;                          // with the static shared memory: <= 227 KB
    const auto kernel = mk_kernel(H, I);
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.bytes) != cudaSuccess) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, MK_THREADS, L.bytes) != cudaSuccess || per_sm < 1)
        return 0;
    return G;
}

// Gather, every layer and the final norm of a decode step of up to MK_ROWS rows as one
// cooperative launch (m->x, m->normed; the LM head follows).
int32_t launch_decode_mk(nc_model *m, int rows) {
    const nc_qwen2_config &c = m->c;
    MkArgs a{};
    a.layers = m->mk_layers; a.nl = (int)c.layers; a.m = rows; a.H = (int)c.hidden; a.I = (int)c.inter;
    a.heads = (int)c.heads; a.kv = (int)c.kv_heads; a.d = (int)c.head_dim; a.cap = (int)c.capacity;
    a.eps = c.eps; a.scale = c.attn_scale; a.slot_stride = m->slot_stride; a.vocab = c.vocab;
    a.slot_rows = m->slot_stride / c.head_dim;
    a.embed = m->embed; a.ids = m->ids; a.err = m->err; a.slot = m->slot; a.pos = m->pos;
    a.cos_tab = m->cos_tab; a.sin_tab = m->sin_tab; a.final_norm = m->final_norm;
    a.normed = m->normed;
    const int H = a.H, Hq = a.heads * a.d, Nqkv = (a.heads + 2 * a.kv) * a.d;
    a.xt = m->mk_xt;
    a.qkvt = a.xt + (int64_t)MK_ROWS * H;
    a.aqt = a.qkvt + (int64_t)MK_ROWS * Nqkv;
    a.hqt = a.aqt + (int64_t)MK_ROWS * (Hq / QBLOCK) * MK_BLOCK_WORDS;
    a.sync = m->mk_sync;
    a.stamps = m->mk_stamps;
    const MkSmem L = mk_smem(a.nl, rows, H, std::max(H, std::max(Hq, a.I)), a.d, a.cap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->mk_ctas);
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = L.bytes;
    cfg.stream = m->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, mk_kernel(a.H, a.I), a, m->kv_map));
    return check_launch("decode_mk_kernel");
}

// The int8-prefiltered LM head + argmax of the model's normed rows (m->normed -> m->tokens).
int32_t launch_lm_head_q8(nc_model *m, int rows) {
    LmHeadQ8Args a{};
    a.m = rows; a.n = (int)m->c.vocab; a.k = (int)m->c.hidden;
    a.q = m->lmq_q; a.s = m->lmq_s; a.x = m->normed; a.w = m->embed; a.approx = m->lmq_approx;
    a.cta_low = m->lmq_low; a.bound = m->lmq_bound; a.pick_val = m->lmq_pval; a.pick_idx = m->lmq_pidx;
    a.counter = m->lmq_counter; a.tokens = m->tokens;
    return launch_lm_head_q8(m->stream, a);
}

// An int8 projection of the step: more than four rows take the tensor cores when the model has
// its weights' tensor maps and NC_TC_I8=1; otherwise the batched dp4a kernel.
int32_t model_i8(nc_model *m, const FusedI8Args &f, int pro, int epi, const CUtensorMap &m1, const CUtensorMap &m2) {
    if (m->tc_i8 && tc_i8_enabled() && f.g.m > PRO_NORM_ROWS && pro != PRO_NORM)
        return launch_i8_tc(m->stream, f, pro, epi, m1, m2);
    return launch_i8_fused(m->stream, f, pro, epi);
}

// Gather, the layers as separate fused-group kernels, and the final norm of the logit rows.
int32_t enqueue_layers(nc_model *m, int rows, int logit_rows, bool fused) {
    const nc_qwen2_config &c = m->c;
    cudaStream_t st = m->stream;
    const int H = (int)c.hidden, I = (int)c.inter, d = (int)c.head_dim;
    const int Hq = (int)(c.heads * d), Nqkv = (int)((c.heads + 2 * c.kv_heads) * d);
    const bool q8 = c.quant == 1;             // int8-vnni: block-32 int8 activations
    const bool i8f = c.quant == 2;            // int8 weights, float32 activations
    const bool norm_fused = rows <= PRO_NORM_ROWS && H <= 8 * CHUNK;
    const bool attn_quant = q8 && d % QBLOCK == 0;

    {
        Probe pr(m, K_GATHER);
        CUDA_TRY(launch_k(gather_kernel, rows, 256, 0, st, m->x, m->ids, m->embed, m->err, c.vocab, H));
        NC_TRY(check_launch("gather_kernel"));
    }

    for (int l = 0; l < (int)c.layers; ++l) {
        const nc_model::Layer &L = m->layers[l];
        // input norm -> q/k/v projections with their biases
        if (q8) {
            FusedI8Args f{};
            f.g.out = m->qkv; f.g.xq = m->xq; f.g.xs = m->xs; f.g.offset = m->off; f.g.w = L.wqkv;
            f.g.scales = L.sqkv; f.g.bias = L.bqkv; f.g.m = rows; f.g.n = Nqkv; f.g.k = H;
            if (norm_fused) {
                f.x = m->x; f.norm_w = L.in_norm; f.eps = c.eps;
                Probe pr(m, K_QKV);
                NC_TRY(launch_i8_fused(st, f, PRO_NORM, EPI_BIAS));
            } else {
                {
                    Probe pr(m, K_NORM);
                    NC_TRY(launch_norm(st, nullptr, m->x, L.in_norm, m->xq, m->xs, m->off, nullptr, nullptr, rows, H, c.eps));
                }
                Probe pr(m, K_QKV);
                NC_TRY(model_i8(m, f, PRO_NONE, EPI_BIAS, L.mqkv, L.mqkv));
            }
        } else {
            {
                Probe pr(m, K_NORM);
                NC_TRY(launch_norm(st, m->normed, m->x, L.in_norm, nullptr, nullptr, nullptr, nullptr, nullptr, rows, H, c.eps));
            }
            Probe pr(m, K_QKV);
            if (i8f) {
                GemvI8fArgs a{};
                a.out = m->qkv; a.x = m->normed; a.w = L.wqkv; a.scales = L.sqkv; a.bias = L.bqkv;
                a.m = rows; a.n = Nqkv; a.k = H;
                NC_TRY(launch_i8f(st, a, EPI_BIAS));
            } else {
                GemvF32Args a{};
                a.out = m->qkv; a.x = m->normed; a.w = L.fqkv; a.bias = L.bqkv; a.m = rows; a.n = Nqkv; a.k = H;
                NC_TRY(launch_f32(st, a, EPI_BIAS, false));
            }
        }
        // RoPE, cache append, attention (and the quantization of its output)
        AttnArgs at{};
        at.ctx = attn_quant ? nullptr : m->ctx; at.qkv = m->qkv; at.cache = m->kv + (int64_t)l * m->layer_stride;
        at.cos_tab = m->cos_tab; at.sin_tab = m->sin_tab; at.slot = m->slot; at.pos = m->pos;
        at.slot_stride = m->slot_stride; at.heads = (int)c.heads; at.kv = (int)c.kv_heads; at.d = d;
        at.cache_row0 = (int64_t)l * m->layer_stride / d;
        at.cap = c.capacity; at.scale = c.attn_scale;
        if (attn_quant) { at.q_out = m->xq; at.xs_out = m->xs; at.bsums_out = m->bsums; }
        if (fused) {
            at.mode = 0;
            Probe pr(m, K_ATTENTION);
            NC_TRY(launch_attention(st, at, rows, m->has_kv_map ? &m->kv_map : nullptr));
        } else {
            Probe pr(m, K_ATTENTION);
            at.mode = 1;
            NC_TRY(launch_attention(st, at, rows, m->has_kv_map ? &m->kv_map : nullptr));
            at.mode = 2;
            NC_TRY(launch_attention(st, at, rows, m->has_kv_map ? &m->kv_map : nullptr));
        }
        // o_proj with the residual add
        if (q8) {
            FusedI8Args f{};
            f.g.out = m->x; f.g.xq = m->xq; f.g.xs = m->xs; f.g.offset = m->off; f.g.w = L.wo; f.g.scales = L.so;
            f.g.residual = m->x; f.g.m = rows; f.g.n = H; f.g.k = Hq;
            if (attn_quant) {
                f.bsums_in = m->bsums;
                Probe pr(m, K_O);
                NC_TRY(model_i8(m, f, PRO_OFFSET, EPI_RESIDUAL, L.mo, L.mo));
            } else {
                {
                    Probe pr(m, K_QUANT);
                    NC_TRY(launch_quant(st, m->xq, m->ctx, m->xs, m->off, nullptr, rows, Hq));
                }
                Probe pr(m, K_O);
                NC_TRY(model_i8(m, f, PRO_NONE, EPI_RESIDUAL, L.mo, L.mo));
            }
        } else {
            Probe pr(m, K_O);
            if (i8f) {
                GemvI8fArgs a{};
                a.out = m->x; a.x = m->ctx; a.w = L.wo; a.scales = L.so; a.residual = m->x; a.m = rows; a.n = H; a.k = Hq;
                NC_TRY(launch_i8f(st, a, EPI_RESIDUAL));
            } else {
                GemvF32Args a{};
                a.out = m->x; a.x = m->ctx; a.w = L.fo; a.residual = m->x; a.m = rows; a.n = H; a.k = Hq;
                NC_TRY(launch_f32(st, a, EPI_RESIDUAL, false));
            }
        }
        // post-attention norm -> gate/up with silu * up (quantized) -> down with the residual add
        if (q8) {
            FusedI8Args f{};
            f.g.xq = m->xq; f.g.xs = m->xs; f.g.offset = m->off; f.g.w = L.wg; f.g.scales = L.sg;
            f.g.w2 = L.wu; f.g.scales2 = L.su; f.g.m = rows; f.g.n = I; f.g.k = H;
            f.q_out = m->hq; f.xs_out = m->hxs; f.bsums_out = m->bsums;
            if (norm_fused) {
                f.x = m->x; f.norm_w = L.post_norm; f.eps = c.eps;
                Probe pr(m, K_GATE_UP);
                NC_TRY(launch_i8_fused(st, f, PRO_NORM, EPI_SWIGLU_QUANT));
            } else {
                {
                    Probe pr(m, K_NORM);
                    NC_TRY(launch_norm(st, nullptr, m->x, L.post_norm, m->xq, m->xs, m->off, nullptr, nullptr, rows, H, c.eps));
                }
                Probe pr(m, K_GATE_UP);
                NC_TRY(model_i8(m, f, PRO_NONE, EPI_SWIGLU_QUANT, L.mg, L.mu));
            }
            FusedI8Args b{};
            b.g.out = m->x; b.g.xq = m->hq; b.g.xs = m->hxs; b.g.w = L.wd; b.g.scales = L.sd;
            b.g.residual = m->x; b.g.m = rows; b.g.n = H; b.g.k = I; b.bsums_in = m->bsums;
            Probe pr(m, K_DOWN);
            NC_TRY(model_i8(m, b, PRO_OFFSET, EPI_RESIDUAL, L.md, L.md));
        } else {
            {
                Probe pr(m, K_NORM);
                NC_TRY(launch_norm(st, m->normed, m->x, L.post_norm, nullptr, nullptr, nullptr, nullptr, nullptr, rows, H, c.eps));
            }
            if (i8f) {
                GemvI8fArgs a{};
                a.out = m->hbuf; a.x = m->normed; a.w = L.wg; a.scales = L.sg; a.w2 = L.wu; a.scales2 = L.su;
                a.m = rows; a.n = I; a.k = H;
                {
                    Probe pr(m, K_GATE_UP);
                    NC_TRY(launch_i8f(st, a, EPI_SWIGLU));
                }
                GemvI8fArgs b{};
                b.out = m->x; b.x = m->hbuf; b.w = L.wd; b.scales = L.sd; b.residual = m->x; b.m = rows; b.n = H; b.k = I;
                Probe pr(m, K_DOWN);
                NC_TRY(launch_i8f(st, b, EPI_RESIDUAL));
            } else {
                GemvF32Args a{};
                a.out = m->hbuf; a.x = m->normed; a.w = L.fg; a.w2 = L.fu; a.m = rows; a.n = I; a.k = H;
                {
                    Probe pr(m, K_GATE_UP);
                    NC_TRY(launch_f32(st, a, EPI_SWIGLU, false));
                }
                GemvF32Args b{};
                b.out = m->x; b.x = m->hbuf; b.w = L.fd; b.residual = m->x; b.m = rows; b.n = H; b.k = I;
                Probe pr(m, K_DOWN);
                NC_TRY(launch_f32(st, b, EPI_RESIDUAL, false));
            }
        }
    }
    // final norm of the rows that need logits, then the tied LM head with the argmax
    {
        Probe pr(m, K_NORM);
        NC_TRY(launch_norm(st, m->normed, m->x, m->final_norm, nullptr, nullptr, nullptr, nullptr, m->logit_row,
                           logit_rows, H, c.eps));
    }
    return NC_OK;
}

int32_t enqueue_step(nc_model *m, int rows, int logit_rows, bool fused, bool tokens_only) {
    const nc_qwen2_config &c = m->c;
    cudaStream_t st = m->stream;
    const int H = (int)c.hidden;
    if (c.quant == 1 && m->mk_ctas && rows <= MK_ROWS && fused && m->logit_identity && logit_rows == rows) {
        Probe pr(m, K_LAYERS);
        NC_TRY(launch_decode_mk(m, rows));
    } else {
        NC_TRY(enqueue_layers(m, rows, logit_rows, fused));
    }
    Probe pr(m, K_LM_HEAD);
    if (tokens_only && m->tc_head && logit_rows > 16 && tc_head_enabled()) {
        // tensor-core logits, then the exact in-order logits of the argmax candidates
        LmHeadTcArgs la{};
        la.m = logit_rows; la.n = (int)c.vocab; la.k = H; la.wmax = m->wmax;
        la.cand_val = m->cand_val; la.cand_idx = m->cand_idx; la.cand_cnt = m->cand_cnt;
        la.cta_best = m->cta_best; la.delta = m->lm_delta; la.tiles = m->lm_tiles;
        la.xhi = m->lm_xhi; la.xlo = m->lm_xlo;
        const int ctas = (int)((c.vocab + LMT_ROWS - 1) / LMT_ROWS);
        CUDA_TRY(launch_k(lm_prep_kernel, logit_rows, 256, 0, st, m->lm_xhi, m->lm_xlo, m->lm_delta,
                          (const float *)m->normed, H, m->wmax, m->wnorm));
        NC_TRY(check_launch("lm_prep_kernel"));
        CUDA_TRY(allow_smem(lm_head_tc_kernel, LMT_SMEM));
        CUDA_TRY(launch_k(lm_head_tc_kernel, dim3(ctas, (logit_rows + LMT_TOK - 1) / LMT_TOK), LMT_THREADS, LMT_SMEM,
                          st, la));
        NC_TRY(check_launch("lm_head_tc_kernel"));
        const size_t psmem = lm_pick_smem(H);
        CUDA_TRY(allow_smem(lm_head_pick_kernel, psmem));
        CUDA_TRY(launch_k(lm_head_pick_kernel, logit_rows, LMP_THREADS, psmem, st, la, (const float *)m->normed,
                          (const float *)m->embed, ctas, m->tokens));
        return check_launch("lm_head_pick_kernel");
    }
    if (tokens_only && m->q8_head && logit_rows <= LMQ_MAXM && q8_head_enabled())
        return launch_lm_head_q8(m, logit_rows);
    GemvF32Args a{};
    a.out = m->logits; a.x = m->normed; a.w = m->embed; a.m = logit_rows; a.n = (int)c.vocab; a.k = H;
    a.part_val = m->part_val; a.part_idx = m->part_idx; a.counter = m->counter; a.tokens = m->tokens;
    NC_TRY(launch_f32(st, a, EPI_NONE, true));
    return NC_OK;
}

}  // namespace

// A step's faults; a persistent step that gave up leaves its barrier counters behind: clear them.
static int32_t model_faults(nc_model *m) {
    const int32_t status = check_device_faults();
    if (status != NC_OK && m->mk_sync) {
        cudaMemset(m->mk_sync, 0, 16);
        cudaMemset(m->mk_xt, 0, (size_t)m->mk_tagged_bytes);
    }
    return status;
}

extern "C" int32_t nc_qwen2_create(const nc_qwen2_config *cfg, const float *inv_freq, nc_model **out) {
    if (!cfg || !out || !inv_freq) return fail(NC_ERR_ARGUMENT, "null argument");
    const nc_qwen2_config c = *cfg;
    if (c.hidden <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads || c.head_dim % 4 ||
        c.head_dim > 256 || c.max_rows <= 0 || c.max_rows > 1024 || c.slots <= 0 || c.capacity <= 0)
        return fail(NC_ERR_ARGUMENT, "unsupported model shape");
    if (c.hidden % 32 || c.inter % 32 || (c.heads * c.head_dim) % 32)
        return fail(NC_ERR_ARGUMENT, "widths must be whole 32-blocks");
    if (c.quant < 0 || c.quant > 2)
        return fail(NC_ERR_ARGUMENT, "projection mode %d: the library implements 0 (float32), 1 (int8-vnni) and 2 "
                                     "(int8 weights, float32 activations)", c.quant);
    if (c.quant == 2 && (c.hidden % 16 || c.inter % 16 || (c.heads * c.head_dim) % 16))
        return fail(NC_ERR_ARGUMENT, "int8 weights with float32 activations take widths that are multiples of 16");
    if (attention_smem((int)(c.heads / c.kv_heads), (int)c.head_dim, c.capacity) > 220 * 1024 &&
        attention_smem(1, (int)c.head_dim, c.capacity) > 220 * 1024)
        return fail(NC_ERR_ARGUMENT, "capacity %d exceeds the attention kernel's shared memory", c.capacity);

    auto m = std::make_unique<nc_model>();
    m->c = c;
    m->dev = c.device;
    CUDA_TRY(cudaSetDevice(c.device));
    CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));

    const int64_t H = c.hidden, I = c.inter, d = c.head_dim, V = c.vocab, R = c.max_rows;
    const int64_t Hq = c.heads * d, Nqkv = (c.heads + 2 * c.kv_heads) * d, half = d / 2;
    const int64_t kmax = std::max(H, std::max(I, Hq));
    Layout lay;
    lay.add(&m->embed, V * H * 4);
    lay.add(&m->final_norm, H * 4);
    lay.add(&m->cos_tab, (int64_t)c.capacity * half * 4);
    lay.add(&m->sin_tab, (int64_t)c.capacity * half * 4);
    m->layers.resize(c.layers);
    for (auto &L : m->layers) {
        std::memset(&L, 0, sizeof L);
        lay.add(&L.in_norm, H * 4);
        lay.add(&L.post_norm, H * 4);
        lay.add(&L.bqkv, Nqkv * 4);
        if (c.quant) {
            lay.add(&L.wqkv, Nqkv * H);
            lay.add(&L.sqkv, Nqkv * 4);
            lay.add(&L.wo, H * Hq);
            lay.add(&L.so, H * 4);
            lay.add(&L.wg, I * H);
            lay.add(&L.sg, I * 4);
            lay.add(&L.wu, I * H);
            lay.add(&L.su, I * 4);
            lay.add(&L.wd, H * I);
            lay.add(&L.sd, H * 4);
        } else {
            lay.add(&L.fqkv, Nqkv * H * 4);
            lay.add(&L.fo, H * Hq * 4);
            lay.add(&L.fg, I * H * 4);
            lay.add(&L.fu, I * H * 4);
            lay.add(&L.fd, H * I * 4);
        }
    }
    m->layer_stride = 2 * c.kv_heads * (int64_t)c.capacity * d;
    m->slot_stride = c.layers * m->layer_stride;
    lay.add(&m->kv, (int64_t)c.slots * m->slot_stride * 4);
    lay.add(&m->x, R * H * 4);
    lay.add(&m->normed, R * H * 4);
    lay.add(&m->xq, R * kmax);
    lay.add(&m->xs, R * (kmax / 32) * 4);
    lay.add(&m->off, R * 4);
    lay.add(&m->hq, R * I);
    lay.add(&m->hxs, R * (I / 32) * 4);
    lay.add(&m->bsums, R * (kmax / 32) * 4);
    lay.add(&m->qkv, R * Nqkv * 4);
    lay.add(&m->ctx, R * Hq * 4);
    lay.add(&m->hbuf, R * I * 4);
    lay.add(&m->logits, R * V * 4);
    const int64_t ctas = (V + F32_ROWS - 1) / F32_ROWS;
    lay.add(&m->part_val, R * ctas * 4);
    lay.add(&m->part_idx, R * ctas * 4);
    const int64_t tc_ctas = (c.vocab + LMT_ROWS - 1) / LMT_ROWS;
    const bool tc_head = H % LMT_KT == 0 && R > 16;
    if (tc_head) {
        lay.add(&m->lm_tiles, tc_ctas * LMT_ROWS * H * 4);
        lay.add(&m->lm_xhi, (R + LMT_TOK - 1) / LMT_TOK * LMT_TOK * H * 4);
        lay.add(&m->lm_xlo, (R + LMT_TOK - 1) / LMT_TOK * LMT_TOK * H * 4);
        lay.add(&m->cand_val, R * tc_ctas * LMT_CAND * 4);
        lay.add(&m->cand_idx, R * tc_ctas * LMT_CAND * 4);
        lay.add(&m->cand_cnt, R * tc_ctas * 4);
        lay.add(&m->cta_best, R * tc_ctas * 4);
        lay.add(&m->lm_delta, R * 4);
    }
    const bool q8_head = H % 128 == 0 && H <= LMQ_MAXK;
    if (q8_head) {
        const int64_t qr = std::min<int64_t>(R, LMQ_MAXM), qctas = (V + LMQ_ROWS - 1) / LMQ_ROWS;
        lay.add(&m->lmq_q, V * H);
        lay.add(&m->lmq_s, V * 4);
        lay.add(&m->lmq_approx, qr * V * 4);
        lay.add(&m->lmq_low, qr * qctas * 4);
        lay.add(&m->lmq_bound, qr * 4);
        lay.add(&m->lmq_pval, qr * LMQ_PICK_CTAS * 4);
        lay.add(&m->lmq_pidx, qr * LMQ_PICK_CTAS * 4);
        lay.add(&m->lmq_counter, 4);
    }
    lay.add(&m->ids, R * 8);
    lay.add(&m->tokens, R * 8);
    lay.add(&m->slot, R * 4);
    lay.add(&m->pos, R * 4);
    lay.add(&m->logit_row, R * 4);
    lay.add(&m->step, 4);
    lay.add(&m->err, 8);
    lay.add(&m->counter, 4);
    lay.add(&m->mk_layers, c.layers * (int64_t)sizeof(MkLayer));
    lay.add(&m->mk_sync, 16);
    {
        const int64_t xt = MK_ROWS * H * 8, qt = MK_ROWS * Nqkv * 8, at = MK_ROWS * (Hq / 32) * MK_BLOCK_WORDS * 8,
                      ht = MK_ROWS * (I / 32) * MK_BLOCK_WORDS * 8;
        lay.add(&m->mk_xt, xt + qt + at + ht);
        m->mk_tagged_bytes = xt + qt + at + ht;
    }
    m->history_steps = 8192;
    lay.add(&m->history, (int64_t)m->history_steps * R * 8);

    m->arena_bytes = lay.top;
    void *base = nullptr;
    CUDA_TRY(cudaMalloc(&base, (size_t)lay.top));
    m->arena = (char *)base;
    for (auto &pc : lay.pieces) *pc.first = m->arena + pc.second;
    CUDA_TRY(cudaMemsetAsync(m->arena, 0, (size_t)lay.top, m->stream));
    // the KV arena as one tensor of rows for the grouped attention kernel's TMA loads
    const int64_t kv_rows = c.slots * m->slot_stride / d;
    if (d % ATB_BOX == 0 && kv_rows < (int64_t(1) << 31))
        m->has_kv_map = make_kv_map(&m->kv_map, m->kv, kv_rows, (int)d) == NC_OK;
    m->tc_head = tc_head;
    m->q8_head = q8_head;
    // int8 weights as tcgen05 operand tiles for the batched projections (more than four rows)
    if (c.quant == 1) {
        bool ok = true;
        for (auto &L : m->layers) {
            ok = ok && make_i8_map(&L.mqkv, L.wqkv, Nqkv, H, I8TC_ROWS) == NC_OK;
            ok = ok && make_i8_map(&L.mo, L.wo, H, Hq, I8TC_ROWS) == NC_OK;
            ok = ok && make_i8_map(&L.mg, L.wg, I, H, 64) == NC_OK;
            ok = ok && make_i8_map(&L.mu, L.wu, I, H, 64) == NC_OK;
            ok = ok && make_i8_map(&L.md, L.wd, H, I, I8TC_ROWS) == NC_OK;
        }
        m->tc_i8 = ok;
    }

    // RoPE tables: angle = float(position) * inv_freq[i] (nanocompile/nn.py:78-94), evaluated with
    // the C library's cosf/sinf -- the functions the reference's generated C calls for them.
    std::vector<float> ct((size_t)c.capacity * half), stt((size_t)c.capacity * half);
    for (int64_t p = 0; p < c.capacity; ++p)
        for (int64_t i = 0; i < half; ++i) {
            volatile float angle = (float)p * inv_freq[i];
            ct[p * half + i] = cosf(angle);
            stt[p * half + i] = sinf(angle);
        }
    CUDA_TRY(cudaMemcpyAsync(m->cos_tab, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaMemcpyAsync(m->sin_tab, stt.data(), stt.size() * 4, cudaMemcpyHostToDevice, m->stream));
    CUDA_TRY(cudaStreamSynchronize(m->stream));

    // the upload registry: checkpoint name -> destination
    auto reg = [&](const std::string &name, void *dst, int64_t bytes, bool int8) {
        m->weights[name] = WeightSlot{(char *)dst, bytes, int8};
    };
    reg("model.embed_tokens.weight", m->embed, V * H * 4, false);
    reg("model.norm.weight", m->final_norm, H * 4, false);
    for (int64_t l = 0; l < c.layers; ++l) {
        auto &L = m->layers[l];
        const std::string p = "model.layers." + std::to_string(l);
        reg(p + ".input_layernorm.weight", L.in_norm, H * 4, false);
        reg(p + ".post_attention_layernorm.weight", L.post_norm, H * 4, false);
        const int64_t rows[3] = {Hq, c.kv_heads * d, c.kv_heads * d};
        const char *names[3] = {"q_proj", "k_proj", "v_proj"};
        int64_t r0 = 0;
        for (int i = 0; i < 3; ++i) {
            const std::string base_name = p + ".self_attn." + names[i];
            reg(base_name + ".bias", L.bqkv + r0, rows[i] * 4, false);
            if (c.quant) {
                reg(base_name + ".weight@int8", L.wqkv + r0 * H, rows[i] * H, true);
                reg(base_name + ".weight@scales", L.sqkv + r0, rows[i] * 4, false);
            } else {
                reg(base_name + ".weight", L.fqkv + r0 * H, rows[i] * H * 4, false);
            }
            r0 += rows[i];
        }
        struct P { const char *name; uint8_t *w8; float *s; float *f; int64_t n, k; };
        const P projs[4] = {{"self_attn.o_proj", L.wo, L.so, L.fo, H, Hq},
                            {"mlp.gate_proj", L.wg, L.sg, L.fg, I, H},
                            {"mlp.up_proj", L.wu, L.su, L.fu, I, H},
                            {"mlp.down_proj", L.wd, L.sd, L.fd, H, I}};
        for (const P &pr : projs) {
            const std::string base_name = p + "." + pr.name + ".weight";
            if (c.quant) {
                reg(base_name + "@int8", pr.w8, pr.n * pr.k, true);
                reg(base_name + "@scales", pr.s, pr.n * 4, false);
            } else {
                reg(base_name, pr.f, pr.n * pr.k * 4, false);
            }
        }
    }
    if (c.quant == 1) {
        std::vector<MkLayer> ml((size_t)c.layers);
        for (int64_t l = 0; l < c.layers; ++l) {
            const auto &L = m->layers[l];
            ml[l] = MkLayer{L.wqkv, L.wo, L.wg, L.wu, L.wd, L.sqkv, L.so, L.sg, L.su, L.sd, L.bqkv, L.in_norm, L.post_norm,
                            m->kv + l * m->layer_stride, l * m->layer_stride / d};
        }
        CUDA_TRY(cudaMemcpy(m->mk_layers, ml.data(), ml.size() * sizeof(MkLayer), cudaMemcpyHostToDevice));
        m->mk_ctas = m->has_kv_map ? mk_capacity(c, m->dev) : 0;
    }
    *out = m.release();
    return NC_OK;
}

extern "C" int32_t nc_qwen2_destroy(nc_model *m) {
    if (!m) return NC_OK;
    cudaSetDevice(m->dev);
    for (auto &g : m->decode_graphs) cudaGraphExecDestroy(g.second);
    for (auto e : m->event_pool) cudaEventDestroy(e);
    if (m->pinned) cudaFreeHost(m->pinned);
    if (m->arena) cudaFree(m->arena);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return NC_OK;
}

extern "C" int64_t nc_qwen2_arena_bytes(const nc_model *m) { return m ? m->arena_bytes : 0; }

extern "C" int32_t nc_qwen2_upload(nc_model *m, const char *name, const void *host, int64_t bytes) {
    if (!m || !name || !host) return fail(NC_ERR_ARGUMENT, "null argument");
    auto it = m->weights.find(name);
    if (it == m->weights.end()) return fail(NC_ERR_ARGUMENT, "no weight named %s", name);
    if (it->second.bytes != bytes)
        return fail(NC_ERR_ARGUMENT, "weight %s has %lld bytes, expected %lld", name, (long long)bytes,
                    (long long)it->second.bytes);
    CUDA_TRY(cudaSetDevice(m->dev));
    CUDA_TRY(cudaMemcpyAsync(it->second.dst, host, (size_t)bytes, cudaMemcpyHostToDevice, m->stream));
    if ((float *)it->second.dst == m->embed) {      // the LM head's candidate margin needs max |w|
        const float *w = (const float *)host;
        float mx = 0.0f;
        for (int64_t i = 0; i < bytes / 4; ++i) {
            const float a = std::fabs(w[i]);
            if (a != a) {                          // a NaN weight: every CTA then rechecks its rows
                mx = a;
                break;
            }
            if (a > mx) mx = a;
        }
        m->wmax = mx;
        // the largest row 2-norm, summed in double and rounded up to a float
        double nmax = 0.0;
        const int64_t hid = m->c.hidden, rows = bytes / 4 / hid;
        for (int64_t r = 0; r < rows && mx == mx; ++r) {
            double q = 0.0;
            for (int64_t i = 0; i < hid; ++i) q += (double)w[r * hid + i] * (double)w[r * hid + i];
            nmax = std::max(nmax, std::sqrt(q));
        }
        m->wnorm = mx == mx ? std::nextafter((float)nmax, INFINITY) : mx;
        if (m->tc_head) {
            lm_tiles_kernel<<<1184, 256, 0, m->stream>>>(m->lm_tiles, m->embed, (int)m->c.vocab, (int)m->c.hidden);
            NC_TRY(check_launch("lm_tiles_kernel"));
        }
        if (m->q8_head) {
            lm_q8_kernel<<<(unsigned)((m->c.vocab + 7) / 8), 256, 0, m->stream>>>(m->lmq_q, m->lmq_s, m->embed,
                                                                                 (int)m->c.vocab, (int)m->c.hidden);
            NC_TRY(check_launch("lm_q8_kernel"));
        }
    }
    if (it->second.int8) {
        xor80_kernel<<<592, 256, 0, m->stream>>>((uint8_t *)it->second.dst, bytes);
        NC_TRY(check_launch("xor80_kernel"));
    }
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->uploaded.insert(name);
    return NC_OK;
}

extern "C" int32_t nc_qwen2_missing_weights(const nc_model *m, int32_t *count) {
    int32_t n = 0;
    std::string first;
    for (auto &w : m->weights)
        if (!m->uploaded.count(w.first)) {
            if (!n) first = w.first;
            ++n;
        }
    *count = n;
    if (n) g_error = "missing weights, first " + first;
    return NC_OK;
}

static int32_t check_ready(nc_model *m) {
    if (m->uploaded.size() != m->weights.size()) {
        int32_t n;
        nc_qwen2_missing_weights(m, &n);
        return fail(NC_ERR_STATE, "%s (%d missing)", g_error.c_str(), n);
    }
    return NC_OK;
}

static int32_t kv_copy(nc_model *m, int32_t slot, int64_t start, int64_t count, float *keys, float *values,
                       bool to_device) {
    const nc_qwen2_config &c = m->c;
    if (slot < 0 || slot >= c.slots || start < 0 || count < 0 || start + count > c.capacity)
        return fail(NC_ERR_ARGUMENT, "KV range slot %d [%lld, %lld) outside the cache", slot, (long long)start,
                    (long long)(start + count));
    if (count == 0) return NC_OK;
    CUDA_TRY(cudaSetDevice(m->dev));
    const int64_t d = c.head_dim;
    for (int64_t l = 0; l < c.layers; ++l)
        for (int64_t kvi = 0; kvi < 2; ++kvi)
            for (int64_t g = 0; g < c.kv_heads; ++g) {
                float *dev = m->kv + slot * m->slot_stride + l * m->layer_stride + (kvi * c.kv_heads + g) * c.capacity * d +
                             start * d;
                float *host = (kvi ? values : keys) + ((l * c.kv_heads + g) * count) * d;
                if (to_device)
                    CUDA_TRY(cudaMemcpyAsync(dev, host, count * d * 4, cudaMemcpyHostToDevice, m->stream));
                else
                    CUDA_TRY(cudaMemcpyAsync(host, dev, count * d * 4, cudaMemcpyDeviceToHost, m->stream));
            }
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    return NC_OK;
}

extern "C" int32_t nc_qwen2_kv_write(nc_model *m, int32_t slot, int64_t start, int64_t count, const float *keys,
                                     const float *values) {
    return kv_copy(m, slot, start, count, (float *)keys, (float *)values, true);
}

extern "C" int32_t nc_qwen2_kv_read(nc_model *m, int32_t slot, int64_t start, int64_t count, float *keys,
                                    float *values) {
    return kv_copy(m, slot, start, count, keys, values, false);
}

static int32_t check_rows(nc_model *m, int32_t rows, const int32_t *slot, const int32_t *pos, bool *fused) {
    const nc_qwen2_config &c = m->c;
    if (rows <= 0 || rows > c.max_rows) return fail(NC_ERR_ARGUMENT, "%d rows, the model takes 1..%d", rows, c.max_rows);
    std::set<int32_t> seen;
    *fused = true;
    for (int r = 0; r < rows; ++r) {
        if (slot[r] < 0 || slot[r] >= c.slots) return fail(NC_ERR_ARGUMENT, "row %d: slot %d out of range", r, slot[r]);
        if (pos[r] < 0 || pos[r] >= c.capacity)
            return fail(NC_ERR_ARGUMENT, "row %d: position %d outside the cache capacity %d", r, pos[r], c.capacity);
        if (!seen.insert(slot[r]).second) {
            *fused = false;
            if (r == 0 || slot[r - 1] != slot[r] || pos[r - 1] + 1 != pos[r])
                return fail(NC_ERR_ARGUMENT, "rows of slot %d must be consecutive positions", slot[r]);
        }
    }
    return NC_OK;
}

extern "C" int32_t nc_qwen2_step(nc_model *m, int32_t rows, const int64_t *ids, const int32_t *slot,
                                 const int32_t *pos, int32_t logit_rows, const int32_t *logit_row, float *logits,
                                 int64_t *tokens, int32_t *bad_row) {
    if (!m || !ids || !slot || !pos) return fail(NC_ERR_ARGUMENT, "null argument");
    NC_TRY(check_ready(m));
    bool fused;
    NC_TRY(check_rows(m, rows, slot, pos, &fused));
    if (logit_rows < 0 || logit_rows > rows) return fail(NC_ERR_ARGUMENT, "bad logit row count");
    for (int i = 0; i < logit_rows; ++i)
        if (logit_row[i] < 0 || logit_row[i] >= rows) return fail(NC_ERR_ARGUMENT, "bad logit row");
    CUDA_TRY(cudaSetDevice(m->dev));
    cudaStream_t st = m->stream;
    CUDA_TRY(cudaMemcpyAsync(m->ids, ids, rows * 8, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->slot, slot, rows * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->pos, pos, rows * 4, cudaMemcpyHostToDevice, st));
    if (logit_rows) CUDA_TRY(cudaMemcpyAsync(m->logit_row, logit_row, logit_rows * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemsetAsync(m->err, 0xff, sizeof(unsigned long long), st));
    m->logit_identity = logit_rows == rows;
    for (int i = 0; i < logit_rows; ++i) m->logit_identity = m->logit_identity && logit_row[i] == i;
    NC_TRY(enqueue_step(m, rows, logit_rows, fused, logits == nullptr));
    unsigned long long err = 0;
    CUDA_TRY(cudaMemcpyAsync(&err, m->err, 8, cudaMemcpyDeviceToHost, st));
    if (logits && logit_rows)
        CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)logit_rows * m->c.vocab * 4, cudaMemcpyDeviceToHost, st));
    if (tokens && logit_rows) CUDA_TRY(cudaMemcpyAsync(tokens, m->tokens, logit_rows * 8, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (err != ~0ull) {
        if (bad_row) *bad_row = (int32_t)err;
        return fail(NC_ERR_KERNEL, "gather index %lld is outside 0..%lld", (long long)ids[err],
                    (long long)(m->c.vocab - 1));
    }
    return model_faults(m);
}

// tokens_only: the step needs no logits (the last step's logits are not read back), so a batch
// may take the tensor-core LM head.
static int32_t decode_graph(nc_model *m, int batch, bool tokens_only, cudaGraphExec_t *out) {
    const int key = 2 * batch + (tokens_only ? 1 : 0);
    auto it = m->decode_graphs.find(key);
    if (it != m->decode_graphs.end()) {
        *out = it->second;
        return NC_OK;
    }
    cudaGraph_t graph;
    if (m->probing) return fail(NC_ERR_STATE, "a decode graph cannot be captured while the kernel-time probe is on");
    CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    m->logit_identity = true;                 // decode_setup makes the logit rows 0..batch-1
    int32_t s = enqueue_step(m, batch, batch, true, tokens_only);
    if (s == NC_OK) {
        if (launch_k(advance_kernel, 1, 1024, 0, m->stream, m->ids, m->pos, m->tokens, m->history, m->step, batch) !=
            cudaSuccess)
            s = fail(NC_ERR_CUDA, "launching advance_kernel");
        s = check_launch("advance_kernel");
    }
    cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (s != NC_OK) return s;
    if (e != cudaSuccess) return fail(NC_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return fail(NC_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
    m->decode_graphs[key] = exec;
    *out = exec;
    return NC_OK;
}

static int32_t decode_setup(nc_model *m, int32_t batch, const int32_t *slot, const int64_t *first,
                            const int32_t *start, int32_t steps, bool tokens_only, cudaGraphExec_t *graph) {
    if (!m || !slot || !first || !start) return fail(NC_ERR_ARGUMENT, "null argument");
    NC_TRY(check_ready(m));
    if (batch <= 0 || batch > m->c.max_rows || batch > 1024)
        return fail(NC_ERR_ARGUMENT, "batch %d outside 1..%d", batch, m->c.max_rows);
    if (steps < 0 || steps > m->history_steps)
        return fail(NC_ERR_ARGUMENT, "%d steps, at most %d per call", steps, m->history_steps);
    bool fused;
    NC_TRY(check_rows(m, batch, slot, start, &fused));
    if (!fused) return fail(NC_ERR_ARGUMENT, "decode rows must be distinct slots");
    for (int b = 0; b < batch; ++b) {
        if (first[b] < 0 || first[b] >= m->c.vocab)
            return fail(NC_ERR_KERNEL, "gather index %lld is outside 0..%lld", (long long)first[b],
                        (long long)(m->c.vocab - 1));
        if ((int64_t)start[b] + steps > m->c.capacity)
            return fail(NC_ERR_ARGUMENT, "row %d: %d steps from position %d pass the capacity %d", b, steps, start[b],
                        m->c.capacity);
    }
    CUDA_TRY(cudaSetDevice(m->dev));
    cudaStream_t st = m->stream;
    std::vector<int32_t> rows(batch);
    for (int b = 0; b < batch; ++b) rows[b] = b;
    CUDA_TRY(cudaMemcpyAsync(m->ids, first, batch * 8, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->slot, slot, batch * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->pos, start, batch * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->logit_row, rows.data(), batch * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemsetAsync(m->step, 0, 4, st));
    NC_TRY(decode_graph(m, batch, tokens_only, graph));
    CUDA_TRY(cudaStreamSynchronize(st));
    return NC_OK;
}

extern "C" int32_t nc_qwen2_decode(nc_model *m, int32_t batch, const int32_t *slot, const int64_t *first,
                                   const int32_t *start, int32_t steps, int32_t per_step, int64_t *tokens,
                                   float *logits) {
    cudaGraphExec_t graph;
    NC_TRY(decode_setup(m, batch, slot, first, start, steps, logits == nullptr, &graph));
    cudaStream_t st = m->stream;
    if (per_step) {
        // the host in the loop: each step's input tokens go host -> device from pinned memory,
        // its argmax comes back, and the host waits for it
        if (!m->pinned) CUDA_TRY(cudaHostAlloc((void **)&m->pinned, 2 * sizeof(int64_t) * m->c.max_rows, 0));
        int64_t *in = m->pinned, *out = m->pinned + m->c.max_rows;
        std::memcpy(in, first, batch * sizeof(int64_t));
        for (int s = 0; s < steps; ++s) {
            CUDA_TRY(cudaMemcpyAsync(m->ids, in, batch * 8, cudaMemcpyHostToDevice, st));
            CUDA_TRY(cudaGraphLaunch(graph, st));
            CUDA_TRY(cudaMemcpyAsync(out, m->tokens, batch * 8, cudaMemcpyDeviceToHost, st));
            CUDA_TRY(cudaStreamSynchronize(st));
            if (tokens) std::memcpy(tokens + (int64_t)s * batch, out, batch * sizeof(int64_t));
            std::memcpy(in, out, batch * sizeof(int64_t));
        }
    } else {
        for (int s = 0; s < steps; ++s) CUDA_TRY(cudaGraphLaunch(graph, st));
    }
    if (!per_step && tokens && steps)
        CUDA_TRY(cudaMemcpyAsync(tokens, m->history, (size_t)steps * batch * 8, cudaMemcpyDeviceToHost, st));
    if (logits && steps)
        CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)batch * m->c.vocab * 4, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    return model_faults(m);
}

extern "C" int32_t nc_qwen2_profile(nc_model *m, int32_t batch, const int32_t *slot, const int64_t *first,
                                    const int32_t *start, int32_t steps, float *ms_per_kind, int32_t *launches_per_kind) {
    cudaGraphExec_t graph;
    NC_TRY(decode_setup(m, batch, slot, first, start, steps, true, &graph));
    for (int k = 0; k < K_KINDS; ++k) {
        ms_per_kind[k] = 0.0f;
        launches_per_kind[k] = 0;
    }
    cudaStream_t st = m->stream;
    for (int s = 0; s < steps; ++s) {
        m->probing = true;
        m->event_next = 0;
        m->probe_marks.clear();
        m->logit_identity = true;
        int32_t status = enqueue_step(m, batch, batch, true, true);
        m->probing = false;
        NC_TRY(status);
        if (launch_k(advance_kernel, 1, 1024, 0, st, m->ids, m->pos, m->tokens, m->history, m->step, batch) != cudaSuccess)
            return fail(NC_ERR_CUDA, "launching advance_kernel");
        CUDA_TRY(cudaStreamSynchronize(st));
        for (auto &pm : m->probe_marks) {
            float ms = 0.0f;
            CUDA_TRY(cudaEventElapsedTime(&ms, pm.second.first, pm.second.second));
            ms_per_kind[pm.first] += ms;
            launches_per_kind[pm.first] += 1;
        }
    }
    return model_faults(m);
}

extern "C" int32_t nc_qwen2_phase_times(nc_model *m, int32_t batch, const int32_t *slot, const int64_t *first,
                                         const int32_t *start, int32_t steps, float *us_per_event) {
    if (!us_per_event) return fail(NC_ERR_ARGUMENT, "null argument");
    cudaGraphExec_t graph;
    NC_TRY(decode_setup(m, batch, slot, first, start, steps, true, &graph));
    if (!(m->c.quant == 1 && m->mk_ctas && batch <= MK_ROWS))
        return fail(NC_ERR_STATE, "the persistent decode kernel does not serve %d rows of this model", batch);
    const int G = m->mk_ctas, nl = (int)m->c.layers;
    const size_t words = (size_t)G * nl * MK_EVENTS;
    unsigned long long *dev = nullptr;
    CUDA_TRY(cudaMalloc(&dev, words * 8));
    std::vector<unsigned long long> host(words);
    std::vector<double> sum(MK_EVENTS, 0.0);
    std::vector<int> count(MK_EVENTS, 0);
    cudaStream_t st = m->stream;
    int32_t status = NC_OK;
    m->logit_identity = true;
    for (int s = 0; s < steps && status == NC_OK; ++s) {
        if (cudaMemsetAsync(dev, 0, words * 8, st) != cudaSuccess) { status = fail(NC_ERR_CUDA, "clearing stamps"); break; }
        m->mk_stamps = dev;
        status = enqueue_step(m, batch, batch, true, true);
        m->mk_stamps = nullptr;
        if (status != NC_OK) break;
        if (launch_k(advance_kernel, 1, 1024, 0, st, m->ids, m->pos, m->tokens, m->history, m->step, batch) != cudaSuccess) {
            status = fail(NC_ERR_CUDA, "launching advance_kernel");
            break;
        }
        if (cudaMemcpyAsync(host.data(), dev, words * 8, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            status = fail(NC_ERR_CUDA, "reading stamps");
            break;
        }
        // per layer and event: the last CTA that wrote it, from the first CTA to start the layer
        for (int l = 0; l < nl; ++l) {
            unsigned long long t0 = ~0ull;
            for (int b = 0; b < G; ++b) {
                const unsigned long long v = host[((size_t)b * nl + l) * MK_EVENTS];
                if (v && v < t0) t0 = v;
            }
            if (t0 == ~0ull) continue;
            for (int e = 0; e < MK_EVENTS; ++e) {
                unsigned long long last = 0;
                for (int b = 0; b < G; ++b) last = std::max(last, host[((size_t)b * nl + l) * MK_EVENTS + e]);
                if (last >= t0) {
                    sum[e] += (double)(last - t0) * 1e-3;
                    count[e] += 1;
                }
            }
        }
    }
    cudaFree(dev);
    NC_TRY(status);
    for (int e = 0; e < MK_EVENTS; ++e) us_per_event[e] = count[e] ? (float)(sum[e] / count[e]) : -1.0f;
    return model_faults(m);
}

extern "C" int32_t nc_qwen2_decode_timed(nc_model *m, int32_t batch, const int32_t *slot, const int64_t *first,
                                         const int32_t *start, int32_t steps, float *ms) {
    cudaGraphExec_t graph;
    NC_TRY(decode_setup(m, batch, slot, first, start, steps, true, &graph));
    cudaStream_t st = m->stream;
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    CUDA_TRY(cudaEventCreate(&b));
    CUDA_TRY(cudaEventRecord(a, st));
    for (int s = 0; s < steps; ++s) CUDA_TRY(cudaGraphLaunch(graph, st));
    CUDA_TRY(cudaEventRecord(b, st));
    CUDA_TRY(cudaEventSynchronize(b));
    CUDA_TRY(cudaEventElapsedTime(ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return model_faults(m);
}

extern "C" int32_t nc_qwen2_probe(nc_model *m, int32_t on, float *ms_per_kind, int32_t *launches_per_kind) {
    if (!m) return fail(NC_ERR_ARGUMENT, "null model");
    if (on) {
        m->probing = true;
        m->event_next = 0;
        m->probe_marks.clear();
        return NC_OK;
    }
    m->probing = false;
    for (int k = 0; k < K_KINDS; ++k) {
        if (ms_per_kind) ms_per_kind[k] = 0.0f;
        if (launches_per_kind) launches_per_kind[k] = 0;
    }
    CUDA_TRY(cudaSetDevice(m->dev));
    CUDA_TRY(cudaStreamSynchronize(m->stream));
    for (auto &pm : m->probe_marks) {
        float ms = 0.0f;
        CUDA_TRY(cudaEventElapsedTime(&ms, pm.second.first, pm.second.second));
        if (ms_per_kind) ms_per_kind[pm.first] += ms;
        if (launches_per_kind) launches_per_kind[pm.first] += 1;
    }
    m->probe_marks.clear();
    return NC_OK;
}

// A float32 projection quantized on the device into its "<name>@int8" / "<name>@scales" slots
// (nanocompile/quantize.py:55-70, the same bytes as the host scheme), staged through a
// temporary device buffer.
extern "C" int32_t nc_qwen2_upload_quantize(nc_model *m, const char *name, const float *host, int64_t bytes) {
    if (!m || !name || !host) return fail(NC_ERR_ARGUMENT, "null argument");
    const std::string base(name);
    auto qi = m->weights.find(base + "@int8"), si = m->weights.find(base + "@scales");
    if (qi == m->weights.end() || si == m->weights.end())
        return fail(NC_ERR_ARGUMENT, "no int8 projection named %s", name);
    const int64_t rows = si->second.bytes / 4, cols = rows ? qi->second.bytes / rows : 0;
    if (bytes != rows * cols * 4)
        return fail(NC_ERR_ARGUMENT, "weight %s has %lld bytes, expected %lld float32", name, (long long)bytes,
                    (long long)(rows * cols * 4));
    CUDA_TRY(cudaSetDevice(m->dev));
    float *staged = nullptr;
    CUDA_TRY(cudaMalloc(&staged, (size_t)bytes));
    cudaError_t e = cudaMemcpyAsync(staged, host, (size_t)bytes, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) {
        quantize_int8_rows_kernel<<<(unsigned)rows, QI8_THREADS, 0, m->stream>>>(
            qi->second.dst, (float *)si->second.dst, staged, cols, 1);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    cudaFree(staged);
    if (e != cudaSuccess) return fail(NC_ERR_CUDA, "quantizing %s: %s", name, cudaGetErrorString(e));
    m->uploaded.insert(base + "@int8");
    m->uploaded.insert(base + "@scales");
    return NC_OK;
}

// Timing hook for benchmarks: `iters` eager steps over the same rows (a prompt of `rows` tokens of
// slot[0] from position pos[0]: its KV positions are rewritten with the same values each time),
// only the last row's token (argmax) produced; CUDA events on the model's stream around all of them.
extern "C" int32_t nc_qwen2_step_timed(nc_model *m, int32_t rows, const int64_t *ids, const int32_t *slot,
                                       const int32_t *pos, int32_t iters, float *ms) {
    if (!m || !ids || !slot || !pos || !ms) return fail(NC_ERR_ARGUMENT, "null argument");
    NC_TRY(check_ready(m));
    bool fused;
    NC_TRY(check_rows(m, rows, slot, pos, &fused));
    if (iters <= 0) return fail(NC_ERR_ARGUMENT, "iters %d", iters);
    CUDA_TRY(cudaSetDevice(m->dev));
    cudaStream_t st = m->stream;
    const int32_t last = rows - 1;
    CUDA_TRY(cudaMemcpyAsync(m->ids, ids, rows * 8, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->slot, slot, rows * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->pos, pos, rows * 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m->logit_row, &last, 4, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemsetAsync(m->err, 0xff, sizeof(unsigned long long), st));
    m->logit_identity = rows == 1;
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    CUDA_TRY(cudaEventCreate(&b));
    CUDA_TRY(cudaEventRecord(a, st));
    int32_t status = NC_OK;
    for (int i = 0; i < iters && status == NC_OK; ++i) status = enqueue_step(m, rows, 1, fused, true);
    CUDA_TRY(cudaEventRecord(b, st));
    CUDA_TRY(cudaEventSynchronize(b));
    CUDA_TRY(cudaEventElapsedTime(ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    NC_TRY(status);
    *ms /= (float)iters;
    return model_faults(m);
}

// ---- the LM head + argmax without any allocation ---------------------------------------------
// Some callers cannot call cudaMalloc: a host that gives this library a fixed device-memory
// budget and forbids allocations it did not make, code that runs while another thread captures
// a CUDA graph in global capture mode (an allocation there breaks the capture), or a latency-
// critical loop that cannot afford an allocation's implicit synchronization.  For them the
// LM head's scratch (a finish counter and one (value, index) pair per row and CTA) lives in
// this file-scope device array instead of caller-provided memory.  Every GPU that loads the
// library holds it until the process exits.
constexpr int64_t NOALLOC_PARTIALS = 32768;    // rows * ceil(vocab / 128) at most
constexpr size_t NOALLOC_SCRATCH_BYTES = 256 + NOALLOC_PARTIALS * (sizeof(float) + sizeof(int32_t));
static __device__ __align__(256) unsigned char g_lm_head_scratch[NOALLOC_SCRATCH_BYTES];

namespace {

// The array's device address, looked up once per device with that device current.  In host
// code g_lm_head_scratch names a host-side stand-in, not device memory.
constexpr int NOALLOC_MAX_DEVICES = 64;
void *g_scratch_addr[NOALLOC_MAX_DEVICES] = {};
std::mutex g_scratch_mutex;

int32_t noalloc_scratch(void **out) {
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(NC_ERR_ARGUMENT, "device %d beyond the scratch table", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        CUDA_TRY(cudaGetSymbolAddress(&p, g_lm_head_scratch));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return NC_OK;
}

}  // namespace

extern "C" int32_t nc_lm_head_argmax_noalloc(void **p, const int64_t *s, void *stream) {
    const int64_t rows = s[0], vocab = s[1], hidden = s[2];
    if (rows <= 0 || vocab <= 0) return NC_OK;
    // refuse sizes whose product could overflow before forming it (rows alone above the limit
    // can never fit; vocab and hidden must also fit the kernel's 32-bit sizes)
    if (rows > NOALLOC_PARTIALS || vocab > INT32_MAX || hidden <= 0 || hidden > INT32_MAX)
        return fail(NC_ERR_ARGUMENT,
                    "nc_lm_head_argmax_noalloc: rows %lld, vocab %lld, hidden %lld are outside what the static "
                    "scratch holds (rows * ceil(vocab / 128) <= %lld, vocab and hidden < 2^31)",
                    (long long)rows, (long long)vocab, (long long)hidden, (long long)NOALLOC_PARTIALS);
    const int64_t partials = rows * ((vocab + F32_ROWS - 1) / F32_ROWS);
    if (partials > NOALLOC_PARTIALS)
        return fail(NC_ERR_ARGUMENT,
                    "nc_lm_head_argmax_noalloc: %lld rows of a %lld-token vocabulary need %lld partial results; the "
                    "static scratch holds %lld (rows * ceil(vocab / 128) <= %lld)",
                    (long long)rows, (long long)vocab, (long long)partials, (long long)NOALLOC_PARTIALS,
                    (long long)NOALLOC_PARTIALS);
    if (hidden % F32_TILE) return fail(NC_ERR_ARGUMENT, "hidden %lld is not a multiple of %d", (long long)hidden, F32_TILE);
    void *scratch = nullptr;
    NC_TRY(noalloc_scratch(&scratch));
    // the finish counter must start at zero (a call that failed midway could leave it set)
    CUDA_TRY(cudaMemsetAsync(scratch, 0, 256, (cudaStream_t)stream));
    GemvF32Args a{};
    a.out = (float *)p[0];
    a.x = (const float *)p[1];
    a.w = (const float *)p[2];
    a.tokens = (int64_t *)p[3];
    a.m = (int)rows;
    a.n = (int)vocab;
    a.k = (int)hidden;
    a.counter = (unsigned int *)scratch;
    a.part_val = (float *)((char *)scratch + 256);
    a.part_idx = (int32_t *)((char *)scratch + 256 + partials * sizeof(float));
    return launch_f32((cudaStream_t)stream, a, EPI_NONE, a.tokens != nullptr);
}
