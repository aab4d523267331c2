/* nc_cuda.h -- the C ABI of libnc_cuda.so, the B200 (sm_100a) backend for nanocompile's
 * Qwen2 decode step.
 *
 * Two layers, both plain C: pointers, sizes, int32 status codes.
 *
 *  1. Fused-group entry points.  nanocompile's generated C exports one function per
 *     fused kernel with the signature  int32_t nc_kN(void **p, const int64_t *s)
 *     (nanocompile/codegen_c.py:3-10, nanocompile/loopir.py:329-336): p[0] is the
 *     output, p[1..] the operands, s the symbol values, 0 = OK.  The functions below
 *     keep that convention -- p[] holds DEVICE pointers, s[] the sizes -- and add the
 *     CUDA stream to launch on (NULL = the default stream).  One per fused group kind
 *     of an int8-vnni Qwen2 step (nanocompile/fusion.py:417-731).
 *
 *  2. The model runtime, the CUDA twin of nanocompile/runtime.py:167-318
 *     (CompiledGraph: compile once, then call per step): one device arena holding the
 *     weights, the KV cache of every sequence slot and the activations; a step is a
 *     fixed sequence of fused kernels, captured once as a CUDA graph and replayed.
 *
 * Every function returns 0 on success or a nonzero NC_* code; nc_last_error() gives
 * the message of the last failure on the calling thread.  No function calls back into
 * the caller.  One host thread should drive one model at a time.
 */
#ifndef NC_CUDA_H
#define NC_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    NC_OK = 0,
    NC_ERR_KERNEL = 1,      /* a kernel rejected its input (gather index out of range), as
                               the reference's kernel status 1 (nanocompile/runtime.py:298-318) */
    NC_ERR_ARGUMENT = 2,    /* bad sizes, names, capacity exceeded */
    NC_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    NC_ERR_STATE = 4,       /* call out of order (e.g. step before every weight is uploaded) */
};

/* The message of the last failure on this thread; returns its full length. */
int32_t nc_last_error(char *buf, int64_t size);

/* Library / device plumbing (device memory for the fused-group entry points). */
int32_t nc_device_count(int32_t *count);
int32_t nc_set_device(int32_t device);
int32_t nc_device_alloc(int64_t bytes, void **ptr);
int32_t nc_device_free(void *ptr);
int32_t nc_copy_to_device(void *dst, const void *src, int64_t bytes);
int32_t nc_copy_to_host(void *dst, const void *src, int64_t bytes);
int32_t nc_device_synchronize(void);

/* ---- 1. fused groups (device pointers; s[] sizes; stream may be NULL) -------------------- */

/* gather (nanocompile/fusion.py:713-731, call 0): rows of the embedding table by token id.
 * p: [0] out f32[rows, hidden]  [1] ids i64[rows]  [2] table f32[vocab, hidden]
 *    [3] error word u64 (device; set every byte to 0xff before the call; after it, the
 *        smallest row whose id was out of range, or still all ones)
 * s: rows, vocab, hidden */
int32_t nc_gather_rows(void **p, const int64_t *s, void *stream);

/* row kernel rms_norm (nanocompile/nn.py:34-38 -> fusion.py:631-650, calls 1/25/40), in the
 * reference's order (in-order float32 sum of squares), fused with block-32 activation
 * quantization (nanocompile/quantize.py:102-124, calls 2-7).
 * p: [0] normed f32[rows, n] (nullable)  [1] x f32[rows, n]  [2] weight f32[n]
 *    [3] xq i8[rows, n] (nullable: no quantization)  [4] xs f32[rows, n/32]  [5] offset f32[rows]
 *    [6] block sums i32[rows, n/32] (nullable)
 * s: rows, n, eps as float32 bits */
int32_t nc_rms_norm_quantize(void **p, const int64_t *s, void *stream);

/* block-32 activation quantization alone (calls 18-23, 33-38).
 * p: [0] xq i8[rows, k]  [1] x f32[rows, k]  [2] xs f32[rows, k/32]  [3] offset f32[rows]
 *    [4] block sums i32[rows, k/32] (nullable)
 * s: rows, k */
int32_t nc_quantize_blocks(void **p, const int64_t *s, void *stream);

/* matmul_i8_vnni with its epilogue (nanocompile/lower.py:363-397, fusion.py:677-711; calls
 * 8/12/16/24/32/39), bit-exact: 32 float32 accumulators per output, one per 4-byte Dp4 lane,
 * FMA'd by the block scale in the reference's k order, combined in its order.
 * Weights are the reference's int8 values offset by 128 (w ^ 0x80, as unsigned bytes; see
 * nc_pack_int8_weights).
 * p: [0] out f32[rows, n]  [1] xq i8[rows, k]  [2] xs f32[rows, k/32]  [3] offset f32[rows]
 *    [4] w u8[n, k]  [5] scales f32[n]  [6] epilogue operand (bias f32[n] / residual
 *    f32[rows, n] / second weight u8[n, k] for SwiGLU)  [7] second scales f32[n] (SwiGLU)
 * s: rows, n, k, epilogue (0 none, 1 bias, 2 residual, 3 silu(y0) * y1) */
int32_t nc_matmul_i8_vnni(void **p, const int64_t *s, void *stream);

/* The same projection on the tensor cores (tcgen05.mma kind::i8, block-diagonal activations so
 * every 4-byte Dp4 lane stays its own int32), bit for bit the reference's matmul_i8_vnni
 * (nanocompile/lower.py:363-397 with _combine, lower.py:298-317, and the fused epilogues of
 * nanocompile/fusion.py:699-711).  The model runtime takes it for steps of more than four rows.
 * p: [0] out f32[m, n] (unused by epilogue 4)  [1] xq i8[m, k]  [2] xs f32[m, k/32]
 *    [3] offset f32[m] (prologue 0)  [4] w u8[n, k] (int8 + 128)  [5] scales f32[n]
 *    [6] bias / residual / second weight (SwiGLU)  [7] second scales (SwiGLU)
 *    [8] block sums i32[m, k/32] (prologue 2: the offset is 128 * in-order sum of sum_b * xs_b)
 *    [9] xq out i8[m, n]  [10] xs out f32[m, n/32]  [11] block sums out i32[m, n/32] (epilogue 4)
 * s: m, n, k, epilogue (0 none, 1 bias, 2 residual, 3 silu(gate)*up, 4 the same block-quantized),
 *    prologue (0 given offsets, 2 from block sums), tokens per work item (0 or 4) */
int32_t nc_matmul_i8_tc(void **p, const int64_t *s, void *stream);

/* float32 matmul with epilogue (nanocompile/lower.py:255-274, fusion.py:652-675):
 * acc = acc + x[k] * w[n, k] in index order, no FMA.
 * p: [0] out f32[rows, n]  [1] x f32[rows, k]  [2] w f32[n, k]  [3] epilogue operand
 *    (bias / residual / second weight)
 * s: rows, n, k, epilogue (as above) */
int32_t nc_matmul_f32(void **p, const int64_t *s, void *stream);

/* matmul_i8 (+epilogue): int8 weights, float32 activations (nanocompile/lower.py:320-356
 * int8_dots, times scales[n]: lower.py:398-412, fusion.py:677-711).  Widths multiples of 16.
 * p: [0] out f32[rows, n]  [1] x f32[rows, k]  [2] w u8[n, k] (int8 + 128)  [3] scales f32[n]
 *    [4] bias / residual / up weights (SwiGLU)  [5] up scales (SwiGLU)
 * s: rows, n, k, epilogue (0 none, 1 bias, 2 residual, 3 silu(gate)*up) */
int32_t nc_matmul_i8_f32(void **p, const int64_t *s, void *stream);

/* The tied LM head (call 41) fused with greedy argmax (nanocompile/models/qwen2.py:364,
 * first maximum wins): logits = x @ embed.T in index order per row, then the argmax of
 * each row.  Scratch holds one (value, index) pair per (row, CTA): nc_lm_head_scratch_bytes.
 * p: [0] logits f32[rows, vocab] (nullable)  [1] x f32[rows, hidden]  [2] embed f32[vocab, hidden]
 *    [3] tokens i64[rows] (nullable)  [4] scratch (device, >= nc_lm_head_scratch_bytes)
 * s: rows, vocab, hidden */
int32_t nc_lm_head_argmax(void **p, const int64_t *s, void *stream);
int64_t nc_lm_head_scratch_bytes(int64_t rows, int64_t vocab);

/* nc_lm_head_argmax for callers that cannot allocate device memory (a host that fixes this
 * library's memory budget, another thread capturing a graph in global capture mode, a loop that
 * cannot take an allocation's implicit synchronization).  No counterpart in the reference: its
 * CPU kernels never needed device scratch.  Same p[] as nc_lm_head_argmax without p[4]: the
 * scratch is a static device array of the library, so nothing is allocated, ever.
 *  - Limit: rows * ceil(vocab / 128) <= 32768 (e.g. 27 rows of a 151,936-token vocabulary);
 *    larger calls fail with NC_ERR_ARGUMENT and a message.
 *  - The first call on each device looks the array's address up (cudaGetSymbolAddress, with
 *    that device current); make that first call before any stream capture.  The address is
 *    kept for the life of the process: it does not survive a cudaDeviceReset of that device
 *    (the library's module is reloaded at a new address), so do not call this entry point on
 *    a device after resetting it.
 *  - Every call shares the array: calls that overlap on the GPU (other streams, other host
 *    threads) race.  Each call clears the finish counter on its stream before the kernel. */
int32_t nc_lm_head_argmax_noalloc(void **p, const int64_t *s, void *stream);

/* The same tokens as nc_lm_head_argmax (np.argmax of the in-order float32 logits,
 * nanocompile/models/qwen2.py:364) for 1..16 rows and a hidden width that is a multiple of 128
 * up to 1024, reading an int8 copy of the embedding instead of the float32 one: approximate
 * logits from the copy, then the exact logits of every row the approximation's error bound
 * cannot rule out.
 *  nc_lm_head_q8_prepare:  p: [0] embedding f32[vocab, hidden]  [1] copy i8[vocab, hidden]
 *                             [2] row scales f32[vocab]    s: [0] vocab  [1] hidden
 *  nc_lm_head_q8_argmax:   p: [0] x f32[rows, hidden]  [1] embedding  [2] copy  [3] row scales
 *                             [4] tokens i64[rows]  [5] scratch (device, >= nc_lm_head_q8_scratch_bytes)
 *                          s: [0] rows  [1] vocab  [2] hidden
 * The scratch's first word must be zero before the first call (it is zero again after each). */
int32_t nc_lm_head_q8_prepare(void **p, const int64_t *s, void *stream);
int32_t nc_lm_head_q8_argmax(void **p, const int64_t *s, void *stream);
int64_t nc_lm_head_q8_scratch_bytes(int64_t rows, int64_t vocab);

/* Decode attention over a KV cache (calls 14-17 with RoPE calls 9-13 fused in): for one new
 * token per row, bias is already in qkv; RoPE q and k, append k/v to the cache at the row's
 * position, scores in index order, softmax (NaN-propagating max, in-order sum of expf),
 * probabilities @ V in index order.
 * p: [0] ctx f32[rows, heads*d]  [1] qkv f32[rows, (heads+2*kv)*d] (biased projections)
 *    [2] cache f32 (layout: slot, {K,V}, kv, capacity, d -- this layer's)  [3] cos f32[cap, d/2]
 *    [4] sin f32[cap, d/2]  [5] slot i32[rows]  [6] pos i32[rows]
 * s: rows, heads, kv_heads, d, capacity, slot stride (floats), append (1 = write k/v),
 *    attention scale as float32 bits */
int32_t nc_attention(void **p, const int64_t *s, void *stream);

/* nc_attention for a cache whose extent is known: s[8] = slots in the cache (p[2] holds
 * s[8] * slot stride floats).  More than eight rows then stream K/V chunks by TMA from a tensor
 * map over the cache (head dims that are multiples of 32).  Same reference interface as
 * nc_attention. */
int32_t nc_attention_cache(void **p, const int64_t *s, void *stream);

/* NC_ERR_KERNEL if a kernel recorded a device-side fault since the last call (a TMA stage of
 * the grouped attention kernel that did not arrive within its bounded wait); clears it. */
int32_t nc_device_faults(void);

/* Bounds the library's abandonable device-side waits (pipeline stages of the tensor-core
 * projection, the self-test below) to `cycles` SM clock cycles on the current device; <= 0
 * restores the default 2^31 (about a second).  A wait that runs out makes its kernel stop, drain
 * the copies and MMAs it has in flight, free its TMEM and record a fault that the next
 * nc_device_faults / model call reports as NC_ERR_KERNEL.  For tests of that path. */
int32_t nc_set_wait_limit(int64_t cycles);

/* Runs one of the bounded waits against a condition that never comes true, with nothing in
 * flight: kind 0 polls hand-over words that never carry their tag (the persistent decode
 * step's wait), kind 1 waits on an mbarrier whose bytes never arrive (a pipeline stage wait).
 * Returns NC_ERR_KERNEL once the wait has given up (and clears the fault), NC_OK never. */
int32_t nc_selftest_wait(int32_t kind);

/* int8 weights as the kernels read them: u8 = int8 + 128 (one XOR per byte). */
int32_t nc_pack_int8_weights(void *dst_device, const int8_t *src_host, int64_t bytes);

/* glibc's expf, bit for bit, evaluated on the device (test hook for the softmax / SiLU math).
 * p: [0] out f32[n]  [1] x f32[n];  s: n */
int32_t nc_expf_exact(void **p, const int64_t *s, void *stream);

/* quantize_int8 (nanocompile/quantize.py:55-70) on the device: per-row symmetric int8 weights,
 * scale = max|row| / 127 (0 -> 1), values sign(v) * floor(|v| + 0.5) of v = w / scale clipped to
 * +-127 -- the same bytes and scales as the host scheme.
 * p: [0] values i8[rows, cols] (packed: u8 value + 128, the layout the projections read)
 *    [1] scales f32[rows]  [2] weights f32[rows, cols]
 * s: rows, cols, packed (0 / 1) */
int32_t nc_quantize_int8_rows(void **p, const int64_t *s, void *stream);

/* The block scale mag / 127 is computed by a branch-free correctly rounded division; this runs
 * it against the IEEE divide on every non-negative float and reports the differences (0). */
int32_t nc_selfcheck_div127(int64_t *mismatches);

/* ---- 2. the model runtime ---------------------------------------------------------------- */

typedef struct nc_model nc_model;

typedef struct {
    int64_t vocab, hidden, inter, layers, heads, kv_heads, head_dim;
    float eps;            /* float32(rms_norm_eps) */
    float attn_scale;     /* float32(head_dim ** -0.5) */
    int32_t quant;        /* 0 = float32 projections, 1 = int8-vnni, 2 = int8 weights + float32 activations */
    int32_t max_rows;     /* token rows per step (prompt length, or sequences in a batch) */
    int32_t slots;        /* KV-cache sequence slots */
    int32_t capacity;     /* KV positions per slot */
    int32_t device;       /* CUDA device ordinal */
} nc_qwen2_config;

/* Allocates the arena on cfg->device.  inv_freq: float32[head_dim/2], RoPE's rates
 * (nanocompile/nn.py:69-75); cos/sin tables of every position are made from it here with
 * the C library's cosf/sinf, the same functions the reference's generated C calls. */
int32_t nc_qwen2_create(const nc_qwen2_config *cfg, const float *inv_freq, nc_model **out);
int32_t nc_qwen2_destroy(nc_model *model);
int64_t nc_qwen2_arena_bytes(const nc_model *model);

/* Upload one weight by its checkpoint name (int8 ones as "<name>@int8" / "<name>@scales",
 * nanocompile/quantize.py:47-52).  Returns NC_ERR_ARGUMENT for an unknown name or size. */
int32_t nc_qwen2_upload(nc_model *model, const char *name, const void *host, int64_t bytes);
int32_t nc_qwen2_missing_weights(const nc_model *model, int32_t *count);
/* A float32 projection "<name>" of an int8 model, quantized on the device (nc_quantize_int8_rows)
 * into its "<name>@int8" / "<name>@scales" weights: the host need not run quantize_int8. */
int32_t nc_qwen2_upload_quantize(nc_model *model, const char *name, const float *host, int64_t bytes);

/* KV cache of one slot: positions [start, start+count) of every layer, host arrays
 * [layers, kv_heads, count, head_dim]. */
int32_t nc_qwen2_kv_write(nc_model *model, int32_t slot, int64_t start, int64_t count,
                          const float *keys, const float *values);
int32_t nc_qwen2_kv_read(nc_model *model, int32_t slot, int64_t start, int64_t count,
                         float *keys, float *values);

/* One step on `rows` token rows: row r is token ids[r] of sequence slot[r] at position
 * pos[r] (its KV history is positions 0..pos[r]-1 of that slot).  Rows of one slot must be
 * consecutive positions in order (a prompt); a slot may also appear once (decode).
 * Logits are produced for the `logit_rows` rows listed in logit_row[] (host), into
 * logits (host, nullable) [logit_rows, vocab], with the argmax of each into tokens (host,
 * nullable).  Returns NC_ERR_KERNEL for an id outside 0..vocab-1; *bad_row (nullable)
 * gets the first such row. */
int32_t nc_qwen2_step(nc_model *model, int32_t rows, const int64_t *ids, const int32_t *slot,
                      const int32_t *pos, int32_t logit_rows, const int32_t *logit_row,
                      float *logits, int64_t *tokens, int32_t *bad_row);

/* Greedy decode of `batch` sequences, one new token each per step, for `steps` steps: row b
 * starts from token first[b] at position start[b] of slot[b].  Each step is one replay of a
 * captured CUDA graph; the argmax feeds the next step on the device.  tokens (host)
 * [steps, batch]; logits (host, nullable) [batch, vocab] of the last step.
 * With per_step != 0 the host is in the loop: every step copies its input tokens host -> device
 * from pinned memory, replays the graph, copies the step's argmax back and synchronizes;
 * otherwise the argmax feeds the next step on the device and the tokens come back once. */
int32_t nc_qwen2_decode(nc_model *model, int32_t batch, const int32_t *slot, const int64_t *first,
                        const int32_t *start, int32_t steps, int32_t per_step, int64_t *tokens,
                        float *logits);

/* Timing hook for benchmarks: runs `steps` replays of the captured decode graph from the given
 * state, timed with CUDA events on the model's stream; *ms gets the elapsed milliseconds. */
int32_t nc_qwen2_decode_timed(nc_model *model, int32_t batch, const int32_t *slot, const int64_t *first,
                              const int32_t *start, int32_t steps, float *ms);

/* Kernel-time probe: runs `steps` decode steps eagerly (not as a graph) with CUDA events around
 * every launch, and sums the milliseconds and launches per fused-group kind into the
 * [NC_KINDS] arrays (kinds: 0 gather, 1 q/k/v projection, 2 attention, 3 o projection,
 * 4 gate/up projection, 5 down projection, 6 rms_norm row kernel, 7 block quantization,
 * 8 LM head + argmax, 9 the persistent decode kernel's layers). */
#define NC_KINDS 10

/* Timing hook for benchmarks: `iters` eager steps of the same `rows` rows (ids / slot / pos as
 * nc_qwen2_step; the rows' KV positions are rewritten with the same values each time), each
 * producing only the last row's argmax; *ms gets the average milliseconds per step, CUDA events
 * on the model's stream.  Configuration 4 (a 512-token prefill) is timed with it. */
int32_t nc_qwen2_step_timed(nc_model *model, int32_t rows, const int64_t *ids, const int32_t *slot,
                            const int32_t *pos, int32_t iters, float *ms);
/* Kernel-time probe around nc_qwen2_step calls: on != 0 starts bracketing every launch of the
 * following steps with CUDA events; on == 0 stops, synchronizes and sums milliseconds and
 * launches per fused-group kind (as nc_qwen2_profile) into the arrays (nullable). */
int32_t nc_qwen2_probe(nc_model *model, int32_t on, float *ms_per_kind, int32_t *launches_per_kind);

int32_t nc_qwen2_profile(nc_model *model, int32_t batch, const int32_t *slot, const int64_t *first,
                         const int32_t *start, int32_t steps, float *ms_per_kind, int32_t *launches_per_kind);

/* Phase table of the persistent decode kernel: `steps` eager decode steps (arguments as
 * nc_qwen2_decode) with globaltimer stamps; us_per_event[NC_MK_EVENTS] gets, per event, the mean
 * over layers and steps of the microseconds from the first CTA starting the layer to the last CTA
 * reaching the event (-1: never reached).  Events: 0 layer start, 1 input words in, 2 input norm +
 * quantization, 3 q/k/v rows out, 4 q/k/v words in (attention), 5 scores, 6 softmax, 7 attention
 * out, 8 attention blocks in, 9 o rows out, 10 residual words in, 11 post norm, 12 gate/up rows
 * staged, 13 SwiGLU blocks out, 14 SwiGLU blocks in, 15 down rows out.  NC_ERR_STATE when the
 * persistent kernel does not serve `batch` rows of the model. */
#define NC_MK_EVENTS 16
int32_t nc_qwen2_phase_times(nc_model *model, int32_t batch, const int32_t *slot, const int64_t *first,
                             const int32_t *start, int32_t steps, float *us_per_event);

#ifdef __cplusplus
}
#endif
#endif
