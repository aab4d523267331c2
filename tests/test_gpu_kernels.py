"""Each fused group on the B200, through the C ABI, against the oracle and the reference's goldens.

Bit-exact for everything: integers (xq, block sums, argmax indices) and float32 (the
kernels follow the reference's operation order, so any difference is a bug).
"""

from __future__ import annotations

import numpy as np
import pytest

from nanocompile_b200 import quantize as q
from oracle import oracle
from tests.conftest import bits, golden
from tests.gpu_util import DeviceArray, call, f32_bits, packed_int8

pytestmark = pytest.mark.gpu


def same_bits(a, b) -> bool:
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and bool(((bits(a) == bits(b)) | (np.isnan(a) & np.isnan(b))).all())


def activations(rng, rows, k, outliers=True):
    x = (rng.standard_normal((rows, k)) * 2).astype(np.float32)
    if outliers:
        x[:, ::13] *= 40.0
    return x


def test_expf_is_glibc_bit_for_bit(cuda):
    u = np.arange(0, 2**32, 257, dtype=np.uint64).astype(np.uint32)
    x = u.view(np.float32)
    x = np.concatenate([x, np.array([-np.inf, np.inf, np.nan, 0.0, -0.0, 88.72, -103.97, -103.9, 88.7, -87.5],
                                    np.float32)])
    dx, dout = DeviceArray(cuda, x), DeviceArray(cuda, shape=x.shape, dtype=np.float32)
    call(cuda, "nc_expf_exact", [dout, dx], [x.size])
    assert same_bits(dout.numpy(), oracle.expf_libm(x))


def test_block_scale_division_is_ieee_for_every_float(cuda):
    import ctypes

    bad = ctypes.c_int64(-1)
    cuda.check(cuda.library().nc_selfcheck_div127(ctypes.byref(bad)))
    assert bad.value == 0


@pytest.mark.parametrize("rows,k", [(1, 896), (3, 4864), (7, 96), (2, 64)])
def test_quantize_blocks(cuda, rows, k):
    rng = np.random.default_rng(rows * k)
    x = activations(rng, rows, k)
    x[0, :32] = 0.0                                  # an all-zero block: scale 1
    x[-1, 32:36] = [0.5, -0.5, 1.5, -2.5]
    if k >= 96:                                      # quotients landing on half-integers
        x[0, 64:96] = np.arange(-16, 16, dtype=np.float32) + 0.5
        x[0, 64] = 127.0
    xq, xs, off, sums = oracle.quantize_blocks(x)
    dx = DeviceArray(cuda, x)
    dq = DeviceArray(cuda, shape=(rows, k), dtype=np.int8)
    dxs = DeviceArray(cuda, shape=(rows, k // 32), dtype=np.float32)
    doff = DeviceArray(cuda, shape=(rows,), dtype=np.float32)
    dsum = DeviceArray(cuda, shape=(rows, k // 32), dtype=np.int32)
    call(cuda, "nc_quantize_blocks", [dq, dx, dxs, doff, dsum], [rows, k])
    assert np.array_equal(dq.numpy(), xq) and np.array_equal(dsum.numpy(), sums)
    assert same_bits(dxs.numpy(), xs) and same_bits(doff.numpy(), off[:, 0])


@pytest.mark.parametrize("rows,n", [(1, 896), (4, 896), (3, 64)])
def test_rms_norm_quantize(cuda, rows, n):
    rng = np.random.default_rng(n + rows)
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    eps = 1e-6
    normed = oracle.rms_norm(x, w, eps)
    xq, xs, off, sums = oracle.quantize_blocks(normed)
    dx, dw = DeviceArray(cuda, x), DeviceArray(cuda, w)
    dn = DeviceArray(cuda, shape=(rows, n), dtype=np.float32)
    dq = DeviceArray(cuda, shape=(rows, n), dtype=np.int8)
    dxs = DeviceArray(cuda, shape=(rows, n // 32), dtype=np.float32)
    doff = DeviceArray(cuda, shape=(rows,), dtype=np.float32)
    dsum = DeviceArray(cuda, shape=(rows, n // 32), dtype=np.int32)
    call(cuda, "nc_rms_norm_quantize", [dn, dx, dw, dq, dxs, doff, dsum], [rows, n, f32_bits(eps)])
    assert same_bits(dn.numpy(), normed)
    assert np.array_equal(dq.numpy(), xq) and np.array_equal(dsum.numpy(), sums)
    assert same_bits(dxs.numpy(), xs) and same_bits(doff.numpy(), off[:, 0])


@pytest.mark.parametrize("k,n", [(896, 72), (4864, 24), (160, 40), (96, 24)])
@pytest.mark.parametrize("tokens", [1, 3, 7])
def test_matmul_i8_vnni_is_the_references_bitwise(cuda, k, n, tokens):
    """The reference's own outputs (tests/test_int8.py widths and inputs) from its generated C."""
    g = golden("proj")
    tag = f"k{k}_n{n}_t{tokens}"
    xq, xs, off = g[f"{tag}_xq"].reshape(tokens, k), g[f"{tag}_xs"].reshape(tokens, -1), g[f"{tag}_offset"].reshape(-1)
    dq, dxs, doff = DeviceArray(cuda, xq), DeviceArray(cuda, xs), DeviceArray(cuda, off)
    dw, ds = packed_int8(cuda, g[f"{tag}_q"]), DeviceArray(cuda, g[f"{tag}_scales"])
    dout = DeviceArray(cuda, shape=(tokens, n), dtype=np.float32)
    call(cuda, "nc_matmul_i8_vnni", [dout, dq, dxs, doff, dw, ds, None, None], [tokens, n, k, 0])
    assert same_bits(dout.numpy(), g[f"{tag}_y"])


@pytest.mark.parametrize("rows,n,k", [(1, 1152, 896), (1, 896, 4864), (5, 200, 896), (64, 96, 4864), (2, 64, 64)])
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_matmul_i8_vnni_epilogues(cuda, rows, n, k, epi):
    rng = np.random.default_rng(rows + n + k + epi)
    x = activations(rng, rows, k)
    xq, xs, off, _ = oracle.quantize_blocks(x)
    w1, s1 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w2, s2 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    y1 = oracle.matmul_i8_vnni(xq, xs, off, w1, s1)
    y2 = oracle.matmul_i8_vnni(xq, xs, off, w2, s2)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    res = rng.standard_normal((rows, n)).astype(np.float32)
    if epi == 1:
        expect, extra, extra2 = y1 + bias, DeviceArray(cuda, bias), None
    elif epi == 2:
        expect, extra, extra2 = res + y1, DeviceArray(cuda, res), None
    else:
        expect, extra, extra2 = oracle.swiglu(y1, y2), packed_int8(cuda, w2), DeviceArray(cuda, s2)
    dq, dxs, doff = DeviceArray(cuda, xq), DeviceArray(cuda, xs), DeviceArray(cuda, off[:, 0])
    dw, ds = packed_int8(cuda, w1), DeviceArray(cuda, s1)
    dout = DeviceArray(cuda, shape=(rows, n), dtype=np.float32)
    call(cuda, "nc_matmul_i8_vnni", [dout, dq, dxs, doff, dw, ds, extra, extra2], [rows, n, k, epi])
    assert same_bits(dout.numpy(), expect)


@pytest.mark.parametrize("rows,n,k,epi", [(1, 1152, 896, 1), (3, 896, 4864, 2), (2, 4864, 896, 3), (9, 100, 64, 0),
                                          (20, 300, 896, 1), (70, 257, 128, 2), (33, 129, 64, 0)])
def test_matmul_f32_in_order(cuda, rows, n, k, epi):
    rng = np.random.default_rng(n * k + rows)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    y = np.stack([oracle.lm_head(x[i], w) for i in range(rows)])
    bias = rng.standard_normal(n).astype(np.float32)
    res = rng.standard_normal((rows, n)).astype(np.float32)
    extra = None
    if epi == 0:
        expect = y
    elif epi == 1:
        expect, extra = y + bias, DeviceArray(cuda, bias)
    elif epi == 2:
        expect, extra = res + y, DeviceArray(cuda, res)
    else:
        y2 = np.stack([oracle.lm_head(x[i], w2) for i in range(rows)])
        expect, extra = oracle.swiglu(y, y2), DeviceArray(cuda, w2)
    dx, dw = DeviceArray(cuda, x), DeviceArray(cuda, w)
    dout = DeviceArray(cuda, shape=(rows, n), dtype=np.float32)
    call(cuda, "nc_matmul_f32", [dout, dx, dw, extra], [rows, n, k, epi])
    assert same_bits(dout.numpy(), expect)


@pytest.mark.parametrize("rows,vocab,hidden", [(1, 151936, 896), (3, 5000, 64), (64, 3000, 896), (17, 4099, 96),
                                               (40, 151936, 896), (100, 2500, 64)])
def test_lm_head_argmax(cuda, rows, vocab, hidden):
    rng = np.random.default_rng(vocab + rows)
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    if rows >= 3:
        embed[vocab - 7] = embed[11]                 # a tie: the first index wins
        x[1] = 0.0                                    # every logit +0: index 0 wins
    logits = np.stack([oracle.lm_head(x[i], embed) for i in range(rows)])
    tokens = [oracle.argmax(logits[i]) for i in range(rows)]
    assert all(t == int(np.argmax(logits[i])) for i, t in enumerate(tokens))
    dx, de = DeviceArray(cuda, x), DeviceArray(cuda, embed)
    dl = DeviceArray(cuda, shape=(rows, vocab), dtype=np.float32)
    dt = DeviceArray(cuda, shape=(rows,), dtype=np.int64)
    scratch = DeviceArray(cuda, shape=(cuda.library().nc_lm_head_scratch_bytes(rows, vocab),), dtype=np.uint8, fill=0)
    for _ in range(2):                                # the finish counter resets itself
        call(cuda, "nc_lm_head_argmax", [dl, dx, de, dt, scratch], [rows, vocab, hidden])
        assert same_bits(dl.numpy(), logits)
        assert list(dt.numpy()) == tokens


def test_lm_head_argmax_nan_is_the_maximum(cuda):
    rng = np.random.default_rng(5)
    vocab, hidden = 2000, 64
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    embed[1500, 3] = np.nan
    embed[1700, 0] = np.nan
    x = rng.standard_normal((1, hidden)).astype(np.float32)
    dx, de = DeviceArray(cuda, x), DeviceArray(cuda, embed)
    dt = DeviceArray(cuda, shape=(1,), dtype=np.int64)
    scratch = DeviceArray(cuda, shape=(cuda.library().nc_lm_head_scratch_bytes(1, vocab),), dtype=np.uint8, fill=0)
    call(cuda, "nc_lm_head_argmax", [None, dx, de, dt, scratch], [1, vocab, hidden])
    assert int(dt.numpy()[0]) == 1500 == int(np.argmax(oracle.lm_head(x[0], embed)))


def q8_head_tokens(cuda, x, embed):
    rows, hidden = x.shape
    vocab = embed.shape[0]
    dx, de = DeviceArray(cuda, x), DeviceArray(cuda, embed)
    dq = DeviceArray(cuda, shape=(vocab, hidden), dtype=np.int8)
    ds = DeviceArray(cuda, shape=(vocab,), dtype=np.float32)
    call(cuda, "nc_lm_head_q8_prepare", [de, dq, ds], [vocab, hidden])
    dt = DeviceArray(cuda, shape=(rows,), dtype=np.int64)
    scratch = DeviceArray(cuda, shape=(cuda.library().nc_lm_head_q8_scratch_bytes(rows, vocab),), dtype=np.uint8, fill=0)
    out = []
    for _ in range(2):                                # the finish counter resets itself
        call(cuda, "nc_lm_head_q8_argmax", [dx, de, dq, ds, dt, scratch], [rows, vocab, hidden])
        out.append([int(v) for v in dt.numpy()])
    assert out[0] == out[1]
    return out[0]


# The int8-prefiltered head: approximate logits from an int8 copy, exact logits for the rows the
# error bound keeps; the tokens must be np.argmax of the reference's float32 logits.
@pytest.mark.parametrize("rows,vocab,hidden", [(1, 151936, 896), (2, 5000, 128), (4, 20000, 896), (7, 3000, 1024),
                                               (16, 4099, 256)])
def test_q8_lm_head_tokens(cuda, rows, vocab, hidden):
    rng = np.random.default_rng(vocab + 3 * rows)
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    logits = np.stack([oracle.lm_head(x[i], embed) for i in range(rows)])
    if rows >= 2:
        best = int(np.argmax(logits[0]))
        embed[vocab - 5] = embed[best]                # an exact tie with the maximum: the first index wins
        embed[vocab - 9] = embed[best]
        embed[vocab - 9, 7] = np.nextafter(embed[best, 7], np.float32(1) if x[0, 7] > 0 else np.float32(-1))
        x[1] = 0.0                                    # every logit +0: index 0 wins
        logits = np.stack([oracle.lm_head(x[i], embed) for i in range(rows)])
    tokens = [oracle.argmax(logits[i]) for i in range(rows)]
    assert q8_head_tokens(cuda, x, embed) == tokens


def test_q8_lm_head_non_finite(cuda):
    rng = np.random.default_rng(11)
    vocab, hidden = 3000, 128
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, hidden)).astype(np.float32)
    embed[2100, 3] = np.nan                           # a NaN logit is np.argmax's answer
    embed[2500, 0] = np.inf
    x[2, 5] = np.inf                                  # every logit of row 2 is +-inf or NaN
    logits = np.stack([oracle.lm_head(x[i], embed) for i in range(3)])
    tokens = [oracle.argmax(logits[i]) for i in range(3)]
    assert tokens[0] == 2100
    assert q8_head_tokens(cuda, x, embed) == tokens


def rope_np(t1, cos, sin):
    half = t1.shape[-1] // 2
    rot = np.concatenate([-t1[..., half:], t1[..., :half]], -1)
    return (t1 * np.concatenate([cos, cos])) + (rot * np.concatenate([sin, sin]))


# Up to eight rows: one CTA per query head. More: the grouped kernel (bulk-copied K/V stages).
@pytest.mark.parametrize("rows,past,heads,kv,d", [(1, 0, 14, 2, 64), (1, 1024, 14, 2, 64), (3, 37, 4, 2, 16),
                                                  (2, 2048, 14, 2, 64), (12, 300, 14, 2, 64), (9, 0, 14, 2, 64),
                                                  (10, 127, 8, 1, 64), (16, 129, 4, 2, 16), (9, 2100, 14, 2, 64)])
@pytest.mark.parametrize("entry", ["nc_attention", "nc_attention_cache"])   # the second: K/V by TMA
def test_decode_attention(cuda, rows, past, heads, kv, d, entry):
    rng = np.random.default_rng(past + rows)
    cap = past + 37 * rows + 8
    n_qkv = (heads + 2 * kv) * d
    qkv = rng.standard_normal((rows, n_qkv)).astype(np.float32)
    cache = rng.standard_normal((rows, 2, kv, cap, d)).astype(np.float32)
    inv = (1.0 / (1e6 ** (np.arange(0, d, 2) / d))).astype(np.float32)
    pos = np.array([past + 37 * r for r in range(rows)], np.int32)   # one sequence per row, ragged lengths
    table_pos = np.arange(cap, dtype=np.float32)[:, None] * inv[None, :]
    cos, sin = oracle.cosf_libm(table_pos), oracle.sinf_libm(table_pos)
    slot = np.arange(rows, dtype=np.int32)
    scale = np.float32(d ** -0.5)
    dctx = DeviceArray(cuda, shape=(rows, heads * d), dtype=np.float32)
    dcache = DeviceArray(cuda, cache)
    call(cuda, entry, [dctx, DeviceArray(cuda, qkv), dcache, DeviceArray(cuda, cos), DeviceArray(cuda, sin),
                       DeviceArray(cuda, slot), DeviceArray(cuda, pos)],
         [rows, heads, kv, d, cap, 2 * kv * cap * d, 1, f32_bits(scale), rows])
    assert cuda.library().nc_device_faults() == 0
    got_ctx, got_cache = dctx.numpy(), dcache.numpy()
    for r in range(rows):
        p = pos[r]
        t = qkv[r].reshape(heads + 2 * kv, d)
        qr = rope_np(t[:heads], cos[p], sin[p])
        kr = rope_np(t[heads:heads + kv], cos[p], sin[p])
        vv = t[heads + kv:]
        keys, values = cache[r, 0].copy(), cache[r, 1].copy()
        keys[:, p], values[:, p] = kr, vv
        assert same_bits(got_cache[r, 0, :, p], kr) and same_bits(got_cache[r, 1, :, p], vv)
        out, _ = oracle.attention_decode(qr, keys, values, heads, kv, p + 1, scale)
        assert same_bits(got_ctx[r], out.reshape(-1))


@pytest.mark.parametrize("rows,heads,kv,d", [(3, 14, 2, 64), (11, 14, 2, 64), (12, 4, 2, 16)])
@pytest.mark.parametrize("entry", ["nc_attention", "nc_attention_cache"])
def test_attention_over_the_cache_only(cuda, rows, heads, kv, d, entry):
    """The prompt path's second pass (mode 2): every position, the row's own included, from the cache."""
    rng = np.random.default_rng(rows + d)
    cap = 64 * rows + 8
    qkv = rng.standard_normal((rows, (heads + 2 * kv) * d)).astype(np.float32)
    cache = rng.standard_normal((rows, 2, kv, cap, d)).astype(np.float32)
    inv = (1.0 / (1e6 ** (np.arange(0, d, 2) / d))).astype(np.float32)
    pos = np.array([61 * r + 5 for r in range(rows)], np.int32)
    table_pos = np.arange(cap, dtype=np.float32)[:, None] * inv[None, :]
    cos, sin = oracle.cosf_libm(table_pos), oracle.sinf_libm(table_pos)
    scale = np.float32(d ** -0.5)
    dctx = DeviceArray(cuda, shape=(rows, heads * d), dtype=np.float32)
    dcache = DeviceArray(cuda, cache)
    call(cuda, entry, [dctx, DeviceArray(cuda, qkv), dcache, DeviceArray(cuda, cos), DeviceArray(cuda, sin),
                       DeviceArray(cuda, np.arange(rows, dtype=np.int32)), DeviceArray(cuda, pos)],
         [rows, heads, kv, d, cap, 2 * kv * cap * d, 0, f32_bits(scale), rows])
    assert cuda.library().nc_device_faults() == 0
    got = dctx.numpy()
    assert same_bits(dcache.numpy(), cache)                          # nothing appended
    for r in range(rows):
        p = pos[r]
        qr = rope_np(qkv[r].reshape(heads + 2 * kv, d)[:heads], cos[p], sin[p])
        out, _ = oracle.attention_decode(qr, cache[r, 0], cache[r, 1], heads, kv, p + 1, scale)
        assert same_bits(got[r], out.reshape(-1))


def test_gather_reports_the_first_bad_row(cuda):
    table = np.arange(12, dtype=np.float32).reshape(4, 3)
    ids = np.array([1, 9, 2, -1], np.int64)
    dout = DeviceArray(cuda, shape=(4, 3), dtype=np.float32)
    err = DeviceArray(cuda, np.full(1, np.iinfo(np.uint64).max, np.uint64))
    call(cuda, "nc_gather_rows", [dout, DeviceArray(cuda, ids), DeviceArray(cuda, table), err], [4, 4, 3])
    assert int(err.numpy()[0]) == 1
    out = dout.numpy()
    assert np.array_equal(out[0], table[1]) and np.array_equal(out[2], table[2])


@pytest.mark.parametrize("packed", [0, 1])
def test_quantize_int8_rows_is_the_references(cuda, packed):
    """Device quantize_int8 (nanocompile/quantize.py:55-70): the reference's own bytes on its edge
    cases (tests/golden/proj.npz), and the host scheme's on rows built to hit each rounding step."""
    g = golden("proj")
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((300, 896)) * 0.02).astype(np.float32)
    w[7] = 0.0                                            # all zero: scale 1
    w[8] = np.float32(1e-44)                              # max / 127 underflows to 0: scale 1
    w[9, 0], w[9, 1:40] = 127.0, np.arange(39, dtype=np.float32) - 19.5       # exact half-integers at scale 1
    w[10, 0], w[10, 1] = 127.0, np.float32(0.5) - np.float32(2.0 ** -25)      # |v| + 0.5 rounds up to 1.0
    w[11] = np.float32(3e38) * np.sign(w[11])             # near the top of the float range
    cases = [(g["qi8_w"], g["qi8_values"], g["qi8_scales"]), (w, *q.quantize_int8(w))]
    for weights, values, scales in cases:
        rows, cols = weights.shape
        dw = DeviceArray(cuda, weights)
        dv = DeviceArray(cuda, shape=(rows, cols), dtype=np.uint8 if packed else np.int8)
        ds = DeviceArray(cuda, shape=(rows,), dtype=np.float32)
        call(cuda, "nc_quantize_int8_rows", [dv, ds, dw], [rows, cols, packed])
        expected = (values.astype(np.int16) + 128).astype(np.uint8) if packed else values
        assert np.array_equal(dv.numpy(), expected)
        assert np.array_equal(bits(ds.numpy()), bits(scales))


# -- the tensor-core int8 projection (tcgen05 kind::i8, block-diagonal activations) ---------------


def call_tc(cuda, out, xq, xs, off, w, s, extra=None, extra2=None, bsums=None, q_out=None, xs_out=None,
            bsums_out=None, sizes=()):
    call(cuda, "nc_matmul_i8_tc", [out, xq, xs, off, w, s, extra, extra2, bsums, q_out, xs_out, bsums_out],
         list(sizes))


@pytest.mark.parametrize("k,n", [(896, 72), (4864, 24), (160, 40), (96, 24)])
@pytest.mark.parametrize("tokens", [1, 3, 7])
@pytest.mark.parametrize("per_item", [0, 4])
def test_matmul_i8_tc_is_the_references_bitwise(cuda, k, n, tokens, per_item):
    """The reference's own projection outputs (tests/golden/proj.npz) through the tensor cores,
    including widths with 32-byte groups past the last whole 128-byte chunk (160, 96)."""
    g = golden("proj")
    tag = f"k{k}_n{n}_t{tokens}"
    xq, xs, off = g[f"{tag}_xq"].reshape(tokens, k), g[f"{tag}_xs"].reshape(tokens, -1), g[f"{tag}_offset"].reshape(-1)
    dq, dxs, doff = DeviceArray(cuda, xq), DeviceArray(cuda, xs), DeviceArray(cuda, off)
    dw, ds = packed_int8(cuda, g[f"{tag}_q"]), DeviceArray(cuda, g[f"{tag}_scales"])
    dout = DeviceArray(cuda, shape=(tokens, n), dtype=np.float32)
    call_tc(cuda, dout, dq, dxs, doff, dw, ds, sizes=[tokens, n, k, 0, 0, per_item])
    assert same_bits(dout.numpy(), g[f"{tag}_y"])


@pytest.mark.parametrize("rows,n,k", [(64, 1152, 896), (64, 896, 4864), (5, 200, 96), (67, 4864, 896),
                                      (16, 96, 160), (130, 256, 896)])
@pytest.mark.parametrize("epi,pro", [(0, 0), (1, 0), (2, 0), (2, 2), (3, 0), (4, 0), (0, 2)])
def test_matmul_i8_tc_epilogues_are_the_oracles(cuda, rows, n, k, epi, pro):
    """Every prologue / epilogue the model runtime uses, against the oracle, bit for bit: offsets
    given or formed from block sums; bias, residual, SiLU(gate) * up and its block quantization."""
    rng = np.random.default_rng(rows * 7 + n + k + epi * 3 + pro)
    x = activations(rng, rows, k)
    xq, xs, off, sums = oracle.quantize_blocks(x)
    w1, s1 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w2, s2 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w1[3] = 127                                         # extreme lanes: |Dp4| up to 4 * 255 * 127
    y1 = oracle.matmul_i8_vnni(xq, xs, off, w1, s1)
    y2 = oracle.matmul_i8_vnni(xq, xs, off, w2, s2)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    res = rng.standard_normal((rows, n)).astype(np.float32)
    extra = extra2 = None
    if epi == 0:
        expect = y1
    elif epi == 1:
        expect, extra = y1 + bias, DeviceArray(cuda, bias)
    elif epi == 2:
        expect, extra = res + y1, DeviceArray(cuda, res)
    else:
        expect, extra, extra2 = oracle.swiglu(y1, y2), packed_int8(cuda, w2), DeviceArray(cuda, s2)
    dq, dxs, doff, dsum = DeviceArray(cuda, xq), DeviceArray(cuda, xs), DeviceArray(cuda, off[:, 0]), DeviceArray(cuda, sums)
    dw, ds = packed_int8(cuda, w1), DeviceArray(cuda, s1)
    dout = DeviceArray(cuda, shape=(rows, n), dtype=np.float32, fill=0)
    outs = [None, None, None]
    if epi == 4:
        outs = [DeviceArray(cuda, shape=(rows, n), dtype=np.int8), DeviceArray(cuda, shape=(rows, max(n // 32, 1)), dtype=np.float32),
                DeviceArray(cuda, shape=(rows, max(n // 32, 1)), dtype=np.int32)]
    if epi == 4 and n % 32:                             # quantized outputs are whole 32-blocks
        with pytest.raises(cuda.InterpreterError, match="quantized output width"):
            call_tc(cuda, dout, dq, dxs, doff, dw, ds, extra, extra2, None, *outs, sizes=[rows, n, k, epi, pro, 4])
        return
    for per_item in (0, 4):
        call_tc(cuda, dout, dq, dxs, None if pro else doff, dw, ds, extra, extra2, dsum if pro else None, *outs,
                sizes=[rows, n, k, epi, pro, per_item])
        if epi == 4:
            hq, hxs, _, hsums = oracle.quantize_blocks(expect)
            assert np.array_equal(outs[0].numpy(), hq) and np.array_equal(outs[2].numpy(), hsums)
            assert same_bits(outs[1].numpy(), hxs)
        else:
            assert same_bits(dout.numpy(), expect)
        if epi == 2:
            extra.upload(res)                           # the residual is read in place: restore it


# -- int8 weights with float32 activations (matmul_i8) ---------------------------------------------


@pytest.mark.parametrize("k,n", [(896, 72), (4864, 24), (160, 40), (96, 24)])
@pytest.mark.parametrize("tokens", [1, 3, 7])
def test_matmul_i8_f32_is_the_references_bitwise(cuda, k, n, tokens):
    """The reference's own matmul_i8 outputs (tests/golden/int8_f32.npz, its generated C)."""
    g = golden("int8_f32")
    tag = f"k{k}_n{n}_t{tokens}"
    dout = DeviceArray(cuda, shape=(tokens, n), dtype=np.float32)
    call(cuda, "nc_matmul_i8_f32", [dout, DeviceArray(cuda, g[f"{tag}_x"]), packed_int8(cuda, g[f"{tag}_q"]),
                                    DeviceArray(cuda, g[f"{tag}_scales"]), None, None], [tokens, n, k, 0])
    assert same_bits(dout.numpy(), g[f"{tag}_y"])


@pytest.mark.parametrize("rows,n,k", [(1, 1152, 896), (3, 896, 4864), (5, 200, 144), (2, 4864, 896), (9, 64, 48)])
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_matmul_i8_f32_epilogues_are_the_oracles(cuda, rows, n, k, epi):
    """Bias, residual and SiLU(gate) * up, and widths with 8-element groups past the last block."""
    rng = np.random.default_rng(rows + n + k + epi)
    x = activations(rng, rows, k)
    w1, s1 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w2, s2 = q.quantize_int8((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    y1, y2 = oracle.matmul_i8(x, w1, s1), oracle.matmul_i8(x, w2, s2)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    res = rng.standard_normal((rows, n)).astype(np.float32)
    if epi == 1:
        expect, extra, extra2 = y1 + bias, DeviceArray(cuda, bias), None
    elif epi == 2:
        expect, extra, extra2 = res + y1, DeviceArray(cuda, res), None
    else:
        expect, extra, extra2 = oracle.swiglu(y1, y2), packed_int8(cuda, w2), DeviceArray(cuda, s2)
    dout = DeviceArray(cuda, shape=(rows, n), dtype=np.float32)
    call(cuda, "nc_matmul_i8_f32", [dout, DeviceArray(cuda, x), packed_int8(cuda, w1), DeviceArray(cuda, s1), extra,
                                    extra2], [rows, n, k, epi])
    assert same_bits(dout.numpy(), expect)
