"""CPU restatement of ttspipe's NF4 hot path - TEST INFRASTRUCTURE ONLY.

This module is the parity checker for the CUDA library in ``ttspipe_b200``.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` may import it; nothing on the product path does, and the product
path fails loudly instead of falling back here.

Everything is plain NumPy on bf16 *bit patterns* (uint16) so that every
rounding point is explicit; the functions with an ``f16`` switch take and
return fp16 bit patterns instead, with the same formulas and fp16 at every
rounding point (the reference's GPU dtype). Each function names the reference file:line whose
arithmetic it restates (paths relative to the ttspipe repository root).

Pinning: the restatement is checked against fixtures produced by running the
reference itself in the build container (``tests/golden/make_golden.py``: the
reference's own C++ CPU kernels ``app/engine/nf4cpu.py`` and its torch
attention ``app/engine/fastpath.py:133-174``). bitsandbytes and the fish-speech
fork are not vendored by the reference, so their parts (the NF4 quantiser, the
8-bit scale codebook, ``precompute_freqs_cis``) are restated from the
published algorithms; the kernels read all of those as data, so parity of the
GPU path does not depend on them matching bitsandbytes bit for bit.
"""

from __future__ import annotations

import math

import numpy as np

# --------------------------------------------------------------------------
# bf16 bit helpers
# --------------------------------------------------------------------------


def f32_to_bf16(a) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even) and return the uint16 bit patterns.

    Same rounding as the reference's `f2bf` (app/engine/nf4cpu.py:70-75) and
    torch's `.to(torch.bfloat16)`; NaN maps to the canonical quiet NaN.
    """
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r = r.copy()
        r[nan] = 0x7FC0
    return r


def bf16_to_f32(b) -> np.ndarray:
    """Widen bf16 bit patterns to fp32 (exact; app/engine/nf4cpu.py:63-68)."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf(a) -> np.ndarray:
    """fp32 -> bf16 -> fp32 (app/engine/nf4cpu.py:77)."""
    return bf16_to_f32(f32_to_bf16(a))


def f32_to_f16(a) -> np.ndarray:
    """Round fp32 to fp16 (nearest-even, overflow to infinity, as the
    reference's `f2h` = __float2half_rn) and return the uint16 bit patterns."""
    return np.ascontiguousarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_to_f32(b) -> np.ndarray:
    """Widen fp16 bit patterns to fp32 (exact)."""
    return np.ascontiguousarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def round_f16(a) -> np.ndarray:
    """fp32 -> fp16 -> fp32."""
    return f16_to_f32(f32_to_f16(a))


def act_to_f32(b, f16: bool = False) -> np.ndarray:
    """Widen bit patterns of the activation type (bf16, or fp16 if `f16`)."""
    return f16_to_f32(b) if f16 else bf16_to_f32(b)


def f32_to_act(a, f16: bool = False) -> np.ndarray:
    """Round fp32 to the activation type's bit patterns."""
    return f32_to_f16(a) if f16 else f32_to_bf16(a)


def round_act(a, f16: bool = False) -> np.ndarray:
    """fp32 -> activation type -> fp32."""
    return act_to_f32(f32_to_act(a, f16), f16)


# --------------------------------------------------------------------------
# the NF4 format (a1-a3)
# --------------------------------------------------------------------------

#: bitsandbytes' NF4 code points in index order (app/engine/nf4gemv.py:69-86).
NF4_CODE = np.array(
    [
        -1.0,
        -0.6961928009986877,
        -0.5250730514526367,
        -0.39491748809814453,
        -0.28444138169288635,
        -0.18477343022823334,
        -0.09105003625154495,
        0.0,
        0.07958029955625534,
        0.16093020141124725,
        0.24611230194568634,
        0.33791524171829224,
        0.44070982933044434,
        0.5626170039176941,
        0.7229568362236023,
        1.0,
    ],
    dtype=np.float32,
)


def nf4_quantize(w, blocksize: int = 64):
    """Blockwise NF4 quantisation, bitsandbytes-style (`quantize_4bit`).

    bitsandbytes is not vendored by the reference; this restates its published
    algorithm as the reference's own layout test pins it
    (tests/test_nf4gemv.py:69-92): per-block absmax over the row-major
    flattened weight, ratio = w * (1 / absmax) in fp32, nearest code point by
    the midpoints between consecutive codes (`bucketize`, right=False), two
    indices per byte with the HIGH nibble first. An all-zero block gets
    absmax 0 and every index maps to code 0.0 (index 7).

    Returns (packed uint8 [N, K/2], absmax fp32 [N*K/blocksize]).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % blocksize or (n * k) % 2:
        raise ValueError("in_features must be a multiple of the blocksize")
    blocks = w.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax > 0, np.float32(1.0) / absmax, np.float32(0.0)).astype(np.float32)
    ratio = (blocks * inv[:, None]).astype(np.float32)
    bounds = ((NF4_CODE[:-1] + NF4_CODE[1:]) / np.float32(2)).astype(np.float32)
    idx = np.searchsorted(bounds, ratio.reshape(-1), side="left").astype(np.uint8)
    zero_rows = np.repeat(absmax == 0, blocksize)
    idx[zero_rows] = 7
    packed = ((idx[0::2] << 4) | idx[1::2]).astype(np.uint8).reshape(n, k // 2)
    return packed, absmax


def nf4_unpack(packed) -> np.ndarray:
    """Code indices [N, K] from packed bytes (high nibble = even k)."""
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    n = p.shape[0]
    out = np.empty((n, p.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = p >> 4
    out[:, 1::2] = p & 15
    return out


def dynamic_code_map() -> np.ndarray:
    """A signed 256-entry "dynamic tree" scale codebook (bitsandbytes'
    `create_dynamic_map(signed=True)` as published: seven decades 1e-6..1e0,
    2**i fraction points per decade and sign, plus 0 and 1, sorted).

    bitsandbytes is absent, so this is a restatement; the kernels read the
    table as data (`state2.code`, app/engine/nf4gemv.py:360-362).
    """
    vals = []
    for i in range(7):
        bounds = np.linspace(0.1, 1.0, 2**i + 1)
        means = (bounds[:-1] + bounds[1:]) / 2.0
        scale = 10.0 ** (i - 6)
        vals.extend((scale * means).tolist())
        vals.extend((-scale * means).tolist())
    vals.extend([0.0, 1.0])
    vals = sorted(vals + [0.0] * (256 - len(vals)))
    return np.asarray(vals, dtype=np.float32)


def double_quantize(absmax, blocksize2: int = 256, code2=None):
    """Second-level quantisation of the fp32 absmax (bitsandbytes'
    `compress_statistics=True`): offset = mean(absmax); the centred values are
    quantised blockwise (blocksize2) to the nearest entry of `code2`, with an
    fp32 absmax2 per block.

    Returns (a8 uint8 [nb], absmax2 fp32 [ceil(nb/blocksize2)], code2, offset).
    """
    if code2 is None:
        code2 = dynamic_code_map()
    absmax = np.ascontiguousarray(absmax, dtype=np.float32)
    offset = np.float32(absmax.astype(np.float64).mean())
    v = (absmax - offset).astype(np.float32)
    nb = v.size
    nb2 = -(-nb // blocksize2)
    pad = np.zeros(nb2 * blocksize2, dtype=np.float32)
    pad[:nb] = v
    blocks = pad.reshape(nb2, blocksize2)
    absmax2 = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax2 > 0, np.float32(1.0) / absmax2, np.float32(0.0)).astype(np.float32)
    ratio = (blocks * inv[:, None]).astype(np.float32).reshape(-1)[:nb]
    mids = ((code2[:-1].astype(np.float64) + code2[1:].astype(np.float64)) / 2.0)
    a8 = np.searchsorted(mids, ratio.astype(np.float64), side="left").astype(np.uint8)
    return a8, absmax2, code2.astype(np.float32), offset


def nested_scales(a8, absmax2, code2, offset, blocksize2: int = 256) -> np.ndarray:
    """absmax[b] = code2[a8[b]] * absmax2[b // blocksize2] + offset, as two
    separately rounded fp32 operations (app/engine/nf4gemv.py:160-161; the
    equality with bitsandbytes' own reconstruction is
    tests/test_nf4gemv.py:95-116)."""
    a8 = np.asarray(a8, dtype=np.int64)
    b = np.arange(a8.size) // blocksize2
    prod = (code2[a8].astype(np.float32) * absmax2[b].astype(np.float32)).astype(np.float32)
    return (prod + np.float32(offset)).astype(np.float32)


def dequantize_bf16(packed, scales, blocksize: int = 64) -> np.ndarray:
    """Dequantised weight as bf16 bits [N, K]: RNE_bf16(NF4[q] * scale) with the
    product in fp32 - what bitsandbytes' `dequantize_4bit` does before its
    GEMM, and the per-element value the reference GPU kernel rounds to its
    compute dtype (app/engine/nf4gemv.py:185-188, bf16 here instead of fp16).
    """
    q = nf4_unpack(packed)
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float32).reshape(n, k // blocksize)
    vals = (NF4_CODE[q].reshape(n, k // blocksize, blocksize) * s[:, :, None]).astype(np.float32)
    return f32_to_bf16(vals.reshape(n, k))


def dequantize_f16(packed, scales, blocksize: int = 64) -> np.ndarray:
    """Dequantised weight as fp16 bits [N, K]: RNE_f16(NF4[q] * scale), the
    per-element value of the reference GPU kernel's A fragments
    (app/engine/nf4gemv.py:185-188, `pack2` of the fp32 products)."""
    q = nf4_unpack(packed)
    n, k = q.shape
    s = np.asarray(scales, dtype=np.float32).reshape(n, k // blocksize)
    vals = (NF4_CODE[q].reshape(n, k // blocksize, blocksize) * s[:, :, None]).astype(np.float32)
    return f32_to_f16(vals.reshape(n, k))


# --------------------------------------------------------------------------
# matmul with the fused epilogues (a4-a7)
# --------------------------------------------------------------------------

EPI_NONE, EPI_RESIDUAL, EPI_SILU_GATE = 0, 1, 2


def silu_bf16(a_bits, f16: bool = False) -> np.ndarray:
    """bf16(silu(a)) with the division done in fp32 (app/engine/nf4gemv.py:224-226,
    app/engine/nf4cpu.py:249-251); fp16 in and out if `f16`."""
    a = act_to_f32(a_bits, f16)
    with np.errstate(over="ignore"):
        s = (a / (np.float32(1.0) + np.exp(-a).astype(np.float32))).astype(np.float32)
    return f32_to_act(s, f16)


def epilogue(acc, epi: int = EPI_NONE, operand=None, f16: bool = False) -> np.ndarray:
    """The matmul's store: its own output rounded to the activation type
    first, then each fused elementwise op rounded where the fork rounds it
    (app/engine/nf4gemv.py:212-228, which is this with f16)."""
    y = round_act(np.asarray(acc, dtype=np.float32), f16)
    if epi == EPI_NONE:
        return f32_to_act(y, f16)
    r = np.asarray(operand, dtype=np.uint16).reshape(y.shape)
    with np.errstate(over="ignore", invalid="ignore"):
        if epi == EPI_RESIDUAL:
            return f32_to_act((act_to_f32(r, f16) + y).astype(np.float32), f16)
        if epi == EPI_SILU_GATE:
            return f32_to_act((act_to_f32(silu_bf16(r, f16), f16) * y).astype(np.float32), f16)
    raise ValueError(f"unknown epilogue {epi}")


def matmul_exact(x_bits, w_bits, f16: bool = False) -> np.ndarray:
    """X @ Wᵀ of bf16 (fp16 if `f16`) inputs, accumulated in fp64 and NOT
    rounded: the value a kernel with outputs of that type approximates (its
    error = accumulation + its own final rounding, at most half an ulp when
    the accumulation is exact)."""
    x = act_to_f32(x_bits, f16).astype(np.float64)
    w = act_to_f32(w_bits, f16).astype(np.float64)
    return x.reshape(-1, w.shape[1]) @ w.T


def matmul_dequant(x_bits, w_bits, epi: int = EPI_NONE, operand=None, f16: bool = False) -> np.ndarray:
    """Y = X @ Wᵀ from the dequantised weight, accumulated exactly (fp64)
    and rounded once: the reference's "dequantise then matmul"
    (app/engine/nf4gemv.py:36-41; tests/test_nf4gemv.py:119-141)."""
    acc = matmul_exact(x_bits, w_bits, f16)
    return epilogue(acc.astype(np.float32), epi, operand, f16)


def nf4cpu_gemv(x_bits, packed, absmax_bf16_bits, code_bf16_bits) -> np.ndarray:
    """The reference CPU kernel's factorisation (app/engine/nf4cpu.py:104-131):
    per 64-block dot of the bf16 code values with x, then times the block's
    bf16 absmax, summed in fp32; output rounded to bf16. Sum order differs
    from the AVX-512 kernel, so this agrees with it to rounding only."""
    x = bf16_to_f32(x_bits).reshape(-1, packed.shape[1] * 2).astype(np.float64)
    q = nf4_unpack(packed)
    n, k = q.shape
    code = bf16_to_f32(code_bf16_bits).astype(np.float64)
    cv = code[q].reshape(n, k // 64, 64)
    am = bf16_to_f32(absmax_bf16_bits).reshape(n, k // 64).astype(np.float64)
    xb = x.reshape(x.shape[0], k // 64, 64)
    part = np.einsum("nbk,mbk->mnb", cv, xb)
    return f32_to_bf16((part * am[None]).sum(-1).astype(np.float32))


# --------------------------------------------------------------------------
# norms, rotary, attention (a8-a10)
# --------------------------------------------------------------------------


def rms_norm(x_bits, w_bits, eps: float, f16: bool = False) -> np.ndarray:
    """The fork's RMSNorm in bf16: y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)
    (fork formula app/engine/fusedops.py:9-13; bf16 rounding points as
    app/engine/nf4cpu.py:456-461; with `f16`, fp16 at both points as the
    reference kernel app/engine/fusedops.py:61-95). The sum of squares is
    exact (fp64); the reciprocal square root is correctly rounded fp32."""
    x = act_to_f32(x_bits, f16)
    d = x.shape[-1]
    xf = x.reshape(-1, d)
    ms = (xf.astype(np.float64) ** 2).sum(-1) / d
    t = (ms.astype(np.float32) + np.float32(eps)).astype(np.float32)
    r = (1.0 / np.sqrt(t.astype(np.float64))).astype(np.float32)
    y1 = round_act((xf * r[:, None]).astype(np.float32), f16)
    w = act_to_f32(w_bits, f16)
    return f32_to_act((y1 * w[None, :]).astype(np.float32), f16).reshape(np.shape(x_bits))


def head_rms_norm(x_f32, w_bits, eps: float, f16: bool = False) -> np.ndarray:
    """Per-head q/k RMSNorm over head_dim with ONE rounding of x*r*w, as both
    reference kernels do it (app/engine/fusedlayer.py:74-84,
    app/engine/nf4cpu.py:501-510). Input fp32 [..., D] (already bf16 values,
    fp16 with `f16`); returns fp32 values exact in that type."""
    x = np.asarray(x_f32, dtype=np.float32)
    d = x.shape[-1]
    ss = (x.astype(np.float64) ** 2).sum(-1, keepdims=True)
    t = ((ss / d).astype(np.float32) + np.float32(eps)).astype(np.float32)
    r = (1.0 / np.sqrt(t.astype(np.float64))).astype(np.float32)
    w = act_to_f32(w_bits, f16)
    return round_act(((x * r).astype(np.float32) * w).astype(np.float32), f16)


def rope(x_bits, freqs, f16: bool = False) -> np.ndarray:
    """Interleaved-pair rotary: (x0*c - x1*s, x1*c + x0*s), each product and the
    sum rounded in fp32 (no FMA contraction), then bf16 (fp16 with `f16`)
    (app/engine/fusedops.py:103-132; pairs (2i, 2i+1), freqs (S, D/2, 2)).

    x: bf16 bits (B, S, H, D); freqs: float array (S, D/2, 2) of fp32 values.
    """
    x = act_to_f32(x_bits, f16)
    b, s, h, d = x.shape
    f = np.asarray(freqs, dtype=np.float32).reshape(s, d // 2, 2)
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    c = f[None, :, None, :, 0]
    sn = f[None, :, None, :, 1]
    y0 = ((x0 * c).astype(np.float32) - (x1 * sn).astype(np.float32)).astype(np.float32)
    y1 = ((x1 * c).astype(np.float32) + (x0 * sn).astype(np.float32)).astype(np.float32)
    out = np.empty_like(x)
    out[..., 0::2] = y0
    out[..., 1::2] = y1
    return f32_to_act(out, f16)


def precompute_freqs_cis(seq_len: int, n_elem: int, base: float = 1e6) -> np.ndarray:
    """(seq_len, n_elem/2, 2) = (cos, sin) of t * base^(-2i/n), as bf16 bits.

    The fork's `precompute_freqs_cis` is not vendored by the reference; this
    is the standard definition it implements (layout (S, D/2, 2) stored bf16,
    app/engine/fusedops.py:96-101, app/engine/nf4cpu.py:518-520). Kernels take
    the table as data."""
    i = np.arange(0, n_elem, 2)[: n_elem // 2].astype(np.float32)
    inv = (np.float32(1.0) / (np.float32(base) ** (i / np.float32(n_elem)))).astype(np.float32)
    t = np.arange(seq_len, dtype=np.float32)
    ang = np.outer(t, inv).astype(np.float32)
    cache = np.stack([np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))], -1)
    return f32_to_bf16(cache.astype(np.float32))


def attention(q_bits, k_cache_bits, v_cache_bits, length: int, n_head: int, n_kv: int,
              f16: bool = False) -> np.ndarray:
    """Grouped decode attention of ONE query position over keys [0, length).

    Follows the fork's rounding points as `decode_attention`
    (app/engine/fastpath.py:133-174) and the CPU kernel
    (app/engine/nf4cpu.py:547-601): score = bf16(q.k) * D^-0.5 in fp32,
    softmax in fp32 (exact sum), probabilities rounded to bf16, output
    sum(p * v) rounded to bf16. Query head h reads KV head h // (n_head/n_kv).

    q: bf16 bits [n_head, D]; caches: bf16 bits [n_kv, max_len, D].
    Returns bf16 bits [n_head, D]. With `f16` every bf16 above is fp16.
    """
    q = act_to_f32(q_bits, f16).reshape(n_head, -1).astype(np.float64)
    kc = act_to_f32(k_cache_bits, f16)
    vc = act_to_f32(v_cache_bits, f16)
    d = q.shape[1]
    groups = n_head // n_kv
    scale = np.float32(1.0 / math.sqrt(d))
    out = np.empty((n_head, d), dtype=np.float32)
    for h in range(n_head):
        kh = h // groups
        k = kc[kh, :length].astype(np.float64)
        v = vc[kh, :length].astype(np.float64)
        sc = (round_act((k @ q[h]).astype(np.float32), f16) * scale).astype(np.float32)
        mx = sc.max()
        e = np.exp((sc - mx).astype(np.float64))
        p = round_act((e / e.sum()).astype(np.float32), f16).astype(np.float64)
        out[h] = (p @ v).astype(np.float32)
    return f32_to_act(out, f16)


def attention_masked(q_bits, k_bits, v_bits, mask, n_head: int, n_kv: int, f16: bool = False) -> np.ndarray:
    """`attention` for S query rows under an explicit visibility mask.

    q: bf16 bits [n_head, S, D]; k/v: [n_kv, L, D]; mask: bool [S, L] (True =
    visible), the (B, 1, S, L) mask of app/engine/fastpath.py:152-166 without
    its unit axes. Masked keys are never read. Returns bf16 bits [n_head, S, D]
    (fp16 throughout with `f16`).
    """
    q = act_to_f32(q_bits, f16).astype(np.float64)
    kc = act_to_f32(k_bits, f16).astype(np.float64)
    vc = act_to_f32(v_bits, f16).astype(np.float64)
    nh, S, d = q.shape
    groups = n_head // n_kv
    scale = np.float32(1.0 / math.sqrt(d))
    mask = np.asarray(mask, dtype=bool).reshape(S, -1)
    out = np.zeros((nh, S, d), dtype=np.float32)
    for h in range(nh):
        kh = h // groups
        for s in range(S):
            vis = np.nonzero(mask[s])[0]
            if vis.size == 0:
                out[h, s] = np.nan
                continue
            sc = (round_act((kc[kh, vis] @ q[h, s]).astype(np.float32), f16) * scale).astype(np.float32)
            e = np.exp((sc - sc.max()).astype(np.float64))
            p = round_act((e / e.sum()).astype(np.float32), f16).astype(np.float64)
            out[h, s] = (p @ vc[kh, vis]).astype(np.float32)
    return f32_to_act(out, f16)


# --------------------------------------------------------------------------
# one decode position through a transformer block (a11)
# --------------------------------------------------------------------------


def decode_block(x_bits, weights: dict, k_cache_bits, v_cache_bits, pos: int, freqs_row,
                 n_head: int, n_kv: int, head_dim: int, eps: float, qk_eps: float | None,
                 length: int | None = None, f16: bool = False):
    """`TransformerBlock.forward` for one position with the fork's rounding
    points, in the order of app/engine/fusedlayer.py:212-269 and
    app/engine/nf4cpu.py:479-617:

        xn = rms_norm(x); qkv = xn @ Wqkvᵀ; [qk-norm]; rope(q, k); cache[pos] = k, v
        a = attention(q, keys [0, length)); h = x + a @ Woᵀ
        hn = rms_norm(h); g = silu(hn @ W1ᵀ) * (hn @ W3ᵀ); out = h + g @ W2ᵀ

    `weights` holds dequantised bf16 bits for "wqkv", "wo", "w1", "w3", "w2",
    norm weights "attn_norm", "ffn_norm" and optional "q_norm", "k_norm".
    Caches are modified in place. Returns bf16 bits of the block output; with
    `f16` every bf16 here (weights, norms, caches, output) is fp16.
    """
    length = pos + 1 if length is None else length
    qs, kvs = n_head * head_dim, n_kv * head_dim
    xn = rms_norm(x_bits.reshape(1, -1), weights["attn_norm"], eps, f16)
    qkv = act_to_f32(matmul_dequant(xn, weights["wqkv"], f16=f16), f16)[0]
    q = qkv[:qs].reshape(n_head, head_dim)
    k = qkv[qs:qs + kvs].reshape(n_kv, head_dim)
    v = qkv[qs + kvs:].reshape(n_kv, head_dim)
    if weights.get("q_norm") is not None:
        q = head_rms_norm(q, weights["q_norm"], qk_eps, f16)
        k = head_rms_norm(k, weights["k_norm"], qk_eps, f16)
    f = np.asarray(freqs_row, dtype=np.float32).reshape(1, head_dim // 2, 2)
    qr = rope(f32_to_act(q, f16).reshape(1, 1, n_head, head_dim), f, f16).reshape(n_head, head_dim)
    kr = rope(f32_to_act(k, f16).reshape(1, 1, n_kv, head_dim), f, f16).reshape(n_kv, head_dim)
    k_cache_bits[:, pos] = kr
    v_cache_bits[:, pos] = f32_to_act(v, f16)
    att = attention(qr, k_cache_bits, v_cache_bits, length, n_head, n_kv, f16).reshape(1, qs)
    h = matmul_dequant(att, weights["wo"], EPI_RESIDUAL, x_bits.reshape(1, -1), f16)
    hn = rms_norm(h, weights["ffn_norm"], eps, f16)
    g1 = matmul_dequant(hn, weights["w1"], f16=f16)
    g = matmul_dequant(hn, weights["w3"], EPI_SILU_GATE, g1, f16)
    return matmul_dequant(g, weights["w2"], EPI_RESIDUAL, h, f16)


# --------------------------------------------------------------------------
# tolerance metrics used by the reference's tests
# --------------------------------------------------------------------------


# --------------------------------------------------------------------------
# output heads and sampling (the frame's tail)
# --------------------------------------------------------------------------


def dense_gemv_exact(x_bits, w_bits) -> np.ndarray:
    """x W^T of a bf16 row and a dense bf16 weight [N, K] in fp64, unrounded:
    the fork's bf16 output heads (app/engine/graphs.py:205-217 replays them)."""
    x = bf16_to_f32(np.asarray(x_bits).reshape(-1)).astype(np.float64)
    w = bf16_to_f32(w_bits).astype(np.float64)
    return w @ x


_MASK64 = (1 << 64) - 1


def splitmix64(z: int) -> int:
    """The counter-based hash the device sampler draws its uniform from."""
    z = (z + 0x9E3779B97F4A7C15) & _MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
    return z ^ (z >> 31)


def sample_uniform(seed: int, step: int) -> float:
    """u in [0, 1) for (seed, step), 24 bits, as the device computes it."""
    h = splitmix64((seed ^ ((step * 0xD1B54A32D192ED03) & _MASK64)) & _MASK64)
    return float(np.float32((h >> 40) * (1.0 / 16777216.0)))


def sample_token(logit_bits, temperature: float, top_p: float, top_k: int, seed: int, step: int):
    """The fork's sampler as the reference calls it (app/engine/graphs.py:55-73):
    sort descending (ties: smaller index first); p = softmax of the sorted,
    unscaled logits over the WHOLE vocabulary; drop position i if
    cumsum(p)[i] > top_p or i >= top_k, never i = 0; divide the kept logits by
    max(temperature, 1e-5); softmax; one inverse-CDF draw with
    sample_uniform(seed, step). Returns (token, kept ids, their probabilities).
    """
    v = bf16_to_f32(np.asarray(logit_bits).reshape(-1)).astype(np.float64)
    order = np.lexsort((np.arange(v.size), -v))
    sv = v[order]
    p = np.exp(sv - sv[0])
    p /= p.sum()
    cum = np.cumsum(p)
    k = max(1, min(int(top_k), 64, v.size))
    keep = 1
    for i in range(1, k):
        if cum[i] > top_p:
            break
        keep = i + 1
    z = sv[:keep] / max(float(temperature), 1e-5)
    q = np.exp(z - z[0])
    q /= q.sum()
    u = sample_uniform(seed, step)
    pick = int(np.searchsorted(np.cumsum(q), u, side="right"))
    pick = min(pick, keep - 1)
    return int(order[pick]), order[:keep].copy(), q


def relative_error(got, ref) -> float:
    """max|got - ref| / max|ref| (tests/test_nf4gemv.py:59-62)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6))


def norm_relative_error(got, ref) -> float:
    """||got - ref|| / ||ref|| (tests/test_nf4cpu.py:56-57)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def rms_relative_max_error(got, ref) -> float:
    """max|got - ref| / rms(ref): the north-star bar for GEMV/GEMM outputs
    (max abs error <= 2e-2 relative to output RMS)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = math.sqrt(float((ref ** 2).mean())) if ref.size else 0.0
    return float(np.abs(got - ref).max() / max(rms, 1e-30)) if ref.size else 0.0
