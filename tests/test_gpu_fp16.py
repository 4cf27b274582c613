"""fp16 activations: the reference's own GPU dtype (B200 only).

The reference's kernels serve fp16 only (app/engine/nf4gemv.py:439,
app/engine/fusedops.py:176,206, app/engine/fusedlayer.py:198) and its
deployment default is fp16 (TTS_HALF, app/config.py:107). Every kernel here is
also instantiated for fp16 and checked against the oracle's fp16 restatement
(`f16=True`: the same formulas with fp16 at every rounding point):

* matmul: the register-fed decode GEMV (1..8 rows) and the tcgen05 GEMM
  (every other row count) against the exactly accumulated product of the
  bit-exact fp16 dequantised weight - max|err| <= 2e-2 x RMS and
  norm-relative < 5e-3, the bars of the bf16 tests; the fused epilogues bit
  for bit against the oracle's fp16 epilogue of the kernel's own output;
* RMSNorm, rotary and the q/k norm + rotary + KV write: bit-exact;
* decode attention: max-relative 5e-3, the reference's own fp16 bar
  (tests/test_nf4gemv.py:224-242);
* the decode block: against the oracle block in fp16;
* against the reference's own fp16 kernel nf4_mma, compiled from its source
  (oracle/build_ref.py), on identical inputs, where that library was built.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import make_linear, oracle_scales, to_bits
from ttspipe_b200 import _lib, fastpath, fusedlayer, fusedops, model, nf4gemv

pytestmark = pytest.mark.gpu

GEMM_TOL = 2e-2
ATTN_TOL = 5e-3
BLOCK_TOL = 1e-2
F16 = torch.float16


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install() and fusedops.install() and fusedlayer.install()


def randn_f16(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(F16).cuda()


def dequant_f16(layer):
    qs = layer.weight.quant_state
    return orc.dequantize_f16(layer.weight.data.cpu().numpy(), oracle_scales(qs), int(qs.blocksize))


def f32(t):
    return orc.f16_to_f32(to_bits(t))


def check_matmul_f16(got, x, layer):
    assert got.dtype == F16
    w = orc.matmul_exact(to_bits(x).reshape(-1, layer.in_features), dequant_f16(layer), f16=True)
    g = f32(got).reshape(w.shape)
    assert np.isfinite(g).all()
    assert orc.rms_relative_max_error(g, w) <= GEMM_TOL
    assert orc.norm_relative_error(g, w) < 5e-3


@pytest.mark.parametrize("shape", [(4096, 2560), (9728, 2560), (2560, 9728), (1024, 2560)])
@pytest.mark.parametrize("rows", [1, 2, 3, 8, 32, 64, 256])
def test_matmul_rows(shape, rows):
    n, k = shape
    layer = make_linear(n, k, seed=n + k + rows)
    x = randn_f16((rows, k), seed=rows * 7 + k)
    before = nf4gemv.stats()["fallback"]
    y = layer(x)   # the installed forward: served, not handed back
    assert nf4gemv.stats()["fallback"] == before
    check_matmul_f16(y, x, layer)


@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("rows", [1, 2, 5])
def test_plain_and_nested_scales_and_ragged_rows(nested, rows):
    layer = make_linear(200, 512, seed=3 + rows, nested=nested)
    x = randn_f16((rows, 512), seed=rows)
    check_matmul_f16(nf4gemv.matmul(layer, x), x, layer)


@pytest.mark.parametrize("rows", [1, 2, 7, 32, 300])
@pytest.mark.parametrize("epi", [nf4gemv.EPI_RESIDUAL, nf4gemv.EPI_SILU_GATE])
def test_fused_epilogues(epi, rows):
    """The fused store equals the oracle's fp16 epilogue of the kernel's own
    un-fused output: bit for bit for the residual add; the gate's exponential
    may differ from NumPy's by an fp32 ulp (a rare fp16 ulp)."""
    layer = make_linear(2560, 9728, seed=11 + rows)
    x = randn_f16((rows, 9728), seed=5000 + rows)
    operand = randn_f16((rows, 2560), seed=7919 + rows)
    y0 = nf4gemv.matmul(layer, x)
    y = nf4gemv.matmul(layer, x, epi=epi, operand=operand)
    check_matmul_f16(y0, x, layer)
    want = orc.epilogue(f32(y0), epi, to_bits(operand), f16=True)
    got = to_bits(y)
    if epi == nf4gemv.EPI_RESIDUAL:
        assert np.array_equal(got, want)
    else:
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3


def _ulp16(v):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -14))) - 10)


@pytest.mark.parametrize("rows", [1, 2, 5])
@pytest.mark.parametrize("nested", [True, False])
def test_gated_pair(rows, nested):
    """silu(x W1) * (x W3) in one launch: within the gate of the separate
    fp16 products, each allowed one ulp (the launch splits the sums its own
    way), widened by one ulp for silu's exponential."""
    w1 = make_linear(9728, 2560, seed=21, nested=nested)
    w3 = make_linear(9728, 2560, seed=22, nested=nested)
    x = randn_f16((rows, 2560), seed=23 + rows)
    got = f32(nf4gemv.matmul_gated(w1, w3, x)).astype(np.float64)
    y1, y3 = f32(nf4gemv.matmul(w1, x)), f32(nf4gemv.matmul(w3, x))
    cands = []
    for a in (y1 - _ulp16(y1), y1, y1 + _ulp16(y1)):
        for b in (y3 - _ulp16(y3), y3, y3 + _ulp16(y3)):
            out = orc.epilogue(b.astype(np.float32), orc.EPI_SILU_GATE, orc.f32_to_f16(a.astype(np.float32)),
                               f16=True)
            cands.append(orc.f16_to_f32(out).astype(np.float64))
    cands = np.stack(cands)
    lo, hi = cands.min(0), cands.max(0)
    lo, hi = lo - _ulp16(lo), hi + _ulp16(hi)
    got = got.reshape(lo.shape)
    assert np.all((got >= lo) & (got <= hi))


@pytest.mark.parametrize("rows", [1, 2, 3, 8])
def test_fused_norm_equals_norm_then_matmul(rows):
    lin = make_linear(6144, 2560, seed=31 + rows)
    g = torch.Generator().manual_seed(rows)
    nw = (1.0 + 0.1 * torch.randn(2560, generator=g)).to(F16).cuda()
    x = randn_f16((rows, 2560), seed=33 + rows, std=3.0)
    want = nf4gemv.matmul(lin, fusedops.rms_norm(x, nw, 1e-6))
    got = nf4gemv.matmul(lin, x, norm=(nw, 1e-6))
    assert got is not None and torch.equal(got, want)
    # beyond the register-fed GEMV's rows a fused norm is declined, not run in bf16
    assert nf4gemv.matmul(lin, randn_f16((9, 2560), seed=1), norm=(nw, 1e-6)) is None


@pytest.mark.parametrize("rows,width", [(1, 2560), (32, 128), (3, 2560), (1, 40)])
def test_rms_norm_is_bit_exact(rows, width):
    x = randn_f16((1, rows, width), seed=rows * 1000 + width)
    g = torch.Generator().manual_seed(width)
    w = (1.0 + 0.1 * torch.randn(width, generator=g)).to(F16).cuda()
    y = fusedops.rms_norm(x, w, 1e-6)
    want = orc.rms_norm(to_bits(x).reshape(rows, width), to_bits(w), 1e-6, f16=True)
    assert y.dtype == F16 and np.array_equal(to_bits(y).reshape(rows, width), want)
    assert fusedops.rms_norm(x, w.to(torch.bfloat16), 1e-6) is None   # mixed types are declined


@pytest.mark.parametrize("fdtype", [torch.bfloat16, torch.float32, torch.float16])
def test_rope_is_bit_exact(fdtype):
    x = randn_f16((1, 4, 32, 128), seed=9)
    f = torch.randn(4, 64, 2, generator=torch.Generator().manual_seed(4)).to(fdtype).cuda()
    y = fusedops.rope(x, f)
    assert np.array_equal(to_bits(y), orc.rope(to_bits(x), f.float().cpu().numpy(), f16=True))


def _qk_rope_kv(qkv, qw, kw, freqs, ftype, p, k, v, nh, nkv, max_len):
    q = torch.empty(nh * 128, dtype=F16, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib().nf4b_qk_rope_kv_ex(
        qkv.data_ptr(), None if qw is None else qw.data_ptr(), None if kw is None else kw.data_ptr(), 1e-6,
        freqs.data_ptr(), ftype, p.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), nh, nkv, 128, max_len,
        _lib.NF4B_F16, st))
    return q


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qk_rope_kv_is_bit_exact(qk_norm):
    nh, nkv, max_len, pos = 32, 8, 64, 17
    qkv = randn_f16(((nh + 2 * nkv) * 128,), seed=41)
    k, v = randn_f16((nkv, max_len, 128), seed=42), randn_f16((nkv, max_len, 128), seed=43)
    k0, v0 = to_bits(k), to_bits(v)
    freqs = model.precompute_freqs_cis(max_len, 128, 1e6, device="cuda")[pos:pos + 1].contiguous()
    g = torch.Generator().manual_seed(5)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(F16).cuda() if qk_norm else None
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(F16).cuda() if qk_norm else None
    p = torch.tensor([pos], dtype=torch.long, device="cuda")
    q = _qk_rope_kv(qkv, qw, kw, freqs, _lib.NF4B_BF16, p, k, v, nh, nkv, max_len)
    torch.cuda.synchronize()
    x = f32(qkv).reshape(nh + 2 * nkv, 128)
    qx, kx = x[:nh], x[nh:nh + nkv]
    if qk_norm:
        qx = orc.head_rms_norm(qx, to_bits(qw), 1e-6, f16=True)
        kx = orc.head_rms_norm(kx, to_bits(kw), 1e-6, f16=True)
    fr = orc.bf16_to_f32(to_bits(freqs)).reshape(1, 64, 2)
    want_q = orc.rope(orc.f32_to_f16(qx).reshape(1, 1, nh, 128), fr, f16=True).reshape(nh, 128)
    want_k = orc.rope(orc.f32_to_f16(kx).reshape(1, 1, nkv, 128), fr, f16=True).reshape(nkv, 128)
    assert np.array_equal(to_bits(q).reshape(nh, 128), want_q)
    gk, gv = to_bits(k), to_bits(v)
    assert np.array_equal(gk[:, pos], want_k)
    assert np.array_equal(gv[:, pos], to_bits(qkv).reshape(-1, 128)[nh + nkv:])
    others = [i for i in range(max_len) if i != pos]
    assert np.array_equal(gk[:, others], k0[:, others]) and np.array_equal(gv[:, others], v0[:, others])


@pytest.mark.parametrize("length", [1, 17, 64, 65, 401, 2048])
def test_decode_attention(length):
    nh, nkv, max_len = 32, 8, 2048
    k, v = randn_f16((nkv, max_len, 128), seed=length), randn_f16((nkv, max_len, 128), seed=length + 1)
    q = randn_f16((nh, 128), seed=length + 7)
    out = torch.empty((nh, 128), dtype=F16, device="cuda")
    pos = torch.tensor([length - 1], dtype=torch.long, device="cuda")
    fastpath.kernel_attention(q, k, v, out, n_head=nh, n_kv=nkv, pos=pos, window=max_len, max_len=max_len)
    want = orc.attention(to_bits(q), to_bits(k), to_bits(v), length, nh, nkv, f16=True)
    assert orc.relative_error(f32(out), orc.f16_to_f32(want)) < ATTN_TOL


def test_decode_attention_api_and_mask():
    nh, nkv, L = 32, 8, 300
    q = randn_f16((1, nh, 1, 128), seed=1)
    k, v = randn_f16((1, nkv, L, 128), seed=2), randn_f16((1, nkv, L, 128), seed=3)
    mask = torch.rand(1, 1, 1, L, generator=torch.Generator().manual_seed(4)) > 0.3
    before = fastpath.stats()["kernel"]
    y = fastpath.decode_attention(q, k, v, mask.cuda(), nh, nkv, 128)
    assert fastpath.stats()["kernel"] == before + 1 and y.dtype == F16
    want = orc.attention_masked(to_bits(q)[0], to_bits(k)[0], to_bits(v)[0], mask.numpy()[0, 0], nh, nkv,
                                f16=True)
    assert orc.relative_error(f32(y)[0, :, 0], orc.f16_to_f32(want)[:, 0]) < ATTN_TOL


@pytest.mark.parametrize("pos", [0, 63, 700])
@pytest.mark.parametrize("qk_norm", [False, True])
def test_qkv_attention_equals_the_two_launches(pos, qk_norm):
    nh, nkv, max_len = 32, 8, 2048
    qkv = randn_f16(((nh + 2 * nkv) * 128,), seed=pos + 11)
    k0, v0 = randn_f16((nkv, max_len, 128), seed=pos + 12), randn_f16((nkv, max_len, 128), seed=pos + 13)
    freqs = model.precompute_freqs_cis(max_len, 128, 1e6, device="cuda")[pos:pos + 1].contiguous()
    g = torch.Generator().manual_seed(pos)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(F16).cuda() if qk_norm else None
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(F16).cuda() if qk_norm else None
    p = torch.tensor([pos], dtype=torch.long, device="cuda")
    k1, v1 = k0.clone(), v0.clone()
    q = _qk_rope_kv(qkv, qw, kw, freqs, _lib.NF4B_BF16, p, k1, v1, nh, nkv, max_len)
    want = torch.empty((nh, 128), dtype=F16, device="cuda")
    fastpath.kernel_attention(q.view(nh, 128), k1, v1, want, n_head=nh, n_kv=nkv, pos=p, window=max_len,
                              max_len=max_len)
    k2, v2 = k0.clone(), v0.clone()
    got = torch.empty((nh, 128), dtype=F16, device="cuda")
    fastpath.qkv_attention(qkv, k2, v2, got, n_head=nh, n_kv=nkv, pos=p, window=max_len, max_len=max_len,
                           freqs=freqs, freqs_dtype=_lib.NF4B_BF16, q_norm_w=qw, k_norm_w=kw, eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(k2, k1) and torch.equal(v2, v1) and torch.equal(got, want)


@pytest.mark.parametrize("pos,qk_norm", [(0, False), (37, True), (1000, False)])
def test_decode_block_matches_the_oracle(pos, qk_norm):
    """A whole decode block in fp16 (the model cast with .half(), as the
    reference's TTS_HALF deployment does) against the oracle's block in fp16."""
    cfg = model.ModelArgs(max_seq_len=2048, attention_qk_norm=qk_norm) if pos >= 64 else \
        model.ModelArgs(dim=512, n_head=4, n_local_heads=2, head_dim=128, intermediate_size=1024,
                        attention_qk_norm=qk_norm, max_seq_len=256)
    blk = model.random_block(cfg, device="cuda", seed=pos).half()
    cache = blk.attention.kv_cache
    assert cache.k_cache.dtype == F16 and blk.attention_norm.weight.dtype == F16
    g = torch.Generator(device="cuda").manual_seed(pos + 1)
    cache.k_cache.copy_(torch.randn(cache.k_cache.shape, generator=g, device="cuda").to(F16))
    cache.v_cache.copy_(torch.randn(cache.v_cache.shape, generator=g, device="cuda").to(F16))
    freqs = model.precompute_freqs_cis(cfg.max_seq_len, cfg.head_dim, cfg.rope_base, device="cuda")
    x = randn_f16((1, 1, cfg.dim), seed=pos + 2)
    ip = torch.tensor([pos], dtype=torch.long, device="cuda")
    window = cfg.max_seq_len
    mask = torch.ones(window, window, dtype=torch.bool, device="cuda").tril()[None, None, ip, :window]
    kc, vc = to_bits(cache.k_cache)[0].copy(), to_bits(cache.v_cache)[0].copy()
    before = fusedlayer.stats()["fused"]
    with torch.inference_mode():
        y = blk(x, freqs[ip], mask, ip)
    assert fusedlayer.stats()["fused"] == before + 1 and y.dtype == F16
    a, ff = blk.attention, blk.feed_forward
    w = {kk: dequant_f16(lin) for kk, lin in
         (("wqkv", a.wqkv), ("wo", a.wo), ("w1", ff.w1), ("w3", ff.w3), ("w2", ff.w2))}
    w["attn_norm"], w["ffn_norm"] = to_bits(blk.attention_norm.weight), to_bits(blk.ffn_norm.weight)
    w["q_norm"] = to_bits(a.q_norm.weight) if qk_norm else None
    w["k_norm"] = to_bits(a.k_norm.weight) if qk_norm else None
    want = orc.decode_block(to_bits(x).reshape(-1), w, kc, vc, pos, orc.bf16_to_f32(to_bits(freqs[pos])),
                            cfg.n_head, cfg.n_local_heads, cfg.head_dim, cfg.norm_eps, cfg.norm_eps, f16=True)
    assert orc.relative_error(f32(y).ravel(), orc.f16_to_f32(want).ravel()) < BLOCK_TOL


def test_unknown_activation_dtype_is_rejected():
    layer = make_linear(256, 512, seed=1)
    x = randn_f16((1, 512), seed=2)
    y = torch.empty((1, 256), dtype=F16, device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    opts = _lib.GemmOpts(None, None, None, 0.0, 7)
    st = _lib.lib().nf4b_gemm_ex(ctypes.byref(layer._nf4_fast["desc"]), x.data_ptr(), y.data_ptr(), 1, 0, None,
                                 ws.data_ptr(), ws.numel(), ctypes.byref(opts), None)
    assert st == _lib.NF4B_ERR_DTYPE
    assert _lib.lib().nf4b_rms_norm_ex(x.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 512, 1e-6, _lib.NF4B_F32,
                                       None) == _lib.NF4B_ERR_DTYPE
    assert nf4gemv.matmul(layer, x.float()) is None


def _reference_kernel():
    from oracle import build_ref

    path = build_ref.gpu_so_path()
    if path is None:
        return None
    ref = ctypes.CDLL(str(path))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    ref.nf4mma_ref_launch.restype = ctypes.c_int
    ref.nf4mma_ref_launch.argtypes = [i32, i32, vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, i32, i32, i32, i32,
                                      i32, vp, i32, vp]
    return ref


@pytest.mark.parametrize("rows", [1, 8, 32])
@pytest.mark.parametrize("epi", [nf4gemv.EPI_NONE, nf4gemv.EPI_RESIDUAL, nf4gemv.EPI_SILU_GATE])
def test_against_the_references_own_fp16_kernel(rows, epi):
    """The reference's nf4_mma (fp16, app/engine/nf4gemv.py:94-231, compiled
    from its source) and this build's fp16 matmul on identical inputs. Both
    are fp32 accumulations of fp16 products rounded once; they differ in where
    the weight is rounded (the reference rounds code x scale to fp16, the
    register-fed GEMV rounds the code and scales the block sums in fp32) and
    in summation order, so the products agree to two fp16 ulps element by
    element. Each kernel's fused epilogue is then the oracle's fp16 epilogue
    of its own product."""
    ref = _reference_kernel()
    if ref is None:
        pytest.skip("oracle/_ref/nf4mma_ref.so was not built here")
    n, k = 2560, 9728
    layer = make_linear(n, k, seed=61 + rows)
    d = layer._nf4_fast["desc"]
    x = randn_f16((rows, k), seed=62 + rows)
    operand = randn_f16((rows, n), seed=63 + rows)
    lut = torch.tensor(orc.NF4_CODE, dtype=torch.float32, device="cuda")

    def reference(e):
        y = torch.empty((rows, n), dtype=F16, device="cuda")
        st = ref.nf4mma_ref_launch(rows, 1, x.data_ptr(), d.packed, d.absmax_code, d.absmax, d.code2, y.data_ptr(),
                                   lut.data_ptr(), d.offset, n, k, k // 64, 6, int(d.blocksize2).bit_length() - 1,
                                   operand.data_ptr() if e else None, e, torch.cuda.current_stream().cuda_stream)
        assert st == 0
        return y

    y0_ref, y_ref = reference(nf4gemv.EPI_NONE), reference(epi)
    y0 = nf4gemv.matmul(layer, x)
    y = nf4gemv.matmul(layer, x, epi=epi, operand=operand if epi else None)
    torch.cuda.synchronize()
    a, b = f32(y0_ref).astype(np.float64), f32(y0).astype(np.float64)
    assert np.isfinite(a).all() and np.isfinite(b).all()
    rms = np.sqrt((a ** 2).mean())
    assert np.all(np.abs(a - b) <= 2 * _ulp16(np.maximum(np.abs(a), np.abs(b))) + 1e-3 * rms)
    assert np.linalg.norm(a - b) / np.linalg.norm(a) < 2e-3
    if epi == nf4gemv.EPI_NONE:
        return
    # this build: deterministic, so its fused store is the epilogue of its own
    # product (the gate's exponential may move an output by one ulp)
    want = orc.epilogue(f32(y0), epi, to_bits(operand), f16=True)
    diff = np.abs(to_bits(y).astype(np.int32) - want.astype(np.int32))
    assert diff.max() <= (1 if epi == nf4gemv.EPI_SILU_GATE else 0) and (diff > 0).mean() < 1e-2
    # the reference: its blocks sum their warps' partials with shared-memory
    # atomics (an order that changes from launch to launch), so its fused
    # launch may round the product one ulp apart from its plain launch; with
    # the residual's cancellation that is many output ulps, so the bar is the
    # product's ulp carried through the epilogue plus the output's own ulp
    y0r = f32(y0_ref).astype(np.float64)
    factor = 1.0 if epi == nf4gemv.EPI_RESIDUAL else \
        np.abs(orc.f16_to_f32(orc.silu_bf16(to_bits(operand), f16=True)).astype(np.float64))
    want = orc.f16_to_f32(orc.epilogue(f32(y0_ref), epi, to_bits(operand), f16=True)).astype(np.float64)
    out = f32(y_ref).astype(np.float64)
    allowed = _ulp16(y0r) * factor + _ulp16(np.maximum(np.abs(out), np.abs(want)))
    assert np.all(np.abs(out - want) <= allowed)
