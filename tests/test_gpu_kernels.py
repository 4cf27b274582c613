"""Parity of every CUDA kernel against the oracle, through the public API and
the C ABI (B200 only).

Bars: dequantisation, RMSNorm, rotary, the q/k norm and the KV-cache write are
bit-exact; GEMV/GEMM outputs within max|err| <= 2e-2 x RMS(output) (the north
star's bar) and norm-relative < 5e-3 (the reference's, tests/test_nf4gemv.py),
both against the exactly accumulated, unrounded product of the bit-exact
dequantised weight - the kernel's bf16 output is then charged with its own
rounding only once; the fused epilogues are checked bit for bit against the
oracle's epilogue applied to the kernel's own un-fused output;
attention within max-relative 1e-2: the reference's 5e-3 bar
(tests/test_nf4gemv.py:224-242) was set in fp16, whose ulp is 8x finer than
bf16's; 1e-2 is ~2.5 bf16 ulps at the largest element. The residual
difference is the fork's bf16 rounding of every probability, which a split-KV
kernel (like the reference's own attn_partial/attn_combine) cannot apply.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from tests.helpers import from_bits, make_linear, oracle_dequant, randn_bf16, to_bits
from ttspipe_b200 import _lib, fastpath, fusedops, nf4gemv

pytestmark = pytest.mark.gpu

GEMM_TOL = 2e-2  # max |err| / rms(ref)
ATTN_TOL = 1e-2  # max |err| / max |ref|

# The S2-Pro slow-AR projections (out, in): q, k, v, o, gate, up, down.
S2PRO = [(4096, 2560), (1024, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (9728, 2560),
         (2560, 9728)]


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available(), "the NF4 library must load on a B200"
    assert nf4gemv.install()
    assert fusedops.install()


def check_matmul(got: torch.Tensor, x: torch.Tensor, layer):
    """Kernel output vs the exact product of x and the dequantised weight."""
    w = orc.matmul_exact(to_bits(x).reshape(-1, layer.in_features), oracle_dequant(layer))
    g = orc.bf16_to_f32(to_bits(got)).reshape(w.shape)
    assert np.isfinite(g).all()
    err = orc.rms_relative_max_error(g, w)
    nrel = orc.norm_relative_error(g, w)
    assert err <= GEMM_TOL, f"max|err|/rms = {err:.4f}"
    assert nrel < 5e-3, f"norm-relative = {nrel:.2e}"


# --------------------------------------------------------------------------
# dequantisation: bit-exact
# --------------------------------------------------------------------------


@pytest.mark.parametrize("shape", [(9728, 2560), (1544, 2560), (13, 64), (64, 4096)])
@pytest.mark.parametrize("nested", [True, False])
@pytest.mark.parametrize("bs", [64, 128])
def test_dequantize_is_bit_exact(shape, nested, bs):
    if shape[1] % bs:
        pytest.skip("in_features must be a multiple of the blocksize")
    layer = make_linear(*shape, seed=shape[0] + bs, nested=nested, blocksize=bs)
    got = nf4gemv.dequantize(layer)
    assert np.array_equal(to_bits(got), oracle_dequant(layer))


# --------------------------------------------------------------------------
# streaming GEMV (rows <= 8) and tcgen05 GEMM (rows > 8)
# --------------------------------------------------------------------------


def test_config1_plain_fp32_absmax_gemv():
    """W [9728, 2560] ~ N(0, 0.02) seed 0, plain fp32 absmax,
    x bf16 [1, 2560] seed 1."""
    layer = make_linear(9728, 2560, seed=0, nested=False)
    x = randn_bf16((1, 2560), seed=1, device="cuda")
    y = layer(x)
    assert y.shape == (1, 9728) and y.dtype == torch.bfloat16
    check_matmul(y, x, layer)


@pytest.mark.parametrize("idx", range(7))
def test_config2_projections_at_m1(idx):
    out_f, in_f = S2PRO[idx]
    layer = make_linear(out_f, in_f, seed=100 + idx, nested=True)
    x = randn_bf16((1, 1, in_f), seed=1000 + idx, device="cuda")
    before = nf4gemv.stats()["fast"]
    y = layer(x)
    assert nf4gemv.stats()["fast"] == before + 1
    assert y.shape == (1, 1, out_f)
    check_matmul(y, x, layer)


@pytest.mark.parametrize("rows", [2, 3, 4, 5, 8, 9, 16, 19, 32])
@pytest.mark.parametrize("shape", [(6144, 2560), (2560, 9728), (1544, 2560)])
def test_rows_match_the_oracle(shape, rows):
    """Batched decode and prefill, including row counts that do not fill a
    tile (tests/test_nf4gemv.py:169-186 restated)."""
    layer = make_linear(*shape, seed=shape[0] + rows)
    x = randn_bf16((1, rows, shape[1]), seed=6000 + rows, device="cuda")
    y = layer(x)
    assert y.shape == (1, rows, shape[0])
    check_matmul(y, x, layer)


@pytest.mark.parametrize("shape", [(13, 64), (48, 128), (16, 64), (100, 192), (17, 256)])
@pytest.mark.parametrize("rows", [1, 3, 31])
def test_tiny_and_ragged_shapes(shape, rows):
    layer = make_linear(*shape, seed=3 * shape[0] + rows)
    x = randn_bf16((rows, shape[1]), seed=7000 + rows, device="cuda")
    y = nf4gemv.matmul(layer, x)
    check_matmul(y, x, layer)


def check_epilogue(layer, x, epi_name):
    """The fused store equals the oracle's epilogue applied to the kernel's own
    un-fused output (same accumulation order): bit for bit for the residual
    add; for the gate, silu's exponential may differ from NumPy's by an fp32
    ulp, so a few elements may land one bf16 ulp apart."""
    rows, n = x.shape[0], layer.out_features
    operand = randn_bf16((rows, n), seed=7919 + rows, device="cuda")
    e = nf4gemv.EPI_RESIDUAL if epi_name == "residual" else nf4gemv.EPI_SILU_GATE
    y0 = nf4gemv.matmul(layer, x)
    y = nf4gemv.matmul(layer, x, epi=e, operand=operand)
    check_matmul(y0, x, layer)
    want = orc.epilogue(orc.bf16_to_f32(to_bits(y0)), e, to_bits(operand))
    got = to_bits(y)
    if e == nf4gemv.EPI_RESIDUAL:
        assert np.array_equal(got, want)
    else:
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() < 1e-3


@pytest.mark.parametrize("rows", [1, 7, 32])
@pytest.mark.parametrize("epi", ["residual", "gate"])
def test_fused_epilogues(epi, rows):
    layer = make_linear(2560, 9728, seed=11 + rows)
    x = randn_bf16((rows, 9728), seed=5000 + rows, device="cuda")
    check_epilogue(layer, x, epi)


@pytest.mark.parametrize("rows", [1, 32])
def test_repeated_calls_are_deterministic(rows):
    """The split-K reduction sums its partials in a fixed order."""
    layer = make_linear(9728, 2560, seed=5)
    x = randn_bf16((rows, 2560), seed=6, device="cuda")
    a = nf4gemv.matmul(layer, x)
    b = nf4gemv.matmul(layer, x)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_single_row_equals_that_row_of_a_batch_within_rounding():
    layer = make_linear(6144, 2560, seed=9)
    x = randn_bf16((4, 2560), seed=10, device="cuda")
    one = nf4gemv.matmul(layer, x[1:2])
    many = nf4gemv.matmul(layer, x)
    d = (one.float() - many[1:2].float()).abs().max().item()
    assert d <= 2 ** -7 * many.float().abs().max().item()


def test_every_input_rank_is_served():
    layer = make_linear(512, 2560, seed=21)
    for shape in [(1, 1, 2560), (1, 2560), (2560,)]:
        x = randn_bf16(shape, seed=22, device="cuda")
        y = layer(x)
        assert y.shape == (*shape[:-1], 512)


def test_bias_is_applied():
    from ttspipe_b200.quant import Linear4bit

    w = torch.randn(512, 2560, generator=torch.Generator().manual_seed(3)).cuda() * 0.02
    b = torch.randn(512, generator=torch.Generator().manual_seed(4)).cuda()
    layer = Linear4bit.from_float(w, bias=b)
    x = randn_bf16((1, 2560), seed=5, device="cuda")
    y = layer(x)
    plain = nf4gemv.matmul(layer, x)
    assert torch.equal(y, plain + layer.bias)


def test_declines_are_counted_and_do_not_launch():
    from ttspipe_b200.quant import Linear4bit

    w = torch.randn(256, 2560, generator=torch.Generator().manual_seed(1)).cuda() * 0.02
    layer = Linear4bit.from_float(w)
    layer.weight.quant_state.blocksize = 96
    assert not nf4gemv.prepare(layer)
    assert nf4gemv.matmul(layer, randn_bf16((1, 2560), seed=1, device="cuda")) is None
    good = make_linear(256, 2560, seed=2)
    assert nf4gemv.prepare(good)
    assert nf4gemv.matmul(good, randn_bf16((1, 2560), seed=1, device="cuda").float()) is None   # fp32 x
    assert nf4gemv.matmul(good, randn_bf16((1, 2048), seed=1, device="cuda")) is None


def test_c_abi_gemm_directly():
    """The C entry point, called with raw pointers as a ctypes/cgo binding would."""
    layer = make_linear(1024, 2560, seed=31)
    assert nf4gemv.prepare(layer)
    desc = layer._nf4_fast["desc"]
    L = _lib.lib()
    x = randn_bf16((3, 2560), seed=32, device="cuda")
    y = torch.empty((3, 1024), dtype=torch.bfloat16, device="cuda")
    need = L.nf4b_gemm_workspace_size(ctypes.byref(desc), 3)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    st = L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), 3, 0, None, ws.data_ptr(),
                     need, None)
    assert st == 0, _lib.last_error()
    torch.cuda.synchronize()
    check_matmul(y, x, layer)
    counters = ws[:256].view(torch.int32)  # partials may remain; the counters are reset
    assert torch.count_nonzero(counters).item() == 0
    assert L.nf4b_gemm(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), 3, 0, None, ws.data_ptr(),
                       need - 1, None) == -5
    assert L.nf4b_device_error(0) == 0


# --------------------------------------------------------------------------
# RMSNorm and rotary: bit-exact
# --------------------------------------------------------------------------


@pytest.mark.parametrize("rows,width", [(1, 2560), (32, 128), (8, 128), (1, 9728), (3, 2560), (1, 40)])
def test_rms_norm_is_bit_exact(rows, width):
    x = randn_bf16((1, rows, width), seed=rows * 1000 + width, device="cuda")
    w = (1.0 + 0.1 * torch.randn(width, generator=torch.Generator().manual_seed(width))).to(torch.bfloat16).cuda()
    y = fusedops.rms_norm(x, w, 1e-6)
    want = orc.rms_norm(to_bits(x).reshape(rows, width), to_bits(w), 1e-6)
    assert np.array_equal(to_bits(y).reshape(rows, width), want)


def test_rms_norm_declines():
    w = torch.ones(128, dtype=torch.bfloat16, device="cuda")
    assert fusedops.rms_norm(torch.randn(1, 1, 128, device="cuda"), w, 1e-6) is None
    wide = randn_bf16((1, 4, 256), seed=1, device="cuda")
    assert fusedops.rms_norm(wide[..., :128], w, 1e-6) is None


@pytest.mark.parametrize("shape", [(1, 1, 32, 128), (1, 1, 8, 128), (1, 4, 32, 128), (2, 3, 8, 64)])
@pytest.mark.parametrize("fdtype", [torch.bfloat16, torch.float32, torch.float16])
def test_rope_is_bit_exact(shape, fdtype):
    b, s, h, d = shape
    x = randn_bf16(shape, seed=sum(shape), device="cuda")
    f = torch.randn(s, d // 2, 2, generator=torch.Generator().manual_seed(s)).to(fdtype).cuda()
    y = fusedops.rope(x, f)
    want = orc.rope(to_bits(x), f.float().cpu().numpy())
    assert np.array_equal(to_bits(y), want)


def test_rope_uses_each_positions_own_frequencies():
    x = randn_bf16((1, 5, 2, 8), seed=3, device="cuda")
    f = torch.randn(5, 4, 2).to(torch.bfloat16).cuda()
    whole = fusedops.rope(x, f)
    for s in range(5):
        alone = fusedops.rope(x[:, s:s + 1].contiguous(), f[s:s + 1].contiguous())
        assert torch.equal(whole[:, s:s + 1], alone)


def test_rope_at_s2pro_positions_up_to_4095():
    from ttspipe_b200.model import precompute_freqs_cis

    freqs = precompute_freqs_cis(4096, 128, 1e6, device="cuda")
    pos = torch.tensor([0, 1, 1000, 2047, 4095])
    x = randn_bf16((1, len(pos), 32, 128), seed=4, device="cuda")
    y = fusedops.rope(x, freqs[pos.cuda()].contiguous())
    want = orc.rope(to_bits(x), orc.bf16_to_f32(to_bits(freqs[pos.cuda()])))
    assert np.array_equal(to_bits(y), want)


# --------------------------------------------------------------------------
# decode attention
# --------------------------------------------------------------------------


def _cache(n_kv, max_len, seed):
    k = randn_bf16((n_kv, max_len, 128), seed=seed, device="cuda")
    v = randn_bf16((n_kv, max_len, 128), seed=seed + 1, device="cuda")
    return k, v


@pytest.mark.parametrize("length", [1, 10, 17, 63, 64, 65, 401, 2048])
def test_decode_attention_by_position(length):
    nh, nkv, max_len = 32, 8, 2048
    k, v = _cache(nkv, max_len, seed=length)
    q = randn_bf16((nh, 128), seed=length + 7, device="cuda")
    out = torch.empty((nh, 128), dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([length - 1], dtype=torch.long, device="cuda")
    fastpath.kernel_attention(q, k, v, out, n_head=nh, n_kv=nkv, pos=pos, window=max_len,
                              max_len=max_len)
    want = orc.attention(to_bits(q), to_bits(k), to_bits(v), length, nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(out)), orc.bf16_to_f32(want)) < ATTN_TOL


@pytest.mark.parametrize("nh,nkv", [(4, 4), (8, 4), (32, 4)])
@pytest.mark.parametrize("length", [17, 300, 1100])
def test_decode_attention_query_groups(nh, nkv, length):
    """Groups of 1, 2 and 8 query heads per KV head (the kernel's tensor-core
    tiles pad a group to 16 rows), at live lengths that occupy one, five and all
    eight CTAs of a KV head's cluster."""
    max_len = 1536
    k, v = _cache(nkv, max_len, seed=nh * 31 + length)
    q = randn_bf16((nh, 128), seed=length + nh, device="cuda")
    out = torch.empty((nh, 128), dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([length - 1], dtype=torch.long, device="cuda")
    fastpath.kernel_attention(q, k, v, out, n_head=nh, n_kv=nkv, pos=pos, window=max_len, max_len=max_len)
    want = orc.attention(to_bits(q), to_bits(k), to_bits(v), length, nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(out)), orc.bf16_to_f32(want)) < ATTN_TOL


@pytest.mark.parametrize("max_len,length", [(16, 1), (16, 5), (16, 16), (100, 64), (100, 65), (100, 100),
                                            (300, 130), (300, 300)])
def test_decode_attention_short_windows(max_len, length):
    """Windows of 1..4 chunks: one CTA per KV head, or clusters of 2..5."""
    nh, nkv = 32, 8
    k, v = _cache(nkv, max_len, seed=max_len + length)
    q = randn_bf16((nh, 128), seed=length + 3, device="cuda")
    out = torch.empty((nh, 128), dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([length - 1], dtype=torch.long, device="cuda")
    fastpath.kernel_attention(q, k, v, out, n_head=nh, n_kv=nkv, pos=pos, window=max_len, max_len=max_len)
    want = orc.attention(to_bits(q), to_bits(k), to_bits(v), length, nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(out)), orc.bf16_to_f32(want)) < ATTN_TOL


@pytest.mark.parametrize("kv_len", [1, 10, 17, 401, 2048])
def test_decode_attention_api_matches_the_oracle(kv_len):
    """fastpath.decode_attention's signature (tests/test_nf4gemv.py:224-242)."""
    nh, nkv = 32, 8
    q = randn_bf16((1, nh, 1, 128), seed=kv_len, device="cuda")
    k = randn_bf16((1, nkv, kv_len, 128), seed=kv_len + 1, device="cuda")
    v = randn_bf16((1, nkv, kv_len, 128), seed=kv_len + 2, device="cuda")
    mask = torch.ones(1, 1, 1, kv_len, dtype=torch.bool, device="cuda")
    before = fastpath.stats()["kernel"]
    y = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    assert fastpath.stats()["kernel"] == before + 1
    want = orc.attention(to_bits(q)[0, :, 0], to_bits(k)[0], to_bits(v)[0], kv_len, nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(y)[0, :, 0]), orc.bf16_to_f32(want)) < ATTN_TOL


def test_decode_attention_honours_the_mask_and_never_reads_masked_rows():
    nh, nkv, L = 32, 8, 64
    q = randn_bf16((1, nh, 1, 128), seed=1, device="cuda")
    k = randn_bf16((1, nkv, L, 128), seed=2, device="cuda")
    v = randn_bf16((1, nkv, L, 128), seed=3, device="cuda")
    mask = torch.ones(1, 1, 1, L, dtype=torch.bool, device="cuda")
    mask[..., 40:] = False
    mask[..., 5] = False
    ours = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    k[:, :, 40:] = float("nan")
    v[:, :, 40:] = float("inf")
    k[:, :, 5] = 1e3
    again = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    assert torch.equal(ours, again)
    want = orc.attention_masked(to_bits(q)[0], to_bits(k)[0], to_bits(v)[0],
                                mask[0, 0].cpu().numpy(), nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(ours)[0]), orc.bf16_to_f32(want)) < ATTN_TOL


def test_query_heads_map_onto_their_kv_head():
    """Query head i reads KV head i // groups (tests/test_nf4gemv.py:297-319)."""
    nh, nkv, L = 8, 2, 3
    q = torch.zeros(1, nh, 1, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, nkv, L, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(1, nkv, L, 128, dtype=torch.bfloat16, device="cuda")
    for h in range(nkv):
        v[0, h] = float(h + 1)
    mask = torch.ones(1, 1, 1, L, dtype=torch.bool, device="cuda")
    out = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    for head in range(nh):
        assert out[0, head, 0, 0].item() == pytest.approx(head // (nh // nkv) + 1)


def test_prefill_attention_uses_the_grouped_formulation():
    nh, nkv, seqlen, prefix = 32, 8, 8, 32
    kv_len = prefix + seqlen
    q = randn_bf16((1, nh, seqlen, 128), seed=1, device="cuda")
    k = randn_bf16((1, nkv, kv_len, 128), seed=2, device="cuda")
    v = randn_bf16((1, nkv, kv_len, 128), seed=3, device="cuda")
    mask = torch.ones(kv_len, kv_len, dtype=torch.bool, device="cuda").tril()[prefix:][None, None]
    y = fastpath.decode_attention(q, k, v, mask, nh, nkv, 128)
    want = orc.attention_masked(to_bits(q)[0], to_bits(k)[0], to_bits(v)[0],
                                mask[0, 0].cpu().numpy(), nh, nkv)
    assert orc.relative_error(orc.bf16_to_f32(to_bits(y)[0]), orc.bf16_to_f32(want)) < ATTN_TOL


# --------------------------------------------------------------------------
# q/k norm + rotary + KV write fused into the attention launch
# --------------------------------------------------------------------------


@pytest.mark.parametrize("max_len,pos", [(2048, 0), (2048, 5), (2048, 63), (2048, 64), (2048, 700), (16, 0),
                                         (16, 9), (16, 15)])
@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("fdtype", [torch.bfloat16, torch.float32])
def test_qkv_attention_equals_qk_rope_kv_then_attention(max_len, pos, qk_norm, fdtype):
    from ttspipe_b200 import _lib, model

    nh, nkv = 32, 8
    ftype = {torch.bfloat16: _lib.NF4B_BF16, torch.float32: _lib.NF4B_F32}[fdtype]
    qkv = randn_bf16(((nh + 2 * nkv) * 128,), seed=pos + 11, device="cuda")
    k0, v0 = _cache(nkv, max_len, seed=pos + 12)
    freqs = model.precompute_freqs_cis(max_len, 128, 1e6, device="cuda").to(fdtype)[pos:pos + 1].contiguous()
    g = torch.Generator().manual_seed(pos)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).cuda() if qk_norm else None
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).cuda() if qk_norm else None
    p = torch.tensor([pos], dtype=torch.long, device="cuda")
    # separate launches
    k1, v1 = k0.clone(), v0.clone()
    q = torch.empty(nh * 128, dtype=torch.bfloat16, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib().nf4b_qk_rope_kv(
        qkv.data_ptr(), None if qw is None else qw.data_ptr(), None if kw is None else kw.data_ptr(), 1e-6,
        freqs.data_ptr(), ftype, p.data_ptr(), q.data_ptr(), k1.data_ptr(), v1.data_ptr(), nh, nkv, 128, max_len, st))
    want = torch.empty((nh, 128), dtype=torch.bfloat16, device="cuda")
    fastpath.kernel_attention(q.view(nh, 128), k1, v1, want, n_head=nh, n_kv=nkv, pos=p, window=max_len,
                              max_len=max_len)
    # one launch
    k2, v2 = k0.clone(), v0.clone()
    got = torch.empty((nh, 128), dtype=torch.bfloat16, device="cuda")
    fastpath.qkv_attention(qkv, k2, v2, got, n_head=nh, n_kv=nkv, pos=p, window=max_len, max_len=max_len,
                           freqs=freqs, freqs_dtype=ftype, q_norm_w=qw, k_norm_w=kw, eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(k2, k1) and torch.equal(v2, v1)
    assert torch.equal(got, want)
