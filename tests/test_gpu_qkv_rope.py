"""The wqkv GEMV with the rotary + KV-cache write fused into its store
(nf4b_gemm_qkv_rope / nf4gemv.matmul_qkv_rope; B200 only).

It must equal, bit for bit, the two launches it replaces: the decode GEMV
(checked against the oracle in test_gpu_kernels / test_gpu_reg_gemv) and
nf4b_qk_rope_kv without q/k norm (checked against the oracle in
test_gpu_kernels) - y, q, and the new K/V cache rows, with every other cache
row untouched.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.helpers import make_linear, randn_bf16
from ttspipe_b200 import _lib, fusedops, nf4gemv

pytestmark = pytest.mark.gpu

FTYPES = {torch.float32: _lib.NF4B_F32, torch.float16: _lib.NF4B_F16, torch.bfloat16: _lib.NF4B_BF16}


@pytest.fixture(scope="module", autouse=True)
def installed():
    assert nf4gemv.available() and nf4gemv.install()


def _freq_row(pos, dtype):
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
    ang = pos * inv
    row = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).reshape(128)
    return row.to(dtype).cuda()


def _caches(nkv, max_len, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(nkv, max_len, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(nkv, max_len, 128, generator=g, device="cuda").to(torch.bfloat16)
    return k, v


def _unfused(lin, x, freqs, pos, kc, vc, nh, nkv, norm):
    xx = fusedops.rms_norm(x, norm[0], norm[1]) if norm is not None else x
    qkv = nf4gemv.matmul(lin, xx)
    q = torch.empty(nh * 128, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().nf4b_qk_rope_kv(
        qkv.data_ptr(), None, None, 1e-6, freqs.data_ptr(), FTYPES[freqs.dtype], pos.data_ptr(), q.data_ptr(),
        kc.data_ptr(), vc.data_ptr(), nh, nkv, 128, kc.shape[1], ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return qkv, q


@pytest.mark.parametrize("nh,nkv,k_in,nested", [(32, 8, 2560, True), (32, 8, 2560, False), (4, 2, 512, True)])
@pytest.mark.parametrize("fdtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("position", [0, 5, 63])
def test_equals_gemv_then_qk_rope_kv(nh, nkv, k_in, nested, fdtype, position):
    max_len = 64
    lin = make_linear((nh + 2 * nkv) * 128, k_in, seed=nh + k_in + position, nested=nested)
    x = randn_bf16((1, k_in), seed=position + 3, device="cuda")
    freqs = _freq_row(position, fdtype)
    pos = torch.tensor([position], dtype=torch.long, device="cuda")
    kc0, vc0 = _caches(nkv, max_len, 11 + position)
    for norm in (None, ((1 + 0.1 * torch.randn(k_in, generator=torch.Generator().manual_seed(5))).to(
            torch.bfloat16).cuda(), 1e-6)):
        k1, v1, k2, v2 = kc0.clone(), vc0.clone(), kc0.clone(), vc0.clone()
        qkv_want, q_want = _unfused(lin, x, freqs, pos, k1, v1, nh, nkv, norm)
        q_got = torch.empty(nh * 128, dtype=torch.bfloat16, device="cuda")
        qkv_got = nf4gemv.matmul_qkv_rope(lin, x, freqs=freqs, pos=pos, q_out=q_got, k_cache=k2, v_cache=v2,
                                          n_head=nh, n_kv=nkv, norm=norm)
        assert qkv_got is not None
        torch.cuda.synchronize()
        assert torch.equal(qkv_got, qkv_want)
        assert torch.equal(q_got, q_want)
        assert torch.equal(k2, k1) and torch.equal(v2, v1)   # the new rows, and nothing else changed


def test_position_outside_the_cache_writes_no_row():
    nh, nkv, max_len = 4, 2, 16
    lin = make_linear((nh + 2 * nkv) * 128, 512, seed=77)
    x = randn_bf16((1, 512), seed=78, device="cuda")
    kc, vc = _caches(nkv, max_len, 79)
    k0, v0 = kc.clone(), vc.clone()
    q = torch.empty(nh * 128, dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([max_len], dtype=torch.long, device="cuda")
    y = nf4gemv.matmul_qkv_rope(lin, x, freqs=_freq_row(3, torch.float32), pos=pos, q_out=q, k_cache=kc,
                                v_cache=vc, n_head=nh, n_kv=nkv)
    assert y is not None
    torch.cuda.synchronize()
    assert torch.equal(kc, k0) and torch.equal(vc, v0)


def test_declines_outside_its_envelope():
    nh, nkv = 4, 2
    kc, vc = _caches(nkv, 16, 80)
    q = torch.empty(nh * 128, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(1, dtype=torch.long, device="cuda")
    fr = _freq_row(0, torch.float32)
    lin = make_linear((nh + 2 * nkv) * 128, 512, seed=81)
    x2 = randn_bf16((2, 512), seed=82, device="cuda")
    assert nf4gemv.matmul_qkv_rope(lin, x2, freqs=fr, pos=pos, q_out=q, k_cache=kc, v_cache=vc, n_head=nh,
                                   n_kv=nkv) is None          # two rows
    odd = make_linear((nh + 2 * nkv) * 128 - 16, 512, seed=83)
    x = randn_bf16((1, 512), seed=84, device="cuda")
    assert nf4gemv.matmul_qkv_rope(odd, x, freqs=fr, pos=pos, q_out=q, k_cache=kc, v_cache=vc, n_head=nh,
                                   n_kv=nkv) is None          # n_out is not whole heads
    k128 = make_linear((nh + 2 * nkv) * 128, 384, seed=85)    # k_in % 256 != 0: not the register-fed kernel
    x3 = randn_bf16((1, 384), seed=86, device="cuda")
    assert nf4gemv.matmul_qkv_rope(k128, x3, freqs=fr, pos=pos, q_out=q, k_cache=kc, v_cache=vc, n_head=nh,
                                   n_kv=nkv) is None
