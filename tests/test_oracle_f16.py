"""The oracle's fp16 switch (CPU): its fp16 rounding is torch's, and its fp16
formulas are the bf16 ones with fp16 at the same rounding points."""

from __future__ import annotations

import numpy as np
import torch

from oracle import nf4_oracle as orc


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_f16_rounding_is_torchs():
    g = torch.Generator().manual_seed(0)
    a = torch.cat([torch.randn(20000, generator=g) * s for s in (1e-7, 1e-5, 1e-3, 1.0, 300.0, 6e4, 1e5)])
    a = torch.cat([a, torch.tensor([65504.0, 65520.0, -65520.0, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -25, 0.0])])
    with np.errstate(over="ignore"):
        assert np.array_equal(orc.f32_to_f16(a.numpy()), bits(a.half()))
    h = a.half()
    assert np.array_equal(orc.f16_to_f32(bits(h)), h.float().numpy())


def test_f16_epilogues_are_torchs_fp16_ops():
    g = torch.Generator().manual_seed(1)
    acc = torch.randn(4096, generator=g) * 3
    r = (torch.randn(4096, generator=g) * 2).half()
    y = acc.half()
    got = orc.epilogue(acc.numpy(), orc.EPI_RESIDUAL, bits(r), f16=True)
    assert np.array_equal(got, bits(r + y))
    got = orc.epilogue(acc.numpy(), orc.EPI_SILU_GATE, bits(r), f16=True)
    want = (torch.nn.functional.silu(r.float()).half().float() * y.float()).half()
    diff = np.abs(got.astype(np.int32) - bits(want).astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-2   # exp in fp32 may differ by an ulp


def test_f16_rms_norm_and_rope_follow_the_fork_formulas():
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(3, 256, generator=g) * 2).half()
    w = (1 + 0.1 * torch.randn(256, generator=g)).half()
    xf = x.float()
    r = torch.rsqrt((xf.double() ** 2).mean(-1, keepdim=True).float() + 1e-6)
    want = ((xf * r).half().float() * w.float()).half()
    got = orc.rms_norm(bits(x), bits(w), 1e-6, f16=True)
    diff = np.abs(got.astype(np.int32) - bits(want).astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 1e-2   # torch's rsqrt is not correctly rounded
    q = (torch.randn(1, 2, 4, 16, generator=g)).half()
    f = torch.randn(2, 8, 2, generator=g)
    q0, q1 = q.float()[..., 0::2], q.float()[..., 1::2]
    c, s = f[None, :, None, :, 0], f[None, :, None, :, 1]
    out = torch.empty_like(q.float())
    out[..., 0::2] = q0 * c - q1 * s
    out[..., 1::2] = q1 * c + q0 * s
    assert np.array_equal(orc.rope(bits(q), f.numpy(), f16=True), bits(out.half()))


def test_f16_dequantise_and_matmul():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(32, 256, generator=g) * 0.05
    packed, absmax = orc.nf4_quantize(w.numpy(), 64)
    wq = orc.dequantize_f16(packed, absmax, 64)
    vals = orc.NF4_CODE[orc.nf4_unpack(packed)].reshape(32, 4, 64) * absmax.reshape(32, 4, 1)
    assert np.array_equal(wq, bits(torch.from_numpy(vals.reshape(32, 256).astype(np.float32)).half()))
    x = (torch.randn(2, 256, generator=g)).half()
    exact = orc.matmul_exact(bits(x), wq, f16=True)
    ref = x.double() @ torch.from_numpy(orc.f16_to_f32(wq)).double().T
    assert np.allclose(exact, ref.numpy(), rtol=1e-12, atol=1e-12)
    y = orc.matmul_dequant(bits(x), wq, f16=True)
    assert np.array_equal(y, bits(torch.from_numpy(exact.astype(np.float32)).half()))
