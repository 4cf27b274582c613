"""Test helpers: bf16 bit conversions between torch and the NumPy oracle, and
seeded NF4 weights made on the device and mirrored for the oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import nf4_oracle as orc


def to_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> uint16 bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)
    return t.to(device)


def randn_bf16(shape, seed: int, device="cpu", std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).to(torch.bfloat16).to(device)


def oracle_scales(qs) -> np.ndarray:
    """The fp32 per-block scales of a QuantState, computed by the oracle."""
    if not qs.nested:
        return qs.absmax.float().cpu().numpy()
    st2 = qs.state2
    off = qs.offset
    off = float(off.item() if hasattr(off, "item") else off)
    return orc.nested_scales(qs.absmax.cpu().numpy(), st2.absmax.cpu().numpy(),
                             st2.code.float().cpu().numpy(), np.float32(off), int(st2.blocksize))


def oracle_dequant(layer) -> np.ndarray:
    """bf16 bits [out, in] of a Linear4bit's weight, dequantised by the oracle."""
    qs = layer.weight.quant_state
    return orc.dequantize_bf16(layer.weight.data.cpu().numpy(), oracle_scales(qs), int(qs.blocksize))


def make_linear(out_f: int, in_f: int, *, seed: int, nested: bool = True, device="cuda",
                std: float = 0.02, blocksize: int = 64):
    """A seeded NF4 Linear4bit; on a GPU it is also `prepare`d, as the
    reference's install does for every layer of a model."""
    from ttspipe_b200 import nf4gemv
    from ttspipe_b200.quant import Linear4bit

    g = torch.Generator(device="cpu").manual_seed(seed)
    w = (torch.randn(out_f, in_f, generator=g) * std).to(device)
    layer = Linear4bit.from_float(w, double_quant=nested, blocksize=blocksize)
    if layer.weight.device.type == "cuda":
        nf4gemv.prepare(layer)
    return layer
