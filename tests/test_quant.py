"""The NF4 format: torch quantiser vs the oracle, the packing layout and the
nested-scale reconstruction (tests/test_nf4gemv.py:69-116 restated without
bitsandbytes)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nf4_oracle as orc
from ttspipe_b200 import quant


@pytest.mark.parametrize("shape,bs", [((8, 256), 64), ((13, 64), 64), ((96, 512), 128), ((40, 1024), 256)])
def test_torch_quantiser_is_bit_identical_to_the_oracle(shape, bs):
    w = (torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape))) * 0.02)
    packed, qs = quant.quantize_nf4(w, blocksize=bs)
    p2, am2 = orc.nf4_quantize(w.numpy(), bs)
    assert np.array_equal(packed.numpy(), p2)
    assert np.array_equal(qs.absmax.numpy(), am2)


def test_packing_layout_is_high_nibble_first():
    """Two indices per byte, high nibble first, row-major flattened: the
    indices recovered from the dequantised values by midpoint bucketing are
    exactly the packed nibbles (tests/test_nf4gemv.py:69-92)."""
    w = torch.randn(8, 256, generator=torch.Generator().manual_seed(1))
    packed, qs = quant.quantize_nf4(w, blocksize=64)
    deq = orc.bf16_to_f32(orc.dequantize_bf16(packed.numpy(), qs.absmax.numpy()))
    ratio = deq.reshape(8, -1, 64) / np.maximum(qs.absmax.numpy().reshape(8, -1, 1), 1e-20)
    bounds = (orc.NF4_CODE[:-1] + orc.NF4_CODE[1:]) / 2
    index = np.searchsorted(bounds, ratio.reshape(-1).astype(np.float32), side="left")
    flat = packed.numpy().reshape(-1)
    assert np.array_equal(flat >> 4, index[0::2])
    assert np.array_equal(flat & 15, index[1::2])


def test_double_quant_matches_the_oracle_and_reconstructs():
    w = torch.randn(64, 512, generator=torch.Generator().manual_seed(2)) * 0.02
    packed, qs = quant.quantize_nf4(w, blocksize=64, double_quant=True, blocksize2=256)
    _, am = orc.nf4_quantize(w.numpy(), 64)
    a8, am2, code2, off = orc.double_quantize(am, 256)
    assert np.array_equal(qs.absmax.numpy(), a8)
    assert np.array_equal(qs.state2.absmax.numpy(), am2)
    assert np.array_equal(qs.state2.code.numpy(), code2)
    assert np.float32(qs.offset.item()) == off
    # code2[a8] * absmax2 + offset, two rounded fp32 ops, equals the oracle's
    assert np.array_equal(quant.scales_fp32(qs).numpy(),
                          orc.nested_scales(a8, am2, code2, off, 256))
    # and the reconstruction is close to the fp32 absmax it encodes
    rel = np.abs(quant.scales_fp32(qs).numpy() - am) / am
    assert rel.max() < 0.05


def test_dynamic_code_map_shape():
    c = quant.dynamic_code_map()
    assert c.numel() == 256 and torch.all(c[1:] >= c[:-1])
    assert c.min().item() == pytest.approx(-0.99296875, abs=1e-6) and c.max().item() == 1.0
    assert np.array_equal(c.numpy(), orc.dynamic_code_map())


def test_all_zero_block_maps_to_code_zero():
    w = torch.zeros(2, 128)
    w[1, 64:] = 1.0
    packed, qs = quant.quantize_nf4(w)
    assert qs.absmax[0].item() == 0.0
    assert torch.all(packed[0] == 0x77)
    deq = orc.bf16_to_f32(orc.dequantize_bf16(packed.numpy(), qs.absmax.numpy()))
    assert np.all(deq[0] == 0) and np.all(deq[1, :64] == 0) and np.all(deq[1, 64:] == 1.0)
