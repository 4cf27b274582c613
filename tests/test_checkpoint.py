"""bitsandbytes-serialised NF4 checkpoints without bitsandbytes (CPU).

The reference fills bnb.nn.Linear4bit modules from its prequantized
checkpoint's state dict (app/engine/worker.py:169-215); ttspipe_b200.checkpoint
reads and writes that layout (QuantState.as_dict(packed=True)) and the
safetensors container.
"""

from __future__ import annotations

import json
import struct

import pytest
import torch

from ttspipe_b200 import checkpoint, model, quant


def _lin(out_f, in_f, nested, seed):
    g = torch.Generator().manual_seed(seed)
    return quant.Linear4bit.from_float(torch.randn(out_f, in_f, generator=g) * 0.02, double_quant=nested)


@pytest.mark.parametrize("nested", [True, False])
def test_linear_round_trips_through_the_bitsandbytes_layout(nested):
    lin = _lin(96, 256, nested, seed=1)
    sd = checkpoint.linear_state_dict(lin, "layers.0.attention.wqkv")
    # bitsandbytes' keys, its [out * in / 2, 1] weight and its packed JSON fields
    base = "layers.0.attention.wqkv.weight"
    assert sd[base].shape == (96 * 256 // 2, 1) and sd[base].dtype == torch.uint8
    meta = json.loads(bytes(sd[f"{base}.quant_state.bitsandbytes__nf4"].tolist()).decode())
    assert meta["quant_type"] == "nf4" and meta["blocksize"] == 64 and meta["shape"] == [96, 256]
    assert meta["dtype"] == "bfloat16"
    if nested:
        assert {"nested_blocksize", "nested_dtype", "nested_offset"} <= set(meta)
        assert f"{base}.nested_absmax" in sd and f"{base}.nested_quant_map" in sd
    else:
        assert "nested_blocksize" not in meta and f"{base}.nested_absmax" not in sd
    back = checkpoint.linear_from_state_dict(sd, "layers.0.attention.wqkv")
    assert (back.out_features, back.in_features) == (96, 256)
    assert torch.equal(back.weight.data, lin.weight.data)
    a, b = lin.weight.quant_state, back.weight.quant_state
    assert b.nested == a.nested and b.blocksize == a.blocksize and tuple(b.shape) == tuple(a.shape)
    assert torch.equal(b.absmax, a.absmax)
    assert torch.equal(quant.scales_fp32(b), quant.scales_fp32(a))
    if nested:
        assert torch.equal(b.state2.absmax, a.state2.absmax) and torch.equal(b.state2.code, a.state2.code)
        assert b.state2.blocksize == a.state2.blocksize


def test_bias_and_errors():
    lin = quant.Linear4bit.from_float(torch.randn(16, 64) * 0.02, bias=torch.arange(16.0))
    sd = checkpoint.linear_state_dict(lin, "p")
    assert torch.equal(checkpoint.linear_from_state_dict(sd, "p").bias, lin.bias)
    assert checkpoint.is_nf4_linear(sd, "p") and not checkpoint.is_nf4_linear(sd, "q")
    with pytest.raises(ValueError, match="not a bitsandbytes NF4"):
        checkpoint.linear_from_state_dict(sd, "q")
    bad = dict(sd)
    bad["p.weight"] = bad["p.weight"][:-1]
    with pytest.raises(ValueError, match="expected uint8"):
        checkpoint.linear_from_state_dict(bad, "p")
    fp4 = dict(sd)
    meta = json.loads(bytes(sd["p.weight.quant_state.bitsandbytes__nf4"].tolist()).decode())
    meta["quant_type"] = "fp4"
    fp4["p.weight.quant_state.bitsandbytes__nf4"] = torch.tensor(list(json.dumps(meta).encode()), dtype=torch.uint8)
    with pytest.raises(ValueError, match="not nf4"):
        checkpoint.linear_from_state_dict(fp4, "p")
    missing = {k: v for k, v in sd.items() if not k.endswith(".absmax")}
    with pytest.raises(ValueError, match="missing"):
        checkpoint.linear_from_state_dict(missing, "p")


def test_safetensors_container_round_trip(tmp_path):
    g = torch.Generator().manual_seed(3)
    tensors = {
        "a.u8": torch.randint(0, 256, (7, 3), generator=g, dtype=torch.uint8),
        "b.bf16": torch.randn(5, 4, generator=g).to(torch.bfloat16),
        "c.f32": torch.randn(9, generator=g),
        "d.i64": torch.arange(6, dtype=torch.int64).reshape(2, 3),
        "e.empty": torch.zeros(0, dtype=torch.float32),
    }
    path = tmp_path / "t.safetensors"
    checkpoint.write_safetensors(path, tensors, metadata={"format": "pt"})
    # the container itself: little-endian header length, JSON header, 8-byte padded
    raw = path.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    header = json.loads(raw[8:8 + n])
    assert header["__metadata__"] == {"format": "pt"}
    assert header["b.bf16"]["dtype"] == "BF16" and header["b.bf16"]["shape"] == [5, 4]
    assert header["a.u8"]["data_offsets"] == [0, 21]
    back = checkpoint.read_safetensors(path)
    assert set(back) == set(tensors)
    for k, v in tensors.items():
        assert back[k].dtype == v.dtype and torch.equal(back[k], v)


def test_blocks_load_from_a_checkpoint_file(tmp_path):
    cfg = model.ModelArgs(dim=256, n_head=4, n_local_heads=2, intermediate_size=512, max_seq_len=32,
                          attention_qk_norm=True)
    blocks = [model.random_block(cfg, device="cpu", seed=s) for s in (1, 2)]
    sd = {}
    for i, b in enumerate(blocks):
        sd.update(checkpoint.block_state_dict(b, f"layers.{i}"))
    path = tmp_path / "model.safetensors"
    checkpoint.write_safetensors(path, sd)
    loaded = checkpoint.read_safetensors(path)
    for i, ref in enumerate(blocks):
        blk = checkpoint.load_block(loaded, f"layers.{i}", cfg, device="cpu")
        for name in ("attention.wqkv", "attention.wo", "feed_forward.w1", "feed_forward.w3", "feed_forward.w2"):
            a, b = ref.get_submodule(name), blk.get_submodule(name)
            assert torch.equal(a.weight.data, b.weight.data)
            assert torch.equal(quant.scales_fp32(a.weight.quant_state), quant.scales_fp32(b.weight.quant_state))
        for name in ("attention_norm", "ffn_norm", "attention.q_norm", "attention.k_norm"):
            assert torch.equal(ref.get_submodule(name).weight, blk.get_submodule(name).weight)
        assert blk.attention.kv_cache.k_cache.shape == (1, 2, 32, 128)
    wrong = model.ModelArgs(dim=256, n_head=4, n_local_heads=2, intermediate_size=1024, max_seq_len=32,
                            attention_qk_norm=True)
    with pytest.raises(ValueError, match="in the checkpoint"):
        checkpoint.load_block(loaded, "layers.0", wrong, device="cpu")
