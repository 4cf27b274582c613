"""A decode block loaded from a bitsandbytes-layout checkpoint file runs the
fused decode path exactly as the block it was saved from (B200 only)."""

from __future__ import annotations

import pytest
import torch

from tests.helpers import randn_bf16
from ttspipe_b200 import checkpoint, fusedlayer, model, nf4gemv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qk_norm", [False, True])
def test_block_from_a_checkpoint_file_decodes_identically(tmp_path, qk_norm):
    assert nf4gemv.available() and nf4gemv.install() and fusedlayer.install()
    cfg = model.ModelArgs(dim=512, n_head=4, n_local_heads=2, intermediate_size=1024, max_seq_len=64,
                          attention_qk_norm=qk_norm)
    ref = model.random_block(cfg, device="cuda", seed=11)
    path = tmp_path / "block.safetensors"
    checkpoint.write_safetensors(path, checkpoint.block_state_dict(ref, "layers.0"))
    blk = checkpoint.load_block(checkpoint.read_safetensors(path, device="cuda"), "layers.0", cfg, device="cuda")
    freqs = model.precompute_freqs_cis(64, 128, 1e6, device="cuda")
    mask = torch.ones(1, 1, 1, 64, dtype=torch.bool, device="cuda")
    x = randn_bf16((1, 1, 512), seed=12, device="cuda")
    outs = []
    for b in (ref, blk):
        y = x
        for p in range(5):  # five positions: the KV caches fill the same way
            ip = torch.tensor([p], device="cuda")
            y = fusedlayer.decode_block(b, y, freqs[p:p + 1], mask, ip)
            assert y is not None
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(ref.attention.kv_cache.k_cache, blk.attention.kv_cache.k_cache)
