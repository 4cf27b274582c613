"""Regenerate the golden fixtures in this directory from the reference itself.

Runs ONLY where the read-only reference checkout is present (``REFERENCE``
below) and the reference's CPU extension has been built by
``oracle/build_ref.py``. Every output below is computed by reference code:

* ``nf4_code.npz``      - ``NF4_CODE`` as the reference states it
                          (app/engine/nf4gemv.py:69-86).
* ``gemv.npz``          - the reference's AVX-512 ``nf4_gemv`` and AMX
                          ``nf4_amx`` (app/engine/nf4cpu.py:256-270, :339-451)
                          on seeded packed weights / bf16 absmax / bf16 codes.
* ``decode_block.npz``  - the reference's C++ ``decode_block`` and
                          ``prefill_block`` (app/engine/nf4cpu.py:479-617,
                          :644-780) on a small seeded block, with the KV caches
                          they leave behind.
* ``attention.npz``     - the reference's torch ``decode_attention``
                          (app/engine/fastpath.py:133-174) for decode and
                          short-prefill shapes.

Inputs are stored next to outputs so the tests need neither the reference nor
a random generator to replay them. Run: ``python tests/golden/make_golden.py``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import build_ref  # noqa: E402
from oracle import nf4_oracle as orc  # noqa: E402

REFERENCE = "/root/reference"


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def nf4_code() -> dict:
    sys.path.insert(0, REFERENCE)
    from app.engine.nf4gemv import NF4_CODE

    return {"nf4_code": np.asarray(NF4_CODE, dtype=np.float32)}


def random_nf4(n: int, k: int, seed: int):
    """Packed bytes and bf16 absmax as the reference's own CPU test makes them
    (tests/test_nf4cpu.py:31-35)."""
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 255, (n, k // 2), dtype=torch.uint8, generator=g)
    absmax = (torch.rand(n, k // 64, generator=g) * 0.1).to(torch.bfloat16)
    return packed, absmax


def gemv(ext) -> dict:
    out = {}
    code16 = torch.tensor(orc.NF4_CODE).to(torch.bfloat16)
    out["code16"] = bits(code16)
    cases = [("g0", 13, 64, 1), ("g1", 256, 512, 1), ("g2", 96, 256, 3), ("g3", 64, 2560, 1),
             ("a0", 64, 256, 9), ("a1", 48, 128, 33), ("a2", 80, 512, 16)]
    for name, n, k, m in cases:
        packed, absmax = random_nf4(n, k, seed=n * 7 + k + m)
        g = torch.Generator().manual_seed(1000 + m + n)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        if name.startswith("a"):
            y = ext.nf4_amx(x, packed, absmax, code16, n)
        else:
            y = ext.nf4_gemv(x, packed, absmax, code16, n)
        out[f"{name}_packed"] = packed.numpy()
        out[f"{name}_absmax"] = bits(absmax)
        out[f"{name}_x"] = bits(x)
        out[f"{name}_y"] = bits(y)
    return out


def block_weights(dim: int, n_head: int, n_kv: int, head_dim: int, inter: int, seed: int):
    """Random-init NF4 weights for one block, quantised by the oracle's
    restated quantiser; the reference kernels get (packed, bf16 absmax)."""
    rng = np.random.default_rng(seed)
    qkv_out = (n_head + 2 * n_kv) * head_dim
    shapes = {"wqkv": (qkv_out, dim), "wo": (dim, n_head * head_dim), "w1": (inter, dim),
              "w3": (inter, dim), "w2": (dim, inter)}
    w = {}
    for name, (o, i) in shapes.items():
        dense = (rng.standard_normal((o, i)) * 0.05).astype(np.float32)
        packed, absmax = orc.nf4_quantize(dense, 64)
        w[name] = (packed, orc.f32_to_bf16(absmax).reshape(o, i // 64))
    norms = {
        "attn_norm": orc.f32_to_bf16((rng.random(dim) + 0.5).astype(np.float32)),
        "ffn_norm": orc.f32_to_bf16((rng.random(dim) + 0.5).astype(np.float32)),
        "q_norm": orc.f32_to_bf16((rng.random(head_dim) + 0.5).astype(np.float32)),
        "k_norm": orc.f32_to_bf16((rng.random(head_dim) + 0.5).astype(np.float32)),
    }
    return w, norms


def decode_blocks(ext) -> dict:
    out = {}
    dim, n_head, n_kv, head_dim, inter, max_len = 256, 4, 2, 128, 512, 96
    eps, qk_eps = 1e-6, 1e-6
    w, norms = block_weights(dim, n_head, n_kv, head_dim, inter, seed=7)
    for name, (packed, absmax) in w.items():
        out[f"w_{name}_packed"] = packed
        out[f"w_{name}_absmax"] = absmax
    for name, v in norms.items():
        out[f"n_{name}"] = v
    freqs = orc.precompute_freqs_cis(max_len, head_dim, 1e6)
    out["freqs"] = freqs
    code16 = torch.tensor(orc.NF4_CODE).to(torch.bfloat16)
    t = {k: (torch.from_numpy(p), from_bits(a)) for k, (p, a) in w.items()}
    w13_p = torch.cat([t["w1"][0], t["w3"][0]]).contiguous()
    w13_a = torch.cat([t["w1"][1], t["w3"][1]]).contiguous()
    empty = torch.empty(0, dtype=torch.bfloat16)
    rng = np.random.default_rng(11)
    kc0 = orc.f32_to_bf16(rng.standard_normal((n_kv, max_len, head_dim)).astype(np.float32))
    vc0 = orc.f32_to_bf16(rng.standard_normal((n_kv, max_len, head_dim)).astype(np.float32))
    out["k_cache0"], out["v_cache0"] = kc0, vc0
    cases = [("d0", 70, True, 1), ("d1", 0, False, 1), ("d2", 37, True, 1), ("p0", 50, True, 3)]
    for name, pos, qk, m in cases:
        x = orc.f32_to_bf16(rng.standard_normal((1, m, dim)).astype(np.float32))
        kc = from_bits(kc0.copy()).view(1, n_kv, max_len, head_dim).clone()
        vc = from_bits(vc0.copy()).view(1, n_kv, max_len, head_dim).clone()
        qn = from_bits(norms["q_norm"]) if qk else empty
        kn = from_bits(norms["k_norm"]) if qk else empty
        args_w = [t["wqkv"][0], t["wqkv"][1], t["wo"][0], t["wo"][1], w13_p, w13_a,
                  t["w2"][0], t["w2"][1], code16]
        if m == 1:
            mask = torch.ones(pos + 1, dtype=torch.bool)
            f = from_bits(freqs[pos]).float()
            y = ext.decode_block(from_bits(x).view(1, 1, dim), from_bits(norms["attn_norm"]),
                                 from_bits(norms["ffn_norm"]), qn, kn, eps, qk_eps, *args_w,
                                 kc, vc, pos, f, mask, n_head, n_kv, head_dim, inter)
        else:
            causal = torch.ones(max_len, max_len, dtype=torch.bool).tril()
            mask = causal[pos:pos + m, :pos + m]
            f = from_bits(freqs[pos:pos + m]).float()
            y = ext.prefill_block(from_bits(x).view(1, m, dim), from_bits(norms["attn_norm"]),
                                  from_bits(norms["ffn_norm"]), qn, kn, eps, qk_eps, *args_w,
                                  kc, vc, pos, f, mask, n_head, n_kv, head_dim, inter)
        out[f"{name}_x"] = x
        out[f"{name}_y"] = bits(y)
        out[f"{name}_meta"] = np.array([pos, int(qk), m], dtype=np.int64)
        # only the rows the call writes; the rest of each cache is k_cache0/v_cache0
        out[f"{name}_k_rows"] = bits(kc)[0][:, pos:pos + m]
        out[f"{name}_v_rows"] = bits(vc)[0][:, pos:pos + m]
    out["dims"] = np.array([dim, n_head, n_kv, head_dim, inter, max_len], dtype=np.int64)
    out["eps"] = np.array([eps, qk_eps], dtype=np.float64)
    return out


def attention() -> dict:
    sys.path.insert(0, REFERENCE)
    from app.engine.fastpath import decode_attention

    out = {}
    n_head, n_kv, d = 8, 2, 128
    # (name, query rows, cache rows, first query position): the query rows are
    # the last `seqlen` positions of the cache, causal within themselves.
    cases = [("s1", 1, 1, 0), ("s17", 1, 17, 16), ("s100", 1, 100, 99), ("p8", 8, 40, 32)]
    for name, seqlen, kv_len, prefix in cases:
        g = torch.Generator().manual_seed(kv_len * 3 + seqlen)
        q = torch.randn(1, n_head, seqlen, d, generator=g).to(torch.bfloat16)
        k = torch.randn(1, n_kv, kv_len, d, generator=g).to(torch.bfloat16)
        v = torch.randn(1, n_kv, kv_len, d, generator=g).to(torch.bfloat16)
        causal = torch.ones(kv_len, kv_len, dtype=torch.bool).tril()
        mask = causal[prefix:prefix + seqlen][None, None]
        y = decode_attention(q, k, v, mask, n_head, n_kv, d)
        out[f"{name}_q"], out[f"{name}_k"], out[f"{name}_v"] = bits(q), bits(k), bits(v)
        out[f"{name}_mask"] = mask.numpy()
        out[f"{name}_y"] = bits(y)
    out["dims"] = np.array([n_head, n_kv, d], dtype=np.int64)
    return out


def main() -> None:
    if build_ref.so_path() is None:
        build_ref.build()
    ext = build_ref.load()
    np.savez_compressed(HERE / "nf4_code.npz", **nf4_code())
    np.savez_compressed(HERE / "gemv.npz", **gemv(ext))
    np.savez_compressed(HERE / "decode_block.npz", **decode_blocks(ext))
    np.savez_compressed(HERE / "attention.npz", **attention())
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
