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
* ``sampler.npz``       - the reference's torch sampler ``_sample_torch``
                          (app/engine/graphs.py:55-73): the kept set and the
                          final probabilities of seeded logit rows. Its last
                          line hands the probabilities to the fish-speech
                          fork's ``multinomial_sample_one_no_sync``; the fork
                          is not in the checkout, so a stand-in module returns
                          the probabilities it is given instead of drawing.
                          Every line that decides the kept set and the
                          probabilities is the reference's own.

Inputs are stored next to outputs so the tests need neither the reference nor
a random generator to replay them. Run: ``python tests/golden/make_golden.py
[fixture ...]`` (all fixtures when none is named). The reference checkout is
``$TTSPIPE_REFERENCE``, or a directory named ``reference`` next to this
repository.
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

REFERENCE = str(build_ref.reference_root())


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


def _fork_stand_in():
    """Register a stand-in for the one fork function `_sample_torch` calls,
    `multinomial_sample_one_no_sync(probs)`: it returns `probs` itself, so the
    reference function hands back the probability row it would draw from."""
    import types

    names = ["fish_speech", "fish_speech.models", "fish_speech.models.text2semantic",
             "fish_speech.models.text2semantic.inference"]
    for n in names:
        sys.modules.setdefault(n, types.ModuleType(n))
    sys.modules[names[-1]].multinomial_sample_one_no_sync = lambda probs: probs


def _bf16_below(b: int) -> int:
    """The largest bf16 value below the bf16 bit pattern b (finite, not -max)."""
    if b & 0x8000:
        return b + 1                  # negative: one step further from zero
    return 0x8001 if b == 0 else b - 1


def _distinct_top(v: np.ndarray, top: int) -> np.ndarray:
    """bf16 bits of the fp32 row v with no two equal values among its `top`
    largest (ties would make the reference's unstable sort order matter):
    walking down from the largest, a value equal to or above its predecessor
    becomes the next bf16 value below it; every other value is then held
    strictly below the last of them."""
    b = orc.f32_to_bf16(v.astype(np.float32))
    f = orc.bf16_to_f32(b)
    idx = np.argsort(-f, kind="stable")
    head, rest = idx[:top], idx[top:]
    prev = None
    for i in head:
        if prev is not None and orc.bf16_to_f32(b[i:i + 1])[0] >= orc.bf16_to_f32(np.array([prev], np.uint16))[0]:
            b[i] = _bf16_below(int(prev))
        prev = int(b[i])
    floor = _bf16_below(prev)
    fl = orc.bf16_to_f32(np.array([floor], np.uint16))[0]
    over = rest[orc.bf16_to_f32(b[rest]) > fl]
    b[over] = floor
    hv = np.sort(orc.bf16_to_f32(b))[::-1][:top + 1]
    assert np.all(np.diff(hv) < 0), "the top values are not distinct"
    return b


def sampler() -> dict:
    """Kept sets and probabilities of the reference's torch sampler."""
    sys.path.insert(0, REFERENCE)
    _fork_stand_in()
    from app.engine.graphs import _sample_torch

    out = {}
    # (name, vocab, logit scale, temperature, top_p, top_k)
    cases = [("flat", 4096, 1.0, 0.7, 0.8, 64), ("peaked", 4096, 4.0, 0.7, 0.8, 64),
             ("high", 4096, 3.0, 1.0, 0.9, 64), ("topk5", 4096, 2.0, 0.7, 0.99, 5),
             ("first", 4096, 2.0, 0.7, 0.01, 64), ("cold", 4096, 2.0, 1e-6, 0.8, 64),
             ("wide", 32768, 5.0, 0.7, 0.8, 64), ("vocab", 155136, 6.0, 0.7, 0.8, 64)]
    for ci, (name, vocab, scale, temp, top_p, top_k) in enumerate(cases):
        rng = np.random.default_rng(500 + ci)
        for attempt in range(50):
            bits_row = _distinct_top(rng.standard_normal(vocab) * scale, 80)
            logits = torch.from_numpy(orc.bf16_to_f32(bits_row)).view(1, 1, vocab)
            probs = _sample_torch(logits, torch.tensor(temp), torch.tensor(top_p),
                                  torch.tensor(top_k))
            p = probs.reshape(-1).double().numpy()
            # The kept set does not depend on the temperature (the reference
            # cuts on the unscaled logits); at temperature 1 every kept entry
            # has a nonzero probability, which shows the set even where a tiny
            # temperature rounds the others' probabilities to zero.
            p1 = _sample_torch(logits, torch.tensor(1.0), torch.tensor(top_p),
                               torch.tensor(top_k)).reshape(-1).double().numpy()
            # keep rows whose cumulative probabilities stay clear of top_p (fp32
            # here, fp64 in the oracle) so the kept set cannot depend on rounding
            sv = np.sort(orc.bf16_to_f32(bits_row).astype(np.float64))[::-1]
            e = np.exp(sv - sv[0])
            cum = np.cumsum(e / e.sum())[:top_k + 1]
            if np.min(np.abs(cum - top_p)) > 1e-4:
                break
        else:
            raise RuntimeError(f"no clear row for {name}")
        kept = np.nonzero(p1 > 0)[0]
        kept = kept[np.argsort(-p1[kept], kind="stable")]
        out[f"{name}_logits"] = bits_row
        out[f"{name}_params"] = np.array([temp, top_p, top_k], dtype=np.float64)
        out[f"{name}_kept"] = kept.astype(np.int64)
        out[f"{name}_probs"] = p[kept].astype(np.float32)
    out["cases"] = np.array([c[0] for c in cases])
    return out


FIXTURES = ("nf4_code", "gemv", "decode_block", "attention", "sampler")


def main(which=None) -> None:
    which = list(which or FIXTURES)
    if any(w in which for w in ("gemv", "decode_block")):
        if build_ref.so_path() is None:
            build_ref.build()
        ext = build_ref.load()
    if "nf4_code" in which:
        np.savez_compressed(HERE / "nf4_code.npz", **nf4_code())
    if "gemv" in which:
        np.savez_compressed(HERE / "gemv.npz", **gemv(ext))
    if "decode_block" in which:
        np.savez_compressed(HERE / "decode_block.npz", **decode_blocks(ext))
    if "attention" in which:
        np.savez_compressed(HERE / "attention.npz", **attention())
    if "sampler" in which:
        np.savez_compressed(HERE / "sampler.npz", **sampler())
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main(sys.argv[1:])
