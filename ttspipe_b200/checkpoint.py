"""Prequantized NF4 checkpoints: bitsandbytes' serialisation, read and written
without bitsandbytes.

The reference loads its prequantized checkpoint through the fish-speech fork,
which turns every ``nn.Linear`` into ``bnb.nn.Linear4bit(quant_type="nf4",
compress_statistics=True)`` and fills it from the checkpoint's state dict
(app/engine/worker.py:169-215). bitsandbytes is not part of this stack, so this
module reads that state-dict layout into ``quant.Linear4bit`` modules, which
``nf4gemv.prepare`` serves in place (zero copy), and writes it back.

The layout is bitsandbytes' ``QuantState.as_dict(packed=True)`` (bitsandbytes
>= 0.45, the reference's requirement; the layout has been stable since 0.41).
For a 4-bit linear whose state-dict prefix is ``P``:

=============================================  ===========================================
``P.weight``                                   packed codes, uint8 (bitsandbytes stores
                                               [out * in / 2, 1]; any shape with that many
                                               bytes is accepted), two codes per byte,
                                               high nibble first
``P.weight.absmax``                            uint8 [blocks] (nested) or fp32 [blocks]
``P.weight.quant_map``                         fp32 [16], the NF4 code points
``P.weight.nested_absmax``                     fp32 [blocks2] (nested only)
``P.weight.nested_quant_map``                  fp32 [256] (nested only)
``P.weight.quant_state.bitsandbytes__nf4``     uint8 bytes of a UTF-8 JSON object with
                                               ``quant_type, blocksize, dtype, shape`` and,
                                               nested, ``nested_blocksize, nested_dtype,
                                               nested_offset``
``P.bias``                                     optional
=============================================  ===========================================

Files: ``read_safetensors`` / ``write_safetensors`` handle the safetensors
container (an 8-byte little-endian header length, a JSON header mapping each
name to ``{dtype, shape, data_offsets}``, then the raw little-endian bytes)
without the safetensors package; ``torch.load`` state dicts work as they are.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import torch

from ttspipe_b200.quant import NF4_CODE, Linear4bit, Params4bit, QuantState

PACKED_KEY = "quant_state.bitsandbytes__nf4"

_ST_DTYPES = {
    "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64,
    "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64, "BOOL": torch.bool,
}
_ST_NAMES = {v: k for k, v in _ST_DTYPES.items()}
_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _dtype_name(dt: torch.dtype) -> str:
    # bitsandbytes writes str(dtype).strip("torch."): "bfloat16", "float16", "float32"
    return str(dt).split(".", 1)[1]


# ----------------------------------------------------------------------------
# one 4-bit linear
# ----------------------------------------------------------------------------


def is_nf4_linear(sd, prefix: str) -> bool:
    """Whether `prefix` names a bitsandbytes NF4 linear in the state dict."""
    return f"{prefix}.weight.{PACKED_KEY}" in sd


def linear_from_state_dict(sd, prefix: str, device=None) -> Linear4bit:
    """The ``Linear4bit`` serialised under `prefix` (tensors moved to `device`).

    Raises ValueError when the entry is not an NF4 linear or its tensors do
    not agree with its recorded shape and block sizes."""
    meta_t = sd.get(f"{prefix}.weight.{PACKED_KEY}")
    if meta_t is None:
        raise ValueError(f"{prefix}: no {PACKED_KEY} entry (not a bitsandbytes NF4 linear)")
    meta = json.loads(bytes(meta_t.to("cpu", torch.uint8).reshape(-1).tolist()).decode("utf-8"))
    if meta.get("quant_type") != "nf4":
        raise ValueError(f"{prefix}: quant_type {meta.get('quant_type')!r} is not nf4")
    out_f, in_f = (int(v) for v in meta["shape"])
    bs = int(meta["blocksize"])
    if in_f % bs or (out_f * in_f) % 2:
        raise ValueError(f"{prefix}: shape {out_f}x{in_f} does not fit blocksize {bs}")
    dev = torch.device(device) if device is not None else None

    def get(key, dtype=None):
        t = sd.get(f"{prefix}.{key}")
        if t is None:
            raise ValueError(f"{prefix}: missing {prefix}.{key}")
        t = t.to(dev) if dev is not None else t
        return t if dtype is None else t.to(dtype)

    packed = get("weight")
    if packed.dtype != torch.uint8 or packed.numel() != out_f * in_f // 2:
        raise ValueError(f"{prefix}: weight is {packed.dtype} x {packed.numel()}, expected uint8 x {out_f * in_f // 2}")
    packed = packed.reshape(out_f, in_f // 2).contiguous()
    nblocks = out_f * in_f // bs
    absmax = get("weight.absmax").reshape(-1).contiguous()
    code = get("weight.quant_map", torch.float32).reshape(-1).contiguous()
    if code.numel() != 16 or absmax.numel() != nblocks:
        raise ValueError(f"{prefix}: quant_map of {code.numel()} / absmax of {absmax.numel()} entries")
    nested = "nested_blocksize" in meta
    if nested:
        if absmax.dtype != torch.uint8:
            raise ValueError(f"{prefix}: nested absmax must be uint8 codes")
        bs2 = int(meta["nested_blocksize"])
        absmax2 = get("weight.nested_absmax", torch.float32).reshape(-1).contiguous()
        code2 = get("weight.nested_quant_map", torch.float32).reshape(-1).contiguous()
        if code2.numel() != 256 or absmax2.numel() != -(-nblocks // bs2):
            raise ValueError(f"{prefix}: nested_quant_map / nested_absmax sizes do not match")
        state2 = QuantState(absmax2, (absmax2.numel(),), bs2, quant_type="dynamic",
                            dtype=_DTYPES.get(meta.get("nested_dtype", "float32"), torch.float32), code=code2)
        offset = torch.tensor(float(meta["nested_offset"]), dtype=torch.float32, device=absmax.device)
        qs = QuantState(absmax, (out_f, in_f), bs, dtype=_DTYPES.get(meta.get("dtype"), torch.bfloat16),
                        code=code, nested=True, offset=offset, state2=state2)
    else:
        qs = QuantState(absmax.to(torch.float32), (out_f, in_f), bs,
                        dtype=_DTYPES.get(meta.get("dtype"), torch.bfloat16), code=code)
    bias = sd.get(f"{prefix}.bias")
    lin = Linear4bit(in_f, out_f, bias=bias is not None, compute_dtype=qs.dtype, device=packed.device)
    lin.weight = Params4bit(packed, qs)
    if bias is not None:
        lin.bias.data.copy_(bias.to(lin.bias.device, lin.bias.dtype))
    return lin


def linear_state_dict(lin, prefix: str) -> dict:
    """`lin` (a ``Linear4bit``) in bitsandbytes' serialisation under `prefix`."""
    w = lin.weight
    qs = w.quant_state
    out_f, in_f = (int(v) for v in qs.shape)
    meta = {"quant_type": "nf4", "blocksize": int(qs.blocksize), "dtype": _dtype_name(qs.dtype),
            "shape": [out_f, in_f]}
    code = qs.code if qs.code is not None else torch.tensor(NF4_CODE, dtype=torch.float32)
    sd = {
        f"{prefix}.weight": w.data.reshape(-1, 1),
        f"{prefix}.weight.absmax": qs.absmax,
        f"{prefix}.weight.quant_map": code.to(torch.float32),
    }
    if qs.nested:
        off = qs.offset.item() if isinstance(qs.offset, torch.Tensor) else float(qs.offset)
        meta.update({"nested_blocksize": int(qs.state2.blocksize), "nested_dtype": _dtype_name(qs.state2.dtype)
                     if isinstance(qs.state2.dtype, torch.dtype) else "float32", "nested_offset": off})
        sd[f"{prefix}.weight.nested_absmax"] = qs.state2.absmax
        sd[f"{prefix}.weight.nested_quant_map"] = qs.state2.code
    sd[f"{prefix}.weight.{PACKED_KEY}"] = torch.tensor(list(json.dumps(meta).encode("utf-8")), dtype=torch.uint8)
    if getattr(lin, "bias", None) is not None:
        sd[f"{prefix}.bias"] = lin.bias.data
    return sd


# ----------------------------------------------------------------------------
# transformer blocks (the fork's module names, as ttspipe_b200.model mirrors them)
# ----------------------------------------------------------------------------

_BLOCK_LINEARS = ("attention.wqkv", "attention.wo", "feed_forward.w1", "feed_forward.w3", "feed_forward.w2")
_BLOCK_NORMS = ("attention_norm", "ffn_norm")


def block_state_dict(block, prefix: str) -> dict:
    """A ``model.TransformerBlock`` as a state dict (NF4 linears serialised)."""
    sd = {}
    for name in _BLOCK_LINEARS:
        mod = block.get_submodule(name)
        sd.update(linear_state_dict(mod, f"{prefix}.{name}"))
    for name in _BLOCK_NORMS:
        sd[f"{prefix}.{name}.weight"] = block.get_submodule(name).weight.data
    if getattr(block.attention, "attention_qk_norm", False):
        sd[f"{prefix}.attention.q_norm.weight"] = block.attention.q_norm.weight.data
        sd[f"{prefix}.attention.k_norm.weight"] = block.attention.k_norm.weight.data
    return sd


@torch.no_grad()
def load_block(sd, prefix: str, cfg, device=None):
    """A ``model.TransformerBlock`` for `cfg` with every weight from `sd` under
    `prefix`, a bf16 KV cache of zeros, and its NF4 linears prepared for the
    kernels when they are available (``nf4gemv.prepare``)."""
    from ttspipe_b200 import model, nf4gemv

    blk = model.TransformerBlock(cfg, device)
    for name in _BLOCK_LINEARS:
        lin = linear_from_state_dict(sd, f"{prefix}.{name}", device)
        expect = blk.get_submodule(name)
        if (lin.in_features, lin.out_features) != (expect.in_features, expect.out_features):
            raise ValueError(f"{prefix}.{name}: {lin.out_features}x{lin.in_features} in the checkpoint, "
                             f"{expect.out_features}x{expect.in_features} in the model")
        parent, leaf = name.rsplit(".", 1)
        setattr(blk.get_submodule(parent), leaf, lin)
    norms = list(_BLOCK_NORMS)
    if cfg.attention_qk_norm:
        norms += ["attention.q_norm", "attention.k_norm"]
    for name in norms:
        w = sd.get(f"{prefix}.{name}.weight")
        if w is None:
            raise ValueError(f"missing {prefix}.{name}.weight")
        blk.get_submodule(name).weight.copy_(w.to(blk.get_submodule(name).weight.dtype))
    blk.attention.kv_cache = model.KVCache(cfg.max_seq_len, cfg.n_local_heads, cfg.head_dim, device=device)
    if nf4gemv.available():
        for name in _BLOCK_LINEARS:
            nf4gemv.prepare(blk.get_submodule(name))
    return blk


# ----------------------------------------------------------------------------
# safetensors container
# ----------------------------------------------------------------------------


def read_safetensors(path, device=None) -> dict:
    """Every tensor of a .safetensors file (CPU, or moved to `device`)."""
    raw = Path(path).read_bytes()
    if len(raw) < 8:
        raise ValueError(f"{path}: too short for a safetensors header")
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n].decode("utf-8"))
    data = memoryview(raw)[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = _ST_DTYPES.get(info["dtype"])
        if dt is None:
            raise ValueError(f"{path}: {name} has unsupported dtype {info['dtype']}")
        b, e = info["data_offsets"]
        shape = [int(s) for s in info["shape"]]
        t = torch.frombuffer(bytearray(data[b:e]), dtype=dt) if e > b else torch.empty(0, dtype=dt)
        t = t.reshape(shape)
        out[name] = t.to(device) if device is not None else t
    return out


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """`tensors` (name -> tensor) as a .safetensors file, names in sorted order."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        if t.dtype not in _ST_NAMES:
            raise ValueError(f"{name}: dtype {t.dtype} cannot be stored")
        b = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _ST_NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
