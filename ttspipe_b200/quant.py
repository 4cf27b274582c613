"""bitsandbytes-format NF4 weights without bitsandbytes.

The reference reads bitsandbytes' ``Params4bit`` buffers and ``QuantState``
fields in place (app/engine/nf4gemv.py:343-377). bitsandbytes is not part of
this stack, so this module provides the same objects:

* ``QuantState`` - the fields the reference's ``prepare`` reads
  (``quant_type, shape, blocksize, nested, absmax, offset, state2.{blocksize,
  absmax, code}``, plus ``code`` for the CPU path, app/engine/nf4cpu.py:850-857);
* ``Params4bit`` - a uint8 parameter [out, in/2] carrying ``quant_state``;
* ``Linear4bit`` - a module holding one, whose forward is routed through the
  NF4 kernels once ``nf4gemv.install()`` has run;
* ``quantize_nf4`` - bitsandbytes' blockwise NF4 quantisation (with optional
  double quantisation of the scales), in torch so it runs where the weights
  live. It is set-up code, not the hot path; results are bit-identical to the
  restatement in ``oracle/nf4_oracle.py``.

Any object with the same attributes works with ``nf4gemv.prepare``; a real
``bitsandbytes.nn.Linear4bit`` does too.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

#: bitsandbytes' NF4 code points in index order (app/engine/nf4gemv.py:69-86).
NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


def dynamic_code_map(device=None) -> torch.Tensor:
    """Signed 256-entry scale codebook of the "dynamic tree" form bitsandbytes
    uses for double quantisation: seven decades 1e-6..1, 2**i points per decade
    and sign, plus 0 and 1, sorted (fp32)."""
    vals = []
    for i in range(7):
        b = torch.linspace(0.1, 1.0, 2**i + 1, dtype=torch.float64)
        means = (b[:-1] + b[1:]) / 2.0
        scale = 10.0 ** (i - 6)
        vals += (scale * means).tolist() + (-scale * means).tolist()
    vals += [0.0, 1.0]
    vals = sorted(vals + [0.0] * (256 - len(vals)))
    return torch.tensor(vals, dtype=torch.float32, device=device)


@dataclass
class QuantState:
    """The subset of bitsandbytes' QuantState the kernels read."""

    absmax: torch.Tensor          # fp32 [nblocks] (plain) or uint8 [nblocks] (nested)
    shape: tuple                  # (out_features, in_features)
    blocksize: int = 64
    quant_type: str = "nf4"
    dtype: torch.dtype = torch.bfloat16
    code: torch.Tensor | None = None  # NF4 code points (fp32)
    nested: bool = False
    offset: torch.Tensor | float | None = None
    state2: "QuantState | None" = None

    def to(self, device):
        def mv(t):
            return t.to(device) if isinstance(t, torch.Tensor) else t
        st2 = self.state2.to(device) if self.state2 is not None else None
        return QuantState(mv(self.absmax), self.shape, self.blocksize, self.quant_type, self.dtype,
                          mv(self.code), self.nested, mv(self.offset), st2)


def _nearest(values: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Index of the nearest table entry by midpoint bucketing (right=False)."""
    mids = (table[:-1] + table[1:]) / 2
    return torch.bucketize(values, mids)


@torch.no_grad()
def quantize_nf4(weight: torch.Tensor, blocksize: int = 64, double_quant: bool = False,
                 blocksize2: int = 256) -> tuple[torch.Tensor, QuantState]:
    """bitsandbytes-style NF4 quantisation of a 2-D fp32/bf16/fp16 weight.

    Blocks of `blocksize` over the row-major flattened weight; ratio =
    w * (1/absmax) in fp32; nearest code point by midpoints; two indices per
    byte, high nibble first (tests/test_nf4gemv.py:69-92). With `double_quant`
    the fp32 absmax is centred on its mean (`offset`) and quantised blockwise
    (`blocksize2`) to the 8-bit dynamic code map with an fp32 absmax2 per block.
    Returns (packed uint8 [out, in/2], QuantState).
    """
    if weight.dim() != 2:
        raise ValueError("weight must be 2-D")
    out_f, in_f = weight.shape
    if in_f % blocksize:
        raise ValueError(f"in_features {in_f} is not a multiple of blocksize {blocksize}")
    dev = weight.device
    w = weight.detach().to(torch.float32).reshape(-1, blocksize)
    absmax = w.abs().amax(dim=1)
    inv = torch.where(absmax > 0, 1.0 / absmax, torch.zeros_like(absmax))
    ratio = w * inv[:, None]
    code = torch.tensor(NF4_CODE, dtype=torch.float32, device=dev)
    idx = _nearest(ratio, code).to(torch.uint8)
    idx[absmax == 0] = 7
    flat = idx.reshape(-1)
    packed = ((flat[0::2] << 4) | flat[1::2]).reshape(out_f, in_f // 2).contiguous()
    if not double_quant:
        return packed, QuantState(absmax.contiguous(), (out_f, in_f), blocksize, code=code)
    offset = absmax.to(torch.float64).mean().to(torch.float32)
    v = absmax - offset
    nb = v.numel()
    nb2 = -(-nb // blocksize2)
    pad = torch.zeros(nb2 * blocksize2, dtype=torch.float32, device=dev)
    pad[:nb] = v
    blocks = pad.reshape(nb2, blocksize2)
    absmax2 = blocks.abs().amax(dim=1)
    inv2 = torch.where(absmax2 > 0, 1.0 / absmax2, torch.zeros_like(absmax2))
    r2 = (blocks * inv2[:, None]).reshape(-1)[:nb]
    code2 = dynamic_code_map(dev)
    a8 = torch.bucketize(r2.double(), ((code2[:-1].double() + code2[1:].double()) / 2)).to(torch.uint8)
    state2 = QuantState(absmax2.contiguous(), (nb2,), blocksize2, quant_type="dynamic", code=code2)
    qs = QuantState(a8.contiguous(), (out_f, in_f), blocksize, code=code, nested=True,
                    offset=offset, state2=state2)
    return packed, qs


class Params4bit(torch.nn.Parameter):
    """uint8 packed NF4 weight with its ``quant_state`` attached."""

    def __new__(cls, data: torch.Tensor, quant_state: QuantState):
        self = super().__new__(cls, data, requires_grad=False)
        self.quant_state = quant_state
        return self

    def __deepcopy__(self, memo):
        return Params4bit(self.data.clone(), self.quant_state)


class Linear4bit(torch.nn.Module):
    """A 4-bit linear layer in bitsandbytes' storage format.

    Its forward goes through ``nf4gemv.matmul`` once ``nf4gemv.install()`` has
    patched the class; before that it raises, because this stack has no
    dequantise-and-matmul fallback of its own.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 compute_dtype=torch.bfloat16, device=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.compute_dtype = compute_dtype
        self.weight = None
        self.bias = torch.nn.Parameter(torch.zeros(out_features, dtype=compute_dtype, device=device),
                                       requires_grad=False) if bias else None

    @classmethod
    def from_float(cls, weight: torch.Tensor, *, blocksize: int = 64, double_quant: bool = True,
                   bias: torch.Tensor | None = None) -> "Linear4bit":
        out_f, in_f = weight.shape
        layer = cls(in_f, out_f, bias=bias is not None, device=weight.device)
        packed, qs = quantize_nf4(weight, blocksize, double_quant)
        layer.weight = Params4bit(packed, qs)
        if bias is not None:
            layer.bias.data.copy_(bias.to(layer.compute_dtype))
        return layer

    def forward(self, x):  # replaced by nf4gemv.install()
        raise RuntimeError("Linear4bit.forward needs nf4gemv.install() (the NF4 kernels)")


def scales_fp32(qs: QuantState) -> torch.Tensor:
    """The per-block fp32 scales the kernels reconstruct (plain: absmax;
    nested: code2[a8] * absmax2 + offset, two rounded fp32 ops)."""
    if not qs.nested:
        return qs.absmax.float()
    st2 = qs.state2
    b = torch.arange(qs.absmax.numel(), device=qs.absmax.device) // st2.blocksize
    prod = st2.code[qs.absmax.long()] * st2.absmax[b]
    off = qs.offset if isinstance(qs.offset, torch.Tensor) else torch.tensor(qs.offset)
    return prod + off.to(prod.device, torch.float32)
