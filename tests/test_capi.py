"""The C ABI library loads on a CPU-only machine, exports every symbol the
header declares, and rejects bad arguments on the host with a status and a
message - before it ever needs a GPU."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from ttspipe_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "nf4b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\w[\w\s\*]*?\b(nf4b_\w+)\s*\(", text, flags=re.M))


def test_header_and_binding_agree():
    assert declared_symbols() == set(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (nf4b_\w+)", out))
    missing = declared_symbols() - exported
    assert not missing, missing
    assert lib.nf4b_version() >= 100


def _weight(**kw):
    w = _lib.Nf4Weight()
    buf = ctypes.create_string_buffer(4096 + 16)
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    w.packed, w.absmax = base, base
    w.n_out, w.k_in, w.blocksize, w.blocksize2, w.nested = 64, 256, 64, 256, 0
    for k, v in kw.items():
        setattr(w, k, v)
    return w, buf


@pytest.mark.parametrize("field,value,status", [
    ("blocksize", 96, -2),      # not a power of two (tests/test_nf4gemv.py:207-221)
    ("blocksize", 32, -2),      # below 64
    ("k_in", 100, -2),          # not a multiple of the blocksize
    ("n_out", 0, -2),           # empty
    ("nested", 1, -1),          # nested without codes
])
def test_gemm_rejects_bad_weights_on_the_host(field, value, status):
    w, _keep = _weight(**{field: value})
    x = ctypes.create_string_buffer(1024)
    st = _lib.lib().nf4b_gemm(ctypes.byref(w), ctypes.addressof(x), ctypes.addressof(x), 1, 0,
                              None, None, 0, None)
    assert st == status
    assert _lib.last_error()


def test_gemm_rejects_misaligned_packed_weight():
    w, _keep = _weight()
    w.packed = w.packed + 1
    st = _lib.lib().nf4b_gemm(ctypes.byref(w), w.absmax, w.absmax, 1, 0, None, None, 0, None)
    assert st == _lib_err("ALIGN")


def _lib_err(name):
    return {"ARG": -1, "SHAPE": -2, "ALIGN": -3, "DTYPE": -4, "WORKSPACE": -5, "LAUNCH": -6,
            "DEVICE": -7}[name]


def test_gemm_rejects_null_and_unknown_epilogue():
    w, _keep = _weight()
    L = _lib.lib()
    assert L.nf4b_gemm(None, None, None, 1, 0, None, None, 0, None) == -1
    assert L.nf4b_gemm(ctypes.byref(w), None, w.absmax, 1, 0, None, None, 0, None) == -1
    assert L.nf4b_gemm(ctypes.byref(w), w.absmax, w.absmax, 1, 7, None, None, 0, None) == -1
    assert L.nf4b_gemm(ctypes.byref(w), w.absmax, w.absmax, 1, 1, None, None, 0, None) == -1
    assert L.nf4b_gemm(ctypes.byref(w), w.absmax, w.absmax, 0, 0, None, None, 0, None) == -2


def test_workspace_size_grows_with_rows_and_is_zero_for_the_gemm_path():
    w, _keep = _weight(n_out=9728, k_in=2560)
    L = _lib.lib()
    s1 = L.nf4b_gemm_workspace_size(ctypes.byref(w), 1)
    s8 = L.nf4b_gemm_workspace_size(ctypes.byref(w), 8)   # the decode GEMV's partial sums grow with rows
    assert 0 < s1 < s8
    assert L.nf4b_gemm_workspace_size(ctypes.byref(w), 33) == 0
    assert L.nf4b_decode_attention_workspace_size(32, 128, 2048) > 0


@pytest.mark.parametrize("n,k", [(1024, 2560), (9728, 2560), (6144, 2560), (2560, 9728)])
def test_prepare_sizes_the_decode_workspace_for_every_decode_row_count(n, k):
    """`prepare` sizes the shared decode workspace once, before any capture; it
    must cover 1..MAX_N rows, whose largest need may come from the GEMV's
    partial sums (few rows) rather than the GEMM's split-K sums (MAX_N rows)."""
    from ttspipe_b200 import nf4gemv

    w, _keep = _weight(n_out=n, k_in=k, nested=1)
    w.absmax_code = w.code2 = w.absmax
    size = _lib.lib().nf4b_gemm_workspace_size
    needs = [int(size(ctypes.byref(w), r)) for r in range(1, nf4gemv.MAX_N + 1)]
    assert nf4gemv.decode_workspace_bytes(w) == max(needs) > 0
    if (n, k) in ((1024, 2560), (9728, 2560)):
        assert max(needs) > needs[-1]       # sizing for MAX_N rows alone would fall short


def test_other_entry_points_reject_bad_arguments():
    L = _lib.lib()
    buf = ctypes.create_string_buffer(4096 + 16)
    p = (ctypes.addressof(buf) + 15) // 16 * 16
    assert L.nf4b_rms_norm(None, p, p, 1, 8, 1e-6, None) == -1
    assert L.nf4b_rms_norm(p, p, p, 0, 8, 1e-6, None) == -2
    assert L.nf4b_rope(p, p, 9, p, 1, 1, 1, 8, None) == -4
    assert L.nf4b_rope(p, p, 0, p, 1, 1, 1, 7, None) == -2
    assert L.nf4b_qk_rope_kv(p, None, None, 1e-6, p, 2, p, p, p, p, 32, 8, 64, 16, None) == -2
    assert L.nf4b_qk_rope_kv(p, p, None, 1e-6, p, 2, p, p, p, p, 32, 8, 128, 16, None) == -1
    assert L.nf4b_decode_attention(p, p, p, p, None, p, 32, 8, 64, 16, 16, p, 1 << 20, None) == -2
    assert L.nf4b_decode_attention(p, p, p, p, None, p, 12, 8, 128, 16, 16, p, 1 << 20, None) == -2
    assert L.nf4b_decode_attention(p, p, p, p, None, p, 32, 8, 128, 16, 32, p, 1 << 20, None) == -2
    assert L.nf4b_decode_attention(p, p, p, p, None, p, 32, 8, 128, 16, 16, p, 16, None) == -5
    assert L.nf4b_dequantize(None, p, None) == -1


def test_misaligned_element_pointers_are_refused_on_the_host():
    """Every pointer a kernel dereferences is checked for its element's
    alignment (2 bytes for bf16/fp16, 4 for an fp32 rotary table, 8 for int64
    positions, steps and token ids) and refused with NF4B_ERR_ALIGN before any
    device work: a C caller's misaligned pointer becomes a status, not a fault.
    Every call below is one the host must refuse."""
    L = _lib.lib()
    buf = ctypes.create_string_buffer(1 << 16)
    p = (ctypes.addressof(buf) + 255) // 256 * 256          # 256-byte aligned
    odd, two, four = p + 1, p + 2, p + 4                    # aligned to 1, 2 and 4 bytes
    ALIGN = _lib_err("ALIGN")
    assert L.nf4b_rms_norm(odd, p, p, 1, 8, 1e-6, None) == ALIGN
    assert L.nf4b_rms_norm(p, odd, p, 1, 8, 1e-6, None) == ALIGN
    assert L.nf4b_rope(p, two, _lib.NF4B_F32, p, 1, 1, 1, 8, None) == ALIGN       # fp32 table
    assert L.nf4b_rope(p, odd, _lib.NF4B_BF16, p, 1, 1, 1, 8, None) == ALIGN
    assert L.nf4b_qk_rope_kv(p, None, None, 1e-6, p, 2, four, p, p, p, 32, 8, 128, 16, None) == ALIGN  # pos
    assert L.nf4b_qk_rope_kv(p, None, None, 1e-6, two, 0, p, p, p, p, 32, 8, 128, 16, None) == ALIGN  # freqs
    assert L.nf4b_qk_rope_kv(odd, None, None, 1e-6, p, 2, p, p, p, p, 32, 8, 128, 16, None) == ALIGN  # qkv
    assert L.nf4b_decode_attention(p, p, p, four, None, p, 32, 8, 128, 16, 16, p, 1 << 20, None) == ALIGN
    assert L.nf4b_decode_attention(p, p, p, p, None, odd, 32, 8, 128, 16, 16, p, 1 << 20, None) == ALIGN
    assert L.nf4b_qkv_attention(odd, None, None, 1e-6, p, 2, p, p, p, p, p, 32, 8, 128, 16, 16, p, 1 << 20,
                                None) == ALIGN
    assert L.nf4b_qkv_attention(p, None, None, 1e-6, p, 2, four, p, p, p, p, 32, 8, 128, 16, 16, p, 1 << 20,
                                None) == ALIGN
    need = L.nf4b_sample_workspace_size(1000)
    assert 0 < need <= (1 << 16) - 512
    assert L.nf4b_sample(p, 1000, 1.0, 0.9, 50, 1, four, p + 256, p + 256, need, None) == ALIGN  # step
    assert L.nf4b_sample(p, 1000, 1.0, 0.9, 50, 1, p, four, p + 256, need, None) == ALIGN        # out
    assert L.nf4b_frame_select(four, p, p, 4, 0, 16, p, p, 8, p, None) == ALIGN
    assert L.nf4b_frame_select(p, p, p, 4, 0, 16, four, p, 8, p, None) == ALIGN
    assert L.nf4b_frame_advance(p, 16, p, 16, 2, four, 8, p, p, 4, p, p, None) == ALIGN
    assert L.nf4b_frame_advance(p, 16, p, 16, 2, p, 8, p, p, 4, p, four, None) == ALIGN
    assert "aligned" in _lib.last_error()
    # the wqkv GEMV's fused rotary store: 4 query heads + 2 x 1 KV head of 128 outputs
    w, _keep = _weight(n_out=(4 + 2) * 128, k_in=256)
    rk = _lib.RopeKv(two, _lib.NF4B_F32, p, p, p, p, 4, 1, 16)           # fp32 table on 2 bytes
    assert L.nf4b_gemm_qkv_rope(ctypes.byref(w), p, p, ctypes.byref(rk), p, 1 << 16, None, None) == ALIGN
    rk = _lib.RopeKv(p, _lib.NF4B_BF16, four, p, p, p, 4, 1, 16)         # pos on 4 bytes
    assert L.nf4b_gemm_qkv_rope(ctypes.byref(w), p, p, ctypes.byref(rk), p, 1 << 16, None, None) == ALIGN


def test_empty_inputs_and_sizes_past_each_maximum_are_refused_on_the_host():
    """Empty inputs and sizes past an entry point's maximum return a status
    before any device work: a 262144-entry vocabulary, 32 codebooks, 1024 KV
    heads, 40 chained and 152 decode-step jobs (the persistent launches'
    parameter blocks) and the dense head's four input widths."""
    L = _lib.lib()
    buf = ctypes.create_string_buffer(1 << 16)
    p = (ctypes.addressof(buf) + 255) // 256 * 256
    SHAPE, ARG = _lib_err("SHAPE"), _lib_err("ARG")
    assert L.nf4b_sample_workspace_size(0) == 0
    assert L.nf4b_sample_workspace_size(262144) > 0
    assert L.nf4b_sample_workspace_size(262145) == 0
    assert L.nf4b_sample(p, 262145, 1.0, 0.9, 50, 1, p, p, p, 1 << 16, None) == SHAPE
    assert L.nf4b_sample(p, 0, 1.0, 0.9, 50, 1, p, p, p, 1 << 16, None) == SHAPE
    assert L.nf4b_frame_advance(p, 16, p, 16, 33, p, 8, p, p, 4, p, p, None) == SHAPE
    assert L.nf4b_decode_attention(p, p, p, p, None, p, 1025, 1025, 128, 16, 16, p, 1 << 20, None) == SHAPE
    jobs = (_lib.ChainJob * 153)()
    assert L.nf4b_gemv_chain(jobs, 41, 1, p, 1 << 16, None) == SHAPE
    assert L.nf4b_gemv_chain(jobs, 0, 1, p, 1 << 16, None) == ARG
    assert L.nf4b_gemv_chain_workspace_size(jobs, 41, 1) == 0
    assert L.nf4b_decode_step(jobs, 153, 1, p, 1 << 16, None) == SHAPE
    assert L.nf4b_decode_step(None, 1, 1, p, 1 << 16, None) == ARG
    assert L.nf4b_decode_step_workspace_size(jobs, 153, 1) == 0
    assert L.nf4b_embed_rows(p, 16, p, 0, 8, p, None) == SHAPE
    assert L.nf4b_dense_gemv(p, p, p, 16, 3072, None, 0.0, None) == SHAPE
    assert L.nf4b_dense_gemv(p, p, p, 0, 2560, None, 0.0, None) == SHAPE


def test_activation_dtypes_are_checked_on_the_host():
    """bf16 (0 or NF4B_BF16) and fp16 (NF4B_F16) are the activation types;
    anything else is NF4B_ERR_DTYPE before any device work."""
    w, _keep = _weight()
    L = _lib.lib()
    buf = ctypes.create_string_buffer(4096 + 16)
    p = (ctypes.addressof(buf) + 15) // 16 * 16
    opts = _lib.GemmOpts(None, None, None, 0.0, 3)    # 0 (zeroed options) means bf16
    assert L.nf4b_gemm_ex(ctypes.byref(w), p, p, 1, 0, None, None, 0, ctypes.byref(opts), None) == -4
    opts.dtype = 9
    assert L.nf4b_gemm_ex(ctypes.byref(w), p, p, 1, 0, None, None, 0, ctypes.byref(opts), None) == -4
    assert L.nf4b_rms_norm_ex(p, p, p, 1, 8, 1e-6, _lib.NF4B_F32, None) == -4
    assert L.nf4b_rope_ex(p, p, 0, p, 1, 1, 1, 8, 3, None) == -4
    assert L.nf4b_qk_rope_kv_ex(p, None, None, 1e-6, p, 2, p, p, p, p, 32, 8, 128, 16, 0, None) == -4
    assert L.nf4b_decode_attention_ex(p, p, p, p, None, p, 32, 8, 128, 16, 16, p, 1 << 20, -1, None) == -4
    assert L.nf4b_qkv_attention_ex(p, None, None, 1e-6, p, 2, p, p, p, p, p, 32, 8, 128, 16, 16, p, 1 << 20, 0,
                                   None) == -4
    # the argument checks still come first for a valid dtype
    assert L.nf4b_rms_norm_ex(None, p, p, 1, 8, 1e-6, _lib.NF4B_F16, None) == -1
