"""B200-native (sm_100a) NF4 hot path of ttspipe: decode GEMV, tcgen05 prefill
GEMM, fused RMSNorm/rotary/KV write and split-KV decode attention, behind the
reference's Python entry points (``nf4gemv``, ``fusedops``, ``fusedlayer``,
``fastpath``) and the C ABI in ``include/nf4b200.h``."""

__version__ = "0.1.0"
