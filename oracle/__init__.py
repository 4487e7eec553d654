"""CPU oracle for the decode-step hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in fp32 torch on the CPU, the reference's own torch
check paths for every kernel on the path. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it, and only as the checker or the timed CPU baseline: the product path
(``fused_kernels_cutedsl_lib_b200``) never calls it and has no CPU fallback.

Parity pinning: the reference ships no golden vectors or fixtures (its checks
regenerate ``torch.randn`` inputs and compare live). The oracle is pinned
against fixtures that ``tests/golden/make_golden.py`` produced by executing the
reference's own torch check functions, extracted from the reference sources,
in float64 on the CPU (see ``tests/test_oracle_golden.py``).
"""
from .ops import (
    dattn1_reference,
    decode_attention,
    decode_layer,
    linear,
    lora_linear,
    prefill_attention,
    rmsnorm,
    rmsnorm_linear,
    silu,
    swiglu,
    swiglu_separate,
)

__all__ = [
    "dattn1_reference",
    "decode_attention",
    "decode_layer",
    "lora_linear",
    "prefill_attention",
    "linear",
    "rmsnorm",
    "rmsnorm_linear",
    "silu",
    "swiglu",
    "swiglu_separate",
]
