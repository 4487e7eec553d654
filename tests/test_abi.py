"""The C-ABI library loads and exports exactly what include/*.h declares (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from fused_kernels_cutedsl_lib_b200 import _native

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^FK_API\s+[\w\s\*]+?\b(fk_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_header_matches_binding_table():
    assert _declared() == set(_native.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.fk_version() == 1


def test_argument_validation_before_launch():
    lib = _native.load()
    # head_dim 64 is rejected before anything touches CUDA
    rc = lib.fk_dec_attn_splitkv_fwd(16, 16, 16, 16, 16, 16, 1, 64, 8, 2, 64, 1, 1.0, None)
    assert rc == -1
    assert "head_dim" in lib.fk_last_error().decode()
    with pytest.raises(ValueError):
        _native.check(rc)
    # GQA group > 8
    assert lib.fk_dec_attn_splitkv_fwd(16, 16, 16, 16, 16, 16, 1, 64, 16, 1, 128, 1, 1.0, None) == -1
    # misaligned pointer
    assert lib.fk_dec_attn_splitkv_fwd(18, 16, 16, 16, 16, 16, 1, 64, 8, 2, 128, 1, 1.0, None) == -1


def test_chunk_rule():
    lib = _native.load()
    from fused_kernels_cutedsl_lib_b200 import chunk_tokens

    for L, s in [(4096, 16), (32768, 64), (100, 3), (1, 1), (65, 1)]:
        assert lib.fk_dec_attn_chunk_tokens(L, s) == chunk_tokens(L, s)
        assert chunk_tokens(L, s) % 64 == 0


def test_python_entry_points_reject_bad_tensors():
    from fused_kernels_cutedsl_lib_b200 import decode_attention

    q = torch.zeros(2, 1, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(2, 16, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        decode_attention(q.float(), k, k, torch.zeros(2, dtype=torch.int32))
    with pytest.raises(ValueError):  # CPU tensors
        decode_attention(q, k, k, torch.zeros(2, dtype=torch.int32))


def test_tvm_ffi_module_loads_and_exports():
    pytest.importorskip("tvm_ffi")
    from fused_kernels_cutedsl_lib_b200 import tvm_ffi_module

    mod = tvm_ffi_module.load()
    for name in ("dec_attn_splitkv_fwd", "dec_attn_combine", "dattn1", "skinny_gemm", "rmsnorm_linear",
                 "swiglu_gemm", "swiglu_gemm2", "lora_gemm", "prefill_attn", "dattn2", "linear_workspace_bytes",
                 "gemm", "gemm_tc", "swiglu2", "dec_attn_fused", "dec_attn_paged", "linear_kv_append"):
        assert getattr(mod, name) is not None


def test_new_entry_points_validate_before_launch():
    """Prefill attention, LoRA, fused KV append, output placement and the peer
    barrier reject bad arguments with a status, before any CUDA call."""
    lib = _native.load()
    # prefill: head_dim 96
    assert lib.fk_prefill_attn_fwd(16, 16, 16, 16, None, 1, 2, 2, 8, 8, 96, 0.1, None) == -1
    assert "head_dim" in lib.fk_last_error().decode()
    # prefill: q heads not a multiple of kv heads
    assert lib.fk_prefill_attn_fwd(16, 16, 16, 16, None, 1, 3, 2, 8, 8, 64, 0.1, None) == -1
    # LoRA: rank 12 is not a multiple of 8
    assert lib.fk_lora_linear(16, 16, 16, 16, None, 16, 4, 128, 128, 12, 256, 1 << 20, None) == -1
    assert "rank" in lib.fk_last_error().decode()
    # fused KV append: next lengths may not alias the input lengths
    assert lib.fk_linear_kv_append(16, None, 16, 16, 4, 1536, 512, 0.0, 16, 16, None, 32, 32, 512, 1024, 2, 128,
                                   64, 0, 256, 1 << 20, None) == -1
    assert "alias" in lib.fk_last_error().decode()
    # fused KV append: K and V column ranges overlap
    assert lib.fk_linear_kv_append(16, None, 16, 16, 4, 1536, 512, 0.0, 16, 16, None, 32, 48, 512, 600, 2, 128,
                                   64, 0, 256, 1 << 20, None) == -1
    # output placement: too many peers, ldy < N
    assert lib.fk_linear_ex(16, None, 16, None, 0, None, 0, 16, 0, None, 8, 4, 128, 128, 0.0, 256, 1 << 20,
                            None) == -1
    assert lib.fk_linear_ex(16, None, 16, None, 0, None, 0, 16, 64, None, 0, 4, 128, 128, 0.0, 256, 1 << 20,
                            None) == -1
    # peer barrier: 9 ranks
    arr = (ctypes.c_void_p * 9)(*([16] * 9))
    assert lib.fk_peer_barrier(16, 16, arr, 0, 9, None) == -1
    # attention with lengths commit aliasing the lengths
    assert lib.fk_dec_attn_fwd_commit(16, 4096, 16, 16, None, 32, 32, 16, 16, 16, 16, 1, 64, 0, 0, 32, 8, 128, 1,
                                      0.1, None) != 0
