"""Parity of the tcgen05 prefill attention (FlashSM90 replacement) against the CPU oracle (GPU)."""
import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import FlashSM90, _native, flash_attention

pytestmark = pytest.mark.gpu

# bf16 output vs fp32 oracle: absolute bounds (outputs are softmax averages of
# V, |out| <~ 3 here), natural-log LSE within 1e-3.
MAX_ERR = 2e-2
MEAN_ERR = 2e-3
LSE_ERR = 1e-3


def _inputs(B, H, Hkv, Lq, Lkv, D, seed, shift=0.5):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(B, H, Lq, D, generator=g, device="cuda") + shift).bfloat16()
    k = (torch.randn(B, Hkv, Lkv, D, generator=g, device="cuda") + shift).bfloat16()
    v = (torch.randn(B, Hkv, Lkv, D, generator=g, device="cuda") + shift).bfloat16()
    return q, k, v


def _check(out, lse, ref_out, ref_lse):
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    o = out.float().cpu()
    assert torch.isfinite(o).all()
    e = (o - ref_out).abs()
    assert e.max().item() <= MAX_ERR, e.max().item()
    assert e.mean().item() <= MEAN_ERR, e.mean().item()
    if lse is not None:
        assert (lse.cpu() - ref_lse).abs().max().item() <= LSE_ERR


@pytest.mark.parametrize("name", ["prefill_d64", "prefill_d128"])
def test_golden(golden, name):
    g = golden(name)
    out, lse = flash_attention(g["q"].cuda(), g["k"].cuda(), g["v"].cuda(), return_lse=True)
    _check(out, lse, g["out"], g["lse"])


@pytest.mark.parametrize("shape", [
    (2, 4, 4, 256, 256, 64),
    (2, 4, 4, 256, 384, 128),
    (1, 8, 2, 100, 300, 128),   # GQA 4, ragged q and kv tails
    (1, 2, 2, 1, 1, 64),        # one query, one key
    (2, 2, 1, 129, 127, 64),    # tails on both sides
    (1, 2, 2, 128, 2048, 64),   # long kv loop (16 tiles)
])
def test_matches_oracle(shape):
    B, H, Hkv, Lq, Lkv, D = shape
    q, k, v = _inputs(B, H, Hkv, Lq, Lkv, D, seed=sum(shape))
    out, lse = flash_attention(q, k, v, return_lse=True)
    ref_out, ref_lse = oracle.prefill_attention(q, k, v)
    _check(out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("D", [64, 128])
def test_running_max_rescale(D):
    # Keys grow along the sequence so the row max rises by more than 2^8 (log2
    # units) across tiles: exercises the O rescale in TMEM.
    B, H, L = 1, 2, 1024
    q, k, v = _inputs(B, H, H, 128, L, D, seed=3, shift=0.0)
    ramp = torch.linspace(0.0, 6.0, L, device="cuda").view(1, 1, L, 1)
    k = (q[:, :, :1, :].float() * ramp + 0.1 * k.float()).bfloat16()
    out, lse = flash_attention(q, k, v, return_lse=True)
    ref_out, ref_lse = oracle.prefill_attention(q, k, v)
    _check(out, lse, ref_out, ref_lse)


def test_custom_scale_and_kernel_object():
    q, k, v = _inputs(1, 2, 2, 256, 200, 64, seed=5)
    o = torch.empty_like(q)
    FlashSM90(qk_mn=(128, 256), num_stages=3, cluster_size_m=1)(q, k, v, o, 0.3)
    ref_out, _ = oracle.prefill_attention(q, k, v, softmax_scale=0.3)
    _check(o, None, ref_out, None)


def test_deterministic():
    q, k, v = _inputs(2, 2, 2, 384, 512, 128, seed=6)
    a = flash_attention(q, k, v)
    b = flash_attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("D", [64, 128])
def test_reference_test_size(D):
    # The reference's FlashSM90 test size (tests.py:138-154): bs 16, heads 16,
    # 4096 x 4096. Two heads against the oracle, all heads against torch SDPA.
    B, H, L = 16, 16, 4096
    q, k, v = _inputs(B, H, H, L, L, D, seed=D)
    out = flash_attention(q, k, v)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    for b, h in ((0, 0), (15, 15)):
        ref_out, _ = oracle.prefill_attention(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1])
        e = (out[b:b + 1, h:h + 1].float().cpu() - ref_out).abs()
        assert e.max().item() <= MAX_ERR and e.mean().item() <= MEAN_ERR
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    assert (out.float() - sdpa.float()).abs().max().item() <= 2 * MAX_ERR


def test_argument_errors():
    q, k, v = _inputs(1, 2, 2, 64, 64, 64, seed=1)
    with pytest.raises(ValueError):
        flash_attention(q, k[:, :, :, :32].contiguous(), v[:, :, :, :32].contiguous())
    q96 = torch.zeros(1, 2, 64, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        flash_attention(q96, q96, q96)
    with pytest.raises(ValueError):
        flash_attention(q, k, v, softmax_scale=0.0)
    q3 = torch.zeros(1, 3, 64, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        flash_attention(q3, k, v)  # 3 q heads over 2 kv heads


def test_tvm_ffi_prefill_matches_ctypes():
    """The TVM-FFI export (FlashSM90's call shape, torch tensors in) gives the ctypes path's result."""
    pytest.importorskip("tvm_ffi")
    from fused_kernels_cutedsl_lib_b200 import tvm_ffi_module

    mod = tvm_ffi_module.load()
    q, k, v = _inputs(1, 4, 2, 200, 300, 128, seed=9)
    o = torch.empty_like(q)
    mod.prefill_attn(q, k, v, o, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(o, flash_attention(q, k, v))
