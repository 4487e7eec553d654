"""Parity of the composed decode step (QKV, KV append, attention, O-proj, SwiGLU FFN) on one GPU."""
import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import _native
from fused_kernels_cutedsl_lib_b200.layer import DecodeLayer, random_layer_weights

pytestmark = pytest.mark.gpu

# Each stage, fed the kernel's own inputs, must meet the per-kernel bound
# (scaled error max 2e-2, mean 2e-3). End to end the two chains round four
# bf16 hand-offs independently; a one-ulp difference in the SwiGLU output
# (~0.008 at |gu| ~ 2) summed over K = 14336 with W ~ N(0, 0.02) gives ~0.01
# std in y (mean |err| ~ 0.008), so the chained comparison allows 5e-2 max
# and 1e-2 mean.
MAX_ERR = 2e-2
MEAN_ERR = 2e-3
CHAIN_MAX_ERR = 5e-2
CHAIN_MEAN_ERR = 1e-2


def _close(out, ref, max_err=MAX_ERR, mean_err=MEAN_ERR):
    out, ref = out.float().cpu(), ref.float().cpu()
    assert torch.isfinite(out).all()
    e = (out - ref).abs() / ref.abs().clamp_min(1.0)
    assert e.max().item() <= max_err, e.max().item()
    assert e.mean().item() <= mean_err, e.mean().item()


def _stagewise(layer, x, k, v, lens_after, w, hq, hkv, eps=1e-6):
    """Every stage against the oracle applied to the kernel's own inputs for that stage."""
    b = layer.buffers(x.shape[0], k.shape[1], x.device)
    wd = w.as_dict()
    _close(b["qkv"], oracle.rmsnorm_linear(x, wd["gamma_attn"], wd["w_qkv"], eps))
    q = b["qkv"][:, :hq * 128].reshape(-1, hq, 128)
    ref_attn, _ = oracle.decode_attention(q, k, v, lens_after)
    _close(b["attn"], ref_attn.reshape(b["attn"].shape))
    _close(b["h"], oracle.linear(b["attn"], wd["w_o"]) + x.float().cpu())
    _close(b["gu"], oracle.swiglu(oracle.rmsnorm(b["h"], wd["gamma_ffn"], eps), wd["w_gate_up"]))
    _close(b["y"], oracle.linear(b["gu"], wd["w_down"]) + b["h"].float().cpu())


def _run(B, L, lens, hidden, ffn, hq, hkv, seed=0):
    w = random_layer_weights(hidden, ffn, hq, hkv, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    x = torch.randn(B, hidden, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, L, hkv, 128, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, L, hkv, 128, generator=g, device="cuda").bfloat16()
    lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ref, k_new, v_new, ref_lens = oracle.decode_layer(x, w.as_dict(), k, v, lens, num_heads_q=hq, num_heads_kv=hkv)
    layer = DecodeLayer(w, hq, hkv)
    lens_before = lens.clone()
    y = layer(x, k, v, lens)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _close(y, ref, CHAIN_MAX_ERR, CHAIN_MEAN_ERR)
    assert torch.equal(lens.cpu(), ref_lens)
    _stagewise(layer, x, k, v, lens, w, hq, hkv)
    for b in range(B):  # the appended rows are the projection's K/V (bf16-rounded like the kernel's output)
        pos = int(lens_before[b])
        assert (k[b, pos].float().cpu() - k_new[b]).abs().max() < 0.05
        assert (v[b, pos].float().cpu() - v_new[b]).abs().max() < 0.05
    return layer, x, k, v, lens


def test_small_layer_ragged():
    _run(B=3, L=300, lens=[0, 100, 299], hidden=512, ffn=1024, hq=4, hkv=2)


def test_llama_dims_skinny_path():
    _run(B=16, L=512, lens=[511] * 8 + [100] * 8, hidden=4096, ffn=14336, hq=32, hkv=8, seed=3)


def test_llama_dims_tensor_core_path():
    _run(B=128, L=260, lens=[256] * 128, hidden=4096, ffn=14336, hq=32, hkv=8, seed=4)


def test_two_steps_and_full_cache():
    layer, x, k, v, lens = _run(B=2, L=64, lens=[62, 63], hidden=512, ffn=1024, hq=4, hkv=2, seed=7)
    y2 = layer(x, k, v, lens)  # row 1 is now full: it attends but is not appended again
    torch.cuda.synchronize()
    assert lens.cpu().tolist() == [64, 64]
    assert torch.isfinite(y2.float()).all()
