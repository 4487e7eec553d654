"""Pin the CPU oracle against fixtures made by executing the reference's own torch checks."""
import torch

import oracle


def _close(a, b, tol=1e-4):
    a, b = a.float(), b.float()
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin)
    assert torch.equal(a[~fin], b[~fin])
    assert (a[fin] - b[fin]).abs().max().item() <= tol * max(1.0, b[fin].abs().max().item())


def test_attention_goldens(golden):
    for name in ("attn_gqa4_ragged", "attn_gqa8", "attn_mha"):
        g = golden(name)
        out, lse = oracle.decode_attention(g["q"], g["k_cache"], g["v_cache"], g["cache_seqlens"])
        _close(out, g["out"])
        _close(lse, g["lse"])


def test_empty_row_is_zero_and_neg_inf(golden):
    g = golden("attn_gqa4_ragged")
    assert int(g["cache_seqlens"][3]) == 0
    out, lse = oracle.decode_attention(g["q"], g["k_cache"], g["v_cache"], g["cache_seqlens"])
    assert torch.all(out[3] == 0) and torch.all(torch.isneginf(lse[3]))


def test_prefill_goldens(golden):
    for name in ("prefill_d64", "prefill_d128"):
        g = golden(name)
        out, lse = oracle.prefill_attention(g["q"], g["k"], g["v"])
        _close(out, g["out"])
        _close(lse, g["lse"])


def test_gemm_goldens(golden):
    g = golden("skinny_gemm")
    _close(oracle.linear(g["x"], g["w"]), g["y"])
    g = golden("rmsnorm_linear")
    _close(oracle.rmsnorm_linear(g["x"], None, g["w"], eps=g["eps"]), g["y"])
    g = golden("swiglu")
    _close(oracle.swiglu(g["x"], g["w_gate_up"]), g["y"])
    g = golden("swiglu_two_weights")
    _close(oracle.swiglu_separate(g["x"], g["b"], g["b1"]), g["y"])
    g = golden("dattn1")
    _close(oracle.dattn1_reference(g["Q"], g["K"], g["V"]), g["O"])
    g = golden("lora")
    _close(oracle.lora_linear(g["x"], g["w"], g["lora_a"], g["lora_b"]), g["y"])


def test_swiglu_forms_agree(golden):
    g = golden("swiglu")
    n = g["w_gate_up"].shape[0] // 2
    a = oracle.swiglu(g["x"], g["w_gate_up"])
    b = oracle.swiglu_separate(g["x"], g["w_gate_up"][:n], g["w_gate_up"][n:])
    assert torch.allclose(a, b)
