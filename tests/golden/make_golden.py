"""Generate the golden fixtures in this folder from the reference's own torch code.

The reference (dungwoong/fused_kernels_cutedsl_lib) ships no golden vectors,
and its modules cannot be imported without a GPU (``STREAM = ...`` runs at
import time, python/cdsl_helpers/cdsl_fn_utils.py:19). Its correctness checks
are plain torch functions and statements inside its demo and ``__main__``
blocks. This script parses those reference source files with ``ast``, takes
exactly the check functions/statements listed in ``SOURCES`` (decorators
such as ``@torch.compile`` dropped), executes them on the CPU in float64 on
seeded bf16-representable inputs, and saves inputs + outputs as ``*.pt``.

It runs only where the reference checkout exists (``--ref``, default
``$FK_REFERENCE_DIR``); the fixtures it writes are
committed so the tests never need the reference.

    python tests/golden/make_golden.py [--ref PATH]
"""
from __future__ import annotations

import argparse
import ast
import math
import os
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent

# fixture -> (reference file, kind, names)
SOURCES = {
    "attn_reimpl": ("python/cutedsl_kernels/attn/attempt6_epi_pipeline/attn.py", "def", "attn_reimpl"),
    "torch_swiglu": ("demo/swiglu.py", "def", "torch_swiglu"),
    "swiglu_two_weights": ("python/cutedsl_kernels/swiglu/attempt1/gemm2.py", "def", "torch_gemm"),
    "skinny_gemm": ("demo/skinny_gemm_test.py", "def", "gemm"),
    "dattn1_check": ("demo/dec_attn_second_part.py", "def", "torch_fn"),
    "rmsnorm_linear": ("python/cutedsl_kernels/rmsnorm_linear/attempt1/gemm.py", "assign", ("norm_a", "ref")),
    "lora": ("python/cutedsl_kernels/lora/attempt1/gemm.py", "def", "torch_lora"),
}


def _find_def(tree: ast.AST, name: str) -> ast.FunctionDef:
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == name:
            node.decorator_list = []
            return node
    raise LookupError(name)


def _find_assigns(tree: ast.AST, names: tuple) -> list[ast.stmt]:
    out = []
    for target in names:
        for node in ast.walk(tree):
            if (isinstance(node, ast.Assign) and len(node.targets) == 1
                    and isinstance(node.targets[0], ast.Name) and node.targets[0].id == target):
                out.append(node)
                break
        else:
            raise LookupError(target)
    return out


def load_reference_code(ref: Path, key: str, namespace: dict):
    """Exec the named reference function (or statements) into ``namespace``."""
    rel, kind, names = SOURCES[key]
    src = (ref / rel).read_text()
    tree = ast.parse(src)
    if kind == "def":
        body = [_find_def(tree, names)]
    else:
        body = _find_assigns(tree, names)
    mod = ast.Module(body=body, type_ignores=[])
    ast.fix_missing_locations(mod)
    exec(compile(mod, f"<reference:{rel}>", "exec"), namespace)
    return namespace


def _ns(**kw):
    ns = {"torch": torch, "math": math, "F": F}
    ns.update(kw)
    return ns


def _bf16_randn(gen, *shape, std=1.0):
    return (torch.randn(*shape, generator=gen, dtype=torch.float64) * std).to(torch.bfloat16)


def make_attention(ref: Path, gen, B, Hq, Hkv, Lmax, lens, name):
    D = 128
    q = _bf16_randn(gen, B, 1, Hq, D)
    k = _bf16_randn(gen, B, Lmax, Hkv, D)
    v = _bf16_randn(gen, B, Lmax, Hkv, D)
    seqlens = torch.tensor(lens, dtype=torch.int32)
    ns = load_reference_code(ref, "attn_reimpl", _ns())
    attn_reimpl = ns["attn_reimpl"]
    G = Hq // Hkv
    out = torch.zeros(B, Hq, D, dtype=torch.float64)
    lse = torch.full((B, Hq), float("-inf"), dtype=torch.float64)
    scale = D ** -0.5
    for b in range(B):
        L = int(lens[b])
        if L == 0:
            continue  # no keys: the zero-row-sum guard gives out = 0, lse = -inf
        qb = q[b].double().permute(1, 0, 2).unsqueeze(0)  # [1, Hq, 1, D]
        kb = k[b, :L].double().permute(1, 0, 2).repeat_interleave(G, dim=0).unsqueeze(0)  # [1, Hq, L, D]
        vb = v[b, :L].double().permute(1, 0, 2).repeat_interleave(G, dim=0).unsqueeze(0)
        out[b] = attn_reimpl(qb, kb, vb)[0, :, 0, :]
        # The reference kernels keep no LSE; it is the logsumexp of the same scaled scores.
        lse[b] = torch.logsumexp((qb @ kb.transpose(2, 3))[0, :, 0, :] * scale, dim=-1)
    torch.save({"q": q, "k_cache": k, "v_cache": v, "cache_seqlens": seqlens,
                "out": out.float(), "lse": lse.float(), "source": SOURCES["attn_reimpl"][0]},
               HERE / f"{name}.pt")


def make_gemms(ref: Path, gen):
    # skinny GEMM: demo/skinny_gemm_test.py `gemm(a, b) = a @ b.t()`
    x = _bf16_randn(gen, 5, 256)
    w = _bf16_randn(gen, 96, 256, std=0.02)
    ns = load_reference_code(ref, "skinny_gemm", _ns())
    y = ns["gemm"](x.double(), w.double())
    torch.save({"x": x, "w": w, "y": y.float(), "source": SOURCES["skinny_gemm"][0]},
               HERE / "skinny_gemm.pt")

    # RMSNorm -> linear: the statements `norm_a = rms_norm(a.float(), (k,), eps=1e-5)` and
    # `ref = (norm_a @ b.t().float()).to(bf16)`; run in float64 by handing in
    # float64 tensors and neutralising the final bf16 cast.
    a = _bf16_randn(gen, 3, 256)
    b = _bf16_randn(gen, 64, 256, std=0.02)
    k = 256
    ns = _ns(a=a.double(), b=b.double(), k=k)

    class _NoCast:  # `x.to(torch.float32)` / `.to(torch.bfloat16)` keep float64 here
        float32 = torch.float64
        bfloat16 = torch.float64

        def __getattr__(self, item):
            return getattr(torch, item)

    ns["torch"] = _NoCast()
    load_reference_code(ref, "rmsnorm_linear", ns)
    torch.save({"x": a, "w": b, "eps": 1e-5, "y": ns["ref"].float(),
                "source": SOURCES["rmsnorm_linear"][0]}, HERE / "rmsnorm_linear.pt")

    # SwiGLU with the concatenated gate/up weight: demo/swiglu.py torch_swiglu(a, bb1)
    x = _bf16_randn(gen, 4, 128)
    wgu = _bf16_randn(gen, 96, 128, std=0.05)
    ns = load_reference_code(ref, "torch_swiglu", _ns())
    y = ns["torch_swiglu"](x.double(), wgu.double())
    torch.save({"x": x, "w_gate_up": wgu, "y": y.float(), "source": SOURCES["torch_swiglu"][0]},
               HERE / "swiglu.pt")

    # SwiGLU with two weights: gemm2.py torch_gemm() over globals a, b, b1
    x = _bf16_randn(gen, 3, 128)
    b_ = _bf16_randn(gen, 40, 128, std=0.05)
    b1 = _bf16_randn(gen, 40, 128, std=0.05)
    ns = load_reference_code(ref, "swiglu_two_weights", _ns(a=x.double(), b=b_.double(), b1=b1.double()))
    y = ns["torch_gemm"]()
    torch.save({"x": x, "b": b_, "b1": b1, "y": y.float(), "source": SOURCES["swiglu_two_weights"][0]},
               HERE / "swiglu_two_weights.pt")

    # DAttn1 check: (Q @ K^T) @ Vt with V stored [H, D, P]
    Q = _bf16_randn(gen, 2, 16, 128)
    K = _bf16_randn(gen, 2, 64, 128)
    V = _bf16_randn(gen, 2, 128, 64)
    ns = load_reference_code(ref, "dattn1_check",
                             _ns(Q=Q.double(), K=K.double(), Vt=V.double().transpose(1, 2).contiguous()))
    y = ns["torch_fn"]()
    torch.save({"Q": Q, "K": K, "V": V, "O": y.float(), "source": SOURCES["dattn1_check"][0]},
               HERE / "dattn1.pt")


def make_lora(ref: Path, gen):
    # LoRA GEMM: gemm.py torch_lora() = (a @ b.t()) + (a @ lA.t() @ lB.t()) over globals a, b, lA, lB
    m, n, k, r = 5, 160, 256, 16
    a = _bf16_randn(gen, m, k)
    b = _bf16_randn(gen, n, k, std=math.sqrt(2 / k))
    lA = _bf16_randn(gen, r, k, std=math.sqrt(2 / k))
    lB = _bf16_randn(gen, n, r, std=math.sqrt(2 / k))
    ns = load_reference_code(ref, "lora", _ns(a=a.double(), b=b.double(), lA=lA.double(), lB=lB.double()))
    y = ns["torch_lora"]()
    torch.save({"x": a, "w": b, "lora_a": lA, "lora_b": lB, "y": y.float(), "source": SOURCES["lora"][0]},
               HERE / "lora.pt")


def make_prefill(ref: Path, gen, B, H, Lq, Lkv, D, name):
    # Full-sequence attention: attn_reimpl(q, k, v) of attn/attempt6_epi_pipeline/attn.py on
    # [b, h, seqlen, d] inputs drawn like that kernel's tests (tests.py generate_input: randn + 0.5).
    q = (torch.randn(B, H, Lq, D, generator=gen, dtype=torch.float64) + 0.5).to(torch.bfloat16)
    k = (torch.randn(B, H, Lkv, D, generator=gen, dtype=torch.float64) + 0.5).to(torch.bfloat16)
    v = (torch.randn(B, H, Lkv, D, generator=gen, dtype=torch.float64) + 0.5).to(torch.bfloat16)
    ns = load_reference_code(ref, "attn_reimpl", _ns())
    out = ns["attn_reimpl"](q.double(), k.double(), v.double())
    lse = torch.logsumexp((q.double() @ k.double().transpose(2, 3)) * D ** -0.5, dim=-1)
    torch.save({"q": q, "k": k, "v": v, "out": out.float(), "lse": lse.float(),
                "source": SOURCES["attn_reimpl"][0]}, HERE / f"{name}.pt")


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--ref", default=os.environ.get("FK_REFERENCE_DIR"),
                    help="reference checkout (default: $FK_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.ref:
        raise SystemExit("give --ref PATH or set FK_REFERENCE_DIR to the reference checkout")
    ref = Path(args.ref)
    if not (ref / "demo").is_dir():
        raise SystemExit(f"reference checkout not found at {ref}")
    gen = torch.Generator().manual_seed(1234)
    make_attention(ref, gen, B=4, Hq=8, Hkv=2, Lmax=136, lens=[136, 77, 1, 0], name="attn_gqa4_ragged")
    make_attention(ref, gen, B=2, Hq=8, Hkv=1, Lmax=200, lens=[200, 65], name="attn_gqa8")
    make_attention(ref, gen, B=3, Hq=4, Hkv=4, Lmax=96, lens=[96, 64, 63], name="attn_mha")
    make_gemms(ref, gen)
    make_lora(ref, gen)
    make_prefill(ref, gen, B=1, H=2, Lq=130, Lkv=200, D=64, name="prefill_d64")
    make_prefill(ref, gen, B=1, H=2, Lq=64, Lkv=136, D=128, name="prefill_d128")
    for p in sorted(HERE.glob("*.pt")):
        print(f"{p.name}: {p.stat().st_size} bytes")


if __name__ == "__main__":
    main()
