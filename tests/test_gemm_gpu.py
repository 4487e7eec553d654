"""Parity of the linear family (skinny stream-K and tcgen05 kernels) against the CPU oracle (GPU)."""
import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import (
    Gemm4SM90,
    LoraGemmSM90,
    RMSNormLinear1SM90,
    Swiglu2SM90,
    _native,
    alloc_workspace,
    compile_cutedsl,
    linear,
    lora_linear,
    rmsnorm_linear,
    skinny_gemm,
    swiglu_gemm,
    swiglu_gemm2,
    workspace_bytes,
)
from fused_kernels_cutedsl_lib_b200 import configs

pytestmark = pytest.mark.gpu

# bf16 outputs vs an fp32 reference. Scaled error |out - ref| / max(1, |ref|):
# the output's own bf16 rounding is 2^-9 relative, so an absolute bound cannot
# hold for |ref| > 8 (SwiGLU products reach tens).
MAX_ERR = 2e-2
MEAN_ERR = 2e-3


def assert_close(out, ref):
    out = out.float().cpu()
    ref = ref.float()
    assert out.shape == ref.shape
    assert torch.isfinite(out).all()
    e = (out - ref).abs() / ref.abs().clamp_min(1.0)
    assert e.max().item() <= MAX_ERR, f"max scaled err {e.max().item():.3e}"
    assert e.mean().item() <= MEAN_ERR, f"mean scaled err {e.mean().item():.3e}"


def mk(M, N, K, seed=0, w_std=0.02):
    return configs.gemm_inputs(M, N, K, seed, w_std=w_std)


def gamma_of(K, seed=9):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).bfloat16()


def finish():
    torch.cuda.synchronize()
    assert _native.device_error() == 0


def test_golden_fixtures(golden):
    g = golden("skinny_gemm")
    y = skinny_gemm(g["x"].cuda(), g["w"].cuda())
    finish()
    assert_close(y, g["y"])
    g = golden("swiglu")
    y = swiglu_gemm(g["x"].cuda(), g["w_gate_up"].cuda())
    finish()
    assert_close(y, g["y"])
    g = golden("swiglu_two_weights")
    y = swiglu_gemm2(g["x"].cuda(), g["b"].cuda(), g["b1"].cuda())
    finish()
    assert_close(y, g["y"])
    g = golden("rmsnorm_linear")
    x = g["x"].cuda()
    y = rmsnorm_linear(x, torch.ones(x.shape[1], dtype=torch.bfloat16, device="cuda"), g["w"].cuda(), eps=g["eps"])
    finish()
    assert_close(y, g["y"])


SKINNY_M = [1, 2, 4, 8, 9, 16]
TC_M = [17, 32, 64, 100, 128, 256]


@pytest.mark.parametrize("M", SKINNY_M + TC_M)
def test_plain_config3_shape(M):
    x, w = mk(M, 14336, 4096, seed=2)
    y = torch.full((M, 14336), float("nan"), dtype=torch.bfloat16, device="cuda")
    skinny_gemm(x, w, y)
    finish()
    assert_close(y, oracle.linear(x, w))


@pytest.mark.parametrize("M", [1, 5, 16, 40, 128])
@pytest.mark.parametrize("N,K", [(200, 136), (1000, 520), (6144, 4096), (4096, 14336)])
def test_plain_ragged_shapes(M, N, K):
    x, w = mk(M, N, K, seed=M + N)
    y = skinny_gemm(x, w)
    finish()
    assert_close(y, oracle.linear(x, w))


@pytest.mark.parametrize("M", [1, 16, 128])
def test_rmsnorm_linear_config4(M):
    x, w = mk(M, 6144, 4096, seed=3)
    gam = gamma_of(4096)
    y = rmsnorm_linear(x, gam, w, eps=1e-6)
    finish()
    assert_close(y, oracle.rmsnorm_linear(x, gam, w, eps=1e-6))


@pytest.mark.parametrize("M", [1, 16, 128])
def test_swiglu_config4(M):
    x, w = mk(M, 2 * 14336, 4096, seed=3)
    y = swiglu_gemm(x, w)
    finish()
    assert_close(y, oracle.swiglu(x, w))


@pytest.mark.parametrize("M", [3, 16, 64, 200])
def test_rmsnorm_swiglu_and_two_weight_forms(M):
    x, w = mk(M, 2 * 1536, 2048, seed=M)
    gam = gamma_of(2048)
    y = swiglu_gemm(x, w, gamma=gam, eps=1e-5)
    finish()
    ref = oracle.swiglu(oracle.rmsnorm(x, gam, 1e-5), w)
    assert_close(y, ref)
    y2 = swiglu_gemm2(x, w[:1536].contiguous(), w[1536:].contiguous())
    finish()
    assert_close(y2, oracle.swiglu(x, w))


@pytest.mark.parametrize("M", [1, 16, 48, 300])
def test_residual_epilogue_in_place(M):
    x, w = mk(M, 4096, 4096, seed=5)
    res = torch.randn(M, 4096, device="cuda").bfloat16()
    ref = oracle.linear(x, w) + res.float().cpu()
    out = res.clone()
    linear(x, w, out, residual=out)  # y = residual + x W^T, written over the residual
    finish()
    assert_close(out, ref)


def test_deterministic_and_workspace_reuse():
    x, w = mk(8, 14336, 4096, seed=1)
    a = skinny_gemm(x, w)
    b = skinny_gemm(x, w)
    x2, w2 = mk(128, 14336, 4096, seed=1)
    c = skinny_gemm(x2, w2)
    d = skinny_gemm(x2, w2)
    finish()
    assert torch.equal(a, b) and torch.equal(c, d)


def test_explicit_workspace_and_stream():
    x, w = mk(16, 6144, 4096, seed=4)
    nb = workspace_bytes(16, 6144, 4096)
    ws = alloc_workspace(nb, "cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y = skinny_gemm(x, w, workspace=ws)
    s.synchronize()
    finish()
    assert_close(y, oracle.linear(x, w))
    assert int(ws[:4 * 48].view(torch.int32).abs().sum()) == 0  # counters back at zero


def test_reference_style_kernel_objects():
    x, w = mk(16, 4096, 4096, seed=6)
    c = torch.empty(16, 4096, dtype=torch.bfloat16, device="cuda")
    k = Gemm4SM90(tile_shape_mnk=(128, 256, 32), epi_tile_mn=(128, 128), cluster_shape_mnk=(2, 1, 1),
                  atom_layout_mn=(2, 1), ab_stage=6, epi_stage=2, is_persistent=True, gemm_n_prologue=1)
    f = compile_cutedsl((x, w, c), k, False)
    f(x, w, c)
    finish()
    assert_close(c, oracle.linear(x, w))
    r = RMSNormLinear1SM90(eps=1e-5)
    r(x, w, c, torch.cuda.current_stream())
    finish()
    assert_close(c, oracle.rmsnorm_linear(x, None, w, eps=1e-5))
    b1 = mk(16, 4096, 4096, seed=7)[1]
    Swiglu2SM90(tile_shape_mnk=(128, 128, 32))(x, w, b1, c)
    finish()
    assert_close(c, oracle.swiglu_separate(x, w, b1))


def test_bad_arguments_raise():
    x, w = mk(4, 256, 256)
    with pytest.raises(TypeError):
        skinny_gemm(x.float(), w)
    with pytest.raises(ValueError):
        skinny_gemm(x[:, :128], w)
    with pytest.raises(ValueError):
        skinny_gemm(x, w, torch.empty(4, 100, dtype=torch.bfloat16, device="cuda"))
    x9 = torch.zeros(4, 260, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        skinny_gemm(x9, torch.zeros(8, 260, dtype=torch.bfloat16, device="cuda"))


def test_shared_workspace_across_shapes():
    """One workspace reused by calls of very different N and M (stale partials must never act as counters)."""
    ws = alloc_workspace(max(workspace_bytes(16, 14336, 4096, True), workspace_bytes(256, 14336, 4096, True)), "cuda")
    shapes = [(1, 256, 4096), (1, 1024, 256), (1, 14336, 256), (5, 96, 256), (16, 14336, 4096),
              (64, 640, 512), (128, 14336, 256), (3, 14336, 4096)]
    for rep in range(2):
        for (M, N, K) in shapes:
            x, w = mk(M, N, K, seed=M * 7 + N + rep)
            y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            skinny_gemm(x, w, y, workspace=ws)
            finish()
            assert_close(y, oracle.linear(x, w))


def test_tvm_ffi_entry_points_match_ctypes():
    """The TVM-FFI module (torch tensors in, reference style) gives the same results as the ctypes path."""
    pytest.importorskip("tvm_ffi")
    from fused_kernels_cutedsl_lib_b200 import tvm_ffi_module

    mod = tvm_ffi_module.load()
    x, w = mk(16, 4096, 4096, seed=8)
    gam = gamma_of(4096)
    ws = alloc_workspace(int(mod.linear_workspace_bytes(16, 4096, 4096, 1)), "cuda")
    y = torch.empty(16, 4096, dtype=torch.bfloat16, device="cuda")
    mod.skinny_gemm(x, w, y, ws)
    torch.cuda.synchronize()
    assert torch.equal(y, skinny_gemm(x, w))
    mod.rmsnorm_linear(x, gam, w, y, 1e-6, ws)
    torch.cuda.synchronize()
    assert torch.equal(y, rmsnorm_linear(x, gam, w, eps=1e-6))
    wgu = mk(16, 2 * 2048, 4096, seed=9)[1]
    y2 = torch.empty(16, 2048, dtype=torch.bfloat16, device="cuda")
    mod.swiglu_gemm(x, wgu, y2, ws)
    torch.cuda.synchronize()
    assert torch.equal(y2, swiglu_gemm(x, wgu))
    xa = mk(16, 16, 16, seed=10)[0]
    lb = mk(16, 4096, 16, seed=11)[1]
    mod.lora_gemm(x, w, xa, lb, y, ws)
    torch.cuda.synchronize()
    assert torch.equal(y, lora_linear(x, w, lb, lora_xa=xa))


# ---- LoRA: y = x W^T + (x A^T) B^T, the reference's lora/attempt1 GemmSM90 ----

def test_lora_golden(golden):
    g = golden("lora")
    x, w, la, lb = (g[k].cuda() for k in ("x", "w", "lora_a", "lora_b"))
    y = lora_linear(x, w, lb, lora_a=la)
    finish()
    assert_close(y, g["y"])


@pytest.mark.parametrize("M", [1, 7, 16, 64, 200, 300])
@pytest.mark.parametrize("rank", [16, 64, 72])
def test_lora_matches_oracle(M, rank):
    N, K = 1536, 1024
    x, w = mk(M, N, K, seed=M + rank)
    g = torch.Generator(device="cuda").manual_seed(rank)
    la = (0.03 * torch.randn(rank, K, generator=g, device="cuda")).bfloat16()
    lb = (0.03 * torch.randn(N, rank, generator=g, device="cuda")).bfloat16()
    res = torch.randn(M, N, generator=g, device="cuda").bfloat16()
    xa = linear(x, la)
    y = lora_linear(x, w, lb, lora_xa=xa, residual=res)
    finish()
    assert_close(y, oracle.lora_linear(x, w, None, lb, lora_xa=xa) + res.float().cpu())
    # the rank-r term matters: without it the check fails
    base = oracle.linear(x, w) + res.float().cpu()
    assert ((y.float().cpu() - base).abs().max() > 0.05)


def test_lora_kernel_object_reference_call_shape():
    M, N, K, r = 32, 512, 256, 16
    x, w = mk(M, N, K, seed=4)
    g = torch.Generator(device="cuda").manual_seed(4)
    la = (0.05 * torch.randn(r, K, generator=g, device="cuda")).bfloat16()
    lb = (0.05 * torch.randn(N, r, generator=g, device="cuda")).bfloat16()
    xa = (x.float() @ la.float().t()).bfloat16()  # the reference computes lora_xA with torch before the call
    c = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    LoraGemmSM90(tile_shape_mn=(128, 256), lora_dim=r)(x, w, xa, lb, c)
    finish()
    assert_close(c, oracle.lora_linear(x, w, None, lb, lora_xa=xa))


def test_lora_argument_errors():
    x, w = mk(4, 256, 128)
    lb = torch.zeros(256, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        lora_linear(x, w, lb, lora_a=torch.zeros(12, 128, dtype=torch.bfloat16, device="cuda"))  # rank 12
    lb = torch.zeros(256, 16, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        lora_linear(x, w, lb)  # neither lora_a nor lora_xa


# ---- output placement (row strides of y / residual), used by the tensor-parallel layer ----

@pytest.mark.parametrize("M", [4, 100])
def test_linear_ex_strided_output_and_residual(M):
    import ctypes

    N, K, ld = 512, 256, 1536
    x, w = mk(M, N, K, seed=M)
    full = torch.full((M, ld), 7.0, dtype=torch.bfloat16, device="cuda")  # [M, ld]; our block at columns 640..
    res_full = torch.randn(M, ld, device="cuda").bfloat16()
    c0 = 640
    ws = alloc_workspace(workspace_bytes(M, N, K), "cuda")
    st = torch.cuda.current_stream().cuda_stream
    _native.check(_native.load().fk_linear_ex(
        x.data_ptr(), None, w.data_ptr(), None, 0, res_full.data_ptr() + 2 * c0, ld, full.data_ptr() + 2 * c0, ld,
        None, 0, M, N, K, 0.0, ws.data_ptr(), ws.numel(), ctypes.c_void_p(st)))
    finish()
    ref = linear(x, w, residual=res_full[:, c0:c0 + N].contiguous())
    assert torch.equal(full[:, c0:c0 + N], ref)
    assert torch.all(full[:, :c0] == 7.0) and torch.all(full[:, c0 + N:] == 7.0)


@pytest.mark.parametrize("M,N,kind", [(4, 512, "plain"), (100, 520, "plain"), (128, 1024, "rms"),
                                      (64, 1792, "swiglu"), (200, 384, "plain")])
def test_linear_ex_output_copies(M, N, kind):
    """Output copies (the tensor-parallel layer's all-gather targets; here local
    buffers stand in for peers' memory): every copy equals y bit for bit, y equals
    the plain call, nothing outside the block is written. Covers the staged
    16-byte path of the tcgen05 epilogue and reduction (M > 16, aligned) and its
    2-byte fallback at a ragged N."""
    import ctypes

    K, ld = 1024, N + 256
    sw = kind == "swiglu"
    x, w = mk(M, 2 * N if sw else N, K, seed=M + N)
    gam = gamma_of(K) if kind == "rms" else None
    c0 = 128
    outs = [torch.full((M, ld), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    ws = alloc_workspace(workspace_bytes(M, N, K, sw), "cuda")
    peers = (ctypes.c_void_p * 2)(outs[1].data_ptr() + 2 * c0, outs[2].data_ptr() + 2 * c0)
    st = torch.cuda.current_stream().cuda_stream
    _native.check(_native.load().fk_linear_ex(
        x.data_ptr(), gam.data_ptr() if gam is not None else None, w.data_ptr(), w.data_ptr() if sw else None,
        N if sw else 0, None, 0, outs[0].data_ptr() + 2 * c0, ld, peers, 2, M, N, K, 1e-6, ws.data_ptr(), ws.numel(),
        ctypes.c_void_p(st)))
    finish()
    if sw:
        ref = linear(x, w, w_up=w, up_row_offset=N)
    else:
        ref = linear(x, w, gamma=gam, eps=1e-6)
    for o in outs:
        assert torch.equal(o[:, c0:c0 + N], ref)
        assert torch.all(o[:, :c0] == 7.0) and torch.all(o[:, c0 + N:] == 7.0)


def test_tvm_ffi_reference_call_shapes_and_compile_cutedsl():
    """TVM-FFI functions with the reference's call shapes (no workspace argument),
    compile_cutedsl returning them, the named tcgen05 entry and the fused QKV +
    KV-append entry: all equal to the ctypes path bit for bit."""
    pytest.importorskip("tvm_ffi")
    import tvm_ffi

    from fused_kernels_cutedsl_lib_b200 import Gemm4SM90, Swiglu2SM90, compile_cutedsl, tvm_ffi_module
    from fused_kernels_cutedsl_lib_b200.layer import linear_kv_append

    mod = tvm_ffi_module.load()
    for M in (3, 16, 96):
        x, w = mk(M, 2048, 1024, seed=30 + M)
        y = torch.empty(M, 2048, dtype=torch.bfloat16, device="cuda")
        f = compile_cutedsl((x, w, y), Gemm4SM90(), False)
        assert isinstance(f, tvm_ffi.Function)
        f(x, w, y)
        torch.cuda.synchronize()
        assert torch.equal(y, linear(x, w))
        s = torch.cuda.Stream()
        fs = compile_cutedsl((x, w, y), Gemm4SM90(), True)
        y.zero_()
        fs(x, w, y, s)
        s.synchronize()
        assert torch.equal(y, linear(x, w))
        if M > 16:
            ws = alloc_workspace(int(mod.linear_workspace_bytes(M, 2048, 1024, 0)), "cuda")
            y2 = torch.empty_like(y)
            mod.gemm_tc(x, w, y2, ws)
            torch.cuda.synchronize()
            assert torch.equal(y2, y)
    x, b = mk(8, 1024, 1024, seed=40)
    b1 = mk(8, 1024, 1024, seed=41)[1]
    c = torch.empty(8, 1024, dtype=torch.bfloat16, device="cuda")
    compile_cutedsl((x, b, b1, c), Swiglu2SM90(), False)(x, b, b1, c)
    torch.cuda.synchronize()
    assert torch.equal(c, swiglu_gemm2(x, b, b1))
    with pytest.raises(ValueError):
        mod.gemm_tc(x, b, c, alloc_workspace(1 << 20, "cuda"))  # M <= 16 is not the tcgen05 path
    # fused QKV projection + KV append through TVM-FFI vs ctypes
    B, Hq, Hkv, L = 4, 8, 2, 64
    x = torch.randn(B, 1024, device="cuda").bfloat16()
    gam = gamma_of(1024)
    wqkv = (0.02 * torch.randn((Hq + 2 * Hkv) * 128, 1024, device="cuda")).bfloat16()
    outs = []
    for use_tvm in (False, True):
        kc = torch.zeros(B, L, Hkv, 128, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        lens = torch.tensor([0, 5, 63, 64], dtype=torch.int32, device="cuda")
        nxt = torch.zeros_like(lens)
        y = torch.empty(B, wqkv.shape[0], dtype=torch.bfloat16, device="cuda")
        ws = alloc_workspace(int(mod.linear_workspace_bytes(B, wqkv.shape[0], 1024, 0)), "cuda")
        if use_tvm:
            mod.linear_kv_append(x, gam, wqkv, y, kc, vc, lens, nxt, Hq, 1e-6, ws)
        else:
            linear_kv_append(x, wqkv, y, kc, vc, lens, nxt, Hq, Hkv, gamma=gam, eps=1e-6, workspace=ws)
        torch.cuda.synchronize()
        outs.append((y, kc, vc, nxt))
    for a, b_ in zip(*outs):
        assert torch.equal(a, b_)
    assert outs[0][3].tolist() == [1, 6, 64, 64]
