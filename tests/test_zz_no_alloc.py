"""The allocation-free skinny GEMM entry point, called through the C ABI (GPU).

``fk_skinny_gemm_noalloc`` serves callers that cannot allocate GPU memory
while they run: it keeps its scratch in a fixed array inside the library.
This file is named to be collected last so a stop-at-first-failure run has
already run every other test; it also passes when run alone.
"""
import ctypes

import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import _native, configs, skinny_gemm

pytestmark = pytest.mark.gpu

MAX_ERR = 2e-2   # same scaled-error tolerance as the other linear-family tests
MEAN_ERR = 2e-3


def _close(out, ref):
    out, ref = out.float().cpu(), ref.float().cpu()
    assert torch.isfinite(out).all()
    e = (out - ref).abs() / ref.abs().clamp_min(1.0)
    assert e.max().item() <= MAX_ERR and e.mean().item() <= MEAN_ERR, e.max().item()


def _noalloc(x, w, y):
    lib = _native.load()
    dev = x.device
    _native.use_device(dev.index if dev.index is not None else torch.cuda.current_device())
    rc = lib.fk_skinny_gemm_noalloc(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.shape[0], w.shape[0],
                                    x.shape[1], torch.cuda.current_stream(dev).cuda_stream)
    _native.check(rc)


def test_noalloc_matches_workspace_entry_point_twice():
    # Two calls in a row with different shapes: the second must not see the
    # first's scratch. Each result is checked against the workspace entry point
    # (the same kernel given caller scratch) and against the CPU oracle.
    for (M, N, K, seed) in [(16, 14336, 4096, 2), (3, 6144, 4096, 5)]:
        x, w = configs.gemm_inputs(M, N, K, seed)
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _noalloc(x, w, y)
        ref = skinny_gemm(x, w)
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        _close(y, ref)
        _close(y, oracle.linear(x, w))


def test_noalloc_rejects_sizes_beyond_limit():
    lib = _native.load()
    x, w = configs.gemm_inputs(17, 256, 256, 0)
    y = torch.empty(17, 256, dtype=torch.bfloat16, device="cuda")
    rc = lib.fk_skinny_gemm_noalloc(x.data_ptr(), w.data_ptr(), y.data_ptr(), 17, 256, 256, None)
    assert rc == -1
    assert "M <= 16" in lib.fk_last_error().decode()
    rc = lib.fk_skinny_gemm_noalloc(x.data_ptr(), w.data_ptr(), y.data_ptr(), 4, 600000, 256, None)
    assert rc == -1
