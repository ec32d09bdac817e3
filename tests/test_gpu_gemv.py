"""Tensor-core GEMV over pre-tiled weights (ls_gemv_bf16) against fp32 torch.

Shapes: the Qwen3-4B decode linears (fused QKV with its RMSNorm, o_proj and
down_proj with the residual epilogue, gate_up with RMSNorm + SiLU*up), their
tensor-parallel shards, and m = 1..8 activation rows.  Bound: max-abs error
<= 2e-2 * max(1, max|ref|) and >= 99% of outputs equal to the fp32 result
rounded to bf16.  Also: the result is bit-identical run to run, the workspace
stays zeroed, and it matches the CUDA-core streaming kernel within the bound.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import tol
from leanstack_b200 import kernels as K
from leanstack_b200 import synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand(shape, std, name, seed=31):
    return synth.normal(shape, std, seed, name, device=DEV)


def _rms(x, w, eps=1e-6):
    xf = x.float()
    return ((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()).bfloat16()


def _check(out, ref):
    err = (out.float() - ref).abs().max().item()
    assert err <= tol(ref), err
    assert (out == ref.bfloat16()).float().mean().item() > 0.99


@pytest.mark.parametrize("m", [1, 2, 5, 8])
@pytest.mark.parametrize("n,k", [(6144, 2560), (2560, 4096), (2560, 9728), (2560, 512), (2560, 1216), (768, 2560)])
def test_gemv_store_and_residual(m, n, k):
    x = _rand((m, k), 1.0, f"gx{m}{k}")
    w = _rand((n, k), 0.02, f"gw{n}{k}")
    wt = K.gemv_tile_weight(w)
    ref = x.float() @ w.float().t()
    _check(K.gemv(x, wt), ref)
    res = _rand((m, n), 1.0, f"gr{m}{n}")
    out = K.gemv(x, wt, epilogue=K.EPI_RESIDUAL, residual=res)
    _check(out, res.float() + ref.bfloat16().float())


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("i,h", [(9728, 2560), (1216, 2560)])
def test_gemv_norm_silu(m, i, h):
    x = _rand((m, h), 1.0, f"sx{m}")
    nw = synth.norm_weight((h,), 31, "snw", device=DEV)
    w = _rand((2 * i, h), 0.02, f"sw{i}")
    wt = K.gemv_tile_weight(w, silu=True)
    out = K.gemv(x, wt, norm_w=nw, eps=1e-6, epilogue=K.EPI_SILU_MUL)
    xn = _rms(x, nw)
    gu = (xn.float() @ w.float().t()).bfloat16()
    g, u = gu[:, :i], gu[:, i:]
    ref = F.silu(g).bfloat16().float() * u.float()
    _check(out, ref)
    # the QKV form: norm + store
    wq = _rand((6144, h), 0.02, "sq")
    _check(K.gemv(x, K.gemv_tile_weight(wq), norm_w=nw, eps=1e-6), xn.float() @ wq.float().t())


def test_gemv_deterministic_and_one_workspace_across_shapes():
    """Calls of different shapes and m share one workspace, as in the decode step,
    and give bit-identical results to calls with fresh workspaces."""
    shapes = [(6144, 2560, K.EPI_STORE, False), (2560, 4096, K.EPI_RESIDUAL, False),
              (19456, 2560, K.EPI_SILU_MUL, True), (2560, 9728, K.EPI_RESIDUAL, False)]
    ws = torch.zeros(max(K.gemv_workspace_bytes(8, n, e) for n, _, e, _ in shapes), device=DEV, dtype=torch.uint8)
    cases = []
    for n, k, epi, silu in shapes:
        w = _rand((n, k), 0.02, f"ow{n}{k}")
        cases.append((K.gemv_tile_weight(w, silu=silu), w, k, n, epi))
    for rep in range(2):
        for m in (1, 8, 3):
            for wt, w, k, n, epi in cases:
                x = _rand((m, k), 1.0, f"ox{m}{k}")
                cols = n // 2 if epi == K.EPI_SILU_MUL else n
                res = _rand((m, cols), 1.0, f"or{m}{cols}")
                shared = K.gemv(x, wt, epilogue=epi, residual=res, workspace=ws)
                fresh = K.gemv(x, wt, epilogue=epi, residual=res)
                assert torch.equal(shared, fresh), (rep, m, n, k)
    x = _rand((1, 9728), 1.0, "dx")
    w = _rand((2560, 9728), 0.02, "dw")
    a = K.gemv(x, K.gemv_tile_weight(w))
    c = K.linear(x, w)
    assert (a.float() - c.float()).abs().max().item() <= tol(c.float())


def test_gemv_rejects_bad_shapes():
    x = _rand((1, 40), 1.0, "bx")
    w = _rand((64, 40), 0.02, "bw")
    with pytest.raises(Exception):
        K.gemv_tile_weight(w)  # k not a multiple of 32
    x9 = _rand((9, 64), 1.0, "bx9")
    w2 = _rand((4096, 64), 0.02, "bw2")
    with pytest.raises(Exception):
        K.gemv(x9, K.gemv_tile_weight(w2))  # m > 8
