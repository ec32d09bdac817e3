"""tcgen05 weight-streaming GEMM (ls_gemm_bf16_tcgen05) against fp32 torch.

Shapes cover the decode / verify linears of Qwen3-4B at m = 1..256 activation
rows, ragged n and k (partial tiles and k-blocks), every epilogue, and both a
whole-tile and a split (stream-K) reduction.  Bound: max-abs error <=
2e-2 * max(1, max|ref|), and at least 99% of outputs equal to the fp32
reference rounded to bf16.
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


def _rand(shape, std, name, seed=21):
    return synth.normal(shape, std, seed, name, device=DEV)


def _check(out, ref):
    err = (out.float() - ref).abs().max().item()
    assert err <= tol(ref), err
    assert (out == ref.bfloat16()).float().mean().item() > 0.99


@pytest.mark.parametrize("m,n,k", [(1, 256, 128), (1, 6144, 2560), (8, 2560, 4096), (16, 2560, 9728),
                                   (32, 6144, 2560), (80, 2560, 4096), (64, 300, 264), (128, 1024, 2560),
                                   (3, 151936 // 8, 2560)])
def test_gemm_tc_store(m, n, k):
    x = _rand((m, k), 1.0, f"x{m}")
    w = _rand((n, k), 0.02, f"w{n}{k}")
    out = K.gemm_tc(x, w)
    _check(out, x.float() @ w.float().t())


@pytest.mark.parametrize("m", [1, 16, 80])
def test_gemm_tc_residual_and_silu(m):
    x = _rand((m, 4096), 1.0, "xa")
    w = _rand((2560, 4096), 0.02, "wo")
    res = _rand((m, 2560), 1.0, "res")
    out = K.gemm_tc(x, w, epilogue=K.EPI_RESIDUAL, residual=res)
    _check(out, res.float() + (x.float() @ w.float().t()).bfloat16().float())
    inter = 9728
    h = _rand((m, 2560), 1.0, "hn")
    gu = _rand((2 * inter, 2560), 0.02, "gu")
    act = K.gemm_tc(h, gu, epilogue=K.EPI_SILU_MUL)
    g_u = (h.float() @ gu.float().t()).bfloat16()
    ref = F.silu(g_u[:, :inter].float()).bfloat16().float() * g_u[:, inter:].float()
    assert act.shape == (m, inter)
    _check(act, ref)


def test_gemm_tc_deterministic_and_reusable_workspace():
    x = _rand((8, 9728), 1.0, "xd")
    w = _rand((2560, 9728), 0.02, "wd")
    ws = torch.zeros(K.gemm_workspace_bytes(8, 9728, 2560, K.EPI_STORE), device=DEV, dtype=torch.uint8)
    a = K.gemm_tc(x, w, workspace=ws)
    for _ in range(3):
        assert torch.equal(K.gemm_tc(x, w, workspace=ws), a)
    # counters are left at zero for the next call
    cnt = ws[:256].view(torch.int32)
    assert int(cnt.abs().sum()) == 0


def test_gemm_tc_one_workspace_across_shapes():
    """Calls of different shapes share one workspace (as the decode engine does):
    every result matches a fresh-workspace call and the counters stay zero."""
    shapes = [(128, 6144, 2560, K.EPI_STORE), (128, 2560, 4096, K.EPI_RESIDUAL), (128, 9728, 2560, K.EPI_SILU_MUL),
              (128, 2560, 9728, K.EPI_RESIDUAL), (1, 151936, 2560, K.EPI_STORE), (1, 6144, 2560, K.EPI_STORE)]
    ws = torch.zeros(max(K.gemm_workspace_bytes(m, k, n, e) for m, n, k, e in shapes), device=DEV, dtype=torch.uint8)
    for rep in range(2):
        for i, (m, n, k, e) in enumerate(shapes):
            x = _rand((m, k), 1.0, f"sx{i}")
            w = _rand((2 * n if e == K.EPI_SILU_MUL else n, k), 0.02, f"sw{i}")
            res = _rand((m, n), 1.0, f"sr{i}") if e == K.EPI_RESIDUAL else None
            K.device_error(clear=True)
            got = K.gemm_tc(x, w, epilogue=e, residual=res, workspace=ws)
            want = K.gemm_tc(x, w, epilogue=e, residual=res)
            assert K.device_error(clear=True) == 0
            assert torch.equal(got, want), (rep, i)
    assert int(ws[:16384].view(torch.int32).abs().sum()) == 0


def test_gemm_tc_rejects_m_beyond_128():
    x = _rand((129, 256), 1.0, "x129")
    w = _rand((256, 256), 0.02, "w129")
    with pytest.raises(Exception, match="1..128|bad arguments"):
        K.gemm_tc(x, w, workspace=torch.zeros(1 << 20, device=DEV, dtype=torch.uint8))


def test_argmax_rows_lowest_index_on_ties():
    logits = torch.full((3, 151936), -1.0, device=DEV, dtype=torch.bfloat16)
    logits[0, 77] = 2.0
    logits[1, 150000] = 3.0
    logits[1, 9] = 3.0
    logits[2] = _rand((151936,), 1.0, "lg")
    ids = K.argmax_rows(logits)
    assert ids[0].item() == 77 and ids[1].item() == 9
    row = logits[2].float()
    assert ids[2].item() == int(torch.nonzero(row == row.max())[0])


@pytest.mark.parametrize("batch", [1, 4, 32])
def test_tc_engine_matches_cuda_core_engine(batch):  # noqa: C901
    """The tensor-core decode step agrees with the CUDA-core one (hidden state after
    prefill within the bound, same first token), and every row of a batch equals
    the batch-1 run of the same sequence exactly."""
    from leanstack_b200.config import TINY
    from leanstack_b200.engine import DecodeEngine
    from leanstack_b200.leanserve import materialize_from_tensors

    rt = materialize_from_tensors(TINY, synth.synth_checkpoint(TINY, 3, device=DEV), device=DEV)
    prompt = synth.token_ids((batch, 21), TINY.vocab_size, 5, "tc/prompt")
    tc_eng = DecodeEngine(rt, batch_size=batch, max_seq_len=96, linear_backend="tc")
    tc_first = tc_eng.prefill(prompt)
    tc_hidden = tc_eng.last_head_rows().clone()
    if batch <= 8:
        cc_eng = DecodeEngine(rt, batch_size=batch, max_seq_len=96, linear_backend="cuda_core")
        cc_first = cc_eng.prefill(prompt)
        cc_hidden = cc_eng.last_head_rows().clone()
        assert (tc_hidden.float() - cc_hidden.float()).abs().max().item() <= tol(cc_hidden.float())
        assert torch.equal(tc_first, cc_first)
    tc = DecodeEngine(rt, batch_size=batch, max_seq_len=96, linear_backend="tc").generate(prompt, 16)
    for r in range(min(batch, 2)):
        one = DecodeEngine(rt, batch_size=1, max_seq_len=96, linear_backend="tc").generate(prompt[r:r + 1], 16)
        assert torch.equal(one[0], tc[r])


@pytest.mark.parametrize("m", [1, 32, 128])
def test_gemm_tc_f32_partials(m):
    """fp32 epilogue (tensor-parallel row-split partials) equals the bf16 store
    epilogue before its rounding."""
    x = _rand((m, 4864), 1.0, "xf")
    w = _rand((2560, 4864), 0.02, "wf")
    out = K.gemm_tc(x, w, epilogue=K.EPI_STORE_F32)
    assert out.dtype == torch.float32
    ref = x.float() @ w.float().t()
    assert (out - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())
    assert torch.equal(out.bfloat16(), K.gemm_tc(x, w))


@pytest.mark.parametrize("m", [1, 32, 80])
@pytest.mark.parametrize("n,k,epi", [(6144, 2560, K.EPI_STORE), (2560, 9728, K.EPI_RESIDUAL),
                                     (19456, 2560, K.EPI_SILU_MUL), (2432, 2560, K.EPI_SILU_MUL),
                                     (300, 264, K.EPI_STORE)])
def test_gemm_tc_pretiled_weights_bit_identical(m, n, k, epi):
    """Pre-tiled weights (one bulk copy per tile) give bit-identical results to the TMA-map path,
    including ragged n and k (zero-padded tiles)."""
    x = _rand((m, k), 1.0, f"tx{m}{k}")
    w = _rand((n, k), 0.02, f"tw{n}{k}")
    cols = n // 2 if epi == K.EPI_SILU_MUL else n
    res = _rand((m, cols), 1.0, f"tr{m}{cols}")
    tl = K.gemm_tc_tile_weight(w, silu=epi == K.EPI_SILU_MUL)
    a = K.gemm_tc(x, w, epilogue=epi, residual=res)
    b = K.gemm_tc(x, w, epilogue=epi, residual=res, tiled=tl)
    assert torch.equal(a, b)


@pytest.mark.parametrize("m,n,k", [(256, 2560, 4096), (1000, 6144, 2560), (4096, 2560, 9728), (777, 300, 264),
                                   (1, 2560, 2560)])
def test_gemm_big_store_residual(m, n, k):
    """Large-M prefill GEMM against fp32 torch, ragged m / n / k (partial tiles)."""
    x = _rand((m, k), 1.0, f"bx{m}{k}")
    w = _rand((n, k), 0.02, f"bw{n}{k}")
    ref = x.float() @ w.float().t()
    _check(K.gemm_big(x, w), ref)
    res = _rand((m, n), 1.0, f"br{m}{n}")
    _check(K.gemm_big(x, w, epilogue=K.EPI_RESIDUAL, residual=res), res.float() + ref.bfloat16().float())
    f32 = K.gemm_big(x, w, epilogue=K.EPI_STORE_F32)
    assert (f32 - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("m", [384, 2048])
def test_gemm_big_silu(m):
    x = _rand((m, 2560), 1.0, f"bsx{m}")
    w = _rand((2 * 9728, 2560), 0.02, "bsw")
    out = K.gemm_big(x, w, epilogue=K.EPI_SILU_MUL)
    gu = (x.float() @ w.float().t()).bfloat16()
    ref = F.silu(gu[:, :9728]).bfloat16().float() * gu[:, 9728:].float()
    _check(out, ref)
    dec = K.gemm_tc(x[:128].contiguous(), w, epilogue=K.EPI_SILU_MUL)  # the decode GEMM on a 128-row slice
    assert (out[:128].float() - dec.float()).abs().max().item() <= tol(dec.float())


@pytest.mark.parametrize("m", [1, 16, 32, 80, 128])
def test_gemm_tc_split_partials_and_residual_norm(m):
    """Split-partial epilogue (QKV / o_proj / down of the one-GPU tensor-core
    step): the splits added in order are the product within the bound, and the
    residual + RMSNorm consumer gives bf16(res + bf16(sum)) and ls_rmsnorm of
    it bit for bit."""
    eps = 1e-6
    for i, (n, k) in enumerate([(6144, 2560), (2560, 4096), (2560, 9728)]):
        x = _rand((m, k), 1.0, f"spx{i}")
        w = _rand((n, k), 0.02, f"spw{i}")
        s = K.gemm_splits(m, k, n)
        part = torch.full((s * m * n + 64,), float("nan"), device=DEV)
        assert K.gemm_tc_splits(x, w, part) == s
        p = part[:s * m * n].view(s, m, n)
        acc = p[0].clone()
        for j in range(1, s):
            acc += p[j]
        assert torch.isnan(part[s * m * n:]).all()  # nothing written past the splits
        _check(acc.bfloat16(), x.float() @ w.float().t())
        if n != 2560:
            continue
        res = _rand((m, n), 1.0, f"spr{i}")
        nw = 1.0 + _rand((n,), 0.01, f"spn{i}")
        h = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
        xn = torch.empty_like(h)
        K.residual_rmsnorm_splits(part, s, res, out_residual=h, norm_w=nw, eps=eps, out_norm=xn)
        want_h = (res.float() + acc.bfloat16().float()).bfloat16()
        assert torch.equal(h, want_h)
        _check(h, res.float() + (x.float() @ w.float().t()).bfloat16().float())
        assert torch.equal(xn, K.rmsnorm(want_h, nw, eps))
        h2 = torch.empty_like(h)
        K.residual_rmsnorm_splits(part, s, res, out_residual=h2)
        assert torch.equal(h2, want_h)


@pytest.mark.parametrize("n,splits", [(8, 3), (256, 1), (512, 2), (1024, 5), (2304, 14), (2560, 14), (3584, 6),
                                      (4096, 16), (12296, 4), (16384, 9)])
def test_residual_norm_splits_rows(n, splits):
    """The residual + RMSNorm consumer of split partials, for rows of one to 32
    warps and rows with more 8-column groups than threads: h is bf16(res +
    bf16(partials summed in split order)) and the norm equals ls_rmsnorm of h,
    bit for bit; without a norm only h is written."""
    eps = 1e-6
    for m in (1, 7, 80):
        p = _rand((splits, m, n), 0.5, f"rnp{n}_{m}").float()
        res = _rand((m, n), 1.0, f"rnr{n}_{m}")
        nw = 1.0 + _rand((n,), 0.01, f"rnw{n}")
        acc = p[0].clone()
        for j in range(1, splits):
            acc += p[j]
        want_h = (res.float() + acc.bfloat16().float()).bfloat16()
        h = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
        xn = torch.empty_like(h)
        K.residual_rmsnorm_splits(p.reshape(-1), splits, res, out_residual=h, norm_w=nw, eps=eps, out_norm=xn)
        assert torch.equal(h, want_h)
        assert torch.equal(xn, K.rmsnorm(want_h, nw, eps))
        h2 = torch.full_like(h, float("nan"))
        K.residual_rmsnorm_splits(p.reshape(-1), splits, res, out_residual=h2)
        assert torch.equal(h2, want_h)


@pytest.mark.parametrize("batch,q_len,splits", [(1, 1, None), (16, 5, None), (32, 1, None), (3, 2, 1), (2, 1, 8),
                                                (4, 3, 9), (1, 1, 16)])
def test_qk_norm_rope_on_split_partials(batch, q_len, splits):
    """q/k norm + RoPE + K/V append fed by split partials equals the same
    kernel fed by the projection those partials sum to (in split order,
    rounded once), bit for bit: the QKV GEMM's own partials (splits None), or
    synthetic ones at split counts around the kernel's 8-load batches."""
    hq, hkv, d, hidden, S = 32, 8, 128, 2560, 64
    m = batch * q_len
    qn = 1.0 + _rand((d,), 0.01, "qn")
    kn = 1.0 + _rand((d,), 0.01, "kn")
    ang = torch.arange(S, device=DEV, dtype=torch.float32)[:, None] * 0.01 * torch.arange(1, d // 2 + 1, device=DEV)
    cos, sin = ang.cos().bfloat16(), ang.sin().bfloat16()
    pos = torch.arange(batch, device=DEV, dtype=torch.int32) % 7
    n = (hq + 2 * hkv) * d
    if splits is None:
        x = _rand((m, hidden), 1.0, "qx")
        w = _rand((n, hidden), 0.02, "qw")
        s = K.gemm_splits(m, hidden, n)
        part = torch.empty(s * m * n, device=DEV)
        K.gemm_tc_splits(x, w, part)
    else:
        s = splits
        part = _rand((s * m * n,), 0.4, f"qp{s}").float()
    p = part.view(s, m, n)
    qkv = p[0].clone()
    for j in range(1, s):
        qkv += p[j]
    qkv = qkv.bfloat16()
    if splits is None:
        _check(qkv, x.float() @ w.float().t())
    outs = []
    for use_split in (False, True):
        kc = torch.zeros(batch, hkv, S, d, device=DEV, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        q = torch.empty(m, hq, d, device=DEV, dtype=torch.bfloat16)
        common = dict(eps=1e-6, cache_pos=pos.clone(), k_cache=kc, v_cache=vc, max_seq=S, q_out=q)
        if use_split:
            K.qk_norm_rope_splits(part, s, batch, q_len, hq, hkv, d, qn, kn, cos, sin, **common)
        else:
            K.qk_norm_rope(qkv, batch, q_len, hq, hkv, d, qn, kn, cos, sin, **common)
        outs.append((q, kc, vc))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("m", [1, 32, 80, 128])
def test_gate_up_plain_split_and_silu_combine(m):
    """gate_up as a plain [2I, H] linear in the split-partial form (whole-K
    tiles: one split) followed by the SiLU*up combine: equal to the combine
    computed in torch from the same partials (up to the last bit of expf), and
    to the fp32 reference within the bound."""
    inter, hidden = 9728, 2560
    x = _rand((m, hidden), 1.0, "gpx")
    w = _rand((2 * inter, hidden), 0.02, "gpw")
    s = K.gemm_splits(m, hidden, 2 * inter)
    part = torch.empty(s * m * 2 * inter, device=DEV)
    assert K.gemm_tc_splits(x, w, part) == s
    act = torch.empty(m, inter, device=DEV, dtype=torch.bfloat16)
    K.silu_mul_splits(part, s, m, inter, out=act)
    p = part.view(s, m, 2 * inter)
    y = p[0].clone()
    for j in range(1, s):
        y += p[j]
    g_u = y.bfloat16().float()
    g = g_u[:, :inter]
    want = ((g / (1.0 + torch.exp(-g))).bfloat16().float() * g_u[:, inter:]).bfloat16()
    # same partials, same rounding points: equal up to the last bit of expf
    assert (act == want).float().mean().item() > 0.999
    assert (act.float() - want.float()).abs().max().item() <= 2 ** -6 * max(1.0, want.float().abs().max().item())
    ref_gu = (x.float() @ w.float().t()).bfloat16()
    _check(act, F.silu(ref_gu[:, :inter].float()).bfloat16().float() * ref_gu[:, inter:].float())
