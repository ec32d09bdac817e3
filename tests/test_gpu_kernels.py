"""Kernel-level parity of libleanb200.so against fp32 references (B200 only).

Each kernel is checked against the same op computed in fp32 by torch with the
reference's bf16 rounding points, within the north star's bound
(max-abs error <= 2e-2 * max(1, max|ref|)); elementwise kernels must also be
bit-exact on nearly every element.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from conftest import tol
from leanstack_b200 import kernels as K
from leanstack_b200 import synth
from oracle import qwen_oracle as qo

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rms_ref(x, w, eps):
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return ((xf * r) * w.float()).bfloat16()


def _rand(shape, std, name, seed=11):
    return synth.normal(shape, std, seed, name, device=DEV)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("k,n", [(2560, 6144), (4096, 2560), (9728, 2560), (264, 136)])
def test_linear_store_and_norm(m, k, n):
    x = _rand((m, k), 1.0, f"x{m}{k}")
    w = _rand((n, k), 0.02, f"w{k}{n}")
    nw = synth.norm_weight((k,), 11, f"nw{k}", device=DEV)
    y = K.linear(x, w)
    ref = (x.float() @ w.float().t())
    assert (y.float() - ref).abs().max().item() <= tol(ref)
    assert (y == ref.bfloat16()).float().mean().item() > 0.99
    yn = K.linear(x, w, norm_w=nw, eps=1e-6)
    xn = _rms_ref(x, nw, 1e-6)
    refn = xn.float() @ w.float().t()
    assert (yn.float() - refn).abs().max().item() <= tol(refn)
    assert (yn == refn.bfloat16()).float().mean().item() > 0.99


@pytest.mark.parametrize("m", [1, 4, 8])
def test_linear_residual_and_silu(m):
    k, n = 2560, 2560
    x = _rand((m, 4096), 1.0, "xo")
    w = _rand((n, 4096), 0.02, "wo")
    res = _rand((m, n), 1.0, "res")
    y = K.oproj_residual(x, w, res)
    ref = res.float() + (x.float() @ w.float().t()).bfloat16().float()
    assert (y.float() - ref).abs().max().item() <= tol(ref)
    assert (y == ref.bfloat16()).float().mean().item() > 0.99
    inter = 1536
    gu = _rand((2 * inter, k), 0.02, "gu")
    nw = synth.norm_weight((k,), 11, "post", device=DEV)
    h = _rand((m, k), 1.0, "h")
    act = K.gateup_silu(h, nw, gu, 1e-6)
    hn = _rms_ref(h, nw, 1e-6)
    g_u = (hn.float() @ gu.float().t()).bfloat16()
    g, u = g_u[:, :inter], g_u[:, inter:]
    ref = (F.silu(g.float()).bfloat16().float() * u.float())
    assert act.shape == (m, inter)
    assert (act.float() - ref).abs().max().item() <= tol(ref)
    assert (act == ref.bfloat16()).float().mean().item() > 0.99
    d = _rand((k, inter), 0.02, "down")
    out = K.down_residual(act, d, h)
    ref = h.float() + (act.float() @ d.float().t()).bfloat16().float()
    assert (out.float() - ref).abs().max().item() <= tol(ref)


def test_linear_is_deterministic():
    x = _rand((1, 9728), 1.0, "xd")
    w = _rand((2560, 9728), 0.02, "wd")
    a = K.linear(x, w)
    for _ in range(3):
        assert torch.equal(K.linear(x, w), a)


def test_rmsnorm_and_embed():
    x = _rand((3, 2560), 1.0, "xr")
    w = synth.norm_weight((2560,), 1, "nr", device=DEV)
    y = K.rmsnorm(x, w, 1e-6)
    ref = qo.rmsnorm(x.cpu(), w.cpu(), 1e-6)
    assert (y.cpu() == ref).float().mean().item() > 0.999
    assert (y.float().cpu() - ref.float()).abs().max().item() <= 2 ** -6
    # a row length that is not a multiple of 8 takes the scalar path
    x2 = _rand((2, 1001), 1.0, "xr2")
    w2 = synth.norm_weight((1001,), 1, "nr2", device=DEV)
    y2 = K.rmsnorm(x2, w2, 1e-6)
    ref2 = qo.rmsnorm(x2.cpu(), w2.cpu(), 1e-6)
    assert (y2.float().cpu() - ref2.float()).abs().max().item() <= 2 ** -6
    emb = _rand((1000, 256), 0.02, "emb")
    ids = torch.tensor([5, 999, 0, 5], device=DEV)
    assert torch.equal(K.embed_gather(ids, emb), emb[ids])


@pytest.mark.parametrize("batch,q_len", [(2, 1), (2, 2), (1, 5), (2, 4)])
def test_qkv_rope_append_matches_oracle(batch, q_len):
    hq, hkv, d, hidden, past = 32, 8, 128, 2560, 37
    x = _rand((batch * q_len, hidden), 1.0, "qx")
    qkv_w = _rand(((hq + 2 * hkv) * d, hidden), 0.02, "qkvw")
    qn = synth.norm_weight((d,), 2, "qn", device=DEV)
    kn = synth.norm_weight((d,), 2, "kn", device=DEV)
    ln = synth.norm_weight((hidden,), 2, "ln", device=DEV)
    cos, sin = qo.rope_cache(qo.rope_inv_freq(d, 1e6), 128, torch.bfloat16)
    kc = torch.zeros(batch, hkv, 128, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    cache_pos = torch.tensor([past + 3 * b for b in range(batch)], device=DEV, dtype=torch.int32)
    q = K.qkv_rope_append(x, batch, q_len, qkv_w, hq, hkv, d, qn, kn, cos.to(DEV), sin.to(DEV), input_norm_w=ln,
                          cache_pos=cache_pos, k_cache=kc, v_cache=vc, max_seq=128)
    # oracle on the CPU with the same inputs, per sequence (positions differ)
    for b in range(batch):
        p0 = past + 3 * b
        xb = x[b * q_len:(b + 1) * q_len].cpu().view(1, q_len, hidden)
        w = qo.LayerWeights(input_layernorm=ln.cpu(), qkv_proj=qkv_w.cpu(), o_proj=None, q_norm=qn.cpu(),
                            k_norm=kn.cpu(), post_attention_layernorm=None, gate_up_proj=None, down_proj=None)
        xn = qo.rmsnorm(xb, w.input_layernorm, 1e-6)
        rq, rk, rv = qo.qkv_project(xn, w, hq, hkv, d, cos[p0:p0 + q_len][None], sin[p0:p0 + q_len][None], 1e-6)
        got_q = q[b * q_len:(b + 1) * q_len].cpu().view(q_len, hq, d).transpose(0, 1)[None]
        for got, want in ((got_q, rq), (kc[b, :, p0:p0 + q_len].cpu()[None], rk),
                          (vc[b, :, p0:p0 + q_len].cpu()[None], rv)):
            assert got.shape == want.shape
            assert (got == want).float().mean().item() > 0.99
            assert (got.float() - want.float()).abs().max().item() <= tol(want.float())


def _attn_ref(q, kc, vc, cache_pos, q_len, hq, hkv, scale):
    """fp32 GQA attention with the causal-suffix visibility rule."""
    batch = kc.shape[0]
    out = []
    for b in range(batch):
        past = int(cache_pos[b])
        L = past + q_len
        qb = q[b * q_len:(b + 1) * q_len].float().transpose(0, 1)  # [Hq, Q, D]
        kb = kc[b, :, :L].float().repeat_interleave(hq // hkv, 0)
        vb = vc[b, :, :L].float().repeat_interleave(hq // hkv, 0)
        s = (qb @ kb.transpose(1, 2)) * scale
        mask = torch.arange(L, device=q.device)[None, :] > (past + torch.arange(q_len, device=q.device))[:, None]
        s = s.masked_fill(mask[None], float("-inf"))
        o = torch.softmax(s, -1) @ vb  # [Hq, Q, D]
        out.append(o.transpose(0, 1).reshape(q_len, -1))
    return torch.cat(out, 0)


@pytest.mark.parametrize("batch,q_len,lens", [(1, 1, [513]), (1, 1, [4000]), (3, 1, [5, 700, 2049]),
                                              (2, 5, [64, 1024]), (1, 8, [504]), (4, 2, [1, 2, 3, 17]),
                                              # 20 / 32 rows per kv head on enough pairs: two 16-row tiles per CTA
                                              (16, 5, [1024 - 61 * i for i in range(16)]),
                                              (3, 6, [0, 5, 300]),  # 24 rows: 8-row tiles, split keys
                                              (10, 8, [0, 1, 15, 16, 17, 300, 511, 512, 1000, 4088])])
def test_decode_attention(batch, q_len, lens):
    hq, hkv, d, S = 32, 8, 128, 4096
    kc = _rand((batch, hkv, S, d), 1.0, "kc")
    vc = _rand((batch, hkv, S, d), 1.0, "vc")
    q = _rand((batch * q_len, hq, d), 1.0, "q")
    cache_pos = torch.tensor(lens, device=DEV, dtype=torch.int32)
    scale = d ** -0.5
    out = K.decode_attention(q, kc, vc, batch, q_len, hq, hkv, d, S, scale, cache_pos=cache_pos)
    ref = _attn_ref(q, kc, vc, lens, q_len, hq, hkv, scale)
    assert (out.float() - ref).abs().max().item() <= tol(ref)
    assert (out.float() - ref).abs().max().item() <= 2 ** -7
    if len(set(lens)) == 1:  # uniform cursor via the host argument
        out2 = K.decode_attention(q, kc, vc, batch, q_len, hq, hkv, d, S, scale, uniform_past=lens[0])
        assert torch.equal(out, out2)


@pytest.mark.parametrize("hq,hkv,lens,S", [(32, 8, [512], 4096),  # config 2
                                           (32, 8, [0], 64),  # first token, empty cache
                                           (32, 8, [15, 16, 4000], 4096),  # 16-key block edges, long context
                                           (16, 8, [1, 31, 32, 700], 1024),  # the 0.6B draft's heads (G 2)
                                           (32, 8, [63, 4094], 4095)])  # the last cache slot
def test_decode_attention_qkv_fused_equals_two_launches(hq, hkv, lens, S):
    """The one-launch decode attention from the raw QKV projection writes the
    same K/V rows into the cache and returns the same output, bit for bit, as
    ls_qk_norm_rope_kvappend followed by ls_decode_attention."""
    d, batch = 128, len(lens)
    qkv = _rand((batch, (hq + 2 * hkv) * d), 1.0, f"fq{hq}_{batch}")
    qn = synth.norm_weight((d,), 2, "fqn", device=DEV)
    kn = synth.norm_weight((d,), 3, "fkn", device=DEV)
    cos, sin = qo.rope_cache(qo.rope_inv_freq(d, 1e6), S, torch.bfloat16)
    cos, sin = cos.to(DEV), sin.to(DEV)
    kc0 = _rand((batch, hkv, S, d), 1.0, f"fkc{batch}")
    vc0 = _rand((batch, hkv, S, d), 1.0, f"fvc{batch}")
    cache_pos = torch.tensor(lens, device=DEV, dtype=torch.int32)
    scale = d ** -0.5
    K.device_error(clear=True)
    kc1, vc1 = kc0.clone(), vc0.clone()
    q = K.qk_norm_rope(qkv, batch, 1, hq, hkv, d, qn, kn, cos, sin, cache_pos=cache_pos, k_cache=kc1, v_cache=vc1,
                       max_seq=S)
    want = K.decode_attention(q, kc1, vc1, batch, 1, hq, hkv, d, S, scale, cache_pos=cache_pos)
    kc2, vc2 = kc0.clone(), vc0.clone()
    got = K.decode_attention_qkv(qkv, batch, hq, hkv, d, qn, kn, cos, sin, kc2, vc2, S, scale, cache_pos=cache_pos)
    assert K.device_error(clear=True) == 0
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    assert torch.equal(got, want)
    if len(set(lens)) == 1:  # uniform cursor via the host argument
        kc3, vc3 = kc0.clone(), vc0.clone()
        got3 = K.decode_attention_qkv(qkv, batch, hq, hkv, d, qn, kn, cos, sin, kc3, vc3, S, scale,
                                      uniform_past=lens[0])
        assert torch.equal(got3, want) and torch.equal(kc3, kc1)


def test_decode_attention_qkv_overflow_sets_flag_and_appends_nothing():
    hq, hkv, d, S = 32, 8, 128, 64
    qkv = _rand((1, (hq + 2 * hkv) * d), 1.0, "fo")
    qn = synth.norm_weight((d,), 2, "foqn", device=DEV)
    cos, sin = qo.rope_cache(qo.rope_inv_freq(d, 1e6), 2 * S, torch.bfloat16)
    kc = _rand((1, hkv, S, d), 1.0, "fokc")
    vc = _rand((1, hkv, S, d), 1.0, "fovc")
    k0, v0 = kc.clone(), vc.clone()
    K.device_error(clear=True)
    cache_pos = torch.tensor([S], device=DEV, dtype=torch.int32)  # one past the arena
    K.decode_attention_qkv(qkv, 1, hq, hkv, d, qn, qn, cos.to(DEV), sin.to(DEV), kc, vc, S, d ** -0.5,
                           cache_pos=cache_pos)
    assert K.device_error(clear=True) == 6  # LS_ERR_KV_OVERFLOW
    assert torch.equal(kc, k0) and torch.equal(vc, v0)
    assert K.device_error(clear=True) == 0


def test_lmhead_argmax_matches_bf16_logits_and_ties():
    vocab, hidden = 151936, 2560
    w = _rand((vocab, hidden), 0.02, "lm")
    h = _rand((2, hidden), 1.0, "hh")
    nw = synth.norm_weight((hidden,), 3, "fn", device=DEV)
    ids = K.lmhead_argmax(h, nw, w, 1e-6)
    hn = _rms_ref(h, nw, 1e-6)
    logits = (hn.float() @ w.float().t()).bfloat16()
    for r in range(2):
        row = logits[r].float()
        top2 = row.topk(2).values
        best = row.max()
        first_max = int(torch.nonzero(row == best)[0])
        if (top2[0] - top2[1]).item() > 2 ** -5:  # no near-tie: must be the reference's argmax
            assert int(ids[r]) == first_max
        else:  # near-tie: a different fp32 summation order may pick the neighbour
            assert row[ids[r]].item() >= best.item() - 2 ** -5
    # exact ties with exactly representable logits: lowest index must win
    w2 = torch.zeros(vocab, 256, device=DEV, dtype=torch.bfloat16)
    w2[:, 0] = 0.25
    w2[100000, 1] = 1.0
    w2[7, 1] = 1.0
    w2[150000, 1] = 1.0
    h2 = torch.zeros(1, 256, device=DEV, dtype=torch.bfloat16)
    h2[0, :2] = 1.0
    assert int(K.lmhead_argmax(h2, None, w2, 1e-6)[0]) == 7
    w2[3, 1] = 1.0
    assert int(K.lmhead_argmax(h2, None, w2, 1e-6)[0]) == 3


def test_kv_overflow_sets_device_flag_without_fault():
    hq, hkv, d, hidden = 4, 2, 128, 512
    x = _rand((1, hidden), 1.0, "ox")
    w = _rand(((hq + 2 * hkv) * d, hidden), 0.02, "ow")
    qn = synth.norm_weight((d,), 2, "oqn", device=DEV)
    cos, sin = qo.rope_cache(qo.rope_inv_freq(d, 1e6), 64, torch.bfloat16)
    kc = torch.zeros(1, hkv, 16, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    K.device_error(clear=True)
    cache_pos = torch.tensor([16], device=DEV, dtype=torch.int32)  # one past the arena
    K.qkv_rope_append(x, 1, 1, w, hq, hkv, d, qn, qn, cos.to(DEV), sin.to(DEV), cache_pos=cache_pos, k_cache=kc,
                      v_cache=vc, max_seq=16)
    assert K.device_error(clear=True) == 6  # LS_ERR_KV_OVERFLOW
    assert kc.abs().sum().item() == 0
    assert K.device_error(clear=True) == 0


@pytest.mark.parametrize("m", [1, 3, 8])
def test_linear_f32_partials_and_residual_add(m):
    """Row-split (tensor-parallel) form of o_proj / down: the fp32 partials of two
    halves of the in-features, summed and passed to the residual-add kernel,
    match the unsplit residual linear within the bound."""
    k, n = 4096, 2560
    x = _rand((m, k), 1.0, "xp")
    w = _rand((n, k), 0.02, "wp")
    res = _rand((m, n), 1.0, "resp")
    parts = [K.linear(x[:, h * k // 2:(h + 1) * k // 2].contiguous(), w[:, h * k // 2:(h + 1) * k // 2].contiguous(),
                      epilogue=K.EPI_STORE_F32) for h in range(2)]
    assert parts[0].dtype == torch.float32
    full = K.linear(x, w, epilogue=K.EPI_STORE_F32)
    ref = x.float() @ w.float().t()
    assert (full - ref).abs().max().item() <= 1e-3 * max(1.0, ref.abs().max().item())
    y = K.residual_add_f32(res, parts[0] + parts[1])
    ref_y = res.float() + ref.bfloat16().float()
    assert (y.float() - ref_y).abs().max().item() <= tol(ref_y)
    # Same rounding points as the fused residual epilogue.
    y1 = K.residual_add_f32(res, full)
    assert (y1 == K.oproj_residual(x, w, res)).float().mean().item() > 0.99


@pytest.mark.parametrize("batch,q_len,past", [(1, 64, 0), (2, 200, 37), (1, 512, 0), (2, 96, 300)])
def test_prefill_attention_matches_fp64(batch, q_len, past):
    """Long query blocks (>= 256 rows per kv head) take the 128-row prefill kernel;
    causal rule key j <= cache_pos + i, against an fp64 softmax of the same bf16 inputs."""
    hq, hkv, d, S = 32, 8, 128, 1024
    gen = torch.Generator(device="cpu").manual_seed(7 + q_len)
    q = torch.randn(batch * q_len, hq, d, generator=gen).bfloat16().to(DEV)
    kc = torch.randn(batch, hkv, S, d, generator=gen).bfloat16().to(DEV)
    vc = torch.randn(batch, hkv, S, d, generator=gen).bfloat16().to(DEV)
    pos = torch.tensor([past + 5 * b for b in range(batch)], dtype=torch.int32, device=DEV)
    scale = d ** -0.5
    out = K.decode_attention(q, kc, vc, batch, q_len, hq, hkv, d, S, scale, cache_pos=pos)
    torch.cuda.synchronize()
    qc, kcc, vcc = q.cpu().double(), kc.cpu().double(), vc.cpu().double()
    G = hq // hkv
    ref = torch.empty(batch * q_len, hq, d, dtype=torch.float64)
    for b in range(batch):
        cp = int(pos[b])
        L = cp + q_len
        for h in range(hq):
            k = kcc[b, h // G, :L]
            v = vcc[b, h // G, :L]
            s = (qc[b * q_len:(b + 1) * q_len, h] @ k.t()) * scale
            mask = torch.arange(L)[None, :] > (cp + torch.arange(q_len))[:, None]
            s = s.masked_fill(mask, float("-inf"))
            ref[b * q_len:(b + 1) * q_len, h] = torch.softmax(s, -1) @ v
    ref = ref.view(batch * q_len, hq * d)
    err = (out.double().cpu() - ref).abs().max().item()
    assert err <= 1e-2, err
    assert (out.cpu() == ref.bfloat16()).float().mean().item() > 0.99
    assert K.device_error() == 0


@pytest.mark.parametrize("hq,hkv,batch,q_len,past", [(16, 8, 2, 150, 19), (32, 8, 1, 300, 0), (32, 8, 3, 70, 1)])
def test_prefill_attention_ignores_cache_past_the_sequence(hq, hkv, batch, q_len, past):
    """Cache positions past each sequence's length hold NaN (the cache is the caller's
    memory): the prefill kernel must keep them out of the result, since 0 x NaN is NaN.
    Also covers 2 query heads per kv head (the 0.6B draft geometry) and lengths that
    end inside a key tile."""
    d, S = 128, 640
    gen = torch.Generator(device="cpu").manual_seed(31 + q_len)
    q = torch.randn(batch * q_len, hq, d, generator=gen).bfloat16()
    kc = torch.randn(batch, hkv, S, d, generator=gen).bfloat16()
    vc = torch.randn(batch, hkv, S, d, generator=gen).bfloat16()
    pos = [past + 7 * b for b in range(batch)]
    for b in range(batch):
        kc[b, :, pos[b] + q_len:] = float("nan")
        vc[b, :, pos[b] + q_len:] = float("nan")
    scale = d ** -0.5
    out = K.decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), batch, q_len, hq, hkv, d, S, scale,
                             cache_pos=torch.tensor(pos, dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    G = hq // hkv
    qd, kd, vd = q.double(), kc.double(), vc.double()
    ref = torch.empty(batch * q_len, hq, d, dtype=torch.float64)
    for b in range(batch):
        L = pos[b] + q_len
        mask = torch.arange(L)[None, :] > (pos[b] + torch.arange(q_len))[:, None]
        for h in range(hq):
            s = (qd[b * q_len:(b + 1) * q_len, h] @ kd[b, h // G, :L].t()) * scale
            ref[b * q_len:(b + 1) * q_len, h] = torch.softmax(s.masked_fill(mask, float("-inf")), -1) @ vd[b, h // G, :L]
    ref = ref.view(batch * q_len, hq * d)
    got = out.double().cpu()
    assert torch.isfinite(got).all()
    assert (got - ref).abs().max().item() <= 1e-2
    assert (out.cpu() == ref.bfloat16()).float().mean().item() > 0.99
    assert K.device_error() == 0
