"""ls_lmhead_argmax_noalloc against ls_lmhead_argmax, both called through the C ABI.

The entry point takes its scratch from a fixed array inside the library, so it
is compared with the workspace form on the same inputs, on two calls in a row
(the second call relies on the first leaving the arrival counter at zero).
The file name sorts last so the test also runs after every other GPU test.
"""
from __future__ import annotations

import pytest
import torch

from leanstack_b200 import _native as nat
from leanstack_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _noalloc(h, norm_w, lm_w, eps, out_ids):
    hidden = h.shape[-1]
    m = h.numel() // hidden
    nat.call("ls_lmhead_argmax_noalloc", h.data_ptr(), m, hidden, norm_w.data_ptr(), float(eps), lm_w.data_ptr(),
             lm_w.shape[0], out_ids.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _with_workspace(h, norm_w, lm_w, eps):
    hidden = h.shape[-1]
    m = h.numel() // hidden
    ws = torch.zeros(K.lmhead_workspace_bytes(m, lm_w.shape[0]), device=h.device, dtype=torch.uint8)
    out = torch.empty(m, device=h.device, dtype=torch.int64)
    nat.call("ls_lmhead_argmax", h.data_ptr(), m, hidden, norm_w.data_ptr(), float(eps), lm_w.data_ptr(),
             lm_w.shape[0], out.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.parametrize("m", [1, 4, 8])
def test_noalloc_head_matches_workspace_head(m):
    dev = torch.device("cuda:0")
    gen = torch.Generator(device="cpu").manual_seed(100 + m)
    hidden, vocab, eps = 2560, 151936, 1e-6
    lm_w = (torch.randn(vocab, hidden, generator=gen) * 0.02).to(torch.bfloat16).to(dev)
    norm_w = (1.0 + 0.1 * torch.randn(hidden, generator=gen)).to(torch.bfloat16).to(dev)
    out = torch.full((m,), -1, device=dev, dtype=torch.int64)
    for call in range(2):
        h = torch.randn(m, hidden, generator=gen).to(torch.bfloat16).to(dev)
        expect = _with_workspace(h, norm_w, lm_w, eps)
        _noalloc(h, norm_w, lm_w, eps, out)
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), expect.cpu()), f"call {call}: {out.tolist()} != {expect.tolist()}"
    assert K.device_error() == 0


def test_noalloc_scratch_limit_arithmetic():
    """The fixed scratch (16 KiB) holds the head's workspace for every m the entry
    point accepts (1..8) on this GPU; the workspace arithmetic it checks against
    grows past the limit for larger m, where the workspace form still works."""
    limit = 16 * 1024
    for m in range(1, 9):
        assert K.lmhead_workspace_bytes(m, 151936) <= limit
    assert K.lmhead_workspace_bytes(16, 151936) > limit


def test_noalloc_rejects_rows_beyond_limit():
    dev = torch.device("cuda:0")
    h = torch.zeros(9, 256, device=dev, dtype=torch.bfloat16)
    w = torch.zeros(512, 256, device=dev, dtype=torch.bfloat16)
    out = torch.empty(9, device=dev, dtype=torch.int64)
    with pytest.raises(nat.LeanB200Error, match="outside 1..8"):
        _noalloc(h, w[0], w, 1e-6, out)
