"""Failure detection on the device: a bounded wait that runs out.

The fused tensor-parallel all-reduce (``ls_linear_allreduce_residual``) waits
for every rank's partials.  Here one GPU plays rank 0 of a world of two whose
rank 1 never calls: both exchange regions are local buffers, so rank 0's
pushes land and its wait for rank 1 can only run out.  With the wait limit
lowered to a few milliseconds the call must come back with LS_ERR_TIMEOUT in
the device error flag, within about one limit (the abort is shared by the
CTA, not re-armed per element), and leave the context usable.  No fault, no
hang: every wait in the kernel is bounded.  (The reference has no device-side
waits; its nearest failure handling is the ValueError cursor checks of
``src/leanstack/runtime/kv_cache.py:100-103``.)
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from conftest import tol
from leanstack_b200 import _native as nat
from leanstack_b200 import kernels as K
from leanstack_b200 import synth

pytestmark = pytest.mark.gpu
DEV = "cuda"
LS_ERR_TIMEOUT = 7


class _LocalExchange:
    """A world-2 exchange descriptor whose two regions both live on this GPU."""

    def __init__(self, width: int, max_rows: int = 8, max_ctas: int = 512):
        nbytes = ctypes.c_int64(0)
        nat.call("ls_p2p_region_bytes", max_rows, width, max_ctas, ctypes.byref(nbytes))
        self.regions = []
        for _ in range(2):
            r = ctypes.c_void_p(0)
            nat.call("ls_p2p_alloc", nbytes.value, ctypes.byref(r))
            self.regions.append(r.value)
        self.desc = nat.P2PExchangeDesc()
        self.desc.peer[0], self.desc.peer[1] = self.regions
        self.desc.rank, self.desc.world = 0, 2
        self.desc.max_ctas, self.desc.max_rows, self.desc.width = max_ctas, max_rows, width

    def close(self):
        for r in self.regions:
            nat.call("ls_p2p_free", ctypes.c_void_p(r))
        self.regions = []


def test_wait_limit_is_settable():
    assert K.wait_limit_ns() == 2_000_000_000
    K.set_wait_limit_ns(3_000_000)
    try:
        assert K.wait_limit_ns() == 3_000_000
        with pytest.raises(nat.LeanB200Error, match="outside"):
            K.set_wait_limit_ns(10)
    finally:
        K.set_wait_limit_ns(2_000_000_000)


@pytest.mark.parametrize("m", [1, 8])
def test_allreduce_wait_for_a_silent_peer_times_out(m):
    H, kdim = 2560, 2048  # a TP-2 o_proj shard
    x = synth.normal((m, kdim), 1.0, 0, "fail/x", device=DEV)
    w = synth.normal((H, kdim), 0.02, 0, "fail/w", device=DEV)
    res = synth.normal((m, H), 1.0, 0, "fail/res", device=DEV)
    out = torch.empty(m, H, device=DEV, dtype=torch.bfloat16)
    ex = _LocalExchange(H)
    assert K.device_error(clear=True) == 0
    limit_ns = 5_000_000
    K.set_wait_limit_ns(limit_ns)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        K.linear_allreduce_residual(x, w, res, ex, out=out)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        code = K.device_error(clear=True)
    finally:
        K.set_wait_limit_ns(2_000_000_000)
        ex.close()
    print(f"m={m}: silent peer -> code {code:#x} after {elapsed * 1e3:.1f} ms (limit {limit_ns / 1e6:.0f} ms)")
    assert code & 0xFF == LS_ERR_TIMEOUT
    assert code >> 8 == 0x30  # the all-reduce's wait site
    assert elapsed < 0.5  # one limit per CTA (plus launch), far below one per element
    # the context is still usable: the plain row-split linear runs and is right
    y = K.linear(x, w)
    ref = x.float() @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= tol(ref)
    assert K.device_error(clear=True) == 0
