"""Megatron-style tensor parallelism of the Qwen3 decode path (one process per GPU).

Partition, per rank r of t (every rank keeps the full residual stream):

* fused QKV, column split by heads: q heads ``[r*Hq/t, (r+1)*Hq/t)`` and kv
  heads ``[r*Hkv/t, (r+1)*Hkv/t)``; with ``Hq/t`` a multiple of the GQA group
  size, local q head i uses local kv head ``i // G`` exactly as in the full
  model.  The KV cache of a rank holds its kv heads only.
* gate_up, column split: gate rows and up rows of the same intermediate slice
  ``[r*I/t, (r+1)*I/t)``, re-fused as ``[gate_r; up_r]`` -- not a contiguous
  slice of the fused ``[gate; up]`` tensor.
* o_proj and down_proj, row split (split of their in-features): each rank
  produces an fp32 partial of the full ``[M, H]`` output, the partials are
  summed by one all-reduce, and the residual epilogue rounds the sum to bf16
  once, as the unsplit linear does (``qwen_explicit.py:819-829``).
* lm_head, split by vocab rows ``[r*V/t, (r+1)*V/t)``: each rank reduces its
  shard to one (logit, id) key per row and a MAX all-reduce of the int64 keys
  picks the global greedy token with torch.argmax's lowest-id tie rule
  (``qwen_explicit.py:952-960``).  With tied embeddings the shard is a view of
  the (replicated) embedding table.

Messages per decode step: two fp32 ``[M, H]`` all-reduces per layer and one
``[M]`` int64 MAX all-reduce for the head.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from .config import QwenGeometry

LAYER_PREFIX = "model.layers.{}."


def check_divisible(geometry: QwenGeometry, world: int) -> None:
    g = geometry
    if world < 1:
        raise ValueError("world size must be >= 1")
    for name, v in (("num_attention_heads", g.num_attention_heads), ("num_key_value_heads", g.num_key_value_heads),
                    ("intermediate_size", g.intermediate_size), ("vocab_size", g.vocab_size)):
        if v % world:
            raise ValueError(f"{name}={v} is not divisible by the tensor-parallel size {world}")
    if (g.intermediate_size // world) % 8:
        raise ValueError(f"intermediate slice {g.intermediate_size // world} is not a multiple of 8")


def local_geometry(geometry: QwenGeometry, world: int) -> QwenGeometry:
    """The geometry one rank computes: heads and intermediate divided by ``world``.

    ``hidden_size`` and ``vocab_size`` stay whole (the residual stream and the
    embedding are replicated; the head shard is described by :class:`TPShard`).
    """
    check_divisible(geometry, world)
    g = geometry
    if world == 1:
        return g
    return replace(g, key=f"{g.key}/tp{world}", num_attention_heads=g.num_attention_heads // world,
                   num_key_value_heads=g.num_key_value_heads // world,
                   intermediate_size=g.intermediate_size // world)


@dataclass(frozen=True)
class TPShard:
    rank: int
    world: int
    vocab_offset: int
    vocab_rows: int


def shard_info(geometry: QwenGeometry, rank: int, world: int) -> TPShard:
    check_divisible(geometry, world)
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside 0..{world - 1}")
    rows = geometry.vocab_size // world
    return TPShard(rank=rank, world=world, vocab_offset=rank * rows, vocab_rows=rows)


def _rows(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    n = t.shape[0] // world
    return t[rank * n:(rank + 1) * n]


def _cols(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    n = t.shape[1] // world
    return t[:, rank * n:(rank + 1) * n]


def shard_layer_tensors(tensors: dict[str, torch.Tensor], geometry: QwenGeometry, layer_idx: int, rank: int,
                        world: int) -> dict[str, torch.Tensor]:
    """Hugging Face-named tensors of one layer, cut to rank ``rank``'s shard (contiguous copies)."""
    check_divisible(geometry, world)
    p = LAYER_PREFIX.format(layer_idx)
    out = {}
    for name in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                 "mlp.gate_proj.weight", "mlp.up_proj.weight"):
        out[p + name] = _rows(tensors[p + name], rank, world).contiguous()
    for name in ("self_attn.o_proj.weight", "mlp.down_proj.weight"):
        out[p + name] = _cols(tensors[p + name], rank, world).contiguous()
    for name in ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                 "self_attn.k_norm.weight"):
        out[p + name] = tensors[p + name]
    return out


def shard_checkpoint(tensors: dict[str, torch.Tensor], geometry: QwenGeometry, rank: int, world: int,
                     layer_indices=None) -> dict[str, torch.Tensor]:
    """Rank ``rank``'s tensors: sharded layers, the replicated embedding / final
    norm, and (for an untied head) the vocab shard of ``lm_head.weight``."""
    idx = range(geometry.num_hidden_layers) if layer_indices is None else layer_indices
    out: dict[str, torch.Tensor] = {}
    for i in idx:
        out.update(shard_layer_tensors(tensors, geometry, i, rank, world))
    for name in ("model.embed_tokens.weight", "model.norm.weight"):
        if name in tensors:
            out[name] = tensors[name]
    if "lm_head.weight" in tensors:
        out["lm_head.weight"] = _rows(tensors["lm_head.weight"], rank, world).contiguous()
    return out


def materialize_tp_shard(geometry: QwenGeometry, tensors: dict[str, torch.Tensor], rank: int, world: int,
                         device="cuda:0", dtype="bfloat16"):
    """Build rank ``rank``'s runtime: local-geometry layers, full embedding, and
    ``lm_head_weight`` set to the rank's vocab shard (a view of the embedding when tied)."""
    from .leanserve import materialize_from_tensors

    shard = shard_info(geometry, rank, world)
    local = shard_checkpoint(tensors, geometry, rank, world)
    untied = "lm_head.weight" in local
    lm_shard = local.pop("lm_head.weight", None)
    rt = materialize_from_tensors(local_geometry(geometry, world), local, device=device, dtype=dtype,
                                  include_output_head=True, free_source=True)
    if untied:
        lm = lm_shard.to(rt.device, rt.dtype).contiguous()
    else:
        lm = rt.embed_tokens_weight[shard.vocab_offset:shard.vocab_offset + shard.vocab_rows]
    rt = replace(rt, lm_head_weight=lm)
    return rt, shard


# ---------------------------------------------------------------------------
# Argmax keys (host mirror of the device encoding in csrc/common.cuh)
# ---------------------------------------------------------------------------

def argmax_key(value: float, token_id: int) -> int:
    """Signed 64-bit key whose max selects the largest value, then the lowest id."""
    import struct

    v = float(torch.tensor(value, dtype=torch.float32).item()) + 0.0
    u = struct.unpack("<I", struct.pack("<f", v))[0]
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    k = (u << 32) | (0xFFFFFFFF - (token_id & 0xFFFFFFFF))
    k ^= 1 << 63
    return k - (1 << 64) if k >= (1 << 63) else k


def argmax_key_id(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


# ---------------------------------------------------------------------------
# Collectives
# ---------------------------------------------------------------------------

class TPComm:
    """The collectives of the tensor-parallel step, over a torch.distributed group.

    NCCL for CUDA tensors (captured into the decode graph like any other
    launch); gloo works for the CPU tests of the partition math.  ``p2p`` (set
    by :meth:`enable_p2p`) is the exchange of the fused one-shot all-reduce
    that the CUDA-core row-split linears use instead of NCCL; ``p2p_tc`` a
    second exchange (up to 128 rows) for the one-shot all-reduce of the
    tensor-core row-split linears' fp32 partials.
    """

    def __init__(self, rank: int, world: int, group=None):
        self.rank = rank
        self.world = world
        self.group = group
        self.p2p: P2PExchange | None = None
        self.p2p_tc: P2PExchange | None = None

    def enable_p2p(self, width: int, max_rows: int = 8, max_ctas: int = 512,
                   tc_rows: int = 128) -> "P2PExchange":
        """Set up the fused all-reduce exchanges (a collective: every rank calls it)."""
        if self.world > 1 and self.p2p is None:
            self.p2p = P2PExchange(self, width, max_rows, max_ctas)
            self.p2p_tc = P2PExchange(self, width, tc_rows, max_ctas)
        return self.p2p

    def close(self) -> None:
        for ex in (self.p2p, self.p2p_tc):
            if ex is not None:
                ex.close()
        self.p2p = self.p2p_tc = None

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def all_reduce_max(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)


class P2PExchange:
    """Exchange regions of the fused one-shot all-reduce (``ls_linear_allreduce_residual``).

    Every rank allocates one region (``cudaMalloc``, zeroed), exports a CUDA
    IPC handle, gathers the others' handles over the process group and maps
    them (plain peer mappings, no multicast).  Refuses to run when two ranks
    share a GPU: the kernel's ranks wait on each other and must run
    concurrently, one per device.
    """

    def __init__(self, comm: TPComm, width: int, max_rows: int = 8, max_ctas: int = 512):
        import ctypes

        import torch.distributed as dist

        from . import _native as nat

        if comm.world > nat.MAX_TP_RANKS:
            raise ValueError(f"the fused all-reduce handles up to {nat.MAX_TP_RANKS} ranks")
        dev = torch.cuda.current_device()
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuids: list = [None] * comm.world
        dist.all_gather_object(uuids, uuid, group=comm.group)
        if len(set(uuids)) != comm.world:
            raise RuntimeError("the fused all-reduce needs one GPU per rank")
        nbytes = ctypes.c_int64(0)
        nat.call("ls_p2p_region_bytes", max_rows, width, max_ctas, ctypes.byref(nbytes))
        region = ctypes.c_void_p(0)
        nat.call("ls_p2p_alloc", nbytes.value, ctypes.byref(region))
        handle = (ctypes.c_ubyte * 64)()
        nat.call("ls_ipc_get_handle", region, handle)
        handles: list = [None] * comm.world
        dist.all_gather_object(handles, bytes(handle), group=comm.group)
        self.region = region.value
        self.opened: list[int] = []
        desc = nat.P2PExchangeDesc()
        for q in range(comm.world):
            if q == comm.rank:
                desc.peer[q] = self.region
                continue
            h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[q])
            ptr = ctypes.c_void_p(0)
            nat.call("ls_ipc_open", h, ctypes.byref(ptr))
            desc.peer[q] = ptr.value
            self.opened.append(ptr.value)
        desc.rank, desc.world, desc.max_ctas, desc.max_rows, desc.width = comm.rank, comm.world, max_ctas, \
            max_rows, width
        self.desc = desc
        self._group = comm.group
        dist.barrier(group=comm.group)  # every region is zeroed and mapped before any kernel signals

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (after every rank has stopped using them)."""
        import torch.distributed as dist

        from . import _native as nat

        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier(group=self._group)
        for ptr in self.opened:
            nat.call("ls_ipc_close", ptr)
        self.opened = []
        if self.region:
            nat.call("ls_p2p_free", self.region)
            self.region = 0
