"""Multi-GPU sharding of the hot-path operators (one process per GPU).

Every operator here splits into independent units, so each rank computes its
own shard with no exchange on the data path:
  * RMSNorm   rows                     (w replicated)
  * GEMM      M-blocks of A / C        (B replicated)
  * SDPA      batch x head pairs       (each rank holds its heads' Q, K, V)
  * decode    sequences of the batch   (weights replicated, KV cache per sequence)
The only collective is the optional all-gather of a result onto every rank
(`gather_rows`), for callers that need the whole output on one device; it
uses torch.distributed (NCCL between GPUs, gloo on CPU).  The reference has
no multi-device path at all (one Metal device, one queue).
"""
from __future__ import annotations

from typing import Optional, Tuple


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank's contiguous share of n units; sizes differ by at most 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int):
    return [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]


def _dist():
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialised (launch one process per GPU)")
    return dist


def world_rank(group=None) -> Tuple[int, int]:
    dist = _dist()
    return dist.get_world_size(group), dist.get_rank(group)


def gather_rows(local, total_rows: int, group=None):
    """All-gather row shards (dim 0, sizes as shard_range gives them) into the full tensor
    on every rank.  Uneven shards are padded to the largest for the collective."""
    import torch
    dist = _dist()
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    sizes = shard_sizes(total_rows, world)
    if local.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, expected {sizes[rank]}")
    cap = max(sizes)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)


# ----------------------------------------------------------------------------- operators
def rmsnorm_rows(x, w, eps: float = 1e-6, gather: bool = False, group=None):
    """RMSNorm of this rank's row shard of x (x may be the full matrix or the shard).

    With a full x [rows, hidden] the rank slices its rows; with gather=True every
    rank returns the full normalised matrix."""
    from . import cuda_ops
    world, rank = world_rank(group)
    rows = x.shape[0]
    lo, hi = shard_range(rows, world, rank)
    y = cuda_ops.rmsnorm(x[lo:hi].contiguous(), w, eps)
    return gather_rows(y, rows, group) if gather else y


def gemm_mblocks(a, b, gather: bool = False, group=None):
    """C = A B with A's rows (M) split across ranks; B replicated."""
    from . import cuda_ops
    world, rank = world_rank(group)
    lo, hi = shard_range(a.shape[0], world, rank)
    c = cuda_ops.gemm(a[lo:hi].contiguous(), b)
    return gather_rows(c, a.shape[0], group) if gather else c


def sdpa_heads(q, k, v, scale: Optional[float] = None, causal: bool = False,
               gather: bool = False, group=None):
    """Attention with the batch x head pairs split across ranks ([B, H, S, D] inputs,
    MHA or GQA; a rank takes whole kv-head groups so no K/V is shared)."""
    from . import cuda_ops
    world, rank = world_rank(group)
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    units = B * Hkv                                  # (b, kv head) groups
    lo, hi = shard_range(units, world, rank)
    qf = q.reshape(B * Hkv, g, S, D)[lo:hi]
    kf = k.reshape(B * Hkv, 1, -1, D)[lo:hi]
    vf = v.reshape(B * Hkv, 1, -1, D)[lo:hi]
    o = cuda_ops.sdpa(qf.contiguous(), kf.contiguous(), vf.contiguous(), scale=scale,
                      causal=causal)                 # [units_local, g, S, D] as B' x g heads
    if not gather:
        return o
    return gather_rows(o, units, group).reshape(B, Hq, S, D)


def decode_shard_config(cfg, group=None):
    """This rank's share of a decode batch: the same layer with `batch` = its sequences
    (shard_range over cfg.batch).  Each rank builds its DecodeLayer from this config and
    so holds only its sequences' KV cache; the weights are replicated."""
    import dataclasses
    world, rank = world_rank(group)
    lo, hi = shard_range(cfg.batch, world, rank)
    return dataclasses.replace(cfg, batch=hi - lo)


def decode_sequences(layer, x, gather: bool = False, group=None, total_batch=None):
    """One decode step of this rank's sequences.  `layer` was built from
    decode_shard_config; x is either the whole batch [total_batch, hidden] (the rank's
    rows are sliced) or this rank's rows [batch_local, hidden] (then gather=True needs
    total_batch).  With gather=True every rank returns the whole batch's output."""
    world, rank = world_rank(group)
    n_local = layer.cfg.batch
    if total_batch is None and (x.shape[0] != n_local or world == 1):
        total_batch = x.shape[0]
    if x.shape[0] != n_local:
        lo, hi = shard_range(x.shape[0], world, rank)
        if hi - lo != n_local:
            raise ValueError(f"rank {rank}: layer holds {n_local} sequences, x gives {hi - lo}")
        x = x[lo:hi].contiguous()
    out = layer.step(x)
    if not gather:
        return out
    if total_batch is None:
        raise ValueError("gather=True with this rank's rows only needs total_batch")
    return gather_rows(out, total_batch, group)
