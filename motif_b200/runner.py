"""Multi-GPU replicas: one process per GPU, requests sharded by rank, no hot-path collective.

Motif Chord inference has no exchange step: every sequence's prefill and decode touch only
that sequence's activations, KV cache and recurrent state, so N GPUs run N full replicas on
disjoint slices of the batch.  The only collectives are host plumbing — a barrier around a
timed region, the max of the ranks' times, and one gather of the per-sequence results to
the rank that needs them — never inside a forward.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 my_job.py

    from motif_b200 import runner
    ctx = runner.init()                          # reads RANK / WORLD_SIZE / LOCAL_RANK
    lo, hi = runner.shard_range(len(prompts), ctx.world, ctx.rank)
    toks = model(prompts[lo:hi].cuda()).next_token()
    all_toks = runner.gather_rows(toks, ctx)     # rank 0: every sequence, in order

The backend is NCCL on GPUs and gloo on CPU (the host-side tests run world_size 2 on gloo).
"""

import datetime
import os
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch


@dataclass
class RankContext:
    world: int
    rank: int
    local: int
    device: torch.device
    backend: Optional[str]   # None when world == 1 (no process group)


def init(backend: Optional[str] = None, timeout_s: float = 300.0) -> RankContext:
    """Join the process group named by the torchrun environment (a no-op at world size 1).

    `backend` defaults to NCCL when CUDA is available, else gloo.  The group gets a short
    timeout so that ranks waiting on a rank that died end with an error instead of hanging."""
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    use_cuda = torch.cuda.is_available() and backend != 'gloo'
    if use_cuda:
        torch.cuda.set_device(local)
        device = torch.device('cuda', local)
    else:
        device = torch.device('cpu')
    if world == 1:
        return RankContext(1, 0, local, device, None)
    import torch.distributed as dist
    backend = backend or ('nccl' if use_cuda else 'gloo')
    kw = {'device_id': device} if backend == 'nccl' else {}
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return RankContext(world, rank, local, device, backend)


def shutdown(ctx: RankContext) -> None:
    if ctx.world > 1:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice [lo, hi) of n items owned by `rank`: sizes differ by at most one and
    the first n % world ranks take the extra item.  Every item lands on exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} outside world size {world}')
    if n < 0:
        raise ValueError(f'negative item count {n}')
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int) -> List[int]:
    return [b - a for a, b in (shard_range(n, world, r) for r in range(world))]


def barrier(ctx: RankContext) -> None:
    if ctx.world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, ctx: RankContext) -> float:
    """The largest value of `x` over all ranks (a timed region is as slow as its slowest rank)."""
    if ctx.world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=ctx.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, ctx: RankContext) -> float:
    if ctx.world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=ctx.device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_rows(t: torch.Tensor, ctx: RankContext, dst: Optional[int] = 0) -> Optional[torch.Tensor]:
    """Concatenate every rank's rows (dim 0) in rank order.

    Ranks may hold different row counts (ragged shards, including zero rows).  Returns the
    full tensor on `dst` and None elsewhere; `dst=None` returns it on every rank.  One size
    exchange plus one all-gather of the padded rows — called once after a step, never inside
    a forward."""
    if ctx.world == 1:
        return t
    import torch.distributed as dist
    t = t.contiguous().to(ctx.device)
    n = torch.tensor([t.shape[0]], dtype=torch.int64, device=ctx.device)
    sizes = [torch.zeros_like(n) for _ in range(ctx.world)]
    dist.all_gather(sizes, n)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    pad = torch.zeros((mx,) + tuple(t.shape[1:]), dtype=t.dtype, device=ctx.device)
    pad[:t.shape[0]] = t
    outs = [torch.empty_like(pad) for _ in range(ctx.world)]
    dist.all_gather(outs, pad)
    if dst is not None and ctx.rank != dst:
        return None
    return torch.cat([o[:s] for o, s in zip(outs, sizes)], 0)


def run_sharded(step: Callable[[torch.Tensor], torch.Tensor], items: torch.Tensor, ctx: RankContext,
                dst: Optional[int] = 0) -> Optional[torch.Tensor]:
    """Apply `step` to this rank's shard of `items` (dim 0) and gather the results in order.

    `step` sees only its own rows (e.g. `lambda ids: model(ids.cuda()).next_token()`); the
    result has one row per input row.  An empty shard calls nothing and contributes no rows,
    but still takes part in the gather so every rank issues the same collectives."""
    lo, hi = shard_range(items.shape[0], ctx.world, ctx.rank)
    local = items[lo:hi]
    if local.shape[0]:
        out = step(local)
        if out.shape[0] != local.shape[0]:
            raise ValueError(f'step returned {out.shape[0]} rows for {local.shape[0]} inputs')
    else:
        out = None
    # every rank needs the row shape / dtype for the gather, even with an empty shard
    proto = _agree_on_prototype(out, ctx)
    if out is None:
        out = torch.empty((0,) + proto[0], dtype=proto[1], device=ctx.device)
    return gather_rows(out, ctx, dst)


def _agree_on_prototype(out: Optional[torch.Tensor], ctx: RankContext):
    if ctx.world == 1:
        return (tuple(out.shape[1:]), out.dtype) if out is not None else ((), torch.float32)
    import torch.distributed as dist
    mine = (tuple(out.shape[1:]), out.dtype) if out is not None else None
    allp: List = [None] * ctx.world
    dist.all_gather_object(allp, mine)
    for p in allp:
        if p is not None:
            return p
    return ((), torch.float32)
