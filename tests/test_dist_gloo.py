"""Multi-process host logic of the replica runner on CPU: world_size 2 over gloo.

The GPU path shards sequences across ranks with no collective inside a forward; what needs
checking without a GPU is the plumbing — every sequence owned by exactly one rank, results
gathered back in order (ragged and empty shards included), the max over ranks of a timing,
and a rank that fails before a collective turning into an error on the others rather than a
hang.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from motif_b200 import runner


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn_name, q):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    ctx = None
    try:
        ctx = runner.init(backend='gloo', timeout_s=20.0)
        res = globals()[fn_name](ctx)
        q.put((rank, 'ok', res))
    except Exception as e:  # reported to the parent, which asserts on it
        q.put((rank, 'err', f'{type(e).__name__}: {e}'))
    finally:
        if ctx is not None:
            try:
                runner.shutdown(ctx)
            except Exception:
                pass


def _spawn(fn_name, world=2, timeout=120):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, res = q.get(timeout=timeout)
            out[rank] = (status, res)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out


# ---------------------------------------------------------------- per-rank bodies
def _body_gather_ragged(ctx):
    # 5 sequences on 2 ranks -> 3 + 2 rows; each row tagged with its global index
    items = torch.arange(5 * 3, dtype=torch.float32).reshape(5, 3)
    out = runner.run_sharded(lambda x: x * 2 + 1, items, ctx, dst=None)
    return out.tolist()


def _body_gather_empty(ctx):
    # 1 sequence on 2 ranks: rank 1 owns nothing but still joins the gather
    items = torch.tensor([[7, 8]], dtype=torch.int64)
    out = runner.run_sharded(lambda x: x + 100, items, ctx, dst=0)
    return None if out is None else out.tolist()


def _body_max(ctx):
    return runner.max_over_ranks(1.5 + ctx.rank, ctx), runner.sum_over_ranks(1.0, ctx)


def _body_token_step(ctx):
    # a stand-in for `model(ids).next_token()`: per-sequence argmax of a fixed projection
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 50, (6, 9), generator=g)
    table = torch.randn(50, 11, generator=g)

    def step(x):
        return table[x].sum(1).argmax(-1, keepdim=True)

    got = runner.run_sharded(step, ids, ctx, dst=0)
    return None if got is None else (got.tolist(), step(ids).tolist())


def _body_rank_dies(ctx):
    # rank 1 leaves between steps (before the collective); rank 0's next collective errors
    if ctx.rank == 1:
        raise RuntimeError('rank 1 exits before the gather')
    runner.gather_rows(torch.ones(2, 2), ctx)
    return 'gathered'


# ---------------------------------------------------------------- tests
def test_shard_range_covers_every_item_once():
    for n in range(0, 40):
        for world in range(1, 9):
            seen = []
            for r in range(world):
                lo, hi = runner.shard_range(n, world, r)
                assert 0 <= lo <= hi <= n
                seen.extend(range(lo, hi))
            assert seen == list(range(n))
            sizes = runner.shard_sizes(n, world)
            assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        runner.shard_range(4, 2, 2)
    with pytest.raises(ValueError):
        runner.shard_range(-1, 2, 0)


def test_single_process_context():
    os.environ.pop('WORLD_SIZE', None)
    ctx = runner.init(backend='gloo')
    assert (ctx.world, ctx.rank) == (1, 0)
    x = torch.arange(4).reshape(2, 2)
    assert runner.gather_rows(x, ctx) is x
    assert runner.max_over_ranks(3.0, ctx) == 3.0
    out = runner.run_sharded(lambda t: t * 2, x, ctx)
    assert torch.equal(out, x * 2)


def test_gloo_gather_ragged_in_order():
    out = _spawn('_body_gather_ragged')
    items = torch.arange(15, dtype=torch.float32).reshape(5, 3)
    want = (items * 2 + 1).tolist()
    for r in range(2):
        assert out[r] == ('ok', want)


def test_gloo_gather_with_empty_shard():
    out = _spawn('_body_gather_empty')
    assert out[0] == ('ok', [[107, 108]])
    assert out[1] == ('ok', None)


def test_gloo_max_and_sum_over_ranks():
    out = _spawn('_body_max')
    for r in range(2):
        assert out[r] == ('ok', (2.5, 2.0))


def test_gloo_sharded_step_matches_single_process():
    out = _spawn('_body_token_step')
    status, res = out[0]
    assert status == 'ok'
    got, want = res
    assert got == want
    assert out[1] == ('ok', None)


def test_gloo_rank_failure_is_an_error_not_a_hang():
    out = _spawn('_body_rank_dies', timeout=180)
    assert out[1][0] == 'err' and 'exits before the gather' in out[1][1]
    assert out[0][0] == 'err'   # the survivor's collective fails within the group timeout
