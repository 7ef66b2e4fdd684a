"""CUDA-graph batched decode (`motif_b200.decode.GraphDecoder`) against the eager decode path
and the reference's greedy tokens.

The graph replays the eager T = 1 kernels with device-side positions, so with the split-KV
count pinned (`model.decode_splits`) graph and eager decode must give identical token ids,
recurrent states and KV caches; against the reference (config 1, fp32) the 64 greedy tokens
must be bit-exact.
"""

import os

import pytest
import torch

from motif_b200.config import MotifChordConfig, tiny_config
from motif_b200.init import init_params

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
# head dim 32: the split-KV decode kernel serves head dims 32 and 64
SMALL = dict(vocab_size=512, model_dim=128, num_heads=4, num_kv_heads=2, head_k_dim=16,
             block=('gdn', 'gdn', 'gdn', 'chord'), block_n=2)


def build(cfg, dtype=torch.float32, jitter=0.0):
    from motif_b200.model import MotifChordModel
    torch.manual_seed(0)
    m = MotifChordModel(cfg)
    init_params(m, seed=0, norm_jitter=jitter)
    return m.to('cuda', dtype).eval()


def eager_decode(m, ids, steps):
    out = m(ids)
    cache, tok = out.cache, out.next_token()
    first = tok
    toks = []
    for _ in range(steps):
        out = m(tok, cache=cache)
        tok = out.next_token()
        toks.append(tok)
    return first, torch.cat(toks, 1), cache


def graph_decode(m, ids, steps, chunks=None):
    from motif_b200.decode import GraphDecoder
    out = m(ids)
    first = out.next_token()
    dec = GraphDecoder(m, out.cache, max_steps=steps)
    parts, tok = [], first
    for n in (chunks or [steps]):
        t = dec.run(tok, n)
        parts.append(t.clone())
        tok = t[:, -1:]
    return first, torch.cat(parts, 1), out.cache, dec


def _gdn_states(cache):
    from motif_b200.cache import GatedDeltaAttentionLayerCache
    return [lc.state for bc in cache for lc in bc.attn if isinstance(lc, GatedDeltaAttentionLayerCache)]


def _kv(cache):
    from motif_b200.cache import KVLayerCache
    return [(lc.k, lc.v) for bc in cache for lc in bc.attn if isinstance(lc, KVLayerCache)]


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_graph_matches_eager_small(dtype):
    m = build(MotifChordConfig(**SMALL), dtype=dtype, jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (3, 40), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        f_e, t_e, c_e = eager_decode(m, ids, 20)
        f_g, t_g, c_g, dec = graph_decode(m, ids, 20)
    assert torch.equal(f_e, f_g)
    assert torch.equal(t_e, t_g), (t_e != t_g).nonzero()
    for a, b in zip(_gdn_states(c_e), _gdn_states(c_g)):
        assert torch.equal(a, b)
    for (ka, va), (kb, vb) in zip(_kv(c_e), _kv(c_g)):
        assert ka.shape == kb.shape and torch.equal(ka, kb) and torch.equal(va, vb)
    assert dec.launches_per_step > 0


def test_graph_run_in_parts_equals_one_run():
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (2, 33), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.no_grad():
        _, whole, _, _ = graph_decode(m, ids, 12)
        _, parts, cache, dec = graph_decode(m, ids, 12, chunks=[5, 7])
    assert torch.equal(whole, parts)
    assert all(lc.length == 33 + 12 for bc in cache for lc in bc.attn)
    with pytest.raises(ValueError):
        dec.run(parts[:, -1:], 1)   # past max_steps


def test_graph_then_eager_continues():
    """After a graph run the cache's host lengths are advanced: the eager path continues."""
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (2, 30), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        _, t_e, _ = eager_decode(m, ids, 10)
        _, t_g, cache, _ = graph_decode(m, ids, 6)
        tok = t_g[:, -1:]
        rest = []
        for _ in range(4):
            out = m(tok, cache=cache)
            tok = out.next_token()
            rest.append(tok)
    assert torch.equal(t_e, torch.cat([t_g] + rest, 1))


def test_tiny_config_graph_greedy64_matches_reference():
    d = torch.load(os.path.join(GOLD, 'tiny.pt'))
    m = build(tiny_config())
    ids = d['ids'].cuda()
    with torch.no_grad():
        first, toks, _, _ = graph_decode(m, ids, 63)
    gen = torch.cat([first, toks], 1).cpu()
    assert torch.equal(gen, d['greedy']), (gen != d['greedy']).nonzero()


@pytest.mark.parametrize('B', [4, 48])
def test_random_filled_cache_decode_172m_matches_eager(B):
    """The benchmark's decode set-up (172M shapes, bf16, caches filled with seeded random
    contents at length 1000): the CUDA-graph steps equal the eager T = 1 forward fed the same
    tokens on a copy of the same caches (same kernels, split count pinned), token for token
    and logit for logit; cache lengths advance by one per step.  4 requests take the
    weight-streaming legacy-MMA products, 48 the tensor-core decode GEMM and its fused gated
    residual."""
    import copy
    from motif_b200.config import config_172m
    from motif_b200.decode import GraphDecoder, fill_cache_random
    m = build(config_172m(), dtype=torch.bfloat16)
    L, steps = 1000, 8
    cache = fill_cache_random(m, m.create_cache(), B, L, L + steps)
    m.decode_splits = 6
    twin = copy.deepcopy(cache)
    with torch.no_grad():
        dec = GraphDecoder(m, cache, max_steps=steps)
        first = torch.arange(B, dtype=torch.int64, device='cuda').view(B, 1) * 7
        tok, g_toks, g_logits = first, [], []
        for _ in range(steps):
            tok = dec.run(tok, 1)
            torch.cuda.synchronize()
            g_toks.append(tok.clone())
            g_logits.append(dec.logits.float().clone())
        tok, e_toks, e_logits = first, [], []
        for _ in range(steps):
            out = m(tok, cache=twin)
            twin = out.cache
            e_logits.append(out.logits[:, 0].float())
            tok = out.next_token()
            e_toks.append(tok)
    m.decode_splits = None
    assert torch.equal(torch.cat(g_toks, 1), torch.cat(e_toks, 1))
    assert torch.equal(torch.stack(g_logits), torch.stack(e_logits))
    assert all(lc.length == L + steps for bc in cache for lc in bc.attn)


@pytest.mark.parametrize('rp', [1.0, 1.3])
def test_graph_sampled_matches_eager_generation(rp):
    """Sampled decode: the graph (Philox offset = sampler offset + device step counter, device
    history buffer for the penalty) draws the same tokens as the eager `Generation` loop with
    an identically seeded sampler."""
    from motif_b200.decode import GraphDecoder
    from motif_b200.generate import Generation
    from motif_b200.sampler import Sampler
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (3, 24), generator=torch.Generator().manual_seed(4)).cuda()
    kw = dict(temperature=0.9, top_k=40, top_p=0.95, repetition_penalty=rp, seed=21)
    steps = 12
    with torch.no_grad():
        gen = Generation(m, ids, max_new_tokens=steps + 1, sampler=Sampler(**kw)).run()
        s = Sampler(**kw)
        out = m(ids)
        first = out.next_token(sampler=s, input_ids=ids)
        seq = torch.cat([ids, first], 1)
        dec = GraphDecoder(m, out.cache, max_steps=steps, sampler=s)
        a = dec.run(first, 5, history=seq)
        b = dec.run(a[:, -1:], steps - 5)
    got = torch.cat([first, a, b], 1)
    assert torch.equal(got, gen.generated), (got != gen.generated).nonzero()
    assert s.offset == 1 + steps
    with pytest.raises(NotImplementedError):
        GraphDecoder(m, out.cache, max_steps=1, sampler=Sampler(**kw).with_constraint(object()))


def _gdn_and_lengths(cache):
    from motif_b200.cache import GatedDeltaAttentionLayerCache
    states = [lc.state.clone() for bc in cache for lc in bc.attn if isinstance(lc, GatedDeltaAttentionLayerCache)]
    return states, [lc.length for bc in cache for lc in bc.attn]


@pytest.mark.parametrize('sampled,sync_every', [(False, 16), (False, 3), (True, 5), (True, 1)])
def test_generation_graph_mode_matches_eager(sampled, sync_every):
    """`generate(graph=True)`: device-side eos bookkeeping, one host read per chunk, and a
    rewind when every row finished inside a chunk — the tokens, finished flags, recurrent
    states and cache lengths equal the step-by-step loop's."""
    from motif_b200.sampler import Sampler
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (3, 20), generator=torch.Generator().manual_seed(5)).cuda()
    kw = dict(temperature=0.9, top_k=30, repetition_penalty=1.2, seed=3) if sampled else None
    mk = (lambda: Sampler(**kw)) if sampled else (lambda: None)
    with torch.no_grad():
        probe = m.generate(ids, max_new_tokens=24, sampler=mk()).run().generated
        # eos ids that end each row at a different step, the last one inside a chunk
        eos = sorted({int(probe[0, 4]), int(probe[1, 9]), int(probe[2, 13])})
        ref = m.generate(ids, max_new_tokens=24, eos_token_id=eos, sampler=mk()).run()
        got = m.generate(ids, max_new_tokens=24, eos_token_id=eos, sampler=mk(), graph=True,
                         sync_every=sync_every).run()
    assert got.graph_steps > 0
    assert torch.equal(got.sequences, ref.sequences), (got.generated, ref.generated)
    assert torch.equal(got.finished, ref.finished) and got.steps == ref.steps
    s_ref, l_ref = _gdn_and_lengths(ref.cache)
    s_got, l_got = _gdn_and_lengths(got.cache)
    assert l_got == l_ref
    for a, b in zip(s_got, s_ref):
        assert torch.equal(a, b)


def test_generation_graph_mode_runs_to_max_tokens():
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    m.decode_splits = 2
    ids = torch.randint(0, 512, (2, 17), generator=torch.Generator().manual_seed(6)).cuda()
    with torch.no_grad():
        ref = m.generate(ids, max_new_tokens=21).run()
        got = m.generate(ids, max_new_tokens=21, graph=True, sync_every=8).run()
    assert got.graph_steps == 20 and torch.equal(got.sequences, ref.sequences)
    # continuing eagerly from the graph's cache gives the eager continuation
    with torch.no_grad():
        a = m.generate(ref.sequences, max_new_tokens=4, cache=ref.cache).run().generated
        b = m.generate(got.sequences, max_new_tokens=4, cache=got.cache).run().generated
    assert torch.equal(a, b)
