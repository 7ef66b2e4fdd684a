"""The CPU oracle against golden vectors produced by the live reference.

`tests/golden/make_golden.py` ran the reference's own torch path; these tests pin
`oracle/` to it before the oracle is trusted as the checker of the CUDA path.
"""

import os

import pytest
import torch

from oracle import model as om
from oracle import ops as oo
from motif_b200.config import MotifChordConfig

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
SMALL = dict(vocab_size=512, model_dim=64, num_heads=4, num_kv_heads=2, head_k_dim=16,
             block=('gdn', 'gdn', 'gdn', 'chord'), block_n=2)
TINY = dict(vocab_size=32000, model_dim=256, num_heads=4, num_kv_heads=None, head_k_dim=64,
            block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)


def load(name):
    return torch.load(os.path.join(GOLD, f'{name}.pt'))


def close(a, b, rtol=1e-5, atol=1e-6):
    assert a.shape == b.shape, (a.shape, b.shape)
    err = (a.double() - b.double()).abs().max().item()
    assert torch.allclose(a.double(), b.double(), rtol=rtol, atol=atol), err


def test_recurrent_delta_rule():
    d = load('gdn_recurrent')
    o, S = oo.recurrent_gated_delta_rule(d['q'], d['k'], d['v'], d['beta'], d['g'], d['S0'])
    close(o, d['o']); close(S, d['S'])


@pytest.mark.parametrize('name', ['gdn_chunk_ragged', 'gdn_chunk_d64'])
def test_chunk_delta_rule(name):
    d = load(name)
    o, S = oo.chunk_gated_delta_rule(d['q'], d['k'], d['v'], d['beta'], d['g'], d.get('S0'), 64)
    close(o, d['o']); close(S, d['S'])


def test_chunk_matches_recurrent():
    d = load('gdn_chunk_ragged')
    o1, S1 = oo.chunk_gated_delta_rule(d['q'], d['k'], d['v'], d['beta'], d['g'], d['S0'], 64)
    o2, S2 = oo.recurrent_gated_delta_rule(d['q'], d['k'], d['v'], d['beta'], d['g'], d['S0'])
    close(o1, o2, rtol=1e-4, atol=1e-5); close(S1, S2, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize('name', ['chord_prefill', 'chord_decode', 'chord_start0'])
def test_chord(name):
    d = load(name)
    B, L = d['q'].shape[0], d['q'].shape[2]
    o = oo.chord_attention(d['q'], d['k'], d['v'], d['alpha'], d['beta'], d['mu'], d['ssmax'],
                           d['log_n'].view(1, L).expand(B, L), int(d['q_start']))
    close(o, d['o'])
    assert torch.equal(oo.log_n_table(int(d['q_start']), L), d['log_n'])


def test_attn_res_and_norms():
    d = load('attn_res')
    srcs = list(d['sources'])
    close(oo.attn_res(srcs[:2], d['query'], d['weight']), d['h2'])
    close(oo.attn_res(srcs, d['query'], d['weight']), d['h4'])
    n = load('norms')
    close(oo.rms_norm(n['x'][..., :48], n['rms_w']), n['rms'])
    close(oo.gated_rms_norm(n['x'], n['gated_w']), n['gated'])
    close(oo.swiglu(n['x']), n['swiglu'])


@pytest.mark.parametrize('dtype_name', ['fp32', 'bf16'])
def test_small_model(dtype_name):
    dtype = torch.float32 if dtype_name == 'fp32' else torch.bfloat16
    d = load(f'small_{dtype_name}')
    cfg = MotifChordConfig(**SMALL)
    P = om.make_params(cfg, seed=0, norm_jitter=0.1, dtype=dtype)
    logits, _, _ = om.forward(P, cfg, d['ids'])
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=0, atol=2e-2)
    close(logits.float(), d['logits'], **tol)
    _, _, cache = om.forward(P, cfg, d['ids'][:, :24])
    steps = []
    for t in range(24, 40):
        lg, _, cache = om.forward(P, cfg, d['ids'][:, t:t + 1], cache)
        steps.append(lg[:, 0].float())
    close(torch.stack(steps, 1), d['decode_logits'], **tol)
    if dtype == torch.float32:
        toks, _ = om.greedy(P, cfg, d['ids'][:, :16], 24)
        assert torch.equal(toks, d['greedy'])


def test_tiny_config():
    d = load('tiny')
    cfg = MotifChordConfig(**TINY)
    P = om.make_params(cfg, seed=0)
    logits, _, _ = om.forward(P, cfg, d['ids'])
    lg = logits[0]
    close(lg[-2:], d['last_logits'], rtol=1e-5, atol=1e-5)
    close(lg.max(-1).values, d['pos_max'], rtol=1e-5, atol=1e-5)
    assert torch.equal(lg.argmax(-1), d['pos_argmax'])
    close(torch.logsumexp(lg, -1), d['pos_lse'], rtol=1e-5, atol=1e-5)
    toks, margins = om.greedy(P, cfg, d['ids'], 64)
    assert torch.equal(toks, d['greedy'])


def test_sampler_oracle_matches_reference_distribution():
    """oracle/sampler.py's filtered distribution == the probabilities the reference Sampler
    hands to torch.multinomial (model/sampler.py:151-219), for six settings."""
    from oracle import sampler as osm
    d = torch.load(os.path.join(GOLD, 'sampler.pt'))
    for case, ref in zip(d['cases'].tolist(), d['probs']):
        t, k, p, rp = case
        got = osm.filtered_probs(d['logits'], d['hist'], t, None if k < 0 else int(k), None if p < 0 else p, rp)
        assert torch.allclose(got, ref.float(), atol=1e-6, rtol=1e-5), case
        assert torch.equal(got > 0, ref > 0), case  # the same support


def test_philox_known_answers():
    """Philox4x32-10 restatement against the Random123 known-answer vectors."""
    from oracle import sampler as osm
    M = 0xFFFFFFFF
    assert osm.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    assert osm.philox4x32_10([M, M, M, M], [M, M]) == [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]
    assert osm.philox4x32_10([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0]) == \
        [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]
    u = osm.philox_uniforms(1234, 7, 64)
    assert u.dtype == torch.float32 and bool((u >= 0).all()) and bool((u < 1).all())


def test_sampler_oracle_draw_is_inverse_cdf():
    """The oracle's draw: first index whose inclusive cumulative mass exceeds u * total."""
    from oracle import sampler as osm
    logits = torch.tensor([[0.0, 1.0, -float('inf'), 2.0]])
    p = torch.softmax(logits, -1)[0]
    c = torch.cumsum(p, 0)
    for u, want in [(0.0, 0), (float(c[0]) * 0.999, 0), (float(c[0]) * 1.001, 1), (float(c[1]) * 1.0001, 3),
                    (0.999999, 3)]:
        got = osm.sample(logits, None, 1.0, None, None, 1.0, torch.tensor([u]))
        assert int(got[0]) == want, (u, int(got[0]))


@pytest.mark.parametrize('kind', ['bool', 'float'])
def test_small_model_masked(kind):
    """The oracle's masked forward (keep-mask with a hole and right padding, additive float
    mask) against the reference: prefill logits, chunked prefill + decode with the mask widened
    every step, and masked greedy generation."""
    d = load('masked')
    cfg = MotifChordConfig(**SMALL)
    P = om.make_params(cfg, seed=0, norm_jitter=0.1, dtype=torch.float32)
    mask = d[f'{kind}_mask']
    logits, _, _ = om.forward(P, cfg, d['ids'], mask=mask)
    close(logits.float(), d[f'{kind}_logits'], rtol=1e-5, atol=1e-5)
    _, _, cache = om.forward(P, cfg, d['ids'][:, :24], mask=mask[:, :24])
    steps = []
    for t in range(24, 40):
        lg, _, cache = om.forward(P, cfg, d['ids'][:, t:t + 1], cache, mask=mask[:, :t + 1])
        steps.append(lg[:, 0].float())
    close(torch.stack(steps, 1), d[f'{kind}_decode_logits'], rtol=1e-5, atol=1e-5)
    toks, _ = om.greedy(P, cfg, d['ids'][:, :16], 8, mask=mask[:, :16])
    assert torch.equal(toks, d[f'{kind}_greedy'])
