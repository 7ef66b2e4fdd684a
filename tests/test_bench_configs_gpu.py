"""Parity at the sizes the benchmark reports: the 172M-class model (kv = 3, 12 heads, 4 blocks
of 3 GDN + 1 Chord, vocab 32000) at T = 4096, against the CPU oracle (the reference's torch
path restated, pinned to the reference's own outputs in `test_oracle_golden.py`).

What a bar can be on this model.  Its random-init weights make it chaotic: a rounding
difference roughly doubles with every decoder (16 of them).  Measured on the oracle itself
at T = 512: its fp32 path lands 1.3e-4 relative (max-abs over max) from its fp64 path on the
logits, and its bf16 path lands 2.2 max-abs (max |logit| 3.2, argmax agreement 35 %) from
its fp32 path, having doubled from 0.7 % after the first decoder.  So:

* fp32 (the parity mode of the north star): logits within 1e-3 relative of the oracle (the
  fp32-vs-fp64 level, with room for the kernels' other summation orders), and greedy ids
  identical wherever the oracle's top-2 margin exceeds four times the logit error of that
  step (below it the two fp32 results are a near-tie apart; those steps are counted and
  printed, and must be rare).
* bf16: no bf16 implementation can sit within 2e-2 of any other after 16 decoders, the
  reference's own bf16 path included.  Bars: the first block's increments (before the
  amplification) are no further from fp32 than the reference's bf16 path is (x1.25, or 2e-2
  relative); over the logits, our mean and max deviation from fp32 are no larger than the
  reference's own bf16 path's (x1.25).  The direct distance to the reference's bf16 logits is
  printed beside the north star's 2e-2.
"""

import os

import pytest
import torch

from motif_b200.config import config_172m
from motif_b200.init import init_params
from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def cpu_threads():
    prev = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    yield
    torch.set_num_threads(prev)


def build(cfg, dtype):
    from motif_b200.model import MotifChordModel
    torch.manual_seed(0)
    m = MotifChordModel(cfg)
    init_params(m, seed=0)
    return m.to('cuda', dtype).eval()


def oracle_params(cfg, dtype):
    """The oracle's copy of the same weights: bf16-rounded for a bf16 model (the fp32
    reference then runs on exactly the bf16 weights), fp32 otherwise."""
    P = om.make_params(cfg, 0, dtype=dtype)
    return P, {k: v.float() for k, v in P.items()}


def test_config4_prefill_t4096_bf16():
    """Config 4's sequence: B = 1 x T = 4096 prefill, bf16, all 32000 logits at every position."""
    cfg = config_172m()
    m = build(cfg, torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (1, 4096), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        out = m(ids.cuda())
        ours = out.logits.float().cpu()
        blk0 = [t.float().cpu() for t in out.cache[0].blocks]
    del out, m
    torch.cuda.empty_cache()
    P16, P32 = oracle_params(cfg, torch.bfloat16)
    ref32, _, rc32 = om.forward(P32, cfg, ids)
    ref16, _, rc16 = om.forward(P16, cfg, ids)
    ref16 = ref16.float()
    e_ours, e_ref, direct = (ours - ref32).abs(), (ref16 - ref32).abs(), (ours - ref16).abs()
    agree_ours = (ours.argmax(-1) == ref32.argmax(-1)).float().mean().item()
    agree_ref = (ref16.argmax(-1) == ref32.argmax(-1)).float().mean().item()
    print(f'config 4 (T=4096, bf16): ours vs fp32 max {e_ours.max():.4f} mean {e_ours.mean():.4f} '
          f'argmax {agree_ours:.3f}; reference bf16 vs fp32 max {e_ref.max():.4f} mean {e_ref.mean():.4f} '
          f'argmax {agree_ref:.3f}; ours vs reference bf16 max {direct.max():.4f} mean {direct.mean():.4f} '
          f'(north star 2e-2); max |logit| {ref32.abs().max():.3f}')
    for i, (o, r32, r16) in enumerate(zip(blk0, rc32.blocks[0].attn_res.blocks, rc16.blocks[0].attn_res.blocks)):
        drift = (r16.float() - r32).abs().max().item()
        err = (o - r32).abs().max().item()
        assert err <= max(2e-2 * r32.abs().max().item(), 1.25 * drift), (i, err, drift)
    assert e_ours.mean().item() <= 1.25 * e_ref.mean().item()
    assert e_ours.max().item() <= 1.25 * max(2e-2, e_ref.max().item())
    assert torch.isfinite(ours).all()


def _graph_decode_steps(m, ids, n):
    """Prefill `ids`, then n CUDA-graph greedy steps one replay at a time; returns the first
    token, the fed tokens [B, n] and each step's logits [B, n, V] (fp32, host)."""
    from motif_b200.decode import GraphDecoder
    with torch.no_grad():
        out = m(ids.cuda())
        first = out.next_token()
        last_prefill = out.logits[:, -1].float().cpu()
        dec = GraphDecoder(m, out.cache, max_steps=n)
        tok, toks, logits = first, [], []
        for _ in range(n):
            nxt = dec.run(tok, 1)
            torch.cuda.synchronize()
            logits.append(dec.logits.float().cpu().clone())
            toks.append(nxt.cpu().clone())
            tok = nxt
        dec.release()
    return first.cpu(), last_prefill, torch.cat(toks, 1), torch.stack(logits, 1)


def _oracle_teacher_forced(P, cfg, ids, first, toks):
    """The oracle fed the same tokens: prefill (its last 16 positions' logits are returned), then
    one step per fed token."""
    lg, _, cache = om.forward(P, cfg, ids)
    tail = lg[:, -16:].float()
    steps, feed = [], torch.cat([first, toks[:, :-1]], 1)
    for i in range(feed.shape[1]):
        lg, _, cache = om.forward(P, cfg, feed[:, i:i + 1], cache)
        steps.append(lg[:, 0].float())
    return tail, torch.stack(steps, 1)


def test_config5_decode_fp32_prefilled_4096():
    """Config 5's decode on a cache PREFILLED to 4096 tokens (2 sequences), fp32: 16 CUDA-graph
    greedy steps against the oracle fed the same tokens."""
    cfg = config_172m()
    m = build(cfg, torch.float32)
    n = 16
    ids = torch.randint(0, cfg.vocab_size, (2, 4096), generator=torch.Generator().manual_seed(5))
    first, pre, toks, lg = _graph_decode_steps(m, ids, n)
    del m
    torch.cuda.empty_cache()
    _, P32 = oracle_params(cfg, torch.float32)
    rtail, rlg = _oracle_teacher_forced(P32, cfg, ids, first, toks)
    rpre = rtail[:, -1]
    rel_pre = ((pre - rpre).abs().max() / rpre.abs().max()).item()
    rel = ((lg - rlg).abs().max() / rlg.abs().max()).item()
    assert torch.equal(first, rpre.argmax(-1, keepdim=True)) or rel_pre < 1e-3
    near_ties, checked = 0, 0
    for i in range(n):
        err = (lg[:, i] - rlg[:, i]).abs().max(-1).values
        top2 = rlg[:, i].topk(2, -1).values
        margin = top2[:, 0] - top2[:, 1]
        decided = margin > 4 * err
        checked += int(decided.sum())
        near_ties += int((~decided).sum())
        ours_id, ref_id = toks[:, i], rlg[:, i].argmax(-1)
        assert torch.equal(ours_id[decided], ref_id[decided]), (i, ours_id, ref_id, margin, err)
    print(f'config 5 (fp32, context 4096, 16 graph steps): prefill rel {rel_pre:.2e}, decode logits rel {rel:.2e}; '
          f'greedy ids equal on {checked} decided steps, {near_ties} near-ties')
    assert rel_pre < 1e-3 and rel < 1e-3, (rel_pre, rel)
    assert near_ties <= 2


def test_config5_decode_bf16_prefilled_4096():
    """The benchmark's decode path (bf16, CUDA graph) on a cache prefilled to 4096 tokens: each
    step's logits against the fp32 oracle fed the same tokens, within the reference's own bf16
    drift over the last 16 positions of the same prefill (x1.25)."""
    cfg = config_172m()
    m = build(cfg, torch.bfloat16)
    n = 8
    ids = torch.randint(0, cfg.vocab_size, (2, 4096), generator=torch.Generator().manual_seed(6))
    first, pre, toks, lg = _graph_decode_steps(m, ids, n)
    del m
    torch.cuda.empty_cache()
    P16, P32 = oracle_params(cfg, torch.bfloat16)
    rtail, rlg = _oracle_teacher_forced(P32, cfg, ids, first, toks)
    r16_tail = om.forward(P16, cfg, ids)[0][:, -16:].float()
    drift_max = (r16_tail - rtail).abs().max().item()
    drift_mean = (r16_tail - rtail).abs().mean().item()
    e = (lg - rlg).abs()
    print(f'config 5 (bf16, context 4096, 8 graph steps): ours vs fp32 max {e.max():.4f} mean {e.mean():.4f}; '
          f'reference bf16 drift over the prefill tail max {drift_max:.4f} mean {drift_mean:.4f}')
    assert torch.isfinite(lg).all()
    assert e.mean().item() <= 1.25 * drift_mean
    assert e.max().item() <= 1.25 * max(2e-2, drift_max)
