"""Model-level parity of `motif_b200.model.MotifChordModel` (CUDA) against the reference.

* fp32: logits within 1e-5 relative of the golden reference outputs / the CPU oracle;
  greedy decode token ids bit-exact (config 1: 64 steps).
* bf16: the reference's own bf16 torch path differs from its fp32 path by far more than
  2e-2 on these random-init models (0.08 on the small model, 0.13 on config 1, measured
  by the golden generator), so the bf16 bar is: our bf16 logits stay within
  max(2e-2, that reference bf16 noise) of the fp32 oracle run on the same bf16 weights.
"""

import os

import pytest
import torch

from motif_b200.config import MotifChordConfig, tiny_config
from motif_b200.init import init_params
from oracle import model as om

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
SMALL = dict(vocab_size=512, model_dim=64, num_heads=4, num_kv_heads=2, head_k_dim=16,
             block=('gdn', 'gdn', 'gdn', 'chord'), block_n=2)


def load(name):
    return torch.load(os.path.join(GOLD, f'{name}.pt'))


def rel_err(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def build(cfg, seed=0, jitter=0.0, dtype=torch.float32):
    from motif_b200.model import MotifChordModel
    torch.manual_seed(0)
    m = MotifChordModel(cfg)
    init_params(m, seed=seed, norm_jitter=jitter)
    return m.to('cuda', dtype).eval()


def test_small_fp32_golden():
    d = load('small_fp32')
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    ids = d['ids'].cuda()
    with torch.no_grad():
        full = m(ids).logits
        assert rel_err(full, d['logits']) < 1e-5, rel_err(full, d['logits'])
        out = m(ids[:, :24])
        steps = []
        for t in range(24, 40):
            out = m(ids[:, t:t + 1], cache=out.cache)
            steps.append(out.logits[:, 0])
        assert rel_err(torch.stack(steps, 1), d['decode_logits']) < 1e-5
    gen = m.generate(ids[:, :16], max_new_tokens=24).run().generated
    assert torch.equal(gen.cpu(), d['greedy'])


def test_small_chunked_prefill_matches_full():
    """`tests/test_unified_cache.py:173-188` on the fused path."""
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    ids = torch.randint(0, 512, (2, 200), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        full = m(ids).logits
        cache = m.create_cache()
        for s in range(0, 200, 70):
            out = m(ids[:, s:s + 70], cache=cache)
            cache = out.cache
            # the reference's bar for this check (tests/test_unified_cache.py:185-187)
            assert (out.logits - full[:, s:s + 70]).abs().max().item() < 1e-4
        assert cache.seq_len == 200


def test_small_cache_structure_and_reset():
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    ids = torch.randint(0, 512, (2, 6), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.no_grad():
        out = m(ids)
        for bc in out.cache:
            assert len(bc.attn) == 4 and bc.seq_len == 6 and len(bc.blocks) == 5
            assert bc.blocks[0].shape == (2, 6, 64)
            assert bc.attn[3].k.shape == (2, 2, 6, 16)
            assert bc.attn[0].state.shape == (2, 4, 16, 32)
            assert [c.shape for c in bc.attn[0].conv_state] == [(2, 64, 3), (2, 64, 3), (2, 128, 3)]
        first = out.logits.clone()
        out.reset_caches()
        again = m(ids, cache=out.cache)
        assert torch.allclose(again.logits, first, atol=1e-6)
        # hidden_states = final RMSNorm output, like the reference
        ref, hid, _ = om.forward(om.make_params(MotifChordConfig(**SMALL), 0, 0.1), MotifChordConfig(**SMALL),
                                 ids.cpu())
        assert rel_err(again.hidden_states, hid) < 1e-5


def test_small_bf16_within_reference_noise():
    """The small model (2 blocks) in bf16 against the reference's own bf16 logits (fixture made
    by the reference) and against fp32: the direct distance is stated beside the north star's
    2e-2; the bar is the reference's own bf16-vs-fp32 distance (x1.25): two bf16 paths that
    round at different points cannot be closer to each other than to fp32 by construction."""
    d = load('small_bf16')
    cfg = MotifChordConfig(**SMALL)
    m = build(cfg, jitter=0.1, dtype=torch.bfloat16)
    ids = d['ids'].cuda()
    with torch.no_grad():
        ours = m(ids).logits.float().cpu()
    P = {k: v.to(torch.bfloat16).float() for k, v in om.make_params(cfg, 0, 0.1).items()}
    fp32, _, _ = om.forward(P, cfg, d['ids'])
    ref_noise = (d['logits'] - fp32).abs().max().item()
    ours_err = (ours - fp32).abs().max().item()
    # the direct comparison: our bf16 logits against the reference's own bf16 logits
    direct = (ours - d['logits']).abs().max().item()
    print(f'bf16 logits: ours vs reference bf16 {direct:.4f} (north star 2e-2); ours vs fp32 {ours_err:.4f}, '
          f'reference bf16 vs fp32 {ref_noise:.4f}')
    assert direct <= 1.25 * max(2e-2, ref_noise)
    assert ours_err <= max(2e-2, ref_noise)


def test_tiny_config_fp32_golden_and_greedy64():
    """Config 1: logits vs the reference (rtol 1e-5) and 64 greedy tokens bit-exact."""
    d = load('tiny')
    m = build(tiny_config())
    ids = d['ids'].cuda()
    with torch.no_grad():
        lg = m(ids).logits[0]
    assert rel_err(lg[-2:], d['last_logits']) < 1e-5
    assert rel_err(lg.max(-1).values, d['pos_max']) < 1e-5
    assert torch.equal(lg.argmax(-1).cpu(), d['pos_argmax'])
    gen = m.generate(ids, max_new_tokens=64).run().generated
    assert torch.equal(gen.cpu(), d['greedy']), (gen.cpu() != d['greedy']).nonzero()


def test_172m_bf16_prefill_and_decode_vs_oracle():
    """172M-class architecture (kv=3, 12 heads, 4 blocks), bf16, B=2 x T=160 prefill + 4 steps.

    This random-init 4-block model amplifies any rounding difference ~3x per block, so the
    reference's own bf16 torch path (the oracle run in bf16) lands ~1.6-1.9 max-abs away from
    its fp32 path here, and any other bf16 kernel (different summation order, P rounded to
    bf16 per key tile) lands at a comparable, not identical, distance.  Bars: the first
    block's increments (before the amplification) are no further from fp32 than the
    reference's own bf16 path (x1.25, or 2e-2 relative); the logits after all four blocks stay
    within 1.25 x max(2e-2, the reference's own bf16 drift) of the fp32 oracle.
    """
    from motif_b200.config import config_172m
    cfg = config_172m()
    m = build(cfg, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (2, 164), generator=g)
    with torch.no_grad():
        full = m(ids[:, :160].cuda())
        blk0 = [t.float().cpu() for t in full.cache[0].blocks]
        steps = []
        cache = full.cache
        for t in range(160, 164):
            o = m(ids[:, t:t + 1].cuda(), cache=cache)
            cache = o.cache
            steps.append(o.logits[:, 0].float().cpu())
    P16 = om.make_params(cfg, 0, dtype=torch.bfloat16)
    P32 = {k: v.float() for k, v in P16.items()}
    ref, _, rc = om.forward(P32, cfg, ids)
    ref16, _, _ = om.forward(P16, cfg, ids[:, :160])
    noise = (ref16.float() - ref[:, :160]).abs().max().item()
    e_pre = (full.logits.float().cpu() - ref[:, :160]).abs().max().item()
    e_dec = (torch.stack(steps, 1) - ref[:, 160:]).abs().max().item()
    print(f'172M bf16: prefill max-abs {e_pre:.4f}, decode {e_dec:.4f}, reference bf16 drift {noise:.4f}')
    _, _, rc0 = om.forward(P32, cfg, ids[:, :160])
    _, _, rc16 = om.forward(P16, cfg, ids[:, :160])
    for ours, theirs, ref16 in zip(blk0, rc0.blocks[0].attn_res.blocks, rc16.blocks[0].attn_res.blocks):
        # first block, before the amplification: per increment no further from fp32 than the
        # reference's own bf16 path (or 2e-2 relative, whichever is looser)
        ref_drift = (ref16.float() - theirs).abs().max().item()
        assert (ours - theirs).abs().max().item() <= max(2e-2 * theirs.abs().max().item(), 1.25 * ref_drift)
    bar = 1.25 * max(2e-2, noise)
    assert e_pre <= bar and e_dec <= bar, (e_pre, e_dec, bar)


@pytest.mark.parametrize('kind', ['bool', 'float'])
def test_small_fp32_masked_golden(kind):
    """Attention masks on the fused path (`motif.py:592-602`, `chord_attn.py:347-356`) against
    the reference: prefill logits, chunked prefill + decode with the mask widened each step,
    and masked greedy generation (fp32, 1e-5 relative; tokens exact)."""
    d = load('masked')
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    ids = d['ids'].cuda()
    mask = d[f'{kind}_mask'].cuda()
    with torch.no_grad():
        full = m(ids, mask=mask).logits
        assert rel_err(full, d[f'{kind}_logits']) < 1e-5, rel_err(full, d[f'{kind}_logits'])
        out = m(ids[:, :24], mask=mask[:, :24])
        steps = []
        for t in range(24, 40):
            out = m(ids[:, t:t + 1], cache=out.cache, mask=mask[:, :t + 1])
            steps.append(out.logits[:, 0])
        assert rel_err(torch.stack(steps, 1), d[f'{kind}_decode_logits']) < 1e-5
        gen = m.generate(ids[:, :16], max_new_tokens=8, mask=mask[:, :16]).run().generated
    assert torch.equal(gen.cpu(), d[f'{kind}_greedy'])


def test_masked_bf16_d64_matches_oracle():
    """bf16, head dim 64 (the tcgen05 prefill and tensor-core decode kernels) with a left-padded
    keep-mask: logits within the bf16 bar of the fp32 oracle on the same weights."""
    cfg = MotifChordConfig(vocab_size=512, model_dim=256, num_heads=4, num_kv_heads=2, head_k_dim=32,
                           block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)
    m = build(cfg, jitter=0.1, dtype=torch.bfloat16)
    ids = torch.randint(0, 512, (2, 150), generator=torch.Generator().manual_seed(9))
    keep = torch.ones(2, 150, dtype=torch.bool)
    keep[1, 100:120] = False
    with torch.no_grad():
        got = m(ids.cuda(), mask=keep.cuda()).logits.float().cpu()
        plain = m(ids.cuda()).logits.float().cpu()
    # positions the mask cannot reach (row 0, and row 1 before the dropped keys) are bitwise
    # those of the unmasked forward: the key bias adds exact zeros there
    assert torch.equal(got[0], plain[0]) and torch.equal(got[1, :100], plain[1, :100])
    P = om.params_from_module(m, dtype=torch.float32)
    ref_m, _, _ = om.forward(P, cfg, ids, mask=keep)
    ref_p, _, _ = om.forward(P, cfg, ids)
    # the masked positions are as close to the fp32 oracle as the unmasked forward is to its own
    err_m = (got[1, 100:] - ref_m[1, 100:].float()).abs().max().item()
    err_p = (plain[1, 100:] - ref_p[1, 100:].float()).abs().max().item()
    assert err_m < max(2 * err_p, 2e-2), (err_m, err_p)


@pytest.mark.parametrize('functional,wide', [(True, False), (False, True), (True, True)])
def test_functional_and_wide_caches_match_grouped(functional, wide):
    """`create_cache(functional=..., wide_kv=...)` (`cache.py:42-70,255-302`) on the fused path:
    prefill + decode logits equal those with the default grouped in-place cache, and a wide
    cache holds one copy of every kv head per query head."""
    m = build(MotifChordConfig(**SMALL), jitter=0.1)
    ids = torch.randint(0, 512, (2, 30), generator=torch.Generator().manual_seed(11)).cuda()
    with torch.no_grad():
        ref = m(ids[:, :24], cache=m.create_cache())
        got = m(ids[:, :24], cache=m.create_cache(functional=functional, wide_kv=wide))
        assert rel_err(got.logits, ref.logits) < 1e-5
        rc, gc = ref.cache, got.cache
        for t in range(24, 30):
            r = m(ids[:, t:t + 1], cache=rc)
            g = m(ids[:, t:t + 1], cache=gc)
            rc, gc = r.cache, g.cache
            assert rel_err(g.logits, r.logits) < 1e-5
    from motif_b200.cache import KVLayerCache
    kv = [lc for bc in gc for lc in bc.attn if isinstance(lc, KVLayerCache)]
    H = m.config.num_heads
    for lc in kv:
        assert lc.length == 30
        if wide:
            assert lc.k.shape[1] == H
            G = H // m.config.kv_heads
            assert torch.equal(lc.k[:, 0], lc.k[:, G - 1])  # copies of kv head 0


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('T', [129, 130, 131, 67])
def test_conv_state_after_prefill_of_any_length(dtype, T):
    """The carried conv state (the raw inputs of the last three tokens) after a prefill whose
    length leaves one or two tokens in the last 8-token run: decoding the next token must give
    the logits of a full prefill that includes it (d = 256, dk = 64, dv = 128)."""
    cfg = MotifChordConfig(vocab_size=512, model_dim=256, num_heads=4, num_kv_heads=2, head_k_dim=64,
                           block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)
    m = build(cfg, jitter=0.1, dtype=dtype)
    ids = torch.randint(0, 512, (2, T + 1), generator=torch.Generator().manual_seed(T)).cuda()
    with torch.no_grad():
        full = m(ids).logits[:, -1].float()
        out = m(ids[:, :T])
        step = m(ids[:, T:], cache=out.cache).logits[:, -1].float()
    tol = 1e-5 if dtype == torch.float32 else 3e-2
    assert rel_err(step, full) < tol, rel_err(step, full)
