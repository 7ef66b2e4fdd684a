"""`motif_b200.install()` against the real reference package: the reference's own
`MotifChordModel`, its layers calling this library's ops through the patched names, must give
the logits of `motif_b200.model.MotifChordModel` on the same weights (fp32).

The bar is 1e-4 relative, not the op-level 1e-5: the two models round differently in fp32
before any op runs (ours folds each RMSNorm weight into the packed projection weight, W * w,
where the reference scales the activations, (x * w) W), and the two blocks amplify that.

The reference package is the unmodified install in `baseline/_ref` (skipped when absent).
"""

import os
import sys

import pytest
import torch

from motif_b200.config import MotifChordConfig
from motif_b200.init import init_params

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), 'baseline', '_ref')
SMALL = dict(vocab_size=512, model_dim=128, num_heads=4, num_kv_heads=2, head_k_dim=32,
             block=('gdn', 'gdn', 'gdn', 'chord'), block_n=2)


@pytest.fixture
def reference():
    if not os.path.isdir(os.path.join(REF, 'motif')):
        pytest.skip('the reference package is not installed in baseline/_ref')
    sys.path.insert(0, REF)
    from motif_b200 import install
    try:
        patched = install.install(strict=True)
        import motif.model.motif as rm
        yield rm, patched
    finally:
        install.uninstall()
        sys.path.remove(REF)


def rel_err(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def test_reference_model_on_patched_ops_matches_ours(reference):
    rm, patched = reference
    assert 'motif.block.attention.gdn_attn.chunk_gated_delta_rule_triton' in patched
    assert 'motif.block.attention.chord_attn.apply_chord_attention' in patched
    from motif.model.config import MotifChordConfig as RefConfig
    from motif_b200.model import MotifChordModel
    cfg = MotifChordConfig(**SMALL)
    torch.manual_seed(0)
    theirs = rm.MotifChordModel(RefConfig(**SMALL))  # built after install(): patched norm / MLP classes
    init_params(theirs, seed=0, norm_jitter=0.1)
    theirs = theirs.cuda().eval()
    torch.manual_seed(0)
    ours = MotifChordModel(cfg)
    init_params(ours, seed=0, norm_jitter=0.1)
    ours = ours.cuda().eval()
    ids = torch.randint(0, cfg.vocab_size, (2, 150), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        a = theirs(ids[:, :140])
        b = ours(ids[:, :140])
        assert rel_err(a.logits, b.logits) < 1e-4, rel_err(a.logits, b.logits)
        ca, cb = a.cache, b.cache
        for t in range(140, 150):   # decode steps through the reference's cache classes
            a = theirs(ids[:, t:t + 1], cache=ca)
            b = ours(ids[:, t:t + 1], cache=cb)
            ca, cb = a.cache, b.cache
            assert rel_err(a.logits, b.logits) < 1e-4, (t, rel_err(a.logits, b.logits))
