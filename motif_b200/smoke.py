"""Tiny end-to-end run of the model on the CUDA path, checked against the CPU oracle."""

import torch

from .config import MotifChordConfig
from .init import init_params


def model_smoke(dev) -> None:
    from oracle import model as om
    from .model import MotifChordModel
    cfg = MotifChordConfig(vocab_size=512, model_dim=64, num_heads=4, num_kv_heads=2, head_k_dim=16,
                           block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)
    m = MotifChordModel(cfg)
    init_params(m, seed=0, norm_jitter=0.1)
    m = m.to(dev).eval()
    ids = torch.randint(0, 512, (2, 70), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        out = m(ids[:, :66].to(dev))
        for t in range(66, 70):
            out = m(ids[:, t:t + 1].to(dev), cache=out.cache)
    torch.cuda.synchronize(dev)
    ref, _, _ = om.forward(om.make_params(cfg, 0, 0.1), cfg, ids)
    err = ((out.logits[:, 0].cpu() - ref[:, -1]).abs().max() / ref.abs().max()).item()
    assert err < 1e-5, f'model smoke parity {err}'
