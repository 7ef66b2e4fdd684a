"""Seeded, name-driven random initialisation shared by every model in this repo.

The reference has no custom initialiser (PyTorch defaults plus `A_log`/`dt_bias`
draws on the global RNG, `block/attention/gdn_attn.py:100-104`), so two models
built from the same seed in two code bases would not agree.  This function sets
every parameter from a private CPU `torch.Generator`, walking the parameter names
in sorted order, so the reference model, the CPU oracle and the CUDA model all
receive bit-identical weights from one seed:

* Linear / Embedding / Conv1d weights: N(0, 0.02);
* RMSNorm / GatedRMSNorm weights: 1 (or 1 + N(0, jitter) when `norm_jitter > 0`);
* `theta_alpha = log U(0.5, 2)`, `theta_beta = U(0, 1)`,
  `theta_mu = asinh(0.5)` (so `mu = 2 sinh(theta_mu) = 1`), `ssmax_s = 1`
  (or `U(0.8, 1.2)` with jitter);
* `pseudo_queries ~ N(0, d^-1/2)`;
* `A_log = log U(1, 16)` and `dt_bias = dt + log(-expm1(-dt))` with
  `dt = exp(U(log 1e-3, log 1e-1))`, the reference's own distributions.
"""

import math

import torch


def _is_norm_weight(name: str) -> bool:
    last = name.rsplit('.', 2)
    if len(last) < 2 or last[-1] != 'weight':
        return False
    owner = last[-2]
    return owner in ('attn_norm', 'mlp_norm', 'norm', 'q_norm', 'k_norm', 'o_norm') or \
        name.split('.')[-3:-2] == ['attn_res_norms']


def init_tensors(shapes: dict, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    """Seeded fp32 CPU values for a `{name: shape}` mapping (names as in `state_dict`).

    Tied parameters must appear once, under the name `named_parameters()` yields.
    """
    gen = torch.Generator().manual_seed(int(seed))
    out = {}
    for name in sorted(shapes):
        shape = tuple(shapes[name])
        leaf = name.rsplit('.', 1)[-1]
        if _is_norm_weight(name):
            val = torch.ones(shape)
            if norm_jitter > 0:
                val = val + norm_jitter * torch.randn(shape, generator=gen)
        elif leaf == 'theta_alpha':
            val = torch.log(0.5 + 1.5 * torch.rand(shape, generator=gen))
        elif leaf == 'theta_beta':
            val = torch.rand(shape, generator=gen)
        elif leaf == 'theta_mu':
            val = torch.full(shape, math.asinh(0.5))
        elif leaf == 'ssmax_s':
            val = torch.ones(shape)
            if norm_jitter > 0:
                val = 0.8 + 0.4 * torch.rand(shape, generator=gen)
        elif name.split('.')[-2:-1] == ['pseudo_queries']:
            val = torch.randn(shape, generator=gen) * (shape[-1] ** -0.5)
        elif leaf == 'A_log':
            val = torch.log(1.0 + 15.0 * torch.rand(shape, generator=gen))
        elif leaf == 'dt_bias':
            u = torch.rand(shape, generator=gen)
            dt = torch.exp(u * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
            val = dt + torch.log(-torch.expm1(-dt))
        else:
            val = 0.02 * torch.randn(shape, generator=gen)
        out[name] = val
    return out


@torch.no_grad()
def init_params(model: torch.nn.Module, seed: int = 0, norm_jitter: float = 0.0) -> torch.nn.Module:
    """Initialise `model` in place from `seed`; returns `model`.

    Works on any module tree with the reference's parameter names: the reference
    `MotifChordModel` or `motif_b200.model.MotifChordModel`.
    """
    named = dict(model.named_parameters())
    vals = init_tensors({k: p.shape for k, p in named.items()}, seed, norm_jitter)
    for name, p in named.items():
        p.copy_(vals[name].to(dtype=p.dtype, device=p.device))
    return model
