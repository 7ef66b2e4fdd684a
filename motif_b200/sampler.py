"""`Sampler` on the device (`motif/model/sampler.py:59-232`).

Same constructor, attributes and call as the reference's sampler: repetition penalty ->
temperature -> grammar constraint -> top-k -> top-p -> multinomial, then the constraint's
forcing and advance.  Everything between the constraint mask and the draw is one launch of
`motif_b200_sample` (one CTA per row, the row held in shared memory); the constraint, a
host-side grammar object, keeps its two host hooks: `mask_logits` runs on the logits before
the kernel (it only writes -inf, which the penalty and the temperature leave at -inf, so the
order does not change the result) and `apply_forcing` / `advance` on the tokens after it.

The multinomial draw reads one uniform per row from Philox4x32-10 inside the kernel: key =
`seed`, counter = (row, 0, call offset).  `seed` defaults to a draw from torch's default
generator, so `torch.manual_seed` makes a run reproducible as it does for the reference; each
call advances the offset by one.  The probabilities are exactly the reference's (fp32 math);
the draw is a different, equally distributed stream than `torch.multinomial`'s.

Differences in error behaviour: a row whose logits are all -inf (a constraint that forbids
everything) yields token -1 instead of the reference's `RuntimeError` from `torch.multinomial`
(checking would cost a host synchronisation on every step).  Vocabularies above 53248 raise
`NotImplementedError`.
"""

import copy
from typing import Optional

import torch

from . import _lib

__all__ = ['Sampler', 'make_sampler', 'sample_tokens']


def _draw_seed() -> int:
    return int(torch.randint(0, 2 ** 62, (1,)).item())


def sample_tokens(logits: torch.Tensor, input_ids: Optional[torch.Tensor] = None, temperature: float = 1.0,
                  top_k: Optional[int] = None, top_p: Optional[float] = None, repetition_penalty: float = 1.0,
                  uniforms: Optional[torch.Tensor] = None, seed: int = 0, offset: int = 0,
                  offset_dev: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                  probs: bool = False):
    """One launch of the sampling kernel on `logits` [B, V] (any float dtype, unit inner stride).

    `input_ids` [B, S] int64 (ids < 0 are ignored) feeds the repetition penalty; `uniforms`
    [B] fp32 in [0, 1) replaces the Philox draw (tests use it to pin the draw); `offset_dev`
    (an int64 device scalar added to `offset`) lets a CUDA graph advance the stream on the
    device.  Returns `(tokens [B] int64, probs [B, V] fp32 or None)`."""
    if logits.dim() != 2:
        raise ValueError(f'logits must be [B, V], got {tuple(logits.shape)}')
    if not logits.is_cuda:
        raise ValueError('the sampling kernel runs on CUDA tensors')
    x = logits if logits.stride(-1) == 1 else logits.contiguous()
    B, V = x.shape
    dev = x.device
    hist, hist_len, hist_ld = None, 0, 0
    if repetition_penalty != 1.0 and input_ids is not None:
        if input_ids.dim() != 2 or input_ids.shape[0] != B:
            raise ValueError(f'input_ids must be [{B}, S], got {tuple(input_ids.shape)}')
        hist = input_ids.to(device=dev, dtype=torch.int64)
        if hist.stride(-1) != 1:
            hist = hist.contiguous()
        hist_len, hist_ld = hist.shape[1], hist.stride(0)
        if hist_len == 0:
            hist = None
    if uniforms is not None:
        uniforms = uniforms.to(device=dev, dtype=torch.float32).contiguous()
        if uniforms.numel() != B:
            raise ValueError(f'uniforms holds {uniforms.numel()} values for {B} rows')
    if out is None:
        out = torch.empty((B,), dtype=torch.int64, device=dev)
    p = torch.empty((B, V), dtype=torch.float32, device=dev) if probs else None
    k = int(top_k) if top_k is not None else 0
    tp = float(top_p) if top_p is not None else 1.0
    _lib.call('motif_b200_sample', _lib.ptr(x), x.stride(0), B, V, _lib.ptr(hist), hist_ld, hist_len,
              float(repetition_penalty), float(temperature), k, tp, _lib.ptr(uniforms), int(seed) & (2 ** 64 - 1),
              int(offset) & (2 ** 64 - 1), _lib.ptr(offset_dev), _lib.ptr(out), _lib.ptr(p), V,
              _lib.dtype_code(x.dtype), _lib.stream_ptr(dev))
    return out, p


class Sampler:
    """Repetition penalty + temperature + top-k / top-p truncation, plus an optional grammar
    constraint (`motif/model/sampler.py:59-219`), sampled by the device kernel."""

    def __init__(self, temperature: float = 0.7, top_k: Optional[int] = None, top_p: Optional[float] = None,
                 repetition_penalty: float = 1.15, constraint=None, seed: Optional[int] = None) -> None:
        self.temperature = temperature
        self.top_k = top_k
        self.top_p = top_p
        self.repetition_penalty = repetition_penalty
        self.constraint = constraint
        self.seed = _draw_seed() if seed is None else int(seed)
        self.offset = 0

    @property
    def eos_token_id(self) -> Optional[int]:
        return getattr(self.constraint, 'eos_token_id', None)

    def __repr__(self) -> str:
        return (f'Sampler(temperature={self.temperature}, top_k={self.top_k}, '
                f'top_p={self.top_p}, repetition_penalty={self.repetition_penalty}, '
                f'constraint={type(self.constraint).__name__ if self.constraint else None})')

    def with_constraint(self, constraint, eos_token_id: Optional[int] = None) -> 'Sampler':
        """A copy bound to `constraint` (`sampler.py:119-146`); self is left untouched."""
        bound = copy.copy(self)
        bound.constraint = constraint
        if constraint is not None and eos_token_id is not None:
            constraint.eos_token_id = int(eos_token_id)
        return bound

    def _kernel_args(self):
        return dict(temperature=self.temperature, top_k=self.top_k, top_p=self.top_p,
                    repetition_penalty=self.repetition_penalty)

    def probs(self, logits: torch.Tensor, input_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The distribution the next call would sample from ([B, V] fp32); draws nothing."""
        if self.constraint is not None:
            logits = self.constraint.mask_logits(logits)
        u = torch.zeros((logits.shape[0],), dtype=torch.float32, device=logits.device)
        return sample_tokens(logits, input_ids, uniforms=u, probs=True, **self._kernel_args())[1]

    @torch.no_grad()
    def __call__(self, logits: torch.Tensor, input_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """`[B, V]` scores -> `[B, 1]` sampled ids (`sampler.py:151-219`)."""
        if self.constraint is not None:
            logits = self.constraint.mask_logits(logits)
        tok, _ = sample_tokens(logits, input_ids, seed=self.seed, offset=self.offset, **self._kernel_args())
        self.offset += 1
        next_token = tok.view(-1, 1)
        if self.constraint is not None:
            next_token = self.constraint.apply_forcing(next_token)
            self.constraint.advance(next_token)
        return next_token


def make_sampler(sampler: Optional[Sampler] = None, **kwargs) -> Optional[Sampler]:
    """`make_sampler` (`sampler.py:222-232`): a ready instance, one built from keyword
    arguments, or None (greedy); both at once is a `ValueError`."""
    if sampler is not None and kwargs:
        raise ValueError('sampler and Sampler(...) constructor arguments are mutually exclusive')
    return Sampler(**kwargs) if kwargs else sampler
