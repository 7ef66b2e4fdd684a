"""`Generation` with the reference's iteration semantics (`motif/model/generate.py:16-200`).

Each step: forward with the cache -> `next_token` (greedy argmax kernel, or a bound
sampler callable) -> append.  The first forward feeds the whole prompt (prefill); later
steps feed the previous token.  Rows that produced an eos keep receiving the eos
placeholder; iteration stops when every row finished or `max_new_tokens` is reached.
"""

from typing import Sequence, Union

import torch

EosTokenId = Union[int, str, Sequence[Union[int, str]], None]


def _resolve_eos(eos_token_id, tokenizer):
    if eos_token_id is None:
        return []
    items = eos_token_id if isinstance(eos_token_id, (list, tuple, set)) else [eos_token_id]
    out = []
    for it in items:
        if isinstance(it, str):
            if tokenizer is None or not hasattr(tokenizer, 'token_to_id'):
                raise ValueError(f'eos token name {it!r} needs a tokenizer that can resolve it')
            out.append(int(tokenizer.token_to_id(it)))
        else:
            out.append(int(it))
    return out


class Generation:
    def __init__(self, model, input_ids, max_new_tokens=32, eos_token_id: EosTokenId = None, sampler=None,
                 cache=None, mask=None, tokenizer=None):
        if input_ids.dim() != 2:
            raise ValueError(f'input_ids must be [B, T], got {tuple(input_ids.shape)}')
        if int(max_new_tokens) < 0:
            raise ValueError(f'max_new_tokens must not be negative, got {max_new_tokens}')
        cached = cache.seq_len if cache is not None else 0
        if cached >= input_ids.shape[1]:
            raise ValueError(f'the cache already holds {cached} positions but the input has only '
                             f'{input_ids.shape[1]} tokens, so there is nothing new to feed')
        self.model = model
        self.cache = cache
        self.sampler = sampler
        self.max_new_tokens = int(max_new_tokens)
        self.sequences = input_ids
        self.prompt_len = input_ids.shape[1]
        self._next_input = input_ids[:, cached:]
        self._key_mask = None if mask is None else mask[:, :cached + input_ids.shape[1]]
        self.eos_ids = _resolve_eos(eos_token_id, tokenizer)
        self.fill_id = min(self.eos_ids) if self.eos_ids else None
        self.finished = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=input_ids.device)
        self.steps = 0

    @property
    def done(self) -> bool:
        return self.steps >= self.max_new_tokens or bool(self.finished.all())

    @property
    def generated(self) -> torch.Tensor:
        return self.sequences[:, self.prompt_len:]

    def step(self) -> torch.Tensor:
        with torch.no_grad():
            out = self.model(self._next_input, cache=self.cache, mask=self._key_mask)
            token = out.next_token(sampler=self.sampler, input_ids=self.sequences)
        self.cache = out.cache
        token = token.to(self.sequences.device)
        if self.fill_id is not None:
            token = token.masked_fill(self.finished.unsqueeze(1), self.fill_id)
        self.sequences = torch.cat([self.sequences, token], dim=1)
        if self._key_mask is not None:
            self._key_mask = torch.cat([self._key_mask, torch.ones_like(token, dtype=torch.bool)], dim=1)
        self._next_input = token
        self.steps += 1
        if self.eos_ids:
            hit = torch.zeros_like(self.finished)
            for e in self.eos_ids:
                hit |= token.squeeze(1) == e
            self.finished |= hit
        return token

    def __iter__(self):
        return self

    def __next__(self):
        if self.done:
            raise StopIteration
        return self.step()

    def run(self):
        for _ in self:
            pass
        return self
