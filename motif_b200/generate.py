"""`Generation` with the reference's iteration semantics (`motif/model/generate.py:16-200`).

Each step: forward with the cache -> `next_token` (greedy argmax kernel, or a bound
sampler callable) -> append.  The first forward feeds the whole prompt (prefill); later
steps feed the previous token.  Rows that produced an eos keep receiving the eos
placeholder; iteration stops when every row finished or `max_new_tokens` is reached.

`graph=True` runs the decode steps of `run()` as replays of one captured CUDA graph
(`motif_b200.decode.GraphDecoder`): the eos placeholder and the finished flags are kept on
the device, and the host reads the all-finished flags once per `sync_every` steps instead
of once per step (`generate.py:127`).  When every row finished inside a chunk, the
recurrent states saved at the chunk's start are restored and exactly the steps up to the
stop are replayed, so the tokens, the finished flags and the cache are those of the
step-by-step loop.  Graph mode needs a Chord layer (the graph reads its positions from the
KV cache), no attention mask, and either greedy decoding or a `motif_b200.sampler.Sampler`
without a grammar constraint; otherwise `run()` steps eagerly.
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
                 cache=None, mask=None, tokenizer=None, graph: bool = False, sync_every: int = 16):
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
        self.graph = bool(graph)
        self.sync_every = max(1, int(sync_every))
        self.graph_steps = 0  # steps taken by graph replays (the rest ran eagerly)

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
        if self.graph and not self.done:
            if self.steps == 0:
                self.step()  # the prefill (and the first token) run eagerly
            if not self.done and self._graph_ok():
                self._run_graph()
        for _ in self:
            pass
        return self

    def _graph_ok(self) -> bool:
        from .model import MotifChordModel
        from .sampler import Sampler
        if not isinstance(self.model, MotifChordModel) or self._key_mask is not None or self.cache is None:
            return False
        s = self.sampler if self.sampler is not None else self.model.sampler
        if s is not None and (not isinstance(s, Sampler) or s.constraint is not None):
            return False
        cfg = self.model.config
        has_chord = any(d.attn_type == 'chord' for blk in self.model.blocks for d in blk.features)
        return has_chord and cfg.head_dim in (32, 64)

    def _run_graph(self):
        from .decode import GraphDecoder
        s = self.sampler if self.sampler is not None else self.model.sampler
        remaining = self.max_new_tokens - self.steps
        dec = GraphDecoder(self.model, self.cache, max_steps=remaining, sampler=s, eos_ids=self.eos_ids or None,
                           fill_id=self.fill_id, finished=self.finished)
        first = self._next_input
        try:
            dec.set_history(self.sequences)
            while remaining > 0:
                k = min(self.sync_every, remaining)
                saved = dec.save() if dec.eos is not None else None
                toks = dec.run(first, k)
                stop = k
                if dec.eos is not None:
                    flags = dec.all_done[dec.taken - k:dec.taken].cpu()  # the one host sync per chunk
                    hit = torch.nonzero(flags).flatten()
                    if hit.numel():
                        stop = int(hit[0]) + 1
                        if stop < k:  # rewind to the chunk's start and take exactly `stop` steps
                            dec.load(saved)
                            toks = dec.run(first, stop)
                toks = toks.to(self.sequences.device)
                self.sequences = torch.cat([self.sequences, toks], dim=1)
                self.steps += stop
                self.graph_steps += stop
                remaining -= stop
                first = toks[:, -1:]
                if dec.eos is not None and bool(dec.finished.all()):
                    break
            self._next_input = first
            if dec.eos is not None:
                self.finished = dec.finished.to(self.finished.device).clone()
        finally:
            dec.release()
