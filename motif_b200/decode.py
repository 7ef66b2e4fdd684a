"""Batched decode as a replayed CUDA graph (greedy, or sampled on the device).

`Generation.step` (`motif/model/generate.py:138-171`) runs one `MotifChordModel.forward`
per new token: at L = 1 every layer is a handful of small launches, so a Python-driven loop
is launch-bound.  `GraphDecoder` captures ONE decode step — embed, for each decoder the
attn-res read, packed projection GEMM, GDN recurrent update (`motif_b200_gdn_decode`) or
Chord cache append + split-KV attention (`motif_b200_chord_prep` / `_chord_decode`), MLP,
residual GEMMs, then lm_head and the greedy argmax (or the sampling kernel) — and replays it
once per token.

Positions live on the device: `lens = [pos, pos + 1]` (int32) is read by the Chord kernels
(cache write position, attended length) and advanced by the graph itself, and the argmax
writes the next input ids in place, so `run(n)` replays n steps back to back with no host
synchronisation.  The KV buffers are grown to hold every step before capture (a graph
cannot regrow them); the GDN recurrent and conv states are updated in place.

The math is the eager T = 1 path's: the same kernels in the same order, except that the
split-KV count is fixed at capture (from the cache capacity) instead of chosen per length;
with `model.decode_splits` set, graph and eager decode give identical tokens.

With a `motif_b200.sampler.Sampler` (no grammar constraint: its hooks run on the host), the
argmax is replaced by `motif_b200_sample`: the Philox offset is the sampler's offset plus the
device step counter, and the repetition-penalty history is a device buffer [B, start + 1 +
max_steps] holding the sequence so far (-1 past its end; the kernel ignores negative ids),
into which each step writes the token it feeds.  The sampled stream is the one the eager
`Generation` loop draws with the same sampler.
"""

from typing import List, Optional, Tuple

import torch

from . import _lib
from .cache import GatedDeltaAttentionLayerCache, KVLayerCache, ModelCache
from .config import GGD_EPS, NORM_EPS
from .model import _chord_tail, _decode_splits, _down_add_gated, _mm, _norm_read

__all__ = ['GraphDecoder', 'fill_cache_random']


class _GDNSlot:
    """A GDN layer's in-place recurrent state (fp32 [B,H,dk,dv]) and conv state ([B,3,C])."""

    def __init__(self, cache: GatedDeltaAttentionLayerCache):
        self.cache = cache
        self.state = cache.state
        self.conv = cache._conv


def _check_layer_caches(model, cache: ModelCache, B: int, need: int):
    kv, gdn = [], []
    dt = model.embed.weight.dtype
    for b, block in enumerate(model.blocks):
        bc = cache[b]
        if len(bc.attn) != len(block.features):
            raise ValueError('the cache must hold one layer cache per decoder (run a prefill first)')
        for i, dec in enumerate(block.features):
            lc = bc.attn[i]
            if dec.attn_type == 'chord':
                if not isinstance(lc, KVLayerCache) or lc._kbuf is None:
                    raise ValueError(f'block {b} decoder {i}: an allocated KVLayerCache is required')
                if lc.wide:
                    raise NotImplementedError('wide KV caches are not used by the decode graph')
                if lc._kbuf.shape[0] != B or lc._kbuf.dtype != dt:
                    raise ValueError(f'block {b} decoder {i}: KV cache batch/dtype mismatch')
                lc.reserve(need)   # room for every step before capture: a graph cannot regrow it
                kv.append(lc)
            else:
                if not isinstance(lc, GatedDeltaAttentionLayerCache) or lc.state is None or lc._conv is None:
                    raise ValueError(f'block {b} decoder {i}: a filled GatedDeltaAttentionLayerCache is required')
                if lc.state.dtype != torch.float32 or not lc.state.is_contiguous():
                    lc.state = lc.state.float().contiguous()
                if lc._conv.dtype != dt or not lc._conv.is_contiguous():
                    lc._conv = lc._conv.to(dt).contiguous()
                gdn.append(_GDNSlot(lc))
    lengths = {lc.length for lc in kv}
    if len(lengths) > 1:
        raise ValueError(f'Chord layer caches disagree on length: {sorted(lengths)}')
    return kv, gdn


class GraphDecoder:
    """Greedy batched decode of `model` from `cache`, one CUDA-graph replay per token.

    >>> dec = GraphDecoder(model, cache, max_steps=256)   # cache: prefilled, batch B
    >>> toks = dec.run(first_ids, 256)                     # [B, 256] int64 on the device

    `first_ids` [B, 1] (or [B]) is the token fed at the first step (the prefill's greedy
    next token); the result holds the token produced by each step.  After `run` the cache's
    host-side lengths are advanced by the steps taken, so the eager API can continue from it.
    """

    def __init__(self, model, cache: ModelCache, max_steps: int, splits: Optional[int] = None, sampler=None,
                 eos_ids: Optional[List[int]] = None, fill_id: Optional[int] = None,
                 finished: Optional[torch.Tensor] = None):
        if model.training:
            raise ValueError('GraphDecoder needs an eval-mode model')
        w = model.embed.weight
        if w.device.type != 'cuda':
            raise ValueError('GraphDecoder runs on a CUDA device')
        self.model = model
        self.cache = cache
        self.dev = w.device
        self.dt = w.dtype
        kv0 = None
        for bc in cache:
            for lc in bc.attn:
                if isinstance(lc, KVLayerCache) and lc._kbuf is not None:
                    kv0 = lc
                    break
            if kv0 is not None:
                break
        if kv0 is None:
            raise ValueError('no allocated KV cache: prefill the cache before building the graph')
        self.B = kv0._kbuf.shape[0]
        self.start = kv0.length
        self.seq_start = cache.seq_len  # the block histories' token count (`ModelCache.seq_len`)
        self.max_steps = int(max_steps)
        self.kv, self.gdn = _check_layer_caches(model, cache, self.B, self.start + self.max_steps)
        self.cap = min(lc.capacity for lc in self.kv)
        cfg = model.config
        Hkv = cfg.kv_heads
        if self.kv and cfg.head_dim not in (32, 64):
            raise NotImplementedError(f'the decode graph uses the split-KV kernel (head dim 32 or 64), '
                                      f'got head dim {cfg.head_dim}')
        self.splits = int(splits) if splits else _decode_splits(model, self.B, Hkv, self.cap)
        self.decs, self.lm = model.packed()
        self.lens = torch.tensor([self.start, self.start + 1], dtype=torch.int32, device=self.dev)
        self.step_idx = torch.zeros((1,), dtype=torch.int64, device=self.dev)
        self.ids = torch.zeros((self.B,), dtype=torch.int64, device=self.dev)
        self.tokens = torch.zeros((self.max_steps, self.B), dtype=torch.int64, device=self.dev)
        self.sampler = None
        self.hist = None
        if sampler is not None:
            from .sampler import Sampler
            if not isinstance(sampler, Sampler):
                raise TypeError('GraphDecoder samples with a motif_b200.sampler.Sampler')
            if sampler.constraint is not None:
                raise NotImplementedError('a grammar constraint runs host hooks every step: use the eager loop')
            self.sampler = sampler
            self.sample_base = sampler.offset
            if sampler.repetition_penalty != 1.0:
                self.hist = torch.full((self.B, self.start + 1 + self.max_steps), -1, dtype=torch.int64,
                                       device=self.dev)
                self.hist_col = torch.tensor([self.start], dtype=torch.int64, device=self.dev)
        # end-of-sequence bookkeeping of `Generation.step` on the device: rows that already
        # produced an eos id receive `fill_id`; `all_done[i]` records whether every row has
        # finished after step i (read by the host once per chunk of steps)
        self.eos = None
        if eos_ids:
            self.eos = torch.tensor([int(e) for e in eos_ids], dtype=torch.int64, device=self.dev)
            self.fill = torch.tensor(int(fill_id if fill_id is not None else min(eos_ids)), dtype=torch.int64,
                                     device=self.dev)
            self.finished = torch.zeros((self.B,), dtype=torch.bool, device=self.dev)
            if finished is not None:
                self.finished.copy_(finished.reshape(-1).to(self.dev, torch.bool))
            self.all_done = torch.zeros((self.max_steps,), dtype=torch.bool, device=self.dev)
        self.launches_per_step = 0
        self.graph = None
        self._capture()

    # ------------------------------------------------------------------ one step
    def _step(self):
        """Every launch of one decode step; reads `ids`, `lens`, writes `ids`, `tokens[step]`."""
        model, cfg = self.model, self.model.config
        B, d, dt, dev = self.B, cfg.model_dim, self.dt, self.dev
        dc = _lib.dtype_code(dt)
        st = _lib.stream_ptr(dev)
        w = model.embed.weight
        x = torch.empty((B, d), dtype=dt, device=dev)
        _lib.call('motif_b200_embed', _lib.ptr(self.ids), _lib.ptr(w), _lib.ptr(x), B, d, cfg.vocab_size, dc, st)
        hn = torch.empty((B, d), dtype=dt, device=dev)
        _norm_read([x], None, None, None, hn)
        kv_i = gdn_i = 0
        for b, block in enumerate(model.blocks):
            fs: List[torch.Tensor] = []
            for i, dec in enumerate(block.features):
                if i > 0:
                    hn = torch.empty((B, d), dtype=dt, device=dev)
                    _norm_read([x] + fs, block.pseudo_queries[i].detach(), block.attn_res_norms[i].weight.detach(),
                               None, hn, eps_src=block.attn_res_norms[i].eps)
                pk = self.decs[b][i]
                proj = _mm(hn, pk.w_in, wp=pk.w_in_sk)
                if dec.attn_type == 'chord':
                    f = self._chord(pk, proj, self.kv[kv_i], dc, st)
                    kv_i += 1
                else:
                    f = self._gdn(pk, proj, self.gdn[gdn_i], dc, st)
                    gdn_i += 1
                fs.append(f)
            x_next = torch.empty((B, d), dtype=dt, device=dev)
            hn = torch.empty((B, d), dtype=dt, device=dev)
            _norm_read(fs, None, None, x_next, hn, eps_out=(model.norm.eps if b == len(model.blocks) - 1 else
                                                             model.blocks[b + 1].features[0].attn_norm.eps))
            x = x_next
        logits = _mm(hn, self.lm, wp=model._lm_sk)
        self.logits = logits  # the step's [B, V] logits buffer: after a replay, the last step's
        sp = self.sampler
        if sp is None:
            _lib.call('motif_b200_argmax', _lib.ptr(logits), B, cfg.vocab_size, logits.stride(0),
                      _lib.ptr(self.ids), dc, st)
        else:
            hist_len = 0
            if self.hist is not None:
                self.hist.index_copy_(1, self.hist_col, self.ids.view(B, 1))
                self.hist_col.add_(1)
                hist_len = self.hist.shape[1]
            _lib.call('motif_b200_sample', _lib.ptr(logits), logits.stride(0), B, cfg.vocab_size,
                      _lib.ptr(self.hist), hist_len, hist_len, float(sp.repetition_penalty), float(sp.temperature),
                      int(sp.top_k) if sp.top_k is not None else 0,
                      float(sp.top_p) if sp.top_p is not None else 1.0, None, sp.seed & (2 ** 64 - 1),
                      self.sample_base & (2 ** 64 - 1), _lib.ptr(self.step_idx), _lib.ptr(self.ids), None, 0,
                      dc, st)
        if self.eos is not None:
            self.ids.copy_(torch.where(self.finished, self.fill, self.ids))
            self.finished.logical_or_(torch.isin(self.ids, self.eos))
            self.all_done.index_copy_(0, self.step_idx, self.finished.all().view(1))
        # token log, step counter and cache lengths in one launch
        _lib.call('motif_b200_decode_advance', _lib.ptr(self.ids), B, _lib.ptr(self.tokens), self.max_steps,
                  _lib.ptr(self.step_idx), _lib.ptr(self.lens), self.lens.numel(), st)

    def _gdn(self, pk, proj, slot: _GDNSlot, dc, st):
        B, dt, dev = self.B, self.dt, self.dev
        H, dk, dv, hid = pk.H, pk.dk, pk.dv, pk.hid
        N_in = proj.shape[1]
        cat = torch.empty((B, H * dv + hid), dtype=dt, device=dev)
        # the recurrent step and the MLP activation in one launch
        _lib.call('motif_b200_gdn_decode_swiglu', _lib.ptr(proj), N_in, _lib.ptr(pk.conv_w), _lib.ptr(pk.A_log),
                  _lib.ptr(pk.dt_bias), _lib.ptr(slot.conv), _lib.ptr(slot.state),
                  proj.data_ptr() + pk.off_g * proj.element_size(), _lib.ptr(pk.onorm_w), _lib.ptr(cat),
                  cat.stride(0), B, H, dk, dv, NORM_EPS, proj.data_ptr() + pk.off_gu * proj.element_size(), N_in,
                  cat.data_ptr() + H * dv * cat.element_size(), cat.stride(0), hid, dc, st)
        return _mm(cat, pk.w_out, wp=pk.w_out_sk)

    def _chord(self, pk, proj, lc: KVLayerCache, dc, st):
        B, dt, dev = self.B, self.dt, self.dev
        H, Hkv, D, hid = pk.H, pk.Hkv, pk.D, pk.hid
        d = H * D
        N_in = proj.shape[1]
        cap = lc._kbuf.shape[2]
        qb = torch.empty((B, d), dtype=dt, device=dev)
        act = torch.empty((B, hid), dtype=dt, device=dev)
        lens_ptr = self.lens.data_ptr()
        # q/k norms + cache append and the MLP activation in one launch
        _lib.call('motif_b200_chord_prep_swiglu', _lib.ptr(proj), N_in, _lib.ptr(pk.qn_w), _lib.ptr(pk.kn_w),
                  _lib.ptr(qb), _lib.ptr(lc._kbuf), _lib.ptr(lc._vbuf), cap, lens_ptr, 0, B, 1, H, Hkv, D, NORM_EPS,
                  proj.data_ptr() + pk.off_gu * proj.element_size(), N_in, _lib.ptr(act), hid, hid, dc, st)
        attn = torch.empty((B, d), dtype=dt, device=dev)
        ws_bytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, 1, D, self.splits)
        ws = torch.empty((max(ws_bytes, 4) // 4,), dtype=torch.float32, device=dev)
        _lib.call('motif_b200_chord_decode', _lib.ptr(qb), _lib.ptr(lc._kbuf), _lib.ptr(lc._vbuf), cap,
                  lens_ptr + 4, 0, _lib.ptr(pk.alpha), _lib.ptr(pk.beta), _lib.ptr(pk.mu), _lib.ptr(pk.ssmax),
                  _lib.ptr(attn), d, B, H, Hkv, 1, D, D ** -0.5, GGD_EPS, self.splits, _lib.ptr(ws), ws_bytes, dc, st)
        gate = proj[:, pk.off_g:pk.off_g + d]
        f = _chord_tail(attn, pk.w_o, act, pk.w_down, gate)
        if f is not None:  # o_proj, down_proj and the gated residual in one launch
            return f
        a = _mm(attn, pk.w_o, wp=pk.w_o_sk)
        f = _down_add_gated(act, pk.w_down, a, gate)
        if f is not None:  # the gated residual in the down projection's epilogue
            return f
        f = _mm(act, pk.w_down, wp=pk.w_down_sk)
        _lib.call('motif_b200_gate_residual', _lib.ptr(a), d, proj.data_ptr() + pk.off_g * proj.element_size(),
                  N_in, _lib.ptr(f), d, _lib.ptr(f), d, B, d, dc, st)
        return f

    # ------------------------------------------------------------------ capture / replay
    def _snapshot(self):
        hist = None if self.hist is None else (self.hist.clone(), self.hist_col.clone())
        fin = None if self.eos is None else self.finished.clone()
        return [s.state.clone() for s in self.gdn], [s.conv.clone() for s in self.gdn], hist, fin

    def _restore(self, snap):
        for s, st_, cv in zip(self.gdn, snap[0], snap[1]):
            s.state.copy_(st_)
            s.conv.copy_(cv)
        if snap[2] is not None:
            self.hist.copy_(snap[2][0])
            self.hist_col.copy_(snap[2][1])
        if snap[3] is not None:
            self.finished.copy_(snap[3])

    def set_history(self, history: torch.Tensor):
        """Seed the repetition-penalty history with the sequence so far ([B, start + 1], ending
        with the first token fed); a no-op for samplers without the penalty."""
        if self.hist is None:
            return
        if self.taken:
            raise ValueError('history seeds the first run only')
        if tuple(history.shape) != (self.B, self.start + 1):
            raise ValueError(f'history must be [{self.B}, {self.start + 1}], got {tuple(history.shape)}')
        self.hist[:, :self.start + 1].copy_(history.to(self.dev, torch.int64))

    def save(self):
        """Everything a later `run` reads or writes, so that `load(save())` rewinds the decoder
        (and the cache's recurrent states and lengths) to this point.  KV entries written after
        the save lie past the restored lengths and are overwritten by the next steps."""
        return (self._snapshot(), self.lens.clone(), self.step_idx.clone(), self.ids.clone(), self.taken)

    def load(self, saved):
        snap, lens, step_idx, ids, taken = saved
        self._restore(snap)
        self.lens.copy_(lens)
        self.step_idx.copy_(step_idx)
        self.ids.copy_(ids)
        self.taken = taken
        if self.sampler is not None:
            self.sampler.offset = self.sample_base + taken
        self._sync_lengths()

    def _capture(self):
        # The warm-up step (required before capture: cuBLAS handles, lazy library load) and the
        # captured step both execute, so the recurrent states are saved and put back, and the
        # cache positions they wrote are rewritten by the first real step.
        snap = self._snapshot()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        tr = _lib.Tracker(timed=None, events=False)
        with torch.cuda.stream(side):
            _lib.set_tracker(tr)
            try:
                self._step()
            finally:
                _lib.set_tracker(None)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        self.launches_per_step = tr.launches
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        torch.cuda.synchronize(self.dev)
        self._restore(snap)
        self.lens.copy_(torch.tensor([self.start, self.start + 1], dtype=torch.int32))
        self.step_idx.zero_()
        self.taken = 0

    def run(self, first_ids: torch.Tensor, steps: int, history: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Replay `steps` decode steps from the current position; returns [B, steps] tokens.

        With a sampler that applies a repetition penalty, `history` ([B, start + 1], the
        sequence so far ending with `first_ids`, as `Generation.sequences`) seeds the penalty
        on the first run; without it the penalty sees only the tokens fed by the graph."""
        steps = int(steps)
        if steps < 0 or self.taken + steps > self.max_steps:
            raise ValueError(f'{steps} steps after {self.taken} exceed max_steps={self.max_steps}')
        ids = first_ids.reshape(-1)
        if ids.numel() != self.B:
            raise ValueError(f'first_ids holds {ids.numel()} ids for a batch of {self.B}')
        if history is not None:
            self.set_history(history)
        self.ids.copy_(ids.to(self.dev, torch.int64), non_blocking=True)
        lo = self.taken
        for _ in range(steps):
            self.graph.replay()
        self.taken += steps
        if self.sampler is not None:
            self.sampler.offset = self.sample_base + self.taken
        self._sync_lengths()
        return self.tokens[lo:self.taken].t()

    def _sync_lengths(self):
        """Host-side lengths after `taken` graph steps: KV / GDN layer caches and the block
        histories' `seq_len` (each step feeds one token)."""
        for lc in self.kv:
            lc.length = self.start + self.taken
        for s in self.gdn:
            s.cache.length = self.start + self.taken
        for bc in self.cache:
            bc.attn_res.seq_len = self.seq_start + self.taken

    def breakdown(self, first_ids: torch.Tensor, steps: int = 32):
        """Run `steps` decode steps eagerly (outside the graph) with CUDA events around every
        launch and return `{entry point or 'cublas_gemm': (calls per step, ms per step)}`,
        averaged over the steps after one untimed warm step.  The states, positions and step
        counter are put back afterwards, so the decoder is unchanged.  Eager launches leave
        gaps the graph does not have, so these times explain the graph step's SHARES; their
        sum exceeds the graph step."""
        snap = self._snapshot()
        lens = self.lens.clone()
        step_idx = self.step_idx.clone()
        self.ids.copy_(first_ids.reshape(-1).to(self.dev, torch.int64))
        self._step()  # warm: the first eager step after capture touches every buffer once
        torch.cuda.synchronize(self.dev)
        tr = _lib.Tracker(timed=None)
        _lib.set_tracker(tr)
        try:
            for _ in range(max(1, int(steps))):
                self._step()
        finally:
            _lib.set_tracker(None)
        torch.cuda.synchronize(self.dev)
        self._restore(snap)
        self.lens.copy_(lens)
        self.step_idx.copy_(step_idx)
        n = max(1, int(steps))
        return {k: (c / n, t / n) for k, (c, t) in tr.summary().items()}

    def release(self):
        """Free the graph (and its memory pool)."""
        self.graph = None


def fill_cache_random(model, cache: ModelCache, batch: int, length: int, capacity: int, seed: int = 0):
    """Fill every layer cache of `cache` as if `length` tokens had been prefilled, with seeded
    random contents: Chord K (unit-RMS rows, as after k_norm) / V, GDN recurrent states and
    conv windows.  Decode speed does not depend on the values; this stands in for a prefill
    of `batch` x `length` tokens (the benchmark's decode context) without its time or memory."""
    cfg = model.config
    w = model.embed.weight
    dev, dt = w.device, w.dtype
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    for b, block in enumerate(model.blocks):
        bc = cache[b]
        bc.ensure_attn([dec.cache_type for dec in block.features])
        for i, dec in enumerate(block.features):
            lc = bc.attn[i]
            if dec.attn_type == 'chord':
                Hkv, D = cfg.kv_heads, cfg.head_dim
                lc._kbuf = torch.empty((batch, Hkv, capacity, D), dtype=dt, device=dev)
                lc._vbuf = torch.empty_like(lc._kbuf)
                lc._kbuf.normal_(0.0, 1.0, generator=g)
                lc._vbuf.normal_(0.0, 0.5, generator=g)
                lc.length = length
            else:
                H, dk, dv = cfg.num_heads, cfg.gdn_dk, cfg.gdn_dv
                C = H * (2 * dk + dv)
                lc.state = torch.empty((batch, H, dk, dv), dtype=torch.float32, device=dev).normal_(0.0, 0.05,
                                                                                                   generator=g)
                lc._conv = torch.empty((batch, 3, C), dtype=dt, device=dev).normal_(0.0, 0.5, generator=g)
                lc._split = (H * dk, H * dk, H * dv)
                lc.length = length
    return cache
