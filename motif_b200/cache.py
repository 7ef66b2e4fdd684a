"""Cache classes with the reference's API (`motif/model/cache.py`), laid out for the kernels.

* `KVLayerCache` keeps one preallocated `[B, H_kv, capacity, D]` buffer per k / v and grows
  it geometrically like the reference (`cache.py:146-168`); `.k` / `.v` are views of the
  valid prefix, so readers see exactly the reference's tensors.  The fused Chord layer
  writes new keys / values straight into the buffer (no concatenation, no copy).
* `GatedDeltaAttentionLayerCache` keeps the recurrent state `[B, H, Dk, Dv]` in fp32 and
  the three conv states in one time-major `[B, 3, C]` buffer (C = q | k | v channels), the
  layout the decode kernel reads; `conv_state` exposes the reference's `[B, D, 3]` views.
* `AttnResCache`, `DecoderBlockCache`, `ModelCache`, `build_cache` follow
  `cache.py:397-847` line for line.
"""

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import torch


class BasicLayerCache:
    """Interface of every per-layer cache (`motif/model/cache.py:7-39`)."""

    @property
    def seq_length(self) -> int:
        raise NotImplementedError

    def reset(self) -> None:
        raise NotImplementedError

    def to(self, device=None, dtype=None):
        raise NotImplementedError


def _widen_heads(x: torch.Tensor, num_heads: int) -> torch.Tensor:
    """Repeat grouped kv heads to every query head (`cache.py:42-70`)."""
    b, kv, n, d = x.shape
    if kv == num_heads:
        return x
    if num_heads % kv:
        raise ValueError(f'cannot store {num_heads} heads from {kv} grouped heads: the '
                         f'query-head count must be a multiple of the key / value head count')
    return x[:, :, None].expand(b, kv, num_heads // kv, n, d).reshape(b, num_heads, n, d)


class KVLayerCache(BasicLayerCache):
    """Key / value cache of a chord layer (`motif/model/cache.py:73-252`)."""

    def __init__(self, num_heads: Optional[int] = None):
        self._kbuf: Optional[torch.Tensor] = None
        self._vbuf: Optional[torch.Tensor] = None
        self.length: int = 0
        self.num_heads: Optional[int] = None if num_heads is None else int(num_heads)

    @property
    def wide(self) -> bool:
        return self.num_heads is not None

    @property
    def k(self) -> Optional[torch.Tensor]:
        return None if self._kbuf is None else self._kbuf[:, :, :self.length]

    @property
    def v(self) -> Optional[torch.Tensor]:
        return None if self._vbuf is None else self._vbuf[:, :, :self.length]

    @property
    def capacity(self) -> int:
        return 0 if self._kbuf is None else self._kbuf.shape[2]

    @property
    def seq_length(self) -> int:
        return self.length

    def reserve(self, need: int, like: torch.Tensor = None, shape=None):
        """Make room for `need` positions (geometric growth, `cache.py:146-168`)."""
        if self._kbuf is not None and need <= self._kbuf.shape[2]:
            return
        if self._kbuf is None:
            b, h, d = shape
            cap = max(need, 1024)
            self._kbuf = torch.empty((b, h, cap, d), dtype=like.dtype, device=like.device)
            self._vbuf = torch.empty_like(self._kbuf)
            return
        old = self._kbuf.shape[2]
        cap = max(need, old + max(old // 4, 1024))
        kb = self._kbuf.new_empty(self._kbuf.shape[:2] + (cap,) + self._kbuf.shape[3:])
        vb = self._vbuf.new_empty(kb.shape)
        kb[:, :, :self.length].copy_(self._kbuf[:, :, :self.length])
        vb[:, :, :self.length].copy_(self._vbuf[:, :, :self.length])
        self._kbuf, self._vbuf = kb, vb

    def update(self, k_new: torch.Tensor, v_new: torch.Tensor, dim: int = 2) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append and return the whole cached sequence (`cache.py:170-215`)."""
        if dim not in (2, -2):
            raise ValueError('KVLayerCache stores the sequence on dim 2')
        if self.num_heads is not None:
            k_new, v_new = _widen_heads(k_new, self.num_heads), _widen_heads(v_new, self.num_heads)
        n = k_new.shape[2]
        if self._kbuf is not None and self._kbuf.device != k_new.device:
            self.to(k_new.device)
        self.reserve(self.length + n, like=k_new, shape=(k_new.shape[0], k_new.shape[1], k_new.shape[3]))
        self._kbuf[:, :, self.length:self.length + n].copy_(k_new.detach())
        self._vbuf[:, :, self.length:self.length + n].copy_(v_new.detach())
        self.length += n
        return self.k, self.v

    def reset(self):
        self._kbuf = None
        self._vbuf = None
        self.length = 0

    def to(self, device=None, dtype=None):
        if self._kbuf is not None:
            self._kbuf = self._kbuf.to(device=device, dtype=dtype)
            self._vbuf = self._vbuf.to(device=device, dtype=dtype)
        return self

    def __repr__(self):
        heads = '' if self.num_heads is None else f', heads={self.num_heads}'
        return f'KVLayerCache(seq_length={self.length}, capacity={self.capacity}{heads})'


class FunctionalKVLayerCache(KVLayerCache):
    """Out-of-place variant (`cache.py:255-302`): `update` concatenates, never pads."""

    def update(self, k_new, v_new, dim: int = 2):
        if self.num_heads is not None:
            k_new, v_new = _widen_heads(k_new, self.num_heads), _widen_heads(v_new, self.num_heads)
        if self._kbuf is None:
            self._kbuf, self._vbuf = k_new.detach(), v_new.detach()
        else:
            self._kbuf = torch.cat([self.k, k_new.detach()], dim=2)
            self._vbuf = torch.cat([self.v, v_new.detach()], dim=2)
        self.length = self._kbuf.shape[2]
        return self.k, self.v


class GatedDeltaAttentionLayerCache(BasicLayerCache):
    """Recurrent + conv state of a GDN layer (`motif/model/cache.py:305-394`)."""

    def __init__(self):
        self.state: Optional[torch.Tensor] = None
        self._conv: Optional[torch.Tensor] = None  # [B, 3, Cq + Ck + Cv], time-major
        self._split: Tuple[int, int, int] = (0, 0, 0)
        self.length: int = 0

    @property
    def seq_length(self) -> int:
        return self.length

    @property
    def conv_state(self) -> Optional[Tuple[torch.Tensor, ...]]:
        if self._conv is None:
            return None
        a, b, c = self._split
        t = self._conv.transpose(1, 2)  # [B, C, 3] view
        return t[:, :a], t[:, a:a + b], t[:, a + b:a + b + c]

    @conv_state.setter
    def conv_state(self, value):
        if value is None:
            self._conv = None
            return
        cq, ck, cv = value
        self._split = (cq.shape[1], ck.shape[1], cv.shape[1])
        self._conv = torch.cat([cq, ck, cv], dim=1).transpose(1, 2).contiguous()

    def update(self, state: torch.Tensor, conv_state, steps: int = 1) -> torch.Tensor:
        """Replace the state with the one produced by the last step (`cache.py:332-356`)."""
        self.state = state.detach()
        if isinstance(conv_state, torch.Tensor):  # the fused path hands over its [B, 3, C] buffer
            self._conv = conv_state.detach()
        else:
            self.conv_state = tuple(c.detach() for c in conv_state)
        self.length += steps
        return self.state

    def reset(self):
        self.state = None
        self._conv = None
        self.length = 0

    def to(self, device=None, dtype=None):
        if self.state is not None:
            self.state = self.state.to(device=device, dtype=dtype)
        if self._conv is not None:
            self._conv = self._conv.to(device=device, dtype=dtype)
        return self

    def __repr__(self):
        return f'GatedDeltaAttentionLayerCache(seq_length={self.length}, has_state={self.state is not None})'


@dataclass
class AttnResCache:
    """Attn-res history of one block (`motif/model/cache.py:397-606`)."""

    blocks: List[torch.Tensor] = field(default_factory=list)
    partial_block: Optional[torch.Tensor] = None
    seq_len: int = 0
    chunk_len: int = 0

    def _cat_or_add(self, cached, new):
        if cached.shape[1] == new.shape[1]:
            return cached + new
        return torch.cat([cached, new], dim=1)

    def _align(self, entries):
        q_len = self.chunk_len
        if q_len <= 0:
            q_len = min(e.shape[1] for e in entries)
        if any(e.shape[1] != q_len for e in entries):
            entries = [e if e.shape[1] == q_len else e[:, max(e.shape[1] - q_len, 0):, :] for e in entries]
        return entries

    def aligned_values(self) -> List[torch.Tensor]:
        if len(self.blocks) == 0:
            raise RuntimeError('AttnResCache is empty, there is no value to read')
        return self._align(list(self.blocks))

    def _stack_values(self):
        return torch.stack(self.aligned_values(), dim=0)

    def init_embedding(self, hidden_states: torch.Tensor):
        q_len = hidden_states.shape[1]
        if len(self.blocks) == 0:
            self.seq_len = q_len
        else:
            self.seq_len = self.seq_len + q_len
            self.partial_block = None
        self.blocks = [hidden_states]
        self.chunk_len = q_len

    def update_increment(self, f_h: torch.Tensor):
        self.blocks.append(f_h)
        if self.partial_block is None:
            self.partial_block = f_h
        else:
            self.partial_block = self._cat_or_add(self.partial_block, f_h)
        self.seq_len = max(self.seq_len, f_h.shape[1])

    def reset(self):
        self.blocks.clear()
        self.partial_block = None
        self.seq_len = 0
        self.chunk_len = 0

    def to(self, device=None, dtype=None):
        self.blocks = [b.to(device=device, dtype=dtype) for b in self.blocks]
        if self.partial_block is not None:
            self.partial_block = self.partial_block.to(device=device, dtype=dtype)
        return self

    def values(self):
        return self._stack_values()

    def num_sources(self) -> int:
        return len(self.blocks)

    @property
    def is_empty(self) -> bool:
        return len(self.blocks) == 0

    @property
    def current_seq_len(self) -> int:
        if self.partial_block is not None:
            return self.partial_block.shape[1]
        if len(self.blocks) > 0:
            return self.blocks[-1].shape[1]
        return 0


@dataclass
class DecoderBlockCache:
    """Cache of one `DecoderBlock` (`motif/model/cache.py:609-700`)."""

    attn_res: AttnResCache = field(default_factory=AttnResCache)
    attn: List[Optional[BasicLayerCache]] = field(default_factory=list)

    def ensure_attn(self, cache_types: Sequence[type]) -> None:
        if len(self.attn) == 0:
            self.attn = [t() for t in cache_types]

    def reset(self):
        self.attn_res.reset()
        self.attn.clear()

    def is_empty(self) -> bool:
        return self.attn_res.is_empty and len(self.attn) == 0

    def to(self, device=None, dtype=None):
        self.attn_res.to(device, dtype)
        for c in self.attn:
            if c is not None:
                c.to(device, dtype)
        return self

    @property
    def blocks(self):
        return self.attn_res.blocks

    @property
    def seq_len(self) -> int:
        return self.attn_res.seq_len


@dataclass
class ModelCache:
    """Cache of the whole model, grouped by block (`motif/model/cache.py:703-799`)."""

    blocks: List[DecoderBlockCache] = field(default_factory=list)

    @classmethod
    def create(cls, num_blocks: int) -> 'ModelCache':
        return cls(blocks=[DecoderBlockCache() for _ in range(num_blocks)])

    def reset(self):
        for b in self.blocks:
            b.reset()

    @property
    def seq_len(self) -> int:
        return self.blocks[0].seq_len if self.blocks else 0

    def to(self, device=None, dtype=None):
        for b in self.blocks:
            b.to(device, dtype)
        return self

    def __len__(self):
        return len(self.blocks)

    def __getitem__(self, idx):
        return self.blocks[idx]

    def __iter__(self):
        return iter(self.blocks)


def build_cache(model, use_attn: Optional[bool] = None, functional: bool = False,
                wide_kv: bool = False) -> ModelCache:
    """`build_cache` (`motif/model/cache.py:802-847`)."""
    if use_attn is None:
        use_attn = not getattr(model, 'training', False)
    if not use_attn:
        return ModelCache.create(len(model.blocks))
    blocks = []
    for block in model.blocks:
        attn = []
        for decoder in block.features:
            t = decoder.cache_type
            if functional and issubclass(t, KVLayerCache):
                t = FunctionalKVLayerCache
            if wide_kv and issubclass(t, KVLayerCache):
                attn.append(t(num_heads=decoder.attn.num_heads))
            else:
                attn.append(t())
        blocks.append(DecoderBlockCache(attn=attn))
    return ModelCache(blocks=blocks)
