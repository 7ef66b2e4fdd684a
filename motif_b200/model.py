"""`MotifChordModel` with the reference's module tree, parameter names, forward, cache and
generation API (`motif/model/motif.py`, `motif/block/decoder.py`, `motif/block/mlp.py`,
`motif/block/attention/{gdn_attn,chord_attn}.py`), computed by the sm_100a kernels.

The parameters are stored exactly as the reference stores them, so `state_dict()` /
`load_state_dict()` interoperate with the reference in both directions.  The forward does
not walk the modules one by one; per decoder a prefill runs

    attn-res read + RMSNorm                motif_b200_attn_res_norm (one pass over the sources)
    every input projection as ONE GEMM, norm weights folded into the packed weight, the MLP's
    SwiGLU in its epilogue                 motif_b200_gemm_proj_swiglu (tcgen05)
    GDN:   conv + SiLU + L2 norms + beta / g, UT transform, state scan, GatedRMSNorm
                                           motif_b200_gdn_prefill_ws
           o_proj + down_proj as ONE GEMM over [o | act] (the parallel residual is a sum of
           two products, so it is one product over the concatenated K dimension)
                                           motif_b200_gemm
    Chord: q/k RMSNorm + cache append      motif_b200_chord_prep
           biased flash attention          motif_b200_chord_attention (tcgen05)
           down_proj, then o_proj with f = attn * sigmoid(g) + mlp in its epilogue
                                           motif_b200_gemm, motif_b200_gemm_gate_residual

and a decode step the same reads with the decode kernels (motif_b200_gdn_decode_swiglu,
motif_b200_chord_prep_swiglu, motif_b200_chord_decode, motif_b200_gate_residual) and the
decode-sized products of `_mm` (weight-streaming GEMMs, the library GEMM for the K = 768 input
projections at 33-64 rows); the block output / final norm use the same fused read (sum mode).
Packed weights are derived from the parameters on first use and rebuilt after
`load_state_dict`, `.to()` or an explicit `invalidate_packed()` (call it after editing
parameters in place).
"""

import builtins
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .cache import (AttnResCache, BasicLayerCache, DecoderBlockCache, GatedDeltaAttentionLayerCache,
                    KVLayerCache, ModelCache, build_cache)
from .config import CHUNK_SIZE, CONV_SIZE, EXPAND_V, GGD_EPS, NORM_EPS, MotifChordConfig
from .ops import GatedRMSNorm, RMSNorm, SwiGLU as SwiGLUOp
from .sampler import Sampler, make_sampler


# ============================================================================ modules
class BasicAttention(nn.Module):
    """Head layout shared by the attention layers (`block/attention/base.py:10-118`)."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: Optional[int] = None, **kwargs):
        super().__init__()
        num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        assert hidden_size % num_heads == 0, f'hidden_size {hidden_size} must be divisible by num_heads {num_heads}'
        assert num_heads % num_kv_heads == 0, f'num_heads {num_heads} must be divisible by num_kv_heads {num_kv_heads}'
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = hidden_size // num_heads
        self.kv_dim = num_kv_heads * self.head_dim
        self.num_kv_queries = num_heads // num_kv_heads


class GatedDeltaAttention(BasicAttention):
    """Gated delta-net attention parameters (`block/attention/gdn_attn.py:19-106`)."""

    def __init__(self, hidden_size, num_heads, head_k_dim=None, expand_v=EXPAND_V, conv_size=CONV_SIZE,
                 chunk_size=CHUNK_SIZE, bias=False, dropout=0.0, use_triton=True, **kwargs):
        super().__init__(hidden_size=hidden_size, num_heads=num_heads, num_kv_heads=num_heads)
        if bias:
            raise NotImplementedError('projection biases are not part of this inference path')
        self.dk = head_k_dim or self.head_dim
        self.dv = int(self.dk * expand_v)
        self.conv_size = conv_size
        self.chunk_size = chunk_size
        self.bias = bias
        self.dropout = dropout
        self.use_triton = True
        dk_all, dv_all = self.num_heads * self.dk, self.num_heads * self.dv
        self.q_proj = nn.Linear(hidden_size, dk_all, bias=False)
        self.k_proj = nn.Linear(hidden_size, dk_all, bias=False)
        self.v_proj = nn.Linear(hidden_size, dv_all, bias=False)
        self.a_proj = nn.Linear(hidden_size, self.num_heads, bias=False)
        self.b_proj = nn.Linear(hidden_size, self.num_heads, bias=False)
        self.g_proj = nn.Linear(hidden_size, dv_all, bias=False)
        self.o_proj = nn.Linear(dv_all, hidden_size, bias=False)
        self.q_conv = nn.Conv1d(dk_all, dk_all, conv_size, groups=dk_all, bias=False)
        self.k_conv = nn.Conv1d(dk_all, dk_all, conv_size, groups=dk_all, bias=False)
        self.v_conv = nn.Conv1d(dv_all, dv_all, conv_size, groups=dv_all, bias=False)
        A = torch.empty(self.num_heads).uniform_(1, 16)
        self.A_log = nn.Parameter(A.log())
        dt = torch.exp(torch.rand(self.num_heads) * (math.log(0.1) - math.log(0.001)) + math.log(0.001))
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.o_norm = GatedRMSNorm(self.dv)

    @classmethod
    def cache_type(cls):
        return GatedDeltaAttentionLayerCache


class ChordAttention(BasicAttention):
    """Chord attention parameters (`block/attention/chord_attn.py:59-124`)."""

    def __init__(self, hidden_size, num_heads, num_kv_heads=None, **kwargs):
        super().__init__(hidden_size=hidden_size, num_heads=num_heads, num_kv_heads=num_kv_heads)
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.kv_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.kv_dim, bias=False)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.g_proj = nn.Linear(hidden_size, hidden_size, bias=False)
        self.q_norm = RMSNorm(self.head_dim)
        self.k_norm = RMSNorm(self.head_dim)
        self.theta_alpha = nn.Parameter(torch.zeros(num_heads))
        self.theta_beta = nn.Parameter(torch.zeros(num_heads))
        self.theta_mu = nn.Parameter(torch.zeros(num_heads), requires_grad=False)
        self.ssmax_s = nn.Parameter(torch.ones(num_heads))

    @classmethod
    def cache_type(cls):
        return KVLayerCache

    def _ggd_parameters(self):
        """`(alpha, beta, mu)` in fp32 (`chord_attn.py:126-138`)."""
        ta, tb, tm = (t.float() for t in (self.theta_alpha, self.theta_beta, self.theta_mu))
        return torch.exp(ta), tb, torch.exp(tm) - torch.exp(-tm)

    @torch.no_grad()
    def relative_prior(self, max_distance: int, device=None, dtype=torch.float32):
        """GGD bias as a function of signed distance (`chord_attn.py:178-202`)."""
        alpha, beta, mu = self._ggd_parameters()
        device = device if device is not None else self.theta_alpha.device
        d = torch.arange(-max_distance, max_distance + 1, device=device, dtype=alpha.dtype)
        b = torch.abs(d[None, :] - mu[:, None].to(device)) + GGD_EPS
        return (-alpha[:, None].to(device) * b ** beta[:, None].to(device)).to(dtype)


class SwiGLU(nn.Module):
    """Gated MLP `down_proj(act(gate_up_proj(x)))` (`block/mlp.py:7-63`)."""

    def __init__(self, in_features: int, hidden_features: int = None, out_features: int = None, bias: bool = False):
        super().__init__()
        if hidden_features is None:
            h = int(in_features * 8 / 3)
            hidden_features = (h + 127) // 128 * 128
        out_features = out_features or in_features
        self.hidden_features = hidden_features
        self.gate_up_proj = nn.Linear(in_features, 2 * hidden_features, bias=bias)
        self.down_proj = nn.Linear(hidden_features, out_features, bias=bias)
        self.act = SwiGLUOp(dim=-1)

    def forward(self, x):
        return F.linear(self.act(F.linear(x, self.gate_up_proj.weight)), self.down_proj.weight)


class Decoder(nn.Module):
    """attn_norm, attn, mlp_norm, mlp (`block/decoder.py:44-104`)."""

    def __init__(self, attn_type: str, config: MotifChordConfig):
        super().__init__()
        self.attn_type = attn_type.lower()
        self.attn_norm = RMSNorm(config.model_dim)
        if self.attn_type == 'chord':
            self.attn = ChordAttention(hidden_size=config.model_dim, num_heads=config.num_heads,
                                       num_kv_heads=config.num_kv_heads)
        else:
            self.attn = GatedDeltaAttention(hidden_size=config.model_dim, num_heads=config.num_heads,
                                            head_k_dim=config.head_k_dim, expand_v=EXPAND_V,
                                            chunk_size=CHUNK_SIZE, bias=False)
        self.mlp_norm = RMSNorm(config.model_dim)
        self.mlp = SwiGLU(in_features=config.model_dim)

    @property
    def cache_type(self):
        return KVLayerCache if self.attn_type == 'chord' else GatedDeltaAttentionLayerCache


class DecoderBlock(nn.Module):
    """Decoders joined by the intra-block attention residual (`block/decoder.py:107-137`)."""

    def __init__(self, config: MotifChordConfig):
        super().__init__()
        self.features = nn.ModuleList([Decoder(t, config) for t in config.block])
        self.pseudo_queries = nn.ParameterList([nn.Parameter(torch.zeros(config.model_dim)) for _ in self.features])
        self.attn_res_norms = nn.ModuleList([RMSNorm(config.model_dim) for _ in self.features])


# ============================================================================ output
class ModelOutput:
    """Result of one forward (`model/motif.py:27-151`).

    `hidden_states` (the final-normed states) is materialised on first access from the
    pre-norm block output, so a decode step that only needs logits does not pay for it.
    """

    def __init__(self, hidden_states=None, logits=None, loss=None, cache=None, sampler=None, _final=None):
        self._hidden = hidden_states
        self._final = _final
        self.logits = logits
        self.loss = loss
        self.cache = cache
        self.sampler = sampler

    @property
    def hidden_states(self) -> torch.Tensor:
        if self._hidden is None and self._final is not None:
            x, norm = self._final
            with torch.no_grad():
                self._hidden = norm(x)
        return self._hidden

    @hidden_states.setter
    def hidden_states(self, v):
        self._hidden = v

    @property
    def last_hidden_state(self):
        return self.hidden_states[:, -1, :]

    @property
    def last_logits(self):
        return None if self.logits is None else self.logits[:, -1, :]

    def next_token(self, temperature: float = 1.0, sampler=None, input_ids=None):
        """Greedy argmax of the last position, or the given / bound sampler (`motif.py:68-98`)."""
        if self.logits is None:
            return None
        last = self.logits[:, -1, :]
        active = sampler if sampler is not None else self.sampler
        if active is not None:
            return active(last, input_ids)
        return greedy_next(last)

    def set_sampler(self, sampler=None, **kwargs):
        """Bind a sampler to this output (`motif.py:100-131`): a ready one, or one built from
        `Sampler` keyword arguments; no arguments unbinds (greedy)."""
        self.sampler = make_sampler(sampler, **kwargs)
        return self

    def reset_caches(self):
        if self.cache is not None:
            self.cache.reset()

    def __repr__(self):
        lg = tuple(self.logits.shape) if self.logits is not None else None
        return f'ModelOutput(logits={lg}, loss={self.loss is not None}, cache={self.cache!r})'


def greedy_next(last_logits: torch.Tensor) -> torch.Tensor:
    """`[B, V] -> [B, 1]` argmax (first maximum) on the argmax kernel."""
    rows, V = last_logits.shape
    x = last_logits if last_logits.stride(-1) == 1 else last_logits.contiguous()
    ids = torch.empty((rows, 1), dtype=torch.int64, device=x.device)
    _lib.call('motif_b200_argmax', _lib.ptr(x), rows, V, x.stride(0), _lib.ptr(ids), _lib.dtype_code(x.dtype),
              _lib.stream_ptr(x.device))
    return ids


# ============================================================================ packing
def _interleave_gate_up(gu: torch.Tensor, hid: int) -> torch.Tensor:
    """gate_up rows `[values (hid) | gates (hid)]` regrouped in blocks of 256: 128 value rows, then
    the 128 gate rows of the same hidden units (the layout `motif_b200_gemm_proj_swiglu` reads)."""
    v, g = gu[:hid].view(hid // 128, 128, -1), gu[hid:].view(hid // 128, 128, -1)
    return torch.cat([v, g], 1).reshape(2 * hid, -1)


@dataclass
class _GDNPack:
    w_in: torch.Tensor      # [N_in, d]: q | k | v | a | b | g | gate_up, norm weights folded in
    conv_w: torch.Tensor    # [C, 4] q | k | v channels
    A_log: torch.Tensor
    dt_bias: torch.Tensor
    onorm_w: torch.Tensor
    w_out: torch.Tensor     # [d, H*dv + hid]: o_proj | down_proj
    H: int
    dk: int
    dv: int
    hid: int
    off_g: int
    off_gu: int
    w_in_il: Optional[torch.Tensor] = None  # w_in with gate_up regrouped for the fused SwiGLU
    w_in_sk: Optional[torch.Tensor] = None  # decode-sized products: w_in / w_out packed for the skinny GEMM
    w_out_sk: Optional[torch.Tensor] = None


@dataclass
class _ChordPack:
    w_in: torch.Tensor      # [N_in, d]: q | k | v | g | gate_up
    qn_w: torch.Tensor
    kn_w: torch.Tensor
    w_o: torch.Tensor
    w_down: torch.Tensor
    alpha: torch.Tensor
    beta: torch.Tensor
    mu: torch.Tensor
    ssmax: torch.Tensor
    H: int
    Hkv: int
    D: int
    hid: int
    off_g: int
    off_gu: int
    w_in_il: Optional[torch.Tensor] = None  # w_in with gate_up regrouped for the fused SwiGLU
    w_in_sk: Optional[torch.Tensor] = None  # decode-sized products: packed for the skinny GEMM
    w_o_sk: Optional[torch.Tensor] = None
    w_down_sk: Optional[torch.Tensor] = None


def _skinny_packed(w: torch.Tensor) -> Optional[torch.Tensor]:
    """w [N, K] in the skinny GEMM's fragment order (`motif_b200_skinny_pack`), or None where
    that kernel does not apply (CPU, fp32, K not a multiple of 16)."""
    if not w.is_cuda or w.dtype not in (torch.bfloat16, torch.float16) or w.dim() != 2:
        return None
    N, K = w.shape
    # K up to 8 cluster splits x 4 warps x 12 k-tiles of 16 (the kernel's split limits)
    if K % 16 or K > 8 * 4 * 12 * 16 or N % 4 or w.stride(1) != 1 or w.stride(0) % 2 or w.data_ptr() % 4:
        return None
    nbytes = _lib.load().motif_b200_skinny_packed_bytes(N, K)
    out = torch.empty(nbytes // w.element_size(), dtype=w.dtype, device=w.device)
    _lib.call('motif_b200_skinny_pack', w.data_ptr(), w.stride(0), N, K, out.data_ptr(), _lib.dtype_code(w.dtype),
              _lib.stream_ptr(w.device))
    return out


@torch.no_grad()
def _pack_decoder(dec: Decoder):
    wa = dec.attn_norm.weight[None, :]
    wm = dec.mlp_norm.weight[None, :]
    a = dec.attn
    hid = dec.mlp.hidden_features
    gu = dec.mlp.gate_up_proj.weight * wm
    if dec.attn_type == 'chord':
        parts = [a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.g_proj.weight]
        off_g = a.hidden_size + 2 * a.kv_dim
        w_in = torch.cat([p * wa for p in parts] + [gu], 0).contiguous()
        w_in_il = (torch.cat([w_in[:off_g + a.hidden_size], _interleave_gate_up(w_in[off_g + a.hidden_size:], hid)],
                             0).contiguous() if hid % 128 == 0 else None)
        al, be, mu = a._ggd_parameters()
        w_o = a.o_proj.weight.detach().contiguous()
        w_down = dec.mlp.down_proj.weight.detach().contiguous()
        return _ChordPack(w_in=w_in, qn_w=a.q_norm.weight.detach().contiguous(),
                          kn_w=a.k_norm.weight.detach().contiguous(), w_o=w_o, w_down=w_down, alpha=al.contiguous(),
                          beta=be.contiguous(), mu=mu.contiguous(), ssmax=a.ssmax_s.detach().float().contiguous(),
                          H=a.num_heads, Hkv=a.num_kv_heads, D=a.head_dim, hid=hid, off_g=off_g,
                          off_gu=off_g + a.hidden_size, w_in_il=w_in_il, w_in_sk=_skinny_packed(w_in),
                          w_o_sk=_skinny_packed(w_o), w_down_sk=_skinny_packed(w_down))
    H, dk, dv = a.num_heads, a.dk, a.dv
    parts = [a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.a_proj.weight, a.b_proj.weight, a.g_proj.weight]
    off_g = 2 * H * dk + H * dv + 2 * H
    w_in = torch.cat([p * wa for p in parts] + [gu], 0).contiguous()
    off_gu = off_g + H * dv
    w_in_il = (torch.cat([w_in[:off_gu], _interleave_gate_up(w_in[off_gu:], hid)], 0).contiguous()
               if hid % 128 == 0 else None)
    conv_w = torch.cat([a.q_conv.weight.reshape(-1, CONV_SIZE), a.k_conv.weight.reshape(-1, CONV_SIZE),
                        a.v_conv.weight.reshape(-1, CONV_SIZE)], 0).contiguous()
    w_out = torch.cat([a.o_proj.weight, dec.mlp.down_proj.weight], 1).contiguous()
    return _GDNPack(w_in=w_in, conv_w=conv_w, A_log=a.A_log.detach().contiguous(),
                    dt_bias=a.dt_bias.detach().contiguous(), onorm_w=a.o_norm.weight.detach().contiguous(),
                    w_out=w_out, H=H, dk=dk, dv=dv, hid=hid, off_g=off_g, off_gu=off_gu, w_in_il=w_in_il,
                    w_in_sk=_skinny_packed(w_in), w_out_sk=_skinny_packed(w_out))


# ============================================================================ model
class MotifChordModel(nn.Module):
    """The Motif Chord decoder-only LM (`model/motif.py:154-630`) on the sm_100a kernels."""

    def __init__(self, config):
        super().__init__()
        config = MotifChordConfig.from_any(config)
        self.config = config
        self.embed = nn.Embedding(config.vocab_size, config.model_dim)
        self.blocks = nn.ModuleList([DecoderBlock(config) for _ in range(config.block_n)])
        self.norm = RMSNorm(config.model_dim)
        self.lm_head = nn.Linear(config.model_dim, config.vocab_size, bias=False)
        if config.tied_weight:
            self.embed.weight = self.lm_head.weight
        self.sampler = None
        self._packed = None
        self._lm_sk = None
        self.decode_splits = None  # split-KV count override for the decode attention

    # ------------------------------------------------------------------ bookkeeping
    def invalidate_packed(self):
        self._packed = None

    def _apply(self, fn, *args, **kwargs):
        self._packed = None
        return super()._apply(fn, *args, **kwargs)

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        self._packed = None
        return super().load_state_dict(state_dict, strict=strict, assign=assign)

    def packed(self):
        if self._packed is None:
            with torch.no_grad():
                decs = [[_pack_decoder(dec) for dec in blk.features] for blk in self.blocks]
                lm = (self.lm_head.weight * self.norm.weight[None, :]).contiguous()
                self._lm_sk = _skinny_packed(lm)
            self._packed = (decs, lm)
        return self._packed

    @classmethod
    def from_pretrained(cls, path, config=None, map_location='cpu', device=None, strict: bool = False,
                        verbose: bool = True, **overrides) -> 'MotifChordModel':
        """Build the model from a checkpoint (`model/motif.py:237-360`): a bare state_dict, a
        pipeline checkpoint or safetensors (file, shard directory, index).  The config is the
        `config` argument (a config, a mapping or a JSON file path), else the file's, else the one
        the tensor shapes imply; `**overrides` replace fields of it.  Tied models take a missing
        `lm_head.weight` from `embed.weight`.  Returns the model in eval mode."""
        import dataclasses
        import json
        import os
        from .checkpoint import config_from_mapping, config_from_state_dict, load_checkpoint
        loaded = load_checkpoint(path, map_location=map_location)
        sd = loaded.state_dict
        if config is not None:
            if isinstance(config, (str, os.PathLike)):
                with open(config, 'r', encoding='utf-8') as f:
                    resolved = config_from_mapping(json.load(f))
            elif isinstance(config, dict):
                resolved = config_from_mapping(config)
            else:
                resolved = MotifChordConfig.from_any(config)
        elif loaded.config is not None:
            resolved = loaded.config
        else:
            try:
                resolved = config_from_state_dict(sd)
            except ValueError:
                resolved = MotifChordConfig()
        if overrides:
            known = {f.name for f in dataclasses.fields(MotifChordConfig)}
            unknown = sorted(set(overrides) - known)
            if unknown:
                raise TypeError(f'unknown MotifChordConfig override(s): {unknown}; valid names are {sorted(known)}.')
            resolved = dataclasses.replace(resolved, **overrides)
        model = cls(resolved)
        emb, head = sd.get('embed.weight'), sd.get('lm_head.weight')
        note = None
        if resolved.tied_weight:
            if head is None and emb is not None:
                sd['lm_head.weight'] = emb
                note = 'lm_head.weight taken from embed.weight (tied weights)'
            elif head is not None and emb is not None and head is not emb and not torch.equal(head, emb):
                note = ('the checkpoint is untied but the config has tied_weight=True: lm_head.weight and '
                        'embed.weight disagree, the last one loaded wins.')
        try:
            incompatible = model.load_state_dict(sd, strict=False)
        except RuntimeError as e:
            raise RuntimeError(f'{os.fspath(path)!r} does not match the model built from {resolved!r}: {e}') from e
        missing, unexpected = list(incompatible.missing_keys), list(incompatible.unexpected_keys)
        if strict and (missing or unexpected):
            raise RuntimeError(f'{os.fspath(path)!r} does not match the model exactly: {len(missing)} missing key(s) '
                               f'{missing[:8]}, {len(unexpected)} unexpected key(s) {unexpected[:8]}.')
        if device is not None:
            model = model.to(device)
        model.eval()
        if verbose:
            builtins.print(f'[MotifChordModel] {os.fspath(path)} -> {loaded.source}: {len(sd):,} tensors, '
                           f'{model.count_param():,} params')
            builtins.print(f'  config: {resolved}')
            if note:
                builtins.print(f'  note: {note}')
            if missing:
                builtins.print(f'  missing ({len(missing)}): {missing[:8]}' + (' ...' if len(missing) > 8 else ''))
            if unexpected:
                builtins.print(f'  unexpected ({len(unexpected)}): {unexpected[:8]}'
                               + (' ...' if len(unexpected) > 8 else ''))
        return model

    def save_pretrained(self, path: str, metadata=None):
        """Write the weights and config as one `.safetensors` file (`save_safetensors`)."""
        from .checkpoint import save_safetensors
        return save_safetensors(self, path, metadata=metadata)

    def count_param(self, print: bool = False) -> int:
        """Parameter count, tied weights once (`model/motif.py:377-400`)."""
        total = int(sum(p.numel() for p in self.parameters()))
        if print:
            builtins.print(f'{type(self).__name__} params: {total:,}')
        return total

    def cache_types(self):
        return [[d.cache_type for d in blk.features] for blk in self.blocks]

    def create_cache(self, use_attn: Optional[bool] = None, functional: bool = False,
                     wide_kv: bool = False) -> ModelCache:
        """`create_cache` (`model/motif.py:413-455`)."""
        return build_cache(self, use_attn=use_attn, functional=functional, wide_kv=wide_kv)

    def set_sampler(self, sampler=None, **kwargs):
        """Model-level sampler carried by every later `ModelOutput` (`motif.py:457-482`)."""
        self.sampler = make_sampler(sampler, **kwargs)
        return self

    def generate(self, input_ids, max_new_tokens: int = 32, eos_token_id=None, sampler=None, cache=None,
                 mask=None, tokenizer=None, graph: bool = False, sync_every: int = 16):
        """`generate` (`model/motif.py:483-543`)."""
        from .generate import Generation
        active = sampler if sampler is not None else self.sampler
        if eos_token_id is None and active is not None:
            eos_token_id = getattr(active, 'eos_token_id', None)
        if eos_token_id is None and tokenizer is not None:
            eos_token_id = getattr(tokenizer, 'token_eos', None)
        return Generation(self, input_ids, max_new_tokens, eos_token_id, sampler, cache, mask, tokenizer,
                          graph=graph, sync_every=sync_every)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: torch.Tensor, cache: Optional[ModelCache] = None, labels=None,
                mask: Optional[torch.Tensor] = None, position: Optional[Union[int, torch.Tensor]] = None):
        """`MotifChordModel.forward` (`model/motif.py:545-630`) on the fused kernels."""
        if input_ids.dim() != 2:
            raise ValueError(f'input_ids must be [B, T], got {tuple(input_ids.shape)}')
        if not self.embed.weight.is_cuda:
            raise ValueError('motif_b200 runs on CUDA only: move the model to a CUDA device')
        cached = cache.seq_len if cache is not None else 0
        if mask is not None:
            width = cached + input_ids.shape[1]
            if mask.dim() != 2:
                raise ValueError(f'mask must be [B, T], got {tuple(mask.shape)}')
            if mask.shape != (input_ids.shape[0], width):
                raise ValueError(f'mask {tuple(mask.shape)} does not cover the {width} keys of a {cached}-position '
                                 f'cache plus {input_ids.shape[1]} inputs')
            key_bias = _key_bias(mask, self.embed.weight.device)
        if isinstance(position, torch.Tensor):
            position = int(position.reshape(-1)[0])
        if cache is None:
            cache = self.create_cache()
        with torch.no_grad():
            logits, x_final = _forward(self, input_ids.to(self.embed.weight.device), cache, position or 0,
                                       key_bias if mask is not None else None)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.view(-1, logits.size(-1)).float(), labels.view(-1).to(logits.device),
                                   ignore_index=-100)
        return ModelOutput(logits=logits, loss=loss, cache=cache, sampler=self.sampler,
                           _final=(x_final, self.norm))


# ============================================================================ engine
# Largest M routed to motif_b200_skinny_gemm (decode: one row per sequence).  Measured on the
# 172M decode step (context 8192, CUDA graph): 0.365 vs 0.447 ms per step at 8 rows, 0.443 vs
# 0.503 at 16, 0.548 vs 0.565 at 32, but 0.908 vs 0.747 at 64, where the legacy-MMA products
# and the cluster's partial-tile exchange cost more than the latency the kernel hides.
SKINNY_MAX_M = 32
# Row counts SKINNY_MAX_M < M <= SKINNY_TC_MAX_M run on the tensor-core decode GEMM
# (motif_b200_skinny_gemm_tc, the weight as it is) for the shapes where it measured faster than
# the library GEMM at 64 rows (CUDA graphs of back-to-back products, weights streamed from HBM):
# long K (the decoders' output and down projections, K >= 2048: e.g. N 768 x K 2816 5.8 vs
# 6.3 us) and the lm_head (N >= 16384: 10.5 vs 10.9 us).  The wide K = 768 input projections
# stay on the library GEMM (N 8728: 7.5 vs 5.1 us): one CTA streams its weight run at only
# ~40-55 GB/s, so they would need more split-K parts than the exchange of the partials allows.
SKINNY_TC_MAX_M = 64


def _tc_skinny_ok(a: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor], fused: bool = False) -> bool:
    """The tensor-core decode GEMM takes the product: above SKINNY_MAX_M rows for the long-K
    products and the lm_head; at SKINNY_MAX_M rows or fewer only the lm_head (at 8 rows 10.6 us
    against 12.2 on the legacy-MMA kernel) and, with `fused`, the Chord down projection that
    carries the gated residual in its epilogue (one launch instead of two)."""
    M, K = a.shape
    N = w.shape[0]
    small_ok = fused or N >= 16384
    return (0 < M <= SKINNY_TC_MAX_M and (M > SKINNY_MAX_M or small_ok) and (K >= 2048 or N >= 16384)
            and a.dtype in (torch.bfloat16, torch.float16) and w.dtype == a.dtype
            and K % 64 == 0 and N % 4 == 0 and a.stride(1) == 1 and w.stride(1) == 1
            and a.stride(0) % 8 == 0 and w.stride(0) % 8 == 0 and a.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0
            and (out is None or (out.stride(1) == 1 and out.stride(0) % 4 == 0 and out.data_ptr() % 8 == 0)))


def _mm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor = None, wp: torch.Tensor = None) -> torch.Tensor:
    """a [M, K] @ w[N, K]^T: decode-sized M (<= 64, 16-bit) on the weight-streaming skinny GEMM
    when `wp` (w packed by `_skinny_packed`) is given and M <= SKINNY_MAX_M, on the tensor-core
    decode GEMM for the larger decode batches, everything else on cuBLAS (plain library GEMM;
    timed as 'cublas_gemm')."""
    M, K = a.shape
    N = w.shape[0]
    if _tc_skinny_ok(a, w, out):
        y = out if out is not None else torch.empty((M, N), dtype=a.dtype, device=a.device)
        _lib.call('motif_b200_skinny_gemm_tc', a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(),
                  y.stride(0), M, N, K, 0, _lib.dtype_code(a.dtype), _lib.stream_ptr(a.device))
        return y
    if (wp is not None and M <= SKINNY_MAX_M and a.dtype == w.dtype and a.stride(1) == 1
            and a.stride(0) % 8 == 0 and a.data_ptr() % 16 == 0
            and (out is None or (out.stride(1) == 1 and out.stride(0) % 4 == 0 and out.data_ptr() % 8 == 0))):
        y = out if out is not None else torch.empty((M, N), dtype=a.dtype, device=a.device)
        _lib.call('motif_b200_skinny_gemm', a.data_ptr(), a.stride(0), wp.data_ptr(), y.data_ptr(), y.stride(0), M, N,
                  K, 0, 0, _lib.dtype_code(a.dtype), _lib.stream_ptr(a.device))
        return y
    tr = _lib._tracker
    if tr is None:
        return torch.mm(a, w.t(), out=out)
    ev = tr.start('cublas_gemm')
    r = torch.mm(a, w.t(), out=out)
    if ev is not None:
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        tr.records.append(('cublas_gemm', ev, end))
    return r


def _down_add_gated(act: torch.Tensor, w_down: torch.Tensor, a: torch.Tensor,
                    gate: torch.Tensor) -> Optional[torch.Tensor]:
    """The Chord decoder's `down_proj(act) + o_proj(out) * sigmoid(g)` for decode-sized batches
    (`chord_attn.py:254,313`, `decoder.py:208`) as ONE launch: the tensor-core decode GEMM with
    the gated residual in its epilogue (`motif_b200_skinny_gemm_tc_add_gated`), given the o_proj
    output `a`; None when that kernel does not take the shapes."""
    M, K = act.shape
    N = w_down.shape[0]
    if not (_tc_skinny_ok(act, w_down, None, fused=True) and a.shape == (M, N) and gate.shape == (M, N)
            and a.dtype == gate.dtype == act.dtype and a.stride(1) == 1 and gate.stride(1) == 1
            and a.stride(0) % 4 == 0 and gate.stride(0) % 4 == 0 and a.data_ptr() % 8 == 0
            and gate.data_ptr() % 8 == 0):
        return None
    y = torch.empty((M, N), dtype=act.dtype, device=act.device)
    _lib.call('motif_b200_skinny_gemm_tc_add_gated', act.data_ptr(), act.stride(0), w_down.data_ptr(),
              w_down.stride(0), a.data_ptr(), a.stride(0), gate.data_ptr(), gate.stride(0), y.data_ptr(),
              y.stride(0), M, N, K, 0, _lib.dtype_code(act.dtype), _lib.stream_ptr(act.device))
    return y


# Decode-sized Chord decoders run their o_proj, down_proj and gated residual as one launch
# (motif_b200_skinny_gemm_tc_chord_tail).
CHORD_TAIL_ONE_LAUNCH = True


def _chord_tail(attn: torch.Tensor, w_o: torch.Tensor, act: torch.Tensor, w_down: torch.Tensor,
                gate: torch.Tensor) -> Optional[torch.Tensor]:
    """The Chord decoder's `o_proj(out) * sigmoid(g) + down_proj(act)` (`chord_attn.py:254,313`,
    `mlp.py:63`, `decoder.py:208`) for decode-sized batches as ONE launch on the tensor-core decode
    GEMM; None when that kernel does not take the shapes."""
    M, K1 = attn.shape
    K2 = act.shape[1]
    N = w_o.shape[0]
    ts = (attn, w_o, act, w_down)
    if not (CHORD_TAIL_ONE_LAUNCH and 0 < M <= SKINNY_TC_MAX_M and act.shape[0] == M and w_down.shape[0] == N
            and attn.dtype in (torch.bfloat16, torch.float16) and all(t.dtype == attn.dtype for t in ts + (gate,))
            and K1 % 64 == 0 and K2 % 64 == 0 and N % 4 == 0 and w_o.shape[1] == K1 and w_down.shape[1] == K2
            and all(t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 for t in ts)
            and gate.shape == (M, N) and gate.stride(1) == 1 and gate.stride(0) % 4 == 0 and gate.data_ptr() % 8 == 0):
        return None
    y = torch.empty((M, N), dtype=attn.dtype, device=attn.device)
    _lib.call('motif_b200_skinny_gemm_tc_chord_tail', attn.data_ptr(), attn.stride(0), w_o.data_ptr(), w_o.stride(0),
              K1, act.data_ptr(), act.stride(0), w_down.data_ptr(), w_down.stride(0), K2, gate.data_ptr(),
              gate.stride(0), y.data_ptr(), y.stride(0), M, N, _lib.dtype_code(attn.dtype),
              _lib.stream_ptr(attn.device))
    return y


def _tc_ok(*ts: torch.Tensor) -> bool:
    """The tcgen05 projection kernels take 16-bit operands with 16-byte aligned rows and K a
    multiple of 64; fp32 (the parity mode) stays on the library GEMM."""
    a = ts[0]
    return (a.dtype in (torch.bfloat16, torch.float16) and a.shape[1] % 64 == 0
            and all(t.dtype == a.dtype and t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0
                    for t in ts))


# Row counts up to this stay on the library GEMM: decode-sized products stream the weights once
# and the persistent 128-row tiles would leave most of the GPU idle.
TC_MIN_M = 65


def _gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor = None, wp: torch.Tensor = None) -> torch.Tensor:
    """a [M, K] @ w[N, K]^T: prefill-sized 16-bit products on the tcgen05 projection kernel
    (`motif_b200_gemm`), decode-sized or fp32 ones on `_mm` (`wp`: w packed for the skinny GEMM)."""
    M, K = a.shape
    N = w.shape[0]
    if M >= TC_MIN_M and _tc_ok(a, w) and (out is None or (out.stride(1) == 1 and out.dtype == a.dtype)):
        y = out if out is not None else torch.empty((M, N), dtype=a.dtype, device=a.device)
        _lib.call('motif_b200_gemm', _lib.ptr(a), a.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(y), y.stride(0),
                  M, N, K, _lib.dtype_code(a.dtype), _lib.stream_ptr(a.device))
        return y
    return _mm(a, w, out, wp)


def _proj_fused(pk, hn: torch.Tensor, act: torch.Tensor):
    """The decoder's packed input projection with its SwiGLU fused (`motif_b200_gemm_proj_swiglu`)
    when the shapes allow it: returns the [M, off_gu] projection (q | k | v | ... | g) and writes
    the MLP activation into `act`; else None."""
    M = hn.shape[0]
    if pk.w_in_il is None or M < TC_MIN_M or not _tc_ok(hn, pk.w_in_il, act):
        return None
    proj = torch.empty((M, pk.off_gu), dtype=hn.dtype, device=hn.device)
    _lib.call('motif_b200_gemm_proj_swiglu', _lib.ptr(hn), hn.stride(0), _lib.ptr(pk.w_in_il), pk.w_in_il.stride(0),
              M, hn.shape[1], pk.off_gu, _lib.ptr(proj), proj.stride(0), pk.hid, _lib.ptr(act), act.stride(0),
              _lib.dtype_code(hn.dtype), _lib.stream_ptr(hn.device))
    return proj


def _norm_read(sources: List[torch.Tensor], query, weight, h_out, hn_out, eps_src=NORM_EPS, eps_out=NORM_EPS):
    x0 = sources[0]
    rows, d = x0.shape
    _lib.call('motif_b200_attn_res_norm', _lib.ptr_array([s.data_ptr() for s in sources]), len(sources),
              x0.stride(0), _lib.ptr(weight), _lib.ptr(query), _lib.ptr(h_out), _lib.ptr(hn_out), hn_out.stride(0),
              rows, d, float(eps_src), float(eps_out), _lib.dtype_code(x0.dtype), _lib.stream_ptr(x0.device))


def _forward(model: MotifChordModel, ids: torch.Tensor, cache: ModelCache, position: int,
             key_bias: Optional[torch.Tensor] = None):
    cfg = model.config
    decs, lm = model.packed()
    B, T = ids.shape
    M = B * T
    d = cfg.model_dim
    w = model.embed.weight
    dt, dev = w.dtype, w.device
    dc = _lib.dtype_code(dt)
    st = _lib.stream_ptr(dev)
    ids = ids.contiguous()

    x = torch.empty((M, d), dtype=dt, device=dev)
    _lib.call('motif_b200_embed', _lib.ptr(ids), _lib.ptr(w), _lib.ptr(x), M, d, cfg.vocab_size, dc, st)
    hn = torch.empty((M, d), dtype=dt, device=dev)
    _norm_read([x], None, None, None, hn)

    for b, block in enumerate(model.blocks):
        bc = cache[b]
        ar = bc.attn_res
        ar.init_embedding(x.view(B, T, d))
        if len(bc.attn) == 0:
            if not model.training:
                bc.ensure_attn([dec.cache_type for dec in block.features])
        elif len(bc.attn) != len(block.features):
            raise ValueError(f'cache.attn has {len(bc.attn)} entries but the block has {len(block.features)} layers')
        use_cache = len(bc.attn) == len(block.features)
        fs: List[torch.Tensor] = []
        for i, dec in enumerate(block.features):
            if i > 0:
                hn = torch.empty((M, d), dtype=dt, device=dev)
                _norm_read([x] + fs, block.pseudo_queries[i].detach(), block.attn_res_norms[i].weight.detach(),
                           None, hn, eps_src=block.attn_res_norms[i].eps)
            pk = decs[b][i]
            layer_cache = bc.attn[i] if use_cache else None
            if dec.attn_type == 'chord':
                if layer_cache is not None and not isinstance(layer_cache, KVLayerCache):
                    raise TypeError(f'ChordAttention requires KVLayerCache, got {type(layer_cache).__name__}')
                f = _chord_decoder(model, pk, hn, B, T, layer_cache, position, dt, dev, dc, st, key_bias)
            else:
                if layer_cache is not None and not isinstance(layer_cache, GatedDeltaAttentionLayerCache):
                    raise TypeError(f'GatedDeltaAttention requires GatedDeltaAttentionLayerCache, '
                                    f'got {type(layer_cache).__name__}')
                f = _gdn_decoder(pk, hn, B, T, layer_cache, dt, dev, dc, st)
            fs.append(f)
        # block output = sum of the increments (decoder.py:215-217), and its RMSNorm for the
        # next block's first decoder (or the final norm before lm_head)
        x_next = torch.empty((M, d), dtype=dt, device=dev)
        hn = torch.empty((M, d), dtype=dt, device=dev)
        _norm_read(fs, None, None, x_next, hn, eps_out=(model.norm.eps if b == len(model.blocks) - 1 else
                                                         model.blocks[b + 1].features[0].attn_norm.eps))
        ar.blocks.extend(f.view(B, T, d) for f in fs)
        ar.partial_block = x_next.view(B, T, d)
        ar.seq_len = max(ar.seq_len, T)
        x = x_next
    logits = _gemm(hn, lm, wp=model._lm_sk)
    return logits.view(B, T, cfg.vocab_size), x.view(B, T, d)


def _gdn_decoder(pk: _GDNPack, hn, B, T, cache: Optional[GatedDeltaAttentionLayerCache], dt, dev, dc, st):
    """`GatedDeltaAttention.forward` + the SwiGLU MLP + the parallel residual (decoder.py:203-208)."""
    M = B * T
    H, dk, dv, hid = pk.H, pk.dk, pk.dv, pk.hid
    C = H * (2 * dk + dv)
    cat = torch.empty((M, H * dv + hid), dtype=dt, device=dev)  # [gated-normed o | act]
    # prefill: the input projection with the MLP activation fused, written into cat's right half
    proj = _proj_fused(pk, hn, cat[:, H * dv:]) if T > 1 else None
    act_done = proj is not None
    if proj is None:
        proj = _mm(hn, pk.w_in, wp=pk.w_in_sk)
    N_in = proj.shape[1]
    state_in = cache.state if cache is not None else None
    conv_in = cache._conv if cache is not None else None
    if state_in is not None and (state_in.dtype != torch.float32 or not state_in.is_contiguous()):
        state_in = state_in.float().contiguous()
    if conv_in is not None and (conv_in.dtype != dt or not conv_in.is_contiguous()):
        conv_in = conv_in.to(dt).contiguous()
    eps = NORM_EPS
    if T == 1:
        # gdn_attn.py:198-199: the L == 1 step is the recurrence, fused with conv and o_norm.
        state = state_in if state_in is not None else torch.zeros((B, H, dk, dv), dtype=torch.float32, device=dev)
        conv = conv_in if conv_in is not None else torch.zeros((B, 3, C), dtype=dt, device=dev)
        # ... and with the MLP activation in the same launch
        _lib.call('motif_b200_gdn_decode_swiglu', _lib.ptr(proj), N_in, _lib.ptr(pk.conv_w), _lib.ptr(pk.A_log),
                  _lib.ptr(pk.dt_bias), _lib.ptr(conv), _lib.ptr(state), proj.data_ptr() + pk.off_g * proj.element_size(),
                  _lib.ptr(pk.onorm_w), _lib.ptr(cat), cat.stride(0), B, H, dk, dv, eps,
                  proj.data_ptr() + pk.off_gu * proj.element_size(), N_in,
                  cat.data_ptr() + H * dv * cat.element_size(), cat.stride(0), hid, dc, st)
        conv_out = conv
    elif dt != torch.float32 and (dk, dv) == (64, 128) and N_in % 8 == 0:
        # three kernels: preparation fused into the parallel per-chunk UT transform (records in a
        # workspace), the state scan, the gated norm
        conv_out = torch.empty((B, 3, C), dtype=dt, device=dev)
        state = torch.empty((B, H, dk, dv), dtype=torch.float32, device=dev)
        ws_bytes = _lib.load().motif_b200_gdn_chunk_workspace_bytes(B, H, T, dk, dv, dc)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        _lib.call('motif_b200_gdn_prefill_ws', _lib.ptr(proj), N_in, _lib.ptr(pk.conv_w), _lib.ptr(pk.A_log),
                  _lib.ptr(pk.dt_bias), _lib.ptr(conv_in), _lib.ptr(conv_out), _lib.ptr(state_in), _lib.ptr(state),
                  _lib.ptr(pk.onorm_w), eps, _lib.ptr(cat), cat.stride(0), B, T, H, dk, dv, dc, _lib.ptr(ws), ws_bytes,
                  st)
    else:
        qb = torch.empty((M, H * dk), dtype=dt, device=dev)
        kb = torch.empty((M, H * dk), dtype=dt, device=dev)
        vb = torch.empty((M, H * dv), dtype=dt, device=dev)
        beta = torch.empty((M, H), dtype=torch.float32, device=dev)
        g = torch.empty((M, H), dtype=torch.float32, device=dev)
        conv_out = torch.empty((B, 3, C), dtype=dt, device=dev)
        _lib.call('motif_b200_gdn_prep', _lib.ptr(proj), N_in, _lib.ptr(pk.conv_w), _lib.ptr(pk.A_log),
                  _lib.ptr(pk.dt_bias), _lib.ptr(conv_in), _lib.ptr(conv_out), _lib.ptr(qb), _lib.ptr(kb),
                  _lib.ptr(vb), _lib.ptr(beta), _lib.ptr(g), B, T, H, dk, dv, dc, st)
        state = torch.empty((B, H, dk, dv), dtype=torch.float32, device=dev)
        cs = cat.stride(0)
        strides = [T * H * dk, dk, H * dk, T * H * dk, dk, H * dk, T * H * dv, dv, H * dv,
                   T * cs, dv, cs, T * H, 1, H, T * H, 1, H]
        # two-kernel chunked delta rule: parallel UT transform into a workspace, then the scan
        ws_bytes = _lib.load().motif_b200_gdn_chunk_workspace_bytes(B, H, T, dk, dv, dc)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
        _lib.call('motif_b200_gdn_chunk_gated_ws', _lib.ptr(qb), _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(beta),
                  _lib.ptr(g), _lib.ptr(state_in), _lib.ptr(state), _lib.ptr(cat), B, H, T, dk, dv,
                  _lib.i64_array(strides), proj.data_ptr() + pk.off_g * proj.element_size(), N_in, dv,
                  _lib.ptr(pk.onorm_w), eps, dc, _lib.ptr(ws), max(ws_bytes, 0), st)
    if T != 1 and not act_done:
        _lib.call('motif_b200_swiglu', proj.data_ptr() + pk.off_gu * proj.element_size(),
                  cat.data_ptr() + H * dv * cat.element_size(), M, hid, N_in, cat.stride(0), dc, st)
    f = _gemm(cat, pk.w_out, wp=pk.w_out_sk)
    if cache is not None:
        cache._split = (H * dk, H * dk, H * dv)
        cache.update(state, conv_out, steps=T)
    return f


_SMS: Dict[int, int] = {}


def _decode_splits(model, B, Hkv, S):
    if model.decode_splits:
        return int(model.decode_splits)
    dev = torch.cuda.current_device()
    if dev not in _SMS:
        _SMS[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    sms = _SMS[dev]
    # about two CTAs per SM, and at least 12 splits: measured on the 172M decode step (context
    # 8192), 12-16 splits were best at 8, 16, 32 and 64 requests (finer splits cost more in
    # per-CTA start-up and merge than they add in parallelism); tiny batches split further
    want = max(12, -(-2 * sms // max(1, B * Hkv)))
    return int(max(1, min(want, 64, (S + 255) // 256)))


def _chord_decoder(model, pk: _ChordPack, hn, B, T, cache: Optional[KVLayerCache], position, dt, dev, dc, st,
                   key_bias: Optional[torch.Tensor] = None):
    """`ChordAttention.forward` (fused path) + SwiGLU MLP + parallel residual.  `key_bias`
    ([B, S] fp32, natural-log units) is the attention mask as an additive key bias."""
    M = B * T
    H, Hkv, D, hid = pk.H, pk.Hkv, pk.D, pk.hid
    d = H * D
    act = torch.empty((M, hid), dtype=dt, device=dev)
    # prefill: the input projection with the MLP activation fused
    proj = _proj_fused(pk, hn, act) if T > 1 else None
    act_done = proj is not None
    fused_proj = act_done
    if proj is None:
        proj = _mm(hn, pk.w_in, wp=pk.w_in_sk)
    N_in = proj.shape[1]
    if cache is None:
        cache = KVLayerCache()  # no layer cache (training-mode forward): attend to this chunk only
    if cache._kbuf is not None and (cache._kbuf.dtype != dt or cache._kbuf.device != dev):
        cache.to(device=dev, dtype=dt)
    cached = cache.length
    q_start = position if position != 0 else cached
    qb = torch.empty((M, d), dtype=dt, device=dev)
    if cache.wide:
        # a wide cache (`cache.py:42-70`) stores every key / value head once per query head: the
        # new keys / values are prepared narrow, widened by the cache's own update, and the
        # attention then reads one kv head per query head (the same arithmetic as grouped)
        kt = torch.empty((B, Hkv, T, D), dtype=dt, device=dev)
        vt = torch.empty_like(kt)
        _lib.call('motif_b200_chord_prep', _lib.ptr(proj), N_in, _lib.ptr(pk.qn_w), _lib.ptr(pk.kn_w), _lib.ptr(qb),
                  _lib.ptr(kt), _lib.ptr(vt), T, None, 0, B, T, H, Hkv, D, NORM_EPS, dc, st)
        cache.update(kt, vt)
        cache.reserve(cache.length, like=proj, shape=(B, H, D))
        Hkv = H
    elif act_done:
        cache.reserve(cached + T, like=proj, shape=(B, Hkv, D))
        # q/k norms + cache append (the MLP activation came with the projection)
        _lib.call('motif_b200_chord_prep', _lib.ptr(proj), N_in, _lib.ptr(pk.qn_w), _lib.ptr(pk.kn_w), _lib.ptr(qb),
                  _lib.ptr(cache._kbuf), _lib.ptr(cache._vbuf), cache._kbuf.shape[2], None, cached, B, T, H, Hkv, D,
                  NORM_EPS, dc, st)
        cache.length = cached + T
    else:
        cache.reserve(cached + T, like=proj, shape=(B, Hkv, D))
        # q/k norms + cache append and the MLP activation in one launch
        _lib.call('motif_b200_chord_prep_swiglu', _lib.ptr(proj), N_in, _lib.ptr(pk.qn_w), _lib.ptr(pk.kn_w),
                  _lib.ptr(qb), _lib.ptr(cache._kbuf), _lib.ptr(cache._vbuf), cache._kbuf.shape[2], None, cached, B,
                  T, H, Hkv, D, NORM_EPS, proj.data_ptr() + pk.off_gu * proj.element_size(), N_in, _lib.ptr(act),
                  hid, hid, dc, st)
        act_done = True
        cache.length = cached + T
    cap = cache._kbuf.shape[2]
    S = cache.length
    attn = torch.empty((M, d), dtype=dt, device=dev)
    scale = D ** -0.5
    G = H // Hkv
    if q_start == S - T and G * T <= 16 and D in (32, 64):
        splits = _decode_splits(model, B, Hkv, S)
        ws_bytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, splits)
        ws = torch.empty((ws_bytes // 4,), dtype=torch.float32, device=dev)
        if key_bias is None:
            _lib.call('motif_b200_chord_decode', _lib.ptr(qb), _lib.ptr(cache._kbuf), _lib.ptr(cache._vbuf), cap,
                      None, S, _lib.ptr(pk.alpha), _lib.ptr(pk.beta), _lib.ptr(pk.mu), _lib.ptr(pk.ssmax),
                      _lib.ptr(attn), d, B, H, Hkv, T, D, scale, GGD_EPS, splits, _lib.ptr(ws), ws_bytes, dc, st)
        else:
            _lib.call('motif_b200_chord_decode_masked', _lib.ptr(qb), _lib.ptr(cache._kbuf), _lib.ptr(cache._vbuf),
                      cap, None, S, _lib.ptr(pk.alpha), _lib.ptr(pk.beta), _lib.ptr(pk.mu), _lib.ptr(pk.ssmax),
                      _lib.ptr(attn), d, B, H, Hkv, T, D, scale, GGD_EPS, splits, _lib.ptr(key_bias),
                      key_bias.stride(0), _lib.ptr(ws), ws_bytes, dc, st)
    else:
        log_n = _log_n(q_start, T, dev)
        strides = [T * d, D, d, Hkv * cap * D, cap * D, D, Hkv * cap * D, cap * D, D, T * d, D, d, 0, 1]
        if key_bias is None:
            _lib.call('motif_b200_chord_attention', _lib.ptr(qb), _lib.ptr(cache._kbuf), _lib.ptr(cache._vbuf),
                      _lib.ptr(pk.alpha), _lib.ptr(pk.beta), _lib.ptr(pk.mu), _lib.ptr(pk.ssmax), _lib.ptr(log_n),
                      _lib.ptr(attn), B, H, Hkv, T, S, D, q_start, scale, GGD_EPS, _lib.i64_array(strides), dc, None,
                      0, st)
        else:
            _lib.call('motif_b200_chord_attention_masked', _lib.ptr(qb), _lib.ptr(cache._kbuf),
                      _lib.ptr(cache._vbuf), _lib.ptr(pk.alpha), _lib.ptr(pk.beta), _lib.ptr(pk.mu),
                      _lib.ptr(pk.ssmax), _lib.ptr(log_n), _lib.ptr(attn), B, H, Hkv, T, S, D, q_start, scale,
                      GGD_EPS, _lib.i64_array(strides), _lib.ptr(key_bias), key_bias.stride(0), dc, st)
    if not act_done:
        _lib.call('motif_b200_swiglu', proj.data_ptr() + pk.off_gu * proj.element_size(), _lib.ptr(act), M, hid,
                  N_in, hid, dc, st)
    gate = proj[:, pk.off_g:pk.off_g + d]
    a = None
    if not fused_proj:  # decode-sized: the whole tail in one launch, else o_proj then down + residual
        f = _chord_tail(attn, pk.w_o, act, pk.w_down, gate)
        if f is not None:
            return f
        a = _mm(attn, pk.w_o, wp=pk.w_o_sk)
        f = _down_add_gated(act, pk.w_down, a, gate)
        if f is not None:
            return f
    f = _gemm(act, pk.w_down, wp=pk.w_down_sk)
    if fused_proj and _tc_ok(attn, pk.w_o, gate, f):
        # o_proj with the gate and the parallel residual in its epilogue: f = attn_o * sigmoid(g) + f
        _lib.call('motif_b200_gemm_gate_residual', _lib.ptr(attn), attn.stride(0), _lib.ptr(pk.w_o),
                  pk.w_o.stride(0), _lib.ptr(gate), gate.stride(0), _lib.ptr(f), f.stride(0), _lib.ptr(f),
                  f.stride(0), M, d, d, dc, st)
        return f
    if a is None:
        a = _mm(attn, pk.w_o, wp=pk.w_o_sk)
    _lib.call('motif_b200_gate_residual', _lib.ptr(a), d, proj.data_ptr() + pk.off_g * proj.element_size(), N_in,
              _lib.ptr(f), d, _lib.ptr(f), d, M, d, dc, st)
    return f


def _key_bias(mask: torch.Tensor, dev) -> Optional[torch.Tensor]:
    """The model's `[B, cached + T]` key mask (`motif.py:592-602`) as the Chord kernels' additive
    key bias ([B, S] fp32): a bool keep-mask becomes 0 / -inf, a float mask is added as is
    (`chord_attn.py:347-356`).  None when it changes nothing (all True, or all zeros)."""
    if mask.dtype == torch.bool:
        if bool(mask.all()):
            return None
        kb = torch.zeros(mask.shape, dtype=torch.float32, device=dev)
        return kb.masked_fill_(~mask.to(dev), float('-inf'))
    kb = mask.to(device=dev, dtype=torch.float32).contiguous()
    return None if not bool(kb.any()) else kb


_LOG_TABLE: Dict[str, torch.Tensor] = {}


def _log_n(q_start: int, T: int, dev) -> torch.Tensor:
    """`log(q_start + 1 .. q_start + T)` from a cached table (`chord_attn.py:21-43,282`)."""
    key = str(dev)
    n = q_start + T
    table = _LOG_TABLE.get(key)
    if table is None or table.numel() < n:
        size = 1 << (max(n, 8192) - 1).bit_length()
        table = torch.log(torch.arange(1, size + 1, device=dev, dtype=torch.float32))
        _LOG_TABLE[key] = table
    return table[q_start:q_start + T].view(1, T)
