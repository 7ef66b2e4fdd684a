"""Drop-in replacements for the reference's `motif.ops` functions and modules.

Same names, argument meanings, return values and exception types as
`motif/ops/__init__.py:1-10` (plus `apply_block_attn_res`, `motif/ops/attn_res.py:596`),
computed by the sm_100a kernels of `libmotif_b200.so`.  The delta rule, Chord attention and
the attn-res read take gradients the way the reference's do (autograd Functions over the
backward kernels, `motif_b200.autograd`); the norm / SwiGLU modules are forward-only and raise
for inputs that require a gradient.  CPU tensors raise `ValueError`; there is no eager
fallback.
"""

from typing import Optional, Sequence

import torch
import torch.nn as nn

from . import _lib
from .autograd import AttnResFunction, ChordAttentionFunction, GatedDeltaRuleFunction, needs_grad
from .sampler import Sampler, make_sampler  # noqa: F401  (install targets)

__all__ = [
    'RMSNorm', 'GatedRMSNorm', 'SwiGLU', 'apply_chord_attention', 'HAS_TRITON',
    'recurrent_gated_delta_rule', 'chunk_gated_delta_rule', 'chunk_gated_delta_rule_triton',
    'attn_res_block', 'can_use_triton_attn_res', 'apply_block_attn_res', 'MAX_SRC',
]

# The reference's switch for its fused-kernel path.  Here the fused path is always the
# sm_100a CUDA library (there is no Triton), so callers that test it take the fast path.
HAS_TRITON = True
MAX_SRC = 8  # sources one fused attn-res read accepts (the reference unrolls 4)


def _cuda(name, t):
    if not isinstance(t, torch.Tensor):
        raise ValueError(f'{name} must be a tensor')
    if not t.is_cuda:
        raise ValueError(f'{name} must live on CUDA')
    return t


def _no_grad(*ts):
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in ts):
        raise NotImplementedError('motif_b200 ops are forward-only (no autograd)')


def _last_contig(t):
    return t if t.stride(-1) == 1 else t.contiguous()


# ------------------------------------------------------------------- gated delta rule
def _delta_args(q, k, v, beta, g, S):
    for n, t in (('q', q), ('k', k), ('v', v), ('beta', beta), ('g', g)):
        _cuda(n, t)
    if q.dim() != 4 or k.shape != q.shape or v.dim() != 4 or v.shape[:3] != q.shape[:3]:
        raise ValueError(f'q/k [B,H,L,Dk] and v [B,H,L,Dv] expected, got {tuple(q.shape)}, {tuple(k.shape)}, '
                         f'{tuple(v.shape)}')
    B, H, L, Dk = q.shape
    Dv = v.shape[-1]
    if beta.shape != (B, H, L) or g.shape != (B, H, L):
        raise ValueError(f'beta / g must be [B,H,L] = {(B, H, L)}')
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError('q / k / v must share one dtype')
    q, k, v = (t if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 else t.contiguous() for t in (q, k, v))
    beta = beta.float()
    g = g.float()
    if S is not None:
        _cuda('S', S)
        if S.shape != (B, H, Dk, Dv):
            raise ValueError(f'S must be [B,H,Dk,Dv] = {(B, H, Dk, Dv)}, got {tuple(S.shape)}')
        S = S.float().contiguous()
    strides = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3]]
    return q, k, v, beta, g, S, (B, H, L, Dk, Dv), strides


def _delta_call(entry, q, k, v, beta, g, S):
    q, k, v, beta, g, S, (B, H, L, Dk, Dv), strides = _delta_args(q, k, v, beta, g, S)
    o = torch.empty(B, H, L, Dv, dtype=q.dtype, device=q.device)
    S_out = torch.empty(B, H, Dk, Dv, dtype=torch.float32, device=q.device)
    strides += [*o.stride()[:3], *beta.stride(), *g.stride()]
    dc = _lib.dtype_code(q.dtype)
    if entry == 'motif_b200_gdn_chunk':
        # the two-kernel path (parallel UT transform, then the state scan) when it exists for
        # this dtype / shape; its workspace comes from torch's caching allocator
        ws_bytes = _lib.load().motif_b200_gdn_chunk_workspace_bytes(B, H, L, Dk, Dv, dc)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes > 0 else None
        _lib.call('motif_b200_gdn_chunk_gated_ws', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(beta),
                  _lib.ptr(g), _lib.ptr(S), _lib.ptr(S_out), _lib.ptr(o), B, H, L, Dk, Dv, _lib.i64_array(strides),
                  None, 0, 0, None, 0.0, dc, _lib.ptr(ws), max(ws_bytes, 0), _lib.stream_ptr(q.device))
        return o, S_out.to(q.dtype)
    _lib.call(entry, _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(beta), _lib.ptr(g), _lib.ptr(S),
              _lib.ptr(S_out), _lib.ptr(o), B, H, L, Dk, Dv, _lib.i64_array(strides), dc,
              _lib.stream_ptr(q.device))
    return o, S_out.to(q.dtype)


def _delta_dispatch(entry, q, k, v, beta, g, S):
    """The forward kernel, under the autograd Function when an input requires a gradient."""
    if needs_grad(q, k, v, beta, g, S):
        _delta_args(q, k, v, beta, g, S)  # validate before recording the graph
        return GatedDeltaRuleFunction.apply(lambda *a: _delta_call(entry, *a), q, k, v, beta, g, S)
    return _delta_call(entry, q, k, v, beta, g, S)


def recurrent_gated_delta_rule(q, k, v, beta, g, S=None):
    """Token-by-token gated delta rule (`motif/ops/gated_deltanet.py:26-59`).

    Returns `(o [B,H,L,Dv], S [B,H,Dk,Dv])`; the state is carried in fp32 inside the kernel
    and returned in q's dtype, as the reference returns it.
    """
    return _delta_dispatch('motif_b200_gdn_recurrent', q, k, v, beta, g, S)


def chunk_gated_delta_rule(q, k, v, beta, g, S=None, chunk_size=64):
    """Chunked gated delta rule (`motif/ops/gated_deltanet.py:287-321`).

    The fused kernel always uses 64-token chunks; `chunk_size` changes only rounding in the
    reference, never the result, and is validated but not otherwise used.
    """
    if int(chunk_size) < 1:
        raise ValueError(f'chunk_size must be positive, got {chunk_size}')
    return _delta_dispatch('motif_b200_gdn_chunk', q, k, v, beta, g, S)


def chunk_gated_delta_rule_triton(q, k, v, beta, g, S=None, chunk_size=64):
    """`chunk_gated_delta_rule_triton` (`motif/ops/gated_deltanet.py:796-834`), same kernel."""
    if int(chunk_size) < 16:
        raise NotImplementedError('chunk_size must be >= 16 (the K-dimension lower bound of tl.dot)')
    return _delta_dispatch('motif_b200_gdn_chunk', q, k, v, beta, g, S)


# -------------------------------------------------------------------- chord attention
def _check_chord(q, k, v, log_n):
    """`_check_tensors` (`motif/ops/chord_attention.py:966-1011`)."""
    for name, t in (('q', q), ('k', k), ('v', v)):
        if not t.is_cuda:
            raise ValueError(f'{name} must live on CUDA')
        if t.dim() != 4:
            raise ValueError(f'{name} must be 4-D [B, H, L, D], got {tuple(t.shape)}')
        if t.stride(-1) != 1:
            raise ValueError(f'{name} must be contiguous along the last dimension (stride(-1) == 1)')
        if t.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError(f'{name} has unsupported dtype {t.dtype} (only fp16 / bf16 / fp32)')
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError('q / k / v must all have the same dtype')
    if k.shape != v.shape:
        raise ValueError(f'k / v must have the same shape, got {tuple(k.shape)} vs {tuple(v.shape)}')
    B, H, L, D = q.shape
    Bk, Hkv, S, Dk = k.shape
    if B != Bk or D != Dk:
        raise ValueError(f'q {tuple(q.shape)} and k {tuple(k.shape)} disagree on B / D')
    if H % Hkv != 0:
        raise ValueError(f'num_heads {H} must be divisible by num_kv_heads {Hkv}')
    if D < 16:
        raise ValueError(f'head_dim {D} is too small (tl.dot requires >= 16)')
    if log_n.shape != (B, L):
        raise ValueError(f'log_n must be [B, q_len] = {(B, L)}, got {tuple(log_n.shape)}')
    if log_n.dtype != torch.float32:
        raise ValueError(f'log_n must be fp32, got {log_n.dtype}')
    if log_n.stride(-1) != 1:
        raise ValueError('log_n must be contiguous along the last dimension')
    return B, H, L, D, Hkv, S


def _check_params(alpha, beta, mu, ssmax, num_heads):
    """`_check_params` (`motif/ops/chord_attention.py:1448-1472`)."""
    for name, t in (('alpha', alpha), ('beta', beta), ('mu', mu), ('ssmax', ssmax)):
        if not t.is_cuda:
            raise ValueError(f'{name} must live on CUDA')
        if t.dtype != torch.float32:
            raise ValueError(f'{name} must be fp32, got {t.dtype}')
        if t.shape != (num_heads,):
            raise ValueError(f'{name} must be [{num_heads}], got {tuple(t.shape)}')
        if not t.is_contiguous():
            raise ValueError(f'{name} must be contiguous')


def apply_chord_attention(q, k, v, alpha, beta, mu, ssmax, log_n, q_start: Optional[int] = None,
                          softmax_scale: Optional[float] = None, eps: float = 1e-5) -> torch.Tensor:
    """Chord attention forward (`motif/ops/chord_attention.py:1557-1625`)."""
    B, H, L, D, Hkv, S = _check_chord(q, k, v, log_n)
    _check_params(alpha, beta, mu, ssmax, H)
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if q_start is None:
        q_start = S - L
    q_start = int(q_start)
    if q_start < 0:
        raise ValueError(f'q_start must not be negative, got {q_start}')
    if needs_grad(q, k, v, alpha, beta, mu, ssmax):
        return ChordAttentionFunction.apply(_chord_forward, q, k, v, alpha, beta, mu, ssmax, log_n, q_start,
                                            float(softmax_scale), float(eps))
    return _chord_forward(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, float(softmax_scale), float(eps))


def _chord_forward(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, softmax_scale, eps):
    B, H, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    out = torch.empty((B, H, L, D), dtype=q.dtype, device=q.device)
    if L == 0:
        return out
    strides = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3], *log_n.stride()]
    _lib.call('motif_b200_chord_attention', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(alpha),
              _lib.ptr(beta), _lib.ptr(mu), _lib.ptr(ssmax), _lib.ptr(log_n), _lib.ptr(out), B, H, Hkv, L, S, D,
              q_start, float(softmax_scale), float(eps), _lib.i64_array(strides), _lib.dtype_code(q.dtype),
              None, 0, _lib.stream_ptr(q.device))
    return out


# --------------------------------------------------------------------------- attn-res
def can_use_triton_attn_res(sources: Sequence[torch.Tensor], weight: Optional[torch.Tensor],
                            query: torch.Tensor) -> bool:
    """Eligibility of the fused read (`motif/ops/attn_res.py:466-515`), widened to 8 sources."""
    if weight is None or not (1 <= len(sources) <= MAX_SRC):
        return False
    d = sources[0].shape[-1]
    dtype = sources[0].dtype
    if dtype not in (torch.float32, torch.float16, torch.bfloat16) or any(t.dtype != dtype for t in sources):
        return False
    if query.dim() != 1 or query.shape[0] != d or not query.is_cuda or weight.numel() != d or not weight.is_cuda:
        return False
    for t in sources:
        if not t.is_cuda or t.dim() != 3 or t.stride(-1) != 1 or t.shape[-1] != d or t.shape[:2] != sources[0].shape[:2]:
            return False
    return True


def attn_res_block(sources: Sequence[torch.Tensor], weight: torch.Tensor, query: torch.Tensor, eps: float,
                   block_t: int = 8) -> torch.Tensor:
    """Fused cross-block attention residual (`motif/ops/attn_res.py:518-540`)."""
    if not can_use_triton_attn_res(sources, weight, query):
        raise ValueError('attn_res_block: unsupported sources / weight / query')
    if needs_grad(weight, query, *sources):
        return AttnResFunction.apply(_attn_res_forward, weight, query, float(eps), *sources)
    return _attn_res_forward(sources, weight, query, eps)


def _attn_res_forward(sources, weight, query, eps):
    sources = [_last_contig(s) for s in sources]
    B, T, D = sources[0].shape
    dt = sources[0].dtype
    out = torch.empty((B, T, D), dtype=dt, device=sources[0].device)
    w = weight.to(dt).contiguous()
    qv = query.to(dt).contiguous()
    strides = []
    for s in sources:
        strides += [s.stride(0), s.stride(1)]
    _lib.call('motif_b200_attn_res', _lib.ptr_array([s.data_ptr() for s in sources]), len(sources),
              _lib.i64_array(strides), _lib.ptr(w), _lib.ptr(qv), _lib.ptr(out), out.stride(0), out.stride(1),
              B, T, D, float(eps), _lib.dtype_code(dt), _lib.stream_ptr(out.device))
    return out


def apply_block_attn_res(cache, query: torch.Tensor, norm) -> torch.Tensor:
    """Cross-block attention residual over a cache's aligned history (`attn_res.py:596-622`)."""
    sources = cache.aligned_values()
    if len(sources) == 1:
        return sources[0]
    return attn_res_block(sources, norm.weight, query, norm.eps)


# ------------------------------------------------------------------ norms / activation
class RMSNorm(nn.Module):
    """`RMSNorm` (`motif/ops/rms_norm.py:419-486`) on the CUDA kernel; parameter `weight`."""

    def __init__(self, dim, eps=1e-6, elementwise_affine=True, use_triton=True):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(dim))
        else:
            self.register_parameter('weight', None)
        self.use_triton = bool(use_triton)

    def forward(self, x):
        _cuda('x', x)
        _no_grad(x, self.weight)
        N = x.shape[-1]
        x2 = x.reshape(-1, N)
        x2 = _last_contig(x2)
        y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
        w = None if self.weight is None else self.weight.to(x.dtype).contiguous()
        _lib.call('motif_b200_rms_norm', _lib.ptr(x2), _lib.ptr(w), _lib.ptr(y), x2.shape[0], N, x2.stride(0),
                  y.stride(0), float(self.eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
        return y.reshape(x.shape)


class GatedRMSNorm(nn.Module):
    """`GatedRMSNorm` (`motif/ops/rms_norm.py:489-553`): rmsnorm(values) * w * silu(gate)."""

    def __init__(self, dim, eps=1e-6, elementwise_affine=True, use_triton=True):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(dim))
        else:
            self.register_parameter('weight', None)
        self.use_triton = bool(use_triton)

    def forward(self, x):
        _cuda('x', x)
        _no_grad(x, self.weight)
        if x.shape[-1] != 2 * self.dim:
            raise ValueError(f'GatedRMSNorm expects last dim {2 * self.dim}, got {x.shape[-1]}')
        x2 = _last_contig(x.reshape(-1, 2 * self.dim))
        y = torch.empty((x2.shape[0], self.dim), dtype=x.dtype, device=x.device)
        w = None if self.weight is None else self.weight.to(x.dtype).contiguous()
        _lib.call('motif_b200_gated_rms_norm', _lib.ptr(x2), _lib.ptr(w), _lib.ptr(y), x2.shape[0], self.dim,
                  x2.stride(0), y.stride(0), float(self.eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
        return y.reshape(*x.shape[:-1], self.dim)


class SwiGLU(nn.Module):
    """`SwiGLU` activation (`motif/ops/swiglu.py:184-253`): values * silu(gate), values first."""

    def __init__(self, dim: int = -1, use_triton: bool = True):
        super().__init__()
        self.dim = dim
        self.use_triton = bool(use_triton)

    def forward(self, x):
        _cuda('x', x)
        _no_grad(x)
        if self.dim not in (-1, x.dim() - 1):
            x = x.movedim(self.dim, -1)
            return self.forward(x).movedim(-1, self.dim)
        if x.shape[-1] % 2:
            raise ValueError('SwiGLU needs an even split dimension')
        n = x.shape[-1] // 2
        x2 = _last_contig(x.reshape(-1, 2 * n))
        y = torch.empty((x2.shape[0], n), dtype=x.dtype, device=x.device)
        _lib.call('motif_b200_swiglu', _lib.ptr(x2), _lib.ptr(y), x2.shape[0], n, x2.stride(0), y.stride(0),
                  _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device))
        return y.reshape(*x.shape[:-1], n)
