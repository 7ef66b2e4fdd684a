"""Autograd for the three hot-path ops: their forwards run the inference kernels, their
backwards the kernels of `csrc/backward.cu` (fp32 arithmetic on CUDA cores).

The reference wraps the same ops in `torch.autograd.Function`s (`_TritonChordFunction`,
`motif/ops/chord_attention.py:1476-1554`; `_AttnResFunction`, `motif/ops/attn_res.py:367-463`;
`_PrepareChunksFunction` / `_FusedScanFunction`, `motif/ops/gated_deltanet.py:107-284,697-765`),
and `motif_b200.ops` routes to these when an input requires a gradient, exactly where the
reference routes to its Functions.  Gradients come back in each input's dtype; the GGD
parameter gradients are accumulated in fp64 and returned in fp32 like the reference's.
"""

import torch

from . import _lib


def needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in ts)


def _c(t):
    return t if t.stride(-1) == 1 else t.contiguous()


class ChordAttentionFunction(torch.autograd.Function):
    """Chord attention with the Chord backward kernels (`motif_b200_chord_backward`): dq, dk, dv
    and the gradients of alpha, beta, mu and ssmax (log_n, q_start, the scale and eps get none,
    as in the reference)."""

    @staticmethod
    def forward(ctx, forward_fn, q, k, v, alpha, beta, mu, ssmax, log_n, q_start, scale, eps):
        with torch.no_grad():
            out = forward_fn(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, scale, eps)
        ctx.save_for_backward(q, k, v, out, alpha, beta, mu, ssmax, log_n)
        ctx.q_start, ctx.scale, ctx.eps = q_start, scale, eps
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, alpha, beta, mu, ssmax, log_n = ctx.saved_tensors
        B, H, L, D = q.shape
        Hkv, S = k.shape[1], k.shape[2]
        dout = _c(dout.to(q.dtype))
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.zeros((B, Hkv, S, D), dtype=q.dtype, device=q.device)
        dv = torch.zeros((B, Hkv, S, D), dtype=q.dtype, device=q.device)
        tq = max(1, (L + 31) // 32)
        part = torch.zeros((B, H, tq, 4), dtype=torch.float64, device=q.device)
        ws = torch.empty(max(16, _lib.load().motif_b200_chord_backward_workspace_bytes(B, H, L)), dtype=torch.uint8,
                         device=q.device)
        strides = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3], *dout.stride()[:3],
                   *dq.stride()[:3], *dk.stride()[:3], *dv.stride()[:3], *log_n.stride()]
        if L > 0 and S > 0:
            _lib.call('motif_b200_chord_backward', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(out),
                      _lib.ptr(dout), _lib.ptr(alpha), _lib.ptr(beta), _lib.ptr(mu), _lib.ptr(ssmax),
                      _lib.ptr(log_n), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), B, H, Hkv, L, S, D, ctx.q_start,
                      float(ctx.scale), float(ctx.eps), _lib.i64_array(strides), _lib.ptr(ws), ws.numel(),
                      _lib.ptr(part), _lib.dtype_code(q.dtype), _lib.stream_ptr(q.device))
        else:
            dq.zero_()
        g4 = part.sum(dim=(0, 2)).float()  # [H, 4]: alpha, beta, mu, ssmax
        need = ctx.needs_input_grad
        return (None,
                dq if need[1] else None, dk if need[2] else None, dv if need[3] else None,
                g4[:, 0].contiguous() if need[4] else None, g4[:, 1].contiguous() if need[5] else None,
                g4[:, 2].contiguous() if need[6] else None, g4[:, 3].contiguous() if need[7] else None,
                None, None, None, None)


class AttnResFunction(torch.autograd.Function):
    """The block attention residual with `motif_b200_attn_res_backward`: gradients of every
    source, of the pseudo-query and of the norm weight."""

    @staticmethod
    def forward(ctx, forward_fn, weight, query, eps, *sources):
        with torch.no_grad():
            out = forward_fn(list(sources), weight, query, eps)
        ctx.save_for_backward(weight, query, *sources)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, dh):
        weight, query, *sources = ctx.saved_tensors
        dt = sources[0].dtype
        B, T, D = sources[0].shape
        srcs = [s.contiguous() for s in sources]
        w = weight.to(dt).contiguous()
        qv = query.to(dt).contiguous()
        dh = dh.to(dt).contiguous()
        dsrc = [torch.empty_like(s) for s in srcs]
        rows = B * T
        parts = max(1, min(148 * 8, (rows + 7) // 8))
        z = torch.zeros((parts, D), dtype=torch.float32, device=dh.device)
        if rows > 0:
            _lib.call('motif_b200_attn_res_backward', _lib.ptr_array([s.data_ptr() for s in srcs]),
                      _lib.ptr_array([s.data_ptr() for s in dsrc]), len(srcs), rows, D, D, _lib.ptr(w), _lib.ptr(qv),
                      float(ctx.eps), _lib.ptr(dh), D, _lib.ptr(z), parts, _lib.dtype_code(dt),
                      _lib.stream_ptr(dh.device))
        Z = z.double().sum(0)
        need = ctx.needs_input_grad
        dw = (qv.double() * Z).to(weight.dtype) if need[1] else None
        dq = (w.double() * Z).to(query.dtype) if need[2] else None
        return (None, dw, dq, None, *[d if need[4 + i] else None for i, d in enumerate(dsrc)])


class GatedDeltaRuleFunction(torch.autograd.Function):
    """The gated delta rule (recurrent or chunked forward: the same function) with
    `motif_b200_gdn_backward`: gradients of q, k, v, beta, g and the initial state, from the
    gradients of the output and of the final state."""

    @staticmethod
    def forward(ctx, forward_fn, q, k, v, beta, g, S):
        with torch.no_grad():
            o, S_out = forward_fn(q, k, v, beta, g, S)
        ctx.save_for_backward(q, k, v, beta, g, S)
        ctx.has_state = S is not None
        return o, S_out

    @staticmethod
    def backward(ctx, do, dS_out):
        q, k, v, beta, g, S = ctx.saved_tensors
        B, H, L, Dk = q.shape
        Dv = v.shape[-1]
        f = lambda t: t.float().contiguous()  # noqa: E731
        q32, k32, v32, b32, g32 = f(q), f(k), f(v), f(beta), f(g)
        s32 = f(S) if S is not None else None
        do32 = f(do) if do is not None else torch.zeros((B, H, L, Dv), device=q.device)
        dS32 = f(dS_out) if dS_out is not None else None
        dq = torch.empty((B, H, L, Dk), device=q.device)
        dk = torch.empty_like(dq)
        dv = torch.empty((B, H, L, Dv), device=q.device)
        db = torch.empty((B, H, L), device=q.device)
        dg = torch.empty_like(db)
        dS0 = torch.empty((B, H, Dk, Dv), device=q.device) if S is not None else None
        ws = torch.empty(max(16, _lib.load().motif_b200_gdn_backward_workspace_bytes(B, H, L, Dk, Dv)),
                         dtype=torch.uint8, device=q.device)
        _lib.call('motif_b200_gdn_backward', _lib.ptr(q32), _lib.ptr(k32), _lib.ptr(v32), _lib.ptr(b32),
                  _lib.ptr(g32), _lib.ptr(s32), _lib.ptr(do32), _lib.ptr(dS32), _lib.ptr(dq), _lib.ptr(dk),
                  _lib.ptr(dv), _lib.ptr(db), _lib.ptr(dg), _lib.ptr(dS0), B, H, L, Dk, Dv, _lib.ptr(ws),
                  ws.numel(), _lib.stream_ptr(q.device))
        need = ctx.needs_input_grad
        return (None,
                dq.to(q.dtype) if need[1] else None, dk.to(k.dtype) if need[2] else None,
                dv.to(v.dtype) if need[3] else None, db.to(beta.dtype) if need[4] else None,
                dg.to(g.dtype) if need[5] else None,
                dS0.to(S.dtype) if (S is not None and need[6]) else None)
