"""Op-level CPU restatements of the reference's torch path (test infrastructure only).

Each function restates one reference function; the citation is in its docstring.
Dtype handling follows the reference line by line (which casts happen where), so
the same function serves as the fp32 oracle and as the bf16 oracle.
"""

import torch
import torch.nn.functional as F

NORM_EPS = 1e-6
GGD_EPS = 1e-5
_HALF = (torch.float16, torch.bfloat16)


# --------------------------------------------------------------------------- norms
def rms_norm(x, weight, eps=NORM_EPS):
    """Eager RMSNorm, `motif/ops/rms_norm.py:481-486`."""
    x_f = x.float()
    var = x_f.pow(2).mean(-1, keepdim=True)
    y = (x_f * torch.rsqrt(var + eps)).to(x.dtype)
    if weight is not None:
        y = y * weight
    return y


def gated_rms_norm(x, weight, eps=NORM_EPS):
    """Eager GatedRMSNorm over a `[..., 2N]` input, `motif/ops/rms_norm.py:547-553`."""
    n = x.shape[-1] // 2
    x_in, gate = x.split(n, dim=-1)
    x_f = x_in.float()
    var = x_f.pow(2).mean(-1, keepdim=True)
    y = (x_f * torch.rsqrt(var + eps)).to(x.dtype)
    if weight is not None:
        y = y * weight
    return y * F.silu(gate)


def swiglu(x):
    """`values * silu(gate)`, values first, `motif/ops/swiglu.py:252-253`."""
    out, gate = torch.split(x, x.size(-1) // 2, dim=-1)
    return out * F.silu(gate)


# ---------------------------------------------------------------------- delta rule
def recurrent_gated_delta_rule(q, k, v, beta, g, S=None):
    """Token-by-token gated delta rule, `motif/ops/gated_deltanet.py:26-59`."""
    B, H, L, Dk = q.shape
    Dv = v.shape[-1]
    if S is None:
        S = q.new_zeros(B, H, Dk, Dv)
    outs = []
    for t in range(L):
        S = S * g[:, :, t].exp()[..., None, None]
        kt, vt = k[:, :, t], v[:, :, t]
        bt = beta[:, :, t, None]
        v_old = (kt.unsqueeze(-2) @ S).squeeze(-2)
        delta = bt * (vt - v_old)
        S = S + kt.unsqueeze(-1) * delta.unsqueeze(-2)
        outs.append((q[:, :, t].unsqueeze(-2) @ S).squeeze(-2))
    return torch.stack(outs, dim=2), S


def prepare_chunks(q, k, v, beta, g, C):
    """Chunk padding and the WY/UT factors, `motif/ops/gated_deltanet.py:137-177`.

    Returns `(q, k, gamma, decay_mask, W, U, N, pad)` with the chunked `[B,H,N,C,.]`
    views; `gamma` is the within-chunk cumulative log decay.
    """
    B, H, L, Dk = q.shape
    Dv = v.shape[-1]
    pad = (C - L % C) % C
    if pad:
        q, k, v = (F.pad(t, (0, 0, 0, pad)) for t in (q, k, v))
        beta, g = (F.pad(t, (0, pad)) for t in (beta, g))
    N = (L + pad) // C
    beta_c = beta.reshape(B, H, N, C)
    k = k.reshape(B, H, N, C, Dk).contiguous()
    vc = v.reshape(B, H, N, C, Dv).contiguous()
    v_beta = vc * beta_c[..., None]
    k_beta = k * beta_c[..., None]
    g = g.reshape(B, H, N, C).contiguous().cumsum(-1)
    tril = torch.tril(torch.ones(C, C, dtype=torch.bool))
    strict = torch.tril(torch.ones(C, C, dtype=torch.bool), diagonal=-1)
    decay_mask = (g[..., :, None] - g[..., None, :]).masked_fill(~tril, float('-inf')).exp()
    G1 = k_beta @ k.transpose(-1, -2)
    A = (-G1 * decay_mask).masked_fill(~strict, 0.0)
    M = torch.eye(C, dtype=A.dtype) - A
    M_inv = torch.linalg.solve_triangular(
        M, torch.eye(C, dtype=A.dtype).expand_as(A), upper=False, unitriangular=True)
    W = M_inv @ (k_beta * g.exp()[..., None])
    U = M_inv @ v_beta
    q = q.reshape(B, H, N, C, Dk).contiguous()
    return q, k, g, decay_mask, W, U, N, pad


def chunk_gated_delta_rule(q, k, v, beta, g, S=None, chunk_size=64):
    """Chunked gated delta rule, `motif/ops/gated_deltanet.py:287-321`."""
    B, H, L, _ = q.shape
    Dk, Dv = q.shape[-1], v.shape[-1]
    qc, kc, gc, decay, W, U, N, _ = prepare_chunks(q, k, v, beta, g, chunk_size)
    if S is None:
        S = qc.new_zeros(B, H, Dk, Dv)
    o = torch.empty(B, H, N, chunk_size, Dv, dtype=qc.dtype)
    for i in range(N):
        qi, ki, gi = qc[:, :, i], kc[:, :, i], gc[:, :, i]
        attn = (qi @ ki.transpose(-1, -2)) * decay[:, :, i]
        u = U[:, :, i] - W[:, :, i] @ S
        o_inter = (qi * gi.exp()[..., None]) @ S
        o[:, :, i] = o_inter + attn @ u
        S = S * gi[:, :, -1].exp()[..., None, None] + \
            (ki * (gi[:, :, -1:] - gi).exp()[..., None]).transpose(-1, -2) @ u
    return o.reshape(B, H, N * chunk_size, Dv)[:, :, :L], S


# ----------------------------------------------------------------- chord attention
def ggd_parameters(theta_alpha, theta_beta, theta_mu):
    """`alpha = e^ta`, `beta = tb`, `mu = e^tm - e^-tm`, `block/attention/chord_attn.py:126-138`."""
    ta, tb, tm = (t.float() if t.dtype in _HALF else t for t in (theta_alpha, theta_beta, theta_mu))
    return torch.exp(ta), tb, torch.exp(tm) - torch.exp(-tm)


def ggd_bias(alpha, beta, mu, q_len, kv_len, q_start, dtype=torch.float32):
    """`[H, L, S]` bias `-alpha (|k - q - mu| + eps)^beta`, `chord_attn.py:140-176`."""
    cd = alpha.dtype
    q_pos = torch.arange(q_len, dtype=cd) + float(q_start)
    k_pos = torch.arange(kv_len, dtype=cd)
    d = k_pos[None, :] - q_pos[:, None]
    b = torch.abs(d[None] - mu[:, None, None]) + GGD_EPS
    return (-alpha[:, None, None] * b ** beta[:, None, None]).to(dtype)


def chord_attention(q, k, v, alpha, beta, mu, ssmax, log_n, q_start=None,
                    softmax_scale=None, eps=GGD_EPS):
    """Biased causal softmax attention, the eager body of `chord_attn.py:316-361`.

    Same arguments as `apply_chord_attention` (`ops/chord_attention.py:1557-1569`):
    q `[B,H,L,D]`, k/v `[B,Hkv,S,D]`, per-head fp32 alpha/beta/mu/ssmax `[H]`,
    log_n `[B,L]` fp32.  Returns `[B,H,L,D]` in q's dtype (attention mask: none).
    """
    B, H, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    if q_start is None:
        q_start = S - L
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    group = H // Hkv
    if group > 1:
        k = k[:, :, None].expand(B, Hkv, group, S, D).reshape(B, H, S, D)
        v = v[:, :, None].expand(B, Hkv, group, S, D).reshape(B, H, S, D)
    scores = (q @ k.transpose(-2, -1)) * softmax_scale
    logit_dtype = torch.float32 if scores.dtype in _HALF else scores.dtype
    cd = alpha.dtype
    q_pos = torch.arange(L, dtype=cd) + float(q_start)
    k_pos = torch.arange(S, dtype=cd)
    d = k_pos[None, :] - q_pos[:, None]
    bias = (-alpha[:, None, None] * (torch.abs(d[None] - mu[:, None, None]) + eps)
            ** beta[:, None, None]).to(logit_dtype)
    logits = scores.to(logit_dtype) + bias.unsqueeze(0)
    logits = logits * (ssmax.to(logit_dtype).view(1, -1, 1, 1)
                       * log_n.view(B, 1, L, 1).to(logit_dtype))
    logits = logits.clamp_min(torch.finfo(logit_dtype).min / 4)
    qp = torch.arange(L) + int(q_start)
    kp = torch.arange(S)
    logits = logits.masked_fill(kp[None, :] > qp[:, None], float('-inf'))
    attn = torch.softmax(logits, dim=-1)
    return attn.to(v.dtype) @ v


def log_n_table(q_start, q_len):
    """`log(q_start + 1 .. q_start + q_len)` fp32, `chord_attn.py:21-43,282`."""
    n = q_start + q_len
    size = max(n, 8192)
    size = 1 << (size - 1).bit_length()
    table = torch.log(torch.arange(1, size + 1, dtype=torch.float32))
    return table[q_start:q_start + q_len]


# ------------------------------------------------------------------------ attn-res
def attn_res(sources, query, norm_weight, eps=NORM_EPS):
    """Depth softmax over sources, the eager path of `motif/ops/attn_res.py:588-593`."""
    V = torch.stack(list(sources), dim=0)
    K = rms_norm(V, norm_weight, eps)
    logits = torch.einsum('d, n b t d -> n b t', query, K)
    alpha = logits.softmax(dim=0)
    return torch.einsum('n b t, n b t d -> b t d', alpha, V)


# --------------------------------------------------------------------- GDN helpers
def causal_conv_silu(x, weight, cache):
    """Depthwise causal conv (k=4) + SiLU with a carried state, `gdn_attn.py:116-136`.

    x `[B,L,D]`, weight `[D,1,K]`, cache `[B,D,K-1]` or None.
    Returns `(y [B,L,D], new_cache [B,D,K-1])`.
    """
    B, _, D = x.shape
    K = weight.shape[-1]
    xt = x.transpose(1, 2)
    if cache is None:
        cache = xt.new_zeros(B, D, K - 1)
    xc = torch.cat([cache, xt], dim=-1)
    new_cache = xc[..., -(K - 1):]
    y = F.conv1d(xc, weight, groups=D)
    return F.silu(y).transpose(1, 2), new_cache
