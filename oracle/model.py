"""Model-level CPU restatement of the reference's `MotifChordModel` torch path.

Test infrastructure only.  A functional restatement over a parameter dict whose
keys are the reference's `state_dict` names, with caches restated as small
classes that keep the reference's semantics:

* `forward` — `motif/model/motif.py:545-630`;
* `block_forward` — `motif/block/decoder.py:139-222`;
* `gdn_layer` — `motif/block/attention/gdn_attn.py:138-219`;
* `chord_layer` — `motif/block/attention/chord_attn.py:204-361` (eager body);
* `KVCache` — `motif/model/cache.py:73-252` (contiguous, append);
* `GDNCache` — `motif/model/cache.py:305-394`;
* `AttnRes` — `motif/model/cache.py:397-606`.
"""

from typing import List, Optional

import torch
import torch.nn.functional as F

from . import ops

EXPAND_V = 2.0
CONV = 4


class KVCache:
    """Key/value cache of a chord layer, `model/cache.py:73-215` (narrow layout)."""

    def __init__(self):
        self.k = None
        self.v = None
        self.length = 0

    def update(self, k_new, v_new):
        if self.k is None:
            self.k, self.v = k_new, v_new
        else:
            self.k = torch.cat([self.k, k_new], dim=2)
            self.v = torch.cat([self.v, v_new], dim=2)
        self.length = self.k.shape[2]
        return self.k, self.v


class GDNCache:
    """Recurrent + conv state of a GDN layer, `model/cache.py:305-356`."""

    def __init__(self):
        self.state = None
        self.conv = None
        self.length = 0

    def update(self, state, conv, steps):
        self.state = state
        self.conv = tuple(conv)
        self.length += steps


class AttnRes:
    """Attn-res history of one block, `model/cache.py:397-534`."""

    def __init__(self):
        self.blocks: List[torch.Tensor] = []
        self.partial = None
        self.seq_len = 0
        self.chunk_len = 0

    def init_embedding(self, x):
        q_len = x.shape[1]
        if len(self.blocks) == 0:
            self.seq_len = q_len
        else:
            self.seq_len += q_len
            self.partial = None
        self.blocks = [x]
        self.chunk_len = q_len

    def aligned(self):
        q_len = self.chunk_len if self.chunk_len > 0 else min(e.shape[1] for e in self.blocks)
        return [e if e.shape[1] == q_len else e[:, max(e.shape[1] - q_len, 0):] for e in self.blocks]

    def update_increment(self, f_h):
        self.blocks.append(f_h)
        if self.partial is None:
            self.partial = f_h
        elif self.partial.shape[1] == f_h.shape[1]:
            self.partial = self.partial + f_h
        else:
            self.partial = torch.cat([self.partial, f_h], dim=1)
        self.seq_len = max(self.seq_len, f_h.shape[1])


class BlockCache:
    def __init__(self, block):
        self.attn_res = AttnRes()
        self.attn = [KVCache() if t == 'chord' else GDNCache() for t in block]


class ModelCache:
    def __init__(self, cfg):
        self.blocks = [BlockCache(cfg.block) for _ in range(cfg.block_n)]

    @property
    def seq_len(self):
        return self.blocks[0].attn_res.seq_len if self.blocks else 0


def _lin(x, w):
    return F.linear(x, w)


def gdn_layer(P, pre, x, cfg, cache: Optional[GDNCache]):
    """Gated delta-net attention, `block/attention/gdn_attn.py:138-219`."""
    B, L, _ = x.shape
    H = cfg.num_heads
    dk = cfg.head_k_dim or (cfg.model_dim // cfg.num_heads)
    dv = int(dk * EXPAND_V)
    conv = cache.conv if (cache is not None and cache.conv is not None) else (None, None, None)
    S0 = cache.state if cache is not None else None
    q, cq = ops.causal_conv_silu(_lin(x, P[pre + 'q_proj.weight']), P[pre + 'q_conv.weight'], conv[0])
    k, ck = ops.causal_conv_silu(_lin(x, P[pre + 'k_proj.weight']), P[pre + 'k_conv.weight'], conv[1])
    v, cv = ops.causal_conv_silu(_lin(x, P[pre + 'v_proj.weight']), P[pre + 'v_conv.weight'], conv[2])
    q = q.view(B, L, H, dk).transpose(1, 2)
    k = k.view(B, L, H, dk).transpose(1, 2)
    v = v.view(B, L, H, dv).transpose(1, 2)
    q = F.normalize(q, dim=-1) * (dk ** -0.5)
    k = F.normalize(k, dim=-1)
    beta = torch.sigmoid(_lin(x, P[pre + 'b_proj.weight'])).transpose(1, 2)
    g = -P[pre + 'A_log'].exp() * F.softplus(_lin(x, P[pre + 'a_proj.weight']) + P[pre + 'dt_bias'])
    g = g.transpose(1, 2)
    qf, kf, vf, bf, gf = (t.float() for t in (q, k, v, beta, g))
    if L == 1:
        o, S = ops.recurrent_gated_delta_rule(qf, kf, vf, bf, gf, S0)
    else:
        o, S = ops.chunk_gated_delta_rule(qf, kf, vf, bf, gf, S0, 64)
    o = o.to(x.dtype).transpose(1, 2)
    gate = _lin(x, P[pre + 'g_proj.weight']).view(B, L, H, dv)
    o = ops.gated_rms_norm(torch.cat([o, gate.to(o.dtype)], dim=-1), P[pre + 'o_norm.weight']).reshape(B, L, -1)
    out = _lin(o, P[pre + 'o_proj.weight'])
    if cache is not None:
        cache.update(S, (cq, ck, cv), L)
    return out


def chord_layer(P, pre, x, cfg, cache: Optional[KVCache], position=0, mask=None):
    """Chord attention, eager body of `block/attention/chord_attn.py:204-361`."""
    B, L, d = x.shape
    H = cfg.num_heads
    Hkv = cfg.num_kv_heads if cfg.num_kv_heads is not None else H
    D = d // H
    G = torch.sigmoid(_lin(x, P[pre + 'g_proj.weight']))
    q = _lin(x, P[pre + 'q_proj.weight']).view(B, L, H, D).transpose(1, 2)
    k = _lin(x, P[pre + 'k_proj.weight']).view(B, L, Hkv, D).transpose(1, 2)
    v = _lin(x, P[pre + 'v_proj.weight']).view(B, L, Hkv, D).transpose(1, 2)
    q = ops.rms_norm(q, P[pre + 'q_norm.weight'])
    k = ops.rms_norm(k, P[pre + 'k_norm.weight'])
    q_start = int(position)
    if cache is not None:
        cached = cache.length
        if q_start == 0 and cached > 0:
            q_start = cached
        k, v = cache.update(k, v)
    S = k.shape[2]
    log_n = ops.log_n_table(q_start, L)
    alpha, beta, mu = ops.ggd_parameters(P[pre + 'theta_alpha'], P[pre + 'theta_beta'], P[pre + 'theta_mu'])
    ssmax = P[pre + 'ssmax_s']
    ssmax = ssmax.float() if ssmax.dtype in (torch.float16, torch.bfloat16) else ssmax
    if mask is None:
        out = ops.chord_attention(q, k, v, alpha, beta, mu, ssmax,
                                  log_n.view(1, L).expand(B, L), q_start, D ** -0.5)
    else:
        out = _chord_masked(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, D, mask)
    out = out.transpose(1, 2).contiguous().view(B, L, d)
    return _lin(out, P[pre + 'o_proj.weight']) * G


def _chord_masked(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, D, mask):
    """Eager chord with a keep/additive key mask, `chord_attn.py:316-361`."""
    B, H, L, _ = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    grp = H // Hkv
    if grp > 1:
        k = k[:, :, None].expand(B, Hkv, grp, S, D).reshape(B, H, S, D)
        v = v[:, :, None].expand(B, Hkv, grp, S, D).reshape(B, H, S, D)
    scores = (q @ k.transpose(-2, -1)) * D ** -0.5
    ld = torch.float32 if scores.dtype in (torch.float16, torch.bfloat16) else scores.dtype
    bias = ops.ggd_bias(alpha, beta, mu, L, S, q_start, ld)
    logits = scores.to(ld) + bias.unsqueeze(0)
    logits = logits * (ssmax.view(1, -1, 1, 1) * log_n.view(1, 1, L, 1).to(ld))
    logits = logits.clamp_min(torch.finfo(ld).min / 4)
    qp = torch.arange(L) + q_start
    kp = torch.arange(S)
    logits = logits.masked_fill(kp[None, :] > qp[:, None], float('-inf'))
    if mask.dtype == torch.bool:
        keep = mask
        if keep.dim() == 2:
            keep = keep[:, None, None, :]
        elif keep.dim() == 3:
            keep = keep[:, None]
        logits = logits.masked_fill(~keep, float('-inf'))
    else:
        logits = logits + mask
    attn = torch.softmax(logits, dim=-1)
    return attn.to(v.dtype) @ v


def block_forward(P, b, x, cfg, bc: BlockCache, position=0, mask=None):
    """`DecoderBlock.forward`, `block/decoder.py:139-222`."""
    ar = bc.attn_res
    ar.init_embedding(x)
    for i, typ in enumerate(cfg.block):
        pre = f'blocks.{b}.features.{i}.'
        srcs = ar.aligned()
        if len(srcs) == 1:
            h = srcs[0]
        else:
            h = ops.attn_res(srcs, P[f'blocks.{b}.pseudo_queries.{i}'],
                             P[f'blocks.{b}.attn_res_norms.{i}.weight'])
        a_in = ops.rms_norm(h, P[pre + 'attn_norm.weight'])
        if typ == 'chord':
            attn_out = chord_layer(P, pre + 'attn.', a_in, cfg, bc.attn[i], position, mask)
        else:
            attn_out = gdn_layer(P, pre + 'attn.', a_in, cfg, bc.attn[i])
        m_in = ops.rms_norm(h, P[pre + 'mlp_norm.weight'])
        mlp_out = _lin(ops.swiglu(_lin(m_in, P[pre + 'mlp.gate_up_proj.weight'])), P[pre + 'mlp.down_proj.weight'])
        ar.update_increment(attn_out + mlp_out)
    return ar.partial if ar.partial is not None else x


@torch.no_grad()
def forward(P, cfg, input_ids, cache: Optional[ModelCache] = None, position=None, mask=None):
    """`MotifChordModel.forward`, `model/motif.py:545-630` (no labels).

    Returns `(logits, hidden_states, cache)`.
    """
    if mask is not None:
        mask = mask[:, None, None, :]
    x = F.embedding(input_ids, P['embed.weight'])
    if cache is None:
        cache = ModelCache(cfg)
    for b in range(cfg.block_n):
        x = block_forward(P, b, x, cfg, cache.blocks[b], 0 if position is None else position, mask)
    x = ops.rms_norm(x, P['norm.weight'])
    logits = _lin(x, P['lm_head.weight'])
    return logits, x, cache


@torch.no_grad()
def greedy(P, cfg, input_ids, steps, mask=None):
    """Prefill then `steps` greedy tokens, `model/generate.py:138-171` + `motif.py:92-98`.  A key
    `mask` over the prompt is widened by one True column per token fed, as `Generation.step`
    does (`torch.cat` with a bool column: a float mask gains 1.0 columns by type promotion)."""
    logits, _, cache = forward(P, cfg, input_ids, mask=mask)
    tok = logits[:, -1].argmax(-1, keepdim=True)
    toks = [tok]
    margins = []
    for _ in range(steps - 1):
        if mask is not None:
            mask = torch.cat([mask, torch.ones_like(tok, dtype=torch.bool)], dim=1)
        logits, _, cache = forward(P, cfg, tok, cache, mask=mask)
        top2 = logits[:, -1].float().topk(2, dim=-1).values
        margins.append((top2[:, 0] - top2[:, 1]).min().item())
        tok = logits[:, -1].argmax(-1, keepdim=True)
        toks.append(tok)
    return torch.cat(toks, dim=1), margins


def params_from_module(module, dtype=None):
    """A `{name: tensor}` dict from any module with the reference's names (tied weights kept)."""
    sd = {k: v.detach().cpu() for k, v in module.state_dict().items()}
    if dtype is not None:
        sd = {k: v.to(dtype) for k, v in sd.items()}
    return sd


def param_shapes(cfg):
    """`{name: shape}` of every parameter `named_parameters()` yields for the reference
    model built from `cfg` (`model/motif.py:168-187`, `block/decoder.py:58-137`,
    `gdn_attn.py:76-106`, `chord_attn.py:97-116`, `block/mlp.py:42-53`)."""
    d, H = cfg.model_dim, cfg.num_heads
    Hkv = cfg.num_kv_heads if cfg.num_kv_heads is not None else H
    D = d // H
    dk = cfg.head_k_dim or D
    dv = int(dk * EXPAND_V)
    hid = (int(d * 8 / 3) + 127) // 128 * 128
    s = {'embed.weight': (cfg.vocab_size, d), 'norm.weight': (d,)}
    if not cfg.tied_weight:
        s['lm_head.weight'] = (cfg.vocab_size, d)
    for b in range(cfg.block_n):
        for i, typ in enumerate(cfg.block):
            pre = f'blocks.{b}.features.{i}.'
            s[pre + 'attn_norm.weight'] = (d,)
            s[pre + 'mlp_norm.weight'] = (d,)
            s[pre + 'mlp.gate_up_proj.weight'] = (2 * hid, d)
            s[pre + 'mlp.down_proj.weight'] = (d, hid)
            a = pre + 'attn.'
            if typ == 'chord':
                s.update({a + 'q_proj.weight': (d, d), a + 'k_proj.weight': (Hkv * D, d),
                          a + 'v_proj.weight': (Hkv * D, d), a + 'o_proj.weight': (d, d),
                          a + 'g_proj.weight': (d, d), a + 'q_norm.weight': (D,),
                          a + 'k_norm.weight': (D,), a + 'theta_alpha': (H,),
                          a + 'theta_beta': (H,), a + 'theta_mu': (H,), a + 'ssmax_s': (H,)})
            else:
                s.update({a + 'q_proj.weight': (H * dk, d), a + 'k_proj.weight': (H * dk, d),
                          a + 'v_proj.weight': (H * dv, d), a + 'a_proj.weight': (H, d),
                          a + 'b_proj.weight': (H, d), a + 'g_proj.weight': (H * dv, d),
                          a + 'o_proj.weight': (d, H * dv),
                          a + 'q_conv.weight': (H * dk, 1, CONV), a + 'k_conv.weight': (H * dk, 1, CONV),
                          a + 'v_conv.weight': (H * dv, 1, CONV), a + 'A_log': (H,),
                          a + 'dt_bias': (H,), a + 'o_norm.weight': (dv,)})
            s[f'blocks.{b}.pseudo_queries.{i}'] = (d,)
            s[f'blocks.{b}.attn_res_norms.{i}.weight'] = (d,)
    return s


def make_params(cfg, seed=0, norm_jitter=0.0, dtype=torch.float32):
    """Seeded parameters by name (same values `motif_b200.init.init_params` writes)."""
    from motif_b200.init import init_tensors
    P = init_tensors(param_shapes(cfg), seed, norm_jitter)
    P = {k: v.to(dtype) for k, v in P.items()}
    P['lm_head.weight'] = P['embed.weight'] if cfg.tied_weight else P['lm_head.weight']
    return P
