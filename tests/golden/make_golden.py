"""Generate the golden vectors that pin the CPU oracle to the live reference.

Run once in a container where the reference source tree is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference <ref-src-dir>

It imports the reference's own `motif` package (its pure-torch CPU path), runs it on
seeded inputs and writes `tests/golden/*.pt`.  Nothing at test time reads the
reference; the tests only compare the oracle with these files.

Models are built from the reference's `MotifChordModel` and initialised with
`motif_b200.init.init_params` (seeded, name-driven), so the oracle / CUDA model can
rebuild bit-identical weights from the same seed without storing them.
"""

import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

# Small model used for full-logit fixtures (GQA, 2 blocks of 3 GDN + 1 Chord).
SMALL = dict(vocab_size=512, model_dim=64, num_heads=4, num_kv_heads=2, head_k_dim=16,
             block=('gdn', 'gdn', 'gdn', 'chord'), block_n=2)
# Config 1 of the benchmark: one block, d=256, 4 heads of 64 (MHA), vocab 32000.
TINY = dict(vocab_size=32000, model_dim=256, num_heads=4, num_kv_heads=None, head_k_dim=64,
            block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def gdn_inputs(B, H, L, dk, dv, seed, with_state=True):
    """Seeded delta-rule inputs in the GDN-op distribution (q,k L2-normalised)."""
    g = _gen(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1)
    v = torch.randn(B, H, L, dv, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=g))
    gg = -torch.nn.functional.softplus(torch.randn(B, H, L, generator=g)) * 0.1
    S0 = 0.1 * torch.randn(B, H, dk, dv, generator=g) if with_state else None
    return q, k, v, beta, gg, S0


def chord_inputs(B, H, Hkv, L, S, D, seed):
    g = _gen(seed)
    q = torch.randn(B, H, L, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    alpha = 0.5 + 1.5 * torch.rand(H, generator=g)
    beta = torch.rand(H, generator=g)
    mu = torch.ones(H)
    ssmax = 0.8 + 0.4 * torch.rand(H, generator=g)
    return q, k, v, alpha, beta, mu, ssmax


def eager_chord_reference(q, k, v, alpha, beta, mu, ssmax, q_start):
    """Drive the reference's own eager ChordAttention math through a bare layer.

    The eager body lives inside `ChordAttention.forward`; to feed it raw q/k/v we run
    the same statements on a layer whose GGD parameters reproduce alpha/beta/mu.
    """
    from motif.block.attention.chord_attn import ChordAttention
    B, H, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    layer = ChordAttention(hidden_size=H * D, num_heads=H, num_kv_heads=Hkv)
    with torch.no_grad():
        layer.theta_alpha.copy_(torch.log(alpha))
        layer.theta_beta.copy_(beta)
        layer.theta_mu.copy_(torch.asinh(mu / 2))
        layer.ssmax_s.copy_(ssmax)
    a, b, m = layer._ggd_parameters()
    grp = H // Hkv
    kk = k[:, :, None].expand(B, Hkv, grp, S, D).reshape(B, H, S, D)
    vv = v[:, :, None].expand(B, Hkv, grp, S, D).reshape(B, H, S, D)
    scores = (q @ kk.transpose(-2, -1)) * D ** -0.5
    bias = layer._compute_ggd_bias(q_len=L, kv_len=S, q_start=q_start, device=q.device)
    logits = scores + bias.unsqueeze(0)
    from motif.block.attention.chord_attn import _log_n_table
    log_n = _log_n_table(q_start + L, q.device)[q_start:q_start + L]
    logits = logits * (layer.ssmax_s.view(1, -1, 1, 1) * log_n.view(1, 1, L, 1))
    logits = logits.clamp_min(torch.finfo(logits.dtype).min / 4)
    qp = torch.arange(L) + q_start
    kp = torch.arange(S)
    logits = logits.masked_fill(kp[None, :] > qp[:, None], float('-inf'))
    attn = torch.softmax(logits, dim=-1)
    return (attn @ vv), (a, b, m), log_n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True, help='reference source tree (contains motif/)')
    ap.add_argument('--only', nargs='*', default=None, help='write only these fixtures (default: all)')
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    sys.path.insert(0, REPO)
    torch.set_num_threads(os.cpu_count())

    from motif.ops import (recurrent_gated_delta_rule, chunk_gated_delta_rule,
                           RMSNorm, GatedRMSNorm, SwiGLU)
    from motif.ops.attn_res import _read_sources
    from motif.model.config import MotifChordConfig
    from motif.model.motif import MotifChordModel
    from motif_b200.init import init_params

    out = {}
    # --- delta rule -------------------------------------------------------------
    q, k, v, beta, g, S0 = gdn_inputs(2, 3, 7, 16, 32, seed=1)
    o, S = recurrent_gated_delta_rule(q, k, v, beta, g, S0)
    out['gdn_recurrent'] = dict(q=q, k=k, v=v, beta=beta, g=g, S0=S0, o=o, S=S)
    q, k, v, beta, g, S0 = gdn_inputs(1, 2, 150, 32, 64, seed=2)
    o, S = chunk_gated_delta_rule(q, k, v, beta, g, S0, 64)
    out['gdn_chunk_ragged'] = dict(q=q, k=k, v=v, beta=beta, g=g, S0=S0, o=o, S=S)
    q, k, v, beta, g, _ = gdn_inputs(1, 1, 128, 64, 128, seed=3, with_state=False)
    o, S = chunk_gated_delta_rule(q, k, v, beta, g, None, 64)
    out['gdn_chunk_d64'] = dict(q=q, k=k, v=v, beta=beta, g=g, o=o, S=S)

    # --- chord (eager math of the layer) ---------------------------------------
    for name, (L, S_, qs) in {'chord_prefill': (37, 50, 13), 'chord_decode': (1, 40, 39),
                              'chord_start0': (24, 24, 0)}.items():
        q, k, v, alpha, beta, mu, ssmax = chord_inputs(2, 4, 2, L, S_, 32, seed=10 + L)
        o, (a, b, m), log_n = eager_chord_reference(q, k, v, alpha, beta, mu, ssmax, qs)
        out[name] = dict(q=q, k=k, v=v, alpha=a.detach(), beta=b.detach(), mu=m.detach(),
                         ssmax=ssmax, log_n=log_n, q_start=torch.tensor(qs), o=o.detach())

    # --- attn-res, norms, swiglu ------------------------------------------------
    gen = _gen(20)
    srcs = [torch.randn(2, 5, 48, generator=gen) for _ in range(4)]
    norm = RMSNorm(48)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(48, generator=gen))
    query = torch.randn(48, generator=gen) / 48 ** 0.5
    with torch.no_grad():
        out['attn_res'] = dict(sources=torch.stack(srcs), weight=norm.weight.detach().clone(), query=query,
                               h2=_read_sources(srcs[:2], query, norm), h4=_read_sources(srcs, query, norm))
        x = torch.randn(3, 7, 96, generator=gen)
        gn = GatedRMSNorm(48)
        gn.weight.copy_(1 + 0.1 * torch.randn(48, generator=gen))
        out['norms'] = dict(x=x, rms_w=norm.weight.detach().clone(), rms=norm(x[..., :48]),
                            gated_w=gn.weight.detach().clone(), gated=gn(x), swiglu=SwiGLU()(x))

    # --- small model: full logits, chunked / decode consistency, greedy ----------
    for dtype_name, dtype in (('fp32', torch.float32), ('bf16', torch.bfloat16)):
        torch.manual_seed(0)
        model = MotifChordModel(MotifChordConfig(**SMALL))
        init_params(model, seed=0, norm_jitter=0.1)
        model = model.to(dtype).eval()
        ids = torch.randint(0, SMALL['vocab_size'], (2, 40), generator=_gen(30))
        with torch.no_grad():
            full = model(ids).logits.float()
            pre = model(ids[:, :24])
            steps = []
            cache = pre.cache
            for t in range(24, 40):
                o = model(ids[:, t:t + 1], cache=cache)
                cache = o.cache
                steps.append(o.logits[:, 0].float())
            gen_ids = model.generate(ids[:, :16], max_new_tokens=24).run().generated
        out[f'small_{dtype_name}'] = dict(ids=ids, logits=full, decode_logits=torch.stack(steps, 1),
                                          greedy=gen_ids)

    # --- small model with attention masks (chord_attn.py:347-356, motif.py:592-602): a bool
    # keep-mask with a hole and right padding, and an additive float mask; prefill logits,
    # chunked prefill + decode with the mask widened every step, masked greedy generation
    torch.manual_seed(0)
    model = MotifChordModel(MotifChordConfig(**SMALL))
    init_params(model, seed=0, norm_jitter=0.1)
    model = model.eval()
    ids = torch.randint(0, SMALL['vocab_size'], (2, 40), generator=_gen(31))
    keep = torch.ones(2, 40, dtype=torch.bool)
    keep[0, 5:8] = False
    keep[1, 32:] = False
    gm = _gen(32)
    additive = -2.0 * torch.rand(2, 40, generator=gm)
    additive[0, 10] = float('-inf')
    additive[1, 3:5] = float('-inf')
    masked = {}
    with torch.no_grad():
        for mname, mask in (('bool', keep), ('float', additive)):
            full = model(ids, mask=mask).logits.float()
            pre = model(ids[:, :24], mask=mask[:, :24])
            steps, cache = [], pre.cache
            for t in range(24, 40):
                o = model(ids[:, t:t + 1], cache=cache, mask=mask[:, :t + 1])
                cache = o.cache
                steps.append(o.logits[:, 0].float())
            gen_ids = model.generate(ids[:, :16], max_new_tokens=8, mask=mask[:, :16]).run().generated
            masked[f'{mname}_mask'] = mask
            masked[f'{mname}_logits'] = full
            masked[f'{mname}_decode_logits'] = torch.stack(steps, 1)
            masked[f'{mname}_greedy'] = gen_ids
    out['masked'] = dict(ids=ids, **masked)

    # --- config 1 (tiny): last-position logits, per-position stats, 64-step greedy
    torch.manual_seed(0)
    model = MotifChordModel(MotifChordConfig(**TINY))
    init_params(model, seed=0, norm_jitter=0.0)
    model.eval()
    ids = torch.randint(0, TINY['vocab_size'], (1, 512), generator=_gen(0))
    with torch.no_grad():
        lg = model(ids).logits.float()
        gen_ids = model.generate(ids, max_new_tokens=64).run().generated
    out['tiny'] = dict(ids=ids, last_logits=lg[0, -2:].clone(), pos_max=lg[0].max(-1).values,
                       pos_argmax=lg[0].argmax(-1), pos_lse=torch.logsumexp(lg[0], -1),
                       pos_sumsq=lg[0].pow(2).sum(-1), greedy=gen_ids)

    # --- sampler: the filtered distribution the reference draws from -------------------
    # (repetition penalty -> temperature -> top-k -> top-p -> softmax, model/sampler.py:151-219);
    # torch.multinomial is wrapped to record the probabilities it is given.
    from motif.model.sampler import Sampler
    gen = _gen(40)
    V = 1000
    logits = torch.randn(4, V, generator=gen) * 3.0
    hist = torch.randint(0, V, (4, 50), generator=gen)
    cases = [(0.7, 50, 0.9, 1.15), (1.0, -1, 0.5, 1.0), (1.3, 10, -1.0, 1.3), (0.5, -1, -1.0, 1.15),
             (1.0, 1, -1.0, 1.0), (0.9, 200, 0.95, 1.05)]
    seen = {}
    real_multinomial = torch.multinomial

    def recording_multinomial(p, num_samples, *a, **kw):
        seen['p'] = p.detach().clone()
        return real_multinomial(p, num_samples, *a, **kw)

    torch.multinomial = recording_multinomial
    try:
        probs = []
        for t, k, p_, rp in cases:
            Sampler(temperature=t, top_k=None if k < 0 else k, top_p=None if p_ < 0 else p_,
                    repetition_penalty=rp)(logits, hist)
            probs.append(seen['p'])
    finally:
        torch.multinomial = real_multinomial
    out['sampler'] = dict(logits=logits, hist=hist, cases=torch.tensor(cases, dtype=torch.float64),
                          probs=torch.stack(probs))

    # --- checkpoints written by the reference's own writers (model/checkpoint.py): its
    # safetensors writer, a wrapper-prefixed bare state_dict and a pipeline-style mapping;
    # plus the logits of those weights and the config the reference resolves from each file
    if args.only is None or 'checkpoints' in args.only:
        from motif.model.checkpoint import save_safetensors, config_to_dict, load_checkpoint
        ck_dir = os.path.join(HERE, 'ckpt')
        os.makedirs(ck_dir, exist_ok=True)
        ccfg = MotifChordConfig(vocab_size=64, model_dim=32, num_heads=2, num_kv_heads=1, head_k_dim=16,
                                block=('gdn', 'chord'), block_n=1)
        torch.manual_seed(0)
        model = MotifChordModel(ccfg)
        init_params(model, seed=0, norm_jitter=0.1)
        model.eval()
        save_safetensors(model, os.path.join(ck_dir, 'model.safetensors'))
        sd = model.state_dict()
        torch.save({'module.' + k: v.clone() for k, v in sd.items() if k != 'lm_head.weight'},
                   os.path.join(ck_dir, 'bare_module.pt'))
        torch.save({'__pipeline__': 'PretrainPipeline',
                    'payload': {'model': {k: v.clone() for k, v in sd.items()}, 'config': config_to_dict(ccfg)}},
                   os.path.join(ck_dir, 'pipeline.pt'))
        ids = torch.randint(0, 64, (2, 12), generator=_gen(33))
        with torch.no_grad():
            lg = model(ids).logits.float()
        resolved = {}
        for f in ('model.safetensors', 'bare_module.pt', 'pipeline.pt'):
            ld = load_checkpoint(os.path.join(ck_dir, f))
            cfg = MotifChordModel._resolve_pretrained_config(None, ld)
            resolved[f] = json.dumps(config_to_dict(cfg))
        out['checkpoints'] = dict(ids=ids, logits=lg, resolved=resolved,
                                  state_dict={k: v.clone() for k, v in sd.items()})

    for name, d in out.items():
        if args.only is not None and name not in args.only:
            continue
        path = os.path.join(HERE, f'{name}.pt')
        torch.save({k: (v.contiguous() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}, path)
        print(f'wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)')


if __name__ == '__main__':
    main()
