"""Gradients of the three hot-path ops through `motif_b200.ops` (autograd over the backward
kernels of `csrc/backward.cu`) against the oracle's autograd in fp64 on the same inputs.

Bar: for fp32 inputs every gradient (q / k / v / sources / state, and the GGD parameters, the
pseudo-query, the norm weight, beta, g) within 1e-5 of the fp64 gradient, relative to that
gradient's largest magnitude; 16-bit inputs within a few 16-bit roundings (2e-2).
"""

import math

import pytest
import torch

from motif_b200 import ops
from oracle import ops as oo

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def chord_inputs(B, H, Hkv, L, S, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    alpha = 0.05 + 0.3 * torch.rand(H, generator=g)
    beta = 0.6 + 0.8 * torch.rand(H, generator=g)
    mu = 2.0 * torch.rand(H, generator=g)
    ssmax = 0.5 + torch.rand(H, generator=g)
    ssmax[0] = -ssmax[0]  # a negative logit scale
    q_start = S - L
    log_n = torch.log(torch.arange(q_start, q_start + L, dtype=torch.float32) + 1.0)[None].repeat(B, 1)
    log_n += 0.1 * torch.rand(B, L, generator=g)
    dout = torch.randn(B, H, L, D, generator=g)
    t = [x.to(dtype) for x in (q, k, v)] + [alpha, beta, mu, ssmax, log_n, dout.to(dtype)]
    return t, q_start


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,H,Hkv,L,S,D', [(2, 4, 2, 70, 90, 32), (1, 4, 4, 65, 65, 64), (2, 6, 2, 33, 130, 16),
                                           (1, 2, 1, 40, 40, 128)])
def test_chord_attention_gradients(dtype, B, H, Hkv, L, S, D):
    (q, k, v, al, be, mu, ss, log_n, dout), q_start = chord_inputs(B, H, Hkv, L, S, D, dtype, L * S + D)
    leaves = [x.clone().cuda().requires_grad_(True) for x in (q, k, v, al, be, mu, ss)]
    out = ops.apply_chord_attention(*leaves, log_n.cuda(), q_start=q_start)
    out.backward(dout.cuda())
    ref = [x.clone().double().requires_grad_(True) for x in (q, k, v, al, be, mu, ss)]
    o_ref = oo.chord_attention(*ref, log_n.double(), q_start=q_start)
    o_ref.backward(dout.double())
    bar = 1e-5 if dtype == torch.float32 else 2e-2
    for name, a, b in zip(('q', 'k', 'v', 'alpha', 'beta', 'mu', 'ssmax'), leaves, ref):
        assert a.grad is not None and a.grad.dtype == a.dtype, name
        e = rel(a.grad, b.grad)
        assert e < bar, (name, e)


def test_chord_attention_gradient_of_some_inputs_only():
    (q, k, v, al, be, mu, ss, log_n, dout), q_start = chord_inputs(1, 2, 2, 20, 20, 32, torch.float32, 7)
    qc = q.cuda().requires_grad_(True)
    out = ops.apply_chord_attention(qc, k.cuda(), v.cuda(), al.cuda(), be.cuda(), mu.cuda(), ss.cuda(), log_n.cuda())
    out.sum().backward()
    qr = q.double().requires_grad_(True)
    oo.chord_attention(qr, k.double(), v.double(), al.double(), be.double(), mu.double(), ss.double(),
                       log_n.double()).sum().backward()
    assert rel(qc.grad, qr.grad) < 1e-5
    # no gradient requested: the inference path, no graph
    with torch.no_grad():
        assert not ops.apply_chord_attention(qc, k.cuda(), v.cuda(), al.cuda(), be.cuda(), mu.cuda(), ss.cuda(),
                                             log_n.cuda()).requires_grad


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('N,B,T,D', [(3, 2, 37, 128), (5, 1, 64, 768), (1, 2, 5, 256), (8, 1, 9, 64)])
def test_attn_res_gradients(dtype, N, B, T, D):
    g = torch.Generator().manual_seed(N * 100 + T)
    srcs = [torch.randn(B, T, D, generator=g).to(dtype) for _ in range(N)]
    w = (1.0 + 0.2 * torch.randn(D, generator=g)).to(dtype)
    qv = (0.5 * torch.randn(D, generator=g)).to(dtype)
    dh = torch.randn(B, T, D, generator=g).to(dtype)
    eps = 1e-6
    leaves = [s.clone().cuda().requires_grad_(True) for s in srcs]
    wl, ql = w.clone().cuda().requires_grad_(True), qv.clone().cuda().requires_grad_(True)
    out = ops.attn_res_block(leaves, wl, ql, eps)
    out.backward(dh.cuda())
    ref = [s.double().requires_grad_(True) for s in srcs]
    wr, qr = w.double().requires_grad_(True), qv.double().requires_grad_(True)
    oo.attn_res(ref, qr, wr, eps).backward(dh.double())
    bar = 1e-5 if dtype == torch.float32 else 2e-2
    for i, (a, b) in enumerate(zip(leaves, ref)):
        assert rel(a.grad, b.grad) < bar, ('source', i, rel(a.grad, b.grad))
    assert rel(wl.grad, wr.grad) < bar, ('weight', rel(wl.grad, wr.grad))
    assert rel(ql.grad, qr.grad) < bar, ('query', rel(ql.grad, qr.grad))


def gdn_inputs(B, H, L, Dk, Dv, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, Dk, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, H, L, Dk, generator=g), dim=-1)
    v = torch.randn(B, H, L, Dv, generator=g)
    beta = torch.rand(B, H, L, generator=g)
    gg = -0.3 * torch.rand(B, H, L, generator=g)
    S0 = 0.1 * torch.randn(B, H, Dk, Dv, generator=g)
    do = torch.randn(B, H, L, Dv, generator=g)
    dS = torch.randn(B, H, Dk, Dv, generator=g)
    return q, k, v, beta, gg, S0, do, dS


@pytest.mark.parametrize('fn', ['recurrent', 'chunk'])
@pytest.mark.parametrize('B,H,L,Dk,Dv,with_state', [(2, 3, 150, 32, 64, True), (1, 2, 64, 64, 128, True),
                                                    (1, 2, 70, 64, 64, False), (2, 1, 5, 16, 32, True)])
def test_gated_delta_rule_gradients(fn, B, H, L, Dk, Dv, with_state):
    q, k, v, beta, gg, S0, do, dS = gdn_inputs(B, H, L, Dk, Dv, L + Dk)
    op = ops.recurrent_gated_delta_rule if fn == 'recurrent' else ops.chunk_gated_delta_rule
    names = ['q', 'k', 'v', 'beta', 'g'] + (['S'] if with_state else [])
    base = [q, k, v, beta, gg] + ([S0] if with_state else [])
    leaves = [x.clone().cuda().requires_grad_(True) for x in base]
    o, S_out = op(*leaves) if with_state else op(*leaves, None)
    torch.autograd.backward([o, S_out], [do.cuda(), dS.cuda()])
    ref = [x.double().requires_grad_(True) for x in base]
    o_r, S_r = oo.recurrent_gated_delta_rule(*ref) if with_state else oo.recurrent_gated_delta_rule(*ref, None)
    torch.autograd.backward([o_r, S_r], [do.double(), dS.double()])
    for name, a, b in zip(names, leaves, ref):
        e = rel(a.grad, b.grad)
        assert e < 1e-5, (name, e)


def test_gated_delta_rule_output_gradient_only():
    q, k, v, beta, gg, S0, do, dS = gdn_inputs(1, 2, 40, 32, 64, 3)
    vl = v.clone().cuda().requires_grad_(True)
    o, _ = ops.chunk_gated_delta_rule(q.cuda(), k.cuda(), vl, beta.cuda(), gg.cuda())
    (o * do.cuda()).sum().backward()
    vr = v.double().requires_grad_(True)
    o_r, _ = oo.recurrent_gated_delta_rule(q.double(), k.double(), vr, beta.double(), gg.double())
    (o_r * do.double()).sum().backward()
    assert rel(vl.grad, vr.grad) < 1e-5
    assert math.isfinite(vl.grad.abs().max().item())
