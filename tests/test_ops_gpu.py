"""Op-level parity of the CUDA kernels (through the C ABI) against the CPU oracle.

Tolerances (stated per the north-star): fp32 inputs -> max relative error 1e-5 against the
fp32 oracle; 16-bit inputs -> the oracle is run in fp32 on the same (rounded) inputs and the
kernel must stay within the 16-bit output rounding (rel 1e-2: outputs and the returned
state are in the input dtype, as the reference returns them).
"""

import os

import pytest
import torch

from oracle import ops as oo

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


@pytest.fixture(scope='module')
def ops():
    assert torch.cuda.is_available(), 'GPU tests need CUDA'
    from motif_b200 import ops as mo
    return mo


def rel_err(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def gdn_inputs(B, H, L, dk, dv, seed, state=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1) * dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1)
    v = torch.randn(B, H, L, dv, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, L, generator=g))
    gg = -torch.nn.functional.softplus(torch.randn(B, H, L, generator=g)) * 0.1
    S0 = 0.1 * torch.randn(B, H, dk, dv, generator=g) if state else None
    return q, k, v, beta, gg, S0


def cuda(*ts, dtype=None):
    return [None if t is None else (t.cuda() if dtype is None else t.to('cuda', dtype)) for t in ts]


# ----------------------------------------------------------------------- delta rule
@pytest.mark.parametrize('name', ['gdn_recurrent'])
def test_recurrent_golden(ops, name):
    d = torch.load(os.path.join(GOLD, f'{name}.pt'))
    o, S = ops.recurrent_gated_delta_rule(*cuda(d['q'], d['k'], d['v'], d['beta'], d['g'], d['S0']))
    assert rel_err(o, d['o']) < 1e-5 and rel_err(S, d['S']) < 1e-5


@pytest.mark.parametrize('name', ['gdn_chunk_ragged', 'gdn_chunk_d64'])
def test_chunk_golden(ops, name):
    d = torch.load(os.path.join(GOLD, f'{name}.pt'))
    o, S = ops.chunk_gated_delta_rule(*cuda(d['q'], d['k'], d['v'], d['beta'], d['g'], d.get('S0')))
    assert rel_err(o, d['o']) < 1e-5, rel_err(o, d['o'])
    assert rel_err(S, d['S']) < 1e-5, rel_err(S, d['S'])


@pytest.mark.parametrize('B,H,L,dk,dv', [(2, 3, 1, 64, 128), (1, 2, 17, 16, 32), (2, 2, 130, 64, 128),
                                         (1, 1, 64, 32, 64), (1, 2, 200, 64, 64)])
def test_recurrent_vs_oracle(ops, B, H, L, dk, dv):
    q, k, v, beta, g, S0 = gdn_inputs(B, H, L, dk, dv, seed=L)
    ro, rS = oo.recurrent_gated_delta_rule(q, k, v, beta, g, S0)
    o, S = ops.recurrent_gated_delta_rule(*cuda(q, k, v, beta, g, S0))
    assert rel_err(o, ro) < 1e-5 and rel_err(S, rS) < 1e-5


@pytest.mark.parametrize('B,H,L,dk,dv,state', [(1, 1, 1, 64, 128, True), (2, 3, 63, 64, 128, False),
                                               (2, 3, 64, 64, 128, True), (1, 2, 300, 64, 128, True),
                                               (2, 2, 129, 16, 32, True), (1, 3, 100, 32, 64, True),
                                               (1, 2, 77, 64, 64, False), (1, 1, 0, 64, 128, True)])
def test_chunk_fp32_vs_oracle(ops, B, H, L, dk, dv, state):
    q, k, v, beta, g, S0 = gdn_inputs(B, H, L, dk, dv, seed=100 + L, state=state)
    if L == 0:
        o, S = ops.chunk_gated_delta_rule(*cuda(q, k, v, beta, g, S0))
        assert o.shape == (B, H, 0, dv) and torch.allclose(S.cpu(), S0)
        return
    ro, rS = oo.chunk_gated_delta_rule(q, k, v, beta, g, S0)
    o, S = ops.chunk_gated_delta_rule(*cuda(q, k, v, beta, g, S0))
    assert rel_err(o, ro) < 1e-5, rel_err(o, ro)
    assert rel_err(S, rS) < 1e-5, rel_err(S, rS)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('L', [64, 257, 1000])
def test_chunk_16bit_vs_oracle(ops, dtype, L):
    q, k, v, beta, g, S0 = gdn_inputs(2, 3, L, 64, 128, seed=7 + L)
    q, k, v = (t.to(dtype) for t in (q, k, v))
    ro, rS = oo.chunk_gated_delta_rule(q.float(), k.float(), v.float(), beta, g, S0)
    o, S = ops.chunk_gated_delta_rule(*cuda(q, k, v, beta, g, S0))
    assert o.dtype == dtype and S.dtype == dtype  # the reference returns S in q's dtype
    assert rel_err(o.float(), ro) < 1e-2, rel_err(o.float(), ro)
    assert rel_err(S.float(), rS) < 1e-2, rel_err(S.float(), rS)


def test_chunk_split_sequence_property(ops):
    """Full sequence == two halves with the state carried (size-independent property)."""
    q, k, v, beta, g, S0 = cuda(*gdn_inputs(2, 4, 1000, 64, 128, seed=5))
    o, S = ops.chunk_gated_delta_rule(q, k, v, beta, g, S0)
    o1, S1 = ops.chunk_gated_delta_rule(q[:, :, :333], k[:, :, :333], v[:, :, :333], beta[:, :, :333],
                                        g[:, :, :333], S0)
    o2, S2 = ops.chunk_gated_delta_rule(q[:, :, 333:], k[:, :, 333:], v[:, :, 333:], beta[:, :, 333:],
                                        g[:, :, 333:], S1)
    assert rel_err(torch.cat([o1, o2], 2), o) < 1e-5 and rel_err(S2, S) < 1e-5


def test_chunk_strided_token_major(ops):
    """[B,T,H,D] memory passed as [B,H,T,D] views (the model's layout)."""
    B, H, L, dk, dv = 2, 3, 150, 64, 128
    q, k, v, beta, g, S0 = gdn_inputs(B, H, L, dk, dv, seed=9)
    qt, kt, vt = (t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (q, k, v))
    bt, gt = (t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (beta, g))
    ro, rS = oo.chunk_gated_delta_rule(q, k, v, beta, g, S0)
    o, S = ops.chunk_gated_delta_rule(qt, kt, vt, bt, gt, S0.cuda())
    assert rel_err(o, ro) < 1e-5 and rel_err(S, rS) < 1e-5


def test_gdn_op_config_full_size(ops):
    """Config 2 (B=8, H=12, T=4096, dk=dv=64, bf16 in, fp32 state) against the fp32 oracle."""
    B, H, L = 8, 12, 4096
    gen = torch.Generator().manual_seed(0)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, 64, generator=gen), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, H, L, 64, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, H, L, 64, generator=gen).bfloat16()
    beta = torch.sigmoid(torch.randn(B, H, L, generator=gen))
    g = -torch.nn.functional.softplus(torch.randn(B, H, L, generator=gen)) * 0.1
    o, S = ops.chunk_gated_delta_rule(*cuda(q, k, v, beta, g))
    ro, rS = oo.chunk_gated_delta_rule(q[:1, :2].float(), k[:1, :2].float(), v[:1, :2].float(),
                                       beta[:1, :2], g[:1, :2])
    assert rel_err(o[:1, :2].float(), ro) < 1e-2
    assert rel_err(S[:1, :2].float(), rS) < 1e-2
    assert torch.isfinite(o).all() and torch.isfinite(S).all()


# ------------------------------------------------------------------ chord attention
def chord_inputs(B, H, Hkv, L, S, D, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    alpha = 0.5 + 1.5 * torch.rand(H, generator=g)
    beta = torch.rand(H, generator=g)
    mu = torch.ones(H) + 0.5 * torch.randn(H, generator=g)
    ssmax = 0.8 + 0.4 * torch.rand(H, generator=g)
    q_start = S - L
    log_n = oo.log_n_table(q_start, L).view(1, L).expand(B, L).contiguous()
    return q, k, v, alpha, beta, mu, ssmax, log_n, q_start


@pytest.mark.parametrize('name', ['chord_prefill', 'chord_decode', 'chord_start0'])
def test_chord_golden(ops, name):
    d = torch.load(os.path.join(GOLD, f'{name}.pt'))
    B, L = d['q'].shape[0], d['q'].shape[2]
    out = ops.apply_chord_attention(*cuda(d['q'], d['k'], d['v'], d['alpha'], d['beta'], d['mu'], d['ssmax'],
                                          d['log_n'].view(1, L).expand(B, L).contiguous()), int(d['q_start']))
    assert rel_err(out, d['o']) < 1e-5


@pytest.mark.parametrize('B,H,Hkv,L,S,D', [(1, 4, 4, 100, 100, 64), (2, 12, 3, 130, 200, 64), (1, 8, 1, 33, 33, 32),
                                           (2, 4, 2, 1, 77, 16), (1, 6, 2, 70, 90, 64), (1, 2, 2, 5, 300, 128)])
def test_chord_fp32_vs_oracle(ops, B, H, Hkv, L, S, D):
    q, k, v, alpha, beta, mu, ssmax, log_n, qs = chord_inputs(B, H, Hkv, L, S, D, seed=L + S)
    ref = oo.chord_attention(q, k, v, alpha, beta, mu, ssmax, log_n, qs)
    out = ops.apply_chord_attention(*cuda(q, k, v, alpha, beta, mu, ssmax, log_n))
    assert rel_err(out, ref) < 1e-5, rel_err(out, ref)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('B,H,Hkv,L,S,D', [(1, 4, 4, 200, 200, 64), (2, 12, 3, 300, 300, 64),
                                           (1, 8, 1, 65, 100, 32), (2, 4, 2, 1, 513, 16),
                                           (1, 16, 2, 129, 129, 64), (1, 12, 3, 1000, 1000, 64),
                                           (2, 12, 3, 100, 350, 64), (1, 4, 2, 3, 5, 64), (3, 8, 4, 257, 600, 64),
                                           (1, 2, 2, 128, 128, 64)])
def test_chord_16bit_vs_oracle(ops, dtype, B, H, Hkv, L, S, D):
    q, k, v, alpha, beta, mu, ssmax, log_n, qs = chord_inputs(B, H, Hkv, L, S, D, seed=3 * L + S, dtype=dtype)
    ref = oo.chord_attention(q.float(), k.float(), v.float(), alpha, beta, mu, ssmax, log_n, qs)
    out = ops.apply_chord_attention(*cuda(q, k, v, alpha, beta, mu, ssmax, log_n))
    assert out.dtype == dtype
    assert rel_err(out.float(), ref) < 1e-2, rel_err(out.float(), ref)


@pytest.mark.parametrize('B,H,Hkv,L,S', [(2, 12, 3, 300, 300), (1, 8, 8, 70, 500), (2, 16, 2, 200, 260)])
def test_chord_tcgen05_matches_mma_sync(ops, B, H, Hkv, L, S):
    """16-bit D = 64 prefill: the tcgen05 kernel (default) against the mma.sync kernel."""
    q, k, v, alpha, beta, mu, ssmax, log_n, qs = chord_inputs(B, H, Hkv, L, S, 64, seed=L + 7 * S,
                                                              dtype=torch.bfloat16)
    args = cuda(q, k, v, alpha, beta, mu, ssmax, log_n)
    tc = ops.apply_chord_attention(*args)
    from motif_b200 import _lib
    with _lib.forced(_lib.FORCE_CHORD_MMA_SYNC):
        ms = ops.apply_chord_attention(*args)
    assert _lib.wait_timeouts() == 0
    ref = oo.chord_attention(q.float(), k.float(), v.float(), alpha, beta, mu, ssmax, log_n, qs)
    assert rel_err(tc.float(), ref) < 1e-2 and rel_err(ms.float(), ref) < 1e-2
    assert rel_err(tc.float(), ms.float()) < 1e-2


@pytest.mark.parametrize('L,S', [(200, 200), (70, 330)])
def test_chord_16bit_negative_ssmax(ops, L, S):
    """ssmax < 0 on some heads flips those heads' logits; first positions have log n = 0."""
    q, k, v, alpha, beta, mu, ssmax, log_n, qs = chord_inputs(2, 12, 3, L, S, 64, seed=L + S, dtype=torch.bfloat16)
    ssmax = ssmax.clone()
    ssmax[::3] *= -1.0
    ref = oo.chord_attention(q.float(), k.float(), v.float(), alpha, beta, mu, ssmax, log_n, qs)
    out = ops.apply_chord_attention(*cuda(q, k, v, alpha, beta, mu, ssmax, log_n))
    assert rel_err(out.float(), ref) < 1e-2, rel_err(out.float(), ref)


def test_chord_op_config_subset(ops):
    """Config 3 (B=8, H=12, T=4096, D=64, bf16): full-size kernel, oracle on two (b, h) slices."""
    B, H, L, D = 8, 12, 4096, 64
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(B, H, L, D, generator=gen).bfloat16()
    k = torch.randn(B, H, L, D, generator=gen).bfloat16()
    v = torch.randn(B, H, L, D, generator=gen).bfloat16()
    alpha = 0.5 + 1.5 * torch.rand(H, generator=gen)
    beta = torch.rand(H, generator=gen)
    mu = torch.ones(H)
    ssmax = torch.ones(H)
    log_n = oo.log_n_table(0, L).view(1, L).expand(B, L).contiguous()
    out = ops.apply_chord_attention(*cuda(q, k, v, alpha, beta, mu, ssmax, log_n))
    for (b, h) in ((0, 0), (7, 11)):
        ref = oo.chord_attention(q[b:b + 1, h:h + 1].float(), k[b:b + 1, h:h + 1].float(),
                                 v[b:b + 1, h:h + 1].float(), alpha[h:h + 1], beta[h:h + 1], mu[h:h + 1],
                                 ssmax[h:h + 1], log_n[b:b + 1], 0)
        assert rel_err(out[b:b + 1, h:h + 1].float(), ref) < 1e-2


def test_chord_errors(ops):
    q, k, v, alpha, beta, mu, ssmax, log_n, _ = cuda(*chord_inputs(1, 4, 2, 8, 8, 32, seed=1)[:8], None)
    with pytest.raises(ValueError):
        ops.apply_chord_attention(q, k, v, alpha, beta, mu, ssmax, log_n[:, :4])
    with pytest.raises(ValueError):
        ops.apply_chord_attention(q, k, v, alpha.double(), beta, mu, ssmax, log_n)
    with pytest.raises(ValueError):
        ops.apply_chord_attention(q, k, v, alpha, beta, mu, ssmax, log_n, q_start=-1)
    with pytest.raises(ValueError):
        ops.apply_chord_attention(q.cpu(), k, v, alpha, beta, mu, ssmax, log_n)


# ------------------------------------------------------------- attn-res / norms / act
def test_attn_res_golden(ops):
    d = torch.load(os.path.join(GOLD, 'attn_res.pt'))
    srcs = [s.cuda() for s in d['sources']]
    h2 = ops.attn_res_block(srcs[:2], d['weight'].cuda(), d['query'].cuda(), 1e-6)
    h4 = ops.attn_res_block(srcs, d['weight'].cuda(), d['query'].cuda(), 1e-6)
    assert rel_err(h2, d['h2']) < 1e-5 and rel_err(h4, d['h4']) < 1e-5


@pytest.mark.parametrize('n', [1, 2, 3, 4, 5, 8])
def test_attn_res_vs_oracle(ops, n):
    g = torch.Generator().manual_seed(n)
    srcs = [torch.randn(3, 17, 768, generator=g) for _ in range(n)]
    w = 1 + 0.1 * torch.randn(768, generator=g)
    qv = torch.randn(768, generator=g) / 768 ** 0.5
    ref = oo.attn_res(srcs, qv, w)
    out = ops.attn_res_block([s.cuda() for s in srcs], w.cuda(), qv.cuda(), 1e-6)
    assert rel_err(out, ref) < 1e-5


def test_norms_golden(ops):
    d = torch.load(os.path.join(GOLD, 'norms.pt'))
    x = d['x'].cuda()
    rn = ops.RMSNorm(48).cuda()
    rn.weight.data.copy_(d['rms_w'])
    gn = ops.GatedRMSNorm(48).cuda()
    gn.weight.data.copy_(d['gated_w'])
    with torch.no_grad():
        assert rel_err(rn(x[..., :48]), d['rms']) < 1e-6
        assert rel_err(gn(x), d['gated']) < 1e-6
        assert rel_err(ops.SwiGLU()(x), d['swiglu']) < 1e-6


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_norms_vs_oracle(ops, dtype):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 33, 2 * 768, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(768, generator=g)).to(dtype)
    rn = ops.RMSNorm(768).cuda().to(dtype)
    rn.weight.data.copy_(w)
    gn = ops.GatedRMSNorm(768).cuda().to(dtype)
    gn.weight.data.copy_(w)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    with torch.no_grad():
        assert rel_err(rn(x[..., :768].cuda()).float(), oo.rms_norm(x[..., :768], w).float()) < tol
        assert rel_err(gn(x.cuda()).float(), oo.gated_rms_norm(x, w).float()) < tol
        assert rel_err(ops.SwiGLU()(x.cuda()).float(), oo.swiglu(x).float()) < tol
