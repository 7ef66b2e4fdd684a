"""Parity of the fused model-level kernels (one C-ABI call each) against the CPU oracle.

Each fused kernel replaces a run of reference statements (cited in `include/motif_b200.h`);
here every one is checked on its own against the oracle statements it replaces.
"""

import pytest
import torch
import torch.nn.functional as F

from motif_b200 import _lib
from oracle import ops as oo

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def st():
    return _lib.stream_ptr()


TOL = {torch.float32: 1e-5, torch.bfloat16: 1.5e-2}


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('D', [64, 256, 768])
@pytest.mark.parametrize('n', [1, 2, 4, 5])
@pytest.mark.parametrize('mode', ['softmax', 'sum'])
@pytest.mark.parametrize('rows', [37, 2500])  # one CTA per row (decode) / one warp per row
def test_attn_res_norm(dtype, D, n, mode, rows):
    g = torch.Generator().manual_seed(D + n)
    srcs = [torch.randn(rows, D, generator=g).to(dtype) for _ in range(n)]
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    qv = (torch.randn(D, generator=g) / D ** 0.5).to(dtype)
    if mode == 'softmax':
        h = oo.attn_res([s.float()[None] for s in srcs], qv.float(), w.float())[0] if n > 1 else srcs[0].float()
    else:
        h = sum(s.float() for s in srcs)
    hn = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
    cs = [s.cuda() for s in srcs]
    h_out = torch.empty(rows, D, dtype=dtype, device='cuda')
    hn_out = torch.empty(rows, D, dtype=dtype, device='cuda')
    wq = (w.cuda(), qv.cuda()) if mode == 'softmax' else (None, None)
    _lib.call('motif_b200_attn_res_norm', _lib.ptr_array([t.data_ptr() for t in cs]), n, D, _lib.ptr(wq[0]),
              _lib.ptr(wq[1]), _lib.ptr(h_out), _lib.ptr(hn_out), D, rows, D, 1e-6, 1e-6, _lib.dtype_code(dtype), st())
    assert rel_err(h_out.float(), h) < TOL[dtype], rel_err(h_out.float(), h)
    assert rel_err(hn_out.float(), hn) < TOL[dtype], rel_err(hn_out.float(), hn)


def gdn_setup(B, T, H, dk, dv, dtype, seed, with_conv=True):
    g = torch.Generator().manual_seed(seed)
    C = H * (2 * dk + dv)
    N = C + 2 * H + 40  # extra trailing columns, as in the packed projection
    proj = (0.5 * torch.randn(B, T, N, generator=g)).to(dtype)
    conv_w = (0.3 * torch.randn(C, 4, generator=g)).to(dtype)
    A_log = torch.log(1 + 15 * torch.rand(H, generator=g)).to(dtype)
    dt_bias = (0.1 * torch.randn(H, generator=g)).to(dtype)
    conv_in = (0.5 * torch.randn(B, 3, C, generator=g)).to(dtype) if with_conv else None
    return proj, conv_w, A_log, dt_bias, conv_in, C, N


def gdn_prep_oracle(proj, conv_w, A_log, dt_bias, conv_in, B, T, H, dk, dv):
    f = proj.float()
    C = H * (2 * dk + dv)
    x = f[..., :C]
    cache = conv_in.float().transpose(1, 2) if conv_in is not None else None
    y, new_cache = oo.causal_conv_silu(x, conv_w.float().view(C, 1, 4), cache)
    q = y[..., :H * dk].view(B, T, H, dk)
    k = y[..., H * dk:2 * H * dk].view(B, T, H, dk)
    v = y[..., 2 * H * dk:].view(B, T, H, dv)
    q = F.normalize(q, dim=-1) * dk ** -0.5
    k = F.normalize(k, dim=-1)
    a = f[..., C:C + H]
    b = f[..., C + H:C + 2 * H]
    beta = torch.sigmoid(b)
    gg = -A_log.float().exp() * F.softplus(a + dt_bias.float())
    return q, k, v, beta, gg, new_cache.transpose(1, 2)


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,T,H,dk,dv,with_conv', [(2, 37, 3, 64, 128, True), (1, 2, 12, 64, 128, False),
                                                   (2, 70, 4, 16, 32, True), (1, 16, 2, 32, 64, True)])
def test_gdn_prep(dtype, B, T, H, dk, dv, with_conv):
    proj, conv_w, A_log, dt_bias, conv_in, C, N = gdn_setup(B, T, H, dk, dv, dtype, seed=T)
    q, k, v, beta, gg, cout = gdn_prep_oracle(proj, conv_w, A_log, dt_bias, conv_in, B, T, H, dk, dv)
    M = B * T
    qb = torch.empty(M, H * dk, dtype=dtype, device='cuda')
    kb = torch.empty_like(qb)
    vb = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    be = torch.empty(M, H, device='cuda')
    ge = torch.empty(M, H, device='cuda')
    co = torch.empty(B, 3, C, dtype=dtype, device='cuda')
    p, cw, al, db = (t.cuda() for t in (proj, conv_w, A_log, dt_bias))
    ci = conv_in.cuda() if conv_in is not None else None
    _lib.call('motif_b200_gdn_prep', _lib.ptr(p), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db), _lib.ptr(ci),
              _lib.ptr(co), _lib.ptr(qb), _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(be), _lib.ptr(ge), B, T, H, dk, dv,
              _lib.dtype_code(dtype), st())
    tol = TOL[dtype]
    assert rel_err(qb.view(B, T, H, dk).float(), q) < tol
    assert rel_err(kb.view(B, T, H, dk).float(), k) < tol
    assert rel_err(vb.view(B, T, H, dv).float(), v) < tol
    assert rel_err(be.view(B, T, H), beta) < tol
    assert rel_err(ge.view(B, T, H), gg) < tol
    assert rel_err(co.float(), cout) < tol


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,H,dk,dv', [(3, 12, 64, 128), (2, 4, 16, 32), (2, 3, 32, 64), (1, 2, 128, 256), (2, 2, 64, 64)])
def test_gdn_decode(dtype, B, H, dk, dv):
    proj, conv_w, A_log, dt_bias, conv_in, C, _ = gdn_setup(B, 1, H, dk, dv, dtype, seed=B * H)
    g = torch.Generator().manual_seed(11)
    N = C + 2 * H + H * dv
    proj = torch.cat([proj[..., :C + 2 * H], (0.5 * torch.randn(B, 1, H * dv, generator=g)).to(dtype)], -1)
    state = 0.1 * torch.randn(B, H, dk, dv, generator=g)
    onw = (1 + 0.1 * torch.randn(dv, generator=g)).to(dtype)
    q, k, v, beta, gg, cout = gdn_prep_oracle(proj, conv_w, A_log, dt_bias, conv_in, B, 1, H, dk, dv)
    o, S = oo.recurrent_gated_delta_rule(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                         beta.transpose(1, 2), gg.transpose(1, 2), state)
    gate = proj[..., C + 2 * H:].float().view(B, 1, H, dv)
    ref = oo.gated_rms_norm(torch.cat([o.transpose(1, 2), gate], -1), onw.float()).reshape(B, H * dv)
    p, cw, al, db, ci, sd, ow = (t.cuda() for t in (proj, conv_w, A_log, dt_bias, conv_in, state, onw))
    out = torch.empty(B, H * dv, dtype=dtype, device='cuda')
    _lib.call('motif_b200_gdn_decode', _lib.ptr(p), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db), _lib.ptr(ci),
              _lib.ptr(sd), p.data_ptr() + (C + 2 * H) * p.element_size(), _lib.ptr(ow), _lib.ptr(out), H * dv,
              B, H, dk, dv, 1e-6, _lib.dtype_code(dtype), st())
    tol = TOL[dtype]
    assert rel_err(sd, S) < max(tol, 1e-5)
    assert rel_err(ci.float(), cout) < tol
    assert rel_err(out.float(), ref) < (1e-5 if dtype == torch.float32 else 3e-2)


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,H,dk,dv,hid', [(64, 12, 64, 128, 2816), (3, 12, 64, 128, 24), (2, 4, 16, 32, 40),
                                           (5, 12, 64, 128, 20)])
def test_gdn_decode_swiglu_matches_separate_launches(dtype, B, H, dk, dv, hid):
    """The fused GDN step + SwiGLU launch gives bit-identical state, conv cache, GDN output and
    MLP activation to motif_b200_gdn_decode followed by motif_b200_swiglu (hid = 20 is not a
    multiple of 8: the entry falls back to a separate SwiGLU launch)."""
    proj, conv_w, A_log, dt_bias, conv_in, C, _ = gdn_setup(B, 1, H, dk, dv, dtype, seed=B + hid)
    g = torch.Generator().manual_seed(5)
    N = C + 2 * H + H * dv + 2 * hid
    proj = torch.cat([proj[..., :C + 2 * H], torch.randn(B, 1, H * dv + 2 * hid, generator=g).to(dtype)], -1)
    proj = proj.view(B, N).cuda()
    state = (0.1 * torch.randn(B, H, dk, dv, generator=g)).cuda()
    onw = (1 + 0.1 * torch.randn(dv, generator=g)).to(dtype).cuda()
    cw, al, db, ci = (t.cuda() for t in (conv_w, A_log, dt_bias, conv_in))
    outs = []
    for fused in (False, True):
        sd, cc = state.clone(), ci.clone()
        cat = torch.full((B, H * dv + hid), 7, dtype=dtype, device='cuda')
        gate = proj.data_ptr() + (C + 2 * H) * proj.element_size()
        gu = proj.data_ptr() + (C + 2 * H + H * dv) * proj.element_size()
        act = cat.data_ptr() + H * dv * cat.element_size()
        if fused:
            _lib.call('motif_b200_gdn_decode_swiglu', _lib.ptr(proj), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db),
                      _lib.ptr(cc), _lib.ptr(sd), gate, _lib.ptr(onw), _lib.ptr(cat), cat.stride(0), B, H, dk, dv,
                      1e-6, gu, N, act, cat.stride(0), hid, _lib.dtype_code(dtype), st())
        else:
            _lib.call('motif_b200_gdn_decode', _lib.ptr(proj), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db),
                      _lib.ptr(cc), _lib.ptr(sd), gate, _lib.ptr(onw), _lib.ptr(cat), cat.stride(0), B, H, dk, dv,
                      1e-6, _lib.dtype_code(dtype), st())
            _lib.call('motif_b200_swiglu', gu, act, B, hid, N, cat.stride(0), _lib.dtype_code(dtype), st())
        outs.append((sd, cc, cat))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    v, gt = proj[:, C + 2 * H + H * dv:].float().split(hid, -1)
    ref = v * F.silu(gt)
    assert rel_err(outs[1][2][:, H * dv:].float(), ref) < (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,T,H,Hkv,D,hid', [(64, 1, 12, 3, 64, 2816), (2, 5, 12, 3, 64, 48), (3, 1, 4, 2, 32, 12)])
def test_chord_prep_swiglu_matches_separate_launches(dtype, B, T, H, Hkv, D, hid):
    """The fused Chord prep + SwiGLU launch writes bit-identical q, cache rows and MLP
    activation to motif_b200_chord_prep followed by motif_b200_swiglu."""
    g = torch.Generator().manual_seed(B + hid)
    N = (H + 2 * Hkv) * D + 2 * hid
    proj = torch.randn(B * T, N, generator=g).to(dtype).cuda()
    qw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).cuda()
    kw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype).cuda()
    cap, pos = T + 9, 4
    gu = proj.data_ptr() + (H + 2 * Hkv) * D * proj.element_size()
    outs = []
    for fused in (False, True):
        qo = torch.empty(B * T, H * D, dtype=dtype, device='cuda')
        kc = torch.zeros(B, Hkv, cap, D, dtype=dtype, device='cuda')
        vc = torch.zeros_like(kc)
        act = torch.full((B * T, hid), 3, dtype=dtype, device='cuda')
        if fused:
            _lib.call('motif_b200_chord_prep_swiglu', _lib.ptr(proj), N, _lib.ptr(qw), _lib.ptr(kw), _lib.ptr(qo),
                      _lib.ptr(kc), _lib.ptr(vc), cap, None, pos, B, T, H, Hkv, D, 1e-6, gu, N, _lib.ptr(act), hid,
                      hid, _lib.dtype_code(dtype), st())
        else:
            _lib.call('motif_b200_chord_prep', _lib.ptr(proj), N, _lib.ptr(qw), _lib.ptr(kw), _lib.ptr(qo),
                      _lib.ptr(kc), _lib.ptr(vc), cap, None, pos, B, T, H, Hkv, D, 1e-6, _lib.dtype_code(dtype), st())
            _lib.call('motif_b200_swiglu', gu, _lib.ptr(act), B * T, hid, N, hid, _lib.dtype_code(dtype), st())
        outs.append((qo, kc, vc, act))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,T,H,Hkv,D,pos', [(2, 5, 12, 3, 64, 0), (3, 1, 4, 2, 16, 17), (1, 33, 8, 8, 32, 4)])
def test_chord_prep(dtype, B, T, H, Hkv, D, pos):
    g = torch.Generator().manual_seed(T + pos)
    N = (H + 2 * Hkv) * D + 24
    proj = torch.randn(B * T, N, generator=g).to(dtype)
    qw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    cap = pos + T + 3
    qo = torch.empty(B * T, H * D, dtype=dtype, device='cuda')
    kc = torch.zeros(B, Hkv, cap, D, dtype=dtype, device='cuda')
    vc = torch.zeros_like(kc)
    # keep every device tensor alive across the call (a temporary's block could be reused)
    pc, qwc, kwc = proj.cuda(), qw.cuda(), kw.cuda()
    _lib.call('motif_b200_chord_prep', _lib.ptr(pc), N, _lib.ptr(qwc), _lib.ptr(kwc),
              _lib.ptr(qo), _lib.ptr(kc), _lib.ptr(vc), cap, None, pos, B, T, H, Hkv, D, 1e-6,
              _lib.dtype_code(dtype), st())
    P = proj.view(B, T, N)
    q = oo.rms_norm(P[..., :H * D].reshape(B, T, H, D), qw)
    k = oo.rms_norm(P[..., H * D:(H + Hkv) * D].reshape(B, T, Hkv, D), kw)
    v = P[..., (H + Hkv) * D:(H + 2 * Hkv) * D].reshape(B, T, Hkv, D)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert rel_err(qo.view(B, T, H, D).float(), q.float()) < tol
    assert rel_err(kc[:, :, pos:pos + T].float(), k.transpose(1, 2).float()) < tol
    assert torch.equal(vc[:, :, pos:pos + T].cpu(), v.transpose(1, 2))
    assert kc[:, :, :pos].abs().sum() == 0 and kc[:, :, pos + T:].abs().sum() == 0


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
@pytest.mark.parametrize('B,H,Hkv,T,S,D,splits', [(2, 12, 3, 1, 1000, 64, 7), (3, 4, 2, 2, 33, 32, 4),
                                                  (1, 8, 8, 1, 5000, 64, 64), (2, 4, 1, 4, 300, 32, 1),
                                                  (2, 8, 2, 2, 8448, 64, 12), (1, 12, 3, 1, 64, 64, 3),
                                                  (1, 16, 2, 2, 777, 64, 5), (2, 12, 3, 1, 8448, 64, 33)])
@pytest.mark.parametrize('scalar', [False, True])
def test_chord_decode(dtype, B, H, Hkv, T, S, D, splits, scalar, request):
    # 16-bit D = 64 runs the tensor-core kernel unless the FORCE_DECODE_SCALAR testing knob is on
    if scalar:
        if dtype == torch.float32 or D != 64:
            pytest.skip('the CUDA-core kernel is the only path for this case')
        _lib.call('motif_b200_testing_force', _lib.FORCE_DECODE_SCALAR, 1)
        request.addfinalizer(lambda: _lib.call('motif_b200_testing_force', _lib.FORCE_DECODE_SCALAR, 0))
    g = torch.Generator().manual_seed(S + T)
    cap = S + 10
    q = torch.randn(B, T, H, D, generator=g).to(dtype)
    kc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)
    vc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)
    # cache slots past the length hold stale data, possibly non-finite: must not leak in
    kc[:, :, S:] = float('nan')
    vc[:, :, S:] = float('nan')
    alpha = 0.5 + 1.5 * torch.rand(H, generator=g)
    beta = torch.rand(H, generator=g)
    mu = torch.ones(H)
    ssmax = 0.8 + 0.4 * torch.rand(H, generator=g)
    q_start = S - T
    log_n = oo.log_n_table(q_start, T).view(1, T).expand(B, T)
    ref = oo.chord_attention(q.transpose(1, 2).float(), kc[:, :, :S].float(), vc[:, :, :S].float(), alpha, beta, mu,
                             ssmax, log_n, q_start)
    out = torch.empty(B * T, H * D, dtype=dtype, device='cuda')
    ws_bytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, splits)
    ws = torch.empty(ws_bytes // 4, device='cuda')
    length = torch.tensor([S], dtype=torch.int32, device='cuda')
    a = [t.cuda() for t in (alpha, beta, mu, ssmax)]
    qc, kcc, vcc = q.cuda(), kc.cuda(), vc.cuda()
    _lib.call('motif_b200_chord_decode', _lib.ptr(qc), _lib.ptr(kcc), _lib.ptr(vcc), cap,
              _lib.ptr(length), 0, *[_lib.ptr(t) for t in a], _lib.ptr(out), H * D, B, H, Hkv, T, D, D ** -0.5,
              1e-5, splits, _lib.ptr(ws), ws_bytes, _lib.dtype_code(dtype), st())
    got = out.view(B, T, H, D).transpose(1, 2).float()
    assert rel_err(got, ref) < (1e-5 if dtype == torch.float32 else 1e-2), rel_err(got, ref)
    assert _lib.wait_timeouts() == 0


def test_decode_advance_matches_torch_ops():
    """One launch = tokens.index_copy_(0, step_idx, ids) + step_idx += 1 + lens += 1, over
    several steps, and no log write once step_idx is past the log."""
    B, steps = 70, 3
    ids = torch.randint(0, 32000, (B,), device='cuda')
    tokens = torch.zeros(steps, B, dtype=torch.int64, device='cuda')
    step_idx = torch.zeros(1, dtype=torch.int64, device='cuda')
    lens = torch.tensor([8192, 8193], dtype=torch.int32, device='cuda')
    ref_tokens = tokens.clone()
    for s in range(steps + 1):
        _lib.call('motif_b200_decode_advance', _lib.ptr(ids), B, _lib.ptr(tokens), steps, _lib.ptr(step_idx),
                  _lib.ptr(lens), 2, st())
        if s < steps:
            ref_tokens[s] = ids
        ids = ids + 1
    torch.cuda.synchronize()
    assert torch.equal(tokens, ref_tokens)
    assert step_idx.item() == steps + 1
    assert lens.tolist() == [8192 + steps + 1, 8193 + steps + 1]


def test_gate_residual_argmax_embed():
    g = torch.Generator().manual_seed(0)
    a, gt, m = (torch.randn(70000, 24, generator=g) for _ in range(3))
    out = torch.empty(70000, 24, device='cuda')
    ac, gc, mc = a.cuda(), gt.cuda(), m.cuda()
    _lib.call('motif_b200_gate_residual', _lib.ptr(ac), 24, _lib.ptr(gc), 24, _lib.ptr(mc), 24,
              _lib.ptr(out), 24, 70000, 24, _lib.MB_F32, st())
    assert rel_err(out, a * torch.sigmoid(gt) + m) < 1e-6
    x = torch.randn(5, 32000, generator=g)
    x[2, 7] = x[2, 9] = x[2].max() + 1  # tie: first index wins, like torch.argmax
    ids = torch.empty(5, dtype=torch.int64, device='cuda')
    xc = x.cuda()
    _lib.call('motif_b200_argmax', _lib.ptr(xc), 5, 32000, 32000, _lib.ptr(ids), _lib.MB_F32, st())
    assert torch.equal(ids.cpu(), x.argmax(-1))
    # 16-bit rows take the vectorised path (V and stride multiples of 8) or the scalar one
    for V, rs in ((32000, 32000), (32000, 32008), (1003, 1003), (40, 48)):
        xb = torch.randn(7, rs, generator=g).to(torch.bfloat16)
        xb[3, 5] = xb[3, V - 2] = xb[3, :V].max() + 1  # tie across a thread's groups
        xb[4, 8] = xb[4, 16] = xb[4, :V].max() + 2
        xb[:, V:] = 100  # past V: never read
        xbc = xb.cuda()
        idb = torch.empty(7, dtype=torch.int64, device='cuda')
        _lib.call('motif_b200_argmax', _lib.ptr(xbc), 7, V, rs, _lib.ptr(idb), _lib.MB_BF16, st())
        assert torch.equal(idb.cpu(), xb[:, :V].float().argmax(-1)), (V, rs)
    table = torch.randn(100, 48, generator=g)
    tok = torch.randint(0, 100, (70000,), generator=g)
    out = torch.empty(70000, 48, device='cuda')
    tc, tbc = tok.cuda(), table.cuda()
    _lib.call('motif_b200_embed', _lib.ptr(tc), _lib.ptr(tbc), _lib.ptr(out), 70000, 48, 100, _lib.MB_F32, st())
    assert torch.equal(out.cpu(), table[tok])


@pytest.mark.parametrize('B,T,H,dk,dv,with_state', [(2, 150, 12, 64, 128, True), (1, 64, 4, 32, 64, False),
                                                    (3, 2, 2, 64, 64, True), (1, 300, 3, 64, 128, False),
                                                    (2, 130, 12, 64, 128, True), (1, 129, 4, 64, 128, False)])
def test_gdn_prefill_fused_matches_two_kernel_path(B, T, H, dk, dv, with_state):
    """motif_b200_gdn_prefill == gdn_prep + gdn_chunk_gated, and both track the fp32 oracle."""
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(T + H)
    C = H * (2 * dk + dv)
    N = (C + 2 * H + H * dv + 24 + 7) // 8 * 8  # projection rows are 16-byte aligned (as packed by the model)
    proj = (0.5 * torch.randn(B, T, N, generator=g)).to(dtype)
    conv_w = (0.3 * torch.randn(C, 4, generator=g)).to(dtype)
    A_log = torch.log(1 + 15 * torch.rand(H, generator=g)).to(dtype)
    dt_bias = (0.1 * torch.randn(H, generator=g)).to(dtype)
    conv_in = (0.5 * torch.randn(B, 3, C, generator=g)).to(dtype)
    s_in = 0.1 * torch.randn(B, H, dk, dv, generator=g) if with_state else None
    onw = (1 + 0.1 * torch.randn(dv, generator=g)).to(dtype)
    p, cw, al, db, ci, ow = (t.cuda() for t in (proj, conv_w, A_log, dt_bias, conv_in, onw))
    si = s_in.cuda() if s_in is not None else None
    M = B * T
    dc, s = _lib.MB_BF16, st()
    # fused
    out1 = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    co1 = torch.empty(B, 3, C, dtype=dtype, device='cuda')
    S1 = torch.empty(B, H, dk, dv, device='cuda')
    _lib.call('motif_b200_gdn_prefill', _lib.ptr(p), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db), _lib.ptr(ci),
              _lib.ptr(co1), _lib.ptr(si), _lib.ptr(S1), _lib.ptr(ow), 1e-6, _lib.ptr(out1), H * dv, B, T, H, dk, dv,
              dc, s)
    # two kernels
    qb = torch.empty(M, H * dk, dtype=dtype, device='cuda')
    kb = torch.empty_like(qb)
    vb = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    be = torch.empty(M, H, device='cuda')
    ge = torch.empty(M, H, device='cuda')
    co2 = torch.empty(B, 3, C, dtype=dtype, device='cuda')
    _lib.call('motif_b200_gdn_prep', _lib.ptr(p), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db), _lib.ptr(ci),
              _lib.ptr(co2), _lib.ptr(qb), _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(be), _lib.ptr(ge), B, T, H, dk, dv, dc, s)
    out2 = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    S2 = torch.empty(B, H, dk, dv, device='cuda')
    strides = [T * H * dk, dk, H * dk, T * H * dk, dk, H * dk, T * H * dv, dv, H * dv,
               T * H * dv, dv, H * dv, T * H, 1, H, T * H, 1, H]
    _lib.call('motif_b200_gdn_chunk_gated', _lib.ptr(qb), _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(be), _lib.ptr(ge),
              _lib.ptr(si), _lib.ptr(S2), _lib.ptr(out2), B, H, T, dk, dv, _lib.i64_array(strides),
              p.data_ptr() + (C + 2 * H) * 2, N, dv, _lib.ptr(ow), 1e-6, dc, s)
    # the same call with a workspace: parallel UT-transform kernel + state-scan kernel
    ws_bytes = _lib.load().motif_b200_gdn_chunk_workspace_bytes(B, H, T, dk, dv, dc)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device='cuda')
    out3 = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    S3 = torch.empty(B, H, dk, dv, device='cuda')
    _lib.call('motif_b200_gdn_chunk_gated_ws', _lib.ptr(qb), _lib.ptr(kb), _lib.ptr(vb), _lib.ptr(be), _lib.ptr(ge),
              _lib.ptr(si), _lib.ptr(S3), _lib.ptr(out3), B, H, T, dk, dv, _lib.i64_array(strides),
              p.data_ptr() + (C + 2 * H) * 2, N, dv, _lib.ptr(ow), 1e-6, dc, _lib.ptr(ws), ws_bytes, s)
    # whole layer with a workspace: preparation fused into the UT-transform kernel
    out4 = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    co4 = torch.empty(B, 3, C, dtype=dtype, device='cuda')
    S4 = torch.empty(B, H, dk, dv, device='cuda')
    _lib.call('motif_b200_gdn_prefill_ws', _lib.ptr(p), N, _lib.ptr(cw), _lib.ptr(al), _lib.ptr(db), _lib.ptr(ci),
              _lib.ptr(co4), _lib.ptr(si), _lib.ptr(S4), _lib.ptr(ow), 1e-6, _lib.ptr(out4), H * dv, B, T, H, dk, dv,
              dc, _lib.ptr(ws), ws_bytes, s)
    torch.cuda.synchronize()
    assert torch.equal(co4, co2)
    if (dk, dv) == (64, 128) and (C + 2 * H) % 8 == 0:
        # same preparation roundings, same split kernels: equal to the split call on prepared inputs
        # (the split prefill takes gate columns on 16-byte boundaries; otherwise it runs the
        # single fused kernel)
        assert rel_err(out4.float(), out3.float()) < 1e-6, rel_err(out4.float(), out3.float())
        assert rel_err(S4, S3) < 1e-6, rel_err(S4, S3)
    else:  # other shapes / alignments run the single fused prefill kernel
        assert torch.equal(out4, out1) and torch.equal(S4, S1)
    assert torch.equal(co1, co2)
    # the split path rounds q e^gamma and k e^(gL - gamma) where the fused kernel rounds the
    # products instead: agreement to the 16-bit operand rounding
    assert rel_err(out3.float(), out2.float()) < 1e-2, rel_err(out3.float(), out2.float())
    assert rel_err(S3, S2) < 5e-3, rel_err(S3, S2)
    assert _lib.wait_timeouts() == 0
    assert rel_err(out1.float(), out2.float()) < 1e-2, rel_err(out1.float(), out2.float())
    assert rel_err(S1, S2) < 1e-3, rel_err(S1, S2)
    # fp32 oracle on the prepared inputs (rounded like the kernels round them)
    q, k, v, beta, gg, _ = gdn_prep_oracle(proj, conv_w, A_log, dt_bias, conv_in, B, T, H, dk, dv)
    o, S = oo.chunk_gated_delta_rule(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), beta.transpose(1, 2),
                                     gg.transpose(1, 2), s_in)
    gate = proj[..., C + 2 * H:C + 2 * H + H * dv].float().view(B, T, H, dv)
    ref = oo.gated_rms_norm(torch.cat([o.transpose(1, 2), gate], -1), onw.float()).reshape(M, H * dv)
    assert rel_err(out1.float(), ref) < 3e-2, rel_err(out1.float(), ref)
    assert rel_err(S1, S) < 2e-2, rel_err(S1, S)


def skinny_pack(w):
    N, K = w.shape
    nbytes = _lib.load().motif_b200_skinny_packed_bytes(N, K)
    assert nbytes == (N + 31) // 32 * 32 * K * 2
    p = torch.empty(nbytes // 2, dtype=w.dtype, device=w.device)
    _lib.call('motif_b200_skinny_pack', w.data_ptr(), w.stride(0), N, K, p.data_ptr(), _lib.dtype_code(w.dtype), st())
    return p


def skinny(x, p, N, y=None, k_warps=0, split_k=0):
    M, K = x.shape
    y = y if y is not None else torch.empty(M, N, dtype=x.dtype, device=x.device)
    _lib.call('motif_b200_skinny_gemm', x.data_ptr(), x.stride(0), p.data_ptr(), y.data_ptr(), y.stride(0), M, N, K,
              k_warps, split_k, _lib.dtype_code(x.dtype), st())
    return y


def within_fp32_product(y, x, w):
    """The kernel accumulates in fp32 and rounds once to the output dtype: each element is
    within one 16-bit rounding of the fp32 product plus a summation-order term."""
    ref = x.float() @ w.float().t()
    err = (y.float() - ref).abs()
    tol = 2.0 ** -7 * ref.abs() + 1e-3 * ref.abs().max()
    return bool((err <= tol).all()), err.max().item()


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M,N,K', [(1, 768, 768), (7, 8728, 768), (64, 768, 3584), (64, 6016, 768),
                                   (33, 768, 2048), (64, 32000, 768), (5, 100, 64), (64, 132, 128), (16, 8728, 768),
                                   (9, 768, 16)])
def test_skinny_gemm_vs_fp32_product(dtype, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    x = (0.5 * torch.randn(M, K, generator=g)).to(dtype).cuda()
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).to(dtype).cuda()
    p = skinny_pack(w)
    outs = []
    for _ in range(2):  # a call leaves no state behind: a repeat gives the same bits
        y = skinny(x, p, N)
        torch.cuda.synchronize()
        ok, e = within_fp32_product(y, x, w)
        assert ok, e
        outs.append(y)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize('k_warps,split_k', [(1, 1), (1, 4), (2, 3), (4, 1), (4, 8), (2, 8), (1, 7)])
def test_skinny_gemm_every_split(k_warps, split_k):
    """Forced splits of K across the warps of a CTA (1, 2, 4) and the CTAs of a cluster (1..8),
    including ragged last parts, all within the fp32 product's bound."""
    M, N, K = 40, 1000, 1536
    g = torch.Generator().manual_seed(k_warps * 10 + split_k)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).bfloat16().cuda()
    p = skinny_pack(w)
    if (K // 16 + split_k - 1) // split_k > 12 * k_warps:
        with pytest.raises(NotImplementedError, match='no split'):
            skinny(x, p, N, k_warps=k_warps, split_k=split_k)
        return
    y = skinny(x, p, N, k_warps=k_warps, split_k=split_k)
    torch.cuda.synchronize()
    ok, e = within_fp32_product(y, x, w)
    assert ok, e


def test_skinny_gemm_strided_rows_and_slices():
    """X a column slice of a wider buffer (ldx > K), Y written into a column slice (ldy > N):
    the columns around the slice are left alone."""
    M, N, K = 64, 768, 2048
    g = torch.Generator().manual_seed(11)
    big_x = torch.randn(M, K + 1536, generator=g).bfloat16().cuda()
    x = big_x[:, 1536:]
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).bfloat16().cuda()
    big_y = torch.full((M, N + 16), 3.0, dtype=torch.bfloat16, device='cuda')
    y = skinny(x, skinny_pack(w), N, y=big_y[:, 8:8 + N])
    torch.cuda.synchronize()
    ok, e = within_fp32_product(y, x, w)
    assert ok, e
    assert bool((big_y[:, :8] == 3).all()) and bool((big_y[:, 8 + N:] == 3).all())


def test_skinny_gemm_decode_shapes_in_a_cuda_graph():
    """The decode step's products back to back on one stream, captured in a CUDA graph (the
    launches carry programmatic-dependent-launch edges there) and replayed: each replay equals
    the eager calls bit for bit, and each product feeds the next (a chain of dependencies)."""
    g = torch.Generator().manual_seed(3)
    M = 64
    shapes = [(8728, 768), (768, 3584), (6016, 768), (768, 2048), (768, 768), (32000, 768)]
    ws = [(K ** -0.5 * torch.randn(N, K, generator=g)).bfloat16().cuda() for N, K in shapes]
    ps = [skinny_pack(w) for w in ws]
    x0 = torch.randn(M, 768, generator=g).bfloat16().cuda()
    bufs = [torch.empty(M, N, dtype=torch.bfloat16, device='cuda') for N, _ in shapes]

    def chain():  # each product reads a column slice of the previous one's output (N >= next K)
        h = x0
        for (N, K), p, out in zip(shapes, ps, bufs):
            skinny(h[:, :K], p, N, y=out)
            h = out

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
        torch.cuda.synchronize()
        eager = [b.clone() for b in bufs]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            chain()
    torch.cuda.current_stream().wait_stream(s)
    for b in bufs:
        b.zero_()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for i, b in enumerate(bufs):
        assert torch.equal(b, eager[i]), i
    ok, e = within_fp32_product(eager[1], eager[0][:, :3584], ws[1])
    assert ok, e
    del graph


def test_skinny_gemm_rejects_bad_arguments():
    x = torch.zeros(65, 64, dtype=torch.bfloat16, device='cuda')
    w = torch.zeros(64, 64, dtype=torch.bfloat16, device='cuda')
    p = skinny_pack(w)
    y = torch.zeros(65, 64, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(NotImplementedError, match='M'):  # M > 64
        _lib.call('motif_b200_skinny_gemm', x.data_ptr(), 64, p.data_ptr(), y.data_ptr(), 64, 65, 64, 64, 0, 0,
                  _lib.MB_BF16, st())
    with pytest.raises(NotImplementedError, match='multiple of 16'):
        _lib.call('motif_b200_skinny_gemm', x.data_ptr(), 64, p.data_ptr(), y.data_ptr(), 64, 8, 64, 40, 0, 0,
                  _lib.MB_BF16, st())
    with pytest.raises(ValueError, match='k_warps'):
        _lib.call('motif_b200_skinny_gemm', x.data_ptr(), 64, p.data_ptr(), y.data_ptr(), 64, 8, 64, 64, 3, 0,
                  _lib.MB_BF16, st())
    with pytest.raises(NotImplementedError, match='16-bit'):
        _lib.call('motif_b200_skinny_gemm', x.data_ptr(), 64, p.data_ptr(), y.data_ptr(), 64, 8, 64, 64, 0, 0,
                  _lib.MB_F32, st())
    assert _lib.load().motif_b200_skinny_packed_bytes(64, 40) == -1


# ------------------------------------------------------------------ attention masks
def _key_bias(B, S, seed, kind):
    """[B, S] fp32 key bias: 'bool' -> 0 / -inf with a dropped run, 'float' -> random additive
    values with some -inf (key 0 is never dropped, so no row loses every key)."""
    g = torch.Generator().manual_seed(seed)
    if kind == 'bool':
        keep = torch.rand(B, S, generator=g) > 0.3
        keep[:, 0] = True
        return torch.zeros(B, S).masked_fill(~keep, float('-inf')), keep
    kb = -3.0 * torch.rand(B, S, generator=g)
    kb[:, 1::7] = float('-inf')
    return kb, kb


def _oracle_masked(q, k, v, alpha, beta, mu, ssmax, q_start, mask):
    from oracle import model as om
    B, H, L, D = q.shape
    log_n = oo.log_n_table(q_start, L)
    m4 = mask[:, None, None, :]
    return om._chord_masked(q, k, v, alpha, beta, mu, ssmax, log_n, q_start, D, m4)


@pytest.mark.parametrize('kind', ['bool', 'float'])
@pytest.mark.parametrize('dtype,B,H,Hkv,L,S,D', [
    (torch.bfloat16, 2, 12, 3, 300, 300, 64),    # tcgen05 kernel
    (torch.bfloat16, 1, 8, 2, 130, 400, 64),     # tcgen05, q_start > 0
    (torch.float16, 2, 4, 2, 70, 70, 32),        # 16-bit D = 32: the simple kernel takes masks
    (torch.float32, 2, 4, 4, 50, 90, 64),        # fp32
])
def test_chord_prefill_masked(kind, dtype, B, H, Hkv, L, S, D):
    g = torch.Generator().manual_seed(L + S + D)
    q = torch.randn(B, H, L, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, S, D, generator=g).to(dtype)
    alpha = 0.5 + 1.5 * torch.rand(H, generator=g)
    beta = torch.rand(H, generator=g)
    mu = torch.ones(H) + 0.5 * torch.randn(H, generator=g)
    ssmax = 0.8 + 0.4 * torch.rand(H, generator=g)
    ssmax[::3] *= -1.0
    qs = S - L
    kb, mask = _key_bias(B, S, seed=S, kind=kind)
    ref = _oracle_masked(q.float(), k.float(), v.float(), alpha, beta, mu, ssmax, qs, mask)
    log_n = oo.log_n_table(qs, L).view(1, L).expand(B, L).contiguous()
    qc, kc, vc, lc, kbc = q.cuda(), k.cuda(), v.cuda(), log_n.cuda(), kb.cuda()
    a = [t.cuda() for t in (alpha, beta, mu, ssmax)]
    out = torch.empty_like(qc)
    strides = [*qc.stride()[:3], *kc.stride()[:3], *vc.stride()[:3], *out.stride()[:3], *lc.stride()]
    _lib.call('motif_b200_chord_attention_masked', _lib.ptr(qc), _lib.ptr(kc), _lib.ptr(vc),
              *[_lib.ptr(t) for t in a], _lib.ptr(lc), _lib.ptr(out), B, H, Hkv, L, S, D, qs, D ** -0.5, 1e-5,
              _lib.i64_array(strides), _lib.ptr(kbc), S, _lib.dtype_code(dtype), st())
    assert torch.isfinite(out).all()
    assert rel_err(out.float(), ref) < (1e-5 if dtype == torch.float32 else 1e-2), rel_err(out.float(), ref)
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize('kind', ['bool', 'float'])
@pytest.mark.parametrize('dtype,B,H,Hkv,T,S,D', [
    (torch.bfloat16, 3, 12, 3, 1, 700, 64),   # tensor-core decode
    (torch.bfloat16, 2, 8, 2, 2, 300, 32),    # CUDA-core decode
    (torch.float32, 2, 4, 2, 1, 257, 64),
])
def test_chord_decode_masked(kind, dtype, B, H, Hkv, T, S, D):
    g = torch.Generator().manual_seed(S + T)
    cap = S + 10
    q = torch.randn(B, T, H, D, generator=g).to(dtype)
    kc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)
    vc = torch.randn(B, Hkv, cap, D, generator=g).to(dtype)
    alpha = 0.5 + 1.5 * torch.rand(H, generator=g)
    beta = torch.rand(H, generator=g)
    mu = torch.ones(H)
    ssmax = 0.8 + 0.4 * torch.rand(H, generator=g)
    qs = S - T
    kb, mask = _key_bias(B, S, seed=S + 1, kind=kind)
    ref = _oracle_masked(q.transpose(1, 2).float(), kc[:, :, :S].float(), vc[:, :, :S].float(), alpha, beta, mu,
                         ssmax, qs, mask)
    splits = 4
    out = torch.empty(B * T, H * D, dtype=dtype, device='cuda')
    ws_bytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, splits)
    ws = torch.empty(ws_bytes // 4, device='cuda')
    a = [t.cuda() for t in (alpha, beta, mu, ssmax)]
    qc, kcc, vcc, kbc = q.cuda(), kc.cuda(), vc.cuda(), kb.cuda()
    _lib.call('motif_b200_chord_decode_masked', _lib.ptr(qc), _lib.ptr(kcc), _lib.ptr(vcc), cap, None, S,
              *[_lib.ptr(t) for t in a], _lib.ptr(out), H * D, B, H, Hkv, T, D, D ** -0.5, 1e-5, splits,
              _lib.ptr(kbc), S, _lib.ptr(ws), ws_bytes, _lib.dtype_code(dtype), st())
    got = out.view(B, T, H, D).transpose(1, 2).float()
    assert rel_err(got, ref) < (1e-5 if dtype == torch.float32 else 1e-2), rel_err(got, ref)
    assert _lib.wait_timeouts() == 0


def test_chord_masked_all_keys_dropped_gives_zeros():
    """A row whose every visible key is dropped yields zeros (the reference's softmax gives NaN)."""
    B, H, Hkv, L, S, D = 1, 4, 4, 8, 8, 64
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(B, n, L, D, generator=g).bfloat16().cuda() for n in (H, Hkv, Hkv))
    kb = torch.zeros(B, S)
    kb[0, :4] = float('-inf')  # rows 0..3 see only keys 0..their own position
    a = [t.cuda() for t in (torch.ones(H), torch.full((H,), 0.5), torch.ones(H), torch.ones(H))]
    log_n = oo.log_n_table(0, L).view(1, L).contiguous().cuda()
    out = torch.full_like(q, 7.0)
    strides = [*q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *out.stride()[:3], *log_n.stride()]
    _lib.call('motif_b200_chord_attention_masked', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), *[_lib.ptr(t) for t in a],
              _lib.ptr(log_n), _lib.ptr(out), B, H, Hkv, L, S, D, 0, D ** -0.5, 1e-5, _lib.i64_array(strides),
              _lib.ptr(kb.cuda()), S, _lib.dtype_code(torch.bfloat16), st())
    assert bool((out[:, :, :4] == 0).all()) and torch.isfinite(out).all()
    assert bool((out[:, :, 4:].abs().sum(-1) > 0).all())


@pytest.mark.parametrize('B,H,T,dk,dv,with_state', [(2, 12, 300, 64, 128, True), (1, 12, 4096, 64, 128, False),
                                                    (1, 3, 70, 64, 128, True)])
def test_gdn_split_narrow_slices_equal_wide(B, H, T, dk, dv, with_state):
    """Tiny batches scan 32-column value slices (twice the CTAs of the 64-column ones); the
    columns of the state evolve independently, so both slicings give the same bits, for the
    whole-layer prefill (preparation fused) and the split call on prepared inputs."""
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(B * T + dv)
    C = H * (2 * dk + dv)
    N = C + 2 * H + H * dv
    N += (-N) % 8
    proj = (0.5 * torch.randn(B * T, N, generator=g)).to(dtype).cuda()
    conv_w = (0.3 * torch.randn(C, 4, generator=g)).to(dtype).cuda()
    A_log = torch.log(1 + 15 * torch.rand(H, generator=g)).to(dtype).cuda()
    dt_bias = (0.1 * torch.randn(H, generator=g)).to(dtype).cuda()
    conv_in = (0.5 * torch.randn(B, 3, C, generator=g)).to(dtype).cuda()
    s_in = (0.1 * torch.randn(B, H, dk, dv, generator=g)).cuda() if with_state else None
    onw = (1 + 0.1 * torch.randn(dv, generator=g)).to(dtype).cuda()
    dc, s = _lib.MB_BF16, st()
    M = B * T

    def layer():
        ws_bytes = _lib.load().motif_b200_gdn_chunk_workspace_bytes(B, H, T, dk, dv, dc)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device='cuda')
        out = torch.empty(M, H * dv, dtype=dtype, device='cuda')
        co = torch.empty(B, 3, C, dtype=dtype, device='cuda')
        S = torch.empty(B, H, dk, dv, device='cuda')
        _lib.call('motif_b200_gdn_prefill_ws', _lib.ptr(proj), N, _lib.ptr(conv_w), _lib.ptr(A_log),
                  _lib.ptr(dt_bias), _lib.ptr(conv_in), _lib.ptr(co), _lib.ptr(s_in), _lib.ptr(S), _lib.ptr(onw), 1e-6,
                  _lib.ptr(out), H * dv, B, T, H, dk, dv, dc, _lib.ptr(ws), ws_bytes, s)
        torch.cuda.synchronize()
        return out, S

    narrow = layer()
    with _lib.forced(_lib.FORCE_GDN_WIDE):
        wide = layer()
    assert torch.equal(narrow[0], wide[0]) and torch.equal(narrow[1], wide[1])
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize('B,H,L,dk,dv', [(2, 4, 300, 64, 64), (2, 12, 1000, 64, 64), (1, 2, 130, 32, 64)])
def test_gdn_chunk_op_narrow_slices_equal_wide(B, H, L, dk, dv):
    """The chunked delta-rule op (config 2's shape family) through the split path: 32- and
    64-column scan slices give the same bits."""
    from motif_b200 import ops
    g = torch.Generator().manual_seed(L + B)
    q = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1).bfloat16().cuda()
    k = torch.nn.functional.normalize(torch.randn(B, H, L, dk, generator=g), dim=-1).bfloat16().cuda()
    v = torch.randn(B, H, L, dv, generator=g).bfloat16().cuda()
    beta = torch.rand(B, H, L, generator=g).cuda()
    gg = (-0.2 * torch.rand(B, H, L, generator=g)).cuda()
    S0 = (0.1 * torch.randn(B, H, dk, dv, generator=g)).cuda()
    o1, s1 = ops.chunk_gated_delta_rule(q, k, v, beta, gg, S0)
    with _lib.forced(_lib.FORCE_GDN_WIDE):
        o2, s2 = ops.chunk_gated_delta_rule(q, k, v, beta, gg, S0)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
