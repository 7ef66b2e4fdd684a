"""The tcgen05 projection kernels (`motif_b200_gemm`, `_gemm_proj_swiglu`, `_gemm_gate_residual`)
through the C ABI.

* plain: against a fp32 product of the same 16-bit operands (the kernels accumulate in fp32 and
  round once to the output dtype), over partial row / feature tiles, long K, fp16 and bf16;
* fused epilogues: bit-identical to the plain kernel followed by the separate elementwise kernel
  (`motif_b200_swiglu`, `motif_b200_gate_residual`): the accumulator of an output element does
  not depend on which tile holds it, and the epilogue rounds where those kernels round.
"""

import pytest
import torch

from motif_b200 import _lib

pytestmark = pytest.mark.gpu


def st():
    return _lib.stream_ptr()


def gemm(x, w, out=None):
    M, K = x.shape
    N = w.shape[0]
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    _lib.call('motif_b200_gemm', _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(y), y.stride(0), M, N,
              K, _lib.dtype_code(x.dtype), st())
    return y


def operands(M, N, K, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=g) * 0.5).to(dtype).cuda()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).to(dtype).cuda()
    return x, w


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M,N,K', [(1000, 768, 768), (257, 8728, 768), (131, 32000, 768), (384, 300, 192),
                                   (128, 24, 64), (512, 768, 3584), (65, 4632, 768), (4096, 1920, 768)])
def test_gemm_matches_fp32_product(dtype, M, N, K):
    x, w = operands(M, N, K, dtype, M + N + K)
    y = gemm(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    err = (y.float() - ref).abs()
    tol = 2.0 ** -7 * ref.abs() + 1e-3 * ref.abs().max()
    assert bool((err <= tol).all()), (err.max().item(), ref.abs().max().item())
    assert _lib.wait_timeouts() == 0


def test_gemm_strided_output_and_repeat_is_deterministic():
    """Writes into a column slice of a wider buffer (row stride > N); a second call is bit-identical."""
    x, w = operands(700, 520, 256, torch.bfloat16, 3)
    big = torch.full((700, 1040), 7.0, dtype=torch.bfloat16, device='cuda')
    a = gemm(x, w, big[:, 8:528])
    b = gemm(x, w)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert bool((big[:, :8] == 7).all()) and bool((big[:, 528:] == 7).all())


def interleave(gu, hid):
    v, g = gu[:hid].view(hid // 128, 128, -1), gu[hid:].view(hid // 128, 128, -1)
    return torch.cat([v, g], 1).reshape(2 * hid, -1).contiguous()


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M,n_plain,hid,K', [(1000, 4632, 2048, 768), (300, 1920, 768, 256), (129, 0, 256, 64),
                                             (200, 72, 384, 128)])
def test_proj_swiglu_equals_plain_then_swiglu(dtype, M, n_plain, hid, K):
    x, w = operands(M, n_plain + 2 * hid, K, dtype, M + hid)
    w_il = torch.cat([w[:n_plain], interleave(w[n_plain:], hid)], 0).contiguous()
    y = torch.empty((M, max(n_plain, 8)), dtype=dtype, device='cuda')
    act = torch.empty((M, hid), dtype=dtype, device='cuda')
    _lib.call('motif_b200_gemm_proj_swiglu', _lib.ptr(x), x.stride(0), _lib.ptr(w_il), w_il.stride(0), M, K, n_plain,
              _lib.ptr(y), y.stride(0), hid, _lib.ptr(act), act.stride(0), _lib.dtype_code(dtype), st())
    full = gemm(x, w)  # natural layout: [plain | values | gates]
    ref_act = torch.empty_like(act)
    _lib.call('motif_b200_swiglu', full.data_ptr() + n_plain * full.element_size(), _lib.ptr(ref_act), M, hid,
              full.stride(0), ref_act.stride(0), _lib.dtype_code(dtype), st())
    torch.cuda.synchronize()
    if n_plain:
        assert torch.equal(y[:, :n_plain], full[:, :n_plain])
    assert torch.equal(act, ref_act)
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize('M,N,K', [(1000, 768, 768), (257, 256, 512), (130, 200, 64)])
def test_gate_residual_equals_plain_then_gate_residual(M, N, K):
    dtype = torch.bfloat16
    x, w = operands(M, N, K, dtype, M + 11 * N)
    g = torch.Generator().manual_seed(N)
    gate = torch.randn(M, N, generator=g).to(dtype).cuda()
    res = torch.randn(M, N, generator=g).to(dtype).cuda()
    out = torch.empty_like(res)
    _lib.call('motif_b200_gemm_gate_residual', _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(gate),
              gate.stride(0), _lib.ptr(res), res.stride(0), _lib.ptr(out), out.stride(0), M, N, K,
              _lib.dtype_code(dtype), st())
    a = gemm(x, w)
    ref = torch.empty_like(res)
    _lib.call('motif_b200_gate_residual', _lib.ptr(a), a.stride(0), _lib.ptr(gate), gate.stride(0), _lib.ptr(res),
              res.stride(0), _lib.ptr(ref), ref.stride(0), M, N, _lib.dtype_code(dtype), st())
    # in place (out aliases the residual), as the model calls it
    inplace = res.clone()
    _lib.call('motif_b200_gemm_gate_residual', _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(gate),
              gate.stride(0), _lib.ptr(inplace), inplace.stride(0), _lib.ptr(inplace), inplace.stride(0), M, N, K,
              _lib.dtype_code(dtype), st())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.equal(inplace, ref)


def test_gemm_rejects_bad_arguments():
    x, w = operands(128, 128, 96, torch.bfloat16, 0)
    y = torch.empty((128, 128), dtype=torch.bfloat16, device='cuda')
    with pytest.raises(NotImplementedError, match='multiple of 64'):
        _lib.call('motif_b200_gemm', _lib.ptr(x), 96, _lib.ptr(w), 96, _lib.ptr(y), 128, 128, 128, 96, _lib.MB_BF16,
                  st())
    xf = torch.randn(128, 128, device='cuda')
    with pytest.raises(NotImplementedError, match='16-bit'):
        _lib.call('motif_b200_gemm', _lib.ptr(xf), 128, _lib.ptr(xf), 128, _lib.ptr(xf), 128, 128, 128, 128,
                  _lib.MB_F32, st())


@pytest.mark.parametrize('B,T,with_state', [(2, 130, False), (1, 4096, True), (3, 3, True), (64, 5, False),
                                            (2, 64, True)])
def test_gdn_prep_equals_plain_then_prep_kernel(B, T, with_state):
    """The GDN projection with the layer's preparation fused (125-row tiles with a 3-row halo)
    against the plain projection followed by the separate preparation kernel: v, the gate, beta,
    g, the SwiGLU and the conv state bit-identical; q / k within one bf16 rounding (their
    per-head sum of squares is accumulated in another order)."""
    dtype = torch.bfloat16
    H, dk, dv, hid, d = 12, 64, 128, 2048, 768
    C = H * (2 * dk + dv)
    n_plain = 2 * H * dk + H * dv + 2 * H + H * dv
    g_ = torch.Generator().manual_seed(B * T)
    M = B * T
    x = (torch.randn(M, d, generator=g_) * 0.5).to(dtype).cuda()
    w = (torch.randn(n_plain + 2 * hid, d, generator=g_) * d ** -0.5).to(dtype).cuda()
    w_il = torch.cat([w[:n_plain], interleave(w[n_plain:], hid)], 0).contiguous()
    conv_w = (torch.randn(C, 4, generator=g_) * 0.5).to(dtype).cuda()
    A_log = torch.rand(H, generator=g_).to(dtype).cuda()
    dt_bias = (torch.randn(H, generator=g_) * 0.5).to(dtype).cuda()
    conv_in = (torch.randn(B, 3, C, generator=g_)).to(dtype).cuda() if with_state else None

    def outs():
        return dict(q=torch.empty(M, H * dk, dtype=dtype, device='cuda'), k=torch.empty(M, H * dk, dtype=dtype, device='cuda'),
                    v=torch.empty(M, H * dv, dtype=dtype, device='cuda'), beta=torch.empty(M, H, device='cuda'),
                    g=torch.empty(M, H, device='cuda'), conv=torch.empty(B, 3, C, dtype=dtype, device='cuda'))
    a = outs()
    gate = torch.empty(M, H * dv, dtype=dtype, device='cuda')
    act = torch.empty(M, hid, dtype=dtype, device='cuda')
    _lib.call('motif_b200_gemm_gdn_prep', _lib.ptr(x), d, _lib.ptr(w_il), d, B, T, d, H, dk, dv, hid, _lib.ptr(conv_w),
              _lib.ptr(A_log), _lib.ptr(dt_bias), _lib.ptr(conv_in), _lib.ptr(a['conv']), _lib.ptr(a['q']),
              _lib.ptr(a['k']), _lib.ptr(a['v']), _lib.ptr(a['beta']), _lib.ptr(a['g']), _lib.ptr(gate), _lib.ptr(act),
              hid, _lib.MB_BF16, st())
    proj = gemm(x, w)
    b = outs()
    _lib.call('motif_b200_gdn_prep', _lib.ptr(proj), proj.stride(0), _lib.ptr(conv_w), _lib.ptr(A_log),
              _lib.ptr(dt_bias), _lib.ptr(conv_in), _lib.ptr(b['conv']), _lib.ptr(b['q']), _lib.ptr(b['k']),
              _lib.ptr(b['v']), _lib.ptr(b['beta']), _lib.ptr(b['g']), B, T, H, dk, dv, _lib.MB_BF16, st())
    ref_act = torch.empty_like(act)
    _lib.call('motif_b200_swiglu', proj.data_ptr() + n_plain * proj.element_size(), _lib.ptr(ref_act), M, hid,
              proj.stride(0), hid, _lib.MB_BF16, st())
    torch.cuda.synchronize()
    for name in ('v', 'beta', 'g', 'conv'):
        assert torch.equal(a[name], b[name]), name
    assert torch.equal(gate, proj[:, 2 * H * dk + H * dv + 2 * H:n_plain])
    assert torch.equal(act, ref_act)
    for name in ('q', 'k'):
        err = (a[name].float() - b[name].float()).abs()
        assert bool((err <= 2.0 ** -7 * b[name].float().abs() + 1e-6).all()), (name, err.max().item())
    assert _lib.wait_timeouts() == 0
