"""The tensor-core decode GEMM (`motif_b200_skinny_gemm_tc`): Y = X W^T for 1..64 token rows on
the weight itself, against the fp32 product, across splits of K over a cluster, strided
operands, and a chain of the decode step's products captured in a CUDA graph."""

import pytest
import torch

from motif_b200 import _lib

pytestmark = pytest.mark.gpu


def st():
    return _lib.stream_ptr()


def tc(x, w, y=None, split_k=0):
    M, K = x.shape
    N = w.shape[0]
    y = y if y is not None else torch.empty(M, N, dtype=x.dtype, device=x.device)
    _lib.call('motif_b200_skinny_gemm_tc', x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(),
              y.stride(0), M, N, K, split_k, _lib.dtype_code(x.dtype), st())
    return y


def within_fp32_product(y, x, w):
    """fp32 accumulation rounded once to the output dtype: each element is within one 16-bit
    rounding of the fp32 product plus a summation-order term."""
    ref = x.float() @ w.float().t()
    err = (y.float() - ref).abs()
    tol = 2.0 ** -7 * ref.abs() + 1e-3 * ref.abs().max()
    return bool((err <= tol).all()), err.max().item()


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M,N,K', [(64, 8728, 768), (64, 768, 3584), (64, 6016, 768), (64, 768, 768),
                                   (64, 768, 2048), (64, 32000, 768), (33, 768, 2048), (48, 1000, 1536),
                                   (1, 768, 768), (7, 132, 64), (64, 4, 128)])
def test_skinny_tc_vs_fp32_product(dtype, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    x = (0.5 * torch.randn(M, K, generator=g)).to(dtype).cuda()
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).to(dtype).cuda()
    outs = []
    for _ in range(2):  # a call leaves no state behind: a repeat gives the same bits
        y = tc(x, w)
        torch.cuda.synchronize()
        ok, e = within_fp32_product(y, x, w)
        assert ok, e
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize('split_k', [1, 2, 3, 5, 7, 8])
@pytest.mark.parametrize('M', [64, 40, 3])
def test_skinny_tc_every_split(split_k, M):
    """Forced splits of K over 1..8 CTAs of a cluster, with ragged last parts (K = 1536 is 24
    blocks of 64) and token rows that do not divide evenly among the CTAs (some own none when
    M < S)."""
    N, K = 1000, 1536
    g = torch.Generator().manual_seed(split_k * 100 + M)
    x = torch.randn(M, K, generator=g).bfloat16().cuda()
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).bfloat16().cuda()
    kbt = K // 64
    kbc = -(-kbt // split_k)
    if -(-kbt // kbc) != split_k:  # this split has the same parts as a smaller one
        with pytest.raises(NotImplementedError, match='no split'):
            tc(x, w, split_k=split_k)
        return
    y = tc(x, w, split_k=split_k)
    torch.cuda.synchronize()
    ok, e = within_fp32_product(y, x, w)
    assert ok, e
    # the sum over the cluster's partials runs in rank order: the same bits on a repeat
    assert torch.equal(y, tc(x, w, split_k=split_k))
    assert _lib.wait_timeouts() == 0


def test_skinny_tc_strided_rows_and_slices():
    """X a column slice of a wider buffer (ldx > K), W a row-strided view (ldw > K), Y written
    into a column slice (ldy > N): the columns around the slice are left alone."""
    M, N, K = 64, 768, 2048
    g = torch.Generator().manual_seed(11)
    big_x = torch.randn(M, K + 1536, generator=g).bfloat16().cuda()
    x = big_x[:, 1536:]
    big_w = (K ** -0.5 * torch.randn(N, K + 64, generator=g)).bfloat16().cuda()
    w = big_w[:, 64:]
    big_y = torch.full((M, N + 16), 3.0, dtype=torch.bfloat16, device='cuda')
    y = tc(x, w, y=big_y[:, 8:8 + N])
    torch.cuda.synchronize()
    ok, e = within_fp32_product(y, x, w)
    assert ok, e
    assert bool((big_y[:, :8] == 3).all()) and bool((big_y[:, 8 + N:] == 3).all())


def test_skinny_tc_decode_shapes_in_a_cuda_graph():
    """The decode step's products back to back on one stream, captured in a CUDA graph (the
    launches carry programmatic-dependent-launch edges there) and replayed: each replay equals
    the eager calls bit for bit, and each product feeds the next (a chain of dependencies)."""
    g = torch.Generator().manual_seed(3)
    M = 64
    shapes = [(8728, 768), (768, 3584), (6016, 768), (768, 2048), (768, 768), (32000, 768)]
    ws = [(K ** -0.5 * torch.randn(N, K, generator=g)).bfloat16().cuda() for N, K in shapes]
    x0 = torch.randn(M, 768, generator=g).bfloat16().cuda()
    bufs = [torch.empty(M, N, dtype=torch.bfloat16, device='cuda') for N, _ in shapes]

    def chain():  # each product reads a column slice of the previous one's output (N >= next K)
        h = x0
        for (N, K), w, out in zip(shapes, ws, bufs):
            tc(h[:, :K], w, y=out)
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
    assert _lib.wait_timeouts() == 0


def test_skinny_tc_rejects_bad_arguments():
    x = torch.zeros(65, 128, dtype=torch.bfloat16, device='cuda')
    w = torch.zeros(64, 128, dtype=torch.bfloat16, device='cuda')
    y = torch.zeros(65, 64, dtype=torch.bfloat16, device='cuda')

    def call(M, N, K, split_k=0, dtype=_lib.MB_BF16, ldx=128):
        _lib.call('motif_b200_skinny_gemm_tc', x.data_ptr(), ldx, w.data_ptr(), 128, y.data_ptr(), 64, M, N, K,
                  split_k, dtype, st())

    with pytest.raises(NotImplementedError, match='M'):  # M > 64
        call(65, 64, 128)
    with pytest.raises(NotImplementedError, match='multiple of 64'):
        call(8, 64, 96)
    with pytest.raises(ValueError, match='split_k'):
        call(8, 64, 128, split_k=9)
    with pytest.raises(NotImplementedError, match='16-bit'):
        call(8, 64, 128, dtype=_lib.MB_F32)
    with pytest.raises(ValueError, match='aligned'):
        call(8, 64, 128, ldx=130)



@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M,K,split_k', [(64, 2048, 0), (40, 2048, 3), (64, 768, 0), (33, 2816, 8)])
def test_skinny_tc_add_gated_equals_product_then_gate_residual(dtype, M, K, split_k):
    """The Chord decoder's down_proj with the gated residual in the epilogue gives the same bits
    as the product followed by the separate gate-residual kernel, with the gate a column slice
    of a wider projection row (as in the model), on two calls in a row."""
    N, N_in, off_g = 768, 6016, 1152
    g = torch.Generator().manual_seed(M * 7 + K)
    x = torch.randn(M, K, generator=g).to(dtype).cuda()
    w = (K ** -0.5 * torch.randn(N, K, generator=g)).to(dtype).cuda()
    a = torch.randn(M, N, generator=g).to(dtype).cuda()
    proj = (2 * torch.randn(M, N_in, generator=g)).to(dtype).cuda()
    gate = proj[:, off_g:off_g + N]
    ref = tc(x, w, split_k=split_k)
    _lib.call('motif_b200_gate_residual', a.data_ptr(), N, gate.data_ptr(), N_in, ref.data_ptr(), N, ref.data_ptr(), N,
              M, N, _lib.dtype_code(dtype), st())
    for _ in range(2):
        y = torch.full((M, N), float('nan'), dtype=dtype, device='cuda')
        _lib.call('motif_b200_skinny_gemm_tc_add_gated', x.data_ptr(), K, w.data_ptr(), K, a.data_ptr(), N,
                  gate.data_ptr(), N_in, y.data_ptr(), N, M, N, K, split_k, _lib.dtype_code(dtype), st())
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    assert _lib.wait_timeouts() == 0


def test_skinny_tc_add_gated_rejects_misaligned_gate():
    x = torch.zeros(64, 2048, dtype=torch.bfloat16, device='cuda')
    w = torch.zeros(768, 2048, dtype=torch.bfloat16, device='cuda')
    a = torch.zeros(64, 768, dtype=torch.bfloat16, device='cuda')
    proj = torch.zeros(64, 6016, dtype=torch.bfloat16, device='cuda')
    y = torch.zeros(64, 768, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(ValueError, match='aligned'):  # the gate starts 2 bytes past an 8-byte boundary
        _lib.call('motif_b200_skinny_gemm_tc_add_gated', x.data_ptr(), 2048, w.data_ptr(), 2048, a.data_ptr(), 768,
                  proj.data_ptr() + 2, 6016, y.data_ptr(), 768, 64, 768, 2048, 0, _lib.MB_BF16, st())


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('M', [64, 33, 8, 1])
def test_skinny_tc_chord_tail(dtype, M):
    """The Chord decoder's tail in one launch, y = o_proj(attn) * sigmoid(g) + down_proj(act) with
    the unfused path's rounding points, against the fp32 products rounded where the separate
    kernels round (each product within one 16-bit rounding plus a summation-order term), on
    two calls in a row that give the same bits."""
    N, K1, K2, N_in, off_g = 768, 768, 2048, 6016, 1152
    g = torch.Generator().manual_seed(M + 5)
    x1 = torch.randn(M, K1, generator=g).to(dtype).cuda()
    w1 = (K1 ** -0.5 * torch.randn(N, K1, generator=g)).to(dtype).cuda()
    x2 = torch.randn(M, K2, generator=g).to(dtype).cuda()
    w2 = (K2 ** -0.5 * torch.randn(N, K2, generator=g)).to(dtype).cuda()
    proj = (2 * torch.randn(M, N_in, generator=g)).to(dtype).cuda()
    gate = proj[:, off_g:off_g + N]
    outs = []
    for _ in range(2):
        y = torch.full((M, N), float('nan'), dtype=dtype, device='cuda')
        _lib.call('motif_b200_skinny_gemm_tc_chord_tail', x1.data_ptr(), K1, w1.data_ptr(), K1, K1, x2.data_ptr(), K2,
                  w2.data_ptr(), K2, K2, gate.data_ptr(), N_in, y.data_ptr(), N, M, N, _lib.dtype_code(dtype), st())
        torch.cuda.synchronize()
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    p1 = x1.float() @ w1.float().t()
    p2 = x2.float() @ w2.float().t()
    sg = torch.sigmoid(gate.float()).to(dtype).float()
    att = (p1.to(dtype).float() * sg).to(dtype).float()
    mlp = p2.to(dtype).float()
    ref = att + mlp
    err = (outs[0].float() - ref).abs()
    # a few 16-bit roundings of each part (the sum may cancel, so the bound follows the parts)
    tol = 2.0 ** -6 * (att.abs() + mlp.abs()) + 1e-3
    assert bool((err <= tol).all()), err.max().item()
    assert _lib.wait_timeouts() == 0
