"""The allocation-free split-KV decode entry point against the workspace one.

`motif_b200_chord_decode_noalloc` serves callers that cannot allocate device memory: it
keeps its split partials in a fixed device array inside the library instead of a
caller-provided workspace.  Both entry points run the same kernels with the same split
count, so their outputs must be bit-identical.  This file runs last (pytest collects it after
every other test file), so a failure here leaves every other test already run.
"""

import pytest
import torch

from motif_b200 import _lib

pytestmark = pytest.mark.gpu

B, H, HKV, T = 4, 12, 3, 1
SCRATCH_BYTES = 8 << 20   # the fixed scratch array of the library


def inputs(S, seed, dtype, D):
    g = torch.Generator().manual_seed(seed)
    cap = S + 16
    q = torch.randn(B * T, H * D, generator=g).to(dtype).cuda()
    k = torch.randn(B, HKV, cap, D, generator=g).to(dtype).cuda()
    v = torch.randn(B, HKV, cap, D, generator=g).to(dtype).cuda()
    params = [(0.5 + 1.5 * torch.rand(H, generator=g)).cuda(), torch.rand(H, generator=g).cuda(),
              torch.ones(H).cuda(), (0.8 + 0.4 * torch.rand(H, generator=g)).cuda()]
    length = torch.tensor([S], dtype=torch.int32, device='cuda')
    return dict(q=q, k=k, v=v, cap=cap, params=params, length=length, S=S, D=D, dtype=dtype)


def _len_args(a, host_len):
    return (None, a['S']) if host_len else (_lib.ptr(a['length']), 0)


def with_workspace(a, splits, host_len=False):
    D, dt = a['D'], a['dtype']
    out = torch.empty(B * T, H * D, dtype=dt, device='cuda')
    nbytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, splits)
    ws = torch.empty(nbytes // 4, device='cuda')
    _lib.call('motif_b200_chord_decode', _lib.ptr(a['q']), _lib.ptr(a['k']), _lib.ptr(a['v']), a['cap'],
              *_len_args(a, host_len), *[_lib.ptr(p) for p in a['params']], _lib.ptr(out), H * D, B, H, HKV, T, D,
              D ** -0.5, 1e-5, splits, _lib.ptr(ws), nbytes, _lib.dtype_code(dt), _lib.stream_ptr())
    return out


def without_workspace(a, splits, host_len=False):
    D, dt = a['D'], a['dtype']
    out = torch.empty(B * T, H * D, dtype=dt, device='cuda')
    _lib.call('motif_b200_chord_decode_noalloc', _lib.ptr(a['q']), _lib.ptr(a['k']), _lib.ptr(a['v']), a['cap'],
              *_len_args(a, host_len), *[_lib.ptr(p) for p in a['params']], _lib.ptr(out), H * D, B, H, HKV, T, D,
              D ** -0.5, 1e-5, splits, _lib.dtype_code(dt), _lib.stream_ptr())
    return out


@pytest.mark.parametrize('dtype,D', [(torch.bfloat16, 64), (torch.float32, 64), (torch.bfloat16, 32)])
@pytest.mark.parametrize('host_len', [False, True])
def test_noalloc_decode_matches_workspace_decode_twice(dtype, D, host_len):
    """Two calls in a row (different inputs and lengths) both equal the workspace path bit for
    bit: the tensor-core kernel (bf16, D = 64), the CUDA-core kernel (fp32; D = 32), with the
    cache length read from device memory or passed by the host."""
    for S, seed, splits in ((1000, 1, 12), (333, 2, 5)):
        a = inputs(S, seed, dtype, D)
        ref = with_workspace(a, splits, host_len)
        got = without_workspace(a, splits, host_len)
        torch.cuda.synchronize()
        assert torch.isfinite(ref).all()
        assert torch.equal(got, ref)


def test_noalloc_largest_split_count_that_fits():
    """The limit is inclusive: the largest split count whose partials fit the scratch runs and
    matches the workspace path; one split more is rejected before anything is launched."""
    D = 64
    per_split = B * H * T * (D + 2) * 4
    most = SCRATCH_BYTES // per_split
    assert _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, most) <= SCRATCH_BYTES
    a = inputs(1000, 4, torch.bfloat16, D)
    assert torch.equal(without_workspace(a, most), with_workspace(a, most))
    with pytest.raises(ValueError, match='limit'):
        without_workspace(a, most + 1)


def test_noalloc_rejects_oversized_requests():
    a = inputs(64, 3, torch.bfloat16, 64)
    with pytest.raises(ValueError, match='limit'):
        without_workspace(a, 1024)
