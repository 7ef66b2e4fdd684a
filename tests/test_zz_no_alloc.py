"""The allocation-free split-KV decode entry point against the workspace one.

`motif_b200_chord_decode_noalloc` serves callers that cannot allocate device memory: it
keeps its split partials in a fixed device array inside the library instead of a
caller-provided workspace.  This file runs last (pytest collects it after every other
test file), so a failure here leaves every other test already run.
"""

import pytest
import torch

from motif_b200 import _lib

pytestmark = pytest.mark.gpu

B, H, HKV, T, D, SPLITS = 4, 12, 3, 1, 64, 12


def inputs(S, seed):
    g = torch.Generator().manual_seed(seed)
    cap = S + 16
    q = torch.randn(B * T, H * D, generator=g).bfloat16().cuda()
    k = torch.randn(B, HKV, cap, D, generator=g).bfloat16().cuda()
    v = torch.randn(B, HKV, cap, D, generator=g).bfloat16().cuda()
    params = [(0.5 + 1.5 * torch.rand(H, generator=g)).cuda(), torch.rand(H, generator=g).cuda(),
              torch.ones(H).cuda(), (0.8 + 0.4 * torch.rand(H, generator=g)).cuda()]
    length = torch.tensor([S], dtype=torch.int32, device='cuda')
    return q, k, v, cap, params, length


def with_workspace(q, k, v, cap, params, length):
    out = torch.empty(B * T, H * D, dtype=torch.bfloat16, device='cuda')
    nbytes = _lib.load().motif_b200_chord_decode_workspace_bytes(B, H, T, D, SPLITS)
    ws = torch.empty(nbytes // 4, device='cuda')
    _lib.call('motif_b200_chord_decode', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), cap, _lib.ptr(length), 0,
              *[_lib.ptr(p) for p in params], _lib.ptr(out), H * D, B, H, HKV, T, D, D ** -0.5, 1e-5, SPLITS,
              _lib.ptr(ws), nbytes, _lib.MB_BF16, _lib.stream_ptr())
    return out


def without_workspace(q, k, v, cap, params, length, splits=SPLITS):
    out = torch.empty(B * T, H * D, dtype=torch.bfloat16, device='cuda')
    _lib.call('motif_b200_chord_decode_noalloc', _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), cap, _lib.ptr(length), 0,
              *[_lib.ptr(p) for p in params], _lib.ptr(out), H * D, B, H, HKV, T, D, D ** -0.5, 1e-5, splits,
              _lib.MB_BF16, _lib.stream_ptr())
    return out


def test_noalloc_decode_matches_workspace_decode_twice():
    """Two calls in a row (different inputs and lengths) both match the workspace path."""
    for S, seed in ((1000, 1), (333, 2)):
        args = inputs(S, seed)
        ref = with_workspace(*args)
        got = without_workspace(*args)
        torch.cuda.synchronize()
        err = ((got.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        assert err <= 1e-2, err


def test_noalloc_rejects_oversized_requests():
    args = inputs(64, 3)
    with pytest.raises(ValueError, match='limit'):
        without_workspace(*args, splits=1024)
