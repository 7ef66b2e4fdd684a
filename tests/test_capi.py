"""The C-ABI library loads and exports every entry point `include/motif_b200.h` declares.

CPU-only: no kernel is launched.  Calls made here fail argument validation before any
CUDA runtime call, which checks the error plumbing and the ctypes signatures.
"""

import ctypes
import os
import re

import pytest

from motif_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, 'include', 'motif_b200.h')).read()
    return sorted(set(re.findall(r'\b(motif_b200_[a-z0-9_]+)\s*\(', src)))


def test_header_and_binding_agree():
    assert declared() == sorted(_lib.SIGNATURES), set(declared()) ^ set(_lib.SIGNATURES)


def declared_arity():
    """{entry point: parameter count} from the header's MB_API declarations."""
    src = open(os.path.join(ROOT, 'include', 'motif_b200.h')).read()
    src = re.sub(r'/\*.*?\*/', ' ', src, flags=re.S)
    out = {}
    for name, params in re.findall(r'MB_API[^;(]*?\b(motif_b200_[a-z0-9_]+)\s*\(([^;]*?)\)\s*;', src, flags=re.S):
        params = params.strip()
        out[name] = 0 if params in ('', 'void') else params.count(',') + 1
    return out


def test_binding_parameter_counts_match_header():
    """Every ctypes signature has as many parameters as the C declaration (an argument added
    on one side only would shift every later argument of the call)."""
    arity = declared_arity()
    assert sorted(arity) == declared()
    bad = {n: (arity[n], len(_lib.SIGNATURES[n][1])) for n in arity if arity[n] != len(_lib.SIGNATURES[n][1])}
    assert not bad, bad


def test_library_exports_every_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared():
        assert hasattr(lib, name), name
    assert _lib.load().motif_b200_abi_version() == _lib.ABI_VERSION


def test_errors_map_to_reference_exceptions():
    lib = _lib.load()
    with pytest.raises(ValueError, match='null pointer'):
        _lib.call('motif_b200_rms_norm', None, None, None, 4, 8, 8, 8, 1e-6, _lib.MB_F32, None)
    with pytest.raises(ValueError, match='unsupported dtype'):
        _lib.call('motif_b200_rms_norm', 16, None, 16, 4, 8, 8, 8, 1e-6, 7, None)
    with pytest.raises(NotImplementedError):
        _lib.call('motif_b200_attn_res', _lib.ptr_array([16] * 9), 9, _lib.i64_array([0] * 18), 16, 16, 16,
                  0, 0, 1, 1, 8, 1e-6, _lib.MB_F32, None)
    with pytest.raises(ValueError, match='not divisible'):
        _lib.call('motif_b200_chord_attention', 16, 16, 16, 16, 16, 16, 16, 16, 16, 1, 4, 3, 1, 1, 64, 0,
                  0.125, 1e-5, _lib.i64_array([0] * 14), _lib.MB_BF16, None, 0, None)
    assert b'not divisible' in lib.motif_b200_last_error()
    # decode workspace size is plain arithmetic
    assert lib.motif_b200_chord_decode_workspace_bytes(2, 4, 1, 64, 3) == 3 * 2 * 4 * 1 * 66 * 4


def test_unaligned_gdn_inputs_rejected():
    with pytest.raises(ValueError, match='aligned'):
        _lib.call('motif_b200_gdn_chunk', 18, 16, 16, 16, 16, None, 16, 16, 1, 1, 4, 64, 128,
                  _lib.i64_array([256, 256, 64] * 3 + [512, 512, 128] + [4, 4, 1] * 2), _lib.MB_BF16, None)
