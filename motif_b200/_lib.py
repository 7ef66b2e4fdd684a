"""ctypes binding of `libmotif_b200.so` (the C ABI declared in `include/motif_b200.h`).

The library is loaded from this package directory.  There is no fallback: if the library
is missing or a call fails, the error surfaces as an exception with the library's own
message, mapped onto the reference's exception types (`ValueError` for argument / shape /
dtype / alignment errors, `NotImplementedError` for shapes this build has no kernel for,
`RuntimeError` for CUDA launch failures).
"""

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'libmotif_b200.so')

MB_OK, MB_ERR_ARG, MB_ERR_SHAPE, MB_ERR_DTYPE, MB_ERR_ALIGN, MB_ERR_UNSUPPORTED, MB_ERR_CUDA = range(7)
MB_F32, MB_F16, MB_BF16 = 0, 1, 2
# testing knobs of motif_b200_testing_force (include/motif_b200.h)
FORCE_CHORD_MMA_SYNC, FORCE_DECODE_SCALAR, FORCE_GDN_PRECISE, FORCE_GDN_FUSED, FORCE_GDN_WIDE = range(5)
ABI_VERSION = 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> (restype, argtypes); must match include/motif_b200.h
SIGNATURES = {
    'motif_b200_last_error': (ctypes.c_char_p, []),
    'motif_b200_abi_version': (_I, []),
    'motif_b200_gdn_recurrent': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I, _P]),
    'motif_b200_gdn_chunk': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I, _P]),
    'motif_b200_gdn_chunk_gated': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P,
                                        _P, _I64, _I64, _P, _F, _I, _P]),
    'motif_b200_chord_workspace_bytes': (_I64, [_I64, _I64, _I64, _I64, _I64, _I64, _I]),
    'motif_b200_chord_attention': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                        _I64, _I64, _F, _F, _P, _I, _P, _I64, _P]),
    'motif_b200_attn_res': (_I, [_P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I, _P]),
    'motif_b200_rms_norm': (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _I, _P]),
    'motif_b200_gated_rms_norm': (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _I, _P]),
    'motif_b200_swiglu': (_I, [_P, _P, _I64, _I64, _I64, _I64, _I, _P]),
    'motif_b200_attn_res_norm': (_I, [_P, _I, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _F, _F, _I, _P]),
    'motif_b200_gdn_prep': (_I, [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                 _I64, _I, _P]),
    'motif_b200_gdn_prefill': (_I, [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _I64,
                                    _I64, _I64, _I, _P]),
    'motif_b200_gdn_decode': (_I, [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                   _F, _I, _P]),
    'motif_b200_chord_prep': (_I, [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64,
                                   _I64, _F, _I, _P]),
    'motif_b200_decode_advance': (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P]),
    'motif_b200_chord_prep_swiglu': (_I, [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64,
                                          _I64, _F, _P, _I64, _P, _I64, _I64, _I, _P]),
    'motif_b200_gdn_decode_swiglu': (_I, [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                          _F, _P, _I64, _P, _I64, _I64, _I, _P]),
    'motif_b200_chord_decode_workspace_bytes': (_I64, [_I64, _I64, _I64, _I64, _I]),
    'motif_b200_chord_decode': (_I, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                     _I64, _I64, _F, _F, _I, _P, _I64, _I, _P]),
    'motif_b200_chord_attention_masked': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                               _I64, _I64, _F, _F, _P, _P, _I64, _I, _P]),
    'motif_b200_chord_decode_masked': (_I, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                            _I64, _I64, _F, _F, _I, _P, _I64, _P, _I64, _I, _P]),
    'motif_b200_chord_decode_noalloc': (_I, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                             _I64, _I64, _I64, _F, _F, _I, _I, _P]),
    'motif_b200_gate_residual': (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I, _P]),
    'motif_b200_argmax': (_I, [_P, _I64, _I64, _I64, _P, _I, _P]),
    'motif_b200_embed': (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _P]),
    'motif_b200_sample': (_I, [_P, _I64, _I64, _I64, _P, _I64, _I64, _F, _F, _I64, _F, _P, ctypes.c_uint64,
                               ctypes.c_uint64, _P, _P, _P, _I64, _I, _P]),
    'motif_b200_wait_timeouts': (_I, [_P]),
    'motif_b200_testing_force': (_I, [_I, _I]),
    'motif_b200_gemm': (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _P]),
    'motif_b200_gemm_proj_swiglu': (_I, [_P, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _I64, _I, _P]),
    'motif_b200_gemm_gdn_prep': (_I, [_P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P,
                                      _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I, _P]),
    'motif_b200_gemm_gate_residual': (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I,
                                           _P]),
    'motif_b200_skinny_packed_bytes': (_I64, [_I64, _I64]),
    'motif_b200_chord_backward_workspace_bytes': (_I64, [_I64, _I64, _I64]),
    'motif_b200_chord_backward': (_I, [_P] * 13 + [_I64] * 7 + [_F, _F, _P, _P, _I64, _P, _I, _P]),
    'motif_b200_attn_res_backward': (_I, [_P, _P, _I, _I64, _I64, _I64, _P, _P, _F, _P, _I64, _P, _I64, _I, _P]),
    'motif_b200_gdn_backward_workspace_bytes': (_I64, [_I64] * 5),
    'motif_b200_gdn_backward': (_I, [_P] * 14 + [_I64] * 5 + [_P, _I64, _P]),
    'motif_b200_skinny_pack': (_I, [_P, _I64, _I64, _I64, _P, _I, _P]),
    'motif_b200_skinny_gemm': (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _P]),
    'motif_b200_skinny_gemm_tc': (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _I, _P]),
    'motif_b200_skinny_gemm_tc_chord_tail': (_I, [_P, _I64, _P, _I64, _I64, _P, _I64, _P, _I64, _I64, _P, _I64, _P,
                                                   _I64, _I64, _I64, _I, _P]),
    'motif_b200_skinny_gemm_tc_add_gated': (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64,
                                                  _I, _I, _P]),
    'motif_b200_gdn_prefill_ws': (_I, [_P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _I64,
                                       _I64, _I64, _I, _P, _I64, _P]),
    'motif_b200_gdn_chunk_workspace_bytes': (_I64, [_I64, _I64, _I64, _I64, _I64, _I]),
    'motif_b200_gdn_chunk_gated_ws': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64,
                                           _I64, _P, _F, _I, _P, _I64, _P]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the ctypes library; raises if it is missing or stale."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f'{LIB_PATH} is missing: build it with `python -m motif_b200.build` '
                    '(there is no CPU or eager fallback)')
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            v = lib.motif_b200_abi_version()
            if v != ABI_VERSION:
                raise RuntimeError(f'libmotif_b200.so ABI {v} != expected {ABI_VERSION}: rebuild it')
            _lib = lib
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return MB_F32
    if dt == torch.float16:
        return MB_F16
    if dt == torch.bfloat16:
        return MB_BF16
    raise ValueError(f'unsupported dtype {dt} (only fp16 / bf16 / fp32)')


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def i64_array(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * len(vals))(*vals)


def ptr_array(ptrs):
    return (ctypes.c_void_p * len(ptrs))(*[int(p) for p in ptrs])


def ptr(t):
    """Device pointer of a tensor (or None -> NULL)."""
    return None if t is None else t.data_ptr()


# Kernels each entry point launches (for launch accounting); 0 = host-only query.
KERNELS_PER_CALL = {n: 1 for n in SIGNATURES}
KERNELS_PER_CALL.update({'motif_b200_last_error': 0, 'motif_b200_abi_version': 0,
                         'motif_b200_chord_workspace_bytes': 0, 'motif_b200_chord_decode_workspace_bytes': 0,
                         'motif_b200_skinny_packed_bytes': 0, 'motif_b200_gdn_chunk_workspace_bytes': 0,
                         'motif_b200_chord_backward_workspace_bytes': 0, 'motif_b200_gdn_backward_workspace_bytes': 0,
                         'motif_b200_chord_backward': 2,
                         'motif_b200_wait_timeouts': 0, 'motif_b200_testing_force': 0,
                         'motif_b200_chord_decode': 2, 'motif_b200_chord_decode_noalloc': 2,
                         'motif_b200_chord_decode_masked': 2,
                         'motif_b200_gdn_chunk_gated_ws': 3, 'motif_b200_gdn_prefill_ws': 3})


class Tracker:
    """Counts kernel launches and (optionally) times calls with CUDA events on the
    current stream.  `timed` names the entry points to bracket with events (None = all)."""

    def __init__(self, timed=None, events=True):
        self.launches = 0
        self.timed = timed
        self.events = events
        self.records = []  # (name, start_event, end_event)

    def start(self, name):
        if self.events and (self.timed is None or name in self.timed):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            return ev
        return None

    def stop(self, name, ev):
        self.launches += KERNELS_PER_CALL.get(name, 1)
        if ev is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            self.records.append((name, ev, end))

    def summary(self):
        """`{name: (calls, total_ms)}` (call after synchronising)."""
        out = {}
        for name, a, b in self.records:
            c, t = out.get(name, (0, 0.0))
            out[name] = (c + 1, t + a.elapsed_time(b))
        return out


_tracker = None


def set_tracker(tr):
    """Install (or remove with None) the launch tracker; returns the previous one."""
    global _tracker
    prev, _tracker = _tracker, tr
    return prev


def call(name: str, *args) -> None:
    """Call one entry point and raise on a nonzero status."""
    lib = load()
    tr = _tracker
    ev = tr.start(name) if tr is not None else None
    rc = getattr(lib, name)(*args)
    if tr is not None and rc == MB_OK:
        tr.stop(name, ev)
    if rc != MB_OK:
        msg = lib.motif_b200_last_error().decode(errors='replace')
        if rc in (MB_ERR_ARG, MB_ERR_SHAPE, MB_ERR_DTYPE, MB_ERR_ALIGN):
            raise ValueError(f'{name}: {msg}')
        if rc == MB_ERR_UNSUPPORTED:
            raise NotImplementedError(f'{name}: {msg}')
        raise RuntimeError(f'{name}: {msg}')


def wait_timeouts() -> int:
    """Chord-attention CTAs whose bounded copy / MMA wait ran out since the last call (clears it)."""
    n = ctypes.c_uint32(0)
    call('motif_b200_wait_timeouts', ctypes.addressof(n))
    return int(n.value)


class forced:
    """Test-only context manager: switch a testing knob of the library on for the block
    (`with _lib.forced(_lib.FORCE_DECODE_SCALAR): ...`), off again on exit."""

    def __init__(self, knob: int):
        self.knob = knob

    def __enter__(self):
        call('motif_b200_testing_force', self.knob, 1)
        return self

    def __exit__(self, *exc):
        call('motif_b200_testing_force', self.knob, 0)
        return False
