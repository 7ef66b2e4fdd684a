"""motif_b200: B200 (sm_100a) inference path for the Motif Chord model.

Drop-in for the reference's `motif.ops` functions (`motif_b200.ops`) and its
`MotifChordModel` forward / cache / generation API (`motif_b200.model`), computed by the
hand-written CUDA kernels of `libmotif_b200.so` through a C ABI (`include/motif_b200.h`).
"""

__version__ = '0.1.0'
