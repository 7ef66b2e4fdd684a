"""Route the reference's own `motif` layers through this library's kernels.

The reference modules bind the `motif.ops` names by value at import time
(`from motif.ops import apply_chord_attention, ...`), so replacing `motif.ops.X` alone
changes nothing for an already-imported layer: the patch targets are the importing modules.

    motif/block/attention/chord_attn.py:6-10   apply_chord_attention, RMSNorm
    motif/block/attention/gdn_attn.py:7-13     recurrent_gated_delta_rule, chunk_gated_delta_rule,
                                               chunk_gated_delta_rule_triton, GatedRMSNorm
    motif/block/decoder.py:12-13               apply_block_attn_res, RMSNorm
    motif/block/mlp.py:4                       SwiGLU (bound as SwiGLUOp)
    motif/model/motif.py:22-23                 Sampler, make_sampler, RMSNorm
    motif/model/sampler.py                     Sampler, make_sampler (the device sampler)
    motif/ops/__init__.py                      every name above, for later importers

Functions take effect at once for existing layers; classes (RMSNorm, GatedRMSNorm, SwiGLU)
take effect for modules constructed after `install()` — build the model after installing.
`uninstall()` puts every original object back.
"""

import importlib
from typing import Dict, List, Tuple

from . import ops

# (module, attribute in that module, attribute of motif_b200.ops that replaces it)
TARGETS: List[Tuple[str, str, str]] = [
    ('motif.ops', 'apply_chord_attention', 'apply_chord_attention'),
    ('motif.ops', 'recurrent_gated_delta_rule', 'recurrent_gated_delta_rule'),
    ('motif.ops', 'chunk_gated_delta_rule', 'chunk_gated_delta_rule'),
    ('motif.ops', 'chunk_gated_delta_rule_triton', 'chunk_gated_delta_rule_triton'),
    ('motif.ops', 'attn_res_block', 'attn_res_block'),
    ('motif.ops', 'RMSNorm', 'RMSNorm'),
    ('motif.ops', 'GatedRMSNorm', 'GatedRMSNorm'),
    ('motif.ops', 'SwiGLU', 'SwiGLU'),
    ('motif.ops.attn_res', 'apply_block_attn_res', 'apply_block_attn_res'),
    ('motif.block.attention.chord_attn', 'apply_chord_attention', 'apply_chord_attention'),
    ('motif.block.attention.chord_attn', 'RMSNorm', 'RMSNorm'),
    ('motif.block.attention.gdn_attn', 'recurrent_gated_delta_rule', 'recurrent_gated_delta_rule'),
    ('motif.block.attention.gdn_attn', 'chunk_gated_delta_rule', 'chunk_gated_delta_rule'),
    ('motif.block.attention.gdn_attn', 'chunk_gated_delta_rule_triton', 'chunk_gated_delta_rule_triton'),
    ('motif.block.attention.gdn_attn', 'GatedRMSNorm', 'GatedRMSNorm'),
    ('motif.block.decoder', 'apply_block_attn_res', 'apply_block_attn_res'),
    ('motif.block.decoder', 'RMSNorm', 'RMSNorm'),
    ('motif.block.mlp', 'SwiGLUOp', 'SwiGLU'),
    ('motif.model.motif', 'RMSNorm', 'RMSNorm'),
    ('motif.model.motif', 'Sampler', 'Sampler'),
    ('motif.model.motif', 'make_sampler', 'make_sampler'),
    ('motif.model.sampler', 'Sampler', 'Sampler'),
    ('motif.model.sampler', 'make_sampler', 'make_sampler'),
]

_saved: Dict[Tuple[str, str], object] = {}


def install(strict: bool = False) -> List[str]:
    """Swap the reference's op names for this library's.  Returns the patched `module.attr` names.

    A target module that cannot be imported (or lacks the attribute) is skipped, or raises
    `ImportError` / `AttributeError` when `strict`.  Installing twice is a no-op for names
    already patched."""
    done = []
    for mod_name, attr, repl in TARGETS:
        try:
            mod = importlib.import_module(mod_name)
        except ImportError:
            if strict:
                raise
            continue
        if not hasattr(mod, attr):
            if strict:
                raise AttributeError(f'{mod_name} has no attribute {attr}')
            continue
        new = getattr(ops, repl)
        key = (mod_name, attr)
        if key not in _saved:
            _saved[key] = getattr(mod, attr)
        setattr(mod, attr, new)
        done.append(f'{mod_name}.{attr}')
    return done


def uninstall() -> None:
    """Restore every name `install()` replaced."""
    for (mod_name, attr), orig in list(_saved.items()):
        mod = importlib.import_module(mod_name)
        setattr(mod, attr, orig)
        del _saved[(mod_name, attr)]


def installed() -> bool:
    return bool(_saved)
