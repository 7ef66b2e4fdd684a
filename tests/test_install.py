"""`motif_b200.install` swaps the reference's imported op names and restores them.

Runs on CPU against a stand-in `motif` package tree with the same module paths and names
as the reference (`motif/block/attention/{chord_attn,gdn_attn}.py`, `motif/block/decoder.py`,
`motif/block/mlp.py`, `motif/model/{motif,sampler}.py`, `motif/ops`), so no reference checkout is needed.
"""

import sys
import types

import pytest

from motif_b200 import install, ops


@pytest.fixture
def fake_motif(monkeypatch):
    names = {
        'motif': [],
        'motif.ops': ['apply_chord_attention', 'recurrent_gated_delta_rule', 'chunk_gated_delta_rule',
                      'chunk_gated_delta_rule_triton', 'attn_res_block', 'RMSNorm', 'GatedRMSNorm', 'SwiGLU'],
        'motif.ops.attn_res': ['apply_block_attn_res'],
        'motif.block': [],
        'motif.block.attention': [],
        'motif.block.attention.chord_attn': ['apply_chord_attention', 'RMSNorm'],
        'motif.block.attention.gdn_attn': ['recurrent_gated_delta_rule', 'chunk_gated_delta_rule',
                                           'chunk_gated_delta_rule_triton', 'GatedRMSNorm'],
        'motif.block.decoder': ['apply_block_attn_res', 'RMSNorm'],
        'motif.block.mlp': ['SwiGLUOp'],
        'motif.model': [],
        'motif.model.motif': ['RMSNorm', 'Sampler', 'make_sampler'],
        'motif.model.sampler': ['Sampler', 'make_sampler'],
    }
    originals = {}
    for mod_name, attrs in names.items():
        m = types.ModuleType(mod_name)
        for a in attrs:
            obj = object()
            setattr(m, a, obj)
            originals[(mod_name, a)] = obj
        monkeypatch.setitem(sys.modules, mod_name, m)
    yield originals
    install.uninstall()


def test_install_patches_every_target(fake_motif):
    done = install.install(strict=True)
    assert len(done) == len(install.TARGETS)
    for mod_name, attr, repl in install.TARGETS:
        assert getattr(sys.modules[mod_name], attr) is getattr(ops, repl), (mod_name, attr)
    assert install.installed()


def test_uninstall_restores_originals(fake_motif):
    install.install()
    install.install()   # idempotent: the saved originals are not overwritten by our own objects
    install.uninstall()
    for (mod_name, attr), obj in fake_motif.items():
        assert getattr(sys.modules[mod_name], attr) is obj
    assert not install.installed()


def test_missing_module_skipped_or_strict(monkeypatch, fake_motif):
    monkeypatch.delitem(sys.modules, 'motif.block.mlp')
    monkeypatch.setattr(install.importlib, 'import_module',
                        lambda n: sys.modules[n] if n in sys.modules else (_ for _ in ()).throw(ImportError(n)))
    done = install.install()
    assert 'motif.block.mlp.SwiGLUOp' not in done
    install.uninstall()
    with pytest.raises(ImportError):
        install.install(strict=True)


def test_every_target_names_a_real_op():
    for _, _, repl in install.TARGETS:
        assert callable(getattr(ops, repl))
