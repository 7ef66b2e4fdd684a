"""Checkpoint I/O (`motif_b200.checkpoint`, `MotifChordModel.from_pretrained`) against files the
reference wrote (`tests/golden/ckpt/`, made by `tests/golden/make_golden.py` with the
reference's own `save_safetensors` / `torch.save`): the weights come back under their
canonical names, the config each layout yields is the one the reference resolves from the
same file, and (GPU) the loaded model's logits equal the reference's."""

import json
import os

import pytest
import torch

from motif_b200.checkpoint import (config_from_mapping, config_from_state_dict, load_checkpoint,
                                   looks_like_safetensors, save_safetensors, strip_wrapper_prefixes)
from motif_b200.config import MotifChordConfig

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
CK = os.path.join(GOLD, 'ckpt')
FILES = ['model.safetensors', 'bare_module.pt', 'pipeline.pt']


def fixture():
    return torch.load(os.path.join(GOLD, 'checkpoints.pt'))


@pytest.mark.parametrize('name', FILES)
def test_weights_come_back_canonical(name):
    d = fixture()
    ld = load_checkpoint(os.path.join(CK, name))
    ref = d['state_dict']
    for k, v in ld.state_dict.items():
        assert k in ref, k
        assert torch.equal(v, ref[k]), k
    # only the tied head may be absent
    assert set(ref) - set(ld.state_dict) <= {'lm_head.weight'}


@pytest.mark.parametrize('name', FILES)
def test_config_resolution_matches_reference(name):
    from motif_b200.model import MotifChordModel
    d = fixture()
    want = config_from_mapping(json.loads(d['resolved'][name]))
    m = MotifChordModel.from_pretrained(os.path.join(CK, name), verbose=False)
    assert m.config == want
    assert not m.training


def test_layout_detection_and_sources():
    assert looks_like_safetensors(os.path.join(CK, 'model.safetensors'))
    assert not looks_like_safetensors(os.path.join(CK, 'pipeline.pt'))
    assert load_checkpoint(os.path.join(CK, 'model.safetensors')).source == 'safetensors'
    assert load_checkpoint(os.path.join(CK, 'bare_module.pt')).source == 'bare state_dict'
    assert load_checkpoint(os.path.join(CK, 'pipeline.pt')).source.startswith('pipeline checkpoint')
    assert load_checkpoint(CK).source == 'safetensors'  # a directory: model.safetensors first
    with pytest.raises(FileNotFoundError):
        load_checkpoint(os.path.join(CK, 'missing.pt'))


def test_prefix_stripping_and_inference():
    sd = {'module._orig_mod.embed.weight': torch.zeros(3), 'module._orig_mod.x': torch.zeros(1)}
    assert set(strip_wrapper_prefixes(sd)) == {'embed.weight', 'x'}
    mixed = {'model.a': torch.zeros(1), 'b': torch.zeros(1)}
    assert strip_wrapper_prefixes(mixed) == mixed
    d = fixture()
    cfg = config_from_state_dict(d['state_dict'])
    assert cfg.block == ('gdn', 'chord') and cfg.num_kv_heads == 1 and cfg.head_k_dim == 16
    with pytest.raises(ValueError):
        config_from_state_dict({'x': torch.zeros(1)})
    assert config_from_mapping({'hidden_size': 48, 'num_attention_heads': 3, 'extra': 1}).model_dim == 48


def test_save_round_trip_and_overrides(tmp_path):
    from motif_b200.model import MotifChordModel
    m = MotifChordModel.from_pretrained(os.path.join(CK, 'pipeline.pt'), verbose=False)
    p = tmp_path / 'out.safetensors'
    info = save_safetensors(m, str(p), metadata={'note': 'x'})
    assert info['dropped'] == ['lm_head.weight'] and info['metadata']['note'] == 'x'
    m2 = MotifChordModel.from_pretrained(str(p), verbose=False)
    assert m2.config == m.config
    assert all(torch.equal(a, b) for a, b in zip(m.state_dict().values(), m2.state_dict().values()))
    with pytest.raises(TypeError):
        MotifChordModel.from_pretrained(str(p), verbose=False, no_such_field=1)
    with pytest.raises(RuntimeError):  # a config that does not fit the weights
        MotifChordModel.from_pretrained(str(p), verbose=False, model_dim=48)


@pytest.mark.gpu
@pytest.mark.parametrize('name', FILES)
def test_loaded_model_logits_match_reference(name):
    from motif_b200.model import MotifChordModel
    d = fixture()
    m = MotifChordModel.from_pretrained(os.path.join(CK, name), device='cuda', verbose=False)
    with torch.no_grad():
        lg = m(d['ids'].cuda()).logits.float().cpu()
    err = ((lg - d['logits']).abs().max() / d['logits'].abs().max()).item()
    assert err < 1e-5, err


def test_pipeline_checkpoint_with_phase_enum_loads_weights_only(tmp_path, monkeypatch):
    """A pipeline checkpoint whose training state holds a `motif.pipeline.base.PipelinePhase`
    member loads through the `weights_only` unpickler (the class is allowlisted under that
    name), without the training pipeline importable and without the full unpickler."""
    import enum
    import sys
    import types
    from motif_b200 import checkpoint as ck

    # write the file the way the training pipeline did: the enum pickled under its own module
    mod = types.ModuleType('motif.pipeline.base')

    class PipelinePhase(enum.Enum):
        INIT = 1
        SETUP = 2
        TRAINING = 3
        EVALUATING = 4
        FINISHED = 5
        INTERRUPTED = 6
        FAILED = 7

    PipelinePhase.__module__ = 'motif.pipeline.base'
    PipelinePhase.__qualname__ = 'PipelinePhase'
    mod.PipelinePhase = PipelinePhase
    for name in ('motif', 'motif.pipeline'):
        monkeypatch.setitem(sys.modules, name, sys.modules.get(name) or types.ModuleType(name))
    monkeypatch.setitem(sys.modules, 'motif.pipeline.base', mod)
    sd = {'embed.weight': torch.randn(8, 4), 'lm_head.weight': torch.randn(8, 4)}
    path = str(tmp_path / 'phase.pt')
    torch.save({'__pipeline__': 'pretrain', 'model': sd, 'state': {'phase': PipelinePhase.FINISHED, 'step': 7}}, path)
    monkeypatch.delitem(sys.modules, 'motif.pipeline.base')

    # the weights_only form must succeed on its own: fail the test if the full unpickler runs
    real = torch.load

    def guarded(*a, **kw):
        assert kw.get('weights_only', True), 'fell back to the full unpickler'
        return real(*a, **kw)

    monkeypatch.setattr(torch, 'load', guarded)
    ld = ck.load_checkpoint(path)
    assert set(ld.state_dict) == set(sd)
    assert all(torch.equal(ld.state_dict[k], sd[k]) for k in sd)
