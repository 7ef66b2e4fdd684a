"""Host-side behaviour of `motif_b200.sampler` (no GPU): construction, `make_sampler`,
`with_constraint`, and argument checks that run before any launch."""

import pytest
import torch

from motif_b200.sampler import Sampler, make_sampler, sample_tokens


def test_defaults_mirror_reference():
    s = Sampler()
    assert (s.temperature, s.top_k, s.top_p, s.repetition_penalty, s.constraint) == (0.7, None, None, 1.15, None)
    assert s.eos_token_id is None
    assert repr(s) == 'Sampler(temperature=0.7, top_k=None, top_p=None, repetition_penalty=1.15, constraint=None)'


def test_seed_follows_torch_manual_seed():
    torch.manual_seed(123)
    a = Sampler().seed
    torch.manual_seed(123)
    assert Sampler().seed == a
    assert Sampler(seed=9).seed == 9


def test_make_sampler_styles():
    assert make_sampler() is None
    s = Sampler(temperature=0.5)
    assert make_sampler(s) is s
    b = make_sampler(temperature=0.3, top_p=0.8)
    assert isinstance(b, Sampler) and b.temperature == 0.3 and b.top_p == 0.8
    with pytest.raises(ValueError):
        make_sampler(s, top_k=3)


def test_with_constraint_copies():
    class C:
        eos_token_id = 1

    s = Sampler(top_k=5)
    c = C()
    b = s.with_constraint(c, eos_token_id=7)
    assert b is not s and s.constraint is None and b.constraint is c
    assert c.eos_token_id == 7 and b.eos_token_id == 7 and b.top_k == 5
    assert s.with_constraint(None).constraint is None


def test_sample_tokens_rejects_host_tensors():
    with pytest.raises(ValueError):
        sample_tokens(torch.zeros(2, 10))
