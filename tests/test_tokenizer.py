"""`motif_b200.tokenizer` against the reference's tokenizer (golden vectors written by
`tests/golden/make_tokenizer_golden.py` from the reference's own `motif.tokenizer`).

* The reference's `tokenizer.zip` (loaded from the reference tree when it is present; the
  GPU box has no reference tree, so these cases skip there): vocabulary, configuration,
  special-token ids, `encode` / `decode` with and without the safe rules, chat templates.
* A tiny BPE trained by `create_tokenizer_trainer` on the generator's fixed corpus: the same
  vocabulary and merges as the reference's trainer, and the same encodings.
* The archive round trip: save -> load keeps ids, configuration, template, rules and extra
  files; reserved names are rejected; entries under a directory prefix are found.
"""

import importlib.util
import json
import os
import zipfile

import pytest

from motif_b200 import tokenizer as mt

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, 'golden', 'tokenizer.json')
REF_ZIP = os.path.join(os.environ.get('MOTIF_REFERENCE', '/root/reference'), 'tokenizer.zip')


def _generator():
    spec = importlib.util.spec_from_file_location('make_tokenizer_golden',
                                                  os.path.join(HERE, 'golden', 'make_tokenizer_golden.py'))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope='module')
def golden():
    with open(GOLDEN, encoding='utf-8') as f:
        return json.load(f)


@pytest.fixture(scope='module')
def ref_tok():
    if not os.path.exists(REF_ZIP):
        pytest.skip('the reference tokenizer archive is not present')
    return mt.PackedTokenizer(REF_ZIP)


def test_special_token_table(golden):
    assert mt.SPEC_TOKEN == golden['spec_token']
    assert len(mt.SPEC_TOKEN) == 256 and mt.SPEC_TOKEN[0] == '<|pad|>' and mt.SPEC_TOKEN[-1].startswith('<|unused_')
    assert mt.token('x') == '<|x|>' and mt.token(['a', 'b']) == ['<|a|>', '<|b|>']
    assert mt.token('u', 2) == ['<|u_0|>', '<|u_1|>']


def test_reference_archive_loads_with_its_configuration(golden, ref_tok):
    assert ref_tok.vocab_size == golden['vocab_size']
    assert ref_tok.config == golden['config']
    assert ref_tok.safe_escape == golden['safe_escape'] and ref_tok.safe_rules == golden['safe_rules']
    assert {s: ref_tok.token_to_id(s) for s in mt.SPEC_TOKEN} == golden['special_ids']
    assert ref_tok.token_eos == golden['config'].get('eos_token', '<|eos|>')
    assert ref_tok.extra_files == {}


def test_reference_archive_encode_decode(golden, ref_tok):
    for case in golden['encode']:
        s = case['text']
        ids = ref_tok.encode(s)
        assert ids == case['ids'], s
        assert ref_tok.encode(s, apply_safe_rule=False) == case['ids_raw'], s
        assert ref_tok.encode(s, add_special_tokens=True) == case['ids_special'], s
        assert ref_tok.decode(ids) == case['decoded'], s
        assert ref_tok.decode(ids, skip_special_tokens=True) == case['decoded_skip'], s
        assert ref_tok.ensure_escape() not in ids


def test_reference_archive_chat_template(golden, ref_tok):
    for case in golden['chat']:
        msgs = json.loads(json.dumps(case['messages']))
        before = json.dumps(msgs)
        assert ref_tok.apply_chat_template(msgs, **case['kwargs']) == case['ids']
        assert json.dumps(msgs) == before  # the caller's messages are not modified


def test_tiny_trainer_matches_reference_trainer(golden):
    gen = _generator()
    tr = mt.create_tokenizer_trainer(vocab_size=300)
    tr.train_from_iterator(gen.corpus())
    tok = tr.packed_tokenizer
    assert tok.vocab_size == golden['tiny']['vocab_size']
    assert gen.digest(tok.tokenizer) == golden['tiny']['digest']
    assert [tok.encode(s) for s in gen.TEXTS] == golden['tiny']['encode']
    # special tokens take the first ids, in table order
    assert [tok.token_to_id(s) for s in mt.SPEC_TOKEN[:8]] == list(range(8))


def test_archive_round_trip(tmp_path):
    gen = _generator()
    tr = mt.create_tokenizer_trainer(vocab_size=300)
    tr.train_from_iterator(gen.corpus())
    tok = tr.packed_tokenizer
    tok.set_chat_template('{% for m in messages %}{{ m.role }}: {{ m.content }}\n{% endfor %}')
    assert tok.set_eos('<|im_end|>') and not tok.set_eos('<|not_a_token|>')
    assert tok.set_pad('<|pad|>')
    tok.add_file('notes/readme.txt', 'hello').add_file('blob.bin', b'\x00\x01')
    path = str(tmp_path / 'tok.zip')
    tok.save(path)
    back = mt.PackedTokenizer(path)
    assert back.config == {'eos_token': '<|im_end|>', 'pad_token': '<|pad|>'}
    assert back.template == tok.template and back.safe_rules == tok.safe_rules
    assert back.get_file('notes/readme.txt') == b'hello' and back.get_file('blob.bin') == b'\x00\x01'
    for s in gen.TEXTS:
        assert back.encode(s) == tok.encode(s)
    assert back.apply_chat_template([{'role': 'human', 'content': 'a [b]'}], add_generation_prompt=False) == \
        tok.apply_chat_template([{'role': 'human', 'content': 'a [b]'}], add_generation_prompt=False)
    with pytest.raises(ValueError, match='reserved'):
        tok.add_file('safe_rules.json', '{}').save(str(tmp_path / 'bad.zip'))


def test_archive_entries_under_a_directory(tmp_path):
    gen = _generator()
    tr = mt.create_tokenizer_trainer(vocab_size=300)
    tr.train_from_iterator(gen.corpus())
    src = str(tmp_path / 'a.zip')
    tr.packed_tokenizer.save(src)
    nested = str(tmp_path / 'nested.zip')
    with zipfile.ZipFile(src) as zi, zipfile.ZipFile(nested, 'w') as zo:
        for n in zi.namelist():
            zo.writestr('pack/' + n, zi.read(n))
    t = mt.PackedTokenizer(nested)
    # 256 special tokens + the 256-symbol byte alphabet already exceed vocab_size = 300
    assert t.vocab_size == 512 and t.extra_files == {}
    with pytest.raises(FileNotFoundError):
        mt.PackedTokenizer(str(tmp_path / 'missing.zip'))
    empty = str(tmp_path / 'empty.zip')
    with zipfile.ZipFile(empty, 'w') as z:
        z.writestr('other.txt', 'x')
    with pytest.raises(ValueError, match='tokenizer.json'):
        mt.PackedTokenizer(empty)


def test_unloaded_wrapper_raises():
    t = mt.PackedTokenizer()
    with pytest.raises(ValueError, match='not loaded'):
        _ = t.tokenizer
    with pytest.raises(ValueError, match='not loaded'):
        _ = t.fast_tokenizer
    with pytest.raises(ValueError, match='No tokenizer'):
        t.save('/nonexistent/x.zip')
    with pytest.raises(TypeError):
        t.set_chat_template(3)
