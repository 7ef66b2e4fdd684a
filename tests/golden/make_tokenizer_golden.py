"""Generate the golden vectors that pin `motif_b200.tokenizer` to the reference's tokenizer.

Run once in a container where the reference source tree (with its `tokenizer.zip`) is present:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_tokenizer_golden.py --reference <ref-src-dir>

It imports the reference's own `motif.tokenizer` (PackedTokenizer, create_tokenizer_trainer,
SPEC_TOKEN), and records into `tests/golden/tokenizer.json`:
  * with the reference's `tokenizer.zip`: vocabulary size, configuration, the ids of every
    special token, `encode` (with and without the safe rules, with special tokens) and `decode`
    of a fixed set of texts, and `apply_chat_template` of fixed conversations;
  * with a tiny BPE trained by the reference's trainer (vocab 300) on a fixed synthetic corpus:
    its vocabulary and merges digest and the encodings of the same texts.
The tests compare `motif_b200.tokenizer` with these values; they load `tokenizer.zip` from the
reference tree when it is present (CPU tests only) and retrain the tiny BPE themselves.
"""

import argparse
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

TEXTS = [
    'Hello, world!',
    'Brackets [like this] and | bars || and ]] [[ mixed',
    'Numbers 1234567890 and 3.14159 and -42',
    'Unicode: héllo naïve café — 你好，世界 🙂',
    '  leading and trailing spaces  ',
    'tabs\tand\nnewlines\r\nhere',
    '<|im_start|>looks special<|im_end|> and <|safe_escape|> literally',
    'code: def f(x): return x[0] | x[1]',
    '',
]

CHATS = [
    ([{'role': 'system', 'content': 'You are terse.'}, {'role': 'human', 'content': 'Hi [there] | friend'}],
     {'add_generation_prompt': True}),
    ([{'role': 'human', 'content': 'What is 2+2?'},
      {'role': 'model', 'content': 'It is 4.', 'thought': 'simple arithmetic'},
      {'role': 'human', 'content': 'And 3+3?'}], {'add_generation_prompt': True}),
    ([{'role': 'user', 'content': 'list parts'},
      {'role': 'assistant', 'content': [{'type': 'text', 'text': 'a [b] c'}], 'reasoning_content': 'think'}],
     {'add_generation_prompt': False}),
    ([{'role': 'system', 'content': 'tools available'}, {'role': 'human', 'content': 'weather?'},
      {'role': 'tool', 'content': '{"temp": 21}'}], {'add_generation_prompt': True}),
]


def corpus():
    """A fixed synthetic corpus, large enough that pairs pass the trainer's min_frequency."""
    words = ['alpha', 'beta', 'gamma', 'delta', 'motif', 'chord', 'token', 'stream', '[x]', 'a|b', '2024', 'héllo']
    out = []
    for i in range(400):
        out.append(' '.join(words[(i * 7 + j * 3) % len(words)] for j in range(12)))
    return out


def digest(tok):
    """sha256 of the tokenizer's vocabulary (sorted) and merges, from its JSON serialisation."""
    m = json.loads(tok.to_str())['model']
    vocab = sorted(m['vocab'].items())
    merges = [' '.join(x) if isinstance(x, list) else x for x in m['merges']]
    return hashlib.sha256(json.dumps([vocab, merges], ensure_ascii=False).encode('utf-8')).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from motif.tokenizer.spec_token import SPEC_TOKEN
    from motif.tokenizer.tokenizer import PackedTokenizer, create_tokenizer_trainer

    t = PackedTokenizer(os.path.join(args.reference, 'tokenizer.zip'))
    out = {'spec_token': SPEC_TOKEN, 'vocab_size': t.vocab_size, 'config': t.config,
           'safe_escape': t.safe_escape, 'safe_rules': t.safe_rules,
           'special_ids': {s: t.token_to_id(s) for s in SPEC_TOKEN}, 'encode': [], 'chat': []}
    for s in TEXTS:
        ids = t.encode(s)
        out['encode'].append({'text': s, 'ids': ids, 'ids_raw': t.encode(s, apply_safe_rule=False),
                              'ids_special': t.encode(s, add_special_tokens=True), 'decoded': t.decode(ids),
                              'decoded_skip': t.decode(ids, skip_special_tokens=True)})
    for msgs, kw in CHATS:
        out['chat'].append({'messages': msgs, 'kwargs': kw, 'ids': t.apply_chat_template(msgs, **kw)})

    tr = create_tokenizer_trainer(vocab_size=300)
    tr.train_from_iterator(corpus())
    small = tr.packed_tokenizer
    out['tiny'] = {'vocab_size': small.vocab_size, 'digest': digest(small.tokenizer),
                   'encode': [small.encode(s) for s in TEXTS]}
    path = os.path.join(HERE, 'tokenizer.json')
    with open(path, 'w', encoding='utf-8') as f:
        json.dump(out, f, ensure_ascii=False, indent=1)
    print('wrote', path, os.path.getsize(path), 'bytes')


if __name__ == '__main__':
    main()
