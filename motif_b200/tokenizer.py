"""The Motif tokenizer: special tokens, BPE trainer and the single-file archive wrapper
(`motif/tokenizer/spec_token.py`, `motif/tokenizer/tokenizer.py`).

Host-side text I/O around the model: it turns text and chat messages into the token ids
`MotifChordModel` / `Generation` consume and back.  It is built on the same libraries as the
reference (`tokenizers` for the byte-level BPE, `transformers.PreTrainedTokenizerFast` for the
Jinja chat template), so an archive the reference wrote (`tokenizer.zip`) loads here and gives
the same ids.

Archive layout (zip; the reference's `PackedTokenizer.save` / `load`):
    tokenizer.json          the `tokenizers.Tokenizer` serialisation
    tokenizer_config.json   {"unk_token", "pad_token", "bos_token", "eos_token"} (any subset)
    chat_template.jinja     the chat template source
    safe_rules.json         {character: replacement}, the replacement may hold "{safe}"
    safe_escape.txt         the escape token's text
    anything else           extra files, kept verbatim
Entries are found by base name, ignoring a directory prefix.

Safe escaping: before encoding, every character with a rule is replaced by its replacement with
the escape token spliced in (default: `]` -> `<esc>]`, `[` -> `[<esc>`, `|` -> `<esc>|<esc>`), so
BPE cannot merge user text into the template's bracket / bar markers; the escape token's id is
then removed from the result.
"""

from __future__ import annotations

import copy
import json
import os
import zipfile
from dataclasses import dataclass
from typing import Any, Dict, Iterable, List, Optional, Union

__all__ = ['token', 'SPEC_TOKEN', 'PackedTokenizer', 'TokenizerTrainerResult', 'create_tokenizer_trainer',
           'RESERVED_ENTRIES']


def token(name: Union[str, List[str]], range_num: Optional[int] = None) -> Union[str, List[str]]:
    """`<|name|>` for one name, a list of those for a list of names, or the indexed series
    `<|name_0|>` .. `<|name_{range_num-1}|>` (`spec_token.py:4-21`)."""
    if isinstance(name, list):
        return [token(n) for n in name]
    if range_num is not None:
        return [f'<|{name}_{i}|>' for i in range(range_num)]
    return f'<|{name}|>'


# The special-token table, in vocabulary order (ids 0.. of a trained tokenizer): the groups of
# `spec_token.py:24-75`, then `<|unused_i|>` up to 256 entries.
_GROUPS = (
    ('pad', 'unk', 'sep', 'mask', 'bos', 'eos', 'end_of_text', 'safe_escape'),
    ('im_start', 'im_end'),
    ('system', 'human', 'tool_response', 'environment', 'model'),
    ('thought_start', 'effort_low', 'effort_high', 'effort_max', 'thought_end'),
    ('tool_declare_start', 'tool_declare_end', 'tool_call_start', 'tool_call_end', 'tool_name_divider'),
    ('fim_prefix', 'fim_suffix', 'fim_middle'),
    ('modality_image_start', 'modality_image_pad', 'modality_image_end',
     'modality_audio_start', 'modality_audio_pad', 'modality_audio_end',
     'modality_video_start', 'modality_video_pad', 'modality_video_end',
     'timestamp_pad', 'timestamp_frame_divider', 'frame_pad', 'frame_sep'),
    ('plan_start', 'plan_sep', 'plan_end'),
    ('action_start', 'action_pad', 'action_end', 'diffusion_start', 'diffusion_pad', 'diffusion_end'),
    ('bbox_start', 'bbox_end'),
    ('object_ref_start', 'object_ref_end'),
)
SPEC_TOKEN: List[str] = [token(n) for group in _GROUPS for n in group]
SPEC_TOKEN += token('unused', 256 - len(SPEC_TOKEN))

RESERVED_ENTRIES = ('tokenizer.json', 'tokenizer_config.json', 'chat_template.jinja', 'safe_rules.json',
                    'safe_escape.txt')

DEFAULT_SAFE_RULES = {']': '{safe}]', '[': '[{safe}', '|': '{safe}|{safe}'}


def _entry(names: List[str], base: str) -> Optional[str]:
    """The archive entry whose base name is `base` (any directory prefix), or None."""
    return next((n for n in names if n == base or n.endswith('/' + base)), None)


@dataclass
class TokenizerTrainerResult:
    """A BPE tokenizer and its trainer (`tokenizer.py:33-73`)."""
    tokenizer: Any
    trainer: Any

    def train_from_iterator(self, iterable: Iterable[str]) -> 'TokenizerTrainerResult':
        self.tokenizer.train_from_iterator(iterable, self.trainer)
        return self

    @property
    def packed_tokenizer(self) -> 'PackedTokenizer':
        return PackedTokenizer(tokenizer=self.tokenizer)


def create_tokenizer_trainer(unk_token: str = token('unk'), vocab_size: int = 5 * (2 ** 13),
                             special_tokens: Optional[List[str]] = None, use_norm: bool = True,
                             use_nfc: bool = True) -> TokenizerTrainerResult:
    """A byte-level BPE tokenizer and trainer configured as `tokenizer.py:76-130` does: NFC (or
    NFKC) normalisation, digits split one by one, byte-level pre-tokenisation without a prefix
    space, byte-level decoding; the trainer starts from the 256-symbol byte alphabet, keeps the
    special tokens first, caps tokens at 32 characters and merges pairs seen at least 10 times."""
    from tokenizers import Tokenizer, decoders, normalizers, pre_tokenizers
    from tokenizers.models import BPE
    from tokenizers.trainers import BpeTrainer

    tok = Tokenizer(BPE(unk_token=unk_token))
    if use_norm:
        tok.normalizer = normalizers.NFC() if use_nfc else normalizers.NFKC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Digits(individual_digits=True),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True),
    ])
    tok.decoder = decoders.ByteLevel()
    trainer = BpeTrainer(vocab_size=vocab_size,
                         special_tokens=list(SPEC_TOKEN if special_tokens is None else special_tokens),
                         initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), max_token_length=32, min_frequency=10)
    return TokenizerTrainerResult(tokenizer=tok, trainer=trainer)


class PackedTokenizer:
    """Tokenizer + chat template + safe escaping + archive I/O (`tokenizer.py:133-570`).

    `PackedTokenizer(path)` loads an archive, `PackedTokenizer(tokenizer)` wraps a trained
    `tokenizers.Tokenizer`, `PackedTokenizer()` is empty until `load`."""

    def __init__(self, tokenizer: Any = None, safe_escape: str = token('safe_escape'),
                 safe_rules: Optional[Dict[str, str]] = None):
        self._tokenizer = None
        self._fast_tokenizer = None
        self.config: Dict[str, Any] = {}
        self.template = ''
        self.extra_files: Dict[str, bytes] = {}
        self.safe_escape = safe_escape
        self.safe_escape_id: Optional[int] = None
        self.safe_rules: Dict[str, str] = dict(safe_rules) if safe_rules else dict(DEFAULT_SAFE_RULES)
        # a path string loads, a Tokenizer is wrapped, anything else leaves the wrapper empty
        # (the reference's constructor, `tokenizer.py:180-184`)
        if isinstance(tokenizer, str):
            self.load(tokenizer)
        elif tokenizer is not None:
            from tokenizers import Tokenizer
            if isinstance(tokenizer, Tokenizer):
                self._tokenizer = tokenizer
                self._rebuild_fast()

    # ------------------------------------------------------------------ configuration
    def _rebuild_fast(self) -> None:
        """The `PreTrainedTokenizerFast` view (chat templates, encode / decode) of the current
        tokenizer, configuration and template; None while nothing is loaded."""
        if self._tokenizer is None:
            self._fast_tokenizer = None
            return
        from transformers import PreTrainedTokenizerFast
        cfg = self.config
        self._fast_tokenizer = PreTrainedTokenizerFast(
            tokenizer_object=self._tokenizer, unk_token=cfg.get('unk_token', token('unk')),
            pad_token=cfg.get('pad_token', token('pad')), bos_token=cfg.get('bos_token', token('bos')),
            eos_token=cfg.get('eos_token', token('eos')), chat_template=self.template,
            clean_up_tokenization_spaces=False)

    def set_chat_template(self, template: str) -> 'PackedTokenizer':
        if not isinstance(template, str):
            raise TypeError(f'template must be str, got {type(template).__name__}')
        self.template = template
        self._rebuild_fast()
        return self

    def _set_special(self, key: str, text: str) -> bool:
        if self._tokenizer.token_to_id(text) is None:
            return False
        self.config[key] = text
        return True

    def set_eos(self, eos: str) -> bool:
        """Make `eos` the end-of-sequence token if the vocabulary has it (True), else False.
        The fast view keeps the previous token until the next rebuild, as in the reference."""
        return self._set_special('eos_token', eos)

    def set_pad(self, pad: str) -> bool:
        return self._set_special('pad_token', pad)

    @property
    def token_eos(self) -> str:
        return self.config.get('eos_token', token('eos'))

    @property
    def token_pad(self) -> str:
        return self.config.get('pad_token', token('pad'))

    # ------------------------------------------------------------------ accessors
    @property
    def tokenizer(self):
        if self._tokenizer is None:
            raise ValueError('Tokenizer is not loaded.')
        return self._tokenizer

    @property
    def fast_tokenizer(self):
        if self._fast_tokenizer is None:
            raise ValueError('Tokenizer is not loaded.')
        return self._fast_tokenizer

    @property
    def vocab_size(self) -> int:
        return self.tokenizer.get_vocab_size()

    def token_to_id(self, text: str) -> Optional[int]:
        return self.tokenizer.token_to_id(text)

    def ensure_escape(self) -> int:
        """The escape token's id (cached); ValueError if the vocabulary lacks it."""
        if self.safe_escape_id is None:
            tid = self.tokenizer.token_to_id(self.safe_escape)
            if tid is None:
                raise ValueError(f'Escape token {self.safe_escape} not found in vocab.')
            self.safe_escape_id = tid
        return self.safe_escape_id

    # ------------------------------------------------------------------ escaping
    def _escape_text(self, text: str) -> str:
        # rules applied one after another in their stored order (a later rule also sees the
        # escape text an earlier one inserted, as in the reference)
        for ch, rep in self.safe_rules.items():
            text = text.replace(ch, rep.format(safe=self.safe_escape))
        return text

    def _escape_content(self, content: Any) -> Any:
        """A message content: a string, or a list of typed parts whose 'text' parts are escaped;
        anything else unchanged."""
        if isinstance(content, str):
            return self._escape_text(content)
        if isinstance(content, list):
            return [{**part, 'text': self._escape_content(part['text'])} if part.get('type') == 'text' else part
                    for part in content]
        return content

    # ------------------------------------------------------------------ text <-> ids
    def encode(self, text: str, add_special_tokens: bool = False, apply_safe_rule: bool = True,
               **kwargs) -> List[int]:
        esc = self.ensure_escape()
        src = self._escape_text(text) if apply_safe_rule else text
        ids = self.fast_tokenizer.encode(src, add_special_tokens=add_special_tokens, **kwargs)
        return [i for i in ids if i != esc]

    def decode(self, token_ids: List[int], skip_special_tokens: bool = False) -> str:
        return self.fast_tokenizer.decode(token_ids, skip_special_tokens=skip_special_tokens)

    def apply_chat_template(self, messages: List[Dict[str, Any]], add_generation_prompt: bool = True,
                            **kwargs) -> List[int]:
        """Token ids of `messages` rendered through the chat template.  Contents are escaped on a
        deep copy, model / assistant messages get `thought=None` unless given (the template then
        falls back to 'reasoning_content'), and the escape id is removed from the result."""
        esc = self.ensure_escape()
        msgs = copy.deepcopy(messages)
        for m in msgs:
            if 'content' in m:
                m['content'] = self._escape_content(m['content'])
            if isinstance(m, dict) and m.get('role') in ('model', 'assistant'):
                m.setdefault('thought', None)
        kwargs.pop('tokenize', None)
        out = self.fast_tokenizer.apply_chat_template(msgs, add_generation_prompt=add_generation_prompt,
                                                      tokenize=True, **kwargs)
        if isinstance(out, dict) or hasattr(out, 'input_ids'):
            out = out['input_ids']
        if out and isinstance(out[0], list):
            out = out[0]
        return [i for i in out if i != esc]

    # ------------------------------------------------------------------ archive
    def add_file(self, name: str, data: Union[str, bytes]) -> 'PackedTokenizer':
        self.extra_files[name] = data.encode('utf-8') if isinstance(data, str) else data
        return self

    def get_file(self, name: str) -> Optional[bytes]:
        return self.extra_files.get(name)

    def save(self, path: str) -> 'PackedTokenizer':
        if self._tokenizer is None:
            raise ValueError('No tokenizer to save.')
        bad = [n for n in self.extra_files if n in RESERVED_ENTRIES]
        with zipfile.ZipFile(path, 'w', zipfile.ZIP_DEFLATED) as z:
            z.writestr('tokenizer.json', self._tokenizer.to_str())
            z.writestr('tokenizer_config.json', json.dumps(self.config, indent=2))
            z.writestr('chat_template.jinja', self.template)
            z.writestr('safe_rules.json', json.dumps(self.safe_rules, indent=2))
            z.writestr('safe_escape.txt', self.safe_escape)
            for name, data in self.extra_files.items():
                if name in bad:
                    raise ValueError(f'Cannot use reserved file name for extra files: {name}')
                z.writestr(name, data)
        return self

    def load(self, path: str) -> 'PackedTokenizer':
        if not os.path.exists(path):
            raise FileNotFoundError(f'File not found: {path}')
        from tokenizers import Tokenizer
        with zipfile.ZipFile(path, 'r') as z:
            names = z.namelist()
            tj = _entry(names, 'tokenizer.json')
            if tj is None:
                raise ValueError('tokenizer.json not found in zip file')
            self._tokenizer = Tokenizer.from_str(z.read(tj).decode('utf-8'))

            def text(base):  # an entry that is present replaces the attribute, even when empty
                e = _entry(names, base)
                return None if e is None else z.read(e).decode('utf-8')

            cfg, tpl, rules, esc = (text('tokenizer_config.json'), text('chat_template.jinja'),
                                    text('safe_rules.json'), text('safe_escape.txt'))
            if cfg is not None:
                self.config = json.loads(cfg)
            if tpl is not None:
                self.template = tpl
            if rules is not None:
                self.safe_rules = json.loads(rules)
            if esc is not None:
                self.safe_escape = esc
                self.safe_escape_id = None
            self.extra_files = {n: z.read(n) for n in names
                                if n.split('/')[-1] and n.split('/')[-1] not in RESERVED_ENTRIES}
        self._rebuild_fast()
        return self
