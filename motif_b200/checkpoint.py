"""Checkpoint I/O for `MotifChordModel.from_pretrained` (`motif/model/checkpoint.py`).

The same three layouts the reference reads, resolved to (weights, config):

* a bare `state_dict` written by `torch.save` (`.pt` / `.pth`);
* a training-pipeline checkpoint: a mapping whose `payload['model']` is the state_dict,
  or a mapping holding it under `state_dict` / `model_state_dict` / `weights` / `model`;
* safetensors: one file, a directory of shards (`model.safetensors` first), or an
  `*.index.json` shard index.

Key prefixes added by wrappers (`module.`, `_orig_mod.`, `_forward_module.`,
`_checkpoint_wrapped_module.`, `model.`) are removed while every key carries them.  The
config comes from the file (a `config`-like entry of the mapping or of the safetensors
metadata, else a `config.json` beside the weights) or, failing that, from the tensor
shapes (`config_from_state_dict`).  `save_safetensors` writes the layout `load_checkpoint`
reads back: the weights (the tied `lm_head.weight` dropped when it shares storage with
`embed.weight`) and the config as JSON under the `config` metadata key.

Loading is host-side and runs on the CPU (`map_location='cpu'` by default); the weights
reach the GPU with the model's `.to()`.
"""

import json
import os
import re
from dataclasses import asdict, dataclass, field, fields
from enum import Enum, auto
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .config import MotifChordConfig

__all__ = ['LoadedCheckpoint', 'load_checkpoint', 'save_safetensors', 'config_from_state_dict',
           'config_from_mapping', 'strip_wrapper_prefixes', 'looks_like_safetensors']

_PREFIXES = ('module.', '_orig_mod.', '_forward_module.', '_checkpoint_wrapped_module.', 'model.')
_CONFIG_KEYS = ('config', 'model_config', 'motif_config', 'modelconfig', 'config_dict')
# common names for the config fields in foreign config files (checkpoint.py:73-84)
_ALIASES = {'hidden_size': 'model_dim', 'd_model': 'model_dim', 'n_embd': 'model_dim',
            'num_hidden_layers': 'block_n', 'n_layers': 'block_n', 'num_layers': 'block_n',
            'num_attention_heads': 'num_heads', 'n_heads': 'num_heads',
            'num_key_value_heads': 'num_kv_heads', 'n_kv_heads': 'num_kv_heads'}
_FIELDS = {f.name for f in fields(MotifChordConfig)}


@dataclass
class LoadedCheckpoint:
    """Weights (canonical names) plus the config the file carried (None: infer it)."""

    state_dict: Dict[str, torch.Tensor]
    config: Optional[MotifChordConfig]
    source: str
    path: str
    metadata: Dict[str, str] = field(default_factory=dict)


def looks_like_safetensors(path: str) -> bool:
    """A `.safetensors` name, or a file that starts with a plausible little-endian header
    length followed by a JSON object."""
    if path.endswith('.safetensors'):
        return True
    if path.endswith('.index.json') or not os.path.isfile(path):
        return False
    try:
        size = os.path.getsize(path)
        with open(path, 'rb') as f:
            raw = f.read(8)
            if len(raw) < 8:
                return False
            n = int.from_bytes(raw, 'little')
            if n <= 0 or n > 256 * 1024 * 1024 or 8 + n > size:
                return False
            return f.read(min(n, 64)).lstrip()[:1] == b'{'
    except OSError:
        return False


def strip_wrapper_prefixes(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Remove wrapper prefixes, one at a time, while every key carries the same one."""
    cur = dict(sd)
    while cur:
        for p in _PREFIXES:
            if all(k.startswith(p) for k in cur):
                cur = {k[len(p):]: v for k, v in cur.items()}
                break
        else:
            break
    return cur


def config_from_mapping(spec: Dict[str, Any]) -> MotifChordConfig:
    """A config from a mapping of fields or their common aliases; other keys are ignored."""
    kw = {}
    for k, v in spec.items():
        name = _ALIASES.get(k, k)
        if name in _FIELDS:
            kw[name] = tuple(v) if name == 'block' and isinstance(v, list) else v
    return MotifChordConfig(**kw)


def _config_from_any(value) -> Optional[MotifChordConfig]:
    if value is None:
        return None
    if isinstance(value, MotifChordConfig):
        return value
    if hasattr(value, 'model_dim') and hasattr(value, 'block'):  # the reference's config object
        return MotifChordConfig.from_any(value)
    if isinstance(value, (str, bytes)):
        try:
            value = json.loads(value)
        except (TypeError, ValueError):
            return None
    return config_from_mapping(value) if isinstance(value, dict) else None


def _find_config(*containers) -> Optional[MotifChordConfig]:
    for c in containers:
        if isinstance(c, dict):
            for k in _CONFIG_KEYS:
                if k in c:
                    cfg = _config_from_any(c[k])
                    if cfg is not None:
                        return cfg
    return None


def config_from_state_dict(sd: Dict[str, torch.Tensor]) -> MotifChordConfig:
    """The hyper-parameters recovered from tensor shapes (`checkpoint.py:441-558`): vocab and
    width from the embedding, `block_n` from the highest block index, the recipe from each
    block-0 layer's marker parameters (`theta_alpha` -> chord, `a_proj` / `q_conv` /
    `A_log` -> gated delta net), heads from the per-head vectors, kv heads from a chord
    `k_proj`, `head_k_dim` from a GDN `q_proj` (64 when there is none), tying from whether the
    head equals the embedding."""
    emb = sd.get('embed.weight', sd.get('lm_head.weight'))
    if emb is None:
        raise ValueError("cannot infer the config: the state_dict has neither 'embed.weight' nor 'lm_head.weight'.")
    if emb.dim() != 2:
        raise ValueError(f"cannot infer the config: 'embed.weight' has shape {tuple(emb.shape)}, "
                         f'expected [vocab_size, model_dim].')
    vocab, dim = int(emb.shape[0]), int(emb.shape[1])
    blocks = sorted({int(m.group(1)) for k in sd if (m := re.match(r'blocks\.(\d+)\.', k))})
    if not blocks:
        raise ValueError("cannot infer the config: the state_dict has no 'blocks.<n>.' keys.")
    feats = sorted({int(m.group(1)) for k in sd if (m := re.match(r'blocks\.0\.features\.(\d+)\.', k))})
    if not feats:
        raise ValueError("cannot infer the config: block 0 has no 'features.<n>.' keys.")
    recipe: List[str] = []
    heads = kv = hk = None
    for i in feats:
        p = f'blocks.0.features.{i}.attn.'
        if p + 'theta_alpha' in sd:
            recipe.append('chord')
            n = int(sd[p + 'theta_alpha'].shape[0])
            heads = heads or n
            hd = dim // n
            kw = sd.get(p + 'k_proj.weight')
            if kw is not None and hd > 0:
                kv = int(kw.shape[0]) // hd
        elif p + 'a_proj.weight' in sd or p + 'q_conv.weight' in sd or p + 'A_log' in sd:
            recipe.append('gdn')
            anchor = sd.get(p + 'a_proj.weight', sd.get(p + 'A_log'))
            if anchor is not None:
                heads = heads or int(anchor.shape[0])
            qw = sd.get(p + 'q_proj.weight')
            if qw is not None and heads:
                hk = int(qw.shape[0]) // int(heads)
        else:
            raise ValueError(f"cannot infer the config: {p} carries neither chord ('theta_alpha') nor gated "
                             f"delta-net ('q_conv' / 'a_proj') weights.")
    if heads is None:
        raise ValueError('cannot infer the config: no per-head parameter was found.')
    head = sd.get('lm_head.weight')
    tied = head is None or head is emb or (tuple(head.shape) == tuple(emb.shape) and torch.equal(head, emb))
    return MotifChordConfig(vocab_size=vocab, model_dim=dim, num_heads=int(heads),
                            num_kv_heads=int(kv if kv is not None else heads),
                            head_k_dim=int(hk) if hk is not None else 64, tied_weight=bool(tied),
                            block=tuple(recipe), block_n=blocks[-1] + 1)


def _is_tensor_dict(v) -> bool:
    return isinstance(v, dict) and len(v) > 0 and all(isinstance(x, torch.Tensor) for x in v.values())


def _from_mapping(obj, path: str) -> LoadedCheckpoint:
    """Weights and config out of a `torch.load` result (`checkpoint.py:629-677`)."""
    if isinstance(obj, nn.Module):
        return LoadedCheckpoint(strip_wrapper_prefixes(obj.state_dict()), None, 'nn.Module', path)
    if not isinstance(obj, dict):
        raise ValueError(f'{path!r} holds {type(obj).__name__}, expected a state_dict / a checkpoint mapping.')
    payload = obj.get('payload')
    if isinstance(payload, dict):
        cfg = _find_config(obj, payload)
        model = payload.get('model')
        if isinstance(model, nn.Module):
            return LoadedCheckpoint(strip_wrapper_prefixes(model.state_dict()), cfg, 'pipeline checkpoint', path)
        if _is_tensor_dict(model):
            name = obj.get('__pipeline__') or 'pipeline'
            return LoadedCheckpoint(strip_wrapper_prefixes(model), cfg, f'pipeline checkpoint ({name!r})', path)
    for key in ('state_dict', 'model_state_dict', 'weights', 'model'):
        cand = obj.get(key)
        if isinstance(cand, nn.Module):
            return LoadedCheckpoint(strip_wrapper_prefixes(cand.state_dict()), _find_config(obj),
                                    f'{key}=nn.Module', path)
        if _is_tensor_dict(cand):
            return LoadedCheckpoint(strip_wrapper_prefixes(cand), _find_config(obj), f'state_dict under {key!r}', path)
    tensors = {k: v for k, v in obj.items() if isinstance(v, torch.Tensor)}
    if tensors:
        return LoadedCheckpoint(strip_wrapper_prefixes(tensors), _find_config(obj), 'bare state_dict', path)
    raise ValueError(f'cannot find model weights in {path!r}: the mapping has keys {sorted(obj)[:8]}.')


class PipelinePhase(Enum):
    """Stand-in for the training pipeline's phase enum.  A pipeline checkpoint's training state
    holds one of its members, pickled under the name `motif.pipeline.base.PipelinePhase`; the
    class is registered under that name for `weights_only` loading so such a checkpoint loads
    without importing the training pipeline and without the full unpickler (the reference does
    the same, `motif/model/checkpoint.py:27-60`).  The member names are the pickle contract."""

    INIT = auto()
    SETUP = auto()
    TRAINING = auto()
    EVALUATING = auto()
    FINISHED = auto()
    INTERRUPTED = auto()
    FAILED = auto()


_SAFE_GLOBALS = [(PipelinePhase, 'motif.pipeline.base.PipelinePhase')]


def _torch_load(path: str, map_location):
    errors = []
    with torch.serialization.safe_globals(_SAFE_GLOBALS):
        for kw in ({'weights_only': True, 'mmap': True}, {'weights_only': True}, {'weights_only': False, 'mmap': True},
                   {'weights_only': False}):
            try:
                return torch.load(path, map_location=map_location, **kw)
            except Exception as e:  # noqa: BLE001 - every form is tried, the errors are reported together
                errors.append(f'{kw}: {type(e).__name__}: {e}')
    raise RuntimeError(f'failed to load {path!r} with torch.load:\n  ' + '\n  '.join(errors))


def _shards(path: str) -> Tuple[List[str], Optional[str]]:
    """The safetensors files of a file / directory / shard index, and a sibling config.json."""
    def sidecar(d):
        c = os.path.join(d, 'config.json')
        return c if os.path.isfile(c) else None

    if path.endswith('.index.json'):
        d = os.path.dirname(os.path.abspath(path)) or '.'
        with open(path, 'r', encoding='utf-8') as f:
            wm = json.load(f).get('weight_map') or {}
        files = sorted({os.path.join(d, n) for n in wm.values()})
        if not files:
            raise FileNotFoundError(f'{path} lists no weight shards.')
        return files, sidecar(d)
    if os.path.isdir(path):
        d = os.path.abspath(path)
        pref = os.path.join(d, 'model.safetensors')
        if os.path.isfile(pref):
            return [pref], sidecar(d)
        files = sorted(os.path.join(d, n) for n in os.listdir(d) if n.endswith('.safetensors'))
        if not files:
            raise FileNotFoundError(f'no .safetensors file under {path!r}.')
        return files, sidecar(d)
    return [os.path.abspath(path)], sidecar(os.path.dirname(os.path.abspath(path)))


def load_checkpoint(path: str, map_location: Any = 'cpu') -> LoadedCheckpoint:
    """Read a checkpoint in any supported layout (`checkpoint.py:716-760`)."""
    path = os.fspath(path)
    if not os.path.exists(path):
        raise FileNotFoundError(f'checkpoint not found: {path!r}')
    if os.path.isdir(path) or looks_like_safetensors(path) or path.endswith('.index.json'):
        try:
            from safetensors import safe_open
        except ImportError as e:
            raise ImportError('reading a safetensors checkpoint needs the `safetensors` package.') from e
        files, side = _shards(path)
        sd: Dict[str, torch.Tensor] = {}
        meta: Dict[str, str] = {}
        for fpath in files:
            with safe_open(fpath, framework='pt', device=str(map_location)) as f:
                for k in f.keys():
                    sd[k] = f.get_tensor(k)
                meta.update(dict(f.metadata() or {}))
        cfg = _find_config(meta)
        if cfg is None and side is not None:
            with open(side, 'r', encoding='utf-8') as f:
                cfg = _config_from_any(json.load(f))
        label = 'safetensors' if len(files) == 1 else f'safetensors ({len(files)} shards)'
        return LoadedCheckpoint(strip_wrapper_prefixes(sd), cfg, label, path, meta)
    return _from_mapping(_torch_load(path, map_location), path)


def config_to_dict(cfg: MotifChordConfig) -> Dict[str, Any]:
    return {k: list(v) if isinstance(v, tuple) else v for k, v in asdict(cfg).items()}


def save_safetensors(model_or_state, path: str, config=None, metadata: Optional[Dict[str, Any]] = None):
    """Write weights + config into one `.safetensors` file (`checkpoint.py:263-368`): the config
    as JSON under `config` in the metadata, `lm_head.weight` dropped when it shares storage
    with `embed.weight`.  Accepts a module, a state_dict or a checkpoint path."""
    from safetensors.torch import save_file
    source = 'state_dict'
    cfg = config if isinstance(config, MotifChordConfig) else None
    if isinstance(model_or_state, (str, os.PathLike)):
        loaded = load_checkpoint(os.fspath(model_or_state))
        sd, source = loaded.state_dict, loaded.source
        cfg = cfg or loaded.config
    elif isinstance(model_or_state, nn.Module):
        sd, source = model_or_state.state_dict(), type(model_or_state).__name__
        if cfg is None and getattr(model_or_state, 'config', None) is not None:
            cfg = MotifChordConfig.from_any(model_or_state.config)
    elif isinstance(model_or_state, dict):
        sd = model_or_state
    else:
        raise ValueError(f'cannot save {type(model_or_state).__name__}: expected an nn.Module, a state_dict or a '
                         f'checkpoint path.')
    if not sd:
        raise ValueError('no weights to save.')
    if isinstance(config, dict):
        cfg = config_from_mapping(config)
    if cfg is None:
        cfg = config_from_state_dict(sd)
    emb, head = sd.get('embed.weight'), sd.get('lm_head.weight')
    dropped = []
    if emb is not None and head is not None and emb is not head and emb.data_ptr() == head.data_ptr() \
            and tuple(emb.shape) == tuple(head.shape) and emb.device == head.device:
        sd = {k: v for k, v in sd.items() if k != 'lm_head.weight'}
        dropped = ['lm_head.weight']
    out = {}
    for k, v in sd.items():
        if not isinstance(v, torch.Tensor):
            raise ValueError(f'{k!r} is not a tensor ({type(v).__name__}).')
        out[k] = v.detach().to('cpu').contiguous()
    info = {'format': 'pt', 'producer': 'motif-checkpoint/1', 'config': json.dumps(config_to_dict(cfg))}
    for k, v in (metadata or {}).items():
        info[str(k)] = v if isinstance(v, str) else json.dumps(v)
    d = os.path.dirname(os.path.abspath(os.fspath(path)))
    if not os.path.isdir(d):
        raise FileNotFoundError(f'destination directory does not exist: {d!r}')
    save_file(out, os.fspath(path), metadata=info)
    return {'path': os.fspath(path), 'source': source, 'tensors': len(out),
            'params': int(sum(v.numel() for v in out.values())), 'bytes': os.path.getsize(path),
            'config': config_to_dict(cfg), 'dropped': dropped, 'metadata': info}
