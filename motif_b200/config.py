"""Model hyper-parameters, field-for-field the reference's `MotifChordConfig`.

Mirrors `motif/model/config.py:5-39` so that a config object (or a mapping of its
fields) built for the reference builds the same architecture here.  Two values the
reference hard-codes inside the layers are exposed as module constants instead of
fields, with the same values: `EXPAND_V = 2.0` and `CHUNK_SIZE = 64`
(`motif/block/decoder.py:82-89`), `CONV_SIZE = 4` (`gdn_attn.py:50`).
"""

from dataclasses import dataclass, fields
from typing import Optional, Tuple

EXPAND_V = 2.0
CHUNK_SIZE = 64
CONV_SIZE = 4
NORM_EPS = 1e-6
GGD_EPS = 1e-5


@dataclass
class MotifChordConfig:
    """Hyper-parameters of `MotifChordModel` (reference `model/config.py:5-39`)."""

    vocab_size: int = 5 * (2 ** 13)
    model_dim: int = 768
    num_heads: int = 12
    num_kv_heads: Optional[int] = 3
    head_k_dim: Optional[int] = 64
    tied_weight: bool = True
    block: Tuple[str, ...] = ('gdn', 'gdn', 'gdn', 'chord')
    block_n: int = 4

    @classmethod
    def from_any(cls, cfg) -> 'MotifChordConfig':
        """Build from this class, the reference's config object or a mapping."""
        if isinstance(cfg, cls):
            return cfg
        names = [f.name for f in fields(cls)]
        if isinstance(cfg, dict):
            return cls(**{k: cfg[k] for k in names if k in cfg})
        return cls(**{k: getattr(cfg, k) for k in names})

    @property
    def head_dim(self) -> int:
        return self.model_dim // self.num_heads

    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads if self.num_kv_heads is not None else self.num_heads

    @property
    def gdn_dk(self) -> int:
        return self.head_k_dim or self.head_dim

    @property
    def gdn_dv(self) -> int:
        return int(self.gdn_dk * EXPAND_V)

    @property
    def mlp_hidden(self) -> int:
        """SwiGLU width, `ceil128(int(8 d / 3))` (reference `block/mlp.py:42-44`)."""
        h = int(self.model_dim * 8 / 3)
        return (h + 127) // 128 * 128


# The five configurations the benchmark and the parity tests are quoted on.
def tiny_config() -> MotifChordConfig:
    """Config 1: one block of 3 GDN + 1 Chord, d=256, 4 heads of 64, vocab 32000."""
    return MotifChordConfig(vocab_size=32000, model_dim=256, num_heads=4,
                            num_kv_heads=None, head_k_dim=64,
                            block=('gdn', 'gdn', 'gdn', 'chord'), block_n=1)


def config_172m() -> MotifChordConfig:
    """Configs 4/5: d=768, 12 heads of 64 (3 kv heads), 4 blocks, vocab 32000."""
    return MotifChordConfig(vocab_size=32000, model_dim=768, num_heads=12,
                            num_kv_heads=3, head_k_dim=64,
                            block=('gdn', 'gdn', 'gdn', 'chord'), block_n=4)
