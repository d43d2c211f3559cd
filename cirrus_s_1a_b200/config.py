"""Model shapes for the cirrus-s-1a decode path.

The field names, defaults and presets are the reference's interface
(``cirrus/config.py:32-79`` for ``ModelConfig``, ``:182-219`` for the presets),
kept identical so that a reference ``ModelConfig`` and this one are
interchangeable: the engine only reads attributes, so either object works.

``baseline_config()`` gives the shapes the B200 benchmarks are quoted on:
the reference default preset with vocab 32000, 12 GDN heads of 64, 12 query /
4 KV heads of 64, window 2048, top-k 512 and a 4 x 64 lightning indexer.
"""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class ModelConfig:
    name: str = "cirrus-s-1a"
    vocab_size: int = 32_768
    d_model: int = 768
    self_pattern: tuple = ("gdn", "gdn", "gdn", "swa")
    n_self_layers: int = 12
    n_cross_layers: int = 6
    gdn_heads: int = 6
    gdn_head_dim_k: int = 128
    gdn_head_dim_v: int = 128
    gdn_conv_size: int = 4
    n_q_heads: int = 6
    n_kv_heads: int = 2
    head_dim: int = 128
    swa_window: int = 1024
    rope_theta: float = 1_000_000.0
    partial_rotary: float = 0.5
    sparse_topk: int | None = 2048
    indexer_heads: int = 4
    indexer_dim: int = 64
    ffn_hidden: int = 2048
    n_mtp_heads: int = 1
    mtp_passes: int = 2
    mtp_draft_vocab: int = 8192
    tie_embeddings: bool = True
    max_seq_len: int = 65_536
    norm_eps: float = 1e-6

    def __post_init__(self) -> None:
        if self.n_q_heads % self.n_kv_heads:
            raise ValueError("n_q_heads must be divisible by n_kv_heads")
        if self.n_self_layers <= 0 or self.n_cross_layers <= 0:
            raise ValueError("need at least one self and one cross layer")

    @property
    def self_layer_kinds(self) -> list:
        p = self.self_pattern
        return [p[i % len(p)] for i in range(self.n_self_layers)]

    @property
    def q_dim(self) -> int:
        return self.n_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def rot_dim(self) -> int:
        """Rotary channels per head; same rounding as ``layers.py:67``."""
        return int(self.head_dim * self.partial_rotary) // 2 * 2


PRESETS: dict[str, ModelConfig] = {
    "cirrus-s-1a": ModelConfig(),
    "cirrus-s-1a-large": ModelConfig(
        name="cirrus-s-1a-large", d_model=1024, n_self_layers=12, n_cross_layers=8, gdn_heads=8,
        n_q_heads=8, n_kv_heads=2, ffn_hidden=2816,
    ),
    "cirrus-s-1a-debug": ModelConfig(
        name="cirrus-s-1a-debug", vocab_size=512, d_model=64, n_self_layers=4, n_cross_layers=2,
        gdn_heads=2, gdn_head_dim_k=16, gdn_head_dim_v=16, n_q_heads=4, n_kv_heads=2, head_dim=16,
        swa_window=8, sparse_topk=6, indexer_heads=2, indexer_dim=8, ffn_hidden=128,
        mtp_draft_vocab=128, max_seq_len=256,
    ),
}


def get_config(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError as e:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}") from e


def baseline_config() -> ModelConfig:
    """The benchmark shapes (about 155M parameters, 83.7 MB of NVFP4 weights per step)."""
    return replace(
        get_config("cirrus-s-1a"), name="cirrus-s-1a-b200", vocab_size=32000, gdn_heads=12,
        gdn_head_dim_k=64, gdn_head_dim_v=64, n_q_heads=12, n_kv_heads=4, head_dim=64,
        swa_window=2048, sparse_topk=512, indexer_heads=4, indexer_dim=64,
    )
