"""Configuration dataclasses for the drafter training step.

Field names and defaults mirror the reference's ``pe.config`` so that a caller
switching packages keeps its configuration code unchanged
(reference ``src/pe/config.py:17-32`` TargetConfig, ``:35-56`` DrafterConfig,
``:59-81`` TrainConfig, ``:84-93`` FeatureConfig).  The decode, distillation and
benchmark configs of the reference configure paths outside the training step and
are not carried here.

Architectural dimensions (hidden size, heads, vocabulary, RoPE base) are left as
``None`` and are taken from the frozen target heads at build time, exactly as the
reference does, so the drafter cannot drift from the model it serves.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

DEFAULT_TARGET = "meta-llama/Llama-3.2-1B-Instruct"


@dataclass
class TargetConfig:
    """Which frozen target the shared embedding / LM head / final norm come from."""

    model_name: str = DEFAULT_TARGET
    feature_layers: tuple[int, ...] | None = None
    dtype: str = "bfloat16"
    device: str = "cuda"
    device_map: object | None = None


@dataclass
class DrafterConfig:
    """Drafter architecture knobs; ``max_depth`` is K, the prediction slots per anchor."""

    num_layers: int = 2
    max_depth: int = 8
    dropout: float = 0.0
    rms_norm_eps: float = 1e-5

    hidden_size: int | None = None
    num_attention_heads: int | None = None
    num_key_value_heads: int | None = None
    intermediate_size: int | None = None
    vocab_size: int | None = None
    rope_theta: float | None = None
    num_feature_layers: int = 3


@dataclass
class TrainConfig:
    """Drafter training on cached features (``save_every`` > 0 adds mid-epoch checkpoints)."""

    feature_cache_dir: Path = Path("features_cache")
    out_dir: Path = Path("checkpoints")
    max_seq_len: int = 2048
    batch_size: int = 1
    grad_accum: int = 8
    num_segments: int = 1
    lr: float = 1e-4
    warmup_ratio: float = 0.0025
    weight_decay: float = 0.0
    epochs: int = 1
    seed: int = 0
    use_8bit_adam: bool = True
    grad_checkpoint: bool = True
    log_every: int = 20
    save_every: int = 0


@dataclass
class FeatureConfig:
    """Layout knobs of the on-disk feature shards read by :class:`FeatureDataset`."""

    out_dir: Path = Path("features_cache")
    dataset: str = "HuggingFaceH4/ultrachat_200k"
    split: str = "train_sft"
    max_examples: int = 2000
    max_seq_len: int = 2048
    shard_size: int = 256
