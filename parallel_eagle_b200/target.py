"""The frozen target heads the drafter shares: embedding, LM head, final norm.

Same surface as the reference's ``TargetHeads`` / ``_heads_from_weights`` /
``load_heads_from_dump`` / ``load_target_heads`` (``src/pe/target.py:227-331``):
the weights are cast to the training dtype, placed on the training device and
frozen.  The full target-model wrapper (hidden-state extraction, KV cache,
tree verification) is inference-side and not part of this package.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import TargetConfig
from .nn import RMSNorm

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


@dataclass
class TargetHeads:
    config: object
    hidden_size: int
    vocab_size: int
    feature_dim: int
    num_feature_layers: int
    feature_layers: tuple[int, ...]
    embed: torch.nn.Module
    head: torch.nn.Module
    norm: torch.nn.Module

    def get_input_embeddings(self):
        return self.embed

    def get_lm_head(self):
        return self.head

    def get_final_norm(self):
        return self.norm


def resolve_feature_layers(feature_layers, num_hidden_layers: int) -> tuple[int, ...]:
    """Hidden-state slots to fuse (reference ``target.py:103-128``): ``None`` picks
    the depth-relative fractions 0.25 / 0.55 / 0.95; explicit (possibly negative)
    indices are clamped to ``[1, n]``; duplicates fall back to the defaults."""
    n = num_hidden_layers
    fracs = (0.25, 0.55, 0.95)
    layers = tuple(round(n * f) for f in fracs) if feature_layers is None else tuple(feature_layers)
    out = [max(1, min(i if i >= 0 else n + 1 + i, n)) for i in layers]
    if len(set(out)) < len(out):
        out = sorted({max(1, min(round(n * f), n)) for f in fracs})
        while len(out) < len(layers):
            out.append(out[-1])
    return tuple(out)


def _heads_from_weights(config, embed_w, head_w, norm_w, feature_layers, device, dtype) -> TargetHeads:
    vocab, hidden = embed_w.shape
    embed = torch.nn.Embedding(vocab, hidden, device="meta")
    embed.weight = torch.nn.Parameter(embed_w.to(device=device, dtype=dtype), requires_grad=False)
    head = torch.nn.Linear(hidden, head_w.shape[0], bias=False, device="meta")
    head.weight = torch.nn.Parameter(head_w.to(device=device, dtype=dtype), requires_grad=False)
    norm = RMSNorm(hidden, getattr(config, "rms_norm_eps", 1e-5))
    norm.weight = torch.nn.Parameter(norm_w.to(device=device, dtype=dtype), requires_grad=False)
    return TargetHeads(
        config=config,
        hidden_size=config.hidden_size,
        vocab_size=config.vocab_size,
        feature_dim=config.hidden_size * len(feature_layers),
        num_feature_layers=len(feature_layers),
        feature_layers=tuple(feature_layers),
        embed=embed,
        head=head,
        norm=norm,
    )


def load_heads_from_dump(dump_path, cfg: TargetConfig, feature_layers, feature_dim_check=None) -> TargetHeads:
    """Shared heads from a ``heads.pt`` dump plus the target's config
    (reference ``target.py:296-305``)."""
    from transformers import AutoConfig

    config = AutoConfig.from_pretrained(cfg.model_name)
    fl = resolve_feature_layers(feature_layers, config.num_hidden_layers)
    w = torch.load(dump_path, map_location="cpu", weights_only=False)
    return _heads_from_weights(config, w["embed"], w["head"], w["norm"], fl, cfg.device,
                               _DTYPES[cfg.dtype])


def load_target_heads(cfg: TargetConfig) -> TargetHeads:
    """Load only the embedding, LM head and final norm of a HF causal LM
    (reference ``target.py:308-331``, unquantized checkpoints)."""
    from transformers import AutoModelForCausalLM

    model = AutoModelForCausalLM.from_pretrained(cfg.model_name, dtype=torch.float16)
    base = model.get_decoder() if hasattr(model, "get_decoder") else model.model
    norm_mod = next(getattr(base, n) for n in ("norm", "final_layernorm", "ln_f") if hasattr(base, n))
    config = model.config
    fl = resolve_feature_layers(cfg.feature_layers, config.num_hidden_layers)
    heads = _heads_from_weights(
        config, model.get_input_embeddings().weight.data, model.get_output_embeddings().weight.data,
        norm_mod.weight.data, fl, cfg.device, _DTYPES[cfg.dtype],
    )
    del model
    return heads
