"""Reader for the cached target-feature shards the drafter trains on.

Format (reference ``src/pe/features.py:116-157``): ``manifest.json`` with
``shards``, ``num_examples``, ``feature_dim``, optional ``feature_layers`` and
``self_distilled``; each shard is a ``torch.save``'d list of dicts with
``input_ids`` (int64 [n]), ``features`` (fp16 [n, feature_dim]) and, for
self-distilled caches, ``prompt_len`` and ``labels``.  An optional
``heads.pt`` holds the frozen embedding / LM head / final norm.

Feature extraction itself (running the frozen target over a dataset) is not
part of the training step and is not provided here.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch


class FeatureDataset:
    """Iterates cached ``(input_ids, features)`` examples across shards, or
    ``(input_ids, features, prompt_len, labels)`` with ``with_prompt_len=True``."""

    def __init__(self, cache_dir: str | Path, with_prompt_len: bool = False, pin_memory: bool = False):
        self.dir = Path(cache_dir)
        manifest = self.dir / "manifest.json"
        if not manifest.exists():
            raise FileNotFoundError(
                f"No feature cache at {self.dir} (missing manifest.json). "
                "Run `python -m pe.features` (or `python -m pe.distill`) first."
            )
        self.manifest = json.loads(manifest.read_text())
        self.feature_dim = self.manifest["feature_dim"]
        self.feature_layers = tuple(self.manifest.get("feature_layers", ()))
        self.self_distilled = bool(self.manifest.get("self_distilled", False))
        self.heads_dump = self.dir / "heads.pt"
        self.with_prompt_len = with_prompt_len
        self.pin_memory = pin_memory

    def __len__(self) -> int:
        return self.manifest["num_examples"]

    def __iter__(self):
        for shard in self.manifest["shards"]:
            for ex in torch.load(self.dir / shard, weights_only=False):
                ids, feats = ex["input_ids"], ex["features"]
                if self.pin_memory and torch.cuda.is_available():
                    # page-locked so the per-sequence host->device copy is asynchronous
                    ids, feats = ids.pin_memory(), feats.pin_memory()
                if self.with_prompt_len:
                    yield ids, feats, int(ex.get("prompt_len", 0)), ex.get("labels")
                else:
                    yield ids, feats
