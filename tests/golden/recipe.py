"""Seeded synthetic inputs shared by the golden-vector generator and the tests.

Everything here is drawn from explicit ``torch.Generator`` objects on the CPU so a
case is fully determined by its seeds; the fixtures store checksums of what the
reference saw so a drift in this recipe is detected instead of silently
changing the comparison.
"""

from __future__ import annotations

import torch

# Each golden case: dims + step arguments.  Shapes follow the reference's own CPU
# test model (hidden 32, 4/2 heads, vocab 64; reference tests/conftest.py:20-30) and
# the tiny BASELINE configuration (hidden 256, 4/2 heads, head_dim 64, I 688,
# vocab 1024, n 128, K 4).
CASES = {
    "tiny_fp32": dict(
        hidden=32, n_heads=4, n_kv_heads=2, intermediate=64, vocab=64, num_layers=2,
        max_depth=4, dtype="float32", n=9, seed=1, runs=[
            dict(num_segments=1), dict(num_segments=3), dict(num_segments=20),
            dict(num_segments=1, prompt_len=5), dict(num_segments=2, prompt_len=5),
            dict(num_segments=1, teacher_labels=True), dict(num_segments=3, loss_scale=0.25),
        ], norm_jitter=0.1, full=True,
    ),
    "tiny_k1_fp32": dict(
        hidden=32, n_heads=4, n_kv_heads=2, intermediate=64, vocab=64, num_layers=1,
        max_depth=1, dtype="float32", n=6, seed=2, runs=[dict(num_segments=1), dict(num_segments=2)],
        norm_jitter=0.1, full=True,
    ),
    "tiny_n2_fp32": dict(
        hidden=32, n_heads=4, n_kv_heads=2, intermediate=64, vocab=64, num_layers=1,
        max_depth=3, dtype="float32", n=2, seed=3, runs=[dict(num_segments=1), dict(num_segments=2)],
        norm_jitter=0.1, full=True,
    ),
    "tiny_bf16": dict(
        hidden=64, n_heads=4, n_kv_heads=2, intermediate=128, vocab=128, num_layers=1,
        max_depth=3, dtype="bfloat16", n=12, seed=4, runs=[dict(num_segments=1), dict(num_segments=2)],
        norm_jitter=0.1, full=True,
    ),
    "config1_fp32": dict(
        hidden=256, n_heads=4, n_kv_heads=2, intermediate=688, vocab=1024, num_layers=1,
        max_depth=4, dtype="float32", n=128, batch=2, seed=0, runs=[
            dict(num_segments=1), dict(num_segments=2),
        ], norm_jitter=0.0, full=False,
    ),
}

# Draft-time runs on the first sequence of each full case: context length p, drafted
# depths k (k - pending fresh ones for the tree / chain), tree beam parameters.
DRAFT_RUNS = [
    dict(p=1, k=1, pending=0, top_k=3, max_nodes=4),
    dict(p=5, k=4, pending=0, top_k=3, max_nodes=9, sequential=True),
    dict(p=6, k=3, pending=1, top_k=2, max_nodes=8),
    dict(p=9, k=5, pending=0, top_k=4, max_nodes=20),
]

SKETCH_ROWS = 64


def make_heads(vocab: int, hidden: int, seed: int, norm_jitter: float, dtype=torch.float32):
    """Frozen shared embedding / LM head ~ N(0, 0.02^2) and final-norm weight."""
    g = torch.Generator().manual_seed(10_000 + seed)
    embed = torch.randn(vocab, hidden, generator=g) * 0.02
    head = torch.randn(vocab, hidden, generator=g) * 0.02
    norm = torch.ones(hidden) + norm_jitter * torch.randn(hidden, generator=g)
    return {"embed": embed.to(dtype), "head": head.to(dtype), "norm": norm.to(dtype)}


def make_sequence(n: int, vocab: int, feature_dim: int, seed: int, index: int):
    """Token ids ~ U[0, vocab) and target features ~ N(0, 1) for sequence ``index``."""
    g = torch.Generator().manual_seed(20_000 + 97 * seed + index)
    ids = torch.randint(0, vocab, (n,), generator=g)
    feats = torch.randn(n, feature_dim, generator=g)
    return ids, feats


def teacher_labels_for(ids: torch.Tensor) -> torch.Tensor:
    """Self-consistent teacher labels (``labels[p] == ids[p+1]``), the reference's
    equivalence case (reference tests/test_distill.py:80-97)."""
    t = torch.empty_like(ids)
    t[:-1] = ids[1:]
    t[-1] = ids[-1]
    return t


def sketch(t: torch.Tensor, salt: int) -> torch.Tensor:
    """64 Gaussian random projections of a tensor (float64) -- a compact,
    position-sensitive fingerprint used where full tensors are too large to commit."""
    flat = t.detach().double().reshape(-1)
    g = torch.Generator().manual_seed(777 + salt)
    proj = torch.randn(SKETCH_ROWS, flat.numel(), generator=g, dtype=torch.float64)
    return proj @ flat


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().double()
    b = b.detach().double()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)
