"""Shared helpers for the GPU parity tests and ``__graft_entry__.smoke()``.

Builds a seeded synthetic drafter case, runs the CUDA training step
(``parallel_eagle_b200.partition.mtp_backward``) and the CPU oracle on the same
inputs, and reports loss / per-parameter relative Frobenius errors.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import oracle  # noqa: E402
import recipe  # noqa: E402


def heads_object(heads: dict, n_heads: int, n_kv_heads: int, intermediate: int,
                 device="cuda", dtype=torch.float32):
    """Frozen shared embedding / LM head / final norm placed like the reference's
    ``_heads_from_weights`` (reference src/pe/target.py:255-281)."""
    from parallel_eagle_b200.nn import RMSNorm

    V, H = heads["embed"].shape
    embed = torch.nn.Embedding(V, H)
    embed.weight.data = heads["embed"].to(dtype)
    head = torch.nn.Linear(H, V, bias=False)
    head.weight.data = heads["head"].to(dtype)
    norm = RMSNorm(H, 1e-5)
    norm.weight.data = heads["norm"].to(dtype)
    for m in (embed, head, norm):
        m.to(device)
        for p in m.parameters():
            p.requires_grad_(False)
    cfg = types.SimpleNamespace(num_attention_heads=n_heads, num_key_value_heads=n_kv_heads,
                                intermediate_size=intermediate, rope_theta=10000.0,
                                rms_norm_eps=1e-5, hidden_size=H, vocab_size=V)
    return types.SimpleNamespace(config=cfg, hidden_size=H, vocab_size=V, feature_dim=3 * H,
                                 get_input_embeddings=lambda: embed, get_lm_head=lambda: head,
                                 get_final_norm=lambda: norm)


def make_case(hidden, n_heads, n_kv_heads, intermediate, vocab, num_layers, max_depth, n,
              dtype=torch.bfloat16, seed=0, batch=1, norm_jitter=0.1):
    dims = oracle.OracleDims(hidden=hidden, n_heads=n_heads, n_kv_heads=n_kv_heads,
                             intermediate=intermediate, vocab=vocab, num_layers=num_layers,
                             max_depth=max_depth)
    heads = recipe.make_heads(vocab, hidden, seed, norm_jitter, dtype)
    params = oracle.init_params(dims, seed, dtype)
    seqs = [recipe.make_sequence(n, vocab, 3 * hidden, seed, b) for b in range(batch)]
    seqs = [(i, f.to(dtype)) for i, f in seqs]
    return dict(dims=dims, heads=heads, params=params, seqs=seqs, dtype=dtype, seed=seed)


def build_drafter(case, device="cuda"):
    from parallel_eagle_b200.config import DrafterConfig
    from parallel_eagle_b200.drafter import ParallelDrafter

    d = case["dims"]
    target = heads_object(case["heads"], d.n_heads, d.n_kv_heads, d.intermediate, device,
                          case["dtype"])
    model = ParallelDrafter.from_target(target, DrafterConfig(num_layers=d.num_layers,
                                                              max_depth=d.max_depth))
    model.load_state_dict({k: v for k, v in case["params"].items()})
    return model.to(device=device, dtype=case["dtype"])


def cuda_step(case, drafter=None, **kw):
    """Run ``mtp_backward`` over every sequence of the case; returns (losses, grads)."""
    from parallel_eagle_b200.partition import mtp_backward

    model = drafter if drafter is not None else build_drafter(case)
    model.zero_grad(set_to_none=True)
    batch = len(case["seqs"])
    losses = []
    for b, (ids, feats) in enumerate(case["seqs"]):
        extra = dict(kw)
        extra.setdefault("loss_scale", 1.0 / batch)
        if extra.pop("teacher_labels_self", False):
            extra["teacher_labels"] = recipe.teacher_labels_for(ids)
        th = extra.pop("teacher_hidden_seed", None)
        if th is not None:
            g = torch.Generator().manual_seed(th + b)
            extra["teacher_hidden"] = torch.randn(ids.shape[0], case["dims"].hidden,
                                                  generator=g).to(case["dtype"])
        losses.append(mtp_backward(model, ids, feats, **extra))
    torch.cuda.synchronize()
    grads = {n: p.grad.detach().float().cpu() for n, p in model.named_parameters()
             if p.grad is not None}
    return losses, grads, model


def oracle_step(case, **kw):
    batch = len(case["seqs"])
    losses, grads = [], None
    for b, (ids, feats) in enumerate(case["seqs"]):
        extra = dict(kw)
        extra.setdefault("loss_scale", 1.0 / batch)
        if extra.pop("teacher_labels_self", False):
            extra["teacher_labels"] = recipe.teacher_labels_for(ids)
        th = extra.pop("teacher_hidden_seed", None)
        if th is not None:
            g = torch.Generator().manual_seed(th + b)
            extra["teacher_hidden"] = torch.randn(ids.shape[0], case["dims"].hidden,
                                                  generator=g).to(case["dtype"])
        loss, grads = oracle.mtp_step(case["params"], case["heads"], ids, feats, case["dims"],
                                      grads=grads, **extra)
        losses.append(loss)
    return losses, {k: v.float() for k, v in grads.items()}


def compare_step(case, **kw):
    losses, grads, _ = cuda_step(case, **kw)
    olosses, ograds = oracle_step(case, **kw)
    loss_rel = max(abs(a - b) / max(1e-12, abs(b)) for a, b in zip(losses, olosses))
    rel = {k: recipe.rel_fro(grads[k], ograds[k]) for k in ograds}
    assert grads.keys() == ograds.keys(), (sorted(grads), sorted(ograds))
    return dict(loss=losses[0], oracle_loss=olosses[0], loss_rel=loss_rel, grad_rel=rel)
