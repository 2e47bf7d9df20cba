"""Functional CPU restatement of the reference's draft-time path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  The drafter's serving-side
consumer: one forward over the confirmed context plus ``k - 1`` prediction
slots, the frozen LM head on the ``k`` prediction rows, and the tree / chain
proposals built from those logits.  Paths are relative to the reference root.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .drafter_step import OracleDims, additive_bias, drafter_forward, mask_input, real_input


def token_shared_input(p, heads, tok, dims: OracleDims):
    """``in_proj([embed(tok); h_shared])`` for drafted tokens the target has not seen
    (``src/pe/drafter.py:139-145``)."""
    dt = p["in_proj.weight"].dtype
    emb = heads["embed"][tok].to(dt)
    shared = p["h_shared"].unsqueeze(0).expand(emb.shape[0], -1)
    return F.linear(torch.cat([emb, shared], dim=-1), p["in_proj.weight"])


def draft_logits(p, heads, ids, feats, k: int, dims: OracleDims) -> torch.Tensor:
    """Logits ``[k, V]`` for the ``k`` tokens after the context
    (``src/pe/drafter.py:195-236``): real slots for the whole context, then ``k - 1``
    prediction slots anchored at the last context position (positions ``p-1+d``);
    prediction slots see the whole context and the prediction slots of depth
    ``<= d``.  Depth 0 is read at the last real slot, depth ``d`` at slot
    ``p + d - 1``."""
    n = ids.shape[0]
    m = n + (k - 1)
    dt = p["in_proj.weight"].dtype
    x = torch.empty(m, dims.hidden, dtype=dt)
    x[:n] = real_input(p, heads, ids, feats, dims)
    if k > 1:
        x[n:] = mask_input(p, k - 1)
    pos = torch.arange(m)
    pos[n:] = (n - 1) + torch.arange(1, k)
    allow = torch.zeros(m, m, dtype=torch.bool)
    allow[:n, :n] = torch.tril(torch.ones(n, n, dtype=torch.bool))
    if k > 1:
        allow[n:, :n] = True
        allow[n:, n:] = torch.tril(torch.ones(k - 1, k - 1, dtype=torch.bool))
    hidden = drafter_forward(p, heads, x, pos, additive_bias(allow, dt), dims)
    logits = F.linear(hidden, heads["head"].to(dt))
    idx = torch.empty(k, dtype=torch.long)
    idx[0] = n - 1
    if k > 1:
        idx[1:] = torch.arange(n, m)
    return logits[idx]


def draft_logits_sequential(p, heads, ids, feats, k: int, dims: OracleDims) -> torch.Tensor:
    """Greedy drafting with ``k`` causal forward passes, each appending the previous
    argmax token as ``token_shared_input`` (``src/pe/drafter.py:239-269``)."""
    dt = p["in_proj.weight"].dtype
    real_x = real_input(p, heads, ids, feats, dims)
    drafted: list[int] = []
    out = []
    for _ in range(k):
        if drafted:
            x = torch.cat([real_x, token_shared_input(p, heads, torch.tensor(drafted), dims)])
        else:
            x = real_x
        s = x.shape[0]
        bias = additive_bias(torch.tril(torch.ones(s, s, dtype=torch.bool)), dt)
        hidden = drafter_forward(p, heads, x, torch.arange(s), bias, dims)
        logits = F.linear(hidden[-1], heads["head"].to(dt))
        out.append(logits)
        drafted.append(int(logits.argmax()))
    return torch.stack(out)


def propose_tree_from_logits(logits, k: int, top_k: int, max_nodes: int, pending: int = 0):
    """Beam tree over per-depth log-probabilities (``src/pe/decode/tree.py:19-57``),
    given the ``[k + pending, V]`` draft logits.  Returns ``(node_tokens, parents)``."""
    logprobs = torch.log_softmax(logits.float(), dim=-1)[pending:]
    beam_width = max(1, min(top_k, max_nodes // max(1, k)))
    beam: list[tuple[int, float]] = [(-1, 0.0)]
    node_tokens: list[int] = []
    parents: list[int] = []
    for d in range(k):
        topv, topi = logprobs[d].topk(beam_width)
        topv, topi = topv.tolist(), topi.tolist()
        cand = [(par, tok, cum + lp) for (par, cum) in beam for lp, tok in zip(topv, topi)]
        cand.sort(key=lambda c: c[2], reverse=True)
        beam = []
        for par, tok, cum in cand[:beam_width]:
            beam.append((len(node_tokens), cum))
            node_tokens.append(tok)
            parents.append(par)
    return node_tokens, parents


def propose_chain_from_logits(logits, pending: int = 0) -> list[int]:
    """Top-1 token per depth (``src/pe/decode/chain.py:15-23``)."""
    return [int(t) for t in logits.argmax(-1)[pending:]]


def tree_allow(parents: list[int], prefix_len: int) -> torch.Tensor:
    """Verification-tree attend mask by a per-pair walk up the parent chain
    (``src/pe/masks.py:127-147``): prefix causal, nodes see the whole prefix and
    their ancestors (themselves included)."""
    t = len(parents)
    n = prefix_len + t
    allow = torch.zeros(n, n, dtype=torch.bool)
    for q in range(n):
        for kk in range(n):
            if kk < prefix_len:
                allow[q, kk] = q >= prefix_len or kk <= q
            elif q >= prefix_len:
                a = q - prefix_len
                while a >= 0 and a != kk - prefix_len:
                    a = parents[a]
                allow[q, kk] = a >= 0
    return allow


def tree_positions(parents: list[int], prefix_len: int) -> list[int]:
    """Prefix positions ``0 .. P-1``, then ``P + depth`` per node, the depth counted
    by walking to the root (``src/pe/masks.py:118-124,150-156``)."""
    out = list(range(prefix_len))
    for t in range(len(parents)):
        depth, a = 0, parents[t]
        while a >= 0:
            depth, a = depth + 1, parents[a]
        out.append(prefix_len + depth)
    return out
