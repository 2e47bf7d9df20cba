"""Draft proposals built on :meth:`ParallelDrafter.draft_logits` (the drafter's
serving-side consumer; reference ``src/pe/decode/tree.py`` and
``src/pe/decode/chain.py``).

One drafter pass gives a distribution at each of the ``k`` prediction depths.
The per-depth selection (log-softmax + top-k, or argmax) runs in one
``pe_topk_logprobs`` launch over all depths; only the small beam bookkeeping
(at most ``k * beam_width^2`` candidates) runs on the host, in the reference's
order, so ties in the cumulative score resolve the same way.
"""

from __future__ import annotations

import torch

from . import ops


def propose_tree(drafter, context_ids: torch.Tensor, context_feats: torch.Tensor, k: int,
                 top_k: int, max_nodes: int, pending: int = 0) -> tuple[list[int], list[int]]:
    """``(node_tokens, parents)`` in topological order (reference ``tree.py:19-57``).

    ``parents[t] == -1`` means the node hangs off the confirmed prefix; ``pending``
    leading depths (already-confirmed tokens) are skipped.  At each depth the
    ``beam_width = max(1, min(top_k, max_nodes // k))`` best tokens are attached to
    every surviving parent and the beam is re-pruned by cumulative log-probability.
    Equal log-probabilities order by token id (the reference leaves that order to
    ``torch.topk``)."""
    logits = drafter.draft_logits(context_ids, context_feats, k + pending)
    beam_width = max(1, min(top_k, max_nodes // max(1, k)))
    if k <= 0:
        return [], []
    vals, toks = ops.topk_logprobs(logits[pending:], beam_width)
    vals, toks = vals.tolist(), toks.tolist()
    beam: list[tuple[int, float]] = [(-1, 0.0)]  # (parent node index, cumulative logprob)
    node_tokens: list[int] = []
    parents: list[int] = []
    for d in range(k):
        cand = [(par, tok, cum + lp) for (par, cum) in beam for lp, tok in zip(vals[d], toks[d])]
        cand.sort(key=lambda c: c[2], reverse=True)
        beam = []
        for par, tok, cum in cand[:beam_width]:
            beam.append((len(node_tokens), cum))
            node_tokens.append(tok)
            parents.append(par)
    return node_tokens, parents


def propose_chain(drafter, context_ids: torch.Tensor, context_feats: torch.Tensor, k: int,
                  pending: int = 0) -> list[int]:
    """Top-1 token per fresh depth from one drafter pass (reference ``chain.py:15-23``)."""
    logits = drafter.draft_logits(context_ids, context_feats, k + pending)
    if k <= 0:
        return []
    _, toks = ops.topk_logprobs(logits[pending:], 1, raw=True)
    return [int(t) for t in toks[:, 0].tolist()]


def propose_chain_sequential(drafter, context_ids: torch.Tensor, context_feats: torch.Tensor,
                             k: int, pending: int = 0) -> list[int]:
    """The same chain from ``k + pending`` sequential drafter passes (reference
    ``chain.py:26-35``), the baseline parallel drafting replaces."""
    logits = drafter.draft_logits_sequential(context_ids, context_feats, k + pending)
    if k <= 0:
        return []
    _, toks = ops.topk_logprobs(logits[pending:], 1, raw=True)
    return [int(t) for t in toks[:, 0].tolist()]


def propose_chain_sampling(drafter, context_ids: torch.Tensor, context_feats: torch.Tensor,
                           k: int, temperature: float,
                           generator: torch.Generator | None = None) -> tuple[list[int], torch.Tensor]:
    """Sample one token per depth from the drafter's distributions at ``temperature``
    (reference ``chain.py:38-53``).  Returns the tokens and the ``[k, V]`` fp32
    distributions ``q`` (for the speculative-sampling residual).  ``q`` comes from
    ``pe_softmax_rows``; the draw is ``torch.multinomial`` with the caller's generator,
    as in the reference, so a seeded generator reproduces its tokens."""
    if not temperature > 0:
        raise ValueError(f"temperature must be positive, got {temperature}")
    logits = drafter.draft_logits(context_ids, context_feats, k)
    q = ops.softmax_rows(logits, temperature)
    tokens = torch.multinomial(q, 1, generator=generator).squeeze(-1)
    return [int(t) for t in tokens.tolist()], q
