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

from . import _lib as L
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


# ---------------------------------------------------------------------------
# Verification: accept the drafts the target agrees with (reference
# src/pe/decode/verify.py).  The target's argmaxes over every position a rule may
# visit come from one pe_topk_logprobs launch (raw mode: the first maximal column,
# as torch.argmax); the walk itself is host bookkeeping over those integers.
# ---------------------------------------------------------------------------


def _argmax_rows(rows: torch.Tensor) -> list[int]:
    """First maximal column of each row (``torch.argmax``; NaN ranks highest) for
    float32, bfloat16 or float16 logits.  float16 is widened to float32, which is
    exact; other dtypes (float64 included, whose distinct maxima could round to
    equal float32 values) are rejected rather than silently rounded."""
    if rows.dtype == torch.float16:
        rows = rows.float()
    elif rows.dtype not in (torch.float32, torch.bfloat16):
        raise L.PeError(f"target logits must be float32, bfloat16 or float16, got {rows.dtype}")
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    _, idx = ops.topk_logprobs(rows, 1, raw=True)
    return [int(t) for t in idx[:, 0].tolist()]


def _check_prefix(prefix_len: int) -> None:
    if prefix_len < 1:
        raise ValueError(f"prefix_len must be at least 1, got {prefix_len}")


def _tree_walk(truth_after, node_tokens, parents) -> tuple[list[int], int]:
    # truth_after(node) = the target's token after `node` (-1: after the prefix)
    children: dict[int, list[int]] = {}
    for t, par in enumerate(parents):
        children.setdefault(int(par), []).append(t)
    path: list[int] = []
    at = -1
    while True:
        want = truth_after(at)
        nxt = next((t for t in children.get(at, ()) if int(node_tokens[t]) == want), None)
        if nxt is None:
            return path, want
        path.append(nxt)
        at = nxt


def accept_chain_greedy(logits: torch.Tensor, prefix_len: int,
                        draft_tokens) -> tuple[list[int], int]:
    """Longest draft prefix equal to the target's greedy tokens, plus the target's
    token after it (reference ``verify.py:17-32``).  ``logits`` ``[P + K, V]`` covers
    ``[prefix | drafts]``; rows P-1 .. P-1+K are read."""
    _check_prefix(prefix_len)
    k = len(draft_tokens)
    truth = _argmax_rows(logits[prefix_len - 1:prefix_len + k])
    a = 0
    while a < k and int(draft_tokens[a]) == truth[a]:
        a += 1
    return [int(t) for t in draft_tokens[:a]], truth[a]


def accept_tree_greedy(logits: torch.Tensor, prefix_len: int, node_tokens,
                       parents) -> tuple[list[int], int]:
    """Follow the target's argmax down a drafted tree (reference ``verify.py:35-57``):
    the accepted node indices and the bonus token.  ``logits`` covers
    ``[prefix | tree nodes]``."""
    _check_prefix(prefix_len)
    truth = _argmax_rows(logits[prefix_len - 1:prefix_len + len(parents)])
    return _tree_walk(lambda node: truth[node + 1], node_tokens, parents)


def accept_chain_cached(root_logit: torch.Tensor, node_logits: torch.Tensor,
                        draft_tokens) -> tuple[list[int], int]:
    """The chain rule over cached predictions (reference ``verify.py:60-72``):
    ``root_logit`` ``[V]`` predicts the first draft, ``node_logits[m]`` the one after
    draft m."""
    k = len(draft_tokens)
    rows = torch.cat([root_logit.reshape(1, -1), node_logits[:k].reshape(-1, root_logit.numel())])
    truth = _argmax_rows(rows)
    a = 0
    while a < k and int(draft_tokens[a]) == truth[a]:
        a += 1
    return [int(t) for t in draft_tokens[:a]], truth[a]


def accept_tree_cached(root_logit: torch.Tensor, node_logits: torch.Tensor, node_tokens,
                       parents) -> tuple[list[int], int]:
    """The tree rule over cached predictions (reference ``verify.py:104-125``):
    ``node_logits[t]`` predicts the token after tree node ``t``."""
    n = len(parents)
    rows = torch.cat([root_logit.reshape(1, -1), node_logits[:n].reshape(-1, root_logit.numel())])
    truth = _argmax_rows(rows)
    return _tree_walk(lambda node: truth[node + 1], node_tokens, parents)


def accept_chain_sampling(target_dists: torch.Tensor, draft_tokens, q_dists: torch.Tensor,
                          generator: torch.Generator | None = None) -> tuple[list[int], int]:
    """Lossless speculative-sampling acceptance of a sampled chain (reference
    ``verify.py:75-101``): draft i is kept with probability min(1, p_i / q_i); the
    first rejection draws the bonus from relu(p - q) normalised, and a fully accepted
    chain draws it from the trailing target distribution.  The draws are the same
    ``torch.rand`` / ``torch.multinomial`` calls in the same order, so a seeded
    generator reproduces the reference's decisions."""
    accepted: list[int] = []
    for i, tok in enumerate(draft_tokens):
        keep = torch.clamp(target_dists[i, tok] / q_dists[i, tok], max=1.0)
        u = torch.rand((), generator=generator, device=target_dists.device)
        if not bool(u < keep):
            resid = torch.clamp(target_dists[i] - q_dists[i], min=0)
            resid = resid / resid.sum()
            return accepted, int(torch.multinomial(resid, 1, generator=generator))
        accepted.append(int(tok))
    return accepted, int(torch.multinomial(target_dists[len(draft_tokens)], 1,
                                           generator=generator))
