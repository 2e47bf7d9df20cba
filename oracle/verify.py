"""CPU restatement of the reference's draft verification (acceptance) rules.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Given the target's outputs
over a drafted chain or tree, these return the accepted drafts and the target's
bonus token (``src/pe/decode/verify.py``; paths relative to the reference root).
Greedy acceptance keeps the longest prefix / tree path whose every token is the
target's argmax at its position; speculative-sampling acceptance keeps draft i
with probability min(1, p_i / q_i) and resamples from the residual on the first
rejection.  Pinned by ``tests/golden/verify_cases.pt`` (made by running the
reference).
"""

from __future__ import annotations

import torch


def _top(row: torch.Tensor) -> int:
    return int(torch.argmax(row))


def accept_chain_greedy(logits, prefix_len: int, draft_tokens):
    """``src/pe/decode/verify.py:17-32``: the target at position p-1+m predicts the
    m-th draft; stop at the first mismatch, bonus = the target's choice there."""
    taken = []
    for m, tok in enumerate(draft_tokens):
        if int(tok) != _top(logits[prefix_len - 1 + m]):
            break
        taken.append(int(tok))
    return taken, _top(logits[prefix_len - 1 + len(taken)])


def _walk_tree(predict, node_tokens, parents):
    # predict(node) -> target logits after `node` (-1: after the prefix)
    path, at = [], -1
    while True:
        want = _top(predict(at))
        step = None
        for t, par in enumerate(parents):  # children in index order
            if par == at and int(node_tokens[t]) == want:
                step = t
                break
        if step is None:
            return path, want
        path.append(step)
        at = step


def accept_tree_greedy(logits, prefix_len: int, node_tokens, parents):
    """``src/pe/decode/verify.py:35-57``: follow the target's argmax down the tree;
    returns the accepted node indices and the bonus token."""
    return _walk_tree(lambda node: logits[prefix_len - 1 if node < 0 else prefix_len + node],
                      node_tokens, parents)


def accept_chain_cached(root_logit, node_logits, draft_tokens):
    """``src/pe/decode/verify.py:60-72``: as the chain rule, with the prediction
    after the last confirmed token and after each draft given separately."""
    def after(m):  # logits predicting draft m (m = 0: after the confirmed prefix)
        return root_logit if m == 0 else node_logits[m - 1]

    taken = []
    for m, tok in enumerate(draft_tokens):
        if int(tok) != _top(after(m)):
            break
        taken.append(int(tok))
    return taken, _top(after(len(taken)))


def accept_tree_cached(root_logit, node_logits, node_tokens, parents):
    """``src/pe/decode/verify.py:104-125``: the tree rule over cached predictions."""
    return _walk_tree(lambda node: root_logit if node < 0 else node_logits[node],
                      node_tokens, parents)


def accept_chain_sampling(target_dists, draft_tokens, q_dists, generator=None):
    """``src/pe/decode/verify.py:75-101``: per draft one uniform draw u; accept when
    u < min(1, p/q), else draw the bonus from relu(p - q) normalised; all accepted:
    draw the bonus from the trailing target distribution.  The same torch RNG calls
    in the same order, so a seeded generator reproduces the reference."""
    taken = []
    dev = target_dists.device
    for i, tok in enumerate(draft_tokens):
        ratio = torch.clamp(target_dists[i, tok] / q_dists[i, tok], max=1.0)
        u = torch.rand((), generator=generator, device=dev)
        if not bool(u < ratio):
            resid = (target_dists[i] - q_dists[i]).clamp(min=0)
            resid = resid / resid.sum()
            return taken, int(torch.multinomial(resid, 1, generator=generator))
        taken.append(int(tok))
    last = target_dists[len(draft_tokens)]
    return taken, int(torch.multinomial(last, 1, generator=generator))
