"""Parallel multi-token (MTP) slot layout: attend rule, positions and labels.

A length-``n`` sequence is expanded into ``n * K`` prediction slots.  Slot
``(i, d)`` (anchor ``i``, depth ``d``) predicts token ``i + 1 + d`` and sits at
rotary position ``i + d``.  The attend rule for a query slot ``(i, d)`` over a key
slot ``(j, e)`` is (reference ``src/pe/masks.py:43-61``):

* real key (``e == 0``): allowed iff ``j <= i``;
* prediction key (``e >= 1``): allowed iff ``j == i`` and ``e <= d``.

The functions here keep the reference's API (``masks.py:29-110``) for callers that
want explicit boolean masks.  The training step itself never builds a dense mask:
the attention kernels re-derive the rule from ``(anchor, depth)`` per slot.
"""

from __future__ import annotations

import torch

NEG_INF_FILL = "min"


def to_additive_bias(allow: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Boolean attend mask -> additive bias ``(1, 1, S, S)``: 0 where allowed,
    ``finfo(dtype).min`` elsewhere (reference ``masks.py:29-33``)."""
    fill = torch.finfo(dtype).min
    bias = torch.where(
        allow,
        torch.zeros((), dtype=dtype, device=allow.device),
        torch.full((), fill, dtype=dtype, device=allow.device),
    )
    return bias[None, None]


def mtp_slot_anchor_depth(num_anchors: int, k: int, device="cpu"):
    """Anchor-major slot coordinates: slot ``i * k + d`` is ``(i, d)``
    (reference ``masks.py:36-40``)."""
    slot = torch.arange(num_anchors * k, device=device)
    return slot // k, slot % k


def allow_from_slots(
    anchor_q: torch.Tensor,
    depth_q: torch.Tensor,
    anchor_k: torch.Tensor | None = None,
    depth_k: torch.Tensor | None = None,
) -> torch.Tensor:
    """Boolean ``[Q, Kv]`` attend mask for arbitrary query/key slot sets
    (reference ``masks.py:43-61``)."""
    if anchor_k is None:
        anchor_k, depth_k = anchor_q, depth_q
    i = anchor_q.unsqueeze(1)
    d = depth_q.unsqueeze(1)
    j = anchor_k.unsqueeze(0)
    e = depth_k.unsqueeze(0)
    causal_real = (e == 0) & (j <= i)
    same_chain = (e > 0) & (j == i) & (e <= d)
    return causal_real | same_chain


def mtp_allow_mask(num_anchors: int, k: int, device="cpu") -> torch.Tensor:
    """Boolean ``(nK, nK)`` mask for the full anchor-major layout (``masks.py:64-67``)."""
    a, d = mtp_slot_anchor_depth(num_anchors, k, device=device)
    return allow_from_slots(a, d)


def mtp_position_ids(num_anchors: int, k: int, device="cpu") -> torch.Tensor:
    """Rotary position ``i + d`` per anchor-major slot (``masks.py:70-73``)."""
    a, d = mtp_slot_anchor_depth(num_anchors, k, device=device)
    return a + d


def mtp_labels(input_ids: torch.Tensor, k: int) -> torch.Tensor:
    """Label ``input_ids[i + 1 + d]`` per anchor-major slot, ``-100`` when the target
    runs past the sequence (``masks.py:76-87``)."""
    n = input_ids.shape[0]
    a, d = mtp_slot_anchor_depth(n, k, device=input_ids.device)
    tgt = a + 1 + d
    inside = tgt < n
    out = torch.full_like(tgt, -100)
    out[inside] = input_ids[tgt[inside]]
    return out


class AmortizedMtpMask:
    """Build the anchor-major mask once at ``max_anchors`` and hand out top-left
    views per length (``masks.py:90-110``)."""

    def __init__(self, max_anchors: int, k: int, device="cpu"):
        self.max_anchors = max_anchors
        self.k = k
        self._allow = mtp_allow_mask(max_anchors, k, device=device)

    def allow(self, num_anchors: int) -> torch.Tensor:
        if num_anchors > self.max_anchors:
            raise ValueError(f"{num_anchors} anchors exceeds max {self.max_anchors}")
        s = num_anchors * self.k
        return self._allow[:s, :s]

    def bias(self, num_anchors: int, dtype: torch.dtype) -> torch.Tensor:
        return to_additive_bias(self.allow(num_anchors), dtype)


# --------------------------------------------------------------------------
# Verification trees: a drafted token tree appended to a prefix, each node
# given by the index of its parent (-1: hangs off the prefix), parents before
# children (reference masks.py:118-156).  These build the target's attend mask
# and positions for verifying a tree from ``decode.propose_tree``.
# --------------------------------------------------------------------------


def _check_tree(parents) -> list[int]:
    parents = [int(p) for p in parents]
    for t, p in enumerate(parents):
        if not -1 <= p < t:
            raise ValueError(
                f"tree node {t} has parent {p}: parents must be -1 or an earlier node"
            )
    return parents


def tree_depths(parents) -> list[int]:
    """Distance of each node from the prefix: 0 for a node whose parent is -1
    (reference ``masks.py:118-124``)."""
    depths: list[int] = []
    for p in _check_tree(parents):
        depths.append(0 if p < 0 else depths[p] + 1)
    return depths


def tree_allow_mask(parents, prefix_len: int, device="cpu") -> torch.Tensor:
    """Boolean ``(P + T, P + T)`` attend mask over ``[prefix | tree nodes]``
    (reference ``masks.py:127-147``): causal inside the prefix, every node sees
    the whole prefix, and among the nodes exactly its ancestor chain, itself
    included.  Nothing in the prefix sees a node."""
    parents = _check_tree(parents)
    t = len(parents)
    # ancestor sets row by row: a node's row is its parent's row plus itself
    anc = torch.zeros(t, t, dtype=torch.bool)
    for node, p in enumerate(parents):
        if p >= 0:
            anc[node, :p + 1] = anc[p, :p + 1]
        anc[node, node] = True
    n = prefix_len + t
    allow = torch.zeros(n, n, dtype=torch.bool)
    allow[:prefix_len, :prefix_len] = torch.ones(prefix_len, prefix_len, dtype=torch.bool).tril()
    allow[prefix_len:, :prefix_len] = True
    allow[prefix_len:, prefix_len:] = anc
    return allow.to(device)


def tree_position_ids(parents, prefix_len: int, device="cpu") -> torch.Tensor:
    """Rotary position per token (reference ``masks.py:150-156``): the prefix at
    ``0 .. P-1``, a node at ``P + depth`` (siblings share a position)."""
    depths = torch.tensor(tree_depths(parents), dtype=torch.long)
    pos = torch.cat([torch.arange(prefix_len, dtype=torch.long), prefix_len + depths])
    return pos.to(device)
