"""Functional CPU restatement of the reference drafter training step.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function cites the
reference lines it restates; paths are relative to the reference project root.

Rounding points follow the reference in low-precision mode: RMSNorm and softmax
run in fp32 and cast back, cos/sin are cast to the activation dtype before the
rotation, logits are produced in the parameter dtype and then upcast, and
cross-entropy runs in fp32.

The soft-target distillation loss (``teacher_hidden``) does not exist in the
reference; it is this oracle's own definition: teacher probabilities for the slot
that predicts position ``t`` come from teacher row ``t - 1`` (the same indexing
the reference uses for hard ``teacher_labels``, ``src/pe/partition.py:105-106``),
``p = softmax(float(h_t @ W_head^T))`` and the slot loss is
``-sum_v p_v * log_softmax(z)_v``.  Its parity is therefore unpinned by any
reference test.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class OracleDims:
    hidden: int
    n_heads: int
    n_kv_heads: int
    intermediate: int
    vocab: int
    num_layers: int
    max_depth: int
    num_feature_layers: int = 3
    rope_theta: float = 10000.0
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads

    @property
    def feature_dim(self) -> int:
        return self.hidden * self.num_feature_layers


def param_names(num_layers: int) -> list[str]:
    """State-dict keys of the drafter in registration order
    (reference ``src/pe/drafter.py:66-76``, ``src/pe/nn.py:114-117``, ``:66-69``, ``:95-97``)."""
    names = ["mask_emb", "h_shared", "feat_norm.weight", "feat_proj.weight", "in_proj.weight"]
    for i in range(num_layers):
        p = f"layers.{i}."
        names += [
            p + "input_norm.weight",
            p + "attn.q_proj.weight",
            p + "attn.k_proj.weight",
            p + "attn.v_proj.weight",
            p + "attn.o_proj.weight",
            p + "post_norm.weight",
            p + "mlp.gate_proj.weight",
            p + "mlp.up_proj.weight",
            p + "mlp.down_proj.weight",
        ]
    return names


def init_params(dims: OracleDims, seed: int, dtype=torch.float32) -> dict[str, torch.Tensor]:
    """Parameters drawn in the reference's construction order from the global RNG
    after ``torch.manual_seed(seed)`` (``src/pe/drafter.py:66-76``): Linear layers use
    torch's default init, norms start at one, ``mask_emb``/``h_shared`` are
    re-drawn N(0, 0.02^2) after the layer stack is built."""
    torch.manual_seed(seed)
    H, I = dims.hidden, dims.intermediate
    hd = dims.head_dim

    def linear(out_f, in_f):
        return torch.nn.Linear(in_f, out_f, bias=False).weight.detach().clone()

    p: dict[str, torch.Tensor] = {}
    p["feat_norm.weight"] = torch.ones(H)
    p["feat_proj.weight"] = linear(H, dims.feature_dim)
    p["in_proj.weight"] = linear(H, 2 * H)
    p["mask_emb"] = torch.zeros(H)
    p["h_shared"] = torch.zeros(H)
    for i in range(dims.num_layers):
        q = f"layers.{i}."
        p[q + "input_norm.weight"] = torch.ones(H)
        p[q + "attn.q_proj.weight"] = linear(dims.n_heads * hd, H)
        p[q + "attn.k_proj.weight"] = linear(dims.n_kv_heads * hd, H)
        p[q + "attn.v_proj.weight"] = linear(dims.n_kv_heads * hd, H)
        p[q + "attn.o_proj.weight"] = linear(H, dims.n_heads * hd)
        p[q + "post_norm.weight"] = torch.ones(H)
        p[q + "mlp.gate_proj.weight"] = linear(I, H)
        p[q + "mlp.up_proj.weight"] = linear(I, H)
        p[q + "mlp.down_proj.weight"] = linear(H, I)
    p["mask_emb"] = torch.empty(H).normal_(std=0.02)
    p["h_shared"] = torch.empty(H).normal_(std=0.02)
    return {k: p[k].to(dtype) for k in param_names(dims.num_layers)}


# ----------------------------------------------------------------------------- #
# building blocks
# ----------------------------------------------------------------------------- #


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMSNorm cast back to the input dtype (``src/pe/nn.py:22-26``)."""
    out_dtype = x.dtype
    xf = x.float()
    scale = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return ((xf * scale) * w.float()).to(out_dtype)


def rope_tables(pos: torch.Tensor, head_dim: int, theta: float):
    """fp32 ``(cos, sin)`` of shape ``pos.shape + (head_dim,)`` for half-split rotary
    embeddings (``src/pe/nn.py:29-37``)."""
    half = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inv_freq = 1.0 / (theta**half)
    ang = pos.float().unsqueeze(-1) * inv_freq
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x * cos + rotate_half(x) * sin`` with cos/sin in x's dtype
    (``src/pe/nn.py:40-49``); x is ``[heads, S, hd]``, cos/sin ``[S, hd]``."""
    c = cos.to(x.dtype).unsqueeze(0)
    s = sin.to(x.dtype).unsqueeze(0)
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
    return x * c + rot * s


def slot_allow(anchor_q, depth_q, anchor_k=None, depth_k=None) -> torch.Tensor:
    """MTP attend rule (``src/pe/masks.py:43-61``)."""
    if anchor_k is None:
        anchor_k, depth_k = anchor_q, depth_q
    i, d = anchor_q[:, None], depth_q[:, None]
    j, e = anchor_k[None, :], depth_k[None, :]
    return torch.where(e == 0, j <= i, (j == i) & (e <= d))


def additive_bias(allow: torch.Tensor, dtype) -> torch.Tensor:
    """``0`` / ``finfo(dtype).min`` bias (``src/pe/masks.py:29-33``)."""
    b = torch.zeros(allow.shape, dtype=dtype)
    b[~allow] = torch.finfo(dtype).min
    return b


def attention(p, pre: str, x, cos, sin, bias, dims: OracleDims):
    """Grouped-query attention with an additive bias (``src/pe/nn.py:71-89``).
    ``x`` is ``[S, H]`` (batch of one), ``bias`` ``[S, S]``."""
    S = x.shape[0]
    hd = dims.head_dim
    q = F.linear(x, p[pre + "q_proj.weight"]).view(S, dims.n_heads, hd).transpose(0, 1)
    k = F.linear(x, p[pre + "k_proj.weight"]).view(S, dims.n_kv_heads, hd).transpose(0, 1)
    v = F.linear(x, p[pre + "v_proj.weight"]).view(S, dims.n_kv_heads, hd).transpose(0, 1)
    q = _rotate(q, cos, sin)
    k = _rotate(k, cos, sin)
    rep = dims.n_heads // dims.n_kv_heads
    k = k.repeat_interleave(rep, dim=0)
    v = v.repeat_interleave(rep, dim=0)
    scores = torch.matmul(q, k.transpose(-1, -2)) / (hd**0.5)
    scores = scores + bias
    probs = torch.softmax(scores.float(), dim=-1).to(q.dtype)
    out = torch.matmul(probs, v).transpose(0, 1).reshape(S, dims.n_heads * hd)
    return F.linear(out, p[pre + "o_proj.weight"])


def swiglu(p, pre: str, x):
    """``down(silu(gate x) * up x)`` (``src/pe/nn.py:99-100``)."""
    g = F.linear(x, p[pre + "gate_proj.weight"])
    u = F.linear(x, p[pre + "up_proj.weight"])
    return F.linear(F.silu(g) * u, p[pre + "down_proj.weight"])


def drafter_forward(p, heads, x, pos, bias, dims: OracleDims):
    """Layer stack plus the frozen shared final norm (``src/pe/drafter.py:150-161``,
    ``src/pe/nn.py:119-124``).  ``x`` ``[S, H]``, ``pos`` ``[S]``, ``bias`` ``[S, S]``."""
    cos, sin = rope_tables(pos, dims.head_dim, dims.rope_theta)
    for li in range(dims.num_layers):
        pre = f"layers.{li}."
        h = rms_norm(x, p[pre + "input_norm.weight"], dims.eps)
        x = x + attention(p, pre + "attn.", h, cos, sin, bias, dims)
        h = rms_norm(x, p[pre + "post_norm.weight"], dims.eps)
        x = x + swiglu(p, pre + "mlp.", h)
    return rms_norm(x, heads["norm"], dims.eps)


def real_input(p, heads, ids, feats, dims: OracleDims):
    """``in_proj([embed(ids); feat_proj(norm(feats per fused layer))])``
    (``src/pe/drafter.py:126-132``)."""
    dt = p["in_proj.weight"].dtype
    emb = heads["embed"][ids].to(dt)
    f = feats.to(dt).unflatten(-1, (dims.num_feature_layers, dims.hidden))
    f = rms_norm(f, p["feat_norm.weight"], dims.eps).flatten(-2)
    feat = F.linear(f, p["feat_proj.weight"])
    return F.linear(torch.cat([emb, feat], dim=-1), p["in_proj.weight"])


def mask_input(p, m: int):
    """One shared input row for prediction slots, repeated ``m`` times
    (``src/pe/drafter.py:134-137``)."""
    v = F.linear(torch.cat([p["mask_emb"], p["h_shared"]]), p["in_proj.weight"])
    return v.unsqueeze(0).expand(m, -1)


# ----------------------------------------------------------------------------- #
# sequence partitioning (src/pe/partition.py)
# ----------------------------------------------------------------------------- #


def segment_edges(n: int, num_segments: int) -> list[tuple[int, int]]:
    """Non-empty ``[a0, a1)`` anchor ranges with edges ``round(n*s/S)``
    (``src/pe/partition.py:25-28``; Python's round-half-to-even)."""
    s_count = max(1, min(num_segments, n))
    edges = [round(n * s / s_count) for s in range(s_count + 1)]
    return [(edges[i], edges[i + 1]) for i in range(s_count) if edges[i + 1] > edges[i]]


def count_loss_slots(n: int, k: int, prompt_len: int = 0) -> int:
    """Slots ``(i, d)`` with ``prompt_len <= i+1+d < n`` (``src/pe/partition.py:31-38``)."""
    total = 0
    for i in range(n):
        for d in range(k):
            t = i + 1 + d
            if prompt_len <= t < n:
                total += 1
    return total


def segment_slots(a0: int, a1: int, k: int):
    """Anchor/depth per slot: real stream ``0..a1-1`` then anchors ``a0..a1-1`` x
    depths ``1..k-1``, anchor-major (``src/pe/partition.py:41-55``)."""
    anchors = list(range(a1))
    depths = [0] * a1
    for i in range(a0, a1):
        for d in range(1, k):
            anchors.append(i)
            depths.append(d)
    return torch.tensor(anchors, dtype=torch.long), torch.tensor(depths, dtype=torch.long)


def _loss_targets(anchor, depth, a0, n, prompt_len):
    tgt = anchor + 1 + depth
    keep = (anchor >= a0) & (tgt < n) & (tgt >= prompt_len)
    return tgt, keep


def mtp_step(
    params: dict[str, torch.Tensor],
    heads: dict[str, torch.Tensor],
    ids: torch.Tensor,
    feats: torch.Tensor,
    dims: OracleDims,
    num_segments: int = 1,
    loss_scale: float = 1.0,
    prompt_len: int = 0,
    teacher_labels: torch.Tensor | None = None,
    teacher_hidden: torch.Tensor | None = None,
    grads: dict[str, torch.Tensor] | None = None,
):
    """One sequence of the partitioned MTP loss with its backward
    (``src/pe/partition.py:58-118``).

    Returns ``(mean_loss, grads)``; ``grads`` accumulates ``d(loss*scale)/dparam``
    in the parameter dtype like ``.grad`` does (pass the previous dict to
    accumulate across sequences).
    """
    leaf = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
    n = int(ids.shape[0])
    k = dims.max_depth
    total = max(1, count_loss_slots(n, k, prompt_len))
    dt = params["in_proj.weight"].dtype
    head_w = heads["head"]
    loss_sum = 0.0
    for a0, a1 in segment_edges(n, num_segments):
        anchor, depth = segment_slots(a0, a1, k)
        x = real_input(leaf, heads, ids[:a1], feats[:a1], dims)
        if k > 1:
            x = torch.cat([x, mask_input(leaf, anchor.shape[0] - a1)])
        bias = additive_bias(slot_allow(anchor, depth), dt)
        hidden = drafter_forward(leaf, heads, x, anchor + depth, bias, dims)
        tgt, keep = _loss_targets(anchor, depth, a0, n, prompt_len)
        if not bool(keep.any()):
            continue
        logits = F.linear(hidden[keep], head_w).float()
        if teacher_hidden is not None:
            t_logits = F.linear(teacher_hidden[tgt[keep] - 1].to(dt), head_w).float()
            p_t = torch.softmax(t_logits, dim=-1)
            seg = -(p_t * torch.log_softmax(logits, dim=-1)).sum()
        else:
            src = teacher_labels[tgt[keep] - 1] if teacher_labels is not None else ids[tgt[keep]]
            seg = F.cross_entropy(logits, src, reduction="sum")
        (seg * (loss_scale / total)).backward()
        loss_sum += float(seg.detach())
    out = {} if grads is None else grads
    for name, t in leaf.items():
        if t.grad is None:
            continue
        out[name] = t.grad if name not in out else out[name] + t.grad
    return loss_sum / total, out


@torch.no_grad()
def mtp_eval_loss(params, heads, ids, feats, dims: OracleDims) -> float:
    """Full-sequence anchor-major mean loss (``src/pe/partition.py:121-131``,
    ``src/pe/drafter.py:166-190``)."""
    n = int(ids.shape[0])
    k = dims.max_depth
    dt = params["in_proj.weight"].dtype
    real = real_input(params, heads, ids, feats, dims)
    x = torch.empty(n * k, dims.hidden, dtype=dt)
    x[0::k] = real
    if k > 1:
        vec = mask_input(params, 1)[0]
        for d in range(1, k):
            x[d::k] = vec
    slot = torch.arange(n * k)
    anchor, depth = slot // k, slot % k
    bias = additive_bias(slot_allow(anchor, depth), dt)
    hidden = drafter_forward(params, heads, x, anchor + depth, bias, dims)
    tgt = anchor + 1 + depth
    keep = tgt < n
    logits = F.linear(hidden[keep], heads["head"]).float()
    return float(F.cross_entropy(logits, ids[tgt[keep]]))


def attention_flops(n: int, k: int, num_segments: int, head_dim: int, n_heads: int) -> float:
    """Masked-attention fwd+bwd FLOPs counted as 12*hd*Hq per allowed pair."""
    pairs = 0
    for a0, a1 in segment_edges(n, num_segments):
        pairs += a1 * (a1 + 1) // 2
        for i in range(a0, a1):
            pairs += (k - 1) * (i + 1) + k * (k - 1) // 2
    return 12.0 * head_dim * n_heads * pairs
