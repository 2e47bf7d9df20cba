"""Fused forward/backward of one drafter training sequence (the hot path).

:func:`parallel_eagle_b200.partition.mtp_backward` hands each sequence to
:class:`StepEngine`, which runs the reference's per-segment computation
(``src/pe/partition.py:91-116``) as an explicit kernel sequence instead of an
autograd graph:

forward  feat RMSNorm -> feat_proj -> [emb | feat] -> in_proj (real slots);
         in_proj([mask_emb; h_shared]) broadcast to the prediction slots;
         per layer: RMSNorm -> fused q/k/v GEMM -> RoPE -> masked flash
         attention (mask re-derived from (a0, a1, K)) -> o_proj + residual ->
         RMSNorm -> fused gate/up GEMM -> SwiGLU -> down_proj + residual;
         frozen final RMSNorm; loss rows gathered; fused LM head + CE.
backward the exact reverse, with weight gradients accumulated in place into a
         flat gradient buffer whose slices are the parameters' ``.grad``.

Parameters live in one flat buffer (:class:`FlatParams`) so q/k/v and gate/up
are single GEMM operands, the data-parallel all-reduce is one contiguous
buffer, and the optimizer is one kernel.  Nothing is materialised at
O(slots^2) and the full-vocabulary logits never exist.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from . import ops

_ALIGN = 128  # elements; keeps every parameter group 256-byte aligned

# parameters that must directly follow their predecessor (fused GEMM operands)
_FOLLOWERS = ("attn.k_proj.weight", "attn.v_proj.weight", "mlp.up_proj.weight", "h_shared")


class FlatParams:
    """All trainable parameters as views of one contiguous buffer, and their
    gradients as views of a second one."""

    def __init__(self, module: torch.nn.Module):
        self.module = module
        self.build()

    def build(self) -> None:
        named = [(n, p) for n, p in self.module.named_parameters() if p.requires_grad]
        self.names = [n for n, _ in named]
        self.params = [p for _, p in named]
        dev, dt = self.params[0].device, self.params[0].dtype
        off = 0
        self.offsets: dict[str, tuple[int, int]] = {}
        for n, p in named:
            if not n.endswith(_FOLLOWERS):
                off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
            self.offsets[n] = (off, p.numel())
            off += p.numel()
        self.numel = (off + _ALIGN - 1) // _ALIGN * _ALIGN
        self.flat = torch.zeros(self.numel, dtype=dt, device=dev)
        self.grad = torch.zeros(self.numel, dtype=dt, device=dev)
        with torch.no_grad():
            for n, p in named:
                o, k = self.offsets[n]
                self.flat[o : o + k].copy_(p.detach().reshape(-1))
                old_grad = p.grad
                p.data = self.flat[o : o + k].view(p.shape)
                if old_grad is not None:
                    self.grad[o : o + k].copy_(old_grad.reshape(-1))
                    p.grad = self.grad[o : o + k].view(p.shape)
        self.dtype, self.device = dt, dev

    def valid(self) -> bool:
        named = [(n, p) for n, p in self.module.named_parameters() if p.requires_grad]
        if [n for n, _ in named] != self.names:
            return False
        esz = self.flat.element_size()
        base = self.flat.data_ptr()
        for n, p in named:
            if p.dtype != self.dtype or p.device != self.device:
                return False
            if p.data_ptr() != base + self.offsets[n][0] * esz:
                return False
        return True

    def view(self, name: str, shape=None, grad: bool = False) -> torch.Tensor:
        o, k = self.offsets[name]
        buf = self.grad if grad else self.flat
        t = buf[o : o + k]
        return t.view(shape) if shape is not None else t

    def span(self, first: str, last: str, cols: int, grad: bool = False) -> torch.Tensor:
        """Rows of the consecutive parameters ``first..last`` as one ``[rows, cols]`` matrix."""
        o0, _ = self.offsets[first]
        o1, k1 = self.offsets[last]
        buf = self.grad if grad else self.flat
        return buf[o0 : o1 + k1].view(-1, cols)

    def attach_grads(self) -> list[str]:
        """Make every ``p.grad`` a view of the flat gradient buffer, keeping the
        values already accumulated (``None`` grads start from zero).  Returns the
        names whose grad was ``None``."""
        fresh = []
        for n, p in zip(self.names, self.params):
            o, k = self.offsets[n]
            region = self.grad[o : o + k]
            g = p.grad
            if g is None:
                region.zero_()
                fresh.append(n)
            elif g.data_ptr() != region.data_ptr():
                region.copy_(g.reshape(-1))
            else:
                continue
            p.grad = region.view(p.shape)
        return fresh

    def detach_grads(self, names) -> None:
        """Return the listed parameters' grads to ``None`` (autograd leaves a
        parameter outside the graph at ``None``; the step mirrors that)."""
        for n, p in zip(self.names, self.params):
            if n in names:
                p.grad = None


@dataclass
class _SegmentPlan:
    a0: int
    a1: int
    q: int
    pos: torch.Tensor  # int64 [Q] rotary position per slot
    loss_idx: torch.Tensor  # int64 [R] slots carrying a loss
    tgt: torch.Tensor  # int64 [R] target position of each loss slot
    rows: int


def count_loss_slots(n: int, k: int, prompt_len: int = 0) -> int:
    """Slots with ``prompt_len <= i+1+d < n``: target position t has min(k, t) slots
    (closed form of reference ``partition.py:36-38``)."""
    lo = max(1, prompt_len)
    return sum(min(k, t) for t in range(lo, n))


def segment_bounds(n: int, num_segments: int) -> list[tuple[int, int]]:
    """Reference ``partition.py:25-28`` (Python ``round``: half to even)."""
    s = max(1, min(num_segments, n))
    edges = [round(n * i / s) for i in range(s + 1)]
    return [(edges[i], edges[i + 1]) for i in range(s) if edges[i + 1] > edges[i]]


class StepEngine:
    """Runs ``mtp_backward`` for one drafter on its device."""

    def __init__(self, drafter):
        self.d = drafter
        self.flat = FlatParams(drafter)
        self._plans: dict[tuple, _SegmentPlan] = {}
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=self.flat.device)

    # --------------------------------------------------------------- plans --
    def _plan(self, a0: int, a1: int, n: int, prompt_len: int) -> _SegmentPlan:
        key = (a0, a1, n, prompt_len)
        p = self._plans.get(key)
        if p is not None:
            return p
        k = self.d.max_depth
        anchor = np.concatenate([np.arange(a1), np.repeat(np.arange(a0, a1), k - 1)])
        depth = np.concatenate([np.zeros(a1, dtype=np.int64), np.tile(np.arange(1, k), a1 - a0)])
        tgt = anchor + 1 + depth
        keep = (anchor >= a0) & (tgt < n) & (tgt >= prompt_len)
        idx = np.nonzero(keep)[0].astype(np.int64)
        dev = self.flat.device
        p = _SegmentPlan(
            a0, a1, int(anchor.shape[0]),
            torch.from_numpy((anchor + depth).astype(np.int64)).to(dev),
            torch.from_numpy(idx).to(dev),
            torch.from_numpy(tgt[idx].astype(np.int64)).to(dev),
            int(idx.size),
        )
        if len(self._plans) > 256:
            self._plans.clear()
        self._plans[key] = p
        return p

    # ---------------------------------------------------------------- step --
    def run(self, input_ids, features, num_segments=1, loss_scale=1.0, prompt_len=0,
            teacher_labels=None, teacher_hidden=None, sync=True):
        """One sequence; returns the mean loss (a host sync) or ``None`` with
        ``sync=False`` (the sum then stays in ``self.loss_sum``)."""
        d = self.d
        if not self.flat.valid():
            self.flat = FlatParams(d)
        fresh = self.flat.attach_grads()
        dev = self.flat.device
        dt = self.flat.dtype
        input_ids = input_ids.to(dev, non_blocking=True)
        features = features.to(dev, non_blocking=True).to(dt)
        if teacher_labels is not None:
            teacher_labels = teacher_labels.to(dev, non_blocking=True)
        if teacher_hidden is not None:
            teacher_hidden = teacher_hidden.to(dev, non_blocking=True).to(dt)
        n = int(input_ids.shape[0])
        k = d.max_depth
        total = max(1, count_loss_slots(n, k, prompt_len))
        self.loss_sum.zero_()
        scale = loss_scale / total
        ran = mask_slots = False
        for a0, a1 in segment_bounds(n, num_segments):
            # a segment contributes iff some target t in [a0+1, a1+k-1] is in [prompt_len, n)
            if max(a0 + 1, prompt_len) > min(a1 + k - 1, n - 1):
                continue
            plan = self._plan(a0, a1, n, prompt_len)
            if plan.rows == 0:
                continue
            self._segment(plan, input_ids, features, scale, teacher_labels, teacher_hidden)
            ran = True
            mask_slots = mask_slots or plan.q > plan.a1
        if fresh:
            untouched = set(fresh) if not ran else (
                set() if mask_slots else {"mask_emb", "h_shared"} & set(fresh))
            if untouched:
                self.flat.detach_grads(untouched)
        if not sync:
            return None
        return float(self.loss_sum.item()) / total

    # ------------------------------------------------------------- segment --
    def _segment(self, plan: _SegmentPlan, ids, feats, scale, teacher_labels, teacher_hidden):
        d, fp = self.d, self.flat
        dt, dev = fp.dtype, fp.device
        H, I = d.hidden, d.intermediate
        nh, nkv, hd = d.n_heads, d.n_kv_heads, d.head_dim
        qc, kc = nh * hd, nkv * hd
        cqkv = qc + 2 * kc
        k = d.max_depth
        a0, a1, Q = plan.a0, plan.a1, plan.q
        nfl = d.num_feature_layers
        eps = d.eps
        E, Wh, wfinal = d.frozen_heads()
        layout = ops.AttnLayout(L.LAYOUT_PARTITION, a0=a0, a1=a1, k=k)

        def W(name, shape=None):
            return fp.view(name, shape)

        def G(name, shape=None):
            return fp.view(name, shape, grad=True)

        # ---------------- input (reference drafter.py:126-137) ----------------
        x = torch.empty(Q, H, dtype=dt, device=dev)
        u = torch.empty(a1, 2 * H, dtype=dt, device=dev)
        ops.embed_rows(ids[:a1], E, u[:, :H])
        f_in = feats[:a1].reshape(a1 * nfl, H)
        fn, rstd_f = ops.rmsnorm_fwd(f_in, W("feat_norm.weight"), eps)
        w_fp = W("feat_proj.weight", (H, nfl * H))
        w_in = W("in_proj.weight", (H, 2 * H))
        ops.linear(fn.view(a1, nfl * H), w_fp, out=u[:, H:])
        ops.linear(u, w_in, out=x[:a1])
        cat_vec = fp.span("mask_emb", "h_shared", 2 * H)  # [1, 2H], adjacent in the flat buffer
        if Q > a1:
            vec = ops.linear(cat_vec, w_in)  # [1, H]
            ops.fill_rows(vec[0], x[a1:])

        # ---------------- layers (reference nn.py:119-124) ----------------
        saved = []
        for li in range(len(d.layers)):
            p = f"layers.{li}."
            w_qkv = fp.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", H)
            w_o = W(p + "attn.o_proj.weight", (H, qc))
            w_gu = fp.span(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", H)
            w_dn = W(p + "mlp.down_proj.weight", (H, I))
            xn, r1 = ops.rmsnorm_fwd(x, W(p + "input_norm.weight"), eps)
            qkv = ops.linear(xn, w_qkv)
            ops.rope_(qkv, nh + nkv, hd, plan.pos, d.rope_theta)
            q3 = qkv.view(1, Q, cqkv)
            o, lse = ops.attn_fwd(q3[:, :, :qc], q3[:, :, qc : qc + kc], q3[:, :, qc + kc :],
                                  nh, nkv, hd, layout)
            x2 = ops.linear(o.view(Q, qc), w_o, residual=x)
            xn2, r2 = ops.rmsnorm_fwd(x2, W(p + "post_norm.weight"), eps)
            gu = ops.linear(xn2, w_gu)
            act = ops.swiglu_fwd(gu, I)
            x3 = ops.linear(act, w_dn, residual=x2)
            saved.append((x, xn, r1, qkv, o, lse, x2, xn2, r2, gu, act))
            x = x3
        hf, rf = ops.rmsnorm_fwd(x, wfinal, eps)

        # ---------------- loss (reference partition.py:101-115) ----------------
        idx = plan.loss_idx
        hv = ops.gather_rows(hf, idx)
        teacher = None
        labels = None
        if teacher_hidden is not None:
            teacher = ops.gather_rows(teacher_hidden, plan.tgt - 1)
        elif teacher_labels is not None:
            labels = teacher_labels[plan.tgt - 1].to(torch.int64)
        else:
            labels = ids[plan.tgt]
        dh = ops.lmhead_ce(hv, Wh, labels, scale, self.loss_sum, teacher=teacher)
        dhf = torch.zeros(Q, H, dtype=dt, device=dev)
        ops.scatter_rows(dh, idx, dhf)
        dx, _ = ops.rmsnorm_bwd(dhf, x, wfinal, rf, want_dw=False)

        # ---------------- layers backward ----------------
        for li in reversed(range(len(d.layers))):
            p = f"layers.{li}."
            x_in, xn, r1, qkv, o, lse, x2, xn2, r2, gu, act = saved[li]
            w_qkv = fp.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", H)
            w_o = W(p + "attn.o_proj.weight", (H, qc))
            w_gu = fp.span(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", H)
            w_dn = W(p + "mlp.down_proj.weight", (H, I))
            # x3 = x2 + act @ W_down^T
            da = ops.linear_dgrad(dx, w_dn)
            ops.linear_wgrad(dx, act, grad=G(p + "mlp.down_proj.weight", (H, I)), accumulate=True)
            dgu = ops.swiglu_bwd(da, gu, I)
            dxn2 = ops.linear_dgrad(dgu, w_gu)
            ops.linear_wgrad(
                dgu, xn2, accumulate=True,
                grad=fp.span(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", H, grad=True),
            )
            dx2, part = ops.rmsnorm_bwd(dxn2, x2, W(p + "post_norm.weight"), r2, residual=dx)
            ops.colsum_into(part, G(p + "post_norm.weight"), accumulate=True)
            # x2 = x + o @ W_o^T
            do = ops.linear_dgrad(dx2, w_o)
            ops.linear_wgrad(dx2, o.view(Q, qc), grad=G(p + "attn.o_proj.weight", (H, qc)),
                             accumulate=True)
            dqkv = torch.empty(Q, cqkv, dtype=dt, device=dev)
            q3 = qkv.view(1, Q, cqkv)
            d3 = dqkv.view(1, Q, cqkv)
            ops.attn_bwd(q3[:, :, :qc], q3[:, :, qc : qc + kc], q3[:, :, qc + kc :], o,
                         do.view(1, Q, qc), lse, nh, nkv, hd, layout,
                         dq=d3[:, :, :qc], dk=d3[:, :, qc : qc + kc], dv=d3[:, :, qc + kc :])
            ops.rope_(dqkv, nh + nkv, hd, plan.pos, d.rope_theta, inverse=True)
            dxn = ops.linear_dgrad(dqkv, w_qkv)
            ops.linear_wgrad(
                dqkv, xn, accumulate=True,
                grad=fp.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", H, grad=True),
            )
            dx, part = ops.rmsnorm_bwd(dxn, x_in, W(p + "input_norm.weight"), r1, residual=dx2)
            ops.colsum_into(part, G(p + "input_norm.weight"), accumulate=True)

        # ---------------- input backward ----------------
        g_in = G("in_proj.weight", (H, 2 * H))
        if Q > a1:
            # the shared row is broadcast to every prediction slot: its gradient is the
            # column sum, rounded to the parameter dtype like autograd's expand backward
            dvec32 = ops.rowsum_cols(dx[a1:])
            dvec = torch.empty(1, H, dtype=dt, device=dev)
            ops.cast_from_f32(dvec32, dvec)
            ops.linear_wgrad(dvec, cat_vec, grad=g_in, accumulate=True)
            g_cat = fp.span("mask_emb", "h_shared", 2 * H, grad=True)
            ops.linear_dgrad(dvec, w_in, out=g_cat, residual=g_cat)
        dreal = dx[:a1]
        dfeat = ops.linear_dgrad(dreal, w_in[:, H:])
        ops.linear_wgrad(dreal, u, grad=g_in, accumulate=True)
        dfn = ops.linear_dgrad(dfeat, w_fp)
        ops.linear_wgrad(dfeat, fn.view(a1, nfl * H), grad=G("feat_proj.weight", (H, nfl * H)),
                         accumulate=True)
        _, part = ops.rmsnorm_bwd(dfn.view(a1 * nfl, H), f_in, W("feat_norm.weight"), rstd_f)
        ops.colsum_into(part, G("feat_norm.weight"), accumulate=True)


def engine_for(drafter) -> StepEngine:
    eng = getattr(drafter, "_engine", None)
    if eng is None or eng.d is not drafter:
        eng = StepEngine(drafter)
        drafter._engine = eng
    return eng
