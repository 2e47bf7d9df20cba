"""Fused forward/backward of one drafter training sequence (the hot path).

:func:`parallel_eagle_b200.partition.mtp_backward` hands each sequence to
:class:`StepEngine`, which runs the reference's per-segment computation
(``src/pe/partition.py:91-116``) as an explicit kernel sequence instead of an
autograd graph:

forward  feat RMSNorm -> feat_proj -> [emb | feat] -> in_proj (real slots);
         in_proj([mask_emb; h_shared]) broadcast to the prediction slots;
         per layer: RMSNorm -> fused q/k/v GEMM with RoPE in its epilogue ->
         masked flash attention (mask re-derived from (a0, a1, K)) -> o_proj + residual ->
         RMSNorm -> fused gate/up GEMM with silu * mul in its epilogue ->
         down_proj + residual;
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
class _PassPlan:
    """Segments executed together: their slot rows stacked segment after segment
    (each segment's rows stay contiguous, ``[real 0..a1) | MTP anchor-major]``)."""

    segs: list  # (a0, a1, Q, row offset) per segment
    q: int  # stacked rows
    pos: torch.Tensor  # int64 [q] rotary position per row
    loss_idx: torch.Tensor  # int64 [R] stacked rows carrying a loss
    tgt: torch.Tensor  # int64 [R] target position of each loss row
    rows: int  # R
    real_tok: torch.Tensor  # int64 [Rt] token index of each stacked real row
    real_row: torch.Tensor  # int64 [Rt] its row in the stack
    nreal: int  # Rt
    has_pred: bool  # some segment has MTP slots
    rope_cs: torch.Tensor | None = None  # [q, head_dim] cos | sin table (fused rotations)


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
        self._plans: dict[tuple, _PassPlan] = {}
        # device bytes of activations one pass of stacked segments may hold
        self.pass_bytes = 24 << 30
        # called (no arguments) once the decoder layers' weight gradients of the current
        # sequence are final -- after its last pass's layer backward, before the input
        # projections' backward -- so a data-parallel caller can start reducing them
        self.after_layers = None
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=self.flat.device)
        # kernel choices (results are identical either way; chosen by step-level timing):
        # RoPE in the q|k|v GEMM epilogue and the attention backward (bf16, head_dim
        # 128); SwiGLU in the gate|up GEMM epilogue and its backward in the epilogue of
        # the down projection's input-gradient GEMM; the fused LM head's tuning bits
        self.fuse_rope = True
        self.fuse_swiglu = True
        self.fuse_swiglu_bwd = False
        self.lmhead_algo = 0
        # per-call-site GEMM tuning bits (pe_gemm's algo: tile width, tile order), keyed
        # "dn_fwd", "gu_dgrad", "gu_wgrad", "dn_dgrad", "dn_wgrad", "o_fwd", "o_dgrad",
        # "o_wgrad", "qkv_dgrad", "qkv_wgrad"; empty = automatic everywhere
        self.gemm_algo = {}

    # --------------------------------------------------------------- plans --
    def _segment_arrays(self, a0: int, a1: int, n: int, prompt_len: int):
        """Slots of one segment (reference ``partition.py:41-55``, ``:101-104``):
        rotary positions, loss-slot indices and their target positions."""
        return self._segment_arrays_static(a0, a1, n, self.d.max_depth, prompt_len)

    @staticmethod
    def _segment_arrays_static(a0: int, a1: int, n: int, k: int, prompt_len: int):
        anchor = np.concatenate([np.arange(a1), np.repeat(np.arange(a0, a1), k - 1)])
        depth = np.concatenate([np.zeros(a1, dtype=np.int64), np.tile(np.arange(1, k), a1 - a0)])
        tgt = anchor + 1 + depth
        keep = (anchor >= a0) & (tgt < n) & (tgt >= prompt_len)
        idx = np.nonzero(keep)[0].astype(np.int64)
        return (anchor + depth).astype(np.int64), idx, tgt[idx].astype(np.int64)

    def _pass_plan(self, bounds: tuple, n: int, prompt_len: int) -> _PassPlan:
        key = (bounds, n, prompt_len)
        p = self._plans.get(key)
        if p is not None:
            return p
        segs, pos, idx, tgt, rtok, rrow = [], [], [], [], [], []
        off = 0
        for a0, a1 in bounds:
            sp, si, st = self._segment_arrays(a0, a1, n, prompt_len)
            q = int(sp.shape[0])
            segs.append((a0, a1, q, off))
            pos.append(sp)
            idx.append(si + off)
            tgt.append(st)
            rtok.append(np.arange(a1, dtype=np.int64))
            rrow.append(off + np.arange(a1, dtype=np.int64))
            off += q
        dev = self.flat.device

        def t(parts):
            return torch.from_numpy(np.concatenate(parts)).to(dev)

        loss_idx = t(idx)
        real_tok = t(rtok)
        p = _PassPlan(segs, off, t(pos), loss_idx, t(tgt), int(loss_idx.numel()), real_tok,
                      t(rrow), int(real_tok.numel()), any(q > a1 for _, a1, q, _ in segs))
        if len(self._plans) > 256:
            self._plans.clear()
        self._plans[key] = p
        return p

    def _row_bytes(self) -> int:
        """Device bytes one stacked slot row holds during a pass: the saved layer
        activations plus the widest transient gradients."""
        d, esz = self.d, self.flat.grad.element_size()
        H, I = d.hidden, d.intermediate
        cqkv = (d.n_heads + 2 * d.n_kv_heads) * d.head_dim
        per_layer = esz * (4 * H + cqkv + d.n_heads * d.head_dim + 3 * I) + 4 * (2 + d.n_heads)
        return per_layer * len(d.layers) + esz * (3 * I + cqkv + 4 * H) + 8 * H

    def _passes(self, bounds: list) -> list:
        """Consecutive segments grouped so each pass stays within ``pass_bytes``
        (a single segment larger than the budget runs alone)."""
        k = self.d.max_depth
        limit = max(1, self.pass_bytes // self._row_bytes())
        groups, cur, rows = [], [], 0
        for a0, a1 in bounds:
            q = a1 + (a1 - a0) * (k - 1)
            if cur and rows + q > limit:
                groups.append(cur)
                cur, rows = [], 0
            cur.append((a0, a1))
            rows += q
        if cur:
            groups.append(cur)
        return groups

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
        # features keep their cached dtype (fp16 shards) until the feature-norm kernel
        # reads and rounds them (reference drafter.py:129 casts first)
        features = features.to(dev, non_blocking=True)
        if not ops.feature_norm_ok(features, d.hidden, d.num_feature_layers):
            features = features.to(dt)
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
        live = []
        for a0, a1 in segment_bounds(n, num_segments):
            # a segment contributes iff some target t in [a0+1, a1+k-1] is in [prompt_len, n)
            if max(a0 + 1, prompt_len) > min(a1 + k - 1, n - 1):
                continue
            live.append((a0, a1))
        groups = self._passes(live)
        for gi, group in enumerate(groups):
            plan = self._pass_plan(tuple(group), n, prompt_len)
            self._pass(plan, input_ids, features, scale, teacher_labels, teacher_hidden,
                       last=gi == len(groups) - 1)
            ran = True
            mask_slots = mask_slots or plan.has_pred
        if fresh:
            untouched = set(fresh) if not ran else (
                set() if mask_slots else {"mask_emb", "h_shared"} & set(fresh))
            if untouched:
                self.flat.detach_grads(untouched)
        if not sync:
            return None
        return float(self.loss_sum.item()) / total

    # ---------------------------------------------------------------- pass --
    def layer_grad_region(self) -> tuple[int, int]:
        """``[start, end)`` of the flat gradient buffer holding the decoder layers'
        parameters: a contiguous suffix (``named_parameters`` lists the drafter's own
        parameters and the input projections before ``layers``)."""
        spans = [self.flat.offsets[n] for n in self.flat.names if n.startswith("layers.")]
        start = min(o for o, _ in spans)
        end = max(o + k for o, k in spans)
        if any(o >= start for n, (o, _) in self.flat.offsets.items() if not n.startswith("layers.")):
            raise L.PeError("layer parameters are not a contiguous suffix of the flat buffer")
        return start, self.flat.numel  # the alignment tail after `end` is zero padding

    def _pass(self, plan: _PassPlan, ids, feats, scale, teacher_labels, teacher_hidden,
              last=True):
        """Forward and backward of the stacked segments of one pass.  Every GEMM,
        norm and element-wise op runs once over all stacked rows; attention runs
        once too, each segment on its row range with that segment's mask."""
        d, fp = self.d, self.flat
        dt, dev = fp.dtype, fp.device
        H, I = d.hidden, d.intermediate
        ga = self.gemm_algo.get
        nh, nkv, hd = d.n_heads, d.n_kv_heads, d.head_dim
        qc, kc = nh * hd, nkv * hd
        cqkv = qc + 2 * kc
        k = d.max_depth
        Q, Rt = plan.q, plan.nreal
        nfl = d.num_feature_layers
        eps = d.eps
        E, Wh, wfinal = d.frozen_heads()
        single = len(plan.segs) == 1
        # bf16 with head_dim 128: RoPE rides in the q|k|v GEMM epilogue and its transpose
        # in the attention backward's dQ store / dK cast, reading a per-plan cos / sin
        # table (the slot positions are fixed per plan)
        fuse_rope = self.fuse_rope and dt == torch.bfloat16 and hd == 128
        if fuse_rope and plan.rope_cs is None:
            plan.rope_cs = ops.rope_table(plan.pos, hd, d.rope_theta, dt)
        rope_cs = plan.rope_cs if fuse_rope else None
        # every segment's attention runs in one call over the stacked rows
        bounds = [(a0, a1) for a0, a1, _, _ in plan.segs]

        def W(name, shape=None):
            return fp.view(name, shape)

        def G(name, shape=None):
            return fp.view(name, shape, grad=True)

        # ---------------- input (reference drafter.py:126-137) ----------------
        # real rows of every segment: [embedding | feat_proj(RMSNorm(features))] -> in_proj
        x = torch.empty(Q, H, dtype=dt, device=dev)
        u = torch.empty(Rt, 2 * H, dtype=dt, device=dev)
        fused_fnorm = ops.feature_norm_ok(feats, H, nfl)
        src_tok = None if single else plan.real_tok
        if single:
            a1 = plan.segs[0][1]
            ops.embed_rows(ids[:a1], E, u[:, :H])
        else:
            ops.embed_rows(ids.index_select(0, plan.real_tok), E, u[:, :H])
        if fused_fnorm:
            # every stacked segment's real prefix rows normalised straight from the shard
            fn, rstd_f = ops.feature_norm_fwd(feats, W("feat_norm.weight"), nfl, H, dt, eps,
                                              src_tok=src_tok, tokens=Rt)
            f_in = None
        else:
            f_in = (feats[:plan.segs[0][1]].reshape(Rt * nfl, H) if single
                    else ops.gather_rows(feats, plan.real_tok).view(Rt * nfl, H))
            fn, rstd_f = ops.rmsnorm_fwd(f_in, W("feat_norm.weight"), eps)
        w_fp = W("feat_proj.weight", (H, nfl * H))
        w_in = W("in_proj.weight", (H, 2 * H))
        ops.linear(fn.view(Rt, nfl * H), w_fp, out=u[:, H:])
        if single:
            ops.linear(u, w_in, out=x[:Rt])
        else:
            ops.scatter_rows(ops.linear(u, w_in), plan.real_row, x)
        cat_vec = fp.span("mask_emb", "h_shared", 2 * H)  # [1, 2H], adjacent in the flat buffer
        if plan.has_pred:
            vec = ops.linear(cat_vec, w_in)  # [1, H]
            for _, a1, q, off in plan.segs:
                if q > a1:
                    ops.fill_rows(vec[0], x[off + a1 : off + q])

        # ---------------- layers (reference nn.py:119-124) ----------------
        saved = []
        for li in range(len(d.layers)):
            p = f"layers.{li}."
            w_qkv = fp.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", H)
            w_o = W(p + "attn.o_proj.weight", (H, qc))
            w_gu = fp.span(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", H)
            w_dn = W(p + "mlp.down_proj.weight", (H, I))
            xn, r1 = ops.rmsnorm_fwd(x, W(p + "input_norm.weight"), eps)
            if fuse_rope:
                qkv = ops.linear_rope(xn, w_qkv, rope_cs, qc + kc, hd)
            else:
                qkv = ops.linear(xn, w_qkv)
                ops.rope_(qkv, nh + nkv, hd, plan.pos, d.rope_theta)
            o, lse = ops.attn_fwd_segments(qkv[:, :qc], qkv[:, qc : qc + kc], qkv[:, qc + kc :],
                                           nh, nkv, hd, bounds, k)
            x2 = ops.linear(o, w_o, residual=x, algo=ga("o_fwd", 0))
            xn2, r2 = ops.rmsnorm_fwd(x2, W(p + "post_norm.weight"), eps)
            if self.fuse_swiglu:
                # the activation in the gate|up GEMM epilogue (gate|up kept for backward)
                gu, act = ops.linear_swiglu(xn2, w_gu, I)
            else:
                gu = ops.linear(xn2, w_gu)
                act = ops.swiglu_fwd(gu, I)
            x3 = ops.linear(act, w_dn, residual=x2, algo=ga("dn_fwd", 0))
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
        dh = ops.lmhead_ce(hv, Wh, labels, scale, self.loss_sum, teacher=teacher,
                           algo=self.lmhead_algo)
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
            if self.fuse_swiglu_bwd:
                dgu = ops.linear_swiglu_bwd(dx, w_dn, gu, I)
            else:
                dgu = ops.swiglu_bwd(ops.linear_dgrad(dx, w_dn, algo=ga("dn_dgrad", 0)), gu, I)
            ops.linear_wgrad(dx, act, grad=G(p + "mlp.down_proj.weight", (H, I)), accumulate=True,
                             algo=ga("dn_wgrad", 0))
            dxn2 = ops.linear_dgrad(dgu, w_gu, algo=ga("gu_dgrad", 0))
            ops.linear_wgrad(
                dgu, xn2, accumulate=True,
                grad=fp.span(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", H, grad=True),
                algo=ga("gu_wgrad", 0),
            )
            dx2, part = ops.rmsnorm_bwd(dxn2, x2, W(p + "post_norm.weight"), r2, residual=dx)
            ops.colsum_into(part, G(p + "post_norm.weight"), accumulate=True)
            # x2 = x + o @ W_o^T
            do = ops.linear_dgrad(dx2, w_o, algo=ga("o_dgrad", 0))
            ops.linear_wgrad(dx2, o, grad=G(p + "attn.o_proj.weight", (H, qc)), accumulate=True,
                             algo=ga("o_wgrad", 0))
            dqkv = torch.empty(Q, cqkv, dtype=dt, device=dev)
            ops.attn_bwd_segments(qkv[:, :qc], qkv[:, qc : qc + kc], qkv[:, qc + kc :], o, do, lse,
                                  nh, nkv, hd, bounds, k, dq=dqkv[:, :qc],
                                  dk=dqkv[:, qc : qc + kc], dv=dqkv[:, qc + kc :],
                                  rope_cs=rope_cs)
            if not fuse_rope:
                ops.rope_(dqkv, nh + nkv, hd, plan.pos, d.rope_theta, inverse=True)
            dxn = ops.linear_dgrad(dqkv, w_qkv, algo=ga("qkv_dgrad", 0))
            ops.linear_wgrad(
                dqkv, xn, accumulate=True,
                grad=fp.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", H, grad=True),
                algo=ga("qkv_wgrad", 0),
            )
            dx, part = ops.rmsnorm_bwd(dxn, x_in, W(p + "input_norm.weight"), r1, residual=dx2)
            ops.colsum_into(part, G(p + "input_norm.weight"), accumulate=True)

        if last and self.after_layers is not None:
            self.after_layers()

        # ---------------- input backward ----------------
        g_in = G("in_proj.weight", (H, 2 * H))
        if plan.has_pred:
            # the shared row is broadcast to every prediction slot: its gradient is the
            # column sum over those slots, rounded to the parameter dtype like
            # autograd's expand backward
            dvec32 = ops.rowsum_cols_ranges(
                dx, [(off + a1, off + q) for _, a1, q, off in plan.segs if q > a1])
            dvec = torch.empty(1, H, dtype=dt, device=dev)
            ops.cast_from_f32(dvec32, dvec)
            ops.linear_wgrad(dvec, cat_vec, grad=g_in, accumulate=True)
            g_cat = fp.span("mask_emb", "h_shared", 2 * H, grad=True)
            ops.linear_dgrad(dvec, w_in, out=g_cat, residual=g_cat)
        dreal = dx[:Rt] if single else ops.gather_rows(dx, plan.real_row)
        dfeat = ops.linear_dgrad(dreal, w_in[:, H:])
        ops.linear_wgrad(dreal, u, grad=g_in, accumulate=True)
        dfn = ops.linear_dgrad(dfeat, w_fp)
        ops.linear_wgrad(dfeat, fn.view(Rt, nfl * H), grad=G("feat_proj.weight", (H, nfl * H)),
                         accumulate=True)
        if fused_fnorm:
            part = ops.feature_norm_dw(dfn.view(Rt * nfl, H), feats, rstd_f, nfl, H,
                                       src_tok=src_tok)
        else:
            _, part = ops.rmsnorm_bwd(dfn.view(Rt * nfl, H), f_in, W("feat_norm.weight"), rstd_f)
        ops.colsum_into(part, G("feat_norm.weight"), accumulate=True)


def engine_for(drafter) -> StepEngine:
    eng = getattr(drafter, "_engine", None)
    if eng is None or eng.d is not drafter:
        eng = StepEngine(drafter)
        drafter._engine = eng
    return eng
