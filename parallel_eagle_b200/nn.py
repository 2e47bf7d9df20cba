"""Llama-style drafter blocks whose compute runs in libpe_b200.

Module names, parameter names/shapes and forward signatures follow the
reference's ``pe.nn`` (``src/pe/nn.py:16-124``) so state dicts and call sites
carry over; every forward/backward is a custom autograd function over the
library's kernels (RMSNorm, rotary embedding, tensor-core GEMMs, the masked
flash attention, SwiGLU).  Inputs must be CUDA tensors.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib as L
from . import ops


def _flat(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2 = _flat(x).contiguous()
        y, rstd = ops.rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, part = ops.rmsnorm_bwd(_flat(dy).contiguous(), x2, w, rstd,
                                   want_dw=ctx.needs_input_grad[1])
        dw = None
        if part is not None:
            dw = ops.colsum_into(part, torch.empty_like(w), accumulate=False)
        return dx.view(ctx.shape), dw, None


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        x2 = _flat(x).contiguous()
        y = ops.linear(x2, w)
        ctx.save_for_backward(x2, w)
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _flat(dy).contiguous()
        dx = ops.linear_dgrad(dy2, w).view(ctx.shape) if ctx.needs_input_grad[0] else None
        dw = ops.linear_wgrad(dy2, x2) if ctx.needs_input_grad[1] else None
        return dx, dw


class _RopeFn(torch.autograd.Function):
    """Rotary embedding on the first ``heads`` head blocks of each row."""

    @staticmethod
    def forward(ctx, x, pos, heads, head_dim, theta):
        y = _flat(x).contiguous().clone()
        p = pos.reshape(-1).to(torch.int64).contiguous()
        ops.rope_(y, heads, head_dim, p, theta, inverse=False)
        ctx.save_for_backward(p)
        ctx.args = (heads, head_dim, theta, x.shape)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        (p,) = ctx.saved_tensors
        heads, head_dim, theta, shape = ctx.args
        dx = _flat(dy).contiguous().clone()
        ops.rope_(dx, heads, head_dim, p, theta, inverse=True)
        return dx.view(shape), None, None, None, None


class _AttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, layout, n_heads, n_kv_heads, head_dim):
        o, lse = ops.attn_fwd(q, k, v, n_heads, n_kv_heads, head_dim, layout)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.args = (layout, n_heads, n_kv_heads, head_dim)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        layout, nh, nkv, hd = ctx.args
        dq, dk, dv = ops.attn_bwd(q, k, v, o, do.contiguous(), lse, nh, nkv, hd, layout)
        return dq, dk, dv, None, None, None, None


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu, inter):
        g2 = _flat(gu).contiguous()
        a = ops.swiglu_fwd(g2, inter)
        ctx.save_for_backward(g2)
        ctx.args = (inter, gu.shape)
        return a.view(*gu.shape[:-1], inter)

    @staticmethod
    def backward(ctx, da):
        (g2,) = ctx.saved_tensors
        inter, shape = ctx.args
        dgu = ops.swiglu_bwd(_flat(da).contiguous(), g2, inter)
        return dgu.view(shape), None


def rms_norm(x, w, eps):
    L.require_cuda(x)
    return _RMSNormFn.apply(x, w, eps)


def linear(x, w):
    L.require_cuda(x)
    return _LinearFn.apply(x, w)


class RMSNorm(nn.Module):
    """``(x * rsqrt(mean(x^2) + eps)) * w`` in fp32, cast back (reference ``nn.py:16-26``)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)


def build_rope_cache(position_ids: torch.Tensor, head_dim: int, theta: float):
    """``(cos, sin)`` of shape ``(B, S, head_dim)`` (reference ``nn.py:29-37``).

    The returned ``cos`` also carries the position ids and base so the fused
    rotary kernel recomputes the angles itself instead of reading the tables.
    """
    dev = position_ids.device
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=dev).float() / head_dim))
    ang = position_ids.float()[..., None] * inv_freq[None, None, :]
    emb = torch.cat([ang, ang], dim=-1)
    cos, sin = emb.cos(), emb.sin()
    cos._pe_positions = position_ids
    cos._pe_theta = float(theta)
    return cos, sin


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding of ``x`` ``(B, heads, S, hd)`` (reference ``nn.py:45-49``)."""
    pos = getattr(cos, "_pe_positions", None)
    if pos is None:
        raise L.PeError("apply_rope needs the (cos, sin) pair returned by build_rope_cache")
    B, nh, S, hd = x.shape
    xr = x.transpose(1, 2).reshape(B, S, nh * hd)
    y = _RopeFn.apply(xr, pos.expand(B, S), nh, hd, cos._pe_theta)
    return y.view(B, S, nh, hd).transpose(1, 2)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """GQA expansion (reference ``nn.py:52-56``); the attention kernels broadcast
    K/V heads themselves and never call this."""
    if n_rep == 1:
        return x
    b, kvh, s, hd = x.shape
    return x[:, :, None, :, :].expand(b, kvh, n_rep, s, hd).reshape(b, kvh * n_rep, s, hd)


def _layout_from_bias(bias) -> ops.AttnLayout:
    if isinstance(bias, ops.AttnLayout):
        return bias
    return ops.AttnLayout(L.LAYOUT_BIAS, bias=bias)


class Attention(nn.Module):
    """GQA attention with RoPE and an additive bias (reference ``nn.py:59-89``).

    ``bias`` may be the reference's dense ``(B|1, 1, S, S)`` additive bias or an
    :class:`ops.AttnLayout` that lets the kernel re-derive the MTP mask.
    """

    def __init__(self, hidden: int, n_heads: int, n_kv_heads: int, theta: float):
        super().__init__()
        self.n_heads = n_heads
        self.n_kv_heads = n_kv_heads
        self.head_dim = hidden // n_heads
        self.theta = theta
        self.q_proj = nn.Linear(hidden, n_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(hidden, n_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(hidden, n_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(n_heads * self.head_dim, hidden, bias=False)

    def forward(self, x, cos, sin, bias):
        pos = getattr(cos, "_pe_positions", None)
        if pos is None:
            raise L.PeError("Attention needs the (cos, sin) pair returned by build_rope_cache")
        B, S, _ = x.shape
        hd, nh, nkv = self.head_dim, self.n_heads, self.n_kv_heads
        q = linear(x, self.q_proj.weight)
        k = linear(x, self.k_proj.weight)
        v = linear(x, self.v_proj.weight)
        pos_full = pos.expand(B, S)
        q = _RopeFn.apply(q, pos_full, nh, hd, cos._pe_theta)
        k = _RopeFn.apply(k, pos_full, nkv, hd, cos._pe_theta)
        layout = _layout_from_bias(bias)
        if layout.bias is not None and layout.bias.dtype != x.dtype:
            layout = ops.AttnLayout(L.LAYOUT_BIAS, bias=layout.bias.to(x.dtype))
        o = _AttnFn.apply(q, k, v, layout, nh, nkv, hd)
        return linear(o, self.o_proj.weight)


class SwiGLU(nn.Module):
    """``down(silu(gate x) * up x)`` (reference ``nn.py:92-100``)."""

    def __init__(self, hidden: int, intermediate: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden, intermediate, bias=False)
        self.up_proj = nn.Linear(hidden, intermediate, bias=False)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False)
        self.intermediate = intermediate

    def forward(self, x):
        w = torch.cat([self.gate_proj.weight, self.up_proj.weight], dim=0)
        gu = linear(x, w)
        return linear(_SwiGLUFn.apply(gu, self.intermediate), self.down_proj.weight)


class DecoderLayer(nn.Module):
    """Pre-norm block ``x += attn(norm x); x += mlp(norm x)`` (reference ``nn.py:103-124``)."""

    def __init__(self, hidden, n_heads, n_kv_heads, intermediate, theta, eps):
        super().__init__()
        self.input_norm = RMSNorm(hidden, eps)
        self.attn = Attention(hidden, n_heads, n_kv_heads, theta)
        self.post_norm = RMSNorm(hidden, eps)
        self.mlp = SwiGLU(hidden, intermediate)

    def forward(self, x, cos, sin, bias):
        x = x + self.attn(self.input_norm(x), cos, sin, bias)
        x = x + self.mlp(self.post_norm(x))
        return x
