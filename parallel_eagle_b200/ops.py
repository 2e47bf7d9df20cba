"""Tensor-level wrappers over the C ABI (one function per kernel entry point).

Each wrapper checks devices/dtypes, passes raw pointers, strides and the current
CUDA stream, and turns a nonzero status into :class:`PeError`.  Outputs are
allocated here (torch owns all memory); the library itself never allocates.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L

_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the tensor-core kernels write a code into when a
    bounded wait times out (0 = healthy)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_status(device: torch.device) -> None:
    """Raise if any tensor-core kernel on ``device`` recorded a timed-out wait."""
    s = status_word(device)
    code = int(s.item())
    if code != 0:
        s.zero_()
        raise L.PeError(f"a tensor-core kernel gave up waiting (fault code {code})")


def _lib():
    return L.load()


def _row_stride(t: torch.Tensor) -> int:
    if t.dim() != 2 or (t.stride(1) != 1 and t.shape[1] > 1):
        raise L.PeError(
            f"expected a 2-D row-major view, got shape {tuple(t.shape)} strides {t.stride()}"
        )
    return t.stride(0) if t.shape[0] > 1 else max(t.stride(0), t.shape[1])


# ----------------------------------------------------------------- norms ----


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None):
    L.require_cuda(x, w)
    rows, H = x.shape
    if out is None:
        out = torch.empty(rows, H, dtype=x.dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    rc = _lib().pe_rmsnorm_fwd(
        L.dtype_code(x.dtype), rows, H, x.data_ptr(), _row_stride(x), w.data_ptr(),
        out.data_ptr(), _row_stride(out), rstd.data_ptr(), float(eps), L.stream_ptr(x.device),
    )
    L.check(rc, "pe_rmsnorm_fwd")
    return out, rstd


def rmsnorm_bwd(dy, x, w, rstd, dx=None, residual=None, want_dw: bool = True):
    """Returns ``(dx, dw_partial)``; ``dx = residual + d/dx``; ``dw_partial`` is the
    fp32 per-block partial reduced by :func:`colsum_into`."""
    L.require_cuda(dy, x, w)
    rows, H = x.shape
    if dx is None:
        dx = torch.empty(rows, H, dtype=x.dtype, device=x.device)
    lib = _lib()
    part = None
    if want_dw:
        nblk = int(lib.pe_rmsnorm_bwd_blocks(rows))
        part = torch.empty(nblk, H, dtype=torch.float32, device=x.device)
    rc = lib.pe_rmsnorm_bwd(
        L.dtype_code(x.dtype), rows, H, dy.data_ptr(), _row_stride(dy), x.data_ptr(),
        _row_stride(x), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), _row_stride(dx),
        L.ptr(residual), _row_stride(residual) if residual is not None else 0, L.ptr(part),
        L.stream_ptr(x.device),
    )
    L.check(rc, "pe_rmsnorm_bwd")
    return dx, part


def colsum_into(partial: torch.Tensor, out: torch.Tensor, accumulate: bool) -> torch.Tensor:
    """``out (+)= partial.sum(0)`` with a fixed summation order."""
    L.require_cuda(partial, out)
    nblk, H = partial.shape
    rc = _lib().pe_colsum_f32(
        L.dtype_code(out.dtype), nblk, H, partial.data_ptr(), out.data_ptr(), int(accumulate),
        L.stream_ptr(out.device),
    )
    L.check(rc, "pe_colsum_f32")
    return out


_SRC_CODES = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16}


def feature_norm_ok(x: torch.Tensor, hidden: int, nfl: int) -> bool:
    """Whether :func:`feature_norm_fwd` takes this feature tensor directly."""
    return (x.is_cuda and x.dtype in _SRC_CODES and x.dim() == 2 and x.stride(1) == 1
            and x.shape[1] == nfl * hidden and hidden % 256 == 0 and hidden <= 8192
            and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0)


def feature_norm_fwd(x, w, nfl: int, hidden: int, dtype, eps: float, src_tok=None, tokens=None):
    """RMSNorm of the ``hidden``-wide blocks of feature rows read straight from ``x`` (fp16,
    bf16 or fp32; row ``src_tok[t]`` for output token ``t``), each element rounded to
    ``dtype`` first (the reference's ``features.to(dtype)``): returns ``y``
    ``[tokens * nfl, hidden]`` in ``dtype`` and ``rstd``."""
    L.require_cuda(x, w)
    tokens = int(x.shape[0] if tokens is None else tokens)
    y = torch.empty(tokens * nfl, hidden, dtype=dtype, device=x.device)
    rstd = torch.empty(tokens * nfl, dtype=torch.float32, device=x.device)
    rc = _lib().pe_feature_norm_fwd(
        _SRC_CODES[x.dtype], L.dtype_code(dtype), tokens, nfl, hidden, x.data_ptr(), x.stride(0),
        L.ptr(src_tok), w.data_ptr(), y.data_ptr(), hidden, rstd.data_ptr(), float(eps),
        L.stream_ptr(x.device),
    )
    L.check(rc, "pe_feature_norm_fwd")
    return y, rstd


def feature_norm_dw(dy, x, rstd, nfl: int, hidden: int, src_tok=None):
    """Weight-gradient partials of :func:`feature_norm_fwd` (``[nblk, hidden]`` fp32, reduce
    with :func:`colsum_into`); ``dy`` ``[tokens * nfl, hidden]``."""
    L.require_cuda(dy, x, rstd)
    rows = dy.shape[0]
    lib = _lib()
    nblk = int(lib.pe_rmsnorm_bwd_blocks(rows))
    part = torch.empty(nblk, hidden, dtype=torch.float32, device=dy.device)
    rc = lib.pe_feature_norm_dw(
        _SRC_CODES[x.dtype], L.dtype_code(dy.dtype), rows // nfl, nfl, hidden, dy.data_ptr(),
        _row_stride(dy), x.data_ptr(), x.stride(0), L.ptr(src_tok), rstd.data_ptr(),
        part.data_ptr(), L.stream_ptr(dy.device),
    )
    L.check(rc, "pe_feature_norm_dw")
    return part


# ------------------------------------------------------------------ rope ----


def rope_(x: torch.Tensor, heads: int, head_dim: int, pos: torch.Tensor, theta: float, inverse=False):
    """In-place rotary embedding on the first ``heads * head_dim`` columns of each row."""
    L.require_cuda(x, pos)
    rc = _lib().pe_rope(
        L.dtype_code(x.dtype), x.shape[0], heads, head_dim, x.data_ptr(), _row_stride(x),
        pos.data_ptr(), float(theta), int(inverse), L.stream_ptr(x.device),
    )
    L.check(rc, "pe_rope")
    return x


def rope_table(pos: torch.Tensor, head_dim: int, theta: float, dtype: torch.dtype) -> torch.Tensor:
    """``[rows, head_dim]`` table of ``[cos | sin]`` per position (rounded to ``dtype``)
    that the fused rotations read: :func:`linear_rope` and
    :func:`attn_bwd_segments` (``rope_cs``)."""
    L.require_cuda(pos)
    rows = pos.shape[0]
    cs = torch.empty(rows, head_dim, dtype=dtype, device=pos.device)
    rc = _lib().pe_rope_table(L.dtype_code(dtype), rows, head_dim, pos.data_ptr(), float(theta),
                              cs.data_ptr(), head_dim, L.stream_ptr(pos.device))
    L.check(rc, "pe_rope_table")
    return cs


def linear_rope(x, w, rope_cs, rot_cols: int, head_dim: int, out=None):
    """``out = x w^T`` with the rotary embedding applied in the GEMM epilogue to the
    ``head_dim`` blocks of columns ``[0, rot_cols)`` (bf16, head_dim 128): the fused
    q|k|v projection + RoPE, bit-identical to :func:`linear` then :func:`rope_`."""
    L.require_cuda(x, w, rope_cs)
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    rc = _lib().pe_linear_rope(
        L.dtype_code(x.dtype), M, N, K, x.data_ptr(), _row_stride(x), w.data_ptr(), _row_stride(w),
        out.data_ptr(), _row_stride(out), rope_cs.data_ptr(), rope_cs.stride(0), int(rot_cols),
        int(head_dim), status_word(x.device).data_ptr(), L.stream_ptr(x.device),
    )
    L.check(rc, "pe_linear_rope")
    return out


def linear_swiglu(x, w_gu, intermediate: int, gu=None, act=None, algo=L.ALGO_AUTO):
    """``gu = x w_gu^T`` (``[M, 2I]``: gate | up) and ``act = silu(gate) * up``
    (``[M, I]``) in one call: the activation comes from the GEMM epilogue on the
    tensor-core pair path (same bits as :func:`linear` then :func:`swiglu_fwd`)."""
    L.require_cuda(x, w_gu)
    M, K = x.shape
    I = int(intermediate)
    if w_gu.shape[0] != 2 * I:
        raise L.PeError(f"linear_swiglu: w_gu has {w_gu.shape[0]} rows, expected 2 * {I}")
    if gu is None:
        gu = torch.empty(M, 2 * I, dtype=x.dtype, device=x.device)
    if act is None:
        act = torch.empty(M, I, dtype=x.dtype, device=x.device)
    rc = _lib().pe_linear_swiglu(
        L.dtype_code(x.dtype), M, I, K, x.data_ptr(), _row_stride(x), w_gu.data_ptr(),
        _row_stride(w_gu), gu.data_ptr(), _row_stride(gu), act.data_ptr(), _row_stride(act), algo,
        status_word(x.device).data_ptr(), L.stream_ptr(x.device),
    )
    L.check(rc, "pe_linear_swiglu")
    return gu, act


def linear_swiglu_bwd(dy, w_dn, gu, intermediate: int, out=None, algo=L.ALGO_AUTO):
    """``dgu = swiglu_bwd(dy w_dn, gu)``: the down projection's input gradient
    (``dy [M, H]``, ``w_dn [H, I]``) carried through the SwiGLU backward into the
    gate | up gradient ``[M, 2I]`` in one call -- on the tensor-core pair path the
    SwiGLU backward runs in the GEMM epilogue and the activation gradient is never
    stored (same bits as :func:`linear_dgrad` then :func:`swiglu_bwd`)."""
    L.require_cuda(dy, w_dn, gu)
    M, K = dy.shape
    I = int(intermediate)
    if w_dn.shape != (K, I) or gu.shape[0] != M or gu.shape[1] < 2 * I:
        raise L.PeError(f"linear_swiglu_bwd: shapes dy {tuple(dy.shape)}, w_dn "
                        f"{tuple(w_dn.shape)}, gu {tuple(gu.shape)} do not match I = {I}")
    if out is None:
        out = torch.empty(M, 2 * I, dtype=dy.dtype, device=dy.device)
    rc = _lib().pe_linear_swiglu_bwd(
        L.dtype_code(dy.dtype), M, I, K, dy.data_ptr(), _row_stride(dy), w_dn.data_ptr(),
        _row_stride(w_dn), gu.data_ptr(), _row_stride(gu), out.data_ptr(), _row_stride(out), algo,
        status_word(dy.device).data_ptr(), L.stream_ptr(dy.device),
    )
    L.check(rc, "pe_linear_swiglu_bwd")
    return out


# ------------------------------------------------------------------ gemm ----


def gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, Cin=None, ldcin=0, alpha=1.0, beta=0.0,
         algo=L.ALGO_AUTO):
    """``C = alpha * A B^T + beta * Cin`` on raw element strides (see the C header)."""
    L.require_cuda(A, B, C)
    rc = _lib().pe_gemm(
        L.dtype_code(A.dtype), M, N, K, A.data_ptr(), a_sm, a_sk, B.data_ptr(), b_sn, b_sk,
        C.data_ptr(), ldc, L.dtype_code(C.dtype), L.ptr(Cin), ldcin, float(alpha), float(beta),
        algo, status_word(C.device).data_ptr(), L.stream_ptr(C.device),
    )
    L.check(rc, "pe_gemm")
    return C


def linear(x, w, out=None, residual=None, algo=L.ALGO_AUTO):
    """``out = x w^T (+ residual)``; x ``[M, K]`` (row view), w ``[N, K]``."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    return gemm(M, N, K, x, _row_stride(x), 1, w, _row_stride(w), 1, out, _row_stride(out),
                residual, _row_stride(residual) if residual is not None else 0, 1.0,
                1.0 if residual is not None else 0.0, algo)


def linear_dgrad(dy, w, out=None, residual=None, algo=L.ALGO_AUTO):
    """``out = dy w (+ residual)``; dy ``[M, N]``, w ``[N, K]`` -> ``[M, K]``."""
    M, N = dy.shape
    K = w.shape[1]
    if out is None:
        out = torch.empty(M, K, dtype=dy.dtype, device=dy.device)
    return gemm(M, K, N, dy, _row_stride(dy), 1, w, 1, _row_stride(w), out, _row_stride(out),
                residual, _row_stride(residual) if residual is not None else 0, 1.0,
                1.0 if residual is not None else 0.0, algo)


def linear_wgrad(dy, x, grad=None, accumulate=False, algo=L.ALGO_AUTO):
    """``grad (+)= dy^T x``; dy ``[M, N]``, x ``[M, K]`` -> ``[N, K]``."""
    M, N = dy.shape
    K = x.shape[1]
    if grad is None:
        grad = torch.empty(N, K, dtype=dy.dtype, device=dy.device)
        accumulate = False
    return gemm(N, K, M, dy, 1, _row_stride(dy), x, 1, _row_stride(x), grad, _row_stride(grad),
                grad if accumulate else None, _row_stride(grad), 1.0, 1.0 if accumulate else 0.0,
                algo)


# ------------------------------------------------------------- attention ----


class AttnLayout:
    """How the attention kernel re-derives the attend rule of a packed sequence.

    ``LAYOUT_PARTITION``: the segment layout of the partitioned step (reference
    ``partition.py:41-55``) -- slots ``0..a1-1`` are real, then anchors
    ``a0..a1-1`` x depths ``1..k-1``; only ``(a0, a1, k)`` is needed.
    ``LAYOUT_INDEXED``: explicit int32 per-slot ``anchor``/``depth``.
    ``LAYOUT_BIAS``: a dense additive bias ``[B|1, 1, S, S]`` (the generic
    ``ParallelDrafter.forward`` contract).
    """

    def __init__(self, kind: int, a0=0, a1=0, k=1, anchor=None, depth=None, bias=None):
        self.kind, self.a0, self.a1, self.k = kind, a0, a1, k
        self.anchor, self.depth, self.bias = anchor, depth, bias

    def bias_strides(self):
        if self.bias is None:
            return 0, 0
        b = self.bias
        return (b.stride(0) if b.shape[0] > 1 else 0), b.stride(2)


def _bsq(t: torch.Tensor):
    if t.stride(2) != 1:
        raise L.PeError("attention operands need unit stride along the head dimension")
    return t.stride(0), t.stride(1)


def attn_fwd(q, k, v, n_heads, n_kv_heads, head_dim, layout: AttnLayout, algo=L.ALGO_AUTO,
             o=None, lse=None):
    """q ``[B, S, Hq*hd]``, k/v ``[B, S, Hkv*hd]`` (row views; last stride 1).  ``o``
    (a row view like q) and ``lse`` (fp32 ``[B, Hq, S]``, contiguous) may be given."""
    L.require_cuda(q, k, v)
    B, S = q.shape[0], q.shape[1]
    if o is None:
        o = torch.empty(B, S, n_heads * head_dim, dtype=q.dtype, device=q.device)
    if lse is None:
        lse = torch.empty(B, n_heads, S, dtype=torch.float32, device=q.device)
    bsb, bsq = layout.bias_strides()
    rc = _lib().pe_attn_fwd(
        L.dtype_code(q.dtype), B, S, n_heads, n_kv_heads, head_dim, q.data_ptr(), *_bsq(q),
        k.data_ptr(), *_bsq(k), v.data_ptr(), *_bsq(v), o.data_ptr(), *_bsq(o), lse.data_ptr(),
        layout.kind, layout.a0, layout.a1, layout.k, L.ptr(layout.anchor), L.ptr(layout.depth),
        L.ptr(layout.bias), bsb, bsq, algo, status_word(q.device).data_ptr(),
        L.stream_ptr(q.device),
    )
    L.check(rc, "pe_attn_fwd")
    return o, lse


def attn_bwd(q, k, v, o, do, lse, n_heads, n_kv_heads, head_dim, layout: AttnLayout,
             dq=None, dk=None, dv=None, algo=L.ALGO_AUTO):
    L.require_cuda(q, k, v, o, do, lse)
    B, S = q.shape[0], q.shape[1]
    if dq is None:
        dq = torch.empty(B, S, n_heads * head_dim, dtype=q.dtype, device=q.device)
    if dk is None:
        dk = torch.empty(B, S, n_kv_heads * head_dim, dtype=k.dtype, device=k.device)
    if dv is None:
        dv = torch.empty(B, S, n_kv_heads * head_dim, dtype=v.dtype, device=v.device)
    lib = _lib()
    nbytes = int(lib.pe_attn_bwd_workspace(L.dtype_code(q.dtype), B, S, n_heads, n_kv_heads,
                                           head_dim))
    ws = _workspace(q.device, nbytes, "attn_bwd")
    bsb, bsq = layout.bias_strides()
    rc = lib.pe_attn_bwd(
        L.dtype_code(q.dtype), B, S, n_heads, n_kv_heads, head_dim, q.data_ptr(), *_bsq(q),
        k.data_ptr(), *_bsq(k), v.data_ptr(), *_bsq(v), o.data_ptr(), *_bsq(o), do.data_ptr(),
        *_bsq(do), lse.data_ptr(), dq.data_ptr(), *_bsq(dq), dk.data_ptr(), *_bsq(dk),
        dv.data_ptr(), *_bsq(dv), ws.data_ptr(), ws.numel(), layout.kind, layout.a0, layout.a1,
        layout.k, L.ptr(layout.anchor), L.ptr(layout.depth), L.ptr(layout.bias), bsb, bsq, algo,
        status_word(q.device).data_ptr(), L.stream_ptr(q.device),
    )
    L.check(rc, "pe_attn_bwd")
    return dq, dk, dv


def _seg_bounds(bounds) -> np.ndarray:
    """(a0, a1) per segment as a contiguous int64 host array (kept alive by the caller)."""
    arr = np.ascontiguousarray(np.asarray(bounds, dtype=np.int64).reshape(-1, 2))
    if arr.shape[0] < 1:
        raise L.PeError("attention segments: no segments")
    return arr


def _row_ss(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise L.PeError("attention segments: operands are [rows, cols] views with unit column stride")
    return t.stride(0)


def segment_rows(bounds, k: int) -> list[int]:
    """Slot count a1 + (a1 - a0)(K - 1) of every segment (its rows in the stack)."""
    return [int(a1 + (a1 - a0) * (k - 1)) for a0, a1 in bounds]


def attn_fwd_segments(q, k, v, n_heads, n_kv_heads, head_dim, bounds, kdepth, o=None, lse=None,
                      algo=L.ALGO_AUTO):
    """Masked attention of all segments of one sequence in one call.  q ``[R, Hq*hd]``,
    k/v ``[R, Hkv*hd]`` row views holding the segments one after another (segment s
    in rows ``[row0_s, row0_s + S_s)``, S_s = a1 + (a1 - a0)(K - 1)).  Returns o (like
    q) and lse: fp32 ``[Hq * R]`` holding one ``[Hq, S_s]`` block per segment at
    ``Hq * row0_s``."""
    L.require_cuda(q, k, v)
    b = _seg_bounds(bounds)
    R = q.shape[0]
    if R != sum(segment_rows(b.tolist(), kdepth)):
        raise L.PeError("attention segments: rows != sum of segment slot counts")
    if o is None:
        o = torch.empty(R, n_heads * head_dim, dtype=q.dtype, device=q.device)
    if lse is None:
        lse = torch.empty(n_heads * R, dtype=torch.float32, device=q.device)
    rc = _lib().pe_attn_fwd_segments(
        L.dtype_code(q.dtype), b.shape[0], b.ctypes.data, kdepth, n_heads, n_kv_heads, head_dim,
        q.data_ptr(), _row_ss(q), k.data_ptr(), _row_ss(k), v.data_ptr(), _row_ss(v),
        o.data_ptr(), _row_ss(o), lse.data_ptr(), algo, status_word(q.device).data_ptr(),
        L.stream_ptr(q.device),
    )
    L.check(rc, "pe_attn_fwd_segments")
    return o, lse


def attn_bwd_segments(q, k, v, o, do, lse, n_heads, n_kv_heads, head_dim, bounds, kdepth,
                      dq=None, dk=None, dv=None, algo=L.ALGO_AUTO, rope_cs=None):
    """Backward of :func:`attn_fwd_segments` (same row and lse conventions); dq/dk/dv
    are overwritten.  With ``rope_cs`` (a :func:`rope_table` over the stacked rows) q
    and k are the rotated projections and dq / dk come back rotated by the transpose
    of the rotary embedding, fused into the dQ store and the dK cast."""
    L.require_cuda(q, k, v, o, do, lse)
    if rope_cs is not None:
        L.require_cuda(rope_cs)
        if rope_cs.dtype != q.dtype or rope_cs.shape[0] != q.shape[0] or rope_cs.stride(1) != 1:
            raise L.PeError("attention segments: rope_cs must be a [rows, >= head_dim] table "
                            "in the operands' dtype with one row per stacked slot")
    b = _seg_bounds(bounds)
    R = q.shape[0]
    if R != sum(segment_rows(b.tolist(), kdepth)):
        raise L.PeError("attention segments: rows != sum of segment slot counts")
    if dq is None:
        dq = torch.empty(R, n_heads * head_dim, dtype=q.dtype, device=q.device)
    if dk is None:
        dk = torch.empty(R, n_kv_heads * head_dim, dtype=k.dtype, device=k.device)
    if dv is None:
        dv = torch.empty(R, n_kv_heads * head_dim, dtype=v.dtype, device=v.device)
    lib = _lib()
    dt = L.dtype_code(q.dtype)
    nbytes = int(lib.pe_attn_bwd_segments_workspace(dt, b.shape[0], b.ctypes.data, kdepth,
                                                    n_heads, n_kv_heads, head_dim))
    ws = _workspace(q.device, nbytes, "attn_bwd")
    rc = lib.pe_attn_bwd_segments(
        dt, b.shape[0], b.ctypes.data, kdepth, n_heads, n_kv_heads, head_dim, q.data_ptr(),
        _row_ss(q), k.data_ptr(), _row_ss(k), v.data_ptr(), _row_ss(v), o.data_ptr(), _row_ss(o),
        do.data_ptr(), _row_ss(do), lse.data_ptr(), dq.data_ptr(), _row_ss(dq), dk.data_ptr(),
        _row_ss(dk), dv.data_ptr(), _row_ss(dv), ws.data_ptr(), ws.numel(), L.ptr(rope_cs),
        rope_cs.stride(0) if rope_cs is not None else 0, algo,
        status_word(q.device).data_ptr(), L.stream_ptr(q.device),
    )
    L.check(rc, "pe_attn_bwd_segments")
    return dq, dk, dv


def topk_logprobs(logits: torch.Tensor, k: int, raw: bool = False):
    """``(values, indices)`` of the ``k`` largest log-softmax entries of every row of
    ``logits`` ``[rows, V]`` (fp32 log-probabilities, int64 columns), ordered by value
    descending then column ascending; ``raw=True`` ranks the logits themselves
    (``k = 1``: argmax with the first maximal column)."""
    L.require_cuda(logits)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise L.PeError("topk_logprobs: logits must be [rows, V] with unit column stride")
    rows, V = logits.shape
    idx = torch.empty(rows, k, dtype=torch.int64, device=logits.device)
    val = torch.empty(rows, k, dtype=torch.float32, device=logits.device)
    rc = _lib().pe_topk_logprobs(L.dtype_code(logits.dtype), rows, V, logits.data_ptr(),
                                 logits.stride(0), k, int(raw), idx.data_ptr(), val.data_ptr(),
                                 L.stream_ptr(logits.device))
    L.check(rc, "pe_topk_logprobs")
    return val, idx


def softmax_rows(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """``softmax(logits.float() / temperature)`` per row of ``[rows, V]`` logits, fp32
    (the per-depth sampling distributions of a sampled draft chain)."""
    L.require_cuda(logits)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise L.PeError("softmax_rows: logits must be [rows, V] with unit column stride")
    rows, V = logits.shape
    q = torch.empty(rows, V, dtype=torch.float32, device=logits.device)
    rc = _lib().pe_softmax_rows(L.dtype_code(logits.dtype), rows, V, logits.data_ptr(),
                                logits.stride(0), float(temperature), q.data_ptr(), V,
                                L.stream_ptr(logits.device))
    L.check(rc, "pe_softmax_rows")
    return q


# --------------------------------------------------------- lm head + loss ----

_ws_cache: dict[tuple, torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int, purpose: str = "lmhead") -> torch.Tensor:
    """Grow-only per-device scratch buffer for one kernel family (reused across
    calls on the same stream; callers never hold it past the call)."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), purpose)
    t = _ws_cache.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _ws_cache[key] = t
    return t


def lmhead_ce(h, W, labels, grad_scale, loss_sum, teacher=None, dh=None, algo=L.ALGO_AUTO):
    """Fused frozen-head projection + CE (or soft-target) loss + input gradient.
    ``loss_sum`` (fp32 [1]) is incremented; returns ``dh``."""
    L.require_cuda(h, W)
    R, H = h.shape
    V = W.shape[0]
    if dh is None:
        dh = torch.empty(R, H, dtype=h.dtype, device=h.device)
    lib = _lib()
    soft = teacher is not None
    nbytes = int(lib.pe_lmhead_ce_workspace(L.dtype_code(h.dtype), R, H, V, int(soft)))
    ws = _workspace(h.device, nbytes)
    rc = lib.pe_lmhead_ce(
        L.dtype_code(h.dtype), R, H, V, h.data_ptr(), _row_stride(h), W.data_ptr(),
        L.ptr(labels), L.ptr(teacher), _row_stride(teacher) if soft else 0, float(grad_scale),
        dh.data_ptr(), _row_stride(dh), loss_sum.data_ptr(), ws.data_ptr(), ws.numel(), algo,
        status_word(h.device).data_ptr(), L.stream_ptr(h.device),
    )
    L.check(rc, "pe_lmhead_ce")
    return dh


# ------------------------------------------------------------ small ops ----


def embed_rows(ids, embed, out):
    L.require_cuda(ids, embed, out)
    rows, H = ids.shape[0], embed.shape[1]
    rc = _lib().pe_embed_rows(L.dtype_code(embed.dtype), rows, H, ids.data_ptr(), embed.data_ptr(),
                              out.data_ptr(), _row_stride(out), L.stream_ptr(out.device))
    L.check(rc, "pe_embed_rows")
    return out


def fill_rows(vec, out):
    L.require_cuda(vec, out)
    rows, H = out.shape
    rc = _lib().pe_fill_rows(L.dtype_code(out.dtype), rows, H, vec.data_ptr(), out.data_ptr(),
                             _row_stride(out), L.stream_ptr(out.device))
    L.check(rc, "pe_fill_rows")
    return out


def swiglu_fwd(gu, inter, out=None):
    L.require_cuda(gu, out)
    rows = gu.shape[0]
    if out is None:
        out = torch.empty(rows, inter, dtype=gu.dtype, device=gu.device)
    rc = _lib().pe_swiglu_fwd(L.dtype_code(gu.dtype), rows, inter, gu.data_ptr(), _row_stride(gu),
                              out.data_ptr(), _row_stride(out), L.stream_ptr(gu.device))
    L.check(rc, "pe_swiglu_fwd")
    return out


def swiglu_bwd(da, gu, inter, out=None):
    L.require_cuda(da, gu, out)
    rows = gu.shape[0]
    if out is None:
        out = torch.empty(rows, 2 * inter, dtype=gu.dtype, device=gu.device)
    rc = _lib().pe_swiglu_bwd(L.dtype_code(gu.dtype), rows, inter, da.data_ptr(), _row_stride(da),
                              gu.data_ptr(), _row_stride(gu), out.data_ptr(), _row_stride(out),
                              L.stream_ptr(gu.device))
    L.check(rc, "pe_swiglu_bwd")
    return out


def rowsum_cols(x, out=None):
    L.require_cuda(x, out)
    rows, H = x.shape
    if out is None:
        out = torch.empty(H, dtype=torch.float32, device=x.device)
    rc = _lib().pe_rowsum_cols(L.dtype_code(x.dtype), rows, H, x.data_ptr(), _row_stride(x),
                               out.data_ptr(), L.stream_ptr(x.device))
    L.check(rc, "pe_rowsum_cols")
    return out


def rowsum_cols_ranges(x, ranges, out=None):
    """fp32 ``[H]`` column sums of ``x`` over the row ranges ``[(begin, end), ...]``
    (host ints), in a fixed order: one launch per 16 ranges."""
    L.require_cuda(x, out)
    rows, H = x.shape
    ranges = [(int(b), int(e)) for b, e in ranges]
    if not ranges:
        raise L.PeError("rowsum_cols_ranges: no row ranges")
    for b, e in ranges:
        if not 0 <= b <= e <= rows:
            raise L.PeError(f"rowsum_cols_ranges: range [{b}, {e}) outside {rows} rows")
    if out is None:
        out = torch.empty(H, dtype=torch.float32, device=x.device)
    part = None
    for i in range(0, len(ranges), 16):
        grp = ranges[i : i + 16]
        if i == 0:
            dst = out
        else:
            if part is None:
                part = torch.empty_like(out)
            dst = part
        flat = (ctypes.c_int64 * (2 * len(grp)))(*[v for r in grp for v in r])
        rc = _lib().pe_rowsum_cols_ranges(L.dtype_code(x.dtype), len(grp), flat, H, x.data_ptr(),
                                          _row_stride(x), dst.data_ptr(), L.stream_ptr(x.device))
        L.check(rc, "pe_rowsum_cols_ranges")
        if i > 0:
            out += part
    return out


def gather_rows(src, idx, out=None):
    L.require_cuda(src, idx, out)
    rows, H = idx.shape[0], src.shape[1]
    if out is None:
        out = torch.empty(rows, H, dtype=src.dtype, device=src.device)
    rc = _lib().pe_gather_rows(L.dtype_code(src.dtype), rows, H, idx.data_ptr(), src.data_ptr(),
                               _row_stride(src), out.data_ptr(), _row_stride(out),
                               L.stream_ptr(src.device))
    L.check(rc, "pe_gather_rows")
    return out


def scatter_rows(src, idx, out):
    L.require_cuda(src, idx, out)
    rows, H = src.shape
    rc = _lib().pe_scatter_rows(L.dtype_code(src.dtype), rows, H, idx.data_ptr(), src.data_ptr(),
                                _row_stride(src), out.data_ptr(), _row_stride(out),
                                L.stream_ptr(src.device))
    L.check(rc, "pe_scatter_rows")
    return out


def cast_from_f32(x, out):
    L.require_cuda(x, out)
    rc = _lib().pe_cast_f32(L.dtype_code(out.dtype), x.numel(), x.data_ptr(), out.data_ptr(),
                            L.stream_ptr(x.device))
    L.check(rc, "pe_cast_f32")
    return out


_SUMSQ_BLOCKS = 1024  # fixed, so the partials (and the sum) do not depend on the device


def sumsq_into(g, out):
    """``out[0] += sum(g ** 2)``, deterministic: the same gradient gives the same bits on
    every run and every data-parallel rank (fixed-grid partials, fixed-order sum)."""
    L.require_cuda(g, out)
    lib = _lib()
    stream = L.stream_ptr(g.device)
    part = _workspace(g.device, _SUMSQ_BLOCKS * 4, "sumsq").view(torch.float32)[:_SUMSQ_BLOCKS]
    rc = lib.pe_sumsq_partials(L.dtype_code(g.dtype), g.numel(), g.data_ptr(), part.data_ptr(),
                               _SUMSQ_BLOCKS, stream)
    L.check(rc, "pe_sumsq_partials")
    rc = lib.pe_sum_f32(_SUMSQ_BLOCKS, part.data_ptr(), out.data_ptr(), 1, stream)
    L.check(rc, "pe_sum_f32")
    return out


def adamw_step(p, g, m, v, sumsq, max_norm, lr, beta1, beta2, eps, weight_decay, step):
    L.require_cuda(p, g, m, v, sumsq)
    rc = _lib().pe_adamw_step(L.dtype_code(p.dtype), p.numel(), p.data_ptr(), g.data_ptr(),
                              m.data_ptr(), v.data_ptr(), L.ptr(sumsq), float(max_norm), float(lr),
                              float(beta1), float(beta2), float(eps), float(weight_decay), int(step),
                              L.stream_ptr(p.device))
    L.check(rc, "pe_adamw_step")


def wait_probe(device: torch.device, limit_ns: int) -> bool:
    """Run the bounded-wait self-test kernel on ``device``: a wait that nothing
    completes gives up after ``limit_ns``, records code 901 in the device's status
    word and unwinds.  Returns whether the wait ran out (read back with a sync);
    :func:`check_status` then raises for the recorded code."""
    waited = torch.zeros(1, dtype=torch.int32, device=device)
    rc = _lib().pe_wait_probe(int(limit_ns), status_word(device).data_ptr(), waited.data_ptr(),
                              L.stream_ptr(device))
    L.check(rc, "pe_wait_probe")
    return bool(waited.item())
