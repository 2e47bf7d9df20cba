"""ctypes binding of ``libpe_b200.so`` (declared in ``include/pe_b200.h``).

The library is the only compute path of this package: if it is missing, or the
tensors are not CUDA tensors, calls fail loudly.  There is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpe_b200.so"

F32, BF16, F16 = 0, 1, 2
ALGO_AUTO, ALGO_SIMT, ALGO_TCGEN05 = 0, 1, 2
LAYOUT_PARTITION, LAYOUT_INDEXED, LAYOUT_BIAS = 0, 1, 2

_vp, _i64, _f32, _int, _sz = C.c_void_p, C.c_int64, C.c_float, C.c_int, C.c_size_t

# name -> (restype, argtypes); mirrors include/pe_b200.h
SIGNATURES: dict[str, tuple] = {
    "pe_last_error": (C.c_char_p, []),
    "pe_version": (_int, []),
    "pe_launch_count": (_i64, []),
    "pe_rmsnorm_fwd": (_int, [_int, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _f32, _vp]),
    "pe_rmsnorm_bwd": (
        _int,
        [_int, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp],
    ),
    "pe_rmsnorm_bwd_blocks": (_i64, [_i64]),
    "pe_rmsnorm_bwd_noalloc": (
        _int, [_int, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _int, _vp]
    ),
    "pe_colsum_f32": (_int, [_int, _i64, _i64, _vp, _vp, _int, _vp]),
    "pe_feature_norm_fwd": (
        _int, [_int, _int, _i64, _int, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _f32, _vp]
    ),
    "pe_feature_norm_dw": (
        _int, [_int, _int, _i64, _int, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp]
    ),
    "pe_rope": (_int, [_int, _i64, _int, _int, _vp, _i64, _vp, _f32, _int, _vp]),
    "pe_rope_table": (_int, [_int, _i64, _int, _vp, _f32, _vp, _i64, _vp]),
    "pe_linear_swiglu": (
        _int, [_int, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _vp]
    ),
    "pe_linear_swiglu_bwd": (
        _int, [_int, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _vp]
    ),
    "pe_linear_rope": (
        _int, [_int, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _int,
               _vp, _vp]
    ),
    "pe_gemm": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _int, _vp, _i64,
         _f32, _f32, _int, _vp, _vp],
    ),
    "pe_attn_fwd": (
        _int,
        [_int, _i64, _i64, _int, _int, _int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64,
         _vp, _i64, _i64, _vp, _int, _i64, _i64, _int, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp],
    ),
    "pe_attn_bwd_workspace": (_sz, [_int, _i64, _i64, _int, _int, _int]),
    "pe_attn_bwd": (
        _int,
        [_int, _i64, _i64, _int, _int, _int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64,
         _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _i64, _vp, _sz, _int, _i64, _i64, _int, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp],
    ),
    "pe_attn_fwd_segments": (
        _int,
        [_int, _int, _vp, _int, _int, _int, _int, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64,
         _vp, _int, _vp, _vp],
    ),
    "pe_attn_bwd_segments_workspace": (_sz, [_int, _int, _vp, _int, _int, _int, _int]),
    "pe_attn_bwd_segments": (
        _int,
        [_int, _int, _vp, _int, _int, _int, _int, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64,
         _vp, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _sz, _vp, _i64, _int, _vp, _vp],
    ),
    "pe_lmhead_ce_workspace": (_sz, [_int, _i64, _i64, _i64, _int]),
    "pe_lmhead_ce": (
        _int,
        [_int, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _f32, _vp, _i64, _vp, _vp, _sz,
         _int, _vp, _vp],
    ),
    "pe_embed_rows": (_int, [_int, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
    "pe_fill_rows": (_int, [_int, _i64, _i64, _vp, _vp, _i64, _vp]),
    "pe_swiglu_fwd": (_int, [_int, _i64, _i64, _vp, _i64, _vp, _i64, _vp]),
    "pe_swiglu_bwd": (_int, [_int, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp]),
    "pe_rowsum_cols": (_int, [_int, _i64, _i64, _vp, _i64, _vp, _vp]),
    "pe_rowsum_cols_ranges": (_int, [_int, _int, _vp, _i64, _vp, _i64, _vp, _vp]),
    "pe_scatter_rows": (_int, [_int, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp]),
    "pe_gather_rows": (_int, [_int, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp]),
    "pe_cast_f32": (_int, [_int, _i64, _vp, _vp, _vp]),
    "pe_topk_logprobs": (_int, [_int, _i64, _i64, _vp, _i64, _int, _int, _vp, _vp, _vp]),
    "pe_softmax_rows": (_int, [_int, _i64, _i64, _vp, _i64, _f32, _vp, _i64, _vp]),
    "pe_sumsq": (_int, [_int, _i64, _vp, _vp, _vp]),
    "pe_sumsq_partials": (_int, [_int, _i64, _vp, _vp, _i64, _vp]),
    "pe_sum_f32": (_int, [_i64, _vp, _vp, _int, _vp]),
    "pe_adamw_step": (
        _int, [_int, _i64, _vp, _vp, _vp, _vp, _vp, _f32, _f32, _f32, _f32, _f32, _f32, _i64, _vp]
    ),
    "pe_wait_probe": (_int, [C.c_uint64, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


class PeError(RuntimeError):
    """A nonzero status returned by libpe_b200, or a call it cannot serve."""


def load(path: Path | str | None = None) -> C.CDLL:
    """Load (once) and return the kernel library; raise if it is not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise PeError(
                f"{p} is not built; run `python -m parallel_eagle_b200.build` "
                "(parallel_eagle_b200 has no CPU fallback)"
            )
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().pe_last_error().decode(errors="replace")
        raise PeError(f"{what} failed ({rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    raise PeError(f"unsupported dtype {dt}: parallel_eagle_b200 kernels take float32 or bfloat16")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise PeError(
                "parallel_eagle_b200 runs on CUDA tensors only (got a tensor on "
                f"{t.device}); there is no CPU fallback"
            )


def launch_count() -> int:
    return int(load().pe_launch_count())
