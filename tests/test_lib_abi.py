"""The C-ABI library loads without a GPU and exports every entry point that
``include/pe_b200.h`` declares, with the ctypes signatures the package binds."""

from __future__ import annotations

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "pe_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pe_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "pe_gemm" in names and "pe_attn_fwd" in names and "pe_lmhead_ce" in names


def test_library_exports_every_declared_symbol():
    from parallel_eagle_b200 import _lib

    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(_lib.SIGNATURES), "ctypes table out of sync with the header"


def test_host_only_queries_work_without_gpu():
    from parallel_eagle_b200 import _lib

    lib = _lib.load()
    assert lib.pe_version() >= 1
    assert lib.pe_rmsnorm_bwd_blocks(10_000) >= 1
    assert lib.pe_lmhead_ce_workspace(1, 100, 64, 1000, 0) > 0
    # argument validation happens before any CUDA call
    assert lib.pe_rope(1, 4, 2, 7, None, 14, None, 10000.0, 0, None) == 1
    assert b"rope" in lib.pe_last_error()


def test_segment_attention_and_topk_validate_before_any_cuda_call():
    import numpy as np

    from parallel_eagle_b200 import _lib

    lib = _lib.load()
    bf16 = 1
    # no segments
    assert lib.pe_attn_fwd_segments(bf16, 0, None, 5, 28, 4, 128, None, 0, None, 0, None, 0,
                                     None, 0, None, 0, None, None) != 0
    assert b"segment" in lib.pe_last_error()
    # a segment with a0 >= a1
    bad = np.array([0, 512, 700, 700], dtype=np.int64)
    assert lib.pe_attn_fwd_segments(bf16, 2, bad.ctypes.data, 5, 28, 4, 128, None, 0, None, 0,
                                     None, 0, None, 0, None, 0, None, None) != 0
    assert b"segment 1" in lib.pe_last_error()
    # kernel-variant bits are not accepted by the stacked-segment entry points
    ok = np.array([0, 512, 512, 1024], dtype=np.int64)
    assert lib.pe_attn_fwd_segments(bf16, 2, ok.ctypes.data, 5, 28, 4, 128, None, 0, None, 0,
                                     None, 0, None, 0, None, 1 << 8, None, None) != 0
    assert b"variant" in lib.pe_last_error()
    # the stacked-segment workspace covers the deltas of every stacked row
    rows = (512 + 512 * 4) + (1024 + 512 * 4)
    assert lib.pe_attn_bwd_segments_workspace(bf16, 2, ok.ctypes.data, 5, 28, 4, 128) >= 28 * rows * 4
    assert lib.pe_attn_bwd_segments_workspace(bf16, 0, None, 5, 28, 4, 128) == 0
    # top-k: k must lie in [1, V]
    assert lib.pe_topk_logprobs(bf16, 2, 7, None, 7, 8, 0, None, None, None) != 0
    assert b"topk" in lib.pe_last_error()
    assert lib.pe_topk_logprobs(bf16, 0, 7, None, 7, 3, 0, None, None, None) == 0
    # sampling distributions: positive finite temperature, strides covering the row
    for t in (0.0, -1.0, float("inf"), float("nan")):
        assert lib.pe_softmax_rows(bf16, 2, 7, None, 7, t, None, 7, None) != 0
        assert b"temperature" in lib.pe_last_error()
    assert lib.pe_softmax_rows(bf16, 2, 7, None, 6, 1.0, None, 7, None) != 0
    assert lib.pe_softmax_rows(bf16, 2, 7, None, 7, 1.0, None, 6, None) != 0
    assert lib.pe_softmax_rows(bf16, 0, 7, None, 7, 0.7, None, 7, None) == 0


def test_ops_reject_host_tensors_before_any_kernel():
    """Every Python wrapper raises PeError for a tensor in host memory instead of
    handing its address to a kernel (there is no CPU fallback); the C side's range
    checks of the multi-range column sum also run before any launch."""
    import pytest
    import torch

    from parallel_eagle_b200 import _lib, ops

    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    idx = torch.zeros(2, dtype=torch.long)
    f32 = torch.zeros(16, dtype=torch.float32)
    calls = [
        lambda: ops.rowsum_cols(x),
        lambda: ops.rowsum_cols_ranges(x, [(0, 2)]),
        lambda: ops.swiglu_fwd(x, 8),
        lambda: ops.swiglu_bwd(x[:, :8], x, 8),
        lambda: ops.gather_rows(x, idx),
        lambda: ops.scatter_rows(x[:2], idx, x),
        lambda: ops.fill_rows(x[0], x),
        lambda: ops.cast_from_f32(f32, x[0]),
        lambda: ops.sumsq_into(x, f32[:1]),
        lambda: ops.colsum_into(f32.view(1, 16), f32, False),
        lambda: ops.linear_swiglu_bwd(x, x[:, :8].t().contiguous(), x, 8),
    ]
    for call in calls:
        with pytest.raises(_lib.PeError, match="CUDA tensors only"):
            call()
    lib = _lib.load()
    import numpy as np

    bad = np.array([5, 3], dtype=np.int64)  # end before begin
    assert lib.pe_rowsum_cols_ranges(1, 1, bad.ctypes.data, 16, None, 16, None, None) != 0
    assert b"range 0" in lib.pe_last_error()
    assert lib.pe_rowsum_cols_ranges(1, 17, bad.ctypes.data, 16, None, 16, None, None) != 0
