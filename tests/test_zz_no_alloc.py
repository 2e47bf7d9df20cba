"""The allocation-free RMSNorm backward (``pe_rmsnorm_bwd_noalloc``).

Some callers cannot allocate device memory -- a host that owns the device's whole
memory budget and forbids its plugins to allocate, or a hot path on which
cudaMalloc's implicit device synchronisation is not allowed.  For them the library
offers one entry point whose scratch (the per-block weight-gradient partials) lives
in a fixed array inside the library.  This test calls it through the C ABI and
checks it against the workspace-taking entry points (``pe_rmsnorm_bwd`` +
``pe_colsum_f32``) on two calls in a row, so the second call also shows that the
shared array's leftover contents from the first call do not leak into the result.

The file name sorts last so a ``-x`` run reaches it only after every other test.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from parallel_eagle_b200 import _lib as L  # noqa: E402

DEV = torch.device("cuda")


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


def _reference(lib, dtype, dy, x, w, rstd, res, dw_init):
    """dx and dw from the workspace-taking entry points."""
    rows, H = x.shape
    code = L.dtype_code(dtype)
    stream = torch.cuda.current_stream().cuda_stream
    dx = torch.empty_like(x)
    nblk = int(lib.pe_rmsnorm_bwd_blocks(rows))
    part = torch.empty(nblk, H, dtype=torch.float32, device=DEV)
    L.check(lib.pe_rmsnorm_bwd(code, rows, H, dy.data_ptr(), H, x.data_ptr(), H, w.data_ptr(),
                               rstd.data_ptr(), dx.data_ptr(), H, res.data_ptr(), H,
                               part.data_ptr(), stream), "pe_rmsnorm_bwd")
    dw = dw_init.clone()
    L.check(lib.pe_colsum_f32(code, nblk, H, part.data_ptr(), dw.data_ptr(), 1, stream),
            "pe_colsum_f32")
    return dx, dw


def _no_alloc(lib, dtype, dy, x, w, rstd, res, dw_init):
    rows, H = x.shape
    dx = torch.empty_like(x)
    dw = dw_init.clone()
    rc = lib.pe_rmsnorm_bwd_noalloc(L.dtype_code(dtype), rows, H, dy.data_ptr(), H, x.data_ptr(),
                                    H, w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), H,
                                    res.data_ptr(), H, dw.data_ptr(), 1,
                                    torch.cuda.current_stream().cuda_stream)
    L.check(rc, "pe_rmsnorm_bwd_noalloc")
    return dx, dw


def _case(dtype, rows, H, seed):
    x = _rand((rows, H), dtype, seed) * 2
    w = (1 + 0.1 * _rand((H,), torch.float32, seed + 1)).to(dtype)
    dy = _rand((rows, H), dtype, seed + 2)
    res = _rand((rows, H), dtype, seed + 3)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-5).contiguous()
    dw_init = _rand((H,), dtype, seed + 4)
    return dy, x, w, rstd, res, dw_init


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_points_twice(dtype):
    lib = L.load()
    tol_dx = 1e-6 if dtype == torch.float32 else 1e-2
    tol_dw = 1e-5 if dtype == torch.float32 else 1e-2
    # a large call that fills many partial rows, then a small one that uses fewer:
    # stale rows from the first call must not reach the second call's dw
    for rows, H, seed in ((5000, 3584, 10), (37, 256, 20)):
        args = _case(dtype, rows, H, seed)
        ref_dx, ref_dw = _reference(lib, dtype, *args)
        dx, dw = _no_alloc(lib, dtype, *args)
        torch.cuda.synchronize()
        assert _rel(dx.float(), ref_dx.float()) < tol_dx, (rows, H)
        assert _rel(dw.float(), ref_dw.float()) < tol_dw, (rows, H)


def test_noalloc_rejects_rows_wider_than_its_scratch():
    lib = L.load()
    H = 8200
    dy, x, w, rstd, res, dw = _case(torch.bfloat16, 4, H, 30)
    rc = lib.pe_rmsnorm_bwd_noalloc(L.BF16, 4, H, dy.data_ptr(), H, x.data_ptr(), H,
                                    w.data_ptr(), rstd.data_ptr(), torch.empty_like(x).data_ptr(),
                                    H, None, 0, dw.data_ptr(), 1,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"8192" in lib.pe_last_error()
