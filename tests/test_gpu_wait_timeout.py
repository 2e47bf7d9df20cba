"""The bounded-wait unwind path on the GPU, made to run out on purpose.

Every mbarrier wait in the tensor-core kernels gives up after a limit, writes a
fault code into the caller's status word and unwinds (frees its tensor memory,
returns) instead of hanging; the Python layer raises on a nonzero word.  Here a
probe kernel waits -- with a 1 ms limit and no copy or MMA in flight -- on an
mbarrier that nothing arrives at, and the test checks the whole chain: the kernel
returns, the word holds the code, ``ops.check_status`` raises and clears it, and the
context still runs tensor-core work correctly afterwards.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from parallel_eagle_b200 import _lib as L  # noqa: E402
from parallel_eagle_b200 import ops  # noqa: E402

DEV = torch.device("cuda")


def test_wait_that_nothing_completes_times_out_and_raises():
    ops.check_status(DEV)  # start from a clean word
    assert ops.wait_probe(DEV, 1_000_000) is True
    assert int(ops.status_word(DEV).item()) == 901
    with pytest.raises(L.PeError, match="fault code 901"):
        ops.check_status(DEV)
    assert int(ops.status_word(DEV).item()) == 0  # cleared by the raise
    ops.check_status(DEV)
    # the context is intact: a tensor-core GEMM right after is still exact enough
    g = torch.Generator(device=DEV).manual_seed(3)
    a = torch.randn(512, 256, generator=g, device=DEV).to(torch.bfloat16)
    w = torch.randn(384, 256, generator=g, device=DEV).to(torch.bfloat16)
    out = ops.linear(a, w, algo=L.ALGO_TCGEN05)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    ref = a.float() @ w.float().t()
    assert ((out.float() - ref).norm() / ref.norm()).item() < 5e-3


def test_wait_probe_rejects_out_of_range_limits():
    with pytest.raises(L.PeError):
        ops.wait_probe(DEV, 10)
    with pytest.raises(L.PeError):
        ops.wait_probe(DEV, 100_000_000_000)
