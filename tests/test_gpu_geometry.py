"""Parity at the benchmarked geometry (BASELINE configs 2 and 4), with the
tensor-core kernels compared directly against fp32 references -- never against
another kernel of this library.

* The masked attention of all four config-2 segments (n 2048, K 5, S 4, 28/4
  heads, head_dim 128; up to 4096 slots per segment) through the stacked
  one-launch entry points, against a dense fp32 PyTorch attention with autograd
  on the GPU, per segment and head (reference ``src/pe/nn.py:84-88`` with the
  mask of ``src/pe/masks.py:43-61`` / ``partition.py:41-55``).
* One full config-2 sequence through ``mtp_backward`` against the CPU oracle
  (``oracle.mtp_step``, a restatement of ``src/pe/partition.py:58-118`` pinned to
  the reference's own outputs): loss within 1e-3, every gradient within 2e-2.
* The same step at 14B-class dims (hidden 5120, 40/8 heads, I 13824).
* The sequence-partitioned gradient against the full-sequence gradient at
  head_dim 128, so both run the tcgen05 attention (reference
  ``tests/test_drafter.py:35-54`` states the property).
"""

from __future__ import annotations

import math

import pytest
import torch

from gpu_harness import build_drafter, compare_step, cuda_step, make_case, oracle, recipe

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from parallel_eagle_b200 import _lib as L  # noqa: E402
from parallel_eagle_b200 import ops  # noqa: E402
from parallel_eagle_b200.engine import segment_bounds  # noqa: E402

DEV = torch.device("cuda")
rel = recipe.rel_fro
LOSS_TOL = 1e-3
BF16_TOL = 2e-2  # the north_star's bf16 gradient bar (relative Frobenius)

SEVEN_B = dict(hidden=3584, n_heads=28, n_kv_heads=4, intermediate=18944, vocab=152064,
               num_layers=1, max_depth=5)
FOURTEEN_B = dict(hidden=5120, n_heads=40, n_kv_heads=8, intermediate=13824, vocab=152064,
                  num_layers=1, max_depth=5)


def _dense_segment(q, k, v, do, allow, nh, nkv, hd):
    """fp32 dense masked attention of one segment, head by head, with autograd on
    the GPU.  q/k/v/do are the segment's bf16 rows; returns o, lse [nh, S], dq, dk, dv
    in fp32."""
    S = q.shape[0]
    rep = nh // nkv
    scale = 1.0 / math.sqrt(hd)
    o = torch.empty(S, nh * hd, device=DEV)
    dq = torch.empty(S, nh * hd, device=DEV)
    dk = torch.zeros(S, nkv * hd, device=DEV)
    dv = torch.zeros(S, nkv * hd, device=DEV)
    lse = torch.empty(nh, S, device=DEV)
    neg = torch.zeros(S, S, device=DEV).masked_fill_(~allow, float("-inf"))
    for h in range(nh):
        g = h // rep
        qh = q[:, h * hd:(h + 1) * hd].float().requires_grad_(True)
        kh = k[:, g * hd:(g + 1) * hd].float().requires_grad_(True)
        vh = v[:, g * hd:(g + 1) * hd].float().requires_grad_(True)
        s = (qh @ kh.t()) * scale + neg
        lse[h] = torch.logsumexp(s.detach(), -1)
        oh = torch.softmax(s, -1) @ vh
        oh.backward(do[:, h * hd:(h + 1) * hd].float())
        o[:, h * hd:(h + 1) * hd] = oh.detach()
        dq[:, h * hd:(h + 1) * hd] = qh.grad
        dk[:, g * hd:(g + 1) * hd] += kh.grad
        dv[:, g * hd:(g + 1) * hd] += vh.grad
        del s, oh, qh, kh, vh
    return o, lse, dq, dk, dv


@pytest.mark.parametrize("n,nseg,K,nh,nkv", [(2048, 4, 5, 28, 4), (1000, 3, 8, 8, 2)])
def test_attention_tcgen05_against_dense_fp32(n, nseg, K, nh, nkv):
    """Forward output, lse, dQ, dK and dV of every stacked segment of one sequence
    (config 2: segments of 2560 / 3072 / 3584 / 4096 slots) against fp32 torch."""
    hd = 128
    bounds = segment_bounds(n, nseg)
    rows = ops.segment_rows(bounds, K)
    R = sum(rows)
    cq, ckv = nh * hd, nkv * hd
    g = torch.Generator(device=DEV).manual_seed(2024)
    qkv = torch.randn(R, cq + 2 * ckv, generator=g, device=DEV).to(torch.bfloat16)
    do = torch.randn(R, cq, generator=g, device=DEV).to(torch.bfloat16)
    q, kt, vt = qkv[:, :cq], qkv[:, cq:cq + ckv], qkv[:, cq + ckv:]
    o, lse = ops.attn_fwd_segments(q, kt, vt, nh, nkv, hd, bounds, K, algo=L.ALGO_TCGEN05)
    dqkv = torch.full((R, cq + 2 * ckv), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.attn_bwd_segments(q, kt, vt, o, do, lse, nh, nkv, hd, bounds, K, dq=dqkv[:, :cq],
                          dk=dqkv[:, cq:cq + ckv], dv=dqkv[:, cq + ckv:], algo=L.ALGO_TCGEN05)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    off = 0
    for (a0, a1), S in zip(bounds, rows):
        anc, dep = oracle.segment_slots(a0, a1, K)
        allow = oracle.slot_allow(anc, dep).to(DEV)
        sl = slice(off, off + S)
        ro, rlse, rdq, rdk, rdv = _dense_segment(q[sl], kt[sl], vt[sl], do[sl], allow, nh, nkv, hd)
        got_lse = lse[nh * off: nh * (off + S)].view(nh, S)
        assert torch.allclose(got_lse, rlse, atol=2e-3, rtol=1e-4), (a0, a1)
        for name, got, ref in (("o", o[sl], ro), ("dq", dqkv[sl, :cq], rdq),
                               ("dk", dqkv[sl, cq:cq + ckv], rdk),
                               ("dv", dqkv[sl, cq + ckv:], rdv)):
            assert not torch.isnan(got).any(), (name, a0, a1)
            err = rel(got.float(), ref)
            assert err < BF16_TOL, (name, a0, a1, err)
        off += S


def test_config2_sequence_against_oracle():
    """One BASELINE config-2 sequence (7B-class dims, n 2048, K 5, S 4, bf16) through
    ``mtp_backward`` against the oracle on the host: the benchmarked step itself."""
    case = make_case(**SEVEN_B, n=2048, dtype=torch.bfloat16, seed=0, norm_jitter=0.0)
    res = compare_step(case, num_segments=4)
    assert res["loss_rel"] < LOSS_TOL, res
    worst = max(res["grad_rel"].items(), key=lambda kv: kv[1])
    assert worst[1] < BF16_TOL, worst


@pytest.mark.parametrize("num_segments", [1, 4])
def test_14b_dims_against_oracle(num_segments):
    """BASELINE config-4 dims (hidden 5120, 40/8 heads, I 13824, vocab 152064) at
    n 320: 1600 slots per sequence at S = 1, so attention spans many 128-slot tiles."""
    case = make_case(**FOURTEEN_B, n=320, dtype=torch.bfloat16, seed=1, norm_jitter=0.0)
    res = compare_step(case, num_segments=num_segments)
    assert res["loss_rel"] < LOSS_TOL, res
    worst = max(res["grad_rel"].items(), key=lambda kv: kv[1])
    assert worst[1] < BF16_TOL, worst


def test_soft_target_config3_dims_against_oracle():
    """The soft-target distillation loss at 7B-class dims: the
    teacher-logits GEMM, the joint combine and both row-rescaled dH accumulations of
    the fused LM head, against the oracle's definition of that loss."""
    case = make_case(**SEVEN_B, n=96, dtype=torch.bfloat16, seed=2, norm_jitter=0.0)
    res = compare_step(case, num_segments=2, teacher_hidden_seed=7)
    assert res["loss_rel"] < LOSS_TOL, res
    worst = max(res["grad_rel"].items(), key=lambda kv: kv[1])
    assert worst[1] < BF16_TOL, worst


@pytest.mark.parametrize("num_segments", [2, 4, 7])
def test_partitioned_gradient_equals_full_on_tensor_cores(num_segments):
    """S-partitioned vs full-sequence gradient with head_dim 128 (the tcgen05
    attention kernels) and enough slots per segment for several 128-slot tiles."""
    case = make_case(hidden=1024, n_heads=8, n_kv_heads=2, intermediate=2048, vocab=8192,
                     num_layers=1, max_depth=5, n=700, dtype=torch.bfloat16, seed=11)
    model = build_drafter(case)
    l1, g1, _ = cuda_step(case, drafter=model, num_segments=1)
    ls, gs, _ = cuda_step(case, drafter=model, num_segments=num_segments)
    assert abs(l1[0] - ls[0]) <= LOSS_TOL * abs(l1[0])
    for k in g1:
        assert rel(gs[k], g1[k]) < BF16_TOL, k
