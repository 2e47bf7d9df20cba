"""Training-step parity on the GPU.

* fp32 mode against the reference's own golden vectors (``tests/golden``):
  every drafter gradient within 1e-4 relative Frobenius, loss within 1e-3.
* bf16 mode against the CPU oracle (which restates the reference's bf16
  rounding points): gradients within 2e-2, loss within 1e-3.
* Size-independent properties at larger sizes: the sequence-partitioned
  gradient equals the full-sequence gradient; teacher-label equivalence.
"""

from __future__ import annotations

import pytest
import torch

from gpu_harness import ROOT, build_drafter, compare_step, cuda_step, make_case, oracle, recipe

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}
LOSS_TOL = 1e-3


def _golden(name):
    return torch.load(ROOT / "tests" / "golden" / f"{name}.pt", weights_only=False)


def _golden_case(g):
    c = g["config"]
    dt = _DT[c["dtype"]]
    case = make_case(c["hidden"], c["n_heads"], c["n_kv_heads"], c["intermediate"], c["vocab"],
                     c["num_layers"], c["max_depth"], c["n"], dtype=dt, seed=c["seed"],
                     batch=c.get("batch", 1), norm_jitter=c["norm_jitter"])
    if "params" in g:
        case["params"] = g["params"]
    # the golden inputs were fp32 features cast to the run dtype
    return case


@pytest.mark.parametrize("name", list(recipe.CASES))
def test_step_matches_reference_golden(name):
    g = _golden(name)
    case = _golden_case(g)
    dt = case["dtype"]
    grad_tol = 1e-4 if dt == torch.float32 else 2e-2
    model = build_drafter(case)
    for rec in g["runs"]:
        run = dict(rec["run"])
        kw = dict(num_segments=run["num_segments"], prompt_len=run.get("prompt_len", 0))
        if "loss_scale" in run:
            kw["loss_scale"] = run["loss_scale"]
        if run.get("teacher_labels"):
            kw["teacher_labels_self"] = True
        losses, grads, model = cuda_step(case, drafter=model, **kw)
        for a, b in zip(losses, rec["losses"]):
            assert abs(a - b) <= LOSS_TOL * abs(b), (run, a, b)
        if "grads" in rec:
            assert grads.keys() == rec["grads"].keys()
            for k, ref in rec["grads"].items():
                assert recipe.rel_fro(grads[k], ref.float()) < grad_tol, (run, k)
        else:
            for i, (k, s) in enumerate(rec["grad_sketch"].items()):
                assert recipe.rel_fro(recipe.sketch(grads[k], 100 + i), s) < grad_tol, (run, k)


@pytest.mark.parametrize("name", [n for n, c in recipe.CASES.items() if c["full"]])
def test_forward_and_eval_loss_match_reference_golden(name):
    from parallel_eagle_b200.partition import mtp_eval_loss

    g = _golden(name)
    case = _golden_case(g)
    model = build_drafter(case)
    pk = g["packed"]
    with torch.no_grad():
        out = model(pk["x"].cuda(), pk["pos"].cuda(), pk["bias"].cuda())
    tol = 1e-5 if case["dtype"] == torch.float32 else 2e-2
    assert recipe.rel_fro(out[0].float().cpu(), pk["hidden"][0].float()) < tol
    ids, feats = case["seqs"][0]
    ev = mtp_eval_loss(model, ids, feats)
    assert abs(ev - g["eval_loss"]) <= LOSS_TOL * abs(g["eval_loss"])


SEVEN_B = dict(hidden=3584, n_heads=28, n_kv_heads=4, intermediate=18944, vocab=152064,
               num_layers=1, max_depth=5)


@pytest.mark.parametrize("num_segments", [1, 2])
def test_7b_dims_bf16_against_oracle(num_segments):
    case = make_case(**SEVEN_B, n=24, dtype=torch.bfloat16, seed=0, norm_jitter=0.0)
    res = compare_step(case, num_segments=num_segments)
    assert res["loss_rel"] < LOSS_TOL, res
    worst = max(res["grad_rel"].items(), key=lambda kv: kv[1])
    assert worst[1] < 2e-2, worst


def test_bf16_variants_against_oracle():
    case = make_case(hidden=256, n_heads=4, n_kv_heads=2, intermediate=512, vocab=2048,
                     num_layers=2, max_depth=5, n=60, dtype=torch.bfloat16, seed=3)
    for kw in (dict(num_segments=3, prompt_len=11), dict(num_segments=2, teacher_labels_self=True),
               dict(num_segments=2, teacher_hidden_seed=99), dict(num_segments=4, loss_scale=0.3)):
        res = compare_step(case, **kw)
        assert res["loss_rel"] < LOSS_TOL, (kw, res)
        assert max(res["grad_rel"].values()) < 2e-2, (kw, res)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_partitioned_gradient_equals_full_gradient(dtype):
    case = make_case(hidden=512, n_heads=8, n_kv_heads=2, intermediate=1024, vocab=4096,
                     num_layers=1, max_depth=5, n=300, dtype=dtype, seed=5)
    model = build_drafter(case)
    l1, g1, _ = cuda_step(case, drafter=model, num_segments=1)
    l4, g4, _ = cuda_step(case, drafter=model, num_segments=4)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-4
    assert abs(l1[0] - l4[0]) <= LOSS_TOL * abs(l1[0])
    for k in g1:
        assert recipe.rel_fro(g4[k], g1[k]) < tol, k


def test_teacher_labels_equal_next_token_when_self_consistent():
    case = make_case(hidden=128, n_heads=4, n_kv_heads=2, intermediate=256, vocab=512,
                     num_layers=1, max_depth=4, n=40, dtype=torch.bfloat16, seed=7)
    model = build_drafter(case)
    base, gb, _ = cuda_step(case, drafter=model, num_segments=2)
    tl, gt, _ = cuda_step(case, drafter=model, num_segments=2, teacher_labels_self=True)
    assert abs(base[0] - tl[0]) < 1e-5
    for k in gb:
        assert torch.equal(gb[k], gt[k]), k


def test_grads_accumulate_across_calls_and_none_grads_restart():
    case = make_case(hidden=64, n_heads=4, n_kv_heads=2, intermediate=128, vocab=256,
                     num_layers=1, max_depth=3, n=20, dtype=torch.float32, seed=8)
    from parallel_eagle_b200.partition import mtp_backward

    model = build_drafter(case)
    ids, feats = case["seqs"][0]
    model.zero_grad(set_to_none=True)
    mtp_backward(model, ids, feats)
    once = {n: p.grad.clone() for n, p in model.named_parameters()}
    mtp_backward(model, ids, feats)
    for n, p in model.named_parameters():
        assert recipe.rel_fro(p.grad.cpu(), 2 * once[n].cpu()) < 1e-5, n
    model.zero_grad(set_to_none=True)
    mtp_backward(model, ids, feats)
    for n, p in model.named_parameters():
        assert recipe.rel_fro(p.grad.cpu(), once[n].cpu()) < 1e-6, n


def test_cpu_tensors_fail_loudly():
    from parallel_eagle_b200._lib import PeError
    from parallel_eagle_b200.partition import mtp_backward

    case = make_case(hidden=64, n_heads=4, n_kv_heads=2, intermediate=128, vocab=256,
                     num_layers=1, max_depth=3, n=10, dtype=torch.float32, seed=9)
    model = build_drafter(case, device="cpu")
    ids, feats = case["seqs"][0]
    with pytest.raises(PeError):
        mtp_backward(model, ids, feats)
    assert oracle is not None
