"""Draft-time path on the GPU: ``ParallelDrafter.draft_logits`` /
``draft_logits_sequential`` and the tree / chain proposals.

* fp32 against the reference's own outputs (``tests/golden/*_draft.pt``): logits
  within 1e-4 relative Frobenius, trees and chains token for token.
* bf16 at head_dim 128 (tensor-core attention, partition layout ``(p-1, p, k)``)
  against the CPU oracle within 2e-2.
* The selection kernel against ``log_softmax`` + ``topk`` / ``argmax``.
"""

from __future__ import annotations

import pytest
import torch

from gpu_harness import ROOT, build_drafter, make_case, oracle, recipe

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}
DEV = torch.device("cuda")


def _golden_case(name):
    c = recipe.CASES[name]
    dt = _DT[c["dtype"]]
    case = make_case(c["hidden"], c["n_heads"], c["n_kv_heads"], c["intermediate"], c["vocab"],
                     c["num_layers"], c["max_depth"], c["n"], dtype=dt, seed=c["seed"],
                     norm_jitter=c["norm_jitter"])
    g = torch.load(ROOT / "tests" / "golden" / f"{name}_draft.pt", weights_only=False)
    case["params"] = g["params"]
    return case, g


@pytest.mark.parametrize("name", [n for n, c in recipe.CASES.items() if c["full"]])
def test_draft_path_matches_reference_golden(name):
    from parallel_eagle_b200 import decode

    case, g = _golden_case(name)
    dt = case["dtype"]
    tol = 1e-4 if dt == torch.float32 else 2e-2
    model = build_drafter(case)
    ids, feats = case["seqs"][0]
    ids, feats = ids.to(DEV), feats.to(DEV)
    for rec in g["runs"]:
        run = rec["run"]
        p, k, pend = run["p"], run["k"], run["pending"]
        logits = model.draft_logits(ids[:p], feats[:p], k)
        assert logits.shape == rec["logits"].shape and logits.dtype == rec["logits"].dtype
        assert recipe.rel_fro(logits.float().cpu(), rec["logits"].float()) < tol, run
        if "logits_sequential" in rec:
            seq = model.draft_logits_sequential(ids[:p], feats[:p], k)
            assert recipe.rel_fro(seq.float().cpu(), rec["logits_sequential"].float()) < tol, run
        if dt == torch.float32:
            tree = decode.propose_tree(model, ids[:p], feats[:p], k - pend, run["top_k"],
                                       run["max_nodes"], pending=pend)
            assert tuple(tree) == tuple(rec["tree"]), run
            chain = decode.propose_chain(model, ids[:p], feats[:p], k - pend, pending=pend)
            assert chain == rec["chain"], run


@pytest.mark.parametrize("p,k", [(1, 5), (300, 5), (129, 8), (256, 1)])
def test_draft_logits_tensor_cores_match_oracle(p, k):
    """hidden 256 / 2 query heads / 1 KV head: head_dim 128, so the draft forward's
    attention runs on the tcgen05 kernels with the partition layout (p-1, p, k)."""
    case = make_case(256, 2, 1, 512, 1000, 1, 5, 300, dtype=torch.bfloat16, seed=7)
    model = build_drafter(case)
    ids, feats = case["seqs"][0]
    got = model.draft_logits(ids[:p].to(DEV), feats[:p].to(DEV), k)
    torch.cuda.synchronize()
    ref = oracle.draft_logits(case["params"], case["heads"], ids[:p], feats[:p], k, case["dims"])
    assert got.shape == (k, 1000)
    assert recipe.rel_fro(got.float().cpu(), ref.float()) < 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,V,k", [(5, 152064, 8), (3, 1000, 1), (2, 7, 7)])
def test_topk_logprobs_matches_torch(dtype, rows, V, k):
    from parallel_eagle_b200 import ops

    g = torch.Generator().manual_seed(rows * 31 + V)
    z = (torch.randn(rows, V, generator=g) * 3).to(dtype)
    vals, idx = ops.topk_logprobs(z.to(DEV), k)
    lp = torch.log_softmax(z.float(), dim=-1)
    for r in range(rows):
        rv, ri = lp[r].topk(k)
        assert torch.allclose(vals[r].cpu(), rv, atol=1e-5, rtol=1e-6), r
        # the selected columns carry the selected values (ties may swap columns)
        assert torch.allclose(lp[r][idx[r].cpu()], vals[r].cpu(), atol=1e-5, rtol=1e-6), r
        assert len(set(idx[r].tolist())) == k
    am_val, am = ops.topk_logprobs(z.to(DEV), 1, raw=True)
    assert torch.equal(am[:, 0].cpu(), z.float().argmax(-1))
    assert torch.equal(am_val[:, 0].cpu(), z.float().max(-1).values)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,V,temp", [(5, 152064, 0.7), (3, 1000, 1.0), (2, 7, 1.6)])
def test_softmax_rows_matches_torch(dtype, rows, V, temp):
    from parallel_eagle_b200 import ops

    g = torch.Generator().manual_seed(rows * 17 + V)
    z = (torch.randn(rows, V, generator=g) * 3).to(dtype)
    q = ops.softmax_rows(z.to(DEV), temp)
    x = z.float() / temp  # the reference's fp32 division
    exact = torch.softmax(x.double(), dim=-1).float()
    ref = torch.softmax(x, dim=-1)
    assert q.dtype == torch.float32 and q.shape == (rows, V)
    # the kernel sums the row in fp64, so it sits within a few ulp of the exact softmax;
    # torch's own fp32 reduction over up to 152K terms is off by ~1.5e-5 relative
    assert torch.allclose(q.cpu(), exact, rtol=2e-6, atol=1e-12)
    assert torch.allclose(q.cpu(), ref, rtol=3e-5, atol=1e-10)
    assert torch.allclose(q.sum(-1).cpu(), torch.ones(rows), atol=1e-5)


def test_propose_chain_sampling_matches_reference_draw():
    """Reference chain.py:38-53: q = softmax(draft_logits.float() / T), tokens drawn by
    torch.multinomial with the caller's generator -- the same seed gives the same chain."""
    from parallel_eagle_b200 import decode

    case = make_case(256, 2, 1, 512, 1000, 1, 5, 300, dtype=torch.bfloat16, seed=7)
    model = build_drafter(case)
    ids, feats = case["seqs"][0]
    ids, feats = ids[:120].to(DEV), feats[:120].to(DEV)
    for temp, seed in ((0.8, 1), (1.3, 2)):
        toks, q = decode.propose_chain_sampling(model, ids, feats, 5, temp,
                                                generator=torch.Generator(device=DEV).manual_seed(seed))
        logits = model.draft_logits(ids, feats, 5)
        ref_q = torch.softmax(logits.float() / temp, dim=-1)
        assert torch.allclose(q, ref_q, rtol=1e-5, atol=1e-10)
        # the draw: torch.multinomial on the returned q with the caller's seeded
        # generator (drawing on torch's own softmax instead could flip a token whose
        # cumulative probability sits within the two q's 1e-5 of a draw boundary)
        ref = torch.multinomial(q, 1, generator=torch.Generator(device=DEV).manual_seed(seed))
        assert toks == [int(t) for t in ref.squeeze(-1).tolist()]
        assert len(toks) == 5 and all(0 <= t < 1000 for t in toks)


def test_verification_rules_match_reference_golden():
    """Draft acceptance (reference pe.decode.verify) with the target's logits on the
    GPU: the greedy and cached rules reproduce the reference's decisions in
    ``verify_cases.pt``; sampled acceptance matches the oracle draw for draw under the
    same seeded CUDA generator."""
    from oracle import verify as ov

    from parallel_eagle_b200 import decode

    cases = torch.load(ROOT / "tests" / "golden" / "verify_cases.pt", weights_only=False)
    for c in cases:
        P, k = c["prefix_len"], len(c["draft"])
        lg, tl = c["logits"].to(DEV), c["tree_logits"].to(DEV)
        assert decode.accept_chain_greedy(lg, P, c["draft"]) == c["chain"]
        _, bonus_bf16 = decode.accept_chain_greedy(lg.bfloat16(), P, c["draft"])  # bf16 dispatch
        assert 0 <= bonus_bf16 < lg.shape[1]
        assert decode.accept_chain_cached(lg[P - 1], lg[P:P + k], c["draft"]) == c["chain_cached"]
        assert decode.accept_tree_greedy(tl, P, c["node_tokens"], c["parents"]) == c["tree"]
        assert decode.accept_tree_cached(tl[P - 1], tl[P:], c["node_tokens"],
                                         c["parents"]) == c["tree_cached"]
        td, qd = c["target_dists"].to(DEV), c["q_dists"].to(DEV)
        got = decode.accept_chain_sampling(td, c["sample_draft"], qd,
                                           generator=torch.Generator(device=DEV).manual_seed(c["seed"]))
        ref = ov.accept_chain_sampling(td, c["sample_draft"], qd,
                                       generator=torch.Generator(device=DEV).manual_seed(c["seed"]))
        assert got == ref


def test_argmax_and_topk_rank_nan_like_torch():
    """NaN ranks above every number (torch.argmax / torch.topk): a row with NaNs
    selects its first NaN column, an all-NaN row its first columns -- never an
    out-of-range index.  float64 target logits are rejected, not rounded."""
    from parallel_eagle_b200 import _lib as L
    from parallel_eagle_b200 import decode, ops

    z = torch.randn(3, 1000, generator=torch.Generator().manual_seed(4))
    z[0, 9] = float("nan")
    z[0, 5] = float("nan")
    z[1, :] = float("nan")
    for dt in (torch.float32, torch.bfloat16):
        _, idx = ops.topk_logprobs(z.to(dt).to(DEV), 3, raw=True)
        idx = idx.cpu()
        zr = z.to(dt).float()
        assert idx[0].tolist() == [5, 9, int(zr[0].nan_to_num(-1e9).argmax())]
        assert idx[1].tolist() == [0, 1, 2]
        assert zr[2][idx[2]].tolist() == torch.topk(zr[2], 3).values.tolist()
        assert int(idx[0, 0]) == int(torch.argmax(zr[0]))
        assert decode._argmax_rows(z.to(dt).to(DEV)) == [5, 0, int(torch.argmax(z[2].to(dt)))]
    with pytest.raises(L.PeError):
        decode._argmax_rows(z.double().to(DEV))
