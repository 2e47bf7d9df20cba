"""Generate golden vectors by running the reference implementation itself.

Run from the repository root in a checkout that has the reference project
available (its ``src`` directory importable as ``pe``)::

    PE_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py [--draft | --verify]

For every case in ``recipe.CASES`` this builds the reference ``ParallelDrafter``
from seeded synthetic frozen heads, runs the reference ``mtp_backward`` (and
``mtp_eval_loss`` / ``forward``) and writes ``tests/golden/<case>.pt`` with the
losses, the accumulated gradients (full tensors for the tiny cases, random-
projection sketches for the larger one) and checksums of every input.  For the
cases that store full tensors it also writes ``<case>_draft.pt`` with the
reference's draft-time outputs (``--draft`` writes only those).  ``--verify``
writes ``verify_cases.pt``: the reference's draft acceptance decisions
(``pe.decode.verify``) on seeded target outputs.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import recipe  # noqa: E402

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _reference():
    src = os.environ.get("PE_REFERENCE_SRC")
    if not src:
        raise SystemExit("set PE_REFERENCE_SRC to the reference project's src directory")
    sys.path.insert(0, src)
    import pe.drafter
    import pe.nn
    import pe.partition

    return pe


def _heads_object(pe, c, heads):
    """The minimal target-heads surface ``ParallelDrafter.from_target`` reads."""
    H, V = c["hidden"], c["vocab"]
    embed = torch.nn.Embedding(V, H)
    embed.weight.data = heads["embed"].clone()
    head = torch.nn.Linear(H, V, bias=False)
    head.weight.data = heads["head"].clone()
    norm = pe.nn.RMSNorm(H, 1e-5)
    norm.weight.data = heads["norm"].clone()
    for m in (embed, head, norm):
        for p in m.parameters():
            p.requires_grad_(False)
    cfg = types.SimpleNamespace(
        num_attention_heads=c["n_heads"], num_key_value_heads=c["n_kv_heads"],
        intermediate_size=c["intermediate"], rope_theta=10000.0, rms_norm_eps=1e-5,
        hidden_size=H, vocab_size=V,
    )
    return types.SimpleNamespace(
        config=cfg, hidden_size=H, vocab_size=V, feature_dim=3 * H,
        get_input_embeddings=lambda: embed, get_lm_head=lambda: head,
        get_final_norm=lambda: norm,
    )


def build_case(pe, name: str, c: dict) -> dict:
    from pe.config import DrafterConfig
    from pe.drafter import ParallelDrafter
    from pe.partition import mtp_backward, mtp_eval_loss

    dt = _DT[c["dtype"]]
    heads = recipe.make_heads(c["vocab"], c["hidden"], c["seed"], c["norm_jitter"], dt)
    target = _heads_object(pe, c, heads)
    torch.manual_seed(c["seed"])
    drafter = ParallelDrafter.from_target(
        target, DrafterConfig(num_layers=c["num_layers"], max_depth=c["max_depth"])
    ).to(dtype=dt)
    drafter.train()
    params = {k: v.detach().clone() for k, v in drafter.state_dict().items()}
    batch = c.get("batch", 1)
    seqs = [recipe.make_sequence(c["n"], c["vocab"], 3 * c["hidden"], c["seed"], b) for b in range(batch)]

    out = {"case": name, "config": {k: v for k, v in c.items() if k != "runs"}, "runs": []}
    out["input_checksum"] = {
        "ids": [int(ids.sum()) for ids, _ in seqs],
        "feats": [float(f.double().sum()) for _, f in seqs],
        "feats_sketch": [recipe.sketch(f, 1) for _, f in seqs],
    }
    if c["full"]:
        out["params"] = params
    else:
        out["param_sketch"] = {k: recipe.sketch(v, i) for i, (k, v) in enumerate(params.items())}
        out["param_sum"] = {k: float(v.double().sum()) for k, v in params.items()}

    for run in c["runs"]:
        drafter.zero_grad(set_to_none=True)
        losses = []
        for ids, feats in seqs:
            kw = dict(
                num_segments=run["num_segments"],
                loss_scale=run.get("loss_scale", 1.0 / batch),
                prompt_len=run.get("prompt_len", 0),
            )
            if run.get("teacher_labels"):
                kw["teacher_labels"] = recipe.teacher_labels_for(ids)
            losses.append(mtp_backward(drafter, ids, feats.to(dt), **kw))
        grads = {k: p.grad.detach().clone() for k, p in drafter.named_parameters() if p.grad is not None}
        rec = {"run": run, "losses": losses}
        if c["full"]:
            rec["grads"] = grads
        else:
            rec["grad_sketch"] = {
                k: recipe.sketch(g, 100 + i) for i, (k, g) in enumerate(grads.items())
            }
            rec["grad_norm"] = {k: float(g.double().norm()) for k, g in grads.items()}
        out["runs"].append(rec)

    ids, feats = seqs[0]
    out["eval_loss"] = mtp_eval_loss(drafter, ids, feats.to(dt))
    if c["full"]:
        # generic forward with an explicit additive bias: the anchor-major packing
        with torch.no_grad():
            x, pos, bias, labels = drafter.build_training_packed(ids, feats.to(dt))
            out["packed"] = {
                "x": x.clone(), "pos": pos.clone(), "bias": bias.clone(), "labels": labels.clone(),
                "hidden": drafter(x, pos, bias).clone(),
            }
    return out


def build_draft_case(pe, name: str, c: dict) -> dict:
    """Draft-time outputs of the reference on the same seeded drafter:
    ``draft_logits`` (src/pe/drafter.py:195-236), ``draft_logits_sequential``
    (:239-269), ``propose_tree`` (src/pe/decode/tree.py:19-57) and ``propose_chain``
    (src/pe/decode/chain.py:15-23) for every entry of ``recipe.DRAFT_RUNS``."""
    from pe.config import DrafterConfig
    from pe.decode.chain import propose_chain
    from pe.decode.tree import propose_tree
    from pe.drafter import ParallelDrafter

    dt = _DT[c["dtype"]]
    heads = recipe.make_heads(c["vocab"], c["hidden"], c["seed"], c["norm_jitter"], dt)
    target = _heads_object(pe, c, heads)
    torch.manual_seed(c["seed"])
    drafter = ParallelDrafter.from_target(
        target, DrafterConfig(num_layers=c["num_layers"], max_depth=c["max_depth"])
    ).to(dtype=dt)
    drafter.eval()
    ids, feats = recipe.make_sequence(c["n"], c["vocab"], 3 * c["hidden"], c["seed"], 0)
    feats = feats.to(dt)
    out = {"case": name, "params": {k: v.detach().clone() for k, v in drafter.state_dict().items()},
           "runs": []}
    for run in recipe.DRAFT_RUNS:
        p, k = run["p"], run["k"]
        rec = {"run": dict(run)}
        with torch.no_grad():
            rec["logits"] = drafter.draft_logits(ids[:p], feats[:p], k).clone()
            if run.get("sequential"):
                rec["logits_sequential"] = drafter.draft_logits_sequential(ids[:p], feats[:p], k).clone()
            kt, pend = k - run["pending"], run["pending"]
            rec["tree"] = propose_tree(drafter, ids[:p], feats[:p], kt, run["top_k"],
                                       run["max_nodes"], pending=pend)
            rec["chain"] = propose_chain(drafter, ids[:p], feats[:p], kt, pending=pend)
        out["runs"].append(rec)
    return out


def build_verify_cases() -> list[dict]:
    """Seeded target outputs over drafted chains / trees and the reference's
    acceptance decisions for them (pe.decode.verify): greedy and cached forms on
    logits whose argmax the drafts follow for a varying prefix / share of nodes, and
    speculative-sampling acceptance with a seeded CPU generator."""
    from pe.decode import verify as ver

    g = torch.Generator().manual_seed(123)
    V = 50
    cases = []
    for ci in range(12):
        P, k, T = 1 + ci, 1 + ci % 5, 3 + ci
        logits = torch.randn(P + k, V, generator=g)
        top = logits.argmax(-1)
        a = ci % (k + 1)  # drafts that follow the target
        draft = [int(top[P - 1 + m]) if m < a else int((top[P - 1 + m] + 1) % V) for m in range(k)]
        parents = [-1 if t == 0 else int(torch.randint(-1, t, (1,), generator=g)) for t in range(T)]
        tlog = torch.randn(P + T, V, generator=g)
        ttop = tlog.argmax(-1)
        nodes = []
        for t, par in enumerate(parents):
            pos = P - 1 if par < 0 else P + par
            follow = float(torch.rand((), generator=g)) < 0.6
            nodes.append(int(ttop[pos]) if follow else int(torch.randint(0, V, (1,), generator=g)))
        tdist = torch.softmax(torch.randn(k + 1, V, generator=g), -1)
        qdist = torch.softmax(torch.randn(k, V, generator=g), -1)
        sdraft = [int(torch.multinomial(qdist[i], 1, generator=g)) for i in range(k)]
        seed = 1000 + ci
        cases.append({
            "prefix_len": P, "logits": logits, "draft": draft,
            "chain": ver.accept_chain_greedy(logits, P, draft),
            "chain_cached": ver.accept_chain_cached(logits[P - 1], logits[P:P + k], draft),
            "tree_logits": tlog, "parents": parents, "node_tokens": nodes,
            "tree": ver.accept_tree_greedy(tlog, P, nodes, parents),
            "tree_cached": ver.accept_tree_cached(tlog[P - 1], tlog[P:], nodes, parents),
            "target_dists": tdist, "q_dists": qdist, "sample_draft": sdraft, "seed": seed,
            "sampling": ver.accept_chain_sampling(tdist, sdraft, qdist,
                                                  generator=torch.Generator().manual_seed(seed)),
        })
    return cases


def main():
    pe = _reference()
    if "--verify" in sys.argv[1:]:
        cases = build_verify_cases()
        torch.save(cases, HERE / "verify_cases.pt")
        print("verify", [(c["chain"], c["tree"], c["sampling"]) for c in cases[:3]])
        return
    draft_only = "--draft" in sys.argv[1:]
    for name, c in recipe.CASES.items():
        if not draft_only:
            rec = build_case(pe, name, c)
            torch.save(rec, HERE / f"{name}.pt")
            print(name, [r["losses"] for r in rec["runs"]], "eval", rec["eval_loss"])
        if c["full"]:
            rec = build_draft_case(pe, name, c)
            torch.save(rec, HERE / f"{name}_draft.pt")
            print(name, "draft", [r["tree"] for r in rec["runs"]])


if __name__ == "__main__":
    main()
