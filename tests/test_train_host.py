"""The training loop's host logic on the CPU: checkpoint/resume after a simulated
preemption, re-entry of a finished run, config-signature mismatch (reference
tests/test_train_resume.py), and data-parallel equivalence over two gloo ranks.

The loop's compute step (``mtp_backward``) and optimizer are replaced by the CPU
oracle and torch AdamW here -- the CUDA path is exercised by the ``gpu`` tests;
these tests pin the bookkeeping around it.
"""

from __future__ import annotations

import json
import os
import sys
import types
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import oracle  # noqa: E402
from parallel_eagle_b200 import target as target_mod  # noqa: E402
from parallel_eagle_b200 import train as train_mod  # noqa: E402
from parallel_eagle_b200.config import DrafterConfig, TargetConfig, TrainConfig  # noqa: E402

H, V = 32, 64


def tiny_heads():
    g = torch.Generator().manual_seed(0)
    cfg = types.SimpleNamespace(hidden_size=H, vocab_size=V, num_attention_heads=4,
                                num_key_value_heads=2, intermediate_size=64, rope_theta=10000.0,
                                rms_norm_eps=1e-5, num_hidden_layers=4)
    return target_mod._heads_from_weights(
        cfg, torch.randn(V, H, generator=g) * 0.02, torch.randn(V, H, generator=g) * 0.02,
        torch.ones(H), (1, 2, 3), "cpu", torch.float32)


def oracle_step(drafter, input_ids, features, num_segments=1, loss_scale=1.0, prompt_len=0,
                teacher_labels=None, teacher_hidden=None):
    """CPU stand-in for mtp_backward with the same contract (adds into p.grad)."""
    dims = oracle.OracleDims(hidden=drafter.hidden, n_heads=drafter.n_heads,
                             n_kv_heads=drafter.n_kv_heads, intermediate=drafter.intermediate,
                             vocab=drafter.vocab, num_layers=len(drafter.layers),
                             max_depth=drafter.max_depth)
    params = {n: p.detach() for n, p in drafter.named_parameters()}
    heads = {"embed": drafter._embed[0].weight.detach(), "head": drafter._lm_head[0].weight.detach(),
             "norm": drafter._final_norm[0].weight.detach()}
    loss, grads = oracle.mtp_step(params, heads, input_ids, features.float(), dims, num_segments,
                                  loss_scale, prompt_len, teacher_labels)
    for n, p in drafter.named_parameters():
        p.grad = grads[n].clone() if p.grad is None else p.grad + grads[n]
    return loss


def build_cache(cache_dir: Path, n=16, seq_len=20, prompt_len=4):
    cache_dir.mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(0)
    buf = []
    for _ in range(n):
        ids = torch.randint(0, V, (seq_len,), generator=g)
        buf.append({"input_ids": ids,
                    "features": torch.randn(seq_len, 3 * H, generator=g).to(torch.float16),
                    "prompt_len": prompt_len,
                    "labels": torch.randint(0, V, (seq_len,), generator=g)})
    torch.save(buf, cache_dir / "shard_00000.pt")
    (cache_dir / "manifest.json").write_text(json.dumps({
        "shards": ["shard_00000.pt"], "num_examples": n, "feature_dim": 3 * H,
        "feature_layers": [1, 2, 3], "self_distilled": True}))


def patch(monkeypatch):
    monkeypatch.setattr(train_mod, "load_target_heads", lambda tcfg: tiny_heads())
    monkeypatch.setattr(train_mod, "mtp_backward", oracle_step)
    monkeypatch.setattr(train_mod, "build_optimizer",
                        lambda params, lr, wd, use_8bit, max_norm=1.0: torch.optim.AdamW(params, lr=lr, weight_decay=wd))


def cfgs(cache, out):
    tcfg = TargetConfig(model_name="tiny", device="cpu", dtype="float32")
    tr = TrainConfig(feature_cache_dir=cache, out_dir=out, epochs=2, grad_accum=2, max_seq_len=64,
                     use_8bit_adam=False, grad_checkpoint=False, save_every=2, log_every=100)
    return tcfg, tr


def test_resume_continues_from_checkpoint(tmp_path, monkeypatch, capsys):
    patch(monkeypatch)
    cache, out = tmp_path / "cache", tmp_path / "ck"
    build_cache(cache)
    tcfg, tr = cfgs(cache, out)
    dcfg = DrafterConfig(num_layers=2, max_depth=4)

    class Preempted(Exception):
        pass

    calls = {"n": 0}

    def boom():
        calls["n"] += 1
        if calls["n"] >= 2:
            raise Preempted

    with pytest.raises(Preempted):
        train_mod.train(tcfg, dcfg, tr, dtype="float32", on_save=boom)
    state = torch.load(out / "train_state.pt", weights_only=False)
    assert (out / "drafter.pt").exists()
    assert 0 < state["update"] < 16 and state["epoch"] < tr.epochs
    resumed = state["update"]
    capsys.readouterr()
    train_mod.train(tcfg, dcfg, tr, dtype="float32", on_save=lambda: None)
    txt = capsys.readouterr().out
    assert f"resuming: epoch {state['epoch']}" in txt
    assert f"update {resumed}/16" in txt
    assert torch.load(out / "train_state.pt", weights_only=False)["epoch"] == tr.epochs
    # checkpoint layout: the reference keys, loadable by load_drafter
    from parallel_eagle_b200.drafter import load_drafter

    ck = torch.load(out / "drafter.pt", weights_only=False)
    assert set(ck) == {"state_dict", "num_layers", "max_depth", "target_name"}
    assert list(ck["state_dict"]) == oracle.param_names(2)
    assert len(load_drafter(out / "drafter.pt", tiny_heads()).layers) == 2


def test_completed_run_is_a_noop_on_reentry(tmp_path, monkeypatch, capsys):
    patch(monkeypatch)
    cache, out = tmp_path / "cache", tmp_path / "ck"
    build_cache(cache)
    tcfg, tr = cfgs(cache, out)
    dcfg = DrafterConfig(num_layers=2, max_depth=4)
    train_mod.train(tcfg, dcfg, tr, dtype="float32")
    capsys.readouterr()
    train_mod.train(tcfg, dcfg, tr, dtype="float32")
    txt = capsys.readouterr().out
    assert "resuming: epoch 2" in txt and "after epoch" not in txt


def test_mismatched_config_starts_fresh(tmp_path, monkeypatch, capsys):
    patch(monkeypatch)
    cache, out = tmp_path / "cache", tmp_path / "ck"
    build_cache(cache)
    tcfg, tr = cfgs(cache, out)
    train_mod.train(tcfg, DrafterConfig(num_layers=2, max_depth=4), tr, dtype="float32")
    capsys.readouterr()
    train_mod.train(tcfg, DrafterConfig(num_layers=3, max_depth=4), tr, dtype="float32")
    assert "different run — starting fresh" in capsys.readouterr().out


def test_missing_cache_and_checkpoint_raise_with_hint(tmp_path):
    from parallel_eagle_b200.drafter import load_drafter
    from parallel_eagle_b200.features import FeatureDataset

    with pytest.raises(FileNotFoundError, match="manifest.json"):
        FeatureDataset(tmp_path / "nope")
    with pytest.raises(FileNotFoundError, match="Train one first"):
        load_drafter(tmp_path / "nope.pt", tiny_heads())


# ------------------------------------------------------------------ gloo DP ----


def _dp_worker(rank, world, port, cache, out, result_path, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=20))
    import parallel_eagle_b200.train as tm

    tm.load_target_heads = lambda tcfg: tiny_heads()
    tm.mtp_backward = oracle_step
    tm.build_optimizer = lambda params, lr, wd, use_8bit, max_norm=1.0: torch.optim.AdamW(params, lr=lr, weight_decay=wd)
    if rank == fail_rank:
        def broken(*a, **k):
            raise RuntimeError("injected rank failure")
        tm.mtp_backward = broken
    tcfg = TargetConfig(model_name="tiny", device="cpu", dtype="float32")
    tr = TrainConfig(feature_cache_dir=Path(cache), out_dir=Path(out), epochs=1, grad_accum=4,
                     max_seq_len=64, use_8bit_adam=False, save_every=0, log_every=100)
    try:
        d = tm.train(tcfg, DrafterConfig(num_layers=1, max_depth=3), tr, dtype="float32")
        if rank == 0:
            torch.save({k: v.clone() for k, v in d.state_dict().items()}, result_path)
        status = "ok"
    except Exception as exc:  # noqa: BLE001
        status = f"error: {type(exc).__name__}: {exc}"
    Path(f"{result_path}.rank{rank}").write_text(status)
    if status == "ok":
        torch.distributed.destroy_process_group()


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _single_process(cache, out, monkeypatch):
    patch(monkeypatch)
    tcfg = TargetConfig(model_name="tiny", device="cpu", dtype="float32")
    tr = TrainConfig(feature_cache_dir=cache, out_dir=out, epochs=1, grad_accum=4, max_seq_len=64,
                     use_8bit_adam=False, save_every=0, log_every=100)
    d = train_mod.train(tcfg, DrafterConfig(num_layers=1, max_depth=3), tr, dtype="float32")
    return {k: v.clone() for k, v in d.state_dict().items()}


def test_data_parallel_two_gloo_ranks_match_single_process(tmp_path, monkeypatch):
    import torch.multiprocessing as mp

    cache = tmp_path / "cache"
    build_cache(cache, n=8)
    ref = _single_process(cache, tmp_path / "single", monkeypatch)
    res = tmp_path / "dp.pt"
    mp.start_processes(_dp_worker, args=(2, _free_port(), str(cache), str(tmp_path / "dp"),
                                         str(res), -1), nprocs=2, start_method="spawn", join=True)
    assert Path(f"{res}.rank0").read_text() == "ok" and Path(f"{res}.rank1").read_text() == "ok"
    got = torch.load(res, weights_only=False)
    for k in ref:
        assert torch.allclose(got[k], ref[k], atol=1e-6, rtol=1e-5), k


def test_failed_rank_surfaces_as_error_on_the_other_rank(tmp_path):
    import torch.multiprocessing as mp

    cache = tmp_path / "cache"
    build_cache(cache, n=8)
    res = tmp_path / "dp.pt"
    ctx = mp.start_processes(_dp_worker, args=(2, _free_port(), str(cache), str(tmp_path / "dp"),
                                               str(res), 1), nprocs=2, start_method="spawn",
                             join=False)
    while not ctx.join(timeout=120):
        pass
    assert "injected rank failure" in Path(f"{res}.rank1").read_text()
    # rank 0 never sees its partner's gradient: the collective ends in an error
    # (connection closed or process-group timeout), not a hang
    assert Path(f"{res}.rank0").read_text().startswith("error")
