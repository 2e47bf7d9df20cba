"""``parallel_eagle_b200.train.train`` itself on the GPU: the loop a user calls,
with the real step engine, the fused clip + AdamW kernel (``FusedAdamW``) and
pinned feature shards, against the same loop on the CPU with the oracle step,
``torch.nn.utils.clip_grad_norm_(1.0)`` and ``torch.optim.AdamW`` -- the
reference's own update (``src/pe/train.py:131-160``).

The cache is a small on-disk shard in the reference's format (fp16 features,
``src/pe/features.py:116-157``); the frozen heads come from a seeded stand-in
for the target (``target.py:255-281`` placement).
"""

from __future__ import annotations

import json
import re
import types
from pathlib import Path

import pytest
import torch

from gpu_harness import oracle, recipe

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from parallel_eagle_b200 import target as target_mod  # noqa: E402
from parallel_eagle_b200 import train as train_mod  # noqa: E402
from parallel_eagle_b200.config import DrafterConfig, TargetConfig, TrainConfig  # noqa: E402

_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _heads(dims, device, dtype):
    H, V = dims["hidden"], dims["vocab"]
    g = torch.Generator().manual_seed(0)
    cfg = types.SimpleNamespace(hidden_size=H, vocab_size=V, num_attention_heads=dims["heads"],
                                num_key_value_heads=dims["kv_heads"],
                                intermediate_size=dims["intermediate"], rope_theta=10000.0,
                                rms_norm_eps=1e-5, num_hidden_layers=4)
    return target_mod._heads_from_weights(
        cfg, torch.randn(V, H, generator=g) * 0.02, torch.randn(V, H, generator=g) * 0.02,
        torch.ones(H), (1, 2, 3), device, dtype)


def _build_cache(cache: Path, dims, n_examples, seq_len, prompt_len):
    cache.mkdir(parents=True, exist_ok=True)
    H, V = dims["hidden"], dims["vocab"]
    g = torch.Generator().manual_seed(1)
    buf = []
    for i in range(n_examples):
        n = seq_len - (i % 3) * 5  # ragged lengths, as real caches are
        buf.append({"input_ids": torch.randint(0, V, (n,), generator=g),
                    "features": torch.randn(n, 3 * H, generator=g).to(torch.float16),
                    "prompt_len": prompt_len,
                    "labels": torch.randint(0, V, (n,), generator=g)})
    torch.save(buf, cache / "shard_00000.pt")
    (cache / "manifest.json").write_text(json.dumps({
        "shards": ["shard_00000.pt"], "num_examples": n_examples, "feature_dim": 3 * H,
        "feature_layers": [1, 2, 3], "self_distilled": True}))


def _oracle_step(drafter, input_ids, features, num_segments=1, loss_scale=1.0, prompt_len=0,
                 teacher_labels=None):
    """The CPU oracle with ``mtp_backward``'s contract (adds into ``p.grad``)."""
    dims = oracle.OracleDims(hidden=drafter.hidden, n_heads=drafter.n_heads,
                             n_kv_heads=drafter.n_kv_heads, intermediate=drafter.intermediate,
                             vocab=drafter.vocab, num_layers=len(drafter.layers),
                             max_depth=drafter.max_depth)
    params = {n: p.detach() for n, p in drafter.named_parameters()}
    heads = {"embed": drafter._embed[0].weight.detach(), "head": drafter._lm_head[0].weight.detach(),
             "norm": drafter._final_norm[0].weight.detach()}
    loss, grads = oracle.mtp_step(params, heads, input_ids, features, dims, num_segments,
                                  loss_scale, prompt_len, teacher_labels)
    for n, p in drafter.named_parameters():
        g = grads[n].to(p.dtype)
        p.grad = g.clone() if p.grad is None else p.grad + g
    return loss


def _run(tmp_path, monkeypatch, capsys, dims, dtype, device, tag, num_segments):
    cache = tmp_path / "cache"
    if not cache.exists():
        _build_cache(cache, dims, n_examples=8, seq_len=dims["seq_len"], prompt_len=3)
    heads = _heads(dims, device, _DT[dtype])
    monkeypatch.setattr(train_mod, "load_target_heads", lambda tcfg: heads)
    if device == "cpu":
        monkeypatch.setattr(train_mod, "mtp_backward", _oracle_step)
        monkeypatch.setattr(train_mod, "build_optimizer",
                            lambda params, lr, wd, use_8bit, max_norm=1.0:
                            torch.optim.AdamW(params, lr=lr, weight_decay=wd))
    tcfg = TargetConfig(model_name="tiny", device=device, dtype=dtype)
    tr = TrainConfig(feature_cache_dir=cache, out_dir=tmp_path / tag, epochs=2, grad_accum=2,
                     max_seq_len=128, lr=3e-3, num_segments=num_segments, use_8bit_adam=False,
                     grad_checkpoint=False, save_every=0, log_every=1)
    capsys.readouterr()
    d = train_mod.train(tcfg, DrafterConfig(num_layers=1, max_depth=dims["K"]), tr, dtype=dtype)
    out = capsys.readouterr().out
    monkeypatch.undo()
    losses = [float(x) for x in re.findall(r"update \d+/\d+ loss ([-0-9.]+)", out)]
    ck = torch.load(tmp_path / tag / "drafter.pt", map_location="cpu", weights_only=False)
    return losses, ck, d


CASES = {
    # fp32: CUDA-core kernels, the north_star's 1e-4 gradient regime
    "fp32": (dict(hidden=64, heads=4, kv_heads=2, intermediate=128, vocab=256, K=4, seq_len=40),
             "float32", 1e-4, 1e-3, 5e-2),
    # bf16 with head_dim 128: the tcgen05 attention and GEMM kernels
    # (no moved-distance check: updates of 3e-3 on bf16 weights near 1.0 are below half
    # an ulp there, so how far such a weight moves is a matter of rounding ties)
    "bf16": (dict(hidden=256, heads=2, kv_heads=1, intermediate=512, vocab=1024, K=5, seq_len=96),
             "bfloat16", 2e-2, 2e-2, None),
}


@pytest.mark.parametrize("name", list(CASES))
def test_train_loop_on_gpu_matches_cpu_reference_update(name, tmp_path, monkeypatch, capsys):
    from parallel_eagle_b200.engine import StepEngine

    dims, dtype, param_tol, loss_tol, moved_tol = CASES[name]
    init_ref = _fresh_params(dims, dtype)
    l_cpu, ck_cpu, _ = _run(tmp_path, monkeypatch, capsys, dims, dtype, "cpu", "cpu", 2)
    l_gpu, ck_gpu, d_gpu = _run(tmp_path, monkeypatch, capsys, dims, dtype, "cuda", "gpu", 2)
    # the CUDA run went through the fused step engine
    assert isinstance(d_gpu._engine, StepEngine)
    assert len(l_cpu) == len(l_gpu) == 8  # 8 examples x 2 epochs / grad_accum 2
    for a, b in zip(l_gpu, l_cpu):
        assert abs(a - b) <= loss_tol * abs(b), (l_gpu, l_cpu)
    assert set(ck_gpu) == {"state_dict", "num_layers", "max_depth", "target_name"}
    for k, ref in ck_cpu["state_dict"].items():
        got = ck_gpu["state_dict"][k].float()
        ref = ref.float()
        # the parameters after 8 updates, and the distance each moved from its init
        assert recipe.rel_fro(got, ref) < param_tol, k
        moved_ref = ref - init_ref[k]
        if moved_tol is not None and moved_ref.norm() > 0:
            assert recipe.rel_fro(got - init_ref[k], moved_ref) < moved_tol, k


def _fresh_params(dims, dtype):
    """The seeded initial parameters ``train()`` starts from (``torch.manual_seed(seed)``
    before the drafter is built, as reference ``train.py:52``)."""
    from parallel_eagle_b200.drafter import ParallelDrafter

    torch.manual_seed(TrainConfig().seed)
    heads = _heads(dims, "cpu", _DT[dtype])
    d = ParallelDrafter.from_target(heads, DrafterConfig(num_layers=1, max_depth=dims["K"]))
    return {n: p.detach().to(_DT[dtype]).float() for n, p in d.named_parameters()}
