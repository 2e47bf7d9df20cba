"""Host-side logic that needs no GPU: the masks API (reference tests/test_masks.py
pins), config defaults, segmenting/counting rules, the LR schedule, feature-layer
resolution and the flat parameter buffer."""

from __future__ import annotations

import pytest
import torch

import oracle
from parallel_eagle_b200 import config, engine, masks, partition, target, train


def test_mtp_allow_small_exact():
    # reference tests/test_masks.py:16-28 (n=2 anchors, K=2)
    expected = torch.tensor([[1, 0, 0, 0], [1, 1, 0, 0], [1, 0, 1, 0], [1, 0, 1, 1]], dtype=torch.bool)
    assert torch.equal(masks.mtp_allow_mask(2, 2), expected)


def test_amortized_equals_naive_and_is_topleft():
    amort = masks.AmortizedMtpMask(max_anchors=8, k=4)
    for n in (1, 3, 5, 8):
        assert torch.equal(amort.allow(n), masks.mtp_allow_mask(n, 4))
    assert torch.equal(masks.mtp_allow_mask(3, 4), masks.mtp_allow_mask(8, 4)[:12, :12])
    with pytest.raises(ValueError):
        amort.allow(9)


def test_positions_labels_and_bias():
    assert masks.mtp_position_ids(4, 3).tolist() == [0, 1, 2, 1, 2, 3, 2, 3, 4, 3, 4, 5]
    labels = masks.mtp_labels(torch.tensor([10, 11, 12, 13]), 3)
    assert labels[:3].tolist() == [11, 12, 13] and labels[-3:].tolist() == [-100] * 3
    allow = masks.mtp_allow_mask(3, 2)
    b = masks.to_additive_bias(allow, torch.bfloat16)
    assert b.shape == (1, 1, 6, 6)
    assert torch.all(b[0, 0][allow] == 0)
    assert torch.all(b[0, 0][~allow] == torch.finfo(torch.bfloat16).min)


def test_allow_rule_matches_oracle_on_random_subsets():
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 20, (50,), generator=g)
    d = torch.randint(0, 5, (50,), generator=g)
    assert torch.equal(masks.allow_from_slots(a, d), oracle.slot_allow(a, d))


def _tree_known_answer(allow, pos):
    # reference tests/test_masks.py:55-75: prefix 2, parents [-1, 0, -1]
    assert allow.shape == (5, 5)
    assert allow[0, 0] and not allow[0, 1] and allow[1, 0] and allow[1, 1]
    assert allow[2:, :2].all()
    assert allow[3, 2] and allow[3, 3] and not allow[3, 4]
    assert allow[2, 2] and not allow[2, 3] and not allow[2, 4]
    assert list(pos) == [0, 1, 2, 3, 2]


def test_tree_masks_reference_known_answer():
    parents = [-1, 0, -1]
    assert masks.tree_depths(parents) == [0, 1, 0]
    _tree_known_answer(masks.tree_allow_mask(parents, prefix_len=2),
                       masks.tree_position_ids(parents, prefix_len=2).tolist())
    # the checker itself against the same pin
    _tree_known_answer(oracle.tree_allow(parents, 2), oracle.tree_positions(parents, 2))


def _random_tree(g, t):
    return [-1 if i == 0 else int(torch.randint(-1, i, (1,), generator=g)) for i in range(t)]


@pytest.mark.parametrize("prefix_len", [0, 1, 7])
def test_tree_masks_match_oracle(prefix_len):
    g = torch.Generator().manual_seed(prefix_len)
    trees = [[], [-1], [-1, 0, 1, 2], [-1, -1, -1]] + [_random_tree(g, t) for t in (5, 17, 40)]
    # beam trees as the draft path builds them (top-k per depth, parents from the beam)
    logits = torch.randn(5, 50, generator=g)
    trees.append(oracle.propose_tree_from_logits(logits, 5, 4, 20)[1])
    for parents in trees:
        allow = masks.tree_allow_mask(parents, prefix_len)
        assert allow.dtype == torch.bool
        assert torch.equal(allow, oracle.tree_allow(parents, prefix_len)), parents
        pos = masks.tree_position_ids(parents, prefix_len)
        assert pos.dtype == torch.long
        assert pos.tolist() == oracle.tree_positions(parents, prefix_len), parents
        assert masks.tree_depths(parents) == [x - prefix_len for x in pos.tolist()[prefix_len:]]
        b = masks.to_additive_bias(allow, torch.float32)
        assert torch.all((b[0, 0] == 0) == allow)


def test_tree_masks_reject_unordered_parents():
    for bad in ([0], [-1, 1], [-1, 2, 0], [-2]):
        with pytest.raises(ValueError):
            masks.tree_allow_mask(bad, 3)
        with pytest.raises(ValueError):
            masks.tree_depths(bad)


def test_config_defaults_match_reference():
    assert config.TrainConfig().num_segments == 1
    assert config.TargetConfig().feature_layers is None
    d = config.DrafterConfig()
    assert d.hidden_size is None and d.vocab_size is None and d.num_layers >= 1 and d.max_depth >= 1


@pytest.mark.parametrize("n,k,p", [(20, 4, 7), (9, 4, 0), (2, 3, 0), (2048, 5, 0), (100, 8, 37), (5, 1, 2)])
def test_loss_slot_count_closed_form(n, k, p):
    assert partition._total_valid_after(n, k, p) == oracle.count_loss_slots(n, k, p)
    assert partition._total_valid(n, k) == oracle.count_loss_slots(n, k, 0)


@pytest.mark.parametrize("n,s", [(9, 3), (5, 2), (2, 20), (2048, 4), (13, 6), (1, 1)])
def test_segment_bounds_match_oracle(n, s):
    assert partition._segment_bounds(n, s) == oracle.segment_edges(n, s)


def test_segment_slots_match_oracle():
    a, d, nr = partition._segment_slots(3, 7, 4, "cpu")
    oa, od = oracle.segment_slots(3, 7, 4)
    assert torch.equal(a, oa) and torch.equal(d, od) and nr == 7


def test_lr_schedule():
    assert train.lr_at(0, 100, 1.0, 0.1) == 0.0
    assert train.lr_at(5, 100, 1.0, 0.1) == 0.5
    assert train.lr_at(10, 100, 1.0, 0.1) == 1.0
    assert train.lr_at(100, 100, 1.0, 0.1) == 0.0


def test_feature_layer_resolution():
    assert target.resolve_feature_layers(None, 28) == (7, 15, 27)
    assert target.resolve_feature_layers((-1, 3), 10) == (10, 3)
    assert target.resolve_feature_layers(None, 2) == (1, 2, 2)


def _tiny_drafter(seed=0):
    from parallel_eagle_b200.drafter import ParallelDrafter
    from parallel_eagle_b200.nn import RMSNorm

    H, V = 32, 64
    embed, head, norm = torch.nn.Embedding(V, H), torch.nn.Linear(H, V, bias=False), RMSNorm(H)
    torch.manual_seed(seed)
    return ParallelDrafter(hidden=H, n_heads=4, n_kv_heads=2, intermediate=48, vocab=V,
                           feature_dim=3 * H, rope_theta=1e4, eps=1e-5, num_layers=2, max_depth=3,
                           embed_module=embed, lm_head_module=head, final_norm_module=norm)


def test_drafter_init_matches_reference_order():
    # the oracle's init is pinned bit-exactly to the reference's (test_oracle_golden);
    # the drafter draws its parameters in the same order from the same seed
    d = _tiny_drafter(seed=5)
    dims = oracle.OracleDims(hidden=32, n_heads=4, n_kv_heads=2, intermediate=48, vocab=64,
                             num_layers=2, max_depth=3)
    ref = oracle.init_params(dims, 5)
    sd = d.state_dict()
    assert list(sd) == oracle.param_names(2)
    for k in sd:
        assert torch.equal(sd[k], ref[k]), k


def test_flat_params_views_and_grad_attachment():
    d = _tiny_drafter()
    before = {k: v.clone() for k, v in d.state_dict().items()}
    fp = engine.FlatParams(d)
    assert fp.valid()
    for k, v in d.state_dict().items():
        assert torch.equal(v, before[k])
    # q/k/v and gate/up are one contiguous matrix each; mask_emb|h_shared adjacent
    qkv = fp.span("layers.0.attn.q_proj.weight", "layers.0.attn.v_proj.weight", 32)
    assert torch.equal(qkv, torch.cat([before[f"layers.0.attn.{n}_proj.weight"] for n in "qkv"]))
    cat = fp.span("mask_emb", "h_shared", 64)
    assert torch.equal(cat[0], torch.cat([before["mask_emb"], before["h_shared"]]))
    assert fp.offsets["feat_proj.weight"][0] % 128 == 0
    # grads: None -> zero view; foreign tensor -> copied in; view kept as is
    p0 = d.in_proj.weight
    p0.grad = torch.ones_like(p0)
    fp.attach_grads()
    assert p0.grad.data_ptr() == fp.view("in_proj.weight", grad=True).data_ptr()
    assert torch.all(p0.grad == 1) and torch.all(d.mask_emb.grad == 0)
    fp.grad.add_(1)
    fp.attach_grads()
    assert torch.all(p0.grad == 2)
    # moving the module invalidates the flat views
    d.to(torch.float64)
    assert not fp.valid()


def test_install_as_pe_resolves_reference_imports():
    """After ``install_as_pe()`` the reference's import lines reach this package
    (run in a child interpreter so this process's ``sys.modules`` stays clean)."""
    import subprocess
    import sys
    from pathlib import Path

    code = (
        "import parallel_eagle_b200 as P; P.install_as_pe()\n"
        "from pe.partition import mtp_backward, mtp_eval_loss\n"
        "from pe.drafter import ParallelDrafter, load_drafter\n"
        "from pe.masks import AmortizedMtpMask, tree_allow_mask, tree_position_ids\n"
        "from pe.config import DrafterConfig, TrainConfig\n"
        "from pe.train import train\n"
        "from pe.features import FeatureDataset\n"
        "from pe.nn import RMSNorm, DecoderLayer\n"
        "from pe.decode.tree import propose_tree\n"
        "from pe.decode.chain import propose_chain, propose_chain_sequential, propose_chain_sampling\n"
        "from pe.decode import propose_tree as t2, accept_tree_greedy, accept_chain_greedy\n"
        "from pe.decode.verify import accept_chain_sampling, accept_tree_cached\n"
        "import pe.decode.tree, pe.partition\n"
        "assert pe.decode.tree.propose_tree is propose_tree is t2\n"
        "assert pe.partition.mtp_backward.__module__.startswith('parallel_eagle_b200')\n"
        "print('ok')\n"
    )
    root = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0 and res.stdout.strip() == "ok", res.stderr


def test_propose_chain_sampling_rejects_non_positive_temperature():
    from parallel_eagle_b200 import decode

    for t in (0.0, -0.5, float("nan")):
        with pytest.raises(ValueError):
            decode.propose_chain_sampling(None, None, None, 3, t)


def test_verification_rejects_empty_prefix():
    from parallel_eagle_b200 import decode

    with pytest.raises(ValueError):
        decode.accept_chain_greedy(torch.zeros(3, 5), 0, [1, 2])
    with pytest.raises(ValueError):
        decode.accept_tree_greedy(torch.zeros(3, 5), 0, [1], [-1])


def test_reference_arm_times_the_full_workload_within_its_budget(monkeypatch, capsys):
    """bench.py --impl reference: warm-up samples are short (n = 256), every timed
    sample is one full sequence of the workload (n = 2048), the config equals this
    framework's arm's, and timed samples stop (after at least three) once they pass
    the budget."""
    import argparse
    import json
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench

    def fake_run(per_sample_s, steps, warmup):
        clock = {"t": 0.0}
        calls = []

        def fake_cpu(args, n=None):
            calls.append(n)
            sec = per_sample_s * n / 2048
            clock["t"] += sec
            return {"seconds": sec, "cores": 4, "sample": f"one sequence, n={n}"}

        monkeypatch.setattr(bench, "cpu_baseline", fake_cpu)
        monkeypatch.setattr(bench.time, "perf_counter", lambda: clock["t"])
        capsys.readouterr()
        bench.run_reference(argparse.Namespace(steps=steps, warmup=warmup, cpu_n=2048))
        return calls, json.loads(capsys.readouterr().out.strip().splitlines()[-1])

    calls, line = fake_run(11.0, steps=20, warmup=5)
    assert calls == [256] * 5 + [2048] * 20
    assert line["steps"] == 20 and line["config"]["n"] == 2048
    assert line["value"] == round(2048 * 5 / 11.0, 2)
    ours = bench.workload_config(bench.WORKLOADS[2][0], dict(bench.CONFIG2), 1)
    assert line["config"] == ours
    # a slow host: the budget cuts the timed samples short, never below three
    calls, line = fake_run(200.0, steps=20, warmup=3)
    assert calls[3:] == [2048] * 3 and line["steps"] == 3 and line["steps_requested"] == 20
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["impl"] == "reference"


def test_speculative_sampling_acceptance_is_lossless():
    """Property of the acceptance rule (reference decode/verify.py:75-101): with the
    draft drawn from q, the first emitted token -- the first draft if kept, else the
    residual bonus -- is distributed as the target's p, whatever q is."""
    from parallel_eagle_b200 import decode

    g = torch.Generator().manual_seed(3)
    V, trials = 6, 6000
    p = torch.softmax(torch.randn(2, V, generator=g) * 1.5, -1)
    q = torch.softmax(torch.randn(1, V, generator=g) * 1.5, -1)
    counts = torch.zeros(V)
    for _ in range(trials):
        draft = [int(torch.multinomial(q[0], 1, generator=g))]
        acc, bonus = decode.accept_chain_sampling(p, draft, q, generator=g)
        counts[acc[0] if acc else bonus] += 1
    tv = 0.5 * (counts / trials - p[0]).abs().sum().item()
    assert tv < 0.03, tv


def test_clock_sampler_follows_cuda_visible_devices(monkeypatch):
    """The bench samples the clocks of the GPU it runs on: nvidia-smi numbers GPUs
    physically, CUDA after CUDA_VISIBLE_DEVICES."""
    import bench

    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "6")
    assert bench.smi_index(0) == 6
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "2,3,4,5")
    assert [bench.smi_index(i) for i in range(4)] == [2, 3, 4, 5]
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.smi_index(3) == 3
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-5f1c")  # UUIDs: left to the index
    assert bench.smi_index(0) == 0
