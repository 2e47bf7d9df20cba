"""Drafter training-step throughput on B200 (slot-tokens/s), one process per GPU.

    python bench.py [--gpus N --steps K --warmup W]            # this framework
    python bench.py --impl reference [...]                      # CPU reference arm
    torchrun --nproc-per-node N bench.py --gpus N ...           # data parallel

A step is one optimizer update over the global batch: for every local sequence
``mtp_backward`` (forward + backward of the partitioned MTP loss, BASELINE
config 2: hidden 3584, 28/4 heads, I 18944, vocab 152064, n 2048, K 5, S 4,
bf16, batch 8 per GPU), then the gradient all-reduce (N > 1), global-norm clip
and AdamW.  Inputs are synthetic (seeded) with the BASELINE shapes.

``value`` is device-timed with inputs resident in HBM; ``e2e`` is the same step
through the public API with ids/features copied from pinned host memory each
step and the loss read back.  The reference arm times the CPU oracle port of
the reference step on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG2 = dict(hidden=3584, n_heads=28, n_kv_heads=4, intermediate=18944, vocab=152064,
               num_layers=1, max_depth=5, n=2048, segments=4, batch=8)
# BASELINE configs 3 (config 2 with the soft-target distillation loss, global batch 64)
# and 4 (14B-class drafter, global batch 64); per-GPU batch = 64 / GPUs (8 on one GPU)
CONFIG3 = dict(CONFIG2, soft=True, global_batch=64)
CONFIG4 = dict(hidden=5120, n_heads=40, n_kv_heads=8, intermediate=13824, vocab=152064,
               num_layers=1, max_depth=5, n=2048, segments=4, batch=8, global_batch=64)
WORKLOADS = {2: ("BASELINE config 2: 7B-class drafter step", CONFIG2),
             3: ("BASELINE config 3: 7B-class drafter, soft-target distillation loss", CONFIG3),
             4: ("BASELINE config 4: 14B-class drafter step", CONFIG4)}
METRIC = "drafter train slot-tokens/sec at 1/2/4/8 B200; masked-attn fwd+bwd TFLOP/s vs peak"
UNIT = "slot-tokens/s"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def attention_pairs(n, k, segments):
    from parallel_eagle_b200.engine import segment_bounds

    pairs = 0
    for a0, a1 in segment_bounds(n, segments):
        pairs += a1 * (a1 + 1) // 2
        pairs += sum((k - 1) * (i + 1) for i in range(a0, a1)) + (a1 - a0) * k * (k - 1) // 2
    return pairs


def step_flops_per_sequence(c):
    """Algorithmic FLOPs of one sequence (2 per MAC, counted at S=1, no recompute)."""
    H, I, V = c["hidden"], c["intermediate"], c["vocab"]
    hd = H // c["n_heads"]
    n, k = c["n"], c["max_depth"]
    r_all = n * k
    r_valid = n * k - k * (k + 1) // 2
    layer = 3 * r_all * (2 * H * (2 * c["n_heads"] * hd + 2 * c["n_kv_heads"] * hd) + 6 * H * I)
    head = 2 * r_valid * 2 * H * V * (1.5 if c.get("soft") else 1.0)  # + teacher logits
    inp = n * (2 * 2 * 3 * H * H + 2 * 2 * 2 * H * H + 2 * H * H)
    attn = 12 * hd * c["n_heads"] * attention_pairs(n, k, 1)
    return c["num_layers"] * layer + head + inp + c["num_layers"] * attn


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:  # noqa: BLE001 - sampling is best effort
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(self.rows)}


# --------------------------------------------------------------------------- #


def smi_index(local: int) -> int:
    """nvidia-smi's index of CUDA device ``local``: CUDA_VISIBLE_DEVICES, when it lists
    plain indices, renumbers the devices this process sees, nvidia-smi does not."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    ids = [x.strip() for x in vis.split(",") if x.strip()]
    if ids and all(x.isdigit() for x in ids) and local < len(ids):
        return int(ids[local])
    return local


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def workload_config(workload, c, world):
    """The ``config`` object of a bench line: the workload's shape, identical in this
    framework's arm and the reference arm."""
    return {"workload": workload, "hidden": c["hidden"], "heads": [c["n_heads"], c["n_kv_heads"]],
            "intermediate": c["intermediate"], "vocab": c["vocab"], "layers": c["num_layers"],
            "n": c["n"], "K": c["max_depth"], "S": c["segments"], "batch_per_gpu": c["batch"],
            "global_batch": c["batch"] * world, "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (features 44 MB/sequence, weights 0.5 GB)"}


def make_heads_gpu(c, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(10_000 + seed)
    V, H = c["vocab"], c["hidden"]
    embed = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    head = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    norm = torch.ones(H, device=dev, dtype=torch.bfloat16)
    return embed, head, norm


def build_drafter(c, dev, seed=0):
    import types

    from parallel_eagle_b200.config import DrafterConfig
    from parallel_eagle_b200.drafter import ParallelDrafter
    from parallel_eagle_b200.nn import RMSNorm

    E, Wh, wn = make_heads_gpu(c, dev, seed)
    V, H = E.shape
    embed = torch.nn.Embedding(V, H, _weight=E)
    head = torch.nn.Linear(H, V, bias=False, device="meta")
    head.weight = torch.nn.Parameter(Wh, requires_grad=False)
    norm = RMSNorm(H, 1e-5)
    norm.weight = torch.nn.Parameter(wn, requires_grad=False)
    embed.weight.requires_grad_(False)
    cfg = types.SimpleNamespace(num_attention_heads=c["n_heads"], num_key_value_heads=c["n_kv_heads"],
                                intermediate_size=c["intermediate"], rope_theta=10000.0,
                                rms_norm_eps=1e-5)
    target = types.SimpleNamespace(config=cfg, hidden_size=H, vocab_size=V, feature_dim=3 * H,
                                   get_input_embeddings=lambda: embed, get_lm_head=lambda: head,
                                   get_final_norm=lambda: norm)
    torch.manual_seed(seed)
    with torch.device(dev):
        d = ParallelDrafter.from_target(target, DrafterConfig(num_layers=c["num_layers"],
                                                              max_depth=c["max_depth"]))
    return d.to(dtype=torch.bfloat16)


class Trainer:
    """One optimizer update over the local sequences (+ all-reduce when N > 1)."""

    def __init__(self, drafter, c, world, lr=1e-4):
        from parallel_eagle_b200.engine import engine_for

        self.d = drafter
        self.c = c
        self.world = world
        self.eng = engine_for(drafter)
        fp = self.eng.flat
        self.m = torch.zeros(fp.numel, dtype=torch.float32, device=fp.device)
        self.v = torch.zeros_like(self.m)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=fp.device)
        self.loss = torch.zeros(1, dtype=torch.float32, device=fp.device)
        self.lr = lr
        self.t = 0
        self.overlap = None
        # (step start, all-reduce finish entered, finish returned) events per step (N > 1)
        self.comm_events = []
        self.record_comm = False
        if world > 1:
            from parallel_eagle_b200.train import OverlappedAllReduce

            self.overlap = OverlappedAllReduce(drafter)

    def _event(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream())
        return e

    def step(self, seqs, global_batch, teachers=None):
        from parallel_eagle_b200 import ops

        fp = self.eng.flat
        rec = self.record_comm and self.overlap is not None
        ev0 = self._event() if rec else None
        fp.grad.zero_()
        self.loss.zero_()
        for i, (ids, feats) in enumerate(seqs):
            if self.overlap is not None and i == len(seqs) - 1:
                self.overlap.arm()  # reduce the layers' gradients during the last backward
            self.eng.run(ids, feats, self.c["segments"], loss_scale=1.0 / global_batch, sync=False,
                         teacher_hidden=None if teachers is None else teachers[i])
            self.loss += self.eng.loss_sum
        if self.overlap is not None:
            ev1 = self._event() if rec else None
            self.overlap.finish()
            if rec:
                self.comm_events.append((ev0, ev1, self._event()))
        self.sumsq.zero_()
        ops.sumsq_into(fp.grad, self.sumsq)
        self.t += 1
        ops.adamw_step(fp.flat, fp.grad, self.m, self.v, self.sumsq, 1.0, self.lr, 0.9, 0.999,
                       1e-8, 0.0, self.t)
        return self.loss


def run_ours(args):
    import torch.distributed as dist

    from parallel_eagle_b200 import _lib, ops

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=600))
    workload, base = WORKLOADS[args.config]
    c = dict(base)
    if "global_batch" in c and world > 1:
        c["batch"] = max(1, c["global_batch"] // world)
    if args.n:
        c["n"] = args.n
    if args.batch:
        c["batch"] = args.batch
    B, n, k = c["batch"], c["n"], c["max_depth"]
    gb = B * world
    drafter = build_drafter(c, dev, seed=0)
    trainer = Trainer(drafter, c, world)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    ids = torch.randint(0, c["vocab"], (B, n), generator=g, device=dev)
    feats = torch.randn(B, n, 3 * c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    seqs = [(ids[b], feats[b]) for b in range(B)]
    # config 3: the teacher's last-layer hidden states ~ N(0, 1)
    teachers = None
    if c.get("soft"):
        teachers = torch.randn(B, n, c["hidden"], generator=g, device=dev).to(torch.bfloat16)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        trainer.step(seqs, gb, teachers)
    torch.cuda.synchronize()
    ops.check_status(dev)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = _lib.launch_count()
    trainer.record_comm = True
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(smi_index(local)) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            # the NVTX range lets a profiler select exactly the timed steps' launches
            torch.cuda.nvtx.range_push("pe_step")
            trainer.step(seqs, gb, teachers)
            torch.cuda.nvtx.range_pop()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    launches = (_lib.launch_count() - l0) // max(1, args.steps)
    trainer.record_comm = False
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    dp = data_parallel_report(trainer, clocks, world, dev) if world > 1 else None
    value = gb * n * k / (ms / 1e3)
    from parallel_eagle_b200.engine import count_loss_slots

    # mean cross entropy per loss slot over this rank's sequences after the timed
    # updates (the same fixed synthetic sequences are trained on every step)
    loss_val = float(trainer.loss.item()) / (B * count_loss_slots(n, k))

    # ---- end to end through the public API: pinned host inputs, loss read back
    from parallel_eagle_b200.partition import mtp_backward

    h_ids = ids.cpu().pin_memory()
    h_feats = feats.cpu().pin_memory()
    h_teach = teachers.cpu().pin_memory() if teachers is not None else None
    fp = trainer.eng.flat

    def e2e_step():
        drafter.zero_grad(set_to_none=True)
        tot = 0.0
        for b in range(B):
            if trainer.overlap is not None and b == B - 1:
                trainer.overlap.arm()
            tot += mtp_backward(drafter, h_ids[b], h_feats[b], c["segments"], loss_scale=1.0 / gb,
                                teacher_hidden=None if h_teach is None else h_teach[b])
        if trainer.overlap is not None:
            trainer.overlap.finish()
        trainer.sumsq.zero_()
        ops.sumsq_into(fp.grad, trainer.sumsq)
        trainer.t += 1
        ops.adamw_step(fp.flat, fp.grad, trainer.m, trainer.v, trainer.sumsq, 1.0, trainer.lr,
                       0.9, 0.999, 1e-8, 0.0, trainer.t)
        return tot

    e2e_ms = wall_ms = None
    if not args.no_e2e:
        e2e_step()
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        t = torch.tensor([e2e_ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
        wall_ms = (time.perf_counter() - w0) * 1e3 / args.steps

    # ---- roofline of the dominant kernel: the tensor-core GEMM, gate/up shape of the step
    # both rooflines time one kernel family alone, so they are set against the burst
    # peak; a short idle first lets the clocks leave the step loop's power-capped state
    hbm, peak_burst, peak_sus, src = _peaks()
    time.sleep(1.0)
    roof = gemm_roofline(c, dev, peak_burst, src)
    time.sleep(1.0)
    attn = attention_roofline(c, dev, peak_burst, src)
    step_tflops = step_flops_per_sequence(c) * B / (ms / 1e3) / 1e12

    if rank == 0:
        # the CPU sample is a config-2 sequence: reported with the config-2 workload only
        cpu = (cpu_baseline(args)
               if (world == 1 and not args.no_cpu_baseline and args.config == 2) else None)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            # configs 3 / 4 fix the global batch (64 sequences split over the ranks)
            "scaling": "strong" if "global_batch" in c else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded ids ~ U[0,V), features ~ N(0,1), heads ~ N(0,0.02^2))",
            "config": workload_config(workload, c, world),
            "loss_ce_per_slot": round(loss_val, 4),
            "step_tflops": round(step_tflops, 1),
            "step_frac_of_peak": round(step_tflops / peak_sus, 4),
            "e2e": None if e2e_ms is None else {
                "value": round(gb * n * k / (e2e_ms / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": int(B * (ids[0].numel() * 8 + feats[0].numel() * 2)
                                          + (teachers.numel() * 2 if teachers is not None else 0)),
                "d2h_bytes_per_step": int(4 * B), "wall_ms_per_step": round(wall_ms, 2)},
            "roofline": roof,
            "attention": attn,
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if dp is not None:
            line["data_parallel"] = dp
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def data_parallel_report(trainer, clocks, world, dev):
    """Per-rank split of the timed steps (N > 1) and a cross-rank consistency check.

    compute_ms: step start -> the all-reduce's ``finish()`` (the local sequences'
    forward/backward, with the layers' reduction already running beside the input
    projections' backward); exposed_comm_ms: ``finish()`` entered -> returned on the
    compute stream (the reduction time the backward did not hide).  Both are CUDA-event
    means over the timed steps.  The flat parameters after the last update are
    checksummed on every rank; ranks that differ fail the run."""
    import torch.distributed as dist

    comp = sum(a.elapsed_time(b) for a, b, _ in trainer.comm_events) / len(trainer.comm_events)
    expo = sum(b.elapsed_time(c) for _, b, c in trainer.comm_events) / len(trainer.comm_events)
    trainer.comm_events.clear()
    sm = clocks.summary().get("sm_mhz") or 0.0
    flat = trainer.eng.flat.flat
    words = flat.view(torch.int16).to(torch.int64)
    pos = torch.arange(words.numel(), device=dev, dtype=torch.int64) % 65521
    mine = torch.stack([words.sum(), (words * pos).sum()])
    sums = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(sums, mine)
    stats = torch.tensor([comp, expo, float(sm)], device=dev, dtype=torch.float64)
    per = [torch.empty_like(stats) for _ in range(world)]
    dist.all_gather(per, stats)
    same = all(torch.equal(sums[0], x) for x in sums[1:])
    if not same:
        raise RuntimeError("data-parallel ranks hold different parameters after the update")
    per = [x.tolist() for x in per]
    return {"rank_compute_ms": [round(x[0], 2) for x in per],
            "rank_exposed_comm_ms": [round(x[1], 3) for x in per],
            "exposed_comm_ms": round(max(x[1] for x in per), 3),
            "rank_sm_mhz": [x[2] for x in per],
            "params_identical_across_ranks": same,
            "grad_bytes": int(trainer.eng.flat.grad.numel() * trainer.eng.flat.grad.element_size())}


def gemm_case(c, dev):
    """The step's largest GEMM: the fused gate/up projection of a 4096-slot segment
    (M=4096, N=2*I, K=H).  Returns (run, flops per run, algorithmic bytes per run)."""
    from parallel_eagle_b200 import ops

    H, I = c["hidden"], c["intermediate"]
    M = 4096
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    out = torch.empty(M, 2 * I, dtype=torch.bfloat16, device=dev)

    def run():
        ops.linear(x, w, out=out)

    return run, 2.0 * M * 2 * I * H, 2.0 * (M * H + 2 * I * H + M * 2 * I)


def attention_case(c, dev):
    """Masked-attention fwd+bwd over the S segments of one config-2 sequence, stacked
    in one row space and run by one call each way (as the step engine does).
    FLOPs = 12 * hd * Hq * allowed pairs (no recompute)."""
    from parallel_eagle_b200 import ops
    from parallel_eagle_b200.engine import segment_bounds

    nh, nkv, hd, k = c["n_heads"], c["n_kv_heads"], c["hidden"] // c["n_heads"], c["max_depth"]
    cols = (nh + 2 * nkv) * hd
    g = torch.Generator(device=dev).manual_seed(11)
    bounds = segment_bounds(c["n"], c["segments"])
    R = sum(ops.segment_rows(bounds, k))
    qkv = torch.randn(R, cols, generator=g, device=dev).to(torch.bfloat16)
    do = torch.randn(R, nh * hd, generator=g, device=dev).to(torch.bfloat16)
    q, kk, vv = qkv[:, : nh * hd], qkv[:, nh * hd:(nh + nkv) * hd], qkv[:, (nh + nkv) * hd:]
    dqkv = torch.empty_like(qkv)
    # the step's backward also rotates dQ / dK back (RoPE's transpose, fused in the dQ
    # store and the dK cast): the same table the step builds for these slots
    from parallel_eagle_b200.engine import StepEngine

    pos = torch.cat([torch.from_numpy(StepEngine._segment_arrays_static(a0, a1, c["n"], k, 0)[0])
                     for a0, a1 in bounds]).to(dev)
    cs = ops.rope_table(pos, hd, 10000.0, torch.bfloat16)

    def run():
        o, lse = ops.attn_fwd_segments(q, kk, vv, nh, nkv, hd, bounds, k)
        ops.attn_bwd_segments(q, kk, vv, o, do, lse, nh, nkv, hd, bounds, k,
                              dq=dqkv[:, : nh * hd], dk=dqkv[:, nh * hd:(nh + nkv) * hd],
                              dv=dqkv[:, (nh + nkv) * hd:], rope_cs=cs)

    return run, 12.0 * hd * nh * attention_pairs(c["n"], k, c["segments"]), None


def lmhead_case(c, dev):
    """Fused LM-head cross entropy (loss + input gradient) over the 2560 loss slots
    of one 512-token segment at K=5 against the full 152064-row head."""
    from parallel_eagle_b200 import ops

    R, H, V = 2560, c["hidden"], c["vocab"]
    g = torch.Generator(device=dev).manual_seed(13)
    h = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    lab = torch.randint(0, V, (R,), generator=g, device=dev)
    loss = torch.zeros(1, device=dev)

    def run():
        ops.lmhead_ce(h, W, lab, 1e-4, loss)

    return run, 2.0 * 2 * R * V * H, None


def elementwise_cases(c, dev):
    """The step's memory-bound kernels on one stacked pass of a config-2 sequence
    (13312 slot rows): name -> (run, algorithmic HBM bytes per run)."""
    from parallel_eagle_b200 import ops

    H, I = c["hidden"], c["intermediate"]
    nh, nkv, hd = c["n_heads"], c["n_kv_heads"], c["hidden"] // c["n_heads"]
    R = 13312
    g = torch.Generator(device=dev).manual_seed(17)
    bf = torch.bfloat16
    x = torch.randn(R, H, generator=g, device=dev).to(bf)
    dy = torch.randn(R, H, generator=g, device=dev).to(bf)
    res = torch.randn(R, H, generator=g, device=dev).to(bf)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(bf)
    y, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    gu = torch.randn(R, 2 * I, generator=g, device=dev).to(bf)
    da = torch.randn(R, I, generator=g, device=dev).to(bf)
    act = torch.empty(R, I, dtype=bf, device=dev)
    dgu = torch.empty(R, 2 * I, dtype=bf, device=dev)
    qkv = torch.randn(R, (nh + 2 * nkv) * hd, generator=g, device=dev).to(bf)
    pos = torch.randint(0, 4096, (R,), generator=g, device=dev)
    e = 2  # bytes per bf16 element
    return {
        "rmsnorm_fwd": (lambda: ops.rmsnorm_fwd(x, w, 1e-5, out=y), R * H * 2 * e + R * 4),
        "rmsnorm_bwd": (lambda: ops.rmsnorm_bwd(dy, x, w, rstd, dx=y, residual=res),
                        R * H * 4 * e + R * 4),
        "swiglu_fwd": (lambda: ops.swiglu_fwd(gu, I, out=act), R * I * 3 * e),
        "swiglu_bwd": (lambda: ops.swiglu_bwd(da, gu, I, out=dgu), R * I * 5 * e),
        "rope": (lambda: ops.rope_(qkv, nh + nkv, hd, pos, 10000.0), R * (nh + nkv) * hd * 2 * e + R * 8),
    }


def time_case(run, reps, warmup=3, flush=None):
    """Average milliseconds of ``run`` over ``reps`` CUDA-event-timed calls on the
    current stream; ``flush`` (a buffer larger than L2) is rewritten before each."""
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    times = []
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        run()
        b.record(s)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return sum(times) / len(times)


def time_variants(runs: dict, reps: int, warmup: int = 2, rounds: int = 5) -> dict:
    """Median milliseconds per call of each variant over ``rounds`` interleaved rounds
    (each round times every variant ``reps`` times, in an order that alternates from
    round to round), so a clock that drifts under the power cap does not favour
    whichever variant runs first."""
    for fn in runs.values():
        for _ in range(warmup):
            fn()
    names = list(runs)
    samples = {n: [] for n in names}
    for r in range(rounds):
        for n in (names if r % 2 == 0 else names[::-1]):
            samples[n].append(time_case(runs[n], reps, warmup=0))
    return {n: sorted(v)[len(v) // 2] for n, v in samples.items()}


def time_case_graph(run, reps, warmup=3):
    """Average milliseconds per call of ``run``, captured ``reps`` times into one CUDA
    graph and replayed (CUDA events on the current stream): device time without the
    host's per-call launch overhead."""
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            run()
    g.replay()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    g.replay()
    b.record(s)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def profiled_traffic(name):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>
    (the ``traffic_bytes_per_launch:`` line), or None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(float(line.split(":", 1)[1].split()[0]))
    return None


GEMM_PROFILE = "gemm_tc_pair_gateup_4096x37888x3584.txt"


def gemm_roofline(c, dev, peak, src):
    """Time the step's largest GEMM with CUDA events on its stream, L2 flushed
    between launches."""
    run, flops, nbytes = gemm_case(c, dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ms = time_case(run, 10, flush=flush)
    achieved = flops / (ms / 1e3) / 1e12
    H, I = c["hidden"], c["intermediate"]
    return {"kernel": f"gemm_tc_pair_kernel (gate/up projection, M=4096 N={2 * I} K={H}; "
                      "CTA-pair tiles)",
            "bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "peak_source": f"{src} bf16_tflops (burst)",
            # the committed ncu summary covers the config-2 shape only
            "traffic": (profiled_traffic(GEMM_PROFILE)
                        if (c["hidden"], c["intermediate"]) == (3584, 18944) else None),
            "algorithmic_bytes": int(nbytes),
            "ms": round(ms, 4)}


def attention_roofline(c, dev, peak, src):
    run, flops, _ = attention_case(c, dev)
    ms = time_case(run, 5)
    achieved = flops / (ms / 1e3) / 1e12
    return {"kernels": "attn_fwd_tc2_kernel + attn_bwd_q2_kernel + attn_bwd_kv2_kernel (+ prep/cast)",
            "segments": c["segments"], "ms_per_sequence": round(ms, 3),
            "tflops": round(achieved, 1), "peak": peak, "frac": round(achieved / peak, 4),
            "peak_source": f"{src} bf16_tflops (burst)", "flops_per_sequence": flops}


def run_sweep(args):
    """config-2 dims, batch 4 per GPU, n in {256..4096}, K in {4, 8},
    S in {1, 2, 4, 8} (``--sweep-n`` / ``--sweep-k`` / ``--sweep-s`` pick a subset); per
    point one JSON line (rank 0) with peak HBM, slot-tokens/s and the masked-attention
    fwd+bwd TFLOP/s of one sequence.  Under torchrun every rank trains its own 4
    sequences and the update all-reduces the gradients (weak scaling); step time and
    peak HBM are the max over ranks."""
    import torch.distributed as dist

    from parallel_eagle_b200 import ops

    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=600))

    def max_over_ranks(x):
        t = torch.tensor([float(x)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    _, peak_burst, _, src = _peaks()
    ns = [int(x) for x in args.sweep_n.split(",")]
    ks = [int(x) for x in args.sweep_k.split(",")]
    ss = [int(x) for x in args.sweep_s.split(",")]
    for K in ks:
        c = dict(CONFIG2, batch=4, max_depth=K)
        drafter = build_drafter(c, dev, seed=0)
        trainer = Trainer(drafter, c, world)
        for n in ns:
            g = torch.Generator(device=dev).manual_seed(n * 131 + rank)
            ids = torch.randint(0, c["vocab"], (c["batch"], n), generator=g, device=dev)
            feats = torch.randn(c["batch"], n, 3 * c["hidden"], generator=g,
                                device=dev).to(torch.bfloat16)
            seqs = [(ids[b], feats[b]) for b in range(c["batch"])]
            gb = c["batch"] * world
            for S in ss:
                cs = dict(c, n=n, segments=S)
                trainer.c = cs
                trainer.step(seqs, gb)
                torch.cuda.synchronize()
                torch.cuda.reset_peak_memory_stats(dev)
                base = torch.cuda.memory_allocated(dev)
                if world > 1:
                    dist.barrier()
                ms = max_over_ranks(time_case(lambda: trainer.step(seqs, gb), max(1, args.steps),
                                              warmup=1))
                peak = max_over_ranks(torch.cuda.max_memory_allocated(dev))
                above = max_over_ranks(torch.cuda.max_memory_allocated(dev) - base)
                run, flops, _ = attention_case(cs, dev)
                ams = max_over_ranks(time_case(run, 3, warmup=1))
                ops.check_status(dev)
                if rank == 0:
                    print(json.dumps({
                        "sweep": "BASELINE config 5", "n_gpus": world, "n": n, "K": K, "S": S,
                        "batch_per_gpu": c["batch"], "global_batch": gb,
                        "ms_per_step": round(ms, 3),
                        "slot_tokens_per_s": round(gb * n * K / (ms / 1e3), 1),
                        "peak_hbm_gb": round(peak / 1e9, 2),
                        "peak_hbm_above_resident_gb": round(above / 1e9, 2),
                        "attn_fwd_bwd_tflops": round(flops / (ams / 1e3) / 1e12, 1),
                        "attn_frac_of_peak": round(flops / (ams / 1e3) / 1e12 / peak_burst, 4),
                        "peak_source": f"{src} bf16_tflops (burst)"}), flush=True)
        del trainer, drafter
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()


AB_VARIANTS = {
    # name -> StepEngine kernel choices (every variant computes the same result)
    "default": {},
    "unfused_rope": {"fuse_rope": False},
    "unfused_swiglu": {"fuse_swiglu": False},
    "fused_swiglu_bwd": {"fuse_swiglu_bwd": True},
    "lmhead_256_256": {"lmhead_algo": (1 << 24) | (1 << 26)},
    "lmhead_auto_dh256": {"lmhead_algo": 1 << 26},
    # two 5120-row groups instead of one of 10240 (all loss rows of a config-2 sequence)
    "lmhead_group5120": {"lmhead_algo": 20 << 16},
    "lmhead_chunk8k": {"lmhead_algo": 8 << 8},
    # 16K / 24K-column vocabulary chunks (the default is 32K): more fp32 dH
    # read-modify-write passes
    "lmhead_chunk16k": {"lmhead_algo": 16 << 8},
    "lmhead_chunk24k": {"lmhead_algo": 24 << 8},
    # every vocabulary chunk two-pass (logits stored, then rewritten as exponentials)
    "lmhead_two_pass": {"lmhead_algo": 1 << 28},
    # 256-wide CTA-pair tiles (two TMEM accumulators, epilogue hidden) instead of the
    # automatic 512 for the long-K MLP GEMMs / every weight gradient
    "mlp_tiles256": {"gemm_algo": {"dn_fwd": 256 << 8, "gu_dgrad": 256 << 8,
                                   "gu_wgrad": 256 << 8, "dn_wgrad": 256 << 8}},
    "wgrad_tiles256": {"gemm_algo": {"gu_wgrad": 256 << 8, "dn_wgrad": 256 << 8,
                                     "o_wgrad": 256 << 8, "qkv_wgrad": 256 << 8}},
}


def run_ab(args):
    """Step-level A/B of the engine's kernel choices on one GPU: one trainer on the
    config-2 workload, whole training steps of each variant in interleaved rounds (the
    order alternating round to round, so a clock drifting under the power cap favours
    none), median step time per variant."""
    from parallel_eagle_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    workload, base = WORKLOADS[args.config]
    c = dict(base)
    B, n, k = c["batch"], c["n"], c["max_depth"]
    drafter = build_drafter(c, dev, seed=0)
    trainer = Trainer(drafter, c, 1)
    g = torch.Generator(device=dev).manual_seed(1000)
    ids = torch.randint(0, c["vocab"], (B, n), generator=g, device=dev)
    feats = torch.randn(B, n, 3 * c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    seqs = [(ids[b], feats[b]) for b in range(B)]
    teachers = None
    if c.get("soft"):
        teachers = torch.randn(B, n, c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    names = [v for v in args.ab.split(",") if v]
    eng = trainer.eng
    defaults = {key: getattr(eng, key)
                for key in ("fuse_rope", "fuse_swiglu", "fuse_swiglu_bwd", "lmhead_algo",
                            "gemm_algo")}

    def use(name):
        for key, val in defaults.items():
            setattr(eng, key, AB_VARIANTS[name].get(key, val))

    samples = {nm: [] for nm in names}
    for nm in names:
        use(nm)
        for _ in range(args.warmup):
            trainer.step(seqs, B, teachers)
    for r in range(args.ab_rounds):
        for nm in (names if r % 2 == 0 else names[::-1]):
            use(nm)
            samples[nm].append(time_case(lambda: trainer.step(seqs, B, teachers), args.steps,
                                         warmup=1))
    ops.check_status(dev)
    out = {}
    for nm, v in samples.items():
        ms = sorted(v)[len(v) // 2]
        out[nm] = {"ms_per_step": round(ms, 2), "slot_tokens_per_s": round(B * n * k / (ms / 1e3), 1),
                   "rounds_ms": [round(x, 2) for x in v]}
    print(json.dumps({"ab": workload, "steps_per_round": args.steps, "rounds": args.ab_rounds,
                      "results": out}), flush=True)


def run_kernel(args):
    """One kernel family on its bench-sized case (the unit an ncu capture covers)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from parallel_eagle_b200 import ops

    c = dict(CONFIG2)
    if args.kernel == "elementwise":
        hbm, _, _, src = _peaks()
        out = {}
        for name, (run, nbytes) in elementwise_cases(c, dev).items():
            # tens of microseconds per launch: replay a captured CUDA graph so the
            # host's per-call overhead does not pace the device
            ms = time_case_graph(run, args.steps, warmup=args.warmup)
            gbs = nbytes / (ms / 1e3) / 1e9
            out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1),
                         "frac_of_hbm": round(gbs / hbm, 3)}
        ops.check_status(dev)
        print(json.dumps({"kernel": "elementwise", "hbm_peak_gbs": hbm, "peak_source": src,
                          "results": out}), flush=True)
        return
    if args.kernel == "swiglu":
        # the step's gate|up projection over one stacked config-2 pass (13312 slot rows):
        # plain GEMM + element-wise SwiGLU against the GEMM with the SwiGLU epilogue
        H, I, M = c["hidden"], c["intermediate"], 13312
        g = torch.Generator(device=dev).manual_seed(19)
        x = torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        gu = torch.empty(M, 2 * I, dtype=torch.bfloat16, device=dev)
        act = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
        flops = 2.0 * M * 2 * I * H
        out = {}
        runs = {"gemm_then_swiglu": lambda: ops.swiglu_fwd(ops.linear(x, w, out=gu), I, out=act),
                "gemm_only": lambda: ops.linear(x, w, out=gu),
                "gemm_only_bn256": lambda: ops.linear(x, w, out=gu, algo=(256 << 8) | (2 << 20)),
                "gemm_only_evict_first": lambda: ops.linear(x, w, out=gu, algo=1 << 22),
                "swiglu_only": lambda: ops.swiglu_fwd(gu, I, out=act)}
        for bn in (0, 256, 512):
            runs[f"fused_bn{bn or 'auto'}"] = (
                lambda bn=bn: ops.linear_swiglu(x, w, I, gu=gu, act=act, algo=bn << 8))
        only = set(args.only.split(",")) if args.only else None
        if only is not None:
            runs = {k: v for k, v in runs.items() if k in only}
        for name, ms in time_variants(runs, args.steps, warmup=args.warmup,
                                      rounds=args.ab_rounds).items():
            out[name] = {"ms": round(ms, 4), "tflops": round(flops / (ms / 1e3) / 1e12, 1)}
        # the q|k|v projection of the same pass: GEMM + rotation kernel vs RoPE epilogue
        nh, nkv, hd = c["n_heads"], c["n_kv_heads"], c["hidden"] // c["n_heads"]
        wq = (torch.randn((nh + 2 * nkv) * hd, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        qkv = torch.empty(M, (nh + 2 * nkv) * hd, dtype=torch.bfloat16, device=dev)
        pos = torch.randint(0, 4096, (M,), generator=g, device=dev)
        cs = ops.rope_table(pos, hd, 10000.0, torch.bfloat16)
        qflops = 2.0 * M * (nh + 2 * nkv) * hd * H
        qruns = {"qkv_gemm_then_rope": lambda: ops.rope_(ops.linear(x, wq, out=qkv), nh + nkv, hd,
                                                         pos, 10000.0),
                 "qkv_gemm_only": lambda: ops.linear(x, wq, out=qkv),
                 "qkv_gemm_only_evict_first": lambda: ops.linear(x, wq, out=qkv, algo=1 << 22),
                 "qkv_fused_rope": lambda: ops.linear_rope(x, wq, cs, (nh + nkv) * hd, hd, out=qkv)}
        if only is not None:
            qruns = {k: v for k, v in qruns.items() if k in only}
        for name, ms in time_variants(qruns, args.steps, warmup=args.warmup,
                                      rounds=args.ab_rounds).items():
            out[name] = {"ms": round(ms, 4), "tflops": round(qflops / (ms / 1e3) / 1e12, 1)}
        ops.check_status(dev)
        print(json.dumps({"kernel": "gate|up + swiglu; q|k|v + rope", "M": M, "N": 2 * I, "K": H,
                          "results": out}), flush=True)
        return
    if args.kernel == "attnfwd":
        # the masked-attention forward over one config-2 sequence's stacked segments, by
        # the share of exponentials taken from the FMA-pipe polynomial (one pair in e)
        from parallel_eagle_b200.engine import segment_bounds

        nh, nkv, hd, k = c["n_heads"], c["n_kv_heads"], c["hidden"] // c["n_heads"], c["max_depth"]
        g = torch.Generator(device=dev).manual_seed(11)
        bounds = segment_bounds(c["n"], c["segments"])
        R = sum(ops.segment_rows(bounds, k))
        qkv = torch.randn(R, (nh + 2 * nkv) * hd, generator=g, device=dev).to(torch.bfloat16)
        q, kk, vv = qkv[:, : nh * hd], qkv[:, nh * hd:(nh + nkv) * hd], qkv[:, (nh + nkv) * hd:]
        flops = 4.0 * hd * nh * attention_pairs(c["n"], k, c["segments"])
        runs = {f"emu{e}": (lambda e=e: ops.attn_fwd_segments(q, kk, vv, nh, nkv, hd, bounds, k,
                                                              algo=(e + 1) << 16))
                for e in (0, 2, 3, 4, 6, 8)}
        out = {n: {"ms": round(ms, 4), "tflops": round(flops / (ms / 1e3) / 1e12, 1)}
               for n, ms in time_variants(runs, args.steps, warmup=args.warmup).items()}
        ops.check_status(dev)
        print(json.dumps({"kernel": "attention forward", "results": out}), flush=True)
        return
    if args.kernel == "lmhead":
        # the fused LM head on all 10240 loss rows of a config-2 sequence (the step's
        # call): one-pass later chunks (default) against every chunk two-pass (algo bit
        # 28), at 32K- and 16K-column chunks, and with forced 256-wide logits tiles
        R, H, V = 10240, c["hidden"], c["vocab"]
        g = torch.Generator(device=dev).manual_seed(13)
        h = torch.randn(R, H, generator=g, device=dev).to(torch.bfloat16)
        W = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        lab = torch.randint(0, V, (R,), generator=g, device=dev)
        loss = torch.zeros(1, device=dev)
        flops = 2.0 * 2 * R * V * H
        out = {}
        variants = {"auto": 0, "two_pass": 1 << 28, "chunk16k": 16 << 8,
                    "chunk16k_two_pass": (16 << 8) | (1 << 28),
                    "logits256_dh512": (1 << 24) | (2 << 26)}
        runs = {n: (lambda b=b: ops.lmhead_ce(h, W, lab, 1e-4, loss, algo=b))
                for n, b in variants.items()}
        for name, ms in time_variants(runs, args.steps, warmup=args.warmup).items():
            out[name] = {"ms": round(ms, 3), "tflops": round(flops / (ms / 1e3) / 1e12, 1)}
        ops.check_status(dev)
        print(json.dumps({"kernel": "lmhead", "R": R, "H": H, "V": V, "results": out}), flush=True)
        return
    case = {"gemm": gemm_case, "attn": attention_case}[args.kernel]
    run, flops, _ = case(c, dev)
    ms = time_case(run, args.steps, warmup=args.warmup)
    ops.check_status(dev)
    print(json.dumps({"kernel": args.kernel, "ms": round(ms, 4),
                      "tflops": round(flops / (ms / 1e3) / 1e12, 1)}), flush=True)


def run_draft(args):
    """The draft path (reference drafter.py:195-269, decode/tree.py:19-57):
    config-2 dims, one context of ``--n`` (default 2048) confirmed tokens, k = 5.
    Times, with CUDA events on the launching stream, ``draft_logits`` (one forward
    over p + k - 1 slots + the LM head on k rows), ``propose_tree`` (k 5, top_k 4,
    max_nodes 20; includes the host beam and its device reads) and the sequential
    baseline ``draft_logits_sequential``; the CPU oracle's ``draft_logits`` on a
    bounded context is reported beside it."""
    from parallel_eagle_b200 import decode, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = dict(CONFIG2)
    p, k = args.n or 2048, c["max_depth"]
    d = build_drafter(c, dev)
    d.eval()
    g = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, c["vocab"], (p,), generator=g, device=dev)
    feats = torch.randn(p, 3 * c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    runs = {
        "draft_logits": lambda: d.draft_logits(ids, feats, k),
        "propose_tree": lambda: decode.propose_tree(d, ids, feats, k, 4, 20),
        "draft_logits_sequential": lambda: d.draft_logits_sequential(ids, feats, k),
    }
    out = {}
    for name, fn in runs.items():
        ms = time_case(fn, args.steps, warmup=args.warmup)
        out[name] = {"ms": round(ms, 3), "draft_tokens_per_s": round(k / (ms / 1e3), 1)}
    ops.check_status(dev)
    line = {"metric": "draft latency (k=5 tokens after a confirmed context)", "unit": "ms",
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config-2 drafter, draft path", "context": p, "k": k},
            "results": out,
            "parallel_vs_sequential": round(out["draft_logits_sequential"]["ms"]
                                            / out["draft_logits"]["ms"], 2)}
    if not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "tests" / "golden"))
        import oracle
        import recipe

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        dims = oracle.OracleDims(hidden=c["hidden"], n_heads=c["n_heads"],
                                 n_kv_heads=c["n_kv_heads"], intermediate=c["intermediate"],
                                 vocab=c["vocab"], num_layers=c["num_layers"], max_depth=k)
        heads = recipe.make_heads(c["vocab"], c["hidden"], 0, 0.0, torch.bfloat16)
        params = oracle.init_params(dims, 0, torch.bfloat16)
        cp = min(p, args.cpu_n)
        cids, cfeats = recipe.make_sequence(cp, c["vocab"], 3 * c["hidden"], 0, 0)
        t0 = time.perf_counter()
        oracle.draft_logits(params, heads, cids, cfeats.to(torch.bfloat16), k, dims)
        sec = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(sec * 1e3, 1), "unit": "ms", "cores": threads,
                                "kind": "port",
                                "sample": f"oracle draft_logits, context {cp}, k {k}, bf16"}
    print(json.dumps(line), flush=True)


def cpu_baseline(args, n=None):
    """The CPU oracle (a port of the reference step) on one bounded sample of the
    workload: one config-2 sequence at reduced length, bf16, all host threads."""
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import oracle
    import recipe

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    c = dict(CONFIG2)
    n = n or args.cpu_n
    dims = oracle.OracleDims(hidden=c["hidden"], n_heads=c["n_heads"], n_kv_heads=c["n_kv_heads"],
                             intermediate=c["intermediate"], vocab=c["vocab"],
                             num_layers=c["num_layers"], max_depth=c["max_depth"])
    dt = torch.bfloat16
    heads = recipe.make_heads(c["vocab"], c["hidden"], 0, 0.0, dt)
    params = oracle.init_params(dims, 0, dt)
    ids, feats = recipe.make_sequence(n, c["vocab"], 3 * c["hidden"], 0, 0)
    feats = feats.to(dt)
    t0 = time.perf_counter()
    oracle.mtp_step(params, heads, ids, feats, dims, num_segments=c["segments"])
    sec = time.perf_counter() - t0
    return {"value": round(n * c["max_depth"] / sec, 2), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"one sequence, n={n} (config 2 dims, K=5, S=4, bf16), {sec:.1f} s",
            "seconds": round(sec, 2)}


REF_BUDGET_S = 420.0  # timed samples of the --impl reference run stop once past this


def run_reference(args):
    """The reference arm: the CPU port of the reference step (pinned to the reference's
    own outputs) on the host cores, on this framework's workload.  Warm-up steps are
    short samples (n = 256: they page in the weights and warm the allocator); each
    timed step is one full sequence of the workload (n = 2048, K 5, S 4, bf16).  Timed
    samples stop early, after at least three, once their total passes REF_BUDGET_S, and
    the line reports how many ran."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    workload, base = WORKLOADS[2]
    c = dict(base)
    for _ in range(max(1, args.warmup)):
        cpu_baseline(args, n=256)
    samples = []
    t0 = time.perf_counter()
    for _ in range(max(1, args.steps)):
        samples.append(cpu_baseline(args, n=c["n"]))
        if len(samples) >= 3 and time.perf_counter() - t0 > REF_BUDGET_S:
            break
    sec = sum(s["seconds"] for s in samples) / len(samples)
    value = c["n"] * c["max_depth"] / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
        "n_gpus": world, "steps": len(samples), "steps_requested": args.steps,
        "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(workload, c, world),
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": samples[0]["cores"],
                         "kind": "port",
                         "sample": "each timed step: " + samples[0]["sample"]},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=None, help="override sequence length")
    ap.add_argument("--batch", type=int, default=None, help="override per-GPU batch")
    ap.add_argument("--cpu-n", type=int, default=2048,
                    help="sequence length of the CPU sample (default: the workload's own n)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end (pinned host inputs) pass; the line carries no e2e")
    ap.add_argument("--config", type=int, choices=[2, 3, 4], default=2,
                    help="BASELINE workload: 2 (default), 3 soft-target loss, 4 14B-class")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 5: peak HBM / throughput over n, K, S (torchrun: DP)")
    ap.add_argument("--sweep-n", default="256,512,1024,2048,4096")
    ap.add_argument("--sweep-k", default="4,8")
    ap.add_argument("--sweep-s", default="1,2,4,8")
    ap.add_argument("--kernel", choices=["gemm", "attn", "attnfwd", "lmhead", "elementwise",
                                         "swiglu"],
                    default=None,
                    help="time one kernel family on its bench-sized case instead of the step")
    ap.add_argument("--ab", default=None,
                    help="comma-separated engine variants to A/B at step level (" +
                    ", ".join(AB_VARIANTS) + ")")
    ap.add_argument("--ab-rounds", type=int, default=4,
                    help="interleaved rounds of --ab and of the --kernel swiglu comparison")
    ap.add_argument("--only", default=None,
                    help="--kernel swiglu: comma-separated subset of its variants")
    ap.add_argument("--draft", action="store_true",
                    help="time the draft path (draft_logits / propose_tree) on config-2 dims")
    args = ap.parse_args(argv)
    if args.ab:
        run_ab(args)
    elif args.draft:
        run_draft(args)
    elif args.sweep:
        run_sweep(args)
    elif args.kernel:
        run_kernel(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
