"""Data-parallel training step on two GPUs (NCCL): the gradient all-reduce that
overlaps the last local sequence's backward (``train.OverlappedAllReduce``) must give
the same summed gradient as one process accumulating every sequence.

Needs at least two visible GPUs; skipped otherwise.  The ranks are child processes
with a short process-group timeout, so a rank that fails ends the other's collective
with an error instead of a hang.
"""

from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs two CUDA devices", allow_module_level=True)

import torch.multiprocessing as mp  # noqa: E402

from gpu_harness import build_drafter, make_case, recipe  # noqa: E402

DIMS = dict(hidden=512, n_heads=4, n_kv_heads=2, intermediate=1024, vocab=4096,
            num_layers=1, max_depth=3, n=96)
PER_RANK = 2


def _rank_main(rank: int, world: int, port: int, out_path: str) -> None:
    import datetime

    import torch.distributed as dist

    from parallel_eagle_b200.engine import engine_for
    from parallel_eagle_b200.partition import mtp_backward
    from parallel_eagle_b200.train import OverlappedAllReduce

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        case = make_case(**DIMS, dtype=torch.bfloat16, seed=3, batch=world * PER_RANK)
        model = build_drafter(case, device=dev)
        nseq = len(case["seqs"])
        overlap = OverlappedAllReduce(model)
        mine = [case["seqs"][i] for i in range(rank, nseq, world)]
        model.zero_grad(set_to_none=True)
        for j, (ids, feats) in enumerate(mine):
            if j == len(mine) - 1:
                overlap.arm()
            mtp_backward(model, ids, feats, num_segments=2, loss_scale=1.0 / nseq)
        overlap.finish()
        dp = {n: p.grad.float().cpu().clone() for n, p in model.named_parameters()
              if p.requires_grad}
        if rank == 0:
            # one process, every sequence, no collective
            ref_model = build_drafter(case, device=dev)
            ref_model.zero_grad(set_to_none=True)
            for ids, feats in case["seqs"]:
                mtp_backward(ref_model, ids, feats, num_segments=2, loss_scale=1.0 / nseq)
            ref = {n: p.grad.float().cpu().clone() for n, p in ref_model.named_parameters()
                   if p.requires_grad}
            errs = {n: recipe.rel_fro(dp[n], ref[n]) for n in ref}
            torch.save(errs, out_path)
        assert engine_for(model).after_layers is None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_overlapped_allreduce_matches_single_process(tmp_path):
    out = str(tmp_path / "errs.pt")
    port = 29600 + os.getpid() % 300
    mp.spawn(_rank_main, args=(2, port, out), nprocs=2, join=True)
    errs = torch.load(out)
    worst = max(errs.values())
    assert worst < 2e-2, errs  # bf16 gradients, different summation order
