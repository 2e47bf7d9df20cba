"""Train the parallel drafter on cached target features (B200 build).

Same loop, CLI, checkpoint/resume files and log lines as the reference
``pe.train`` (``src/pe/train.py:45-211``): per-sequence ``mtp_backward`` with
``loss_scale = 1/grad_accum``, an update every ``grad_accum`` sequences with
linear warmup/decay LR, global-norm clip 1.0 and AdamW, mid-epoch checkpoints
every ``save_every`` updates written atomically, and resume guarded by a config
signature.

Additions for B200: data parallelism (one process per GPU, ``torch.distributed``
over NCCL; each rank trains the sequences ``i % world == rank`` of every update
and the flat gradient buffer is all-reduced before the step, which reproduces
the single-GPU update), and a fused clip + AdamW kernel over the flat
parameter buffer.
"""

from __future__ import annotations

import argparse
import math
from pathlib import Path

import torch

from . import ops
from .config import DrafterConfig, TargetConfig, TrainConfig
from .drafter import ParallelDrafter
from .features import FeatureDataset
from .partition import mtp_backward
from .target import load_heads_from_dump, load_target_heads

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


class FusedAdamW(torch.optim.Optimizer):
    """AdamW (decoupled weight decay, bias-corrected moments, fp32 moments) whose
    update runs in one libpe_b200 kernel per contiguous parameter buffer.

    ``max_norm`` > 0 fuses ``clip_grad_norm_(params, max_norm)`` into the same
    pass: the squared gradient norm is reduced on the device and the clipping
    coefficient is applied inside the update kernel (no host sync).
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2,
                 max_norm: float = 0.0):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, max_norm=max_norm)
        super().__init__(params, defaults)
        for g in self.param_groups:
            for p in g["params"]:
                if not p.is_cuda:
                    raise ops.L.PeError("FusedAdamW runs on CUDA parameters only")

    @staticmethod
    def _runs(params):
        """Group parameters into runs that are contiguous in one storage (the flat
        buffer of the step engine) with gradients contiguous the same way."""
        items = sorted(
            ((p.data_ptr(), p) for p in params if p.grad is not None), key=lambda t: t[0]
        )
        runs, cur = [], []
        for ptr, p in items:
            if cur:
                last = cur[-1]
                same = (p.untyped_storage().data_ptr() == last.untyped_storage().data_ptr()
                        and p.grad.untyped_storage().data_ptr() == last.grad.untyped_storage().data_ptr())
                if not same:
                    runs.append(cur)
                    cur = []
            cur.append(p)
        if cur:
            runs.append(cur)
        return runs

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            dev = params[0].device
            sumsq = None
            if group["max_norm"] and group["max_norm"] > 0:
                sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
                for p in params:
                    ops.sumsq_into(p.grad, sumsq)
            b1, b2 = group["betas"]
            for run in self._runs(params):
                first, last = run[0], run[-1]
                esz = first.element_size()
                n = (last.data_ptr() - first.data_ptr()) // esz + last.numel()
                gspan = (last.grad.data_ptr() - first.grad.data_ptr()) // esz + last.numel()
                # one kernel over the whole run when params and grads share the same
                # offsets (padding between slices has zero gradient and is untouched data)
                fused = gspan == n and all(
                    p.data_ptr() - first.data_ptr() == p.grad.data_ptr() - first.grad.data_ptr()
                    for p in run
                )
                targets = [run] if fused else [[p] for p in run]
                for tgt in targets:
                    key = tgt[0]
                    st = self.state[key]
                    cnt = n if fused else key.numel()
                    if "m" not in st:
                        st["m"] = torch.zeros(cnt, dtype=torch.float32, device=dev)
                        st["v"] = torch.zeros(cnt, dtype=torch.float32, device=dev)
                        st["step"] = 0
                    st["step"] += 1
                    pv = torch.as_strided(key, (cnt,), (1,)) if fused else key.view(-1)
                    gv = torch.as_strided(key.grad, (cnt,), (1,)) if fused else key.grad.view(-1)
                    ops.adamw_step(pv, gv, st["m"], st["v"], sumsq, group["max_norm"] or 0.0,
                                   group["lr"], b1, b2, group["eps"], group["weight_decay"],
                                   st["step"])
        return loss


def build_optimizer(params, lr: float, weight_decay: float, use_8bit: bool, max_norm: float = 1.0):
    """Reference ``train.py:26-34``: 8-bit Adam when bitsandbytes is present,
    otherwise AdamW -- here the fused AdamW kernel with the clip folded in."""
    params = list(params)
    if use_8bit:
        try:
            import bitsandbytes as bnb

            return bnb.optim.AdamW8bit(params, lr=lr, weight_decay=weight_decay)
        except Exception as exc:  # noqa: BLE001
            print(f"8-bit Adam unavailable ({exc}); falling back to AdamW")
    return FusedAdamW(params, lr=lr, weight_decay=weight_decay, max_norm=max_norm)


def lr_at(step: int, total: int, peak: float, warmup_ratio: float) -> float:
    """Linear warmup then linear decay (reference ``train.py:37-42``)."""
    warmup = max(1, int(total * warmup_ratio))
    if step < warmup:
        return peak * step / warmup
    progress = (step - warmup) / max(1, total - warmup)
    return peak * max(0.0, 1.0 - progress)


def _world():
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        return torch.distributed.get_world_size(), torch.distributed.get_rank()
    return 1, 0


def allreduce_gradients(drafter) -> None:
    """SUM-all-reduce the drafter's gradients across ranks (one contiguous
    buffer when the step engine owns them)."""
    world, _ = _world()
    if world == 1:
        return
    eng = getattr(drafter, "_engine", None)
    if eng is not None and eng.flat.valid():
        torch.distributed.all_reduce(eng.flat.grad)
        return
    for p in drafter.trainable_parameters():
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        torch.distributed.all_reduce(p.grad)


class OverlappedAllReduce:
    """Data-parallel gradient reduction overlapped with backward.  Armed before a
    rank's last local sequence of an update: the decoder layers' region of the flat
    gradient buffer starts its NCCL all-reduce (asynchronously, on NCCL's stream) as
    soon as the step engine reports those gradients final, while the input
    projections' backward still runs; ``finish`` then reduces the input projections'
    region and waits.  Every rank issues the same two collectives in the same order
    (layers, then inputs) whether or not its hook fired."""

    def __init__(self, drafter):
        from .engine import engine_for

        self.eng = engine_for(drafter)
        self.work = None

    def arm(self) -> None:
        eng = self.eng
        o0, o1 = eng.layer_grad_region()

        def launch():
            self.work = torch.distributed.all_reduce(eng.flat.grad[o0:o1], async_op=True)

        eng.after_layers = launch

    def finish(self) -> None:
        eng = self.eng
        eng.after_layers = None
        o0, o1 = eng.layer_grad_region()
        if self.work is None:
            torch.distributed.all_reduce(eng.flat.grad[o0:o1])
        torch.distributed.all_reduce(eng.flat.grad[:o0])
        if self.work is not None:
            self.work.wait()
            self.work = None


def train(tcfg: TargetConfig, dcfg: DrafterConfig, tr: TrainConfig, dtype: str = "float32",
          on_save=None):
    """Train the drafter on cached features (reference ``train.py:45-173``).
    ``on_save`` runs after every checkpoint write."""
    torch.manual_seed(tr.seed)
    param_dtype = _DTYPES[dtype]
    world, rank = _world()

    # shards are read into page-locked memory on CUDA runs, so each sequence's
    # host->device copy is an asynchronous DMA on the step's stream
    on_cuda = torch.device(tcfg.device).type == "cuda"
    data = FeatureDataset(tr.feature_cache_dir, with_prompt_len=True, pin_memory=on_cuda)
    if data.self_distilled:
        print("self-distilled cache detected — masking prompt region out of the loss")
    if data.heads_dump.exists():
        heads = load_heads_from_dump(data.heads_dump, tcfg, data.feature_layers)
    else:
        heads = load_target_heads(tcfg)
    if data.feature_dim != heads.feature_dim:
        raise ValueError(
            f"cached feature_dim {data.feature_dim} != target feature_dim {heads.feature_dim}; "
            "regenerate the feature cache for this target."
        )

    drafter = ParallelDrafter.from_target(heads, dcfg).to(tcfg.device, param_dtype)
    drafter.grad_checkpoint = tr.grad_checkpoint
    drafter.train()

    opt = build_optimizer(drafter.trainable_parameters(), tr.lr, tr.weight_decay, tr.use_8bit_adam)
    fused_clip = isinstance(opt, FusedAdamW)
    # data-parallel runs on CUDA overlap the gradient all-reduce with the backward
    overlap = (OverlappedAllReduce(drafter)
               if world > 1 and drafter.device.type == "cuda" else None)
    total_updates = max(1, math.ceil(len(data) * tr.epochs / tr.grad_accum))

    Path(tr.out_dir).mkdir(parents=True, exist_ok=True)
    ckpt = Path(tr.out_dir) / "drafter.pt"
    state_path = Path(tr.out_dir) / "train_state.pt"
    config_sig = f"{dcfg.num_layers}|{dcfg.max_depth}|{tr.epochs}|{tcfg.model_name}"
    update, micro, running = 0, 0, 0.0

    def save_state(next_epoch: int, consumed: int) -> None:
        """Atomically persist model + position (temp file + rename), then ``on_save``."""
        if rank == 0:
            tmp_ckpt = ckpt.with_suffix(".tmp")
            drafter.save_checkpoint(tmp_ckpt, target_name=tcfg.model_name)
            tmp_ckpt.replace(ckpt)
            tmp_state = state_path.with_suffix(".tmp")
            torch.save({"config_sig": config_sig, "epoch": next_epoch, "consumed": consumed,
                        "update": update}, tmp_state)
            tmp_state.replace(state_path)
        if world > 1:
            torch.distributed.barrier()
        if on_save is not None:
            on_save()

    start_epoch, start_consumed = 0, 0
    if state_path.exists() and ckpt.exists():
        st = torch.load(state_path, map_location="cpu", weights_only=False)
        if st.get("config_sig") == config_sig:
            saved = torch.load(ckpt, map_location="cpu", weights_only=False)
            drafter.load_state_dict(saved["state_dict"])
            start_epoch, start_consumed, update = st["epoch"], st["consumed"], st["update"]
            print(f"resuming: epoch {start_epoch}, {start_consumed} examples in, "
                  f"update {update}/{total_updates}", flush=True)
        else:
            print("existing checkpoint is for a different run — starting fresh", flush=True)

    opt.zero_grad(set_to_none=True)

    for epoch in range(start_epoch, tr.epochs):
        consumed = start_consumed if epoch == start_epoch else 0
        to_skip = consumed
        for input_ids, features, prompt_len, labels in data:
            if to_skip > 0:
                to_skip -= 1
                continue
            consumed += 1
            input_ids = input_ids[: tr.max_seq_len]
            features = features[: tr.max_seq_len]
            if labels is not None:
                labels = labels[: tr.max_seq_len]
            if input_ids.shape[0] < 2:
                continue

            if micro % world == rank:
                # last sequence of this update on this rank: overlap the reduction
                boundary = (micro // tr.grad_accum + 1) * tr.grad_accum
                if overlap is not None and micro + world >= boundary:
                    overlap.arm()
                running += mtp_backward(
                    drafter, input_ids, features, tr.num_segments,
                    loss_scale=1.0 / tr.grad_accum,
                    prompt_len=min(prompt_len, input_ids.shape[0]),
                    teacher_labels=labels,
                )
            micro += 1
            if micro % tr.grad_accum != 0:
                continue

            if overlap is not None:
                overlap.finish()
            else:
                allreduce_gradients(drafter)
            for g in opt.param_groups:
                g["lr"] = lr_at(update, total_updates, tr.lr, tr.warmup_ratio)
            if not fused_clip:
                torch.nn.utils.clip_grad_norm_(drafter.trainable_parameters(), 1.0)
            opt.step()
            opt.zero_grad(set_to_none=True)
            update += 1
            if update % tr.log_every == 0:
                avg = running / (tr.grad_accum * tr.log_every)
                print(f"epoch {epoch} update {update}/{total_updates} loss {avg:.4f}", flush=True)
                running = 0.0
            if tr.save_every and update % tr.save_every == 0:
                save_state(epoch, consumed)

        save_state(epoch + 1, 0)
        print(f"saved {ckpt} after epoch {epoch}", flush=True)

    return drafter


def _parse():
    d, t = DrafterConfig(), TrainConfig()
    p = argparse.ArgumentParser(description="Train the parallel drafter on cached features.")
    p.add_argument("--target", default=TargetConfig().model_name)
    p.add_argument("--device", default=TargetConfig().device)
    p.add_argument("--dtype", default="float32", choices=list(_DTYPES))
    p.add_argument("--cache-dir", default=str(t.feature_cache_dir))
    p.add_argument("--out-dir", default=str(t.out_dir))
    p.add_argument("--num-layers", type=int, default=d.num_layers)
    p.add_argument("--max-depth", type=int, default=d.max_depth, help="K_train")
    p.add_argument("--max-seq-len", type=int, default=t.max_seq_len)
    p.add_argument("--epochs", type=int, default=t.epochs)
    p.add_argument("--lr", type=float, default=t.lr)
    p.add_argument("--grad-accum", type=int, default=t.grad_accum)
    p.add_argument("--num-segments", type=int, default=t.num_segments)
    p.add_argument("--no-8bit-adam", action="store_true")
    p.add_argument("--no-grad-checkpoint", action="store_true")
    return p.parse_args()


def main():
    import os

    a = _parse()
    device = a.device
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        device = f"cuda:{local}"
        torch.distributed.init_process_group("nccl", device_id=torch.device(device))
    tcfg = TargetConfig(model_name=a.target, device=device, dtype=a.dtype)
    dcfg = DrafterConfig(num_layers=a.num_layers, max_depth=a.max_depth)
    tr = TrainConfig(feature_cache_dir=Path(a.cache_dir), out_dir=Path(a.out_dir),
                     max_seq_len=a.max_seq_len, epochs=a.epochs, lr=a.lr, grad_accum=a.grad_accum,
                     num_segments=a.num_segments, use_8bit_adam=not a.no_8bit_adam,
                     grad_checkpoint=not a.no_grad_checkpoint)
    train(tcfg, dcfg, tr, dtype=a.dtype)
    if torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
