"""Batch x head sharding of attention across the GPUs of one box (one process per GPU).

Each (batch, head) slice of an attention call is independent, so the forward path has no exchange
step: rank r of N owns a contiguous range of the flattened B*H slices and runs the kernel on its own
range with no collective.  A collective appears only after the work, to bring a sample of every
rank's output to rank 0 for verification (``gather_samples``: NCCL all_gather over NVLink on GPUs,
gloo in the CPU tests).

The reference is single-GPU and has no counterpart; its kernels already split work on the same axis
(grid (q-tiles, B*H), src/cuda/fp16_flash_attention_hfma2.cu:258 in the reference).
"""
from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist


def shard_range(n_units: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the units rank ``rank`` owns: contiguous, sizes differing by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sample_units(start: int, stop: int, count: int, seed: int) -> list[int]:
    """``count`` distinct units of [start, stop), seeded: always the first and last unit, the rest
    drawn without replacement."""
    n = stop - start
    if n <= 0 or count <= 0:
        return []
    if count >= n:
        return list(range(start, stop))
    picks = {start, stop - 1}
    g = torch.Generator().manual_seed(seed)
    for i in torch.randperm(n, generator=g).tolist():
        if len(picks) >= count:
            break
        picks.add(start + i)
    return sorted(picks)


def init_process_group(backend: str, timeout_s: float = 120.0) -> tuple[int, int]:
    """Initialise torch.distributed from the torchrun environment (RANK, WORLD_SIZE, MASTER_*)."""
    if not dist.is_initialized():
        kwargs = {"backend": backend, "timeout": timedelta(seconds=timeout_s)}
        if backend == "nccl":
            import os
            kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(**kwargs)
    return dist.get_rank(), dist.get_world_size()


def gather_samples(local: torch.Tensor) -> torch.Tensor | None:
    """All-gather equally shaped per-rank sample tensors; rank 0 gets them stacked [world, ...].

    Used only for verification, after the timed work.  Every rank calls it (a collective); ranks
    other than 0 get None.
    """
    world = dist.get_world_size()
    local = local.contiguous()
    out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local)
    return out.view(world, *local.shape) if dist.get_rank() == 0 else None


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Max of a per-rank scalar (e.g. a device-timed duration) across ranks."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_floats(values, device: torch.device | None = None) -> list[list[float]] | None:
    """All-gather a short per-rank vector of floats (the same length on every rank); rank 0 gets
    one list per rank, in rank order, the others None.  Used after the timed region, to bring
    per-rank records (device time, median SM clock) to the rank that prints the result."""
    world = dist.get_world_size()
    local = torch.tensor([float(x) for x in values], dtype=torch.float64, device=device or "cpu")
    out = torch.empty(world * local.numel(), dtype=torch.float64, device=local.device)
    dist.all_gather_into_tensor(out, local)
    if dist.get_rank() != 0:
        return None
    return out.view(world, -1).cpu().tolist()
