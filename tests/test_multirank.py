"""Multi-process sharding / verification-gather logic on CPU ranks (gloo, world_size 2).

The GPU path shards (batch, head) slices across ranks with no collective on the forward path and
gathers a sample of outputs to rank 0 for verification (cmpext3.sharding).  Here the same helpers
run on CPU ranks with the gloo backend, with the per-shard attention computed by the reference's
CPU path, so no GPU can hang.  Failure cases are made on the host: a rank that raises before the
collective, which the surviving rank must see as an error within its process-group timeout.
"""
from __future__ import annotations

import json
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from cmpext3 import sharding

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, outdir: str, mode: str) -> None:
    sys.path[:0] = [str(ROOT / "torch-cmp-patch_b200"), str(ROOT)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch.distributed as dist
    from cmpext3 import sharding as S
    from oracle import reference_path as RP
    result = {"rank": rank}
    try:
        S.init_process_group("gloo", timeout_s=8 if mode == "fail" else 60)
        B, H, L, D = 4, 3, 40, 16
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(B, H, L, D, generator=g) for _ in range(3))
        b0, b1 = S.shard_range(B, rank, world)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the verification gather")
        local = RP.sdpa(q[b0:b1], k[b0:b1], v[b0:b1], is_causal=True)  # this rank's shard
        samples = torch.stack([local[0, 0], local[-1, -1]])
        got = S.gather_samples(samples)
        t = S.max_over_ranks(float(rank + 1))
        per_rank = S.gather_floats([rank, 10.0 * rank + 0.5])
        if rank == 0:
            result["per_rank"] = per_rank
        if rank == 0:
            full = RP.sdpa(q, k, v, is_causal=True)
            per = B // world
            want = torch.stack([torch.stack([full[r * per, 0], full[r * per + per - 1, H - 1]])
                                for r in range(world)])
            result["gather_ok"] = bool(torch.allclose(got, want, atol=1e-6))
        result["max"] = t
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        result["error"] = f"{type(exc).__name__}: {exc}"
        result["trace"] = traceback.format_exc(limit=3)
    Path(outdir, f"rank{rank}.json").write_text(json.dumps(result))
    if "error" in result:
        os._exit(3)


def _run(world: int, mode: str, tmp_path) -> dict:
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            p.join()
    out = {}
    for r in range(world):
        f = Path(tmp_path, f"rank{r}.json")
        out[r] = json.loads(f.read_text()) if f.exists() else {"missing": True}
        out[r]["exitcode"] = procs[r].exitcode
    return out


def test_shard_range_partitions_exactly():
    for n in (1, 7, 64, 2048):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)


def test_sample_units_is_seeded_and_in_range():
    a = sharding.sample_units(10, 50, 6, seed=3)
    assert a == sharding.sample_units(10, 50, 6, seed=3)
    assert len(a) == 6 and a[0] == 10 and a[-1] == 49 and all(10 <= x < 50 for x in a)
    assert sharding.sample_units(0, 3, 10, seed=0) == [0, 1, 2]


def test_two_ranks_shard_and_gather(tmp_path):
    res = _run(2, "ok", tmp_path)
    assert all("error" not in res[r] for r in res), res
    assert res[0]["gather_ok"] is True
    assert res[0]["max"] == 2.0 and res[1]["max"] == 2.0
    assert res[0]["per_rank"] == [[0.0, 0.5], [1.0, 10.5]]


def test_rank_failure_is_seen_by_the_survivor(tmp_path):
    res = _run(2, "fail", tmp_path)
    assert "rank 1 fails" in res[1].get("error", "")
    assert res[1]["exitcode"] == 3
    # rank 0 must not hang: its collective ends with an error (timeout / peer closed) in bounded time
    assert "error" in res[0], res[0]
