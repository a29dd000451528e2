"""Host logic of the multi-GPU path, on CPU: the b*h sharding, per-head input
generation, max-over-ranks timing and the gather to rank 0, run as two gloo
ranks (world_size 2) through the same public API step that bench.py times.
On CPU the step takes the reference's math path, so these tests check the
plumbing around the kernels, not the kernels."""

import multiprocessing as mp
import os
import socket
import traceback

import pytest
import torch

from testtimeideas_b200.sharding import gather_heads, head_inputs, head_range, max_over_ranks


@pytest.mark.parametrize("total", [0, 1, 5, 8, 256, 257])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_head_range_partitions_the_heads(total, world):
    parts = [head_range(total, world, r) for r in range(world)]
    assert [h for p in parts for h in p] == list(range(total))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_head_range_rejects_bad_arguments():
    for args in ((4, 0, 0), (4, 2, 2), (4, 2, -1), (-1, 2, 0)):
        with pytest.raises(ValueError):
            head_range(*args)


def test_head_inputs_do_not_depend_on_the_split():
    full = head_inputs(range(0, 5), 16, 8, torch.float32, "cpu", seed=3, scale_in=0.5)
    lo = head_inputs(range(0, 2), 16, 8, torch.float32, "cpu", seed=3, scale_in=0.5)
    hi = head_inputs(range(2, 5), 16, 8, torch.float32, "cpu", seed=3, scale_in=0.5)
    for n in full:
        assert torch.equal(full[n], torch.cat([lo[n], hi[n]], dim=1)), n
    other = head_inputs(range(0, 5), 16, 8, torch.float32, "cpu", seed=4)
    assert not torch.equal(full["q"], other["q"])


def test_single_process_helpers_pass_through():
    x = torch.randn(1, 3, 4, 2)
    assert gather_heads(x, 3) is x
    assert max_over_ranks(2.5) == 2.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, total: int, q: "mp.Queue") -> None:
    try:
        import datetime

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        import bench

        cfg = dict(t=40, d=16, causal=True, scale_in=0.5)
        mine = head_range(total, world, rank)
        x = head_inputs(mine, cfg["t"], cfg["d"], torch.float64, "cpu", seed=11, scale_in=cfg["scale_in"])
        gq, gk, gv = bench.gradgrad_step(x, cfg["causal"])
        slow = max_over_ranks(float(rank + 1) * 1.5)
        full = [gather_heads(r, total) for r in (gq, gk, gv)]
        out = {"rank": rank, "max": slow, "heads": len(mine)}
        if rank == 0:
            ref = bench.gradgrad_step(head_inputs(range(total), cfg["t"], cfg["d"], torch.float64, "cpu", seed=11,
                                                  scale_in=cfg["scale_in"]), cfg["causal"])
            out["shape"] = tuple(full[0].shape)
            out["err"] = max(float((a - b).abs().max()) for a, b in zip(full, ref))
        else:
            out["none_elsewhere"] = all(f is None for f in full)
        dist.barrier()
        dist.destroy_process_group()
        q.put(out)
    except Exception:  # reported to the parent, which fails the test
        q.put({"rank": rank, "error": traceback.format_exc()})


@pytest.mark.parametrize("total", [4, 5])
def test_gloo_world2_sharded_step_matches_unsharded(total):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r = q.get(timeout=240)
            results[r["rank"]] = r
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    for r in results.values():
        assert "error" not in r, r["error"]
    assert results[0]["max"] == results[1]["max"] == 3.0
    assert results[0]["heads"] + results[1]["heads"] == total
    assert results[0]["shape"] == (1, total, 40, 16)
    assert results[0]["err"] < 1e-12
    assert results[1]["none_elsewhere"]
