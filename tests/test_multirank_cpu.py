"""Multi-rank host logic on CPU: the unit split, the cross-rank parameter-gradient sum and the
max-over-ranks timing rule, run as world_size-2 ``gloo`` process groups; and ``bench.py``'s
reference arm under ``torch.distributed.run`` (rank 0 alone prints).

The attention itself is the float64 oracle here (no GPU): each rank computes its shard, the
shards are gathered, and the result must equal the oracle on the whole problem.
"""
from __future__ import annotations

import itertools
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import flash_born_oracle as fo
from quantumdlblocks_b200 import sharding

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ------------------------------------------------------------------------------ plans (no ranks)


@pytest.mark.parametrize("B,H,world", [(8, 16, 1), (8, 16, 2), (8, 16, 8), (4, 3, 2), (5, 7, 3), (2, 6, 4)])
def test_plan_covers_every_unit_once(B, H, world):
    T = 40
    rng = np.random.default_rng(B * 100 + H)
    doc = np.sort(rng.integers(0, 4, (B, T)), axis=1).astype(np.int32)
    try:
        plan = sharding.plan_shards(B, H, T, world, doc_ids=doc)
    except ValueError:
        assert H % world != 0 and B < world
        return
    assert [s.rank for s in plan] == list(range(world))
    seen = np.zeros((B, H), dtype=np.int64)
    for s in plan:
        seen[s.b0:s.b1, s.h0:s.h1] += 1
        assert s.units > 0
    assert (seen == 1).all()
    total = sum(fo.count_valid_pairs(T, True, 0, doc[b]) for b in range(B)) * H
    assert sum(s.pairs for s in plan) == total
    if H % world == 0:
        assert len({s.pairs for s in plan}) == 1  # a head split is exactly balanced


def test_plan_refuses_unsplittable_grid():
    with pytest.raises(ValueError, match="cannot split"):
        sharding.plan_shards(2, 3, 16, 4)


@pytest.mark.parametrize("window,causal", [(0, True), (0, False), (5, True), (5, False)])
def test_row_valid_pairs_match_oracle_count(window, causal):
    T = 37
    rng = np.random.default_rng(window + 7 * causal)
    doc = rng.integers(0, 3, (3, T)).astype(np.int32)  # unsorted ids too
    got = sharding.row_valid_pairs(3, T, causal, window, doc)
    want = [fo.count_valid_pairs(T, causal, window, doc[b]) for b in range(3)]
    assert got.tolist() == want
    got_nd = sharding.row_valid_pairs(2, T, causal, window, None)
    assert got_nd.tolist() == [fo.count_valid_pairs(T, causal, window, None)] * 2


def test_linear_partition_is_optimal():
    rng = np.random.default_rng(0)
    for _ in range(30):
        n = int(rng.integers(2, 8))
        parts = int(rng.integers(1, n + 1))
        costs = rng.integers(1, 50, n).astype(np.int64)
        got = sharding._linear_partition(costs, parts)
        assert got[0][0] == 0 and got[-1][1] == n and all(a[1] == b[0] for a, b in zip(got, got[1:]))
        assert all(b > a for a, b in got)
        best = min(
            max(costs[a:b].sum() for a, b in zip((0,) + cuts, cuts + (n,)))
            for cuts in itertools.combinations(range(1, n), parts - 1))
        assert max(costs[a:b].sum() for a, b in got) == best


# ------------------------------------------------------------------------------ gloo ranks


def _problem(B, H, T, D, with_doc):
    rng = np.random.default_rng(11)
    q, k, v, do = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    scale = rng.uniform(0.5, 2.0, H)
    doc = np.sort(rng.integers(0, 3, (B, T)), axis=1).astype(np.int32) if with_doc else None
    return q, k, v, do, scale, doc


def _rank_main(rank, world, port, B, H, T, D, with_doc, out_path):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, do, scale, doc = _problem(B, H, T, D, with_doc)
        plan = sharding.plan_shards(B, H, T, world, doc_ids=doc)
        me = plan[rank]
        tq, tk, tv, tdo = (torch.from_numpy(x) for x in (q, k, v, do))
        sq, sk, sv, ssc, sdoc = sharding.shard_inputs(me, tq, tk, tv, torch.from_numpy(scale), None if doc is None
                                                      else torch.from_numpy(doc))
        sdo = tdo[me.b0:me.b1, me.h0:me.h1]
        sdoc_np = None if sdoc is None else sdoc.numpy()
        out, z = fo.born_forward(sq.numpy(), sk.numpy(), sv.numpy(), ssc.numpy(), True, 1e-12, 0, sdoc_np)
        g = fo.born_backward(sq.numpy(), sk.numpy(), sv.numpy(), out, z, sdo.numpy(), ssc.numpy(), True, 0, sdoc_np)
        # assemble the full tensors: every rank adds its rectangle into zeros, one all-reduce each
        full = {}
        for name, part in (("out", out), ("dq", g.dq), ("dk", g.dk), ("dv", g.dv)):
            t = torch.zeros(B, H, T, D, dtype=torch.float64)
            t[me.b0:me.b1, me.h0:me.h1] = torch.from_numpy(part)
            dist.all_reduce(t)
            full[name] = t.numpy()
        dscale = sharding.gather_param_grad(torch.from_numpy(g.dscale), me, H).numpy()
        shared = sharding.gather_param_grad(torch.tensor([g.dscale.sum()]), me, H, per_head=False).numpy()
        times = sharding.max_over_ranks([1.0 + rank, 10.0 - rank])
        if rank == 0:
            np.savez(out_path, dscale=dscale, shared=shared, times=np.array(times), **full)
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("B,H,with_doc", [(2, 4, False), (4, 3, True)], ids=["head-split", "batch-split-doc"])
def test_gloo_two_ranks_shards_equal_whole_problem(tmp_path, B, H, with_doc):
    import torch.multiprocessing as mp

    T, D, world = 24, 8, 2
    out_path = str(tmp_path / "r0.npz")
    mp.spawn(_rank_main, args=(world, _free_port(), B, H, T, D, with_doc, out_path), nprocs=world, join=True)
    res = np.load(out_path)
    q, k, v, do, scale, doc = _problem(B, H, T, D, with_doc)
    out, z = fo.born_forward(q, k, v, scale, True, 1e-12, 0, doc)
    g = fo.born_backward(q, k, v, out, z, do, scale, True, 0, doc)
    np.testing.assert_allclose(res["out"], out, rtol=0, atol=1e-12)
    np.testing.assert_allclose(res["dq"], g.dq, rtol=0, atol=1e-10)
    np.testing.assert_allclose(res["dk"], g.dk, rtol=0, atol=1e-10)
    np.testing.assert_allclose(res["dv"], g.dv, rtol=0, atol=1e-10)
    np.testing.assert_allclose(res["dscale"], g.dscale, rtol=1e-12, atol=1e-10)
    np.testing.assert_allclose(res["shared"], [g.dscale.sum()], rtol=1e-12, atol=1e-10)
    assert res["times"].tolist() == [2.0, 10.0]  # max over ranks of [1 + r, 10 - r]


def test_bench_reference_arm_two_ranks_rank0_prints_once():
    env = dict(os.environ, FB_REF_STEP_SECONDS="0.2", OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3", "--workload", "c1"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
