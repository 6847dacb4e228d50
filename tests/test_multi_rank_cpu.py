"""The multi-GPU path's host logic on two CPU ranks (``gloo``, world size 2,
rendezvous on 127.0.0.1): independent inferences sharded by rank, each rank
running ``GpuSimulator`` on its own units (kernel calls replayed on the
oracle's CPU job models, ``tests/cpu_replay.py``), and the verification step
``bench.py`` runs after its timed regions — every rank's first unit and its
sampled MatMul-sweep grids gathered to rank 0 (``all_gather_into_tensor``),
where the CPU oracle checks them.  A mistake planted in rank 0's copy of the
oracle's answer for rank 1's unit must be reported as one mismatching unit."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, outq):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from cormorant_b200 import workloads as WL
        from oracle import graph as og
        from oracle import spec
        from tests.cpu_replay import install
        sim_cls = install(setattr)
        res = {}
        # the sharded model: a global batch of 2 BERT sequences (2 layers x 32 tokens), one per rank
        B = 1
        build = lambda b, first: WL.bert_base(seed=17, batch=b, seq=32, layers=2, first=first)  # noqa: E731
        g, feeds, _ = build(B, rank * B)
        sim = sim_cls(g, fuse=False, device="cpu")  # the replay has no fused epilogue jobs
        raw = {t.onnx_name: sim._to_raw(t, feeds[t.onnx_name]) for t in g.input_tensors}
        out_t = g.output_tensors[0]
        out, _ = sim.forward_raw(raw, keep=[out_t.onnx_name])
        unit = out[out_t.onnx_name][:out_t.numel // B]

        def check(r, got, plant=False):
            g1, f1, _ = build(1, r * B)
            ref = og.forward(g1, f1)[g1.output_tensors[0].onnx_name].reshape(-1).copy()
            if plant and r == 1:
                ref[3] += 1  # the planted mistake: in the oracle's answer, on the CPU
            return bool(np.array_equal(got, ref))
        res["units"] = bench._verify_units(torch, dist, world, rank, unit, check)
        res["units_planted"] = bench._verify_units(torch, dist, world, rank, unit,
                                                   lambda r, got: check(r, got, plant=True))
        # distinct units per rank: rank 0 holds two different outputs
        got = bench._gather_to_root(torch, dist, world, rank, unit.to(torch.int32).contiguous())
        res["distinct"] = (not bool(torch.equal(got[0], got[1]))) if rank == 0 else None
        # the sweep check on small problems, each rank with its own operands
        probs = [(1, 3, 64, 32), (2, 40, 96, 24), (16, 8, 512, 256)]
        gen = torch.Generator().manual_seed(100 + rank)
        bufs = []
        for b, m, k, n in probs:
            A = torch.randint(-256, 256, (b * m * k,), dtype=torch.int16, generator=gen)
            Bm = torch.randint(-256, 256, (b * k * n,), dtype=torch.int16, generator=gen)
            C = torch.from_numpy(spec.matmul_raw(A.numpy().reshape(b, m, k), Bm.numpy().reshape(b, k, n))
                                 .astype(np.int16).reshape(-1).copy())
            bufs.append((A, Bm, C))
        res["sweep"] = bench.sweep_parity(torch, probs, bufs, torch.device("cpu"), rank, world, dist)
        outq.put((rank, res))
    except Exception:  # the parent fails at once with the rank's traceback
        import traceback
        outq.put((rank, {"error": traceback.format_exc()}))
        raise
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_gather_verify():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, res = q.get(timeout=300)
            assert "error" not in res, res.get("error")
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    r0 = got[0]
    assert r0["units"] == {"units_checked": 2, "mismatching_units": 0, "ranks_checked": [0, 1]}
    assert r0["units_planted"]["mismatching_units"] == 1
    assert r0["distinct"]
    sw = r0["sweep"]
    assert sw["ranks"] == 2 and sw["problems"] == 3 and sw["mismatches"] == 0 and sw["checked"] > 0
    assert got[1]["units"] is None and got[1]["sweep"] is None  # only rank 0 checks
