"""The multi-GPU host logic on CPU ranks (gloo, world size 2): the weight
replicas broadcast once from rank 0 arrive bit-identical, each rank's
positions are its own slice of one seeded sequence (weak scaling by batch),
and the timing reduction takes the maximum over ranks. The GPU path of the
same code runs each rank on its own device over NCCL with no per-step
collective."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path[:0] = [ROOT, os.path.join(ROOT, "alphazero-go_b200")]
    import azb200 as E
    import bench

    d = bench.Dist(world, backend="gloo")
    desc = E.NetDesc(9, 1, 2, 16, 32, 0)
    if d.rank == 0:
        params, buffers = E.synth_network(desc, 11, 0)
    else:
        n_p, n_b = E.arena_floats(desc)
        params, buffers = np.zeros(n_p, np.float32), np.zeros(n_b, np.float32)
    params, buffers = d.broadcast(params), d.broadcast(buffers)
    x = E.synth_positions(desc, 11, 4, first=d.rank * 4)
    d.barrier()
    worst = d.max(float(rank + 1) * 1.5)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), params=params, buffers=buffers, x=x, worst=worst)
    d.close()


def test_two_ranks_gloo(tmp_path):
    import torch.multiprocessing as mp

    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in range(2))
    import azb200 as E

    desc = E.NetDesc(9, 1, 2, 16, 32, 0)
    p, b = E.synth_network(desc, 11, 0)
    for r in (r0, r1):
        assert np.array_equal(r["params"], p) and np.array_equal(r["buffers"], b)
        assert float(r["worst"]) == 3.0
    whole = E.synth_positions(desc, 11, 8)
    assert np.array_equal(r0["x"], whole[:4]) and np.array_equal(r1["x"], whole[4:])
