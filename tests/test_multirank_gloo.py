"""The multi-GPU host logic on CPU ranks (gloo, world size 2): the weight
replicas broadcast once from rank 0 arrive bit-identical, each rank's
positions are its own slice of one seeded sequence (weak scaling by batch),
the timing reduction takes the maximum over ranks, and self-play split by
game slice across ranks plays the same games as one process playing them
all. The GPU path of the
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
    total = d.sum(float(rank + 1))
    # Self-play by game slice: rank r plays games [3r, 3r + 3) of one
    # generation (the reference's naive engine here; the bench runs the
    # engine's "cuda" backend the same way, one slice per GPU).
    sp_positions = -1.0
    lib = _selfplay_lib()
    if lib:
        import selfplay as SP

        sd = E.NetDesc(5, 1, 1, 8, 16, 0)
        sp_p, sp_b = E.synth_network(sd, 801, 1)
        r = SP.play(sd, sp_p, sp_b, backend="naive", workers=2, simulations=16, temperature_moves=6, seed=802,
                    generation=3, first=3 * rank, count=3, lib_path=lib)
        sp_positions = d.sum(float(r["positions"]))
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), params=params, buffers=buffers, x=x, worst=worst,
             total=total, sp_positions=sp_positions)
    d.close()


def _selfplay_lib():
    for p in (os.path.join(ROOT, "oracle", "_ref", "libazselfplay_ref.so"),
              os.path.join(ROOT, "alphazero-go_b200", "host", "_ref", "libazselfplay.so")):
        if os.path.exists(p):
            return p
    return None


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
        assert float(r["total"]) == 3.0
    lib = _selfplay_lib()
    if lib:
        sys.path.insert(0, os.path.join(ROOT, "alphazero-go_b200"))
        import selfplay as SP

        sd = E.NetDesc(5, 1, 1, 8, 16, 0)
        sp_p, sp_b = E.synth_network(sd, 801, 1)
        whole_sp = SP.play(sd, sp_p, sp_b, backend="naive", workers=2, simulations=16, temperature_moves=6,
                           seed=802, generation=3, first=0, count=6, lib_path=lib)
        assert float(r0["sp_positions"]) == float(whole_sp["positions"]) == float(r1["sp_positions"])
    whole = E.synth_positions(desc, 11, 8)
    assert np.array_equal(r0["x"], whole[:4]) and np.array_equal(r1["x"], whole[4:])
