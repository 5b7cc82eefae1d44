"""The self-play driver's host logic, on the reference's naive CPU engine.

alphazero-go_b200/host/selfplay_driver.cpp plays a slice the way the
reference's playSelfPlayQueue does (src/selfplay_slice.cpp:93-149): game i's
randomness depends only on i, so the records (hashed in index order) must
not depend on the number of workers (the reference's determinism contract,
include/azgo/selfplay_slice.hpp:85-90). The package build (with the GPU
engine linked in, naive backend here) and the oracle build (the reference's
CPU engines only) must play the same games.
"""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_LIB = os.path.join(ROOT, "alphazero-go_b200", "host", "_ref", "libazselfplay.so")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libazselfplay_ref.so")


def _need(path):
    if not os.path.exists(path):
        pytest.skip(f"{path} is not built (needs the reference tree)")


@pytest.mark.parametrize("shape", [(5, 1, 8, 16), (9, 2, 16, 32)])
def test_slice_independent_of_workers(shape):
    _need(PKG_LIB)
    _need(REF_LIB)
    import azb200 as E
    import selfplay as SP

    d = E.NetDesc(shape[0], 1, shape[1], shape[2], shape[3], 0)
    p, b = E.synth_network(d, 801, 1)
    hashes = set()
    for lib in (PKG_LIB, REF_LIB):
        for workers in (1, 3, 8):
            r = SP.play(d, p, b, backend="naive", workers=workers, simulations=16, mcts_batch=8,
                        temperature_moves=6, seed=802, generation=3, first=10, count=4, lib_path=lib)
            assert r["positions"] > 0 and r["evaluations"] > 0
            hashes.add(r["record_hash"])
    assert len(hashes) == 1


def test_bad_arenas_are_refused():
    _need(REF_LIB)
    import azb200 as E
    import selfplay as SP

    d = E.NetDesc(5, 1, 1, 8, 16, 0)
    p, b = E.synth_network(d, 1, 0)
    with pytest.raises(RuntimeError, match="arena sizes"):
        SP.play(d, p[:-64], b, backend="naive", workers=1, simulations=8, count=1, lib_path=REF_LIB)
    with pytest.raises(RuntimeError):
        SP.play(d, p, b, backend="no-such-engine", workers=1, simulations=8, count=1, lib_path=REF_LIB)


WAVE = [(0, 1, 6, 901), (0, ("bot", 8), 4, 902), (0, 2, 4, 903)]


def _wave_nets(E):
    d = E.NetDesc(5, 1, 1, 8, 16, 0)
    return d, [E.synth_network(d, s, 1) for s in (811, 812, 813)]


def test_arena_wave_independent_of_workers_and_slicing():
    """The reference's arena-wave contract (tests/test_cuda.cpp:1301-1348) on its naive engine: the same
    games for any number of workers, and a wave played in two slices equals the whole wave."""
    _need(REF_LIB)
    import azb200 as E
    import selfplay as SP

    d, nets = _wave_nets(E)
    kw = dict(simulations=16, mcts_batch=4, temperature_moves=2, backend="naive", lib_path=REF_LIB)
    whole = {SP.arena(d, nets, WAVE, first=0, count=14, workers=w, **kw)["record_hash"] for w in (1, 3, 0)}
    assert len(whole) == 1
    a = SP.arena(d, nets, WAVE, first=0, count=5, workers=2, **kw)
    b = SP.arena(d, nets, WAVE, first=5, count=9, workers=2, **kw)
    total = SP.arena(d, nets, WAVE, first=0, count=14, workers=2, **kw)
    assert a["games"] + b["games"] == total["games"]
    assert a["score_a"] + b["score_a"] == total["score_a"]
    assert total["evaluations"] > 0
