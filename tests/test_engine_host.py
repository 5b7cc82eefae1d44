"""The engine's host side, without a GPU: the C ABI library loads and exports
every function include/azb200.h declares, its ParamLayout and its seeded
generators agree bit for bit with the oracle (and so with the reference),
and it refuses what the reference's upload refuses, with the reference's
messages (src/cuda/cuda_network.cu:24-41)."""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import azb200 as E
import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_library_exports_every_declared_symbol():
    syms = E.header_symbols()
    assert len(syms) >= 40
    lib = E.lib()
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert E.cuda_built()


@pytest.mark.parametrize("shape", [(5, 1, 4, 32, 64, False), (9, 8, 2, 16, 16, True), (19, 1, 20, 256, 256, False)])
def test_layout_matches_oracle(oracle, shape):
    cfg = O.NetConfig(*shape)
    d = E.NetDesc.of(cfg)
    assert E.layout(d, 0) == O.layout(cfg, 0)
    assert E.layout(d, 1) == O.layout(cfg, 1)
    assert E.arena_floats(d) == O.arena_floats(cfg)


def test_synthetic_data_matches_golden(oracle):
    """The engine's seeded generator reproduces the reference's networks and inputs."""
    with open(os.path.join(GOLDEN, "nets.json")) as f:
        nets = json.load(f)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    for name, case in nets.items():
        c = case["config"]
        cfg = O.NetConfig(c["board"], c["history"], c["blocks"], c["filters"], c["value_hidden"], c["ownership"])
        d = E.NetDesc.of(cfg)
        kind = -1 if case["kind"] is None else case["kind"]
        p, b = E.synth_network(d, case["seed"], kind)
        assert sha(p) == case["sha256"]["params"], name
        assert sha(b) == case["sha256"]["buffers"], name
        if case["inputs"]["kind"] == "positions":
            x = E.synth_positions(d, case["inputs"]["seed"], case["inputs"]["batch"])
            assert sha(x) == case["sha256"]["inputs"], name


def test_synthetic_positions_slices():
    """Rank r's slice of a weak-scaling run is samples [r*B, (r+1)*B) of one sequence."""
    d = E.NetDesc(9, 1, 1, 16, 16, 0)
    whole = E.synth_positions(d, 3, 8)
    assert np.array_equal(E.synth_positions(d, 3, 4, first=4), whole[4:])
    planes = whole.reshape(8, 4, 81)
    assert np.all((planes[:, 2] + planes[:, 3]) == 1)          # exactly one side-to-move plane
    assert np.all(planes[:, 0] + planes[:, 1] <= 1)            # no point holds two stones


def test_workspace_bytes():
    d = E.NetDesc(19, 1, 20, 256, 256, 0)
    small = E.workspace_bytes(d, 8, E.BF16)
    big = E.workspace_bytes(d, 1024, E.BF16)
    assert 0 < small < big
    assert E.workspace_bytes(d, 1024, E.TF32X3) > E.workspace_bytes(d, 1024, E.TF32) > big


def test_bad_shapes_refused():
    params = np.zeros(10, np.float32)
    for desc, msg in [(E.NetDesc(19, 1, 2, 12, 16, 0), "filters"), (E.NetDesc(4, 1, 2, 16, 16, 0), "board"),
                      (E.NetDesc(19, 1, 2, 512, 16, 0), "filters")]:
        with pytest.raises(E.CudaError, match=msg):
            E.CudaInference(desc, params, params, 4)


@pytest.mark.skipif(E.cuda_available(0)[0], reason="a GPU is present")
def test_no_gpu_reports_why():
    ok, why = E.cuda_available(0)
    assert not ok and why
    assert E.cuda_description(0) == why
    d = E.NetDesc(9, 1, 1, 16, 16, 0)
    p, b = E.synth_network(d, 1)
    with pytest.raises(E.CudaError, match="cuda"):
        E.CudaInference(d, p, b, 4)
