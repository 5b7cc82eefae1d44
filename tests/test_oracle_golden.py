"""The CPU oracle, pinned against the reference's own outputs.

tests/golden holds what the reference's code (compiled from its sources, see
tests/golden/make_golden.py) produced for fixed seeds. The oracle's C
restatement must reproduce its generator, its ParamLayout, its seeded
networks and inputs bit for bit, and its naive-backend forward bit for bit
(the naive backend sums each output in one fixed float order,
src/backend.cpp:115-140); its OpenBLAS forward within the reference's own
ceiling of 1e-5 maxErr (tests/test_cuda.cpp:756-776).
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


NETS = load("nets.json")
RNG = load("rng.json")


def cfg_of(case):
    c = case["config"]
    return O.NetConfig(c["board"], c["history"], c["blocks"], c["filters"], c["value_hidden"], c["ownership"])


def inputs_of(case, cfg):
    i = case["inputs"]
    if i["kind"] == "positions":
        return O.positions(cfg, i["seed"], i["batch"])
    return O.random_planes(cfg, i["seed"], i["batch"])


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("seed", list(RNG["seeds"]))
def test_rng_known_answers(oracle, seed):
    ref = RNG["seeds"][seed]
    s = int(seed)
    assert O.rng_sample(s, 0, 8).astype(np.int64).tolist() == ref["next"]
    assert O.rng_sample(s, 1, 8).tolist() == ref["uniform"]
    assert O.rng_sample(s, 2, 8, 7).astype(int).tolist() == ref["below7"]
    assert O.rng_sample(s, 3, 8).tolist() == ref["normal"]


def test_derive_seed(oracle):
    for a, b, c, d, h in RNG["derive"]:
        assert O.derive_seed(a, b, c, d) == int(h)


@pytest.mark.parametrize("name", list(NETS))
def test_layout_weights_inputs(oracle, name):
    case = NETS[name]
    cfg = cfg_of(case)
    assert [list(e) for e in O.layout(cfg, 0)] == case["layout"]["params"]
    assert [list(e) for e in O.layout(cfg, 1)] == case["layout"]["buffers"]
    params, buffers = O.make_network(cfg, case["seed"], case["kind"])
    assert sha(params) == case["sha256"]["params"]
    assert sha(buffers) == case["sha256"]["buffers"]
    assert sha(inputs_of(case, cfg)) == case["sha256"]["inputs"]


@pytest.mark.parametrize("name", list(NETS))
def test_forward_matches_reference(oracle, name):
    case = NETS[name]
    cfg = cfg_of(case)
    params, buffers = O.make_network(cfg, case["seed"], case["kind"])
    x = inputs_of(case, cfg)
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    logits, values, own = O.forward(cfg, params, buffers, x)
    # bit for bit with the naive backend
    assert np.array_equal(logits.view(np.uint32), gold["logits_naive"].view(np.uint32))
    assert np.array_equal(values.view(np.uint32), gold["values_naive"].view(np.uint32))
    if cfg.ownership:
        assert np.array_equal(own.view(np.uint32), gold["ownership_naive"].view(np.uint32))
    # within the reference's own ceiling of OpenBLAS
    assert O.max_err(logits, gold["logits_blas"]) <= 1e-5
    assert np.max(np.abs(values - gold["values_blas"])) <= 1e-5


def test_double_precision_restatement(oracle):
    """doubleInfer (tests/test_cuda.cpp:659-752): the float forward sits within
    float noise of it."""
    for name in ("c1_5x5_b4_f32", "h8_9x9_b2_f16_own"):
        case = NETS[name]
        cfg = cfg_of(case)
        params, buffers = O.make_network(cfg, case["seed"], case["kind"])
        x = inputs_of(case, cfg)
        lf, vf, of = O.forward(cfg, params, buffers, x)
        ld, vd, od = O.forward(cfg, params, buffers, x, "f64")
        assert O.max_err(lf, ld) <= 1e-5
        assert np.max(np.abs(vf - vd)) <= 1e-5


def test_inference_is_per_sample(oracle):
    """A sample's outputs do not depend on its batch (the property the
    inference hub rests on, tests/test_network.cpp:322): bit for bit."""
    cfg = O.NetConfig(9, 1, 2, 16, 32, True)
    params, buffers = O.make_network(cfg, 3, O.KIND_TEST)
    x = O.positions(cfg, 4, 6)
    whole = O.forward(cfg, params, buffers, x)
    for b in (0, 3, 5):
        alone = O.forward(cfg, params, buffers, x[b:b + 1])
        for k in range(3):
            assert np.array_equal(whole[k][b], alone[k][0])


@pytest.mark.skipif(not O.ref_available(), reason="the reference build (oracle/_ref) is not present")
@pytest.mark.parametrize("shape", [(5, 1, 1, 8, 8, False), (7, 2, 1, 24, 16, True), (13, 1, 2, 32, 64, False)])
def test_live_reference(shape):
    """Against the reference itself, on shapes outside the fixtures."""
    cfg = O.NetConfig(*shape)
    ref = O.RefNetwork(cfg, 99, O.KIND_TEST)
    rp, rb = ref.arenas()
    p, b = O.make_network(cfg, 99, O.KIND_TEST)
    assert np.array_equal(rp.view(np.uint32), p.view(np.uint32))
    assert np.array_equal(rb.view(np.uint32), b.view(np.uint32))
    x = O.positions(cfg, 5, 3)
    assert np.array_equal(x, O.ref_positions(cfg, 5, 3))
    ln, vn, on = ref.infer(x, "naive")
    l, v, o = O.forward(cfg, p, b, x)
    assert np.array_equal(l.view(np.uint32), ln.view(np.uint32))
    assert np.array_equal(v.view(np.uint32), vn.view(np.uint32))
