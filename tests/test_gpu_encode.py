"""The device encoder (azb_infer_run_stones): position records in, the same
outputs, bit for bit, as the planes the reference's encodePlanes makes from
them (src/encode.cpp:15-43) evaluated by azb_infer_run; history, missing
history, side to move and all eight symmetries covered."""
import numpy as np
import pytest

from test_encode_host import random_records

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,H,precision", [(5, 1, "tf32x3"), (9, 8, "bf16"), (19, 2, "tf32"), (13, 1, "bf16")])
def test_records_equal_encoded_planes(engine, oracle, n, H, precision):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libazref.so is not built")
    E = engine
    cfg = oracle.NetConfig(n, H, 2, 32, 32, True)
    params, buffers = oracle.make_network(cfg, 71, oracle.KIND_TEST)
    _, _, _, _, rec = random_records(E, n, H, 40, 70 + n)
    planes = oracle.ref_encode_records(cfg, rec)
    with E.CudaInference(E.NetDesc.of(cfg), params, buffers, 40, 0, E.PRECISIONS[precision]) as net:
        l1, v1, o1 = net.infer(planes)
        l2, v2, o2 = net.infer_stones(rec)
    assert np.array_equal(l1, l2) and np.array_equal(v1, v2) and np.array_equal(o1, o2)


def test_bench_positions_as_records(engine, oracle):
    """The benchmark's own positions (history 1, no symmetry) through records match the oracle."""
    E, O = engine, oracle
    cfg = O.NetConfig(19, 1, 2, 64, 64, False)
    params, buffers = O.make_network(cfg, 1, O.KIND_BENCH)
    x = O.positions(cfg, 1, 16)
    stones = np.zeros((16, 1, 361), np.uint8)
    to_move = np.where(x[:, 2, 0] == 1.0, 1, 2)
    for b in range(16):
        own, opp = (1, 2) if to_move[b] == 1 else (2, 1)
        stones[b, 0][x[b, 0] == 1.0] = own
        stones[b, 0][x[b, 1] == 1.0] = opp
    rec = E.stones_records(stones, to_move)
    lr, vr, _ = O.forward(cfg, params, buffers, x)
    with E.CudaInference(E.NetDesc.of(cfg), params, buffers, 16, 0, E.TF32X3) as net:
        lg, vg, _ = net.infer_stones(rec)
    assert O.max_err(lg, lr) <= 1e-4 and np.max(np.abs(vg - vr)) <= 1e-4
