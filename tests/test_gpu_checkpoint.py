"""A reference-written checkpoint (tests/golden/*.azn, the reference's
saveNetwork) loaded by the engine's loader straight into a GPU pass: the
outputs equal the pass on the same network built from its seed (bitwise)
and match the reference's float forward within the tf32x3 gate."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name,seed", [("ckpt_9x9_b2_f16.azn", 5), ("ckpt_9x9_h8_b1_f8_own.azn", 6)])
def test_checkpoint_into_the_engine(engine, oracle, name, seed):
    O = oracle
    desc, params, buffers = engine.load_checkpoint(os.path.join(GOLDEN, name))
    cfg = O.NetConfig(desc.board, desc.history, desc.blocks, desc.filters, desc.value_hidden, bool(desc.ownership))
    x = O.random_planes(cfg, 77, 9)
    with engine.CudaInference(desc, params, buffers, 16, 0, engine.TF32X3) as net:
        got = net.infer(x)
    p2, b2 = O.make_network(cfg, seed, O.KIND_TEST)
    with engine.CudaInference(engine.NetDesc.of(cfg), p2, b2, 16, 0, engine.TF32X3) as net:
        same = net.infer(x)
    for a, b in zip(got, same):
        if a is not None:
            assert np.array_equal(a, b)
    lr, vr, orf = O.forward(cfg, params, buffers, x)
    assert O.max_err(got[0], lr) <= 1e-4
    assert np.max(np.abs(got[1] - vr)) <= 1e-4
    if cfg.ownership:
        assert np.max(np.abs(got[2] - orf)) <= 1e-4
