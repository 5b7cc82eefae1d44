"""The reference's own CUDA engine rebuilt for sm_100 (oracle/_ref/libazrefcuda.so,
`make -C oracle refcuda`): the comparison arm. It must run on the B200 and
agree with the CPU oracle as the reference requires of it
(tests/test_cuda.cpp:756-776: maxErr <= 1e-5 against the CPU forward on
small seeded networks), so that its timings are of a correct engine.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rc(engine, oracle):
    if not oracle.refcuda_built():
        pytest.skip("oracle/_ref/libazrefcuda.so is not built (needs the reference tree)")
    ok, why = oracle.refcuda_available()
    assert ok, why
    return oracle


def test_describes_the_b200(rc):
    d = rc.refcuda_description()
    assert "sm_100" in d and "kernels ref100r0" in d, d


@pytest.mark.parametrize("shape", [(5, 1, 8, 16), (9, 2, 16, 32), (19, 2, 32, 64)])
def test_matches_the_cpu_forward(rc, shape):
    O = rc
    c = O.NetConfig(shape[0], 1, shape[1], shape[2], shape[3], False)
    params, buffers = O.make_network(c, 44, O.KIND_TEST)
    x = O.random_planes(c, 45, 16)
    lr, vr, _ = O.forward(c, params, buffers, x)
    with O.RefCudaInference(c, params, buffers, 16) as net:
        lg, vg = net.infer(x)
    assert O.max_err(lg, lr) <= 1e-5, O.max_err(lg, lr)
    assert np.max(np.abs(vg - vr)) <= 1e-5


def test_engine_agrees_with_the_reference_cuda_engine(rc, engine):
    """This engine (TF32X3) and the reference's CUDA engine on the same seeded net and inputs."""
    O = rc
    c = O.NetConfig(19, 1, 3, 64, 64, False)
    params, buffers = O.make_network(c, 46, O.KIND_BENCH)
    x = O.positions(c, 46, 32)
    with O.RefCudaInference(c, params, buffers, 32) as ref_net:
        lr, vr = ref_net.infer(x)
    with engine.CudaInference(engine.NetDesc.of(c), params, buffers, 32, 0, engine.TF32X3) as net:
        lg, vg, _ = net.infer(x)
    assert O.max_err(lg, lr) <= 1e-4
    assert np.max(np.abs(vg - vr)) <= 1e-4
