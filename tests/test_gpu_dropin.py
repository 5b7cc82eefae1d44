"""The drop-in: the reference's own InferenceHub and WorkerEvaluators
(robominds/alphazero-go src/inference_hub.cpp, built from its sources) driving
the engine through alphazero-go_b200/host/azgo_cuda_bridge.cpp, i.e. the
reference's include/azgo/cuda.hpp implemented over include/azb200.h.

Mirrors tests/test_cuda.cpp:1096-1217 of the reference: hub chaos mode
(random batch caps, shuffles and pauses) with 1/4/64 clients must return
every row bit-identical to the position evaluated alone; an injected failure
reaches every waiter as "GPU inference failed: ..."; the memory check refuses
before allocating; cuda_probe::tanhInPlace within 2 ulp; runners leave no
thread behind.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HUB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libazhub.so")


@pytest.fixture(scope="module")
def hub(engine):
    if not os.path.exists(HUB):
        pytest.skip("oracle/_ref/libazhub.so is not built (needs the reference tree: make -C oracle hub)")
    L = C.CDLL(HUB)
    L.azhub_chaos.argtypes = [C.c_int] * 5 + [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_int,
                                              C.c_int, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong), C.c_char_p,
                                              C.c_size_t]
    L.azhub_fail_after.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
    L.azhub_memory_refusal.argtypes = [C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
    return L


@pytest.mark.parametrize("precision", ["bf16", "tf32x3"])
@pytest.mark.parametrize("clients,batch,slots,chaos", [(1, 8, 1, 0), (4, 64, 2, 5), (64, 512, 2, 7), (64, 64, 1, 9)])
def test_hub_chaos_bitwise(engine, hub, precision, clients, batch, slots, chaos):
    bad, done = C.c_longlong(), C.c_longlong()
    err = C.create_string_buffer(512)
    rc = hub.azhub_chaos(13, 1, 2, 32, 32, 602, clients, 12, batch, slots, chaos, 0, engine.PRECISIONS[precision],
                         C.byref(bad), C.byref(done), err, 512)
    assert rc == 0, err.value.decode()
    assert done.value >= clients * 12
    assert bad.value == 0, f"{bad.value} of {done.value} rows differ from the position evaluated alone"


def test_injected_failure_reaches_every_waiter(engine, hub):
    msg = C.create_string_buffer(512)
    threw = hub.azhub_fail_after(3, 10, 0, engine.BF16, msg, 512)
    assert threw == 7, threw          # the 4th pass fails, and the hub fails every later request
    assert msg.value.decode().startswith("GPU inference failed: cuda: injected failure")


def test_memory_check_refuses_before_allocating(engine, hub):
    msg = C.create_string_buffer(512)
    assert hub.azhub_memory_refusal(1 << 20, 0, msg, 512) == 1
    text = msg.value.decode()
    assert text.startswith("cuda: inference needs") and text.endswith("lower inference_batch"), text


def _ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in float32 units in the last place, through the ordered integer
    image of the bit patterns (-0 and +0 are 0 apart)."""
    def ordered(x):
        i = np.ascontiguousarray(x, np.float32).view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)
    return np.abs(ordered(a) - ordered(b))


def test_tanh_within_two_ulp(engine, hub):
    """cuda_probe::tanhInPlace runs the tanhf the value head uses; it is held
    within 2 ulp of tanh in double, rounded (tests/test_cuda.cpp:492-512)."""
    hub.azhub_tanh.argtypes = [C.POINTER(C.c_float), C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
    rng = np.random.default_rng(404)
    x = (rng.random(1_000_000) * 40.0 - 20.0).astype(np.float32)
    extra = np.array([0.0, -0.0, 1e-8, -1e-8, 1e-40, 0.5, -0.5, 9.0, -9.0, 20.0, -20.0, 100.0], np.float32)
    x = np.concatenate([x, extra])
    y = x.copy()
    err = C.create_string_buffer(512)
    assert hub.azhub_tanh(y.ctypes.data_as(C.POINTER(C.c_float)), y.size, 0, err, 512) == 0, err.value.decode()
    ref = np.tanh(x.astype(np.float64)).astype(np.float32)
    worst = int(_ulp_distance(y, ref).max())
    print(f"tanh worst {worst} ulp (ceiling 2)")
    assert worst <= 2
    special = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0], np.float32)
    assert hub.azhub_tanh(special.ctypes.data_as(C.POINTER(C.c_float)), 5, 0, err, 512) == 0, err.value.decode()
    assert special[0] == 1.0 and special[1] == -1.0 and np.isnan(special[2])
    assert special[3] == 0.0 and not np.signbit(special[3]) and special[4] == 0.0 and np.signbit(special[4])


def test_runner_no_thread_leak(engine, hub):
    """Fifty runners created and destroyed, every other one with a pass in
    flight, leave no thread behind (tests/test_cuda.cpp:1220-1238)."""
    hub.azhub_runner_cycles.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_char_p,
                                        C.c_size_t]
    before, after = C.c_int(), C.c_int()
    err = C.create_string_buffer(512)
    assert hub.azhub_runner_cycles(50, 0, C.byref(before), C.byref(after), err, 512) == 0, err.value.decode()
    assert after.value <= before.value, (before.value, after.value)
