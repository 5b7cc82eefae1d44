"""The drop-in: the reference's own InferenceHub and WorkerEvaluators
(robominds/alphazero-go src/inference_hub.cpp, built from its sources) driving
the engine through alphazero-go_b200/host/azgo_cuda_bridge.cpp, i.e. the
reference's include/azgo/cuda.hpp implemented over include/azb200.h.

Mirrors tests/test_cuda.cpp:1096-1217 of the reference: hub chaos mode
(random batch caps, shuffles and pauses) with 1/4/64 clients must return
every row bit-identical to the position evaluated alone; an injected failure
reaches every waiter as "GPU inference failed: ..."; the memory check refuses
before allocating.
"""
import ctypes as C
import os

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
