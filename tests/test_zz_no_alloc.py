"""azb_infer_run_noalloc through the C ABI: the forward pass for callers that
may not allocate device memory when they evaluate (hosts whose pool
allocator owns the GPU's memory or that run under a fixed device-memory
budget, latency-critical paths). Its scratch lives in the library's static device array; its results
must equal azb_infer_run's on the same handle and inputs (tolerance 0: the
same kernels run on the same weights), on two calls in a row, including a
call whose frame padding lies where the previous call wrote real points.

This file is collected last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

_F = C.POINTER(C.c_float)


def noalloc(engine):
    fn = engine.lib().azb_infer_run_noalloc
    fn.argtypes = [C.c_void_p, _F, C.c_int, _F, _F, _F, C.c_char_p, C.c_size_t]
    fn.restype = C.c_int
    return fn


def run_noalloc(engine, net, x, ownership):
    fn = noalloc(engine)
    x = np.ascontiguousarray(x, np.float32)
    B = x.shape[0]
    d = net.desc
    logits = np.full((B, d.actions), np.nan, np.float32)
    values = np.full(B, np.nan, np.float32)
    own = np.full((B, d.area), np.nan, np.float32) if ownership else None
    err = C.create_string_buffer(512)
    rc = fn(net.h, x.ctypes.data_as(_F), B, logits.ctypes.data_as(_F), values.ctypes.data_as(_F),
            own.ctypes.data_as(_F) if own is not None else None, err, 512)
    return rc, err.value.decode(), logits, values, own


@pytest.mark.parametrize("precision", ["bf16", "tf32x3"])
def test_noalloc_matches_infer_two_calls(engine, precision):
    prec = engine.PRECISIONS[precision]
    big = engine.NetDesc(19, 1, 2, 64, 32, 0)
    small = engine.NetDesc(9, 1, 2, 32, 32, 1)
    bp, bb = engine.synth_network(big, 21, 1)
    sp, sb = engine.synth_network(small, 22, 1)
    with engine.CudaInference(big, bp, bb, 8, 0, prec) as nb, engine.CudaInference(small, sp, sb, 16, 0, prec) as ns:
        xb = engine.synth_positions(big, 23, 8)
        xs = engine.synth_positions(small, 24, 16)
        # 1st call: the 19x19 network writes real points all over the array
        rc, msg, l1, v1, _ = run_noalloc(engine, nb, xb, False)
        assert rc == 0, msg
        rl, rv, _ = nb.infer(xb)
        np.testing.assert_array_equal(l1, rl)
        np.testing.assert_array_equal(v1, rv)
        # 2nd call, right after: a 9x9 network whose padding rows lie where the
        # first call wrote; it must read them as zero again
        rc, msg, l2, v2, o2 = run_noalloc(engine, ns, xs, True)
        assert rc == 0, msg
        rl, rv, ro = ns.infer(xs)
        np.testing.assert_array_equal(l2, rl)
        np.testing.assert_array_equal(v2, rv)
        np.testing.assert_array_equal(o2, ro)
        # and the first network again, unchanged
        rc, msg, l3, v3, _ = run_noalloc(engine, nb, xb, False)
        assert rc == 0, msg
        np.testing.assert_array_equal(l3, l1)
        np.testing.assert_array_equal(v3, v1)


def test_noalloc_refuses_beyond_its_array(engine):
    d = engine.NetDesc(19, 1, 2, 256, 32, 0)
    p, b = engine.synth_network(d, 25, 1)
    with engine.CudaInference(d, p, b, 256, 0, engine.BF16) as net:
        x = engine.synth_positions(d, 26, 256)
        rc, msg, *_ = run_noalloc(engine, net, x, False)
        assert rc != 0
        assert "more than the static array" in msg and "32 MiB" in msg
