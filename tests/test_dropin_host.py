"""The drop-in's upload checks, which need no GPU: the reference's
cuda_probe::checkUpload and checkForwardReadsEveryTensor
(tests/test_cuda.cpp:918-949) through the bridge
(alphazero-go_b200/host/azgo_cuda_bridge.cpp), built with the reference's
Network into oracle/_ref/libazhub.so.

A tensor the engine's layout does not know (a layer added on the CPU
without a GPU port) is refused at upload, by name; one the layout knows but
the pass for the shape it encodes never reads is refused too, every such
tensor named.
"""
import ctypes as C
import os

import pytest

HUB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libazhub.so")


@pytest.fixture(scope="module")
def hub():
    if not os.path.exists(HUB):
        pytest.skip("oracle/_ref/libazhub.so is not built (needs the reference tree: make -C oracle hub)")
    L = C.CDLL(HUB)
    for f in (L.azhub_check_upload, L.azhub_check_reads):
        f.argtypes = [C.c_int] * 7 + [C.c_char_p, C.c_size_t]
        f.restype = C.c_int
    return L


def test_unknown_tensor_refused(hub):
    msg = C.create_string_buffer(1024)
    assert hub.azhub_check_upload(9, 1, 1, 8, 64, 0, 0, msg, 1024) == 0, msg.value.decode()
    assert hub.azhub_check_upload(9, 1, 1, 8, 64, 1, 1, msg, 1024) == 0, msg.value.decode()
    assert hub.azhub_check_upload(9, 1, 1, 8, 64, 0, 1, msg, 1024) == 1
    assert "ownership.conv.w" in msg.value.decode(), msg.value.decode()


def test_missing_tensor_refused(hub):
    """The other way round: the layout wants a tensor the network lacks."""
    msg = C.create_string_buffer(1024)
    assert hub.azhub_check_upload(9, 1, 1, 8, 64, 1, 0, msg, 1024) == 1
    assert "ownership" in msg.value.decode(), msg.value.decode()


def test_unread_tensor_refused(hub):
    msg = C.create_string_buffer(1024)
    assert hub.azhub_check_reads(9, 1, 1, 8, 64, 1, 1, msg, 1024) == 0, msg.value.decode()
    assert hub.azhub_check_reads(9, 1, 1, 8, 64, 1, 0, msg, 1024) == 1
    what = msg.value.decode()
    assert "ownership.conv.w" in what and "ownership.bn.runVar" in what, what
