"""Python access to the B200 engine through its C ABI (include/azb200.h).

Mirrors the reference's CUDA-engine interface (include/azgo/cuda.hpp,
include/azgo/inference_hub.hpp) under the same names, so tests and the
benchmark read like the reference's own:

    cuda_built(), cuda_available(), cuda_description()
    CudaInference(desc, params, buffers, max_batch).infer(x) -> logits, values, ownership
    make_cuda_runner(desc, params, buffers, max_batch, slots) -> BatchRunner
    check_cuda_inference_memory(desc, inference_batch, hubs, slots_per_hub)
    cuda_probe.*: the test hooks

The engine is the in-tree libazb200.so; importing this module fails loudly
when it is missing (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libazb200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "azb200.h")

TF32, TF32X3, BF16 = 0, 1, 2
PRECISIONS = {"tf32": TF32, "tf32x3": TF32X3, "bf16": BF16}


class NetDesc(C.Structure):
    """NetConfig (include/azgo/network.hpp:23-36)."""

    _fields_ = [(n, C.c_int) for n in ("board", "history", "blocks", "filters", "value_hidden", "ownership")]

    @classmethod
    def of(cls, cfg) -> "NetDesc":
        return cls(cfg.board, cfg.history, cfg.blocks, cfg.filters, cfg.value_hidden, int(cfg.ownership))

    @property
    def planes(self):
        return 2 * self.history + 2

    @property
    def area(self):
        return self.board * self.board

    @property
    def actions(self):
        return self.area + 1


_F = C.POINTER(C.c_float)
DONE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_char_p)

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is not built: run `python {os.path.join(HERE, 'build_ext.py')}`")
            L = C.CDLL(LIB_PATH)
            D = C.POINTER(NetDesc)
            s = C.c_size_t
            err = [C.c_char_p, s]
            L.azb_cuda_built.restype = C.c_int
            L.azb_cuda_available.argtypes = [C.c_int, C.c_char_p, s]
            L.azb_describe.argtypes = [C.c_int, C.c_int, C.c_char_p, s]
            L.azb_layout_count.argtypes = [D, C.c_int]
            L.azb_layout_entry.argtypes = [D, C.c_int, C.c_int, C.c_char_p, s, C.POINTER(s), C.POINTER(s)]
            L.azb_layout_floats.argtypes = [D, C.c_int]
            L.azb_layout_floats.restype = s
            L.azb_checkpoint_config.argtypes = [C.c_char_p, D, C.POINTER(s), C.POINTER(s), C.c_char_p, s]
            L.azb_checkpoint_read.argtypes = [C.c_char_p, D, _F, s, _F, s, C.c_char_p, s]
            L.azb_infer_create.argtypes = [D, _F, s, _F, s, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)] + err
            L.azb_infer_destroy.argtypes = [C.c_void_p]
            L.azb_infer_run.argtypes = [C.c_void_p, _F, C.c_int, _F, _F, _F, _F] + err
            L.azb_stones_record_bytes.argtypes = [C.c_int, C.c_int]
            L.azb_stones_record_bytes.restype = C.c_size_t
            L.azb_infer_run_stones.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _F, _F, _F] + err
            L.azb_infer_bytes.argtypes = [C.c_void_p]
            L.azb_infer_bytes.restype = s
            L.azb_infer_stage.argtypes = [C.c_void_p, _F, C.c_int] + err
            L.azb_infer_enqueue.argtypes = [C.c_void_p, C.c_int]
            L.azb_infer_sync.argtypes = [C.c_void_p] + err
            L.azb_infer_stream.argtypes = [C.c_void_p]
            L.azb_infer_stream.restype = C.c_void_p
            L.azb_infer_time.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double),
                                         C.POINTER(C.c_double)] + err
            L.azb_infer_time_stages.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_double), C.c_char_p, C.c_size_t]
            L.azb_infer_read.argtypes = [C.c_void_p, C.c_int, _F, _F, _F, _F] + err
            L.azb_runner_create.argtypes = [D, _F, s, _F, s, C.c_int, C.c_int, C.c_int, C.c_int,
                                            C.POINTER(C.c_void_p)] + err
            L.azb_runner_destroy.argtypes = [C.c_void_p]
            L.azb_runner_slots.argtypes = [C.c_void_p]
            L.azb_runner_max_batch.argtypes = [C.c_void_p]
            L.azb_runner_input.argtypes = [C.c_void_p, C.c_int]
            L.azb_runner_input.restype = _F
            L.azb_runner_begin.argtypes = [C.c_void_p, C.c_int, C.c_int, DONE_FN, C.c_void_p]
            L.azb_runner_begin_stones.argtypes = [C.c_void_p, C.c_int, C.c_int, DONE_FN, C.c_void_p]
            L.azb_runner_records.argtypes = [C.c_void_p, C.c_int]
            L.azb_runner_records.restype = C.POINTER(C.c_uint8)
            for fn in (L.azb_runner_logits, L.azb_runner_values, L.azb_runner_ownership):
                fn.argtypes = [C.c_void_p, C.c_int]
                fn.restype = _F
            PI = C.POINTER(C.c_int)
            L.azb_hub_create.argtypes = [D, _F, s, _F, s, PI, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.POINTER(C.c_void_p)] + err
            L.azb_hub_create_fake.argtypes = [C.c_int] * 9 + [C.POINTER(C.c_void_p)] + err
            L.azb_hub_destroy.argtypes = [C.c_void_p]
            L.azb_hub_lanes.argtypes = [C.c_void_p]
            L.azb_hub_pass_cap.argtypes = [C.c_void_p]
            L.azb_hub_evaluate.argtypes = [C.c_void_p, C.c_int, _F, C.c_int, _F, _F] + err
            L.azb_hub_evaluate_records.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, _F, _F] + err
            L.azb_hub_stats.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong),
                                        C.POINTER(C.c_longlong), C.POINTER(C.c_double)]
            L.azb_workspace_bytes.argtypes = [D, C.c_int, C.c_int]
            L.azb_workspace_bytes.restype = s
            L.azb_check_memory.argtypes = [D, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int] + err
            L.azb_probe_set_hub_chaos_seed.argtypes = [C.c_uint64]
            L.azb_probe_hub_chaos_seed.restype = C.c_uint64
            L.azb_probe_fail_passes_after.argtypes = [C.c_int]
            L.azb_probe_set_memory_limit.argtypes = [s]
            L.azb_probe_passes_completed.restype = C.c_longlong
            L.azb_probe_set_copy_out_delay.argtypes = [C.c_int]
            L.azb_probe_set_conv_path.argtypes = [C.c_int]
            L.azb_probe_set_conv_segment.argtypes = [C.c_int]
            L.azb_probe_set_tower_fused.argtypes = [C.c_int]
            L.azb_probe_set_tower_persistent.argtypes = [C.c_int]
            L.azb_probe_starve_tower.argtypes = [C.c_int]
            L.azb_probe_binary_version.argtypes = [C.c_int]
            L.azb_probe_device_architecture.argtypes = [C.c_int]
            L.azb_probe_fill.argtypes = [C.c_int, _F, s, C.c_float, s] + err
            L.azb_probe_tanh.argtypes = [C.c_int, _F, s] + err
            L.azb_probe_bounded_wait.argtypes = [C.c_int, C.c_ulonglong] + err
            L.azb_probe_umma.argtypes = [C.c_int] * 7 + [_F, _F, _F] + err
            L.azb_synth_network.argtypes = [D, C.c_uint64, C.c_int, _F, _F]
            L.azb_synth_positions.argtypes = [D, C.c_uint64, C.c_long, C.c_int, _F]
            L.azb_device_pci_bus_id.argtypes = [C.c_int, C.c_char_p, s]
            _lib = L
    return _lib


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, "float32 C-contiguous arrays only"
    return a.ctypes.data_as(_F)


class CudaError(RuntimeError):
    pass


def _err():
    return C.create_string_buffer(1024)


# ------------------------------------------------------------------ device


def cuda_built() -> bool:
    return bool(lib().azb_cuda_built())


def cuda_available(device: int = 0) -> tuple[bool, str]:
    why = C.create_string_buffer(512)
    ok = bool(lib().azb_cuda_available(device, why, 512))
    return ok, why.value.decode()


def cuda_description(device: int = 0, precision: int = TF32) -> str:
    out = C.create_string_buffer(512)
    lib().azb_describe(device, precision, out, 512)
    return out.value.decode()


def device_count() -> int:
    return lib().azb_device_count()


def layout(desc: NetDesc, which: int):
    """[(name, size, offset)] of ParamLayout::of for this shape."""
    L = lib()
    out = []
    name = C.create_string_buffer(64)
    size, off = C.c_size_t(), C.c_size_t()
    for i in range(L.azb_layout_count(C.byref(desc), which)):
        L.azb_layout_entry(C.byref(desc), which, i, name, 64, C.byref(size), C.byref(off))
        out.append((name.value.decode(), size.value, off.value))
    return out


def pci_bus_id(device: int = 0) -> str:
    out = C.create_string_buffer(64)
    return out.value.decode() if lib().azb_device_pci_bus_id(device, out, 64) == 0 else ""


def arena_floats(desc: NetDesc) -> tuple[int, int]:
    return lib().azb_layout_floats(C.byref(desc), 0), lib().azb_layout_floats(C.byref(desc), 1)


def checkpoint_config(path: str) -> NetDesc:
    """readCheckpointConfig (include/azgo/checkpoint.hpp:25): the header's shape.
    Raises RuntimeError with the reference loader's message."""
    return _checkpoint_header(path)[0]


def _checkpoint_header(path: str):
    d, e = NetDesc(), _err()
    np_, nb = C.c_size_t(), C.c_size_t()
    if lib().azb_checkpoint_config(os.fsencode(path), C.byref(d), C.byref(np_), C.byref(nb), e, 1024) != 0:
        raise RuntimeError(e.value.decode())
    return d, np_.value, nb.value


def load_checkpoint(path: str):
    """loadNetwork (include/azgo/checkpoint.hpp:24) into the engine's arenas:
    (NetDesc, params, buffers), ready for CudaInference / make_cuda_runner.
    Raises RuntimeError with the reference loader's message."""
    d, np_, nb = _checkpoint_header(path)
    params = np.zeros(np_, np.float32)
    buffers = np.zeros(nb, np.float32)
    e = _err()
    if lib().azb_checkpoint_read(os.fsencode(path), C.byref(d), _fp(params), np_, _fp(buffers), nb, e, 1024) != 0:
        raise RuntimeError(e.value.decode())
    return d, params, buffers


def synth_network(desc: NetDesc, seed: int, kind: int = 0):
    """Network(cfg, seed) plus a batch-norm randomiser (0 benchmark, 1 tests, -1 none):
    the two ParamLayout arenas (params, buffers)."""
    np_, nb = arena_floats(desc)
    params = np.zeros(np_, np.float32)
    buffers = np.zeros(nb, np.float32)
    if lib().azb_synth_network(C.byref(desc), seed, kind, _fp(params), _fp(buffers)) != 0:
        raise ValueError("azb_synth_network: bad network shape")
    return params, buffers


def synth_positions(desc: NetDesc, seed: int, B: int, first: int = 0) -> np.ndarray:
    """B encoded positions [B][planes][area] (samples first .. first+B-1)."""
    out = np.zeros((B, desc.planes, desc.area), np.float32)
    if lib().azb_synth_positions(C.byref(desc), seed, first, B, _fp(out)) != 0:
        raise ValueError("azb_synth_positions: bad network shape")
    return out


def workspace_bytes(desc: NetDesc, max_batch: int, precision: int) -> int:
    return lib().azb_workspace_bytes(C.byref(desc), max_batch, precision)


def check_cuda_inference_memory(desc: NetDesc, inference_batch: int, hubs: int, slots_per_hub: int = 2,
                                device: int = 0, precision: int = TF32) -> None:
    e = _err()
    if lib().azb_check_memory(C.byref(desc), inference_batch, hubs, slots_per_hub, device, precision, e, 1024) != 0:
        raise CudaError(e.value.decode())


# --------------------------------------------------------------- inference


class CudaInference:
    """CudaInference (include/azgo/cuda.hpp:72-84) for one device."""

    def __init__(self, desc: NetDesc, params: np.ndarray, buffers: np.ndarray, max_batch: int, device: int = 0,
                 precision: int = TF32):
        self.desc = desc
        self.max_batch = max_batch
        self._params = np.ascontiguousarray(params, np.float32)
        self._buffers = np.ascontiguousarray(buffers, np.float32)
        h = C.c_void_p()
        e = _err()
        rc = lib().azb_infer_create(C.byref(desc), _fp(self._params), self._params.size, _fp(self._buffers),
                                    self._buffers.size, max_batch, device, precision, C.byref(h), e, 1024)
        if rc != 0:
            raise CudaError(e.value.decode())
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().azb_infer_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def infer(self, x: np.ndarray, probs: bool = False, ownership: bool = None):
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        d = self.desc
        logits = np.empty((B, d.actions), np.float32)
        values = np.empty(B, np.float32)
        own = np.empty((B, d.area), np.float32) if (d.ownership if ownership is None else ownership) else None
        pr = np.empty((B, d.actions), np.float32) if probs else None
        e = _err()
        if lib().azb_infer_run(self.h, _fp(x), B, _fp(logits), _fp(values), _fp(own), _fp(pr), e, 1024) != 0:
            raise CudaError(e.value.decode())
        return (logits, values, own, pr) if probs else (logits, values, own)

    def infer_stones(self, records: np.ndarray, ownership: bool = None):
        """infer() from position records (stones_records): the planes are encoded on the device."""
        records = np.ascontiguousarray(records, np.uint8)
        B = records.shape[0]
        d = self.desc
        if records.shape[1] != stones_record_bytes(d.history, d.board):
            raise ValueError("records: wrong record size")
        logits = np.empty((B, d.actions), np.float32)
        values = np.empty(B, np.float32)
        own = np.empty((B, d.area), np.float32) if (d.ownership if ownership is None else ownership) else None
        e = _err()
        if lib().azb_infer_run_stones(self.h, records.ctypes.data, B, _fp(logits), _fp(values), _fp(own), e,
                                      1024) != 0:
            raise CudaError(e.value.decode())
        return logits, values, own

    def bytes(self) -> int:
        return lib().azb_infer_bytes(self.h)

    # device-resident use (timing)
    def stage(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        e = _err()
        if lib().azb_infer_stage(self.h, _fp(x), x.shape[0], e, 1024) != 0:
            raise CudaError(e.value.decode())

    def enqueue(self, B: int):
        if lib().azb_infer_enqueue(self.h, B) != 0:
            raise CudaError("enqueue failed")

    def sync(self):
        e = _err()
        if lib().azb_infer_sync(self.h, e, 1024) != 0:
            raise CudaError(e.value.decode())

    def stream(self) -> int:
        return lib().azb_infer_stream(self.h)

    def time(self, B: int, warmup: int, steps: int, with_copies: bool = False, conv: bool = False):
        """(ms for `steps` passes, summed conv-kernel ms or None), CUDA events on the engine's stream."""
        ms, cms = C.c_double(), C.c_double()
        e = _err()
        rc = lib().azb_infer_time(self.h, B, warmup, steps, int(with_copies), C.byref(ms),
                                  C.byref(cms) if conv else None, e, 1024)
        if rc != 0:
            raise CudaError(e.value.decode())
        return ms.value, (cms.value if conv else None)

    STAGES = ("stem_operand", "stem_gemm", "tower", "head_conv", "head_tail", "unused")

    def time_stages(self, B: int, steps: int) -> dict:
        """Device ms per stage, summed over `steps` passes (events around every launch)."""
        out = (C.c_double * len(self.STAGES))()
        e = _err()
        if lib().azb_infer_time_stages(self.h, B, steps, out, e, 1024) != 0:
            raise CudaError(e.value.decode())
        return dict(zip(self.STAGES, list(out)))

    def read(self, B: int):
        d = self.desc
        logits = np.empty((B, d.actions), np.float32)
        values = np.empty(B, np.float32)
        own = np.empty((B, d.area), np.float32) if d.ownership else None
        pr = np.empty((B, d.actions), np.float32)
        e = _err()
        if lib().azb_infer_read(self.h, B, _fp(logits), _fp(values), _fp(own), _fp(pr), e, 1024) != 0:
            raise CudaError(e.value.decode())
        return logits, values, own, pr


# ----------------------------------------------------------- position records


def stones_record_bytes(history: int, board: int) -> int:
    """Bytes of one position record (include/azb200.h, azb_stones_record_bytes)."""
    return int(lib().azb_stones_record_bytes(history, board))


def stones_records(stones: np.ndarray, to_move: np.ndarray, available: np.ndarray | None = None,
                   sym: np.ndarray | None = None) -> np.ndarray:
    """Position records from stones [B][H][n*n] (0 empty, 1 Black, 2 White; row k = k plies ago),
    to_move [B] (1 Black, 2 White), the history positions present [B] (default H) and the
    symmetries [B] (default 0): [B][stones_record_bytes] uint8."""
    stones = np.asarray(stones, np.uint8)
    B, H, A = stones.shape
    n = int(round(A ** 0.5))
    rec = np.zeros((B, stones_record_bytes(H, n)), np.uint8)
    rec[:, :H * A] = stones.reshape(B, H * A)
    rec[:, H * A] = np.asarray(to_move, np.uint8)
    rec[:, H * A + 1] = H if available is None else np.asarray(available, np.uint8)
    rec[:, H * A + 2] = 0 if sym is None else np.asarray(sym, np.uint8)
    return rec


# ------------------------------------------------------------------ runner


class BatchRunner:
    """BatchRunner (include/azgo/inference_hub.hpp:41-53) over the engine's runner."""

    def __init__(self, desc: NetDesc, params, buffers, max_batch: int, slots: int = 2, device: int = 0,
                 precision: int = TF32):
        self.desc = desc
        self._params = np.ascontiguousarray(params, np.float32)
        self._buffers = np.ascontiguousarray(buffers, np.float32)
        h = C.c_void_p()
        e = _err()
        rc = lib().azb_runner_create(C.byref(desc), _fp(self._params), self._params.size, _fp(self._buffers),
                                     self._buffers.size, max_batch, slots, device, precision, C.byref(h), e, 1024)
        if rc != 0:
            msg = e.value.decode()
            raise (ValueError(msg) if "must be" in msg else CudaError(msg))
        self.h = h
        self._callbacks = {}
        self._cb_lock = threading.Lock()
        self._next = 0

    def close(self):
        if getattr(self, "h", None):
            lib().azb_runner_destroy(self.h)   # drains passes in flight first
            self.h = None
            self._callbacks.clear()

    def __del__(self):
        self.close()

    def slots(self) -> int:
        return lib().azb_runner_slots(self.h)

    def max_batch(self) -> int:
        return lib().azb_runner_max_batch(self.h)

    def input(self, slot: int) -> np.ndarray:
        p = lib().azb_runner_input(self.h, slot)
        d = self.desc
        return np.ctypeslib.as_array(p, shape=(self.max_batch(), d.planes, d.area))

    def logits(self, slot: int, B: int) -> np.ndarray:
        return np.ctypeslib.as_array(lib().azb_runner_logits(self.h, slot), shape=(B, self.desc.actions))

    def values(self, slot: int, B: int) -> np.ndarray:
        return np.ctypeslib.as_array(lib().azb_runner_values(self.h, slot), shape=(B,))

    def ownership(self, slot: int, B: int) -> np.ndarray:
        return np.ctypeslib.as_array(lib().azb_runner_ownership(self.h, slot), shape=(B, self.desc.area))

    def records(self, slot: int) -> np.ndarray:
        """The slot's pinned position-record staging, [max_batch][stones_record_bytes]."""
        d = self.desc
        p = lib().azb_runner_records(self.h, slot)
        return np.ctypeslib.as_array(p, shape=(self.max_batch(), stones_record_bytes(d.history, d.board)))

    def begin_stones(self, slot: int, B: int, done) -> None:
        """begin() from the first B records of records(slot), encoded on the device."""
        self.begin(slot, B, done, _entry=lib().azb_runner_begin_stones)

    def begin(self, slot: int, B: int, done, _entry=None) -> None:
        """done(slot, error) is called exactly once, from the runner's thread."""
        with self._cb_lock:
            key = self._next
            self._next += 1

        def trampoline(ctx, s, err, key=key):
            with self._cb_lock:
                fn, _ = self._callbacks.pop(key, (None, None))
            if fn is not None:
                fn(s, err.decode() if err else "")

        cb = DONE_FN(trampoline)
        with self._cb_lock:
            self._callbacks[key] = (done, cb)
        if (_entry or lib().azb_runner_begin)(self.h, slot, B, cb, None) != 0:
            with self._cb_lock:
                self._callbacks.pop(key, None)
            raise IndexError(f"slot {slot} out of range")


# ------------------------------------------------------------------ hub

HUB_PLANES, HUB_RECORDS = 0, 1


class Hub:
    """azb_hub: leaf batching for many worker threads over one runner per GPU
    (the role of the reference's InferenceHub + WorkerEvaluators for "cuda",
    include/azgo/inference_hub.hpp:83-150). evaluate() blocks until the
    worker's positions are back; ctypes releases the GIL meanwhile."""

    def __init__(self, desc: NetDesc, params=None, buffers=None, devices=(0,), max_batch: int = 256,
                 slots: int = 2, precision: int = TF32, input_mode: int = HUB_PLANES, *, fake: dict | None = None):
        self.desc = desc
        h = C.c_void_p()
        e = _err()
        if fake is not None:   # the CPU stand-in for the GPU passes (host-logic tests)
            rc = lib().azb_hub_create_fake(desc.board, desc.history, fake.get("lanes", 1), max_batch, slots,
                                           fake.get("quantum", 1), input_mode, fake.get("delay_us", 0),
                                           fake.get("fail_after", 0), C.byref(h), e, 1024)
        else:
            self._params = np.ascontiguousarray(params, np.float32)
            self._buffers = np.ascontiguousarray(buffers, np.float32)
            devs = (C.c_int * len(devices))(*devices)
            rc = lib().azb_hub_create(C.byref(desc), _fp(self._params), self._params.size, _fp(self._buffers),
                                      self._buffers.size, devs, len(devices), max_batch, slots, precision,
                                      input_mode, C.byref(h), e, 1024)
        if rc != 0:
            raise CudaError(e.value.decode())
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().azb_hub_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def lanes(self) -> int:
        return lib().azb_hub_lanes(self.h)

    def pass_cap(self) -> int:
        return lib().azb_hub_pass_cap(self.h)

    def evaluate(self, lane: int, x: np.ndarray):
        """(logits [B][A+1], values [B]) for planes [B][P][A]."""
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        logits = np.empty((B, self.desc.actions), np.float32)
        values = np.empty(B, np.float32)
        e = _err()
        if lib().azb_hub_evaluate(self.h, lane, _fp(x), B, _fp(logits), _fp(values), e, 1024) != 0:
            raise CudaError(e.value.decode())
        return logits, values

    def evaluate_records(self, lane: int, records: np.ndarray):
        records = np.ascontiguousarray(records, np.uint8)
        B = records.shape[0]
        logits = np.empty((B, self.desc.actions), np.float32)
        values = np.empty(B, np.float32)
        e = _err()
        if lib().azb_hub_evaluate_records(self.h, lane, records.ctypes.data, B, _fp(logits), _fp(values), e,
                                          1024) != 0:
            raise CudaError(e.value.decode())
        return logits, values

    def stats(self, lane: int) -> dict:
        p, n, f, t = C.c_longlong(), C.c_longlong(), C.c_longlong(), C.c_double()
        lib().azb_hub_stats(self.h, lane, C.byref(p), C.byref(n), C.byref(f), C.byref(t))
        return {"passes": p.value, "positions": n.value, "full_passes": f.value, "gpu_seconds": t.value}


def make_cuda_runner(desc, params, buffers, max_batch: int, slots: int = 2, device: int = 0,
                     precision: int = TF32) -> BatchRunner:
    """makeCudaRunner (include/azgo/cuda.hpp:58)."""
    return BatchRunner(desc, params, buffers, max_batch, slots, device, precision)


# -------------------------------------------------------------- cuda_probe


class cuda_probe:
    """The test hooks of include/azgo/cuda.hpp:91-155."""

    @staticmethod
    def set_hub_chaos_seed(seed: int):
        lib().azb_probe_set_hub_chaos_seed(seed)

    @staticmethod
    def hub_chaos_seed() -> int:
        return lib().azb_probe_hub_chaos_seed()

    @staticmethod
    def fail_passes_after(n: int):
        lib().azb_probe_fail_passes_after(n)

    @staticmethod
    def set_memory_limit(nbytes: int):
        lib().azb_probe_set_memory_limit(nbytes)

    @staticmethod
    def passes_completed() -> int:
        return lib().azb_probe_passes_completed()

    @staticmethod
    def set_copy_out_delay(us: int):
        lib().azb_probe_set_copy_out_delay(us)

    @staticmethod
    def set_conv_path(path: int):
        """0 default (by width), 1 one tile per CTA, 2 CTA pairs (M = 256), 3 two tiles per CTA (N <= 128)."""
        lib().azb_probe_set_conv_path(path)

    @staticmethod
    def set_tower_fused(mode: int):
        """-1 default (one launch for the tower of boards up to 10x10 with <= 64 channels; tf32x3 at 64
        channels runs two groups of boards per CTA where that saves a round of CTAs), 0 per-layer kernels,
        1 fused with one group per CTA, 2 fused with two groups per CTA wherever the shape allows."""
        lib().azb_probe_set_tower_fused(mode)

    @staticmethod
    def set_tower_persistent(mode: int):
        """Towers too large to fuse: -1 default (one persistent launch at <= 128 channels), 0 per layer, 1 at any width (bf16/tf32)."""
        lib().azb_probe_set_tower_persistent(mode)

    @staticmethod
    def starve_tower(on: bool):
        """Failure detection: the persistent tower's waits for a previous layer run out (0.5 s) and the pass fails."""
        lib().azb_probe_starve_tower(1 if on else 0)

    @staticmethod
    def set_conv_segment(steps: int):
        """tf32x3 (<= 128 channels): -1 default (accumulation segments of 3 taps, 9 at <= 64 channels), 0 one run per tile."""
        lib().azb_probe_set_conv_segment(steps)

    @staticmethod
    def binary_version(device: int = 0) -> int:
        return lib().azb_probe_binary_version(device)

    @staticmethod
    def device_architecture(device: int = 0) -> int:
        return lib().azb_probe_device_architecture(device)

    @staticmethod
    def fill(data: np.ndarray, n: int, value: float, tail: int = 0, device: int = 0):
        e = _err()
        if lib().azb_probe_fill(device, _fp(data), n, value, tail, e, 1024) != 0:
            raise CudaError(e.value.decode())

    @staticmethod
    def tanh(x: np.ndarray, device: int = 0) -> np.ndarray:
        """cuda_probe::tanhInPlace: tanhf on the device, as the heads compute the value and ownership."""
        y = np.ascontiguousarray(x, np.float32).copy()
        e = _err()
        if lib().azb_probe_tanh(device, _fp(y), y.size, e, 1024) != 0:
            raise CudaError(e.value.decode())
        return y

    @staticmethod
    def bounded_wait(limit_ns: int, device: int = 0) -> int:
        e = _err()
        code = lib().azb_probe_bounded_wait(device, limit_ns, e, 1024)
        if code < 0:
            raise CudaError(e.value.decode())
        return code

    @staticmethod
    def umma(precision: int, n_out: int, halo_rows: int, shift: int, k_chunks: int, a: np.ndarray, w: np.ndarray,
             base_offset_mode: int = 0, device: int = 0) -> np.ndarray:
        d = np.zeros((128, n_out), np.float32)
        e = _err()
        a = np.ascontiguousarray(a, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        if lib().azb_probe_umma(device, precision, n_out, halo_rows, shift, k_chunks, base_offset_mode, _fp(a), _fp(w),
                                _fp(d), e, 1024) != 0:
            raise CudaError(e.value.decode())
        return d


def header_symbols() -> list[str]:
    """Every function include/azb200.h declares."""
    import re

    text = open(HEADER).read()
    return sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(azb_\w+)\s*\(", text, re.M)))
