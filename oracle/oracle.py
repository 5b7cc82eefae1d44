"""ctypes access to the CPU oracle (test infrastructure only).

Two libraries, both built by oracle/Makefile:
  * liboracle.so - the C restatement of the reference's CPU forward
    (azoracle.c), plus its seeded network, batch-norm and input generators;
  * _ref/libazref.so - the reference's own CPU network (robominds/alphazero-go
    src/network.cpp, src/layers.cpp, src/backend*.cpp ...) compiled from its
    sources, behind ref_shim.cpp's C ABI.
Only tests/, the smoke check and bench.py's CPU-baseline / reference arm use
this module. The GPU engine never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libazref.so")


@dataclass(frozen=True)
class NetConfig:
    """NetConfig (include/azgo/network.hpp:23-36)."""

    board: int
    history: int = 1
    blocks: int = 1
    filters: int = 32
    value_hidden: int = 64
    ownership: bool = False

    @property
    def planes(self) -> int:
        return 2 * self.history + 2

    @property
    def area(self) -> int:
        return self.board * self.board

    @property
    def actions(self) -> int:
        return self.area + 1


class _CCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("board", "history", "blocks", "filters", "value_hidden", "ownership")]


def _ccfg(cfg: NetConfig) -> _CCfg:
    return _CCfg(cfg.board, cfg.history, cfg.blocks, cfg.filters, cfg.value_hidden, int(cfg.ownership))


_F = C.POINTER(C.c_float)


def _fp(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"oracle not built: run `make -C {HERE} oracle`")
        L = C.CDLL(ORACLE_SO)
        P = C.POINTER(_CCfg)
        L.az_layout_count.argtypes = [P, C.c_int]
        L.az_layout_entry.argtypes = [P, C.c_int, C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t),
                                      C.POINTER(C.c_size_t), C.POINTER(C.c_int)]
        L.az_layout_floats.argtypes = [P, C.c_int]
        L.az_layout_floats.restype = C.c_size_t
        L.az_network_init.argtypes = [P, C.c_uint64, _F, _F]
        L.az_randomize.argtypes = [P, C.c_int, C.c_uint64, _F, _F]
        L.az_inputs_positions.argtypes = [P, C.c_uint64, C.c_long, C.c_int, _F]
        L.az_inputs_planes.argtypes = [C.c_uint64, C.c_size_t, _F]
        for fn in (L.az_forward_f32, L.az_forward_f64):
            fn.argtypes = [P, _F, _F, _F, C.c_int, _F, _F, _F, C.c_int]
        L.az_derive_seed.argtypes = [C.c_uint64] * 4
        L.az_derive_seed.restype = C.c_uint64
        _lib = L
    return _lib


def layout(cfg: NetConfig, which: int):
    """[(name, size, offset)] in params() (which=0) or buffers() (1) order."""
    L = lib()
    c = _ccfg(cfg)
    out = []
    name = C.create_string_buffer(64)
    size, off, decay = C.c_size_t(), C.c_size_t(), C.c_int()
    for i in range(L.az_layout_count(C.byref(c), which)):
        L.az_layout_entry(C.byref(c), which, i, name, 64, C.byref(size), C.byref(off), C.byref(decay))
        out.append((name.value.decode(), size.value, off.value))
    return out


def arena_floats(cfg: NetConfig):
    c = _ccfg(cfg)
    return lib().az_layout_floats(C.byref(c), 0), lib().az_layout_floats(C.byref(c), 1)


KIND_BENCH, KIND_TEST = 0, 1


def make_network(cfg: NetConfig, seed: int, kind: int | None = KIND_BENCH):
    """Network(cfg, seed), then the batch-norm randomiser `kind` (None: none).
    Returns the (params, buffers) arenas in ParamLayout order."""
    np_, nb = arena_floats(cfg)
    params = np.zeros(np_, np.float32)
    buffers = np.zeros(nb, np.float32)
    c = _ccfg(cfg)
    lib().az_network_init(C.byref(c), seed, _fp(params), _fp(buffers))
    if kind is not None:
        lib().az_randomize(C.byref(c), kind, seed, _fp(params), _fp(buffers))
    return params, buffers


def positions(cfg: NetConfig, seed: int, B: int, first: int = 0) -> np.ndarray:
    out = np.zeros((B, cfg.planes, cfg.area), np.float32)
    c = _ccfg(cfg)
    lib().az_inputs_positions(C.byref(c), seed, first, B, _fp(out))
    return out


def random_planes(cfg: NetConfig, seed: int, B: int) -> np.ndarray:
    out = np.zeros((B, cfg.planes, cfg.area), np.float32)
    lib().az_inputs_planes(seed, out.size, _fp(out))
    return out


def forward(cfg: NetConfig, params, buffers, x: np.ndarray, precision: str = "f32", threads: int = 1):
    """(logits [B][A+1], values [B], ownership [B][A] or None)."""
    x = np.ascontiguousarray(x, np.float32)
    B = x.shape[0]
    logits = np.zeros((B, cfg.actions), np.float32)
    values = np.zeros(B, np.float32)
    own = np.zeros((B, cfg.area), np.float32) if cfg.ownership else None
    c = _ccfg(cfg)
    fn = lib().az_forward_f32 if precision == "f32" else lib().az_forward_f64
    fn(C.byref(c), _fp(params), _fp(buffers), _fp(x), B, _fp(logits), _fp(values), _fp(own), threads)
    return logits, values, own


# ------------------------------------------------------------ the reference


_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError("oracle/_ref/libazref.so not built (needs the reference tree)")
        R = C.CDLL(REF_SO)
        R.azref_net_create.argtypes = [C.c_int] * 6 + [C.c_uint64, C.c_int]
        R.azref_net_create.restype = C.c_void_p
        R.azref_net_destroy.argtypes = [C.c_void_p]
        R.azref_floats.argtypes = [C.c_void_p, C.c_int]
        R.azref_floats.restype = C.c_size_t
        R.azref_layout_count.argtypes = [C.c_void_p, C.c_int]
        R.azref_layout_entry.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t,
                                         C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        R.azref_export.argtypes = [C.c_void_p, _F, _F]
        R.azref_import.argtypes = [C.c_void_p, _F, _F]
        R.azref_infer_threads.argtypes = [C.c_void_p, C.c_char_p, _F, C.c_int, _F, _F, _F, C.c_int, C.c_char_p,
                                          C.c_size_t]
        R.azref_infer.argtypes = [C.c_void_p, C.c_char_p, _F, C.c_int, _F, _F, _F, C.c_char_p, C.c_size_t]
        R.azref_inputs_positions.argtypes = [C.c_int, C.c_int, C.c_uint64, C.c_long, C.c_int, _F]
        R.azref_inputs_planes.argtypes = [C.c_uint64, C.c_size_t, _F]
        R.azref_bench_workers.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, _F, C.c_double,
                                          C.c_longlong, C.POINTER(C.c_longlong), C.c_char_p, C.c_size_t]
        R.azref_bench_workers.restype = C.c_double
        R.azref_blas_description.restype = C.c_char_p
        R.azref_rng_sample.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]
        R.azref_derive_seed.argtypes = [C.c_uint64] * 4
        R.azref_derive_seed.restype = C.c_uint64
        R.azref_save_checkpoint.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_size_t]
        R.azref_load_checkpoint.argtypes = [C.c_char_p, C.POINTER(C.c_int), _F, C.c_size_t, _F, C.c_size_t,
                                            C.c_char_p, C.c_size_t]
        _ref = R
    return _ref


class RefNetwork:
    """The reference's Network(cfg, seed) plus a randomiser, in its own code."""

    def __init__(self, cfg: NetConfig, seed: int, kind: int | None = KIND_BENCH):
        self.cfg = cfg
        self.h = ref().azref_net_create(cfg.board, cfg.history, cfg.blocks, cfg.filters, cfg.value_hidden,
                                        int(cfg.ownership), seed, -1 if kind is None else kind)
        if not self.h:
            raise RuntimeError("reference Network construction failed")

    def __del__(self):
        if getattr(self, "h", None):
            ref().azref_net_destroy(self.h)
            self.h = None

    def layout(self, which: int):
        R = ref()
        out = []
        name = C.create_string_buffer(64)
        size, off = C.c_size_t(), C.c_size_t()
        for i in range(R.azref_layout_count(self.h, which)):
            R.azref_layout_entry(self.h, which, i, name, 64, C.byref(size), C.byref(off))
            out.append((name.value.decode(), size.value, off.value))
        return out

    def arenas(self):
        R = ref()
        params = np.zeros(R.azref_floats(self.h, 0), np.float32)
        buffers = np.zeros(R.azref_floats(self.h, 1), np.float32)
        R.azref_export(self.h, _fp(params), _fp(buffers))
        return params, buffers

    @classmethod
    def from_arenas(cls, cfg: NetConfig, params: np.ndarray, buffers: np.ndarray) -> "RefNetwork":
        """The reference's Network of this shape holding the given arenas' tensors."""
        net = cls(cfg, 0, None)
        p = np.ascontiguousarray(params, np.float32)
        b = np.ascontiguousarray(buffers, np.float32)
        R = ref()
        assert p.size == R.azref_floats(net.h, 0) and b.size == R.azref_floats(net.h, 1)
        R.azref_import(net.h, _fp(p), _fp(b))
        return net

    def infer(self, x: np.ndarray, backend: str = "naive", threads: int = 1):
        """Network::infer (src/network.cpp:171-183); with threads > 1 the
        batch is split over that many workers (same outputs, position by position)."""
        cfg = self.cfg
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        logits = np.zeros((B, cfg.actions), np.float32)
        values = np.zeros(B, np.float32)
        own = np.zeros((B, cfg.area), np.float32) if cfg.ownership else None
        err = C.create_string_buffer(256)
        if threads > 1:
            rc = ref().azref_infer_threads(self.h, backend.encode(), _fp(x), B, _fp(logits), _fp(values), _fp(own),
                                           threads, err, 256)
        else:
            rc = ref().azref_infer(self.h, backend.encode(), _fp(x), B, _fp(logits), _fp(values), _fp(own), err, 256)
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return logits, values, own

    def save_checkpoint(self, path: str):
        """The reference's saveNetwork (src/checkpoint.cpp:80-100) of this network."""
        err = C.create_string_buffer(512)
        if ref().azref_save_checkpoint(self.h, os.fsencode(path), err, 512) != 0:
            raise RuntimeError(err.value.decode())

    def bench_workers(self, backend: str, workers: int, batch: int, x: np.ndarray, seconds: float = 0.0,
                      max_calls: int = 0):
        """(positions/s, positions) with `workers` threads of Network::infer at `batch`."""
        x = np.ascontiguousarray(x, np.float32)
        pos = C.c_longlong()
        err = C.create_string_buffer(256)
        rate = ref().azref_bench_workers(self.h, backend.encode(), workers, batch, _fp(x), seconds, max_calls,
                                         C.byref(pos), err, 256)
        if rate < 0:
            raise RuntimeError(err.value.decode())
        return rate, pos.value


def ref_load_checkpoint(path: str):
    """The reference's loadNetwork (src/checkpoint.cpp:102-133): (shape tuple
    (board, history, blocks, filters, value_hidden, ownership), params,
    buffers) when it loads, else the RuntimeError message it threw (a str)."""
    R = ref()
    shape = (C.c_int * 6)()
    err = C.create_string_buffer(1024)
    if R.azref_load_checkpoint(os.fsencode(path), shape, None, 0, None, 0, err, 1024) != 0:
        return err.value.decode()
    cfg = NetConfig(shape[0], shape[1], shape[2], shape[3], shape[4], bool(shape[5]))
    np_, nb = arena_floats(cfg)
    params = np.zeros(np_, np.float32)
    buffers = np.zeros(nb, np.float32)
    if R.azref_load_checkpoint(os.fsencode(path), shape, _fp(params), np_, _fp(buffers), nb, err, 1024) != 0:
        return err.value.decode()
    return tuple(shape), params, buffers


def ref_encode_records(cfg: NetConfig, records: np.ndarray) -> np.ndarray:
    """The reference's encodePlanes on position records (see stones_records in the package)."""
    records = np.ascontiguousarray(records, np.uint8)
    B = records.shape[0]
    out = np.zeros((B, cfg.planes, cfg.area), np.float32)
    L = ref()
    L.azref_encode_records.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_float)]
    L.azref_encode_records(cfg.board, cfg.history, B, records.ctypes.data, records.shape[1], _fp(out))
    return out


def ref_positions(cfg: NetConfig, seed: int, B: int, first: int = 0) -> np.ndarray:
    out = np.zeros((B, cfg.planes, cfg.area), np.float32)
    ref().azref_inputs_positions(cfg.board, cfg.history, seed, first, B, _fp(out))
    return out


def ref_rng_sample(seed: int, what: int, count: int, n: int = 0) -> np.ndarray:
    """The reference Rng's outputs: what 0 next() as (hi, lo) pairs, 1 uniform, 2 below(n), 3 normal."""
    out = np.zeros(count * (2 if what == 0 else 1), np.float64)
    ref().azref_rng_sample(seed, what, n, count, out.ctypes.data_as(C.POINTER(C.c_double)))
    return out


def rng_sample(seed: int, what: int, count: int, n: int = 0) -> np.ndarray:
    """The oracle's restated generator, same encoding as ref_rng_sample."""
    L = lib()
    L.az_rng_seed.argtypes = [C.c_void_p, C.c_uint64]
    L.az_rng_next.argtypes = [C.c_void_p]
    L.az_rng_next.restype = C.c_uint64
    L.az_rng_uniform.argtypes = [C.c_void_p]
    L.az_rng_uniform.restype = C.c_double
    L.az_rng_below.argtypes = [C.c_void_p, C.c_int]
    L.az_rng_normal.argtypes = [C.c_void_p]
    L.az_rng_normal.restype = C.c_double
    state = (C.c_uint64 * 4)()
    L.az_rng_seed(state, seed)
    out = []
    for _ in range(count):
        if what == 0:
            v = L.az_rng_next(state)
            out += [float(v >> 32), float(v & 0xFFFFFFFF)]
        elif what == 1:
            out.append(L.az_rng_uniform(state))
        elif what == 2:
            out.append(float(L.az_rng_below(state, n)))
        else:
            out.append(L.az_rng_normal(state))
    return np.array(out, np.float64)


def derive_seed(a: int, b: int = 0, c: int = 0, d: int = 0) -> int:
    return int(lib().az_derive_seed(a, b, c, d))


def blas_description() -> str:
    return ref().azref_blas_description().decode()


# ------------------------------------------------------------------ metrics


def max_err(x: np.ndarray, ref_: np.ndarray) -> float:
    """maxErr = max|x - ref| / max|ref| (tests/test_cuda.cpp:150-171)."""
    x = np.asarray(x, np.float64)
    r = np.asarray(ref_, np.float64)
    num = float(np.max(np.abs(x - r))) if x.size else 0.0
    den = float(np.max(np.abs(r))) if r.size else 0.0
    return num / den if den > 0 else num


def softmax(logits: np.ndarray) -> np.ndarray:
    z = np.asarray(logits, np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


# ------------------------------------------------ the reference's CUDA engine

REFCUDA_PATH = os.path.join(HERE, "_ref", "libazrefcuda.so")
_refcuda = None


def refcuda_built() -> bool:
    return os.path.exists(REFCUDA_PATH)


def refcuda() -> C.CDLL:
    """oracle/_ref/libazrefcuda.so: the reference's src/cuda engine built for sm_100 (`make -C oracle refcuda`)."""
    global _refcuda
    if _refcuda is None:
        L = C.CDLL(REFCUDA_PATH)
        F = C.POINTER(C.c_float)
        L.azrefcuda_available.argtypes = [C.c_char_p, C.c_size_t]
        L.azrefcuda_description.argtypes = [C.c_char_p, C.c_size_t]
        L.azrefcuda_create.argtypes = [C.c_int] * 5 + [F, C.c_size_t, F, C.c_size_t, C.c_int, C.c_char_p, C.c_size_t]
        L.azrefcuda_create.restype = C.c_void_p
        L.azrefcuda_destroy.argtypes = [C.c_void_p]
        L.azrefcuda_infer.argtypes = [C.c_void_p, F, C.c_int, F, F, C.c_char_p, C.c_size_t]
        L.azrefcuda_time.argtypes = [C.c_void_p, F, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double), C.c_char_p,
                                     C.c_size_t]
        _refcuda = L
    return _refcuda


def refcuda_available() -> tuple[bool, str]:
    why = C.create_string_buffer(512)
    ok = refcuda().azrefcuda_available(why, 512) == 1
    return ok, why.value.decode()


def refcuda_description() -> str:
    out = C.create_string_buffer(512)
    refcuda().azrefcuda_description(out, 512)
    return out.value.decode()


class RefCudaInference:
    """The reference's CudaInference (include/azgo/cuda.hpp:72-84) on the given arenas."""

    def __init__(self, cfg: NetConfig, params: np.ndarray, buffers: np.ndarray, max_batch: int):
        self.cfg = cfg
        p = np.ascontiguousarray(params, np.float32)
        b = np.ascontiguousarray(buffers, np.float32)
        err = C.create_string_buffer(1024)
        self.h = refcuda().azrefcuda_create(cfg.board, cfg.history, cfg.blocks, cfg.filters, cfg.value_hidden,
                                            _fp(p), p.size, _fp(b), b.size, max_batch, err, 1024)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def infer(self, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        B = x.shape[0]
        logits = np.empty((B, self.cfg.area + 1), np.float32)
        values = np.empty(B, np.float32)
        err = C.create_string_buffer(1024)
        if refcuda().azrefcuda_infer(self.h, _fp(x), B, _fp(logits), _fp(values), err, 1024) != 0:
            raise RuntimeError(err.value.decode())
        return logits, values

    def time(self, x: np.ndarray, warmup: int, steps: int) -> float:
        """Wall seconds of `steps` synchronous infer calls on x (copies included)."""
        x = np.ascontiguousarray(x, np.float32)
        secs = C.c_double()
        err = C.create_string_buffer(1024)
        if refcuda().azrefcuda_time(self.h, _fp(x), x.shape[0], warmup, steps, C.byref(secs), err, 1024) != 0:
            raise RuntimeError(err.value.decode())
        return secs.value

    def close(self):
        if self.h:
            refcuda().azrefcuda_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
