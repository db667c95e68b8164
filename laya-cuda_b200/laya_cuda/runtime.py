"""Runtime: resident weights and shape-class CUDA graphs, executed by liblaya_b200.so.

Drop-in for the reference Runtime (laya_cuda/runtime.py:136-197): same constructor,
`predict(items, capture=True) -> (logits[b, k], acts[b, n_act], metrics)`, `close()`, and the
attributes its tests read (`slots`, `pool.used_bytes()/total_bytes()`, `weights[name].get()`).
`span` and `classes` are importable without any GPU library (BatchEngine imports `span`).
"""
import ctypes as ct
from itertools import chain

import numpy as np


def span(tokens):
    """Rows start at multiples of 16 tokens, the attention tile (runtime.py:15-17)."""
    return -(-tokens // 16) * 16


def classes(items):
    """Shape class (runtime.py:20-25): packed rows (rounded to 32/64/128 steps), question count
    and option count (powers of two, options at least 8)."""
    rows = sum(span(len(item[0])) for item in items)
    step = 32 if rows <= 256 else 64 if rows <= 512 else 128
    pow2 = lambda n, low: max(low, 1 << (n - 1).bit_length())  # noqa: E731
    return -(-rows // step) * step, pow2(len(items), 1), pow2(max(len(item[1]) for item in items), 8)


PRECISIONS = {"bfloat16": 0, "float16": 1}


def flatten(items):
    """Items -> the C ABI's flat int32 arrays (tokens, lengths, markers, marker_counts, kinds)."""
    lengths = np.fromiter((len(item[0]) for item in items), np.int32, len(items))
    counts = np.fromiter((len(item[1]) for item in items), np.int32, len(items))
    kinds = np.fromiter((item[2] for item in items), np.int32, len(items))
    tokens = np.fromiter(chain.from_iterable(item[0] for item in items), np.int32, int(lengths.sum()))
    markers = np.fromiter(chain.from_iterable(item[1] for item in items), np.int32, int(counts.sum()))
    return tokens, lengths, markers, counts, kinds


def config_of(adapter, precision):
    from ._lib import Config
    return Config(vocab=adapter.config["vocab_size"], width=adapter.width, heads=adapter.heads,
                  layers=adapter.layers, intermediate=adapter.intermediate, global_every=adapter.global_every,
                  window=adapter.window, theta_global=adapter.theta[0], theta_local=adapter.theta[1],
                  eps=adapter.eps, max_len=adapter.max_len, head_layers=adapter.head_layers, n_act=adapter.n_act,
                  precision=PRECISIONS[precision])


def _ptr(array):
    return ct.c_void_p(array.ctypes.data) if array.size else ct.c_void_p(0)


class _Tensor:
    def __init__(self, runtime, name, shape):
        self.runtime, self.name, self.shape = runtime, name, shape

    def get(self):
        """The tensor as stored on the device, read back as fp32."""
        from . import _lib
        out = np.empty(self.shape, np.float32)
        _lib.check(self.runtime._lib.laya_read_tensor(self.runtime._handle, self.name.encode(),
                                                      out.ctypes.data_as(ct.POINTER(ct.c_float)), out.size),
                   self.runtime._handle)
        return out


class _Weights:
    def __init__(self, runtime, shapes):
        self._runtime, self._shapes = runtime, shapes

    def __getitem__(self, name):
        if name not in self._shapes or name == "temperature":
            raise KeyError(name)
        return _Tensor(self._runtime, name, self._shapes[name])

    def get(self, name, default=None):
        try:
            return self[name]
        except KeyError:
            return default

    def __contains__(self, name):
        return name in self._shapes and name != "temperature"

    def keys(self):
        return [n for n in self._shapes if n != "temperature"]

    def clear(self):
        self._shapes = {}


class _Pool:
    def __init__(self, runtime):
        self._runtime = runtime

    def _bytes(self):
        if self._runtime._handle is None:
            return 0, 0
        used, total = ct.c_uint64(), ct.c_uint64()
        self._runtime._lib.laya_pool_bytes(self._runtime._handle, ct.byref(used), ct.byref(total))
        return used.value, total.value

    def used_bytes(self):
        return self._bytes()[0]

    def total_bytes(self):
        return self._bytes()[1]


class _Slots:
    def __init__(self, runtime):
        self._runtime = runtime

    def __len__(self):
        if self._runtime._handle is None:
            return 0
        n = ct.c_int32()
        self._runtime._lib.laya_cached_shapes(self._runtime._handle, ct.byref(n))
        return n.value


class Runtime:
    def __init__(self, adapter, device, max_cached_shapes=16, precision="float16"):
        from . import _lib
        if precision not in PRECISIONS:
            raise ValueError("precision must be 'bfloat16' or 'float16'")
        self.adapter, self.device, self.limit, self.precision = adapter, device, max_cached_shapes, precision
        self._lib = _lib.load()
        self._handle = None
        self._pending = {}  # ticket -> (items, options, shape class) of submitted batches
        self.pool, self.slots = _Pool(self), _Slots(self)
        handle = ct.c_void_p()
        cfg = config_of(adapter, precision)
        _lib.check(self._lib.laya_create(ct.byref(cfg), device, max_cached_shapes, ct.byref(handle)))
        self._handle = handle
        try:
            shapes = adapter.weight_shapes()
            # The library maps the file, checks names and shapes (the reference's ValueErrors) and
            # streams it to the device (runtime.py:147-158 of the reference).
            path = str(adapter.path / "model.safetensors").encode()
            _lib.check(self._lib.laya_load_checkpoint(self._handle, path), self._handle)
            _lib.check(self._lib.laya_finalize(self._handle), self._handle)
            self.weights = _Weights(self, shapes)
        except BaseException:
            self.close()
            raise

    def predict(self, items, capture=True):
        """capture=True runs the class's CUDA graph (captured on first use) for classes of up
        to 8192 packed rows and an eager pass above that; capture=False always runs eagerly."""
        from . import _lib
        if self._handle is None:
            raise RuntimeError("Runtime is closed")
        rows, batch, options = classes(items)
        tokens, lengths, markers, counts, kinds = flatten(items)
        logits = np.empty((len(items), options), np.float32)
        acts = np.empty((len(items), self.adapter.n_act), np.float32)
        m = _lib.Metrics()
        _lib.check(self._lib.laya_predict(self._handle, _ptr(tokens), _ptr(lengths), _ptr(markers), _ptr(counts),
                                          _ptr(kinds), len(items), 2 if capture else 0, _ptr(logits), _ptr(acts),
                                          ct.byref(m)), self._handle)
        metrics = {"gpu_ms": m.gpu_ms, "shape": (rows, batch, options), "cache_miss": bool(m.cache_miss),
                   "graph_capture": bool(m.graph_capture), "graph_replay": bool(m.graph_replay),
                   "owned_gpu_bytes": m.owned_gpu_bytes, "kernel_launches": m.kernel_launches}
        return logits, acts, metrics

    def submit(self, items, capture=True):
        """Packs and launches one batch without waiting for it (at most two in flight); returns a
        ticket for collect().  The pair lets a caller prepare batch i+1 while batch i runs."""
        from . import _lib
        if self._handle is None:
            raise RuntimeError("Runtime is closed")
        rows, batch, options = classes(items)
        tokens, lengths, markers, counts, kinds = flatten(items)
        ticket = ct.c_int64()
        _lib.check(self._lib.laya_submit(self._handle, _ptr(tokens), _ptr(lengths), _ptr(markers), _ptr(counts),
                                         _ptr(kinds), len(items), 2 if capture else 0, ct.byref(ticket)), self._handle)
        self._pending[ticket.value] = (len(items), options, (rows, batch, options))
        return ticket.value

    def collect(self, ticket):
        """(logits, acts, metrics) of a submitted batch, as predict() returns them."""
        from . import _lib
        n, options, shape = self._pending.pop(ticket)
        logits = np.empty((n, options), np.float32)
        acts = np.empty((n, self.adapter.n_act), np.float32)
        m = _lib.Metrics()
        _lib.check(self._lib.laya_collect(self._handle, ticket, _ptr(logits), _ptr(acts), ct.byref(m)), self._handle)
        metrics = {"gpu_ms": m.gpu_ms, "shape": shape, "cache_miss": bool(m.cache_miss),
                   "graph_capture": bool(m.graph_capture), "graph_replay": bool(m.graph_replay),
                   "owned_gpu_bytes": m.owned_gpu_bytes, "kernel_launches": m.kernel_launches}
        return logits, acts, metrics

    def predict_many(self, batches, capture=True):
        """predict() over a sequence of batches with two in flight: each batch is packed and
        launched while the previous one runs.  Returns the results in order."""
        results, pending = [], []
        for items in batches:
            if len(pending) == 2:
                results.append(self.collect(pending.pop(0)))
            pending.append(self.submit(items, capture))
        results.extend(self.collect(t) for t in pending)
        return results

    def close(self):
        if self._handle is not None:
            handle, self._handle = self._handle, None
            self._lib.laya_destroy(handle)
        if hasattr(self, "weights"):
            self.weights.clear()
