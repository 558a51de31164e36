"""Drop-in for ggmlc's nanobind module ``ggmlc._runtime`` (runtime/bindings/python_bindings.cpp).

Same class and method names as the reference binding — ``ModelLoader``, ``SerializedModelGraph``,
``SerializedTensor``, ``SerializedOp``, ``ModelExecutor``, ``get_available_devices`` — backed by
the C ABI of ``libggmlc_b200.so`` (include/ggmlc_b200.h) through ctypes.  The executor runs on
CUDA only; there is no CPU fallback, and the module raises on import if the library is missing.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libggmlc_b200.so"


def _load() -> ctypes.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"ggmlc_b200 native library not found at {_LIB_PATH}; build it with "
            "`python -m ggmlc_b200.build` (nvcc, sm_100a)")
    L = ctypes.CDLL(str(_LIB_PATH))
    P, I, I64, U32, SZ, D, CP = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint32,
                                 ctypes.c_size_t, ctypes.c_double, ctypes.c_char_p)
    PP = ctypes.POINTER(ctypes.c_void_p)
    sigs = {
        "gb_last_error": ([], CP),
        "gb_version": ([], I),
        "gb_get_available_devices": ([ctypes.c_char_p, SZ], I),
        "gb_loader_load_from_file": ([CP, PP], I),
        "gb_loader_load_from_bytes": ([P, SZ, PP], I),
        "gb_graph_free": ([P], None),
        "gb_graph_name": ([P], CP),
        "gb_graph_num_symbols": ([P], I),
        "gb_graph_symbol": ([P, I], CP),
        "gb_graph_num_ids": ([P, I], I),
        "gb_graph_id": ([P, I, I, ctypes.POINTER(U32)], I),
        "gb_graph_num_tensors": ([P], I),
        "gb_graph_tensor_id": ([P, I, ctypes.POINTER(U32)], I),
        "gb_graph_tensor_info": ([P, U32, ctypes.POINTER(CP), ctypes.POINTER(I),
                                  ctypes.POINTER(I), ctypes.POINTER(ctypes.c_uint64)], I),
        "gb_graph_tensor_symbol_index": ([P, U32, I], I),
        "gb_graph_num_ops": ([P], I),
        "gb_graph_op_info": ([P, I, ctypes.POINTER(U32), ctypes.POINTER(I), ctypes.POINTER(CP)], I),
        "gb_graph_metadata_str": ([P, CP], CP),
        "gb_executor_create": ([P, CP, PP], I),
        "gb_executor_free": ([P], None),
        "gb_executor_device": ([P], CP),
        "gb_executor_prepare": ([P, ctypes.POINTER(CP), ctypes.POINTER(I64), I, I], I),
        "gb_executor_set_input": ([P, U32, P, SZ], I),
        "gb_executor_set_input_by_name": ([P, CP, P, SZ], I),
        "gb_executor_run": ([P, I], I),
        "gb_executor_synchronize": ([P], I),
        "gb_executor_get_output": ([P, U32, PP, ctypes.POINTER(SZ)], I),
        "gb_executor_get_tensor_shape": ([P, U32, ctypes.POINTER(I64)], I),
        "gb_executor_get_tensor_size_bytes": ([P, U32, ctypes.POINTER(SZ)], I),
        "gb_executor_set_state": ([P, U32, P, SZ], I),
        "gb_executor_get_state": ([P, U32, PP, ctypes.POINTER(SZ)], I),
        "gb_executor_reset_state": ([P], I),
        "gb_executor_init_kv_cache": ([P, I64], I),
        "gb_executor_reset_kv_cache": ([P], I),
        "gb_executor_has_kv_cache": ([P], I),
        "gb_executor_set_logits_last_only": ([P, I], I),
        "gb_executor_logits_last_only": ([P], I),
        "gb_executor_set_enable_cuda_graph": ([P, I], I),
        "gb_executor_is_cuda_graph_enabled": ([P], I),
        "gb_executor_is_cuda_graph_captured": ([P], I),
        "gb_executor_set_enable_profile": ([P, I], I),
        "gb_executor_reset_profile": ([P], I),
        "gb_executor_get_profile": ([P, ctypes.POINTER(D), ctypes.POINTER(D),
                                     ctypes.POINTER(I), ctypes.POINTER(I)], I),
        "gb_executor_graph_summary": ([P], CP),
        "gb_executor_mul_mat_shape_summary": ([P], CP),
        "gb_executor_launches_per_run": ([P], I64),
        "gb_executor_set_kernel_timing": ([P, I], I),
        "gb_executor_reset_kernel_times": ([P], I),
        "gb_executor_kernel_times": ([P], CP),
        "gb_executor_stream": ([P], P),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


_lib = _load()


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(_lib.gb_last_error().decode("utf-8", "replace"))


def lib() -> ctypes.CDLL:
    """The loaded libggmlc_b200.so handle."""
    return _lib


def get_available_devices() -> list[str]:
    """``["cpu", "cuda:0", ..., "cuda"]`` like the reference (python_bindings.cpp:133).

    "cpu" is listed because callers gate on it, but the B200 engine refuses it: the CPU path
    belongs to the reference runtime.
    """
    buf = ctypes.create_string_buffer(4096)
    n = _lib.gb_get_available_devices(buf, 4096)
    if n < 0:
        raise RuntimeError(_lib.gb_last_error().decode())
    return [d for d in buf.value.decode().split("\n") if d]


class SerializedTensor:
    """Read-only tensor record (python_bindings.cpp:71-92)."""

    __slots__ = ("_g", "id", "name", "data_size", "storage", "type")

    def __init__(self, graph: "SerializedModelGraph", tid: int):
        name = ctypes.c_char_p()
        ty = ctypes.c_int()
        st = ctypes.c_int()
        ds = ctypes.c_uint64()
        _check(_lib.gb_graph_tensor_info(graph._h, tid, ctypes.byref(name), ctypes.byref(ty),
                                         ctypes.byref(st), ctypes.byref(ds)))
        self._g = graph
        self.id = int(tid)
        self.name = name.value.decode()
        self.type = int(ty.value)
        self.storage = int(st.value)
        self.data_size = int(ds.value)

    def symbol_index(self, axis: int) -> int:
        return int(_lib.gb_graph_tensor_symbol_index(self._g._h, self.id, int(axis)))

    def __repr__(self) -> str:
        return f"SerializedTensor(id={self.id}, name={self.name!r}, type={self.type})"


class SerializedOp:
    """Read-only op record (python_bindings.cpp:93-98)."""

    __slots__ = ("id", "opcode", "name")

    def __init__(self, oid: int, opcode: int, name: str):
        self.id, self.opcode, self.name = oid, opcode, name


class SerializedModelGraph:
    """Loaded model graph (python_bindings.cpp:99-106)."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        self.name = _lib.gb_graph_name(self._h).decode()
        self.symbol_table = [_lib.gb_graph_symbol(self._h, i).decode()
                             for i in range(_lib.gb_graph_num_symbols(self._h))]

        def ids(which: int) -> list[int]:
            out = []
            for i in range(_lib.gb_graph_num_ids(self._h, which)):
                v = ctypes.c_uint32()
                _check(_lib.gb_graph_id(self._h, which, i, ctypes.byref(v)))
                out.append(int(v.value))
            return out

        self.inputs = ids(0)
        self.outputs = ids(1)
        self.parameters = ids(2)
        self.tensors: dict[int, SerializedTensor] = {}
        for i in range(_lib.gb_graph_num_tensors(self._h)):
            v = ctypes.c_uint32()
            _check(_lib.gb_graph_tensor_id(self._h, i, ctypes.byref(v)))
            self.tensors[int(v.value)] = SerializedTensor(self, int(v.value))
        self.ops = []
        for i in range(_lib.gb_graph_num_ops(self._h)):
            oid, opc, nm = ctypes.c_uint32(), ctypes.c_int(), ctypes.c_char_p()
            _check(_lib.gb_graph_op_info(self._h, i, ctypes.byref(oid), ctypes.byref(opc),
                                         ctypes.byref(nm)))
            self.ops.append(SerializedOp(int(oid.value), int(opc.value), nm.value.decode()))

    def metadata(self, key: str) -> str | None:
        v = _lib.gb_graph_metadata_str(self._h, key.encode())
        return None if v is None else v.decode()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.gb_graph_free(h)
            self._h = ctypes.c_void_p()


class ModelLoader:
    """GGUF loader (python_bindings.cpp:108-130)."""

    @staticmethod
    def load_from_file(filepath: str) -> SerializedModelGraph:
        h = ctypes.c_void_p()
        _check(_lib.gb_loader_load_from_file(str(filepath).encode(), ctypes.byref(h)))
        return SerializedModelGraph(h.value)

    @staticmethod
    def load_from_bytes(data: bytes) -> SerializedModelGraph:
        h = ctypes.c_void_p()
        buf = bytes(data)
        _check(_lib.gb_loader_load_from_bytes(buf, len(buf), ctypes.byref(h)))
        return SerializedModelGraph(h.value)


def _as_c(array: Any) -> np.ndarray:
    a = np.ascontiguousarray(array)
    return a


class ModelExecutor:
    """CUDA executor with the reference ModelExecutor's interface (python_bindings.cpp:136-217).

    ``run`` and ``synchronize`` do not hold the interpreter in C for long: kernels are queued
    on the executor's stream and ``get_output_bytes`` waits for them.
    """

    def __init__(self, graph: SerializedModelGraph, device: str = "cpu"):
        h = ctypes.c_void_p()
        _check(_lib.gb_executor_create(graph._h, str(device).encode(), ctypes.byref(h)))
        self._h = h
        self._graph = graph  # keeps the mmap'd GGUF alive
        self._names = {t.name: tid for tid, t in graph.tensors.items()}

    @property
    def device(self) -> str:
        return _lib.gb_executor_device(self._h).decode()

    def prepare(self, symbols: dict[str, int] | None = None, enable_arena_reuse: bool = True):
        symbols = dict(symbols or {})
        n = len(symbols)
        names = (ctypes.c_char_p * max(n, 1))(*[k.encode() for k in symbols])
        vals = (ctypes.c_int64 * max(n, 1))(*[int(v) for v in symbols.values()])
        _check(_lib.gb_executor_prepare(self._h, names, vals, n, int(bool(enable_arena_reuse))))

    def set_input_by_id(self, tensor_id: int, array: np.ndarray) -> None:
        a = _as_c(array)
        _check(_lib.gb_executor_set_input(self._h, int(tensor_id), a.ctypes.data, a.nbytes))

    def set_input_by_name(self, name: str, array: np.ndarray) -> None:
        a = _as_c(array)
        _check(_lib.gb_executor_set_input_by_name(self._h, name.encode(), a.ctypes.data, a.nbytes))

    def set_state_by_id(self, tensor_id: int, array: np.ndarray) -> None:
        a = _as_c(array)
        _check(_lib.gb_executor_set_state(self._h, int(tensor_id), a.ctypes.data, a.nbytes))

    def set_state_by_name(self, name: str, array: np.ndarray) -> None:
        if name not in self._names:
            raise RuntimeError(f"no state tensor named '{name}'")
        self.set_state_by_id(self._names[name], array)

    def run(self, n_threads: int = 1) -> None:
        _check(_lib.gb_executor_run(self._h, int(n_threads)))

    def synchronize(self) -> None:
        _check(_lib.gb_executor_synchronize(self._h))

    def _bytes(self, fn, tensor_id: int) -> bytes:
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        _check(fn(self._h, int(tensor_id), ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p.value, n.value)

    def get_output_bytes(self, tensor_id: int) -> bytes:
        return self._bytes(_lib.gb_executor_get_output, tensor_id)

    def get_output_array(self, tensor_id: int) -> np.ndarray:
        """f32 view of an output without the extra bytes copy (engine extension)."""
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        _check(_lib.gb_executor_get_output(self._h, int(tensor_id), ctypes.byref(p),
                                           ctypes.byref(n)))
        buf = (ctypes.c_char * n.value).from_address(p.value)
        return np.frombuffer(buf, dtype=np.float32).copy()

    def get_state_bytes(self, tensor_id: int) -> bytes:
        return self._bytes(_lib.gb_executor_get_state, tensor_id)

    def get_state_bytes_by_name(self, name: str) -> bytes:
        if name not in self._names:
            raise RuntimeError(f"no state tensor named '{name}'")
        return self.get_state_bytes(self._names[name])

    def get_tensor_shape(self, tensor_id: int) -> list[int]:
        ne = (ctypes.c_int64 * 4)()
        _check(_lib.gb_executor_get_tensor_shape(self._h, int(tensor_id), ne))
        return [int(x) for x in ne]

    def get_tensor_size_bytes(self, tensor_id: int) -> int:
        n = ctypes.c_size_t()
        _check(_lib.gb_executor_get_tensor_size_bytes(self._h, int(tensor_id), ctypes.byref(n)))
        return int(n.value)

    def reset_state(self) -> None:
        _check(_lib.gb_executor_reset_state(self._h))

    def init_kv_cache(self, max_ctx: int = 2048) -> None:
        _check(_lib.gb_executor_init_kv_cache(self._h, int(max_ctx)))

    def reset_kv_cache(self) -> None:
        _check(_lib.gb_executor_reset_kv_cache(self._h))

    def has_kv_cache(self) -> bool:
        return bool(_lib.gb_executor_has_kv_cache(self._h))

    def set_logits_last_only(self, enable: bool) -> None:
        _check(_lib.gb_executor_set_logits_last_only(self._h, int(bool(enable))))

    def logits_last_only(self) -> bool:
        return bool(_lib.gb_executor_logits_last_only(self._h))

    def set_enable_cuda_graph(self, enable: bool) -> None:
        _check(_lib.gb_executor_set_enable_cuda_graph(self._h, int(bool(enable))))

    def is_cuda_graph_enabled(self) -> bool:
        return bool(_lib.gb_executor_is_cuda_graph_enabled(self._h))

    def is_cuda_graph_captured(self) -> bool:
        return bool(_lib.gb_executor_is_cuda_graph_captured(self._h))

    # bucketed graphs: one decode program (and CUDA graph) per batch bucket is kept anyway
    def set_enable_cuda_graph_buckets(self, enable: bool) -> None:
        self.set_enable_cuda_graph(enable)

    def is_cuda_graph_buckets_enabled(self) -> bool:
        return self.is_cuda_graph_enabled()

    def is_cuda_graph_bucket_captured(self, batch_size: int) -> bool:
        return self.is_cuda_graph_captured()

    def set_enable_profile(self, enable: bool) -> None:
        _check(_lib.gb_executor_set_enable_profile(self._h, int(bool(enable))))

    def reset_profile(self) -> None:
        _check(_lib.gb_executor_reset_profile(self._h))

    def get_profile(self) -> dict[str, float]:
        a, b = ctypes.c_double(), ctypes.c_double()
        c, d = ctypes.c_int(), ctypes.c_int()
        _check(_lib.gb_executor_get_profile(self._h, ctypes.byref(a), ctypes.byref(b),
                                            ctypes.byref(c), ctypes.byref(d)))
        return {"prepare_ms": a.value, "run_ms": b.value, "n_prepare": c.value, "n_run": d.value}

    def runtime_graph_summary(self) -> str:
        return _lib.gb_executor_graph_summary(self._h).decode()

    def runtime_mul_mat_shape_summary(self) -> str:
        return _lib.gb_executor_mul_mat_shape_summary(self._h).decode()

    def launches_per_run(self) -> int:
        return int(_lib.gb_executor_launches_per_run(self._h))

    def set_kernel_timing(self, enable: bool) -> None:
        _check(_lib.gb_executor_set_kernel_timing(self._h, int(bool(enable))))

    def reset_kernel_times(self) -> None:
        _check(_lib.gb_executor_reset_kernel_times(self._h))

    def kernel_times(self) -> dict[str, list[float]]:
        import json

        return json.loads(_lib.gb_executor_kernel_times(self._h).decode())

    def stream(self) -> int:
        return int(_lib.gb_executor_stream(self._h) or 0)

    @staticmethod
    def ggml_cuda_graphs_compiled() -> bool:
        return True

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.gb_executor_free(h)
            self._h = ctypes.c_void_p()
