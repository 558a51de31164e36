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
        "gb_executor_create_tp": ([P, CP, I, I, P, PP], I),
        "gb_nccl_unique_id": ([P], I),
        "gb_tp_plan": ([P, I, I], CP),
        "gb_executor_tp_size": ([P], I),
        "gb_executor_tp_rank": ([P], I),
        "gb_executor_tp_error": ([P], I),
        "gb_executor_free": ([P], None),
        "gb_executor_device": ([P], CP),
        "gb_executor_prepare": ([P, ctypes.POINTER(CP), ctypes.POINTER(I64), I, I], I),
        "gb_executor_set_input": ([P, U32, P, SZ], I),
        "gb_executor_set_input_by_name": ([P, CP, P, SZ], I),
        "gb_executor_run": ([P, I], I),
        "gb_executor_synchronize": ([P], I),
        "gb_executor_get_output": ([P, U32, PP, ctypes.POINTER(SZ)], I),
        "gb_executor_output_argmax": ([P, U32, I, ctypes.POINTER(ctypes.c_int32)], I),
        "gb_executor_get_tensor_shape": ([P, U32, ctypes.POINTER(I64)], I),
        "gb_executor_get_tensor_size_bytes": ([P, U32, ctypes.POINTER(SZ)], I),
        "gb_executor_set_state": ([P, U32, P, SZ], I),
        "gb_executor_get_state": ([P, U32, PP, ctypes.POINTER(SZ)], I),
        "gb_executor_reset_state": ([P], I),
        "gb_executor_init_kv_cache": ([P, I64], I),
        "gb_executor_reset_kv_cache": ([P], I),
        "gb_executor_has_kv_cache": ([P], I),
        "gb_executor_set_logits_last_only": ([P, I], I),
        "gb_executor_set_output_rows": ([P, P, I], I),
        "gb_executor_logits_last_only": ([P], I),
        "gb_executor_set_enable_cuda_graph": ([P, I], I),
        "gb_executor_is_cuda_graph_enabled": ([P], I),
        "gb_executor_is_cuda_graph_captured": ([P], I),
        "gb_executor_set_decode_chain": ([P, I], I),
        "gb_executor_decode_chain": ([P], I),
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
        "gb_executor_init_paged_kv_cache": ([P, I64, I64], I),
        "gb_executor_is_paged_kv_cache_enabled": ([P], I),
        "gb_executor_paged_kv_alloc_slot": ([P, I64], I),
        "gb_executor_paged_kv_free_slot": ([P, I64], I),
        "gb_executor_paged_kv_ensure_tokens": ([P, I64, I64], I),
        "gb_executor_paged_active_vram_bytes": ([P], I64),
        "gb_executor_tokens_per_page": ([P], I64),
        "gb_executor_set_tokens_per_page": ([P, I64], I),
        "gb_executor_prepare_batch": ([P, I, P, P], I),
        "gb_scheduler_create": ([P, I, I, PP], I),
        "gb_scheduler_free": ([P], None),
        "gb_scheduler_add_request": ([P, P, I64, I, ctypes.c_float, I,
                                      ctypes.POINTER(ctypes.c_uint64)], I),
        "gb_scheduler_step": ([P, P, P, I, ctypes.POINTER(I), P, I, ctypes.POINTER(I)], I),
        "gb_scheduler_has_work": ([P], I),
        "gb_scheduler_active_count": ([P], I64),
        "gb_scheduler_pending_count": ([P], I64),
        "gb_scheduler_max_batch_size": ([P], I),
        "gb_scheduler_enable_prefix_caching": ([P, I], I),
        "gb_scheduler_is_prefix_caching_enabled": ([P], I),
        "gb_scheduler_get_request": ([P, ctypes.c_uint64, P], I),
        "gb_scheduler_request_tokens": ([P, ctypes.c_uint64, I, P, I64, ctypes.POINTER(I64)], I),
        "gb_scheduler_prefix_stats": ([P, ctypes.POINTER(I64), ctypes.POINTER(I64)], I),
        "gb_executor_configure_prefix_pool": ([P, I64], I),
        "gb_executor_configure_kv_pool_pages": ([P, I64], I),
        "gb_executor_kv_pool_pages": ([P], I64),
        "gb_executor_kv_free_pages": ([P], I64),
        "gb_radix_create": ([I64, PP], I),
        "gb_radix_free": ([P], None),
        "gb_radix_tokens_per_page": ([P], I64),
        "gb_radix_total_cached_pages": ([P], I64),
        "gb_radix_total_nodes": ([P], I64),
        "gb_radix_reset": ([P], None),
        "gb_radix_match_prefix": ([P, P, I64, ctypes.POINTER(I64), ctypes.POINTER(I64)], I),
        "gb_radix_insert_prefix": ([P, P, I64, ctypes.POINTER(I64)], I),
        "gb_radix_evict_lru": ([P], I64),
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


def nccl_unique_id() -> bytes:
    """128-byte NCCL unique id for a tensor-parallel group (made once, by rank 0)."""
    buf = ctypes.create_string_buffer(128)
    _check(_lib.gb_nccl_unique_id(buf))
    return buf.raw


def tensor_parallel_plan(graph: SerializedModelGraph, tp_rank: int, tp_size: int) -> dict:
    """One rank's tensor-parallel plan (weight slices, partial sums, rewritten shapes); host only."""
    import json

    out = _lib.gb_tp_plan(graph._h, int(tp_rank), int(tp_size))
    if not out:
        raise RuntimeError(_lib.gb_last_error().decode())
    return json.loads(out.decode())


class ModelExecutor:
    """CUDA executor with the reference ModelExecutor's interface (python_bindings.cpp:136-217).

    ``run`` and ``synchronize`` do not hold the interpreter in C for long: kernels are queued
    on the executor's stream and ``get_output_bytes`` waits for them.
    """

    def __init__(self, graph: SerializedModelGraph, device: str = "cpu", tp_rank: int = 0,
                 tp_size: int = 1, nccl_id: bytes | None = None):
        """``tp_size > 1``: rank ``tp_rank`` of a tensor-parallel group (no counterpart in the
        reference).  ``nccl_id`` is the group's ``nccl_unique_id()`` made by rank 0 and shared
        by the caller; every rank constructs its executor at the same time (collective)."""
        h = ctypes.c_void_p()
        if int(tp_size) > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tensor parallelism needs the group's 128-byte nccl_unique_id()")
            idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128)
            _check(_lib.gb_executor_create_tp(graph._h, str(device).encode(), int(tp_rank),
                                              int(tp_size), idbuf, ctypes.byref(h)))
        else:
            _check(_lib.gb_executor_create(graph._h, str(device).encode(), ctypes.byref(h)))
        self._h = h
        self._graph = graph  # keeps the mmap'd GGUF alive
        self._names = {t.name: tid for tid, t in graph.tensors.items()}

    @property
    def device(self) -> str:
        return _lib.gb_executor_device(self._h).decode()

    @property
    def tp_size(self) -> int:
        return int(_lib.gb_executor_tp_size(self._h))

    @property
    def tp_rank(self) -> int:
        return int(_lib.gb_executor_tp_rank(self._h))

    def tp_allreduce_error(self) -> int:
        """0 while every peer all-reduce completed its waits; 1 once one gave up on a peer."""
        return int(_lib.gb_executor_tp_error(self._h))

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

    def output_argmax(self, tensor_id: int, rows: int = 1) -> np.ndarray:
        """Greedy token (first maximum) of each of `rows` rows of an f32 output, computed on the
        device; only the indices are copied (engine extension, no reference twin)."""
        out = np.empty(rows, np.int32)
        _check(_lib.gb_executor_output_argmax(
            self._h, int(tensor_id), int(rows), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out

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

    def set_output_rows(self, rows=None) -> None:
        """Compute the output projections of the next prefills for these rows of the call's
        tokens only (llama's out_ids; at most 64), logits [len(rows), vocab]; None or [] turns it
        off.  Takes precedence over set_logits_last_only."""
        r = np.ascontiguousarray([] if rows is None else rows, np.int32).reshape(-1)
        _check(_lib.gb_executor_set_output_rows(self._h, r.ctypes.data if len(r) else None,
                                                len(r)))

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

    def set_decode_chain(self, enable: bool) -> None:
        """Engine switch (no reference twin): run single-sequence decode steps as one persistent
        launch (off by default; GGMLC_B200_CHAIN=1 turns the default on)."""
        _check(_lib.gb_executor_set_decode_chain(self._h, int(bool(enable))))

    def decode_chain(self) -> bool:
        return bool(_lib.gb_executor_decode_chain(self._h))

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

    # ---- paged KV cache (python_bindings.cpp:196-204) ----------------------------------------
    def init_paged_kv_cache(self, max_batch: int = 8, max_ctx: int = 2048) -> None:
        _check(_lib.gb_executor_init_paged_kv_cache(self._h, int(max_batch), int(max_ctx)))

    def is_paged_kv_cache_enabled(self) -> bool:
        return bool(_lib.gb_executor_is_paged_kv_cache_enabled(self._h))

    def paged_kv_alloc_slot(self, slot_id: int, prefix_hash: str = "") -> None:
        _check(_lib.gb_executor_paged_kv_alloc_slot(self._h, int(slot_id)))

    def paged_kv_free_slot(self, slot_id: int) -> None:
        _check(_lib.gb_executor_paged_kv_free_slot(self._h, int(slot_id)))

    def paged_kv_ensure_tokens(self, slot_id: int, total_tokens: int) -> None:
        _check(_lib.gb_executor_paged_kv_ensure_tokens(self._h, int(slot_id), int(total_tokens)))

    def get_paged_active_vram_bytes(self) -> int:
        return int(_lib.gb_executor_paged_active_vram_bytes(self._h))

    def configure_vmm_pool(self, max_warm_pages: int = 64, prealloc_pages: int = 0) -> None:
        """Pages kept for the prefix cache on top of max_batch full sequences (max_warm_pages),
        read at the next init_paged_kv_cache.  The whole pool is allocated at init, so
        prealloc_pages is accepted and has nothing left to do."""
        _check(_lib.gb_executor_configure_prefix_pool(self._h, int(max_warm_pages)))

    def configure_kv_pool_pages(self, pages: int) -> None:
        """Exact page count of the pool at the next init_paged_kv_cache (0: max_batch full
        sequences plus the prefix pages).  A smaller pool serves more short sequences: the
        scheduler admits requests as their pages allow."""
        _check(_lib.gb_executor_configure_kv_pool_pages(self._h, int(pages)))

    @property
    def kv_pool_pages(self) -> int:
        return int(_lib.gb_executor_kv_pool_pages(self._h))

    @property
    def kv_free_pages(self) -> int:
        return int(_lib.gb_executor_kv_free_pages(self._h))

    @property
    def tokens_per_page(self) -> int:
        return int(_lib.gb_executor_tokens_per_page(self._h))

    def set_tokens_per_page(self, tokens_per_page: int) -> None:
        _check(_lib.gb_executor_set_tokens_per_page(self._h, int(tokens_per_page)))

    def prepare_batch(self, pos: np.ndarray, slot: np.ndarray) -> None:
        """One decode token for each of len(pos) sequences (row r at pos[r] in slot slot[r])."""
        p = np.ascontiguousarray(pos, np.int32)
        s = np.ascontiguousarray(slot, np.int32)
        if p.shape != s.shape or p.ndim != 1:
            raise ValueError("pos and slot must be 1-D arrays of equal length")
        _check(_lib.gb_executor_prepare_batch(self._h, len(p), p.ctypes.data, s.ctypes.data))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.gb_executor_free(h)
            self._h = ctypes.c_void_p()


# ---- prefix cache index (radix_tree.h; python_bindings.cpp:248-258) --------------------------
class PrefixMatchResult:
    def __init__(self, matched_pages: int, matched_tokens: int):
        self.matched_pages = matched_pages
        self.matched_tokens = matched_tokens


class PagedRadixTree:
    """Trie over whole pages of tokens_per_page tokens (FNV-1a chunk hashes checked token by
    token, least-recently-used leaf eviction), the index the scheduler's prefix cache uses."""

    def __init__(self, tokens_per_page: int = 1024):
        h = ctypes.c_void_p()
        _check(_lib.gb_radix_create(int(tokens_per_page), ctypes.byref(h)))
        self._h = h

    @property
    def tokens_per_page(self) -> int:
        return int(_lib.gb_radix_tokens_per_page(self._h))

    @property
    def total_cached_pages(self) -> int:
        return int(_lib.gb_radix_total_cached_pages(self._h))

    @property
    def total_nodes(self) -> int:
        return int(_lib.gb_radix_total_nodes(self._h))

    def match_prefix(self, prompt_tokens) -> PrefixMatchResult:
        t = np.ascontiguousarray(prompt_tokens, np.int32).reshape(-1)
        pages, toks = ctypes.c_int64(), ctypes.c_int64()
        _check(_lib.gb_radix_match_prefix(self._h, t.ctypes.data, len(t), ctypes.byref(pages),
                                          ctypes.byref(toks)))
        return PrefixMatchResult(int(pages.value), int(toks.value))

    def insert_prefix(self, prompt_tokens) -> int:
        """Index the whole pages of prompt_tokens not yet present; returns how many were added."""
        t = np.ascontiguousarray(prompt_tokens, np.int32).reshape(-1)
        added = ctypes.c_int64()
        _check(_lib.gb_radix_insert_prefix(self._h, t.ctypes.data, len(t), ctypes.byref(added)))
        return int(added.value)

    def evict_lru(self) -> int:
        """Drop the least recently used leaf page; its page id, or -1 when none can go."""
        return int(_lib.gb_radix_evict_lru(self._h))

    def reset(self) -> None:
        _lib.gb_radix_reset(self._h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib is not None:
            _lib.gb_radix_free(h)
            self._h = ctypes.c_void_p()


# ---- continuous batching (batch_scheduler.h:35-77; python_bindings.cpp:261-295) -------------
class _RequestInfo(ctypes.Structure):
    _fields_ = [("request_id", ctypes.c_uint64), ("slot_id", ctypes.c_int),
                ("current_pos", ctypes.c_int64), ("max_new_tokens", ctypes.c_int),
                ("temperature", ctypes.c_float), ("eos_token_id", ctypes.c_int),
                ("finished", ctypes.c_int), ("finish_reason", ctypes.c_char_p),
                ("n_prompt_tokens", ctypes.c_int64), ("n_generated_tokens", ctypes.c_int64),
                ("prefix_tokens_matched", ctypes.c_int64)]


class GenerationRequest:
    """Read-only snapshot of a request (python_bindings.cpp:261-272)."""

    def __init__(self, info: _RequestInfo, prompt: list[int], generated: list[int]):
        self.request_id = int(info.request_id)
        self.prompt_tokens = prompt
        self.generated_tokens = generated
        self.slot_id = int(info.slot_id)
        self.current_pos = int(info.current_pos)
        self.max_new_tokens = int(info.max_new_tokens)
        self.temperature = float(info.temperature)
        self.eos_token_id = int(info.eos_token_id)
        self.finished = bool(info.finished)
        self.finish_reason = (info.finish_reason or b"").decode()
        self.prefix_tokens_matched = int(info.prefix_tokens_matched)


class StepResult:
    """new_tokens: [(request_id, token_id)], completed_request_ids (python_bindings.cpp:274-276)."""

    def __init__(self, new_tokens: list[tuple[int, int]], completed: list[int]):
        self.new_tokens = new_tokens
        self.completed_request_ids = completed


class ContinuousBatchScheduler:
    """Iteration-level continuous batching over the executor's paged KV cache.

    Same interface as the reference scheduler (python_bindings.cpp:278-294).  Each step admits
    every pending request that finds a free slot (prefill in it) or decodes one token of every
    active sequence, each at its own position.  Prefix caching (on by default) maps the pages of
    whole cached prompt pages (executor.tokens_per_page tokens each) into the new sequence's page
    table, shared rather than copied, and prefills the rest.  A request waits while the KV pool
    lacks the pages it may claim (prompt + max_new_tokens).
    """

    def __init__(self, executor: ModelExecutor, max_batch_size: int = 8, eos_token_id: int = 0):
        h = ctypes.c_void_p()
        _check(_lib.gb_scheduler_create(executor._h, int(max_batch_size), int(eos_token_id),
                                        ctypes.byref(h)))
        self._h = h
        self._executor = executor  # the scheduler drives this executor

    def add_request(self, prompt_tokens, max_new_tokens: int = 32, temperature: float = 0.0,
                    eos_token_id: int = -1) -> int:
        p = np.ascontiguousarray(prompt_tokens, np.int32).reshape(-1)
        rid = ctypes.c_uint64()
        _check(_lib.gb_scheduler_add_request(self._h, p.ctypes.data, len(p), int(max_new_tokens),
                                             float(temperature), int(eos_token_id),
                                             ctypes.byref(rid)))
        return int(rid.value)

    def step(self) -> StepResult:
        cap = 64
        ids = (ctypes.c_uint64 * cap)()
        toks = (ctypes.c_int32 * cap)()
        done = (ctypes.c_uint64 * cap)()
        n_new, n_done = ctypes.c_int(), ctypes.c_int()
        _check(_lib.gb_scheduler_step(self._h, ids, toks, cap, ctypes.byref(n_new), done, cap,
                                      ctypes.byref(n_done)))
        return StepResult([(int(ids[i]), int(toks[i])) for i in range(n_new.value)],
                          [int(done[i]) for i in range(n_done.value)])

    def has_work(self) -> bool:
        return bool(_lib.gb_scheduler_has_work(self._h))

    def active_count(self) -> int:
        return int(_lib.gb_scheduler_active_count(self._h))

    def pending_count(self) -> int:
        return int(_lib.gb_scheduler_pending_count(self._h))

    def max_batch_size(self) -> int:
        return int(_lib.gb_scheduler_max_batch_size(self._h))

    def enable_prefix_caching(self, enable: bool) -> None:
        _check(_lib.gb_scheduler_enable_prefix_caching(self._h, int(bool(enable))))

    def is_prefix_caching_enabled(self) -> bool:
        return bool(_lib.gb_scheduler_is_prefix_caching_enabled(self._h))

    def _prefix_stats(self) -> tuple[int, int]:
        hits, saved = ctypes.c_int64(), ctypes.c_int64()
        _check(_lib.gb_scheduler_prefix_stats(self._h, ctypes.byref(hits), ctypes.byref(saved)))
        return int(hits.value), int(saved.value)

    @property
    def total_prefix_cache_hits(self) -> int:
        return self._prefix_stats()[0]

    @property
    def total_prefix_tokens_saved(self) -> int:
        return self._prefix_stats()[1]

    def _tokens(self, rid: int, which: int) -> list[int]:
        n = ctypes.c_int64()
        _check(_lib.gb_scheduler_request_tokens(self._h, rid, which, None, 0, ctypes.byref(n)))
        buf = np.empty(n.value, np.int32)
        _check(_lib.gb_scheduler_request_tokens(self._h, rid, which, buf.ctypes.data, n.value,
                                                ctypes.byref(n)))
        return [int(t) for t in buf]

    def get_request(self, request_id: int) -> GenerationRequest:
        info = _RequestInfo()
        _check(_lib.gb_scheduler_get_request(self._h, int(request_id), ctypes.byref(info)))
        return GenerationRequest(info, self._tokens(int(request_id), 0),
                                 self._tokens(int(request_id), 1))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value and _lib is not None:
            _lib.gb_scheduler_free(h)
            self._h = ctypes.c_void_p()
