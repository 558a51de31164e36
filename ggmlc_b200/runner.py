"""``ModelRunner`` / ``load`` over the B200 engine, mirroring python/ggmlc/runtime/runner.py.

Same constructor, ``__call__`` symbol deduction (GGUF-loaded graphs bind ggml ``ne[i]`` to numpy
axis ``-1-i`` through ``SerializedTensor.symbol_index``, runner.py:143-156; a lone ``s`` symbol
fills every sequence-like symbol, :164-171), input binding (int64 -> int32 for I32 inputs,
:182-209), outputs reshaped from ggml ``ne`` to C order (:216-255) and the KV-cache helpers
(:295-316).  The executor is the CUDA one; ``device="cpu"`` raises.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import numpy as np

from . import _runtime

# ggml type id -> numpy dtype (runner.py:23-31)
GGML_TYPE_TO_NUMPY: dict[int, np.dtype] = {
    0: np.dtype(np.float32),
    1: np.dtype(np.float16),
    24: np.dtype(np.int8),
    25: np.dtype(np.int16),
    26: np.dtype(np.int32),
    27: np.dtype(np.int64),
    28: np.dtype(np.float64),
}
_I32 = 26


def get_available_devices() -> list[str]:
    return _runtime.get_available_devices()


class ModelRunner:
    def __init__(self, model_source: str | Path | bytes, n_threads: int = 1,
                 device: str = "cuda") -> None:
        self.n_threads = n_threads
        if isinstance(model_source, (str, Path)):
            p = Path(model_source).resolve()
            if not p.exists():
                raise FileNotFoundError(f"Model file not found: {p}")
            self.graph = _runtime.ModelLoader.load_from_file(str(p))
        elif isinstance(model_source, (bytes, bytearray)):
            self.graph = _runtime.ModelLoader.load_from_bytes(bytes(model_source))
        else:
            raise TypeError(f"Expected file path or bytes, got {type(model_source)}")
        self.executor = _runtime.ModelExecutor(self.graph, device)
        self.device = self.executor.device
        self.name = self.graph.name
        self.symbol_table = list(self.graph.symbol_table)
        self.inputs = list(self.graph.inputs)
        self.outputs = list(self.graph.outputs)
        self.parameters = list(self.graph.parameters)
        self.input_name_to_id: dict[str, int] = {}
        self.tensor_info: dict[int, Any] = {}
        for tid, t in self.graph.tensors.items():
            self.tensor_info[tid] = t
            if tid in self.inputs:
                self.input_name_to_id[t.name] = tid

    def _bind(self, tid: int, arr: np.ndarray) -> None:
        t = self.tensor_info.get(tid)
        a = np.ascontiguousarray(arr)
        if t is not None and t.type == _I32 and a.dtype == np.int64:
            a = a.astype(np.int32)
        self.executor.set_input_by_id(tid, a)

    def __call__(self, *args: np.ndarray, symbols: dict[str, int] | None = None,
                 n_threads: int | None = None, enable_arena_reuse: bool = True,
                 **kwargs: np.ndarray):
        if len(args) == 1 and isinstance(args[0], dict) and not kwargs:
            kwargs = args[0]
            args = ()
        env: dict[str, int] = dict(symbols or {})
        if args and self.symbol_table and hasattr(args[0], "shape") and self.inputs:
            t0 = self.tensor_info.get(self.inputs[0])
            shp = args[0].shape
            for i in range(min(4, len(shp))):
                sidx = int(t0.symbol_index(i)) if t0 is not None else -1
                if 0 <= sidx < len(self.symbol_table):
                    name = self.symbol_table[sidx]
                    env.setdefault(name, int(shp[len(shp) - 1 - i]))
        if symbols and len(self.symbol_table) == len(symbols):
            for reg, val in zip(self.symbol_table, symbols.values()):
                env.setdefault(reg, int(val))
        if "s" in env:
            for sym in self.symbol_table:
                if (sym.startswith("s") or "seq" in sym) and sym not in env:
                    env[sym] = env["s"]
            if len(self.symbol_table) == 1:
                env.setdefault(self.symbol_table[0], env["s"])
        self.executor.prepare(env, enable_arena_reuse)
        for idx, arr in enumerate(args):
            if idx >= len(self.inputs):
                raise ValueError(f"Too many positional arguments: model expects "
                                 f"{len(self.inputs)} inputs, got {len(args)}")
            self._bind(self.inputs[idx], arr)
        for name, arr in kwargs.items():
            if name in self.input_name_to_id:
                self._bind(self.input_name_to_id[name], arr)
            elif len(self.inputs) == 1 and len(kwargs) == 1:
                self._bind(self.inputs[0], arr)
            else:
                self.executor.set_input_by_name(name, np.ascontiguousarray(arr))
        self.executor.run(n_threads if n_threads is not None else self.n_threads)
        ndim = args[0].ndim if args else (next(iter(kwargs.values())).ndim if kwargs else 2)
        return self.get_outputs(input_ndim=ndim)

    def get_outputs(self, input_ndim: int = 2):
        results: dict[Any, np.ndarray] = {}
        for tid in self.outputs:
            t = self.tensor_info.get(tid)
            raw = self.executor.get_output_bytes(tid)
            ne = self.executor.get_tensor_shape(tid)
            dtype = GGML_TYPE_TO_NUMPY.get(t.type if t else 0, np.dtype(np.float32))
            full = [ne[3], ne[2], ne[1], ne[0]]
            rank = max(2, input_ndim)
            arr = np.frombuffer(raw, dtype=dtype)
            try:
                arr = arr.reshape(full[-rank:])
            except ValueError:
                pass
            results[t.name if t else str(tid)] = arr
            results[tid] = arr
        if len(self.outputs) == 1:
            return next(iter(results.values()))
        return results

    def run_benchmark(self, runs: int = 5, n_threads: int | None = None) -> list[float]:
        import time

        lat = []
        for _ in range(runs):
            t0 = time.perf_counter()
            self.executor.run(n_threads or self.n_threads)
            self.executor.synchronize()
            lat.append((time.perf_counter() - t0) * 1000.0)
        return lat

    def set_state(self, state_name_or_id, array: np.ndarray) -> None:
        if isinstance(state_name_or_id, int):
            self.executor.set_state_by_id(state_name_or_id, np.ascontiguousarray(array))
        else:
            self.executor.set_state_by_name(state_name_or_id, np.ascontiguousarray(array))

    def get_state(self, state_name_or_id) -> np.ndarray:
        if isinstance(state_name_or_id, int):
            raw = self.executor.get_state_bytes(state_name_or_id)
            t = self.tensor_info.get(state_name_or_id)
        else:
            raw = self.executor.get_state_bytes_by_name(state_name_or_id)
            t = None
        return np.frombuffer(raw, dtype=GGML_TYPE_TO_NUMPY.get(t.type if t else 0, np.float32))

    def reset_state(self) -> None:
        self.executor.reset_state()

    def init_kv_cache(self, max_ctx: int = 2048) -> None:
        self.executor.init_kv_cache(max_ctx)

    def reset_kv_cache(self) -> None:
        self.executor.reset_kv_cache()

    def has_kv_cache(self) -> bool:
        return bool(self.executor.has_kv_cache())


def load(model_source: str | Path | bytes, n_threads: int = 1, device: str = "cuda") -> ModelRunner:
    """``ggmlc.load`` over the B200 engine (runner.py:319-334)."""
    return ModelRunner(model_source, n_threads=n_threads, device=device)


def greedy_generate(runner: ModelRunner, prompt: list[int], max_new_tokens: int,
                    chunk_size: int = 0, max_ctx: int | None = None) -> list[int]:
    """Token-level twin of GGMLCGenerator.generate (generator.py:123-241) without a tokenizer:
    chunked prefill through the KV cache, then one greedy token per decode step."""
    tokens = list(int(t) for t in prompt)
    runner.init_kv_cache(max_ctx or (len(tokens) + max_new_tokens + 256))
    use_kv = runner.has_kv_cache()
    has_pos = any("pos" in n for n in runner.input_name_to_id) or len(runner.inputs) > 1
    n = len(tokens)
    c = chunk_size if (chunk_size > 0 and use_kv) else n
    last = None
    for c0 in range(0, n, c):
        c1 = min(c0 + c, n)
        ids = np.array([tokens[c0:c1]], dtype=np.int32)
        args = (ids, np.arange(c0, c1, dtype=np.int32).reshape(1, -1)) if has_pos else (ids,)
        out = runner(*args, symbols={"pos": c0, "s": c1 - c0} if use_kv else None)
        last = np.asarray(out).reshape(c1 - c0, -1)[-1]
    out_tokens = []
    if max_new_tokens > 0:
        nxt = int(np.argmax(last))
        out_tokens.append(nxt)
        tokens.append(nxt)
    pos = n
    for _ in range(1, max_new_tokens):
        if use_kv:
            ids = np.array([[tokens[-1]]], dtype=np.int32)
            args = (ids, np.array([[pos]], dtype=np.int32)) if has_pos else (ids,)
            out = runner(*args, symbols={"pos": pos, "s": 1})
            pos += 1
        else:
            ids = np.array([tokens], dtype=np.int32)
            args = (ids, np.arange(len(tokens), dtype=np.int32).reshape(1, -1)) if has_pos else (ids,)
            out = runner(*args)
        logits = np.asarray(out).reshape(-1, np.asarray(out).shape[-1])[-1]
        nxt = int(np.argmax(logits))
        out_tokens.append(nxt)
        tokens.append(nxt)
    return out_tokens
