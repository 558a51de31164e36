"""CPU ORACLE — test infrastructure, not product code.

Drives the reference's own CPU runtime (``oracle/_ref/libggmlc_ref.so``: the vendored ggml CPU
backend and ``ggmlc::ModelExecutor`` compiled from the reference sources by ``oracle/Makefile``)
on a whole GGUF model: prefill through the KV cache, then greedy decode, the loop of
``python/ggmlc/runtime/generator.py:161-241`` over ``ModelExecutor::prepare/set_input/run``
(``runtime/src/executor.cpp:1453``, ``:2984``).  Only ``tests/`` and ``bench.py``'s parity and
reference legs use it, as the checker.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# "avx2": the default build (-march=x86-64-v3), the checker; "native": the same sources built as
# the reference's default cmake build does on the benchmark hosts (oracle/Makefile `native`)
REF_LIBS = {"avx2": HERE / "_ref" / "libggmlc_ref.so",
            "native": HERE / "_ref" / "native" / "libggmlc_ref.so"}
REF_LIB = REF_LIBS["avx2"]

_libs: dict[str, ctypes.CDLL] = {}


def available(build: str = "avx2") -> bool:
    return REF_LIBS[build].exists()


def lib(build: str = "avx2") -> ctypes.CDLL:
    if build not in _libs:
        path = REF_LIBS[build]
        if not path.exists():
            raise RuntimeError(f"{path} is not built (make -C oracle, needs the reference sources)")
        # RTLD_LOCAL (the default): the two builds export the same symbols and stay apart
        L = ctypes.CDLL(str(path))
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.ref_model_open.argtypes = [ctypes.c_char_p, I]
        L.ref_model_open.restype = P
        L.ref_model_close.argtypes = [P]
        L.ref_model_init_kv.argtypes = [P, I64]
        L.ref_model_reset_kv.argtypes = [P]
        L.ref_model_set_logits_last_only.argtypes = [P, I]
        L.ref_model_forward.argtypes = [P, P, I64, I64, P, I64]
        L.ref_model_forward.restype = I64
        L.ref_last_error.restype = ctypes.c_char_p
        _libs[build] = L
    return _libs[build]


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


class RefRunner:
    """One reference CPU executor over a GGUF, with its padded KV cache."""

    def __init__(self, gguf: str | Path, vocab: int, n_threads: int | None = None,
                 max_ctx: int = 2048, build: str = "avx2"):
        self.L = lib(build)
        self.V = vocab
        self.n_threads = n_threads or host_threads()
        self.h = self.L.ref_model_open(str(gguf).encode(), self.n_threads)
        if not self.h:
            raise RuntimeError(self.L.ref_last_error().decode())
        if self.L.ref_model_init_kv(self.h, max_ctx) != 1:
            raise RuntimeError(f"reference KV cache: {self.L.ref_last_error().decode()}")
        # llama n_outputs = 1: the last token's logits only, as ggmlc-bench runs it
        self.L.ref_model_set_logits_last_only(self.h, 1)
        self.out = np.empty(self.V, np.float32)

    def close(self):
        if self.h:
            self.L.ref_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, tokens, pos: int) -> np.ndarray:
        """Last-token logits of tokens[] fed at positions pos.."""
        t = np.ascontiguousarray(tokens, np.int32)
        n = self.L.ref_model_forward(self.h, t.ctypes.data_as(ctypes.c_void_p), t.size, pos,
                                     self.out.ctypes.data_as(ctypes.c_void_p), self.out.size)
        if n != self.V:
            raise RuntimeError(f"reference forward returned {n}: {self.L.ref_last_error().decode()}")
        return self.out.copy()

    def greedy(self, prompt, n_new: int, teacher=None) -> tuple[list[int], np.ndarray]:
        """Prefill prompt, then n_new greedy steps.  Returns (tokens, logits[n_new + 1, V]):
        row 0 the prefill's last-token logits, row i the logits of decode step i.  With
        `teacher` (a token list), step i is fed teacher[i] instead of this run's own argmax."""
        self.L.ref_model_reset_kv(self.h)
        rows = [self.forward(prompt, 0)]
        toks = [int(np.argmax(rows[0]))]
        pos = len(prompt)
        for i in range(n_new):
            feed = toks[-1] if teacher is None else int(teacher[i])
            rows.append(self.forward([feed], pos))
            toks.append(int(np.argmax(rows[-1])))
            pos += 1
        return toks, np.stack(rows)
