"""ggmlc_b200 — B200-native (sm_100a) execution engine for ggmlc-compiled GGUF decoder graphs.

``ggmlc_b200._runtime`` is a drop-in for ggmlc's nanobind ``ggmlc._runtime`` module and
``ggmlc_b200.runner`` mirrors ``ggmlc.runtime.runner`` (``load`` / ``ModelRunner``).  All compute
runs in the CUDA library ``libggmlc_b200.so`` (include/ggmlc_b200.h); there is no CPU fallback.
"""

from __future__ import annotations

__version__ = "0.1.0"


def load(model_source, n_threads: int = 1, device: str = "cuda"):
    """``ggmlc.load(path, device="cuda")`` on the B200 engine."""
    from .runner import load as _load

    return _load(model_source, n_threads=n_threads, device=device)
