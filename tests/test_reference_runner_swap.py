"""The reference's own ModelRunner (python/ggmlc/runtime/runner.py) over this package's `_runtime`:
`ggmlc._runtime` is bound to `ggmlc_b200._runtime` before the reference module is imported from
its sources, which is the one-line swap a ggmlc user makes.  Host only: the loader is the real
one (the runner reads the graph's names, inputs, outputs, symbol table and tensor types from it),
and the executor is a recorder standing in for `ggmlc_b200._runtime.ModelExecutor` that checks
every call the runner makes binds to the real method's signature, so the runner's whole control
flow (construction, symbol deduction, input binding, run, output reshaping, KV-cache helpers)
executes against this package's interface without a GPU.

The runner's source is read where it lies (the reference checkout); without it the tests skip."""

from __future__ import annotations

import ast
import importlib
import inspect
import os
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN

REF = Path(os.environ.get("GGMLC_REF", "/root/reference"))
RUNNER = REF / "python" / "ggmlc" / "runtime" / "runner.py"

pytestmark = pytest.mark.skipif(not RUNNER.exists(), reason="the reference sources are not here")


def _runtime_calls() -> dict[tuple[str, str], set[int]]:
    """(receiver, method) -> positional argument counts of every call the runner makes on
    `_runtime`, `_runtime.ModelLoader` and `self.executor`."""
    calls: dict[tuple[str, str], set[int]] = {}
    for n in ast.walk(ast.parse(RUNNER.read_text())):
        if not (isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute)):
            continue
        v = n.func.value
        if isinstance(v, ast.Name) and v.id == "_runtime":
            key = ("_runtime", n.func.attr)
        elif isinstance(v, ast.Attribute) and isinstance(v.value, ast.Name):
            if v.value.id == "_runtime":
                key = (v.attr, n.func.attr)
            elif v.value.id == "self" and v.attr == "executor":
                key = ("ModelExecutor", n.func.attr)
            else:
                continue
        else:
            continue
        calls.setdefault(key, set()).add(len(n.args))
    return calls


def test_every_runtime_call_of_the_runner_binds_to_this_package():
    from ggmlc_b200 import _runtime as ours

    calls = _runtime_calls()
    assert ("ModelExecutor", "run") in calls and ("ModelLoader", "load_from_file") in calls
    for (recv, meth), nargs in sorted(calls.items()):
        owner = ours if recv == "_runtime" else getattr(ours, recv)
        fn = getattr(owner, meth, None)
        assert fn is not None, f"{recv}.{meth} is missing"
        sig = inspect.signature(fn)
        for k in nargs:
            args = [object()] * k
            if recv == "ModelExecutor":  # an instance method: self is bound first
                sig.bind(object(), *args)
            else:
                sig.bind(*args)


class _Recorder:
    """Stands in for ggmlc_b200._runtime.ModelExecutor: every attribute the runner uses must exist
    on the real class and every call must bind to its signature; outputs are zero logits of the
    fixture's shape."""

    real = None
    vocab = 0

    def __init__(self, graph, device="cpu"):
        inspect.signature(self.real.__init__).bind(self, graph, device)
        self.graph = graph
        self.device = device
        self.log: list[tuple] = []
        self.env: dict[str, int] = {}
        self.kv = False

    def __getattr__(self, name):
        fn = getattr(self.real, name)  # AttributeError for anything the real class lacks
        sig = inspect.signature(fn)

        def call(*args, **kwargs):
            sig.bind(self, *args, **kwargs)
            self.log.append((name, args))
            if name == "prepare":
                self.env = dict(args[0])
            if name == "init_kv_cache":
                self.kv = True
            if name == "has_kv_cache":
                return self.kv
            s = int(self.env.get("s", 1))
            if name == "get_tensor_shape":
                return [self.vocab, s, 1, 1]
            if name == "get_output_bytes":
                return np.zeros(self.vocab * s, np.float32).tobytes()
            return None

        return call


def test_reference_runner_drives_this_runtime(monkeypatch):
    from ggmlc_b200 import _runtime as ours

    monkeypatch.syspath_prepend(str(REF / "python"))
    monkeypatch.setitem(sys.modules, "ggmlc._runtime", ours)
    monkeypatch.delitem(sys.modules, "ggmlc.runtime.runner", raising=False)
    runner = importlib.import_module("ggmlc.runtime.runner")
    assert runner._RUNTIME_AVAILABLE and runner._runtime is ours

    fixture = "tiny_llama_q8_0"
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    rec = type("Rec", (_Recorder,), {"real": ours.ModelExecutor, "vocab": vocab})
    monkeypatch.setattr(ours, "ModelExecutor", rec)

    r = runner.load(str(GOLDEN / f"{fixture}.gguf"), device="cuda")
    g = ours.ModelLoader.load_from_file(str(GOLDEN / f"{fixture}.gguf"))
    assert r.name == g.name and r.inputs == list(g.inputs) and r.outputs == list(g.outputs)
    assert r.symbol_table == list(g.symbol_table) and r.device == "cuda"
    (in_name,) = [g.tensors[t].name for t in g.inputs]
    assert r.input_name_to_id == {in_name: g.inputs[0]}

    # the generate loop's calls (python/ggmlc/runtime/generator.py:149-220): a KV cache, a
    # prompt with its symbols, then one-token steps
    r.init_kv_cache(64)
    assert r.has_kv_cache()
    prompt = np.arange(1, 8, dtype=np.int64)[None, :]
    out = r(prompt, symbols={"pos": 0, "s": 7})
    # a file-loaded graph has no Python-side ranks: the runner keeps the input's rank (2)
    assert out.shape == (7, vocab) and out.dtype == np.float32
    step = r(np.array([[5]], np.int64), symbols={"pos": 7, "s": 1})
    assert step.shape == (1, vocab)
    r.reset_kv_cache()
    lat = r.run_benchmark(runs=2)
    assert len(lat) == 2

    ex = r.executor
    names = [c[0] for c in ex.log]
    assert names[:2] == ["init_kv_cache", "has_kv_cache"]
    prep = [c[1] for c in ex.log if c[0] == "prepare"]
    # the runner deduced the graph's own sequence symbol from the input shape
    (sym,) = g.symbol_table
    assert prep[0][0] == {"pos": 0, "s": 7, sym: 7} and prep[1][0] == {"pos": 7, "s": 1, sym: 1}
    fed = [c[1] for c in ex.log if c[0] == "set_input_by_id"]
    assert fed[0][0] == g.inputs[0] and fed[0][1].dtype == np.int32  # int64 ids narrowed for I32
    assert names.count("run") == 4 and names.count("get_output_bytes") == 2
