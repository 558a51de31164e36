"""The synthetic-model builder (ggmlc_b200/synth.py, used by bench.py for the Llama shapes) writes
the same graph the reference compiler writes: a tiny Llama and a tiny GPT-2 synthesized at the
shapes of the reference-compiled fixtures (tests/golden/make_golden.py LLAMA, GPT2) are compared
node by node with them.  Host only: the numpy quantizers build the payload, the C++ loader reads the result."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle as O

# attributes the compiler records for provenance only (no executor reads them)
INFO_ATTRS = {"source_op", "module_path", "fused_pass"}


def _tensor_sig(spec: dict, tid: int) -> tuple:
    t = spec["tensors"][str(tid)]
    return t["type"], json.dumps(t["ne"]), t["storage"], t["role"]


def _synth(tmp_path, quant: str, theta: float, kv8: bool = False):
    from ggmlc_b200 import synth

    if kv8:  # the eight-KV-head fixture (tests/golden/make_golden.py LLAMA_KV8)
        shape = synth.LlamaShape(2, 512, 8, 8, 64, 1024, 512, theta)
    else:
        shape = synth.LlamaShape(2, 256, 4, 2, 64, 512, 512, theta)
    path = tmp_path / f"tiny_{quant}.gguf"
    synth.synth_llama(path, shape, synth.Q8_0 if quant == "q8_0" else synth.Q4_0,
                      name="tiny_llama_kv8" if kv8 else "tiny_llama")
    return path


def _synth_gpt2(tmp_path):
    from ggmlc_b200 import synth

    shape = synth.GPT2Shape(2, 256, 4, 1024, 500, 512)
    path = tmp_path / "tiny_gpt2_q8_0.gguf"
    synth.synth_gpt2(path, shape, synth.Q8_0, name="tiny_gpt2")
    return path


@pytest.mark.parametrize("quant,theta", [("q8_0", 10000.0), ("q4_0", 500000.0), ("gpt2", None),
                                         ("kv8", 500000.0)])
def test_synthesized_graph_matches_reference_compiled(tmp_path, quant, theta):
    if quant == "gpt2":
        path = _synth_gpt2(tmp_path)
        ref_path = GOLDEN / "tiny_gpt2_q8_0.gguf"
    elif quant == "kv8":
        path = _synth(tmp_path, "q4_0", theta, kv8=True)
        ref_path = GOLDEN / "tiny_llama_kv8_q4_0.gguf"
    else:
        path = _synth(tmp_path, quant, theta)
        ref_path = GOLDEN / f"tiny_llama_{quant}.gguf"
    kv, _, data = O.read_gguf(path)
    ref_kv, _, ref_data = O.read_gguf(ref_path)
    assert sorted(kv) == sorted(ref_kv)
    spec = json.loads(kv["ggmlc.graph_spec"])
    ref = json.loads(ref_kv["ggmlc.graph_spec"])
    assert spec["symbol_table"] == ref["symbol_table"]
    assert [n["opcode"] for n in spec["nodes"]] == [n["opcode"] for n in ref["nodes"]]
    for n, r in zip(spec["nodes"], ref["nodes"]):
        assert [_tensor_sig(spec, i) for i in n["inputs"]] == [_tensor_sig(ref, i) for i in r["inputs"]]
        assert [_tensor_sig(spec, i) for i in n["outputs"]] == [_tensor_sig(ref, i) for i in r["outputs"]]
        strip = lambda a: {k: v for k, v in a.items() if k not in INFO_ATTRS}
        assert strip(n["attributes"]) == strip(r["attributes"]), n["opcode"]
    for key in ("inputs", "outputs"):
        assert [_tensor_sig(spec, i) for i in spec[key]] == [_tensor_sig(ref, i) for i in ref[key]]
    # every weight is present with the reference's name, type, shape and byte size; the reference
    # also lists runtime constants (positions, RoPE frequencies) as parameters
    names = {spec["tensors"][str(i)]["name"]: i for i in spec["parameters"]}
    ref_names = {ref["tensors"][str(i)]["name"]: i for i in ref["parameters"]}
    assert set(names) <= set(ref_names)
    for name in set(ref_names) - set(names):
        assert ref["tensors"][str(ref_names[name])]["role"] == "constant", name
    for name, tid in names.items():
        assert _tensor_sig(spec, tid) == _tensor_sig(ref, ref_names[name]), name
        assert data[name].size == ref_data[name].size, name


def test_synthesized_file_loads_and_quantizes_like_the_reference(tmp_path):
    from ggmlc_b200 import _runtime, synth

    path = _synth(tmp_path, "q8_0", 10000.0)
    g = _runtime.ModelLoader.load_from_file(str(path))
    ref = _runtime.ModelLoader.load_from_file(str(GOLDEN / "tiny_llama_q8_0.gguf"))
    assert [op.opcode for op in g.ops] == [op.opcode for op in ref.ops]
    assert g.symbol_table == ref.symbol_table
    # the block quantizers restate the compiler's: an exact round trip of representable values
    x = np.random.default_rng(0).normal(0, 0.02, size=(4, 64)).astype(np.float32)
    q8 = synth.quantize_q8_0_np(x).reshape(-1)
    assert q8.size == 4 * 2 * 34
    q4 = synth.quantize_q4_0_np(x).reshape(-1)
    assert q4.size == 4 * 2 * 18
