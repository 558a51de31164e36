"""Decode chains (k_chain.cu): a single-sequence decode step runs its GEMVs, attention and row
norms as one persistent launch.  Checked against the same engine with chains off, where every op
is its own kernel (launch_dgemv, launch_attn_decode, the row kernels), and against the
reference's golden logits.

- The chain replaces the per-op launches of a decode step (launch count of the prepared step).
- Teacher-forced decode over a prefill and several steps: every logits row within cosine
  0.99999 of the per-kernel engine, identical argmax, and within the model bar of the
  reference's goldens.  The GEMVs of a chain compute exactly what launch_dgemv computes (same
  work split and summation order); attention sums its splits in another order (fp32 online
  softmax), so rows agree to rounding, not bit for bit.
- Graph replay of a chained step is bit-identical to direct launches, and two runs of the same
  step give identical bits (the split merge has a fixed order)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import FIXTURES, GOLDEN, cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

COS_CHAIN = 0.99999  # chain vs per-kernel engine, per row
COS_REF = 0.9998     # against the reference goldens (tests/test_model_gpu.py)


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def _args(r, ids, pos0):
    ids = np.asarray(ids, np.int32).reshape(1, -1)
    if len(r.inputs) > 1:
        return (ids, np.arange(pos0, pos0 + ids.shape[1], dtype=np.int32).reshape(1, -1))
    return (ids,)


def _decode(fixture, chain: bool, graph: bool = True, steps: int | None = None):
    from ggmlc_b200.runner import load

    gold = np.load(GOLDEN / f"{fixture}.npz")
    r = load(str(GOLDEN / f"{fixture}.gguf"), device="cuda")
    r.executor.set_decode_chain(chain)
    assert r.executor.decode_chain() == chain
    r.executor.set_enable_cuda_graph(graph)
    r.init_kv_cache(1024)
    prompt = gold["prompt"]
    r(*_args(r, prompt, 0), symbols={"pos": 0, "s": len(prompt)})
    toks = [int(t) for t in gold["greedy_tokens"]]
    n = len(gold["decode_logits"]) if steps is None else steps
    rows, pos = [], len(prompt)
    for i in range(n):
        o = np.asarray(r(*_args(r, [toks[i]], pos), symbols={"pos": pos, "s": 1})).ravel()
        rows.append(o.copy())
        pos += 1
    launches = r.executor.launches_per_run()
    return np.stack(rows), gold["decode_logits"][:n], launches


@pytest.mark.parametrize("fixture", FIXTURES)
def test_chain_matches_per_kernel_decode(fixture):
    on, ref, n_on = _decode(fixture, True)
    off, _, n_off = _decode(fixture, False)
    assert n_on < n_off, f"the chain did not replace launches ({n_on} vs {n_off})"
    if fixture.startswith("tiny_llama"):
        # llama layers chain whole: embedding lookup, one chain, nothing else
        assert n_on <= 3, f"{n_on} launches per llama decode step"
    for i, (a, b) in enumerate(zip(on, off)):
        assert cos(a, b) >= COS_CHAIN, f"step {i}: chain vs per-kernel cosine {cos(a, b)}"
        assert int(np.argmax(a)) == int(np.argmax(b)), f"step {i}: argmax differs"
        assert cos(a, ref[i]) >= COS_REF, f"step {i}: chain vs reference cosine {cos(a, ref[i])}"


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_chain_graph_replay_bit_identical_and_repeatable(fixture):
    direct, _, _ = _decode(fixture, True, graph=False, steps=6)
    graph, _, _ = _decode(fixture, True, graph=True, steps=6)
    again, _, _ = _decode(fixture, True, graph=True, steps=6)
    assert np.array_equal(direct, graph)
    assert np.array_equal(graph, again)
