"""Model-level parity on the GPU through the drop-in runner (ggmlc_b200.runner.load ->
ggmlc_b200._runtime -> libggmlc_b200.so) against the reference's own golden outputs
(tests/golden/*.npz, written by oracle/_ref) on the committed fixtures.

Bars.  The north star asks for logits cosine >= 0.99999 and identical greedy tokens.  Integer
work is bit-exact against the reference (tests/test_ops_gpu.py); fp32 sums run in another order
than the CPU's SIMD lanes, attention accumulates in fp32 where the CPU kernel rounds its V
accumulator to fp16 after every position (ggml-cpu/ops.cpp:8689-8696), and the Q8_0
re-quantization in front of each matmul turns those last-bit differences into occasional +-1
quant flips.  The reference itself moves by the same amount between its own thread counts
(decode logits cosine 0.99989 between 1 and 4 threads on these fixtures, split-KV path
ops.cpp:9179-9209).  The bar is therefore cosine >= 0.9998 per logits row set, and identical
greedy tokens (argmax) at every prefill position and decode step whose reference top-2 gap
exceeds 1% of that row's logit range: random-weight fixtures have near-ties that the reference
also flips between thread counts.  Decode is teacher-forced with the reference's tokens.
CUDA-graph replay must be bit-identical to direct launches."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import FIXTURES, GOLDEN, cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


COS_MIN = 0.9998


def argmax_agrees(out, ref, rel_gap=0.01):
    """argmax equal wherever the reference's top-2 gap is above rel_gap of the row range."""
    out = np.asarray(out).reshape(ref.shape)
    srt = np.sort(ref, axis=1)
    gap = srt[:, -1] - srt[:, -2]
    clear = gap > rel_gap * (srt[:, -1] - srt[:, 0])
    same = np.argmax(out, 1) == np.argmax(ref, 1)
    return bool(np.all(same[clear])), int(np.sum(~same)), int(np.sum(clear))


def _runner(fixture):
    from ggmlc_b200.runner import load

    return load(str(GOLDEN / f"{fixture}.gguf"), device="cuda")


def _args(r, ids, pos0):
    ids = np.asarray(ids, np.int32).reshape(1, -1)
    if len(r.inputs) > 1:
        return (ids, np.arange(pos0, pos0 + ids.shape[1], dtype=np.int32).reshape(1, -1))
    return (ids,)


@pytest.mark.parametrize("fixture", FIXTURES)
def test_full_forward_matches_reference(fixture):
    gold = np.load(GOLDEN / f"{fixture}.npz")
    r = _runner(fixture)
    V = gold["full_logits"].shape[1]
    out = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1, V)
    ref = gold["full_logits"]
    assert out.shape == ref.shape
    assert cos(out, ref) >= COS_MIN
    ok, n_diff, n_clear = argmax_agrees(out, ref)
    assert ok, f"{n_diff} argmax differences among {n_clear} clear positions"


@pytest.mark.parametrize("fixture", FIXTURES)
def test_kv_prefill_then_greedy_decode_matches_reference(fixture):
    gold = np.load(GOLDEN / f"{fixture}.npz")
    r = _runner(fixture)
    V = gold["full_logits"].shape[1]
    r.init_kv_cache(1024)
    assert r.has_kv_cache()
    prompt = gold["prompt"]
    out = np.asarray(r(*_args(r, prompt, 0), symbols={"pos": 0, "s": len(prompt)})).reshape(-1, V)
    assert cos(out, gold["kv_prefill_logits"]) >= COS_MIN
    # teacher-forced: each step is fed the reference's greedy token, so one near-tie cannot
    # derail the comparison of every later step
    ref_toks = [int(t) for t in gold["greedy_tokens"]]
    toks = [int(np.argmax(out[-1]))]
    pos = len(prompt)
    logits = [out[-1]]
    for i, ref in enumerate(gold["decode_logits"]):
        o = np.asarray(r(*_args(r, [ref_toks[i]], pos), symbols={"pos": pos, "s": 1})).reshape(-1)
        assert cos(o, ref) >= COS_MIN, f"decode step {i}: cos {cos(o, ref)}"
        toks.append(int(np.argmax(o)))
        logits.append(o)
        pos += 1
    refs = np.stack([gold["kv_prefill_logits"].reshape(-1, V)[-1]] + list(gold["decode_logits"]))
    ok, n_diff, n_clear = argmax_agrees(np.stack(logits), refs)
    assert ok, f"{n_diff} greedy-token differences at clear (non-tie) steps"


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_cuda_graph_replay_bit_identical(fixture):
    gold = np.load(GOLDEN / f"{fixture}.npz")
    prompt = gold["prompt"][:12]
    outs = []
    for graph in (False, True):
        r = _runner(fixture)
        r.executor.set_enable_cuda_graph(graph)
        r.init_kv_cache(512)
        r(*_args(r, prompt, 0), symbols={"pos": 0, "s": len(prompt)})
        seq = []
        tok, pos = 7, len(prompt)
        for _ in range(6):
            o = np.asarray(r(*_args(r, [tok], pos), symbols={"pos": pos, "s": 1})).ravel()
            seq.append(o.copy())
            tok, pos = int(np.argmax(o)), pos + 1
        if graph:
            assert r.executor.is_cuda_graph_captured()
        outs.append(np.stack(seq))
    assert np.array_equal(outs[0], outs[1])


def test_logits_last_only_matches_last_row():
    gold = np.load(GOLDEN / "tiny_llama_q8_0.npz")
    r = _runner("tiny_llama_q8_0")
    r.executor.set_logits_last_only(True)
    assert r.executor.logits_last_only()
    V = gold["full_logits"].shape[1]
    out = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1)
    assert out.size == V
    assert cos(out, gold["full_logits"][-1]) >= COS_MIN


def test_greedy_generate_chunked_prefill_matches_reference():
    """Chunked prefill (chunks of 16 through the KV cache) + greedy decode, the generator loop
    of python/ggmlc/runtime/generator.py:161-241."""
    from ggmlc_b200.runner import greedy_generate

    gold = np.load(GOLDEN / "tiny_llama_q4_0.npz")
    r = _runner("tiny_llama_q4_0")
    toks = greedy_generate(r, list(gold["prompt"]), max_new_tokens=len(gold["greedy_tokens"]),
                           chunk_size=16, max_ctx=1024)
    assert toks == [int(t) for t in gold["greedy_tokens"]]


def test_errors_are_raised_not_crashing():
    r = _runner("tiny_llama_q8_0")
    r.init_kv_cache(64)
    with pytest.raises(RuntimeError, match="KV cache overflow"):
        r.executor.prepare({"pos": 60, "s": 10, "s70": 10})
    r.executor.prepare({"s": 4, "s70": 4})
    with pytest.raises(RuntimeError, match="size mismatch"):
        r.executor.set_input_by_id(r.inputs[0], np.zeros(3, np.int32))


@pytest.mark.parametrize("fixture", FIXTURES)
def test_output_rows_select_prompt_logits(fixture):
    """Output rows (the per-request output indices of the reference's doc gap 3; llama's
    out_ids): a full prompt forward restricted to chosen rows returns exactly those rows of the
    reference's logits (cosine and argmax bar), in the order asked; the last row alone is
    bit-identical to the last-row mode, and clearing the rows restores full logits."""
    gold = np.load(GOLDEN / f"{fixture}.npz")
    ref = gold["full_logits"]
    n, V = ref.shape
    r = _runner(fixture)
    rows = [n - 1, 0, n // 2, 3]
    r.executor.set_output_rows(rows)
    out = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1, V)
    assert out.shape == (len(rows), V)
    assert cos(out, ref[rows]) >= COS_MIN
    ok, n_diff, n_clear = argmax_agrees(out, ref[rows])
    assert ok, f"{n_diff} argmax differences among {n_clear} clear rows"
    r.executor.set_output_rows([n - 1])
    one = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1)
    r.executor.set_output_rows(None)
    r.executor.set_logits_last_only(True)
    last = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1)
    assert np.array_equal(one, last)
    r.executor.set_logits_last_only(False)
    full = np.asarray(r(*_args(r, gold["prompt"], 0))).reshape(-1, V)
    assert full.shape == ref.shape
    with pytest.raises(RuntimeError, match="not among"):
        r.executor.set_output_rows([n])
        r(*_args(r, gold["prompt"], 0))


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_gpt2_q8_0"])
def test_queued_steps_read_their_own_positions(fixture):
    """Steps enqueued back to back, with no host sync between them (a prefill, 40 decode steps,
    a second prefill, 40 more), each read the step parameters (position) their own prepare set,
    though the host runs ahead of the device and rewrites them for later steps: the final
    logits equal those of the same steps with a sync after each one, bit for bit."""
    from ggmlc_b200 import _runtime as R

    def run(sync_each: bool):
        g = R.ModelLoader.load_from_file(str(GOLDEN / f"{fixture}.gguf"))
        ex = R.ModelExecutor(g, "cuda")
        ex.init_kv_cache(256)
        ex.set_logits_last_only(True)
        ex.set_enable_cuda_graph(True)
        prompt = np.arange(1, 17, dtype=np.int32)

        def step(toks, pos):
            toks = np.asarray(toks, np.int32)
            ex.prepare({"s": len(toks), "pos": pos, **{s: len(toks) for s in g.symbol_table}})
            ex.set_input_by_id(g.inputs[0], toks)
            if len(g.inputs) > 1:
                ex.set_input_by_id(g.inputs[1], np.arange(pos, pos + len(toks), dtype=np.int32))
            ex.run()
            if sync_each:
                ex.synchronize()

        for seed in (3, 1):
            step(prompt, 0)
            for i in range(40):
                step([(7 * i + seed) % 200], len(prompt) + i)
        ex.synchronize()
        return ex.get_output_array(g.outputs[0]).reshape(-1).copy()

    assert np.array_equal(run(True), run(False))


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_gpt2_q8_0"])
def test_output_argmax_on_device_matches_host(fixture):
    """output_argmax (the greedy token of each row computed on the device, first maximum) equals
    numpy's argmax of the copied logits, for a prefill's rows and for decode steps."""
    from ggmlc_b200 import _runtime as R

    g = R.ModelLoader.load_from_file(str(GOLDEN / f"{fixture}.gguf"))
    ex = R.ModelExecutor(g, "cuda")
    ex.init_kv_cache(256)
    gold = np.load(GOLDEN / f"{fixture}.npz")
    prompt = gold["prompt"][:12]

    def step(toks, pos):
        toks = np.asarray(toks, np.int32)
        ex.prepare({"s": len(toks), "pos": pos, **{s: len(toks) for s in g.symbol_table}})
        ex.set_input_by_id(g.inputs[0], toks)
        if len(g.inputs) > 1:
            ex.set_input_by_id(g.inputs[1], np.arange(pos, pos + len(toks), dtype=np.int32))
        ex.run()

    step(prompt, 0)
    lg = ex.get_output_array(g.outputs[0]).reshape(len(prompt), -1)
    assert np.array_equal(ex.output_argmax(g.outputs[0], len(prompt)), np.argmax(lg, axis=1))
    tok, pos = int(np.argmax(lg[-1])), len(prompt)
    for _ in range(4):
        step([tok], pos)
        t_dev = int(ex.output_argmax(g.outputs[0])[0])
        t_host = int(np.argmax(ex.get_output_array(g.outputs[0])))
        assert t_dev == t_host
        tok, pos = t_dev, pos + 1
