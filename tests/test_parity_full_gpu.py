"""Model-level parity at the benchmark configurations ([2], [3]): the engine
against the reference's own CPU runtime (oracle/_ref, ggmlc::ModelExecutor and the ggml CPU
backend compiled from the reference sources) on the SAME seeded GGUF, synthesized at full size:
GPT-2-small Q8_0, SmolLM2-135M Q8_0 and Llama-3-8B Q4_0.

Each case prefills a seeded random prompt through the KV cache and decodes greedily.  Checked:

- greedy tokens: the engine's free-running greedy sequence equals the reference's;
- logits: teacher-forced with the reference's tokens, every row (the prefill's last token and
  each decode step) has cosine >= COS_MIN with the reference's row;
- the reference against itself: the same run at another thread count.  The reference's
  decode attention splits the KV range over its threads once the padded cache holds >= 512
  positions (ggml-cpu/ops.cpp:9179-9209) and rounds each split's V accumulator to fp16, so its
  logits move with the thread count; the Llama-3-8B case uses a 512-token prompt, so its decode
  steps run on that split path.  Both cosines are printed (pytest -s) beside each other.

The bar COS_MIN = 0.9998 (tests/test_model_gpu.py) is below the north star's 0.99999: the
engine's fp32 attention accumulator and its matmul summation order differ from the CPU's, and
the Q8_0 re-quantization in front of every matmul turns last-bit differences into +-1 quant
flips that grow over 12-32 layers.  Integer paths are bit-exact (tests/test_ops_gpu.py).

The GGUFs are synthesized on the GPU box (ggmlc_b200/synth.py, torch on cuda:0) into the bench
directory shared with bench.py; the reference library travels prebuilt in oracle/_ref."""

from __future__ import annotations

import json
import os
import time
from pathlib import Path

import numpy as np
import pytest

from conftest import cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

COS_MIN = 0.9998
BENCH_DIR = Path(os.environ.get("GGMLC_B200_BENCH_DIR", "/tmp/ggmlc_b200_bench"))

# (model, quant, prompt tokens, greedy steps, reference thread count for the self-comparison)
CASES = [
    ("gpt2-small", "q8_0", 128, 16, 4),
    ("smollm2-135m", "q8_0", 512, 16, 4),
    ("llama3-8b", "q4_0", 512, 16, 4),
]


def cos(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def gguf_for(model: str, quant: str) -> Path:
    from ggmlc_b200 import synth

    path = BENCH_DIR / f"{model}_{quant}.gguf"
    if not path.exists():
        BENCH_DIR.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        synth.synth_model(tmp, model, synth.Q4_0 if quant == "q4_0" else synth.Q8_0,
                          device="cuda:0", name=f"{model}_{quant}")
        os.replace(tmp, path)
    return path


def engine_greedy(r, prompt, n_new: int, teacher=None):
    """Prefill + greedy decode through the drop-in runner; same contract as RefRunner.greedy."""
    V = r.executor.get_tensor_shape(r.outputs[0])[0]

    def call(ids, pos):
        ids = np.asarray(ids, np.int32).reshape(1, -1)
        args = (ids,)
        if len(r.inputs) > 1:  # GPT-2 position ids
            args = (ids, np.arange(pos, pos + ids.shape[1], dtype=np.int32).reshape(1, -1))
        out = np.asarray(r(*args, symbols={"pos": pos, "s": ids.shape[1]}), np.float32)
        return out.reshape(-1)[-V:].copy()

    r.reset_kv_cache()
    rows = [call(prompt, 0)]
    toks = [int(np.argmax(rows[0]))]
    pos = len(prompt)
    for i in range(n_new):
        feed = toks[-1] if teacher is None else int(teacher[i])
        rows.append(call([feed], pos))
        toks.append(int(np.argmax(rows[-1])))
        pos += 1
    return toks, np.stack(rows)


@pytest.fixture(scope="module", params=CASES, ids=[c[0] for c in CASES])
def parity_run(request):
    from oracle import refrun

    if not refrun.available():
        pytest.skip("oracle/_ref is not built")
    model, quant, P, G, t_alt = request.param
    from ggmlc_b200 import synth
    from ggmlc_b200.runner import load

    path = gguf_for(model, quant)
    V = synth.SHAPES[model].vocab
    prompt = np.random.default_rng(11).integers(0, V, size=P).astype(np.int32)
    max_ctx = P + G + 256

    t0 = time.time()
    ref = refrun.RefRunner(path, V, max_ctx=max_ctx)
    ref_toks, ref_rows = ref.greedy(prompt, G)
    t_ref = time.time() - t0
    ref.close()
    alt = refrun.RefRunner(path, V, n_threads=t_alt, max_ctx=max_ctx)
    alt_toks, alt_rows = alt.greedy(prompt, G, teacher=ref_toks)
    alt.close()

    r = load(str(path), device="cuda:0")
    r.executor.set_logits_last_only(True)
    r.init_kv_cache(max_ctx)
    own_toks, _ = engine_greedy(r, prompt, G)
    _, tf_rows = engine_greedy(r, prompt, G, teacher=ref_toks)
    del r

    res = {
        "model": model, "quant": quant, "prompt": P, "gen": G,
        "ref_threads": ref.n_threads, "alt_threads": t_alt, "ref_s": round(t_ref, 1),
        "cos_engine_min": min(cos(a, b) for a, b in zip(tf_rows, ref_rows)),
        "cos_engine_all": cos(tf_rows, ref_rows),
        "cos_ref_threads_min": min(cos(a, b) for a, b in zip(alt_rows, ref_rows)),
        "tokens_equal": own_toks == ref_toks,
        "ref_tokens_equal_across_threads": alt_toks == ref_toks,
        "first_token_diff": next((i for i, (a, b) in enumerate(zip(own_toks, ref_toks)) if a != b),
                                 None),
    }
    print("\nparity", json.dumps(res))
    return res, tf_rows, ref_rows, own_toks, ref_toks


def test_logits_cosine_every_row(parity_run):
    res, tf_rows, ref_rows, _, _ = parity_run
    per_row = [cos(a, b) for a, b in zip(tf_rows, ref_rows)]
    assert min(per_row) >= COS_MIN, f"{res['model']}: per-row cosine {per_row}"


def test_greedy_tokens_identical(parity_run):
    res, _, _, own, ref = parity_run
    assert own == ref, f"{res['model']}: engine {own} vs reference {ref}"
