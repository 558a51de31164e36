"""The CPU oracle (oracle/oracle.c) against golden vectors written by the reference itself
(tests/golden/make_golden.py through oracle/_ref).  Every comparison here is bit-exact: the
oracle restates the reference's x86 AVX2 arithmetic order, including the FMA contractions of
its GNU build."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import FIXTURES, GOLDEN
from oracle import oracle as O


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "ops_golden.npz")


def test_fp16_roundtrip_rne():
    L = O.lib()
    vals = np.array([0.0, -0.0, 1.0, 65504.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 0.333333,
                     -7.123456, 3.0e-5, 6.1e-5], np.float32)
    for v in vals:
        h = L.oracle_fp32_to_fp16(float(v))
        with np.errstate(over="ignore"):  # 65520 rounds to +inf on purpose
            ref = np.array([v]).astype(np.float16).view(np.uint16)[0]
        assert h == ref, v
    for h in range(0, 65536, 7):
        if (h & 0x7C00) == 0x7C00:
            continue
        f = L.oracle_fp16_to_fp32(h)
        assert np.float32(f) == np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]


def test_quantize_q8_0_matches_reference_incl_ties(g):
    assert np.array_equal(O.quantize_q8_0(g["quant_x"]), g["quant_q8_0"])


def test_quantize_ref_variant_differs_on_ties(g):
    """The scalar reference quantizer rounds half away from zero; the AVX2 build (the one the
    oracle follows) rounds half to even — the tie row shows the difference."""
    x = np.ascontiguousarray(g["quant_x"][-2:-1])
    a = O.quantize_q8_0(x)
    b = np.empty_like(a)
    O.lib().oracle_quantize_row_q8_0_ref(O._p(x), O._p(b), x.size)
    assert not np.array_equal(a, b)


@pytest.mark.parametrize("name,t", [("q8_0", O.Q8_0), ("q4_0", O.Q4_0)])
def test_dequant_and_dots_bit_exact(g, name, t):
    w = g[f"w_{name}"]
    K = 256
    assert np.array_equal(O.dequantize(t, w, K), g[f"deq_{name}"])
    q = g["quant_q8_0"]
    dots = np.array([[O.lib().oracle_vec_dot(t, K, O._p(np.ascontiguousarray(w[n])),
                                              O._p(np.ascontiguousarray(q[m])))
                      for m in range(q.shape[0])] for n in range(w.shape[0])], np.float32)
    assert np.array_equal(dots, g[f"dot_{name}"])


@pytest.mark.parametrize("name,t", [("q8_0", O.Q8_0), ("q4_0", O.Q4_0)])
def test_mul_mat_bit_exact(g, name, t):
    w = g[f"w_{name}"]
    y = O.mul_mat(t, w, w.shape[0], 256, g[f"mm_x_{name}"])
    assert np.array_equal(y, g[f"mm_y_{name}"])


def test_rms_norm_bit_exact(g):
    assert np.array_equal(O.rms_norm(g["rms_x"], 1e-5), g["rms_y"])
    assert np.array_equal(O.rms_norm(g["rms_x"], 1e-5, g["rms_gamma"]), g["rms_y_gamma"])


@pytest.mark.parametrize("tag,base", [("1e4", 10000.0009765625), ("5e5", 500000.0)])
def test_rope_bit_exact(g, tag, base):
    y = O.rope_neox(g["rope_x"], g["rope_pos"], 64, np.float32(base))
    assert np.array_equal(y, g[f"rope_y_{tag}"])


def test_swiglu_bit_exact(g):
    assert np.array_equal(O.swiglu(g["swiglu_x"]), g["swiglu_y"])


def test_flash_attn_bit_exact(g):
    y = O.flash_attn(g["fa_q"], g["fa_k"].view(np.uint16), g["fa_v"].view(np.uint16),
                     g["fa_mask"].view(np.uint16), np.float32(1.0) / np.sqrt(np.float32(64)))
    assert np.array_equal(y, g["fa_y"])


@pytest.mark.parametrize("fixture", FIXTURES + ["tiny_llama_kv8_q4_0"])
def test_model_forward_bit_exact(fixture):
    gold = np.load(GOLDEN / f"{fixture}.npz")
    M = O.ModelOracle(GOLDEN / f"{fixture}.gguf")
    V = gold["full_logits"].shape[1]
    y = M.forward(gold["prompt"]).reshape(-1, V)
    assert np.array_equal(y, gold["full_logits"])


@pytest.mark.parametrize("fixture", FIXTURES + ["tiny_llama_kv8_q4_0"])
def test_model_kv_decode_bit_exact(fixture):
    gold = np.load(GOLDEN / f"{fixture}.npz")
    M = O.ModelOracle(GOLDEN / f"{fixture}.gguf")
    V = gold["full_logits"].shape[1]
    assert M.init_kv_cache(1024)
    y = M.forward(gold["prompt"], pos=0).reshape(-1, V)
    assert np.array_equal(y, gold["kv_prefill_logits"])
    toks = [int(np.argmax(y[-1]))]
    pos = len(gold["prompt"])
    for i in range(len(gold["decode_logits"])):
        y = M.forward(np.array([toks[-1]]), pos=pos).reshape(-1)
        assert np.array_equal(y, gold["decode_logits"][i]), f"decode step {i}"
        toks.append(int(np.argmax(y)))
        pos += 1
    assert toks == list(gold["greedy_tokens"])


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_batch_goldens_pinned_by_oracle(fixture):
    """The per-sequence goldens of the batched-decode test (written by the reference build) are
    reproduced bit for bit by the oracle's own KV decode, for the first two sequences (the rest
    run the same code path); every golden token is the argmax of its logits row."""
    gold = np.load(GOLDEN / f"{fixture}_batch.npz")
    lengths = [int(n) for n in gold["lengths"]]
    offs = np.concatenate([[0], np.cumsum(lengths)])
    V = gold["logits"].shape[2]
    assert np.array_equal(np.argmax(gold["logits"], axis=2), gold["tokens"])
    for k in range(2):
        M = O.ModelOracle(GOLDEN / f"{fixture}.gguf")
        assert M.init_kv_cache(1024)
        prompt = gold["prompts"][offs[k]:offs[k + 1]]
        y = M.forward(prompt, pos=0).reshape(-1, V)
        assert np.array_equal(y[-1], gold["logits"][k][0])
        for i in range(gold["tokens"].shape[1] - 1):
            y = M.forward(np.array([gold["tokens"][k][i]]), pos=lengths[k] + i).reshape(-1)
            assert np.array_equal(y, gold["logits"][k][i + 1]), f"sequence {k} step {i}"
