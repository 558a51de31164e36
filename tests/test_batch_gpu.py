"""Continuous batching over the paged KV cache (the reference's ContinuousBatchScheduler,
runtime/src/batch_scheduler.cpp:130-403, and its e2e test tests/e2e/test_continuous_batching.py).

Every sequence in a batched step decodes at its own position in its own slot.  Steps of up to 2
rows run the decode GEMV, whose per-row arithmetic does not depend on the row count, so with at
most 2 slots a request's tokens equal the same prompt decoded alone.  3-16 rows run the
tensor-core decode kernel (its rows are batch-invariant among themselves but summed in another
order than the GEMV's): those requests are checked teacher-forced against single-sequence decode,
token by token wherever the single-sequence top-2 gap exceeds 1% of the logit range."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, cuda_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

MAX_CTX = 256


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def _executor(fixture):
    from ggmlc_b200 import _runtime as R

    g = R.ModelLoader.load_from_file(str(GOLDEN / f"{fixture}.gguf"))
    return g, R.ModelExecutor(g, "cuda")


def _single(fixture, prompt, n_new):
    """Greedy tokens and per-step logits of one sequence decoded alone (paged slot 0)."""
    g, ex = _executor(fixture)
    ex.init_paged_kv_cache(1, MAX_CTX)
    ex.set_logits_last_only(True)
    ex.paged_kv_alloc_slot(0)
    ex.paged_kv_ensure_tokens(0, len(prompt) + n_new)
    sym = g.symbol_table
    in_id, out_id = g.inputs[0], g.outputs[0]
    env = {"s": len(prompt), "pos": 0, "slot": 0, **{s: len(prompt) for s in sym}}
    ex.prepare(env)
    ex.set_input_by_id(in_id, np.asarray(prompt, np.int32))
    ex.run()
    lg = [ex.get_output_array(out_id).reshape(-1)]
    toks = [int(np.argmax(lg[-1]))]
    pos = len(prompt)
    while len(toks) < n_new:
        ex.prepare_batch(np.array([pos], np.int32), np.array([0], np.int32))
        ex.set_input_by_id(in_id, np.array([toks[-1]], np.int32))
        ex.run()
        lg.append(ex.get_output_array(out_id).reshape(-1))
        toks.append(int(np.argmax(lg[-1])))
        pos += 1
    return toks, lg


def _forced(fixture, prompt, toks):
    """Logits of one sequence decoded alone, fed the given tokens (teacher forcing)."""
    g, ex = _executor(fixture)
    ex.init_paged_kv_cache(1, MAX_CTX)
    ex.set_logits_last_only(True)
    ex.paged_kv_alloc_slot(0)
    ex.paged_kv_ensure_tokens(0, len(prompt) + len(toks))
    in_id, out_id = g.inputs[0], g.outputs[0]
    ex.prepare({"s": len(prompt), "pos": 0, "slot": 0, **{s: len(prompt) for s in g.symbol_table}})
    ex.set_input_by_id(in_id, np.asarray(prompt, np.int32))
    ex.run()
    lg = [ex.get_output_array(out_id).reshape(-1)]
    pos = len(prompt)
    for t in toks[:-1]:
        ex.prepare_batch(np.array([pos], np.int32), np.array([0], np.int32))
        ex.set_input_by_id(in_id, np.array([t], np.int32))
        ex.run()
        lg.append(ex.get_output_array(out_id).reshape(-1))
        pos += 1
    return np.stack(lg)


def _prompts(rng, lengths, vocab):
    return [rng.integers(1, vocab, size=n).astype(np.int32) for n in lengths]


def _serve(fixture, prompts, n_new, max_batch):
    from ggmlc_b200 import _runtime as R

    g, ex = _executor(fixture)
    sched = R.ContinuousBatchScheduler(ex, max_batch_size=max_batch, eos_token_id=-1)
    ex.init_paged_kv_cache(max_batch, MAX_CTX)  # same cache length as the single-sequence runs
    ids = [sched.add_request(p, max_new_tokens=n_new, temperature=0.0) for p in prompts]
    assert sched.pending_count() == len(prompts)
    streamed = {i: [] for i in ids}
    steps = 0
    peak_active = 0
    while sched.has_work():
        res = sched.step()
        for rid, tok in res.new_tokens:
            streamed[rid].append(tok)
        peak_active = max(peak_active, sched.active_count())
        steps += 1
        assert steps < 500
    assert peak_active == max_batch  # the slots were shared, more requests than slots
    assert ex.get_paged_active_vram_bytes() == 0  # every slot returned
    out = []
    for rid in ids:
        req = sched.get_request(rid)
        assert req.finished and req.finish_reason == "length"
        assert req.generated_tokens == streamed[rid]
        out.append(req.generated_tokens)
    return out


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_scheduler_tokens_match_single_sequence_decode(fixture):
    rng = np.random.default_rng(11)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    prompts = _prompts(rng, [5, 17, 33, 9, 40, 3], vocab)
    for p, toks in zip(prompts, _serve(fixture, prompts, 10, 2)):
        ref, _ = _single(fixture, p, 10)
        assert toks == ref, f"prompt {len(p)}"


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_scheduler_batches_of_4_to_8_follow_single_sequence_decode(fixture):
    rng = np.random.default_rng(12)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    prompts = _prompts(rng, [5, 17, 33, 9, 40, 3, 21, 12, 7, 30], vocab)
    n_clear = 0
    for p, toks in zip(prompts, _serve(fixture, prompts, 10, 8)):
        lg = _forced(fixture, p, toks)
        srt = np.sort(lg, axis=1)
        clear = (srt[:, -1] - srt[:, -2]) > 0.01 * (srt[:, -1] - srt[:, 0])
        same = np.argmax(lg, axis=1) == np.asarray(toks)
        assert np.all(same[clear]), f"prompt {len(p)}: {np.flatnonzero(~same)}"
        n_clear += int(clear.sum())
    assert n_clear >= 50


def test_batched_step_of_16_matches_single_sequences():
    fixture = "tiny_llama_q8_0"
    rng = np.random.default_rng(5)
    g, ex = _executor(fixture)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    lengths = list(rng.integers(3, 60, size=16))
    prompts = _prompts(rng, lengths, vocab)
    ex.init_paged_kv_cache(16, MAX_CTX)
    ex.set_logits_last_only(True)
    sym = g.symbol_table
    in_id, out_id = g.inputs[0], g.outputs[0]
    first = []
    for slot, p in enumerate(prompts):
        ex.paged_kv_alloc_slot(slot)
        ex.paged_kv_ensure_tokens(slot, len(p) + 1)
        ex.prepare({"s": len(p), "pos": 0, "slot": slot, **{s: len(p) for s in sym}})
        ex.set_input_by_id(in_id, p)
        ex.run()
        first.append(int(np.argmax(ex.get_output_array(out_id))))
    assert ex.get_paged_active_vram_bytes() > 0
    pos = np.array([len(p) for p in prompts], np.int32)
    ex.prepare_batch(pos, np.arange(16, dtype=np.int32))
    ex.set_input_by_id(in_id, np.array(first, np.int32))
    ex.run()
    out = ex.get_output_array(out_id).reshape(16, -1)
    for r, p in enumerate(prompts):
        _, lg = _single(fixture, p, 2)
        assert cos(out[r], lg[1]) >= 0.9999, f"row {r}"
    for slot in range(16):
        ex.paged_kv_free_slot(slot)
    assert ex.get_paged_active_vram_bytes() == 0


def test_scheduler_rejects_bad_requests():
    from ggmlc_b200 import _runtime as R

    g, ex = _executor("tiny_llama_q8_0")
    sched = R.ContinuousBatchScheduler(ex, max_batch_size=2, eos_token_id=0)
    with pytest.raises(RuntimeError):
        sched.add_request([], max_new_tokens=4)
    with pytest.raises(RuntimeError):
        sched.add_request([1, 2, 3], max_new_tokens=4096)  # beyond the 2048-position cache
    with pytest.raises(RuntimeError):
        ex.prepare_batch(np.array([0], np.int32), np.array([7], np.int32))  # no such slot


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_prefix_caching_reuses_prompt_pages(fixture):
    """The reference's prefix-caching e2e flow (tests/e2e/test_prefix_caching.py:76-142) on the
    tiny models with 16-token pages: a cold request indexes its two whole prompt pages, three
    requests sharing them are admitted in one step with 32 prompt tokens matched each, a prompt
    that is cached whole re-evaluates only its last token; every request finishes, the slots are
    returned, and the tokens follow single-sequence decode wherever its top-2 gap is clear."""
    from ggmlc_b200 import _runtime as R

    rng = np.random.default_rng(21)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    g, ex = _executor(fixture)
    ex.set_tokens_per_page(16)
    ex.configure_vmm_pool(max_warm_pages=8)
    sched = R.ContinuousBatchScheduler(ex, max_batch_size=4, eos_token_id=-1)
    ex.init_paged_kv_cache(4, MAX_CTX)  # same cache length as the single-sequence runs
    assert sched.is_prefix_caching_enabled()
    shared = list(rng.integers(1, vocab, size=32))
    tails = [list(rng.integers(1, vocab, size=3)) for _ in range(4)]
    prompts = [shared + t for t in tails]
    n_new = 6
    ids = [sched.add_request(prompts[0], max_new_tokens=n_new, temperature=0.0)]
    sched.step()
    assert sched.get_request(ids[0]).current_pos == len(prompts[0])
    assert sched.total_prefix_cache_hits == 0
    ids += [sched.add_request(p, max_new_tokens=n_new, temperature=0.0) for p in prompts[1:]]
    sched.step()  # admits all three
    assert sched.pending_count() == 0 and sched.active_count() == 4
    assert sched.total_prefix_cache_hits == 3
    assert sched.total_prefix_tokens_saved == 3 * 32
    for rid in ids[1:]:
        assert sched.get_request(rid).prefix_tokens_matched == 32
    while sched.has_work():
        sched.step()
    # a prompt that is two whole cached pages
    whole = sched.add_request(shared, max_new_tokens=n_new, temperature=0.0)
    while sched.has_work():
        sched.step()
    assert sched.get_request(whole).prefix_tokens_matched == 32
    assert sched.total_prefix_cache_hits == 4
    assert ex.get_paged_active_vram_bytes() == 0
    n_clear = 0
    for rid, p in zip(ids + [whole], prompts + [shared]):
        req = sched.get_request(rid)
        assert req.finished and len(req.generated_tokens) == n_new
        lg = _forced(fixture, p, req.generated_tokens)
        srt = np.sort(lg, axis=1)
        clear = (srt[:, -1] - srt[:, -2]) > 0.01 * (srt[:, -1] - srt[:, 0])
        same = np.argmax(lg, axis=1) == np.asarray(req.generated_tokens)
        assert np.all(same[clear]), f"request {rid}: {np.flatnonzero(~same)}"
        n_clear += int(clear.sum())
    assert n_clear >= 20


def _row_ok(out, ref, rel_gap=0.01) -> tuple[float, bool]:
    """(cosine, argmax agreement where the reference's top-2 gap is above rel_gap of its range)"""
    s = np.sort(np.asarray(ref, np.float64))
    clear = s[-1] - s[-2] > rel_gap * (s[-1] - s[0])
    return cos(out, ref), (not clear) or int(np.argmax(out)) == int(np.argmax(ref))


@pytest.mark.parametrize("rows", [2, 6])
@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_batched_decode_follows_reference_per_sequence(fixture, rows):
    """Every row of a batched decode step follows its OWN sequence's run in the reference CPU
    runtime (tests/golden/<fixture>_batch.npz: six prompts of 3-40 tokens, each prefilled and
    greedily decoded alone by oracle/_ref).  Each prompt is prefilled into its own paged slot,
    then the sequences decode together, `rows` per batched step, each at its own position and
    slot, teacher-forced with the reference's tokens; every logits row (prefill last rows
    included) is within the model bar (cosine 0.9998) of the reference's row and has its argmax
    wherever the reference's top-2 gap is clear.  2 rows run the decode GEMV, 6 the tensor-core
    decode matmul."""
    gold = np.load(GOLDEN / f"{fixture}_batch.npz")
    lengths = [int(n) for n in gold["lengths"]]
    offs = np.concatenate([[0], np.cumsum(lengths)])
    prompts = [gold["prompts"][offs[k]:offs[k + 1]] for k in range(len(lengths))]
    toks, ref = gold["tokens"], gold["logits"]  # [K, n + 1], [K, n + 1, V]
    K, n_rows = len(prompts), toks.shape[1]
    g, ex = _executor(fixture)
    ex.init_paged_kv_cache(K, MAX_CTX)
    ex.set_logits_last_only(True)
    sym = g.symbol_table
    in_id, out_id = g.inputs[0], g.outputs[0]
    for slot, p in enumerate(prompts):
        ex.paged_kv_alloc_slot(slot)
        ex.paged_kv_ensure_tokens(slot, len(p) + n_rows)
        ex.prepare({"s": len(p), "pos": 0, "slot": slot, **{s: len(p) for s in sym}})
        ex.set_input_by_id(in_id, np.asarray(p, np.int32))
        ex.run()
        c, ok = _row_ok(ex.get_output_array(out_id).reshape(-1), ref[slot][0])
        assert c >= 0.9998 and ok, f"prefill of sequence {slot}: cosine {c}, argmax {ok}"
    worst = 1.0
    for start in range(0, K, rows):
        grp = list(range(start, min(K, start + rows)))
        for i in range(n_rows - 1):
            ex.prepare_batch(np.array([lengths[k] + i for k in grp], np.int32),
                             np.array(grp, np.int32))
            ex.set_input_by_id(in_id, np.array([toks[k][i] for k in grp], np.int32))
            ex.run()
            out = ex.get_output_array(out_id).reshape(len(grp), -1)
            for r, k in enumerate(grp):
                c, ok = _row_ok(out[r], ref[k][i + 1])
                worst = min(worst, c)
                assert c >= 0.9998 and ok, f"sequence {k} step {i}: cosine {c}, argmax {ok}"
    for slot in range(K):
        ex.paged_kv_free_slot(slot)
    print(f"{fixture} rows={rows}: worst cosine {worst:.6f}")
