"""Paged KV cache with a page table (the reference's VMM page pool, runtime/src/vmm_pool.cu:154-236,
and its page sharing for prefix hits, runtime/src/executor.cpp:853-920).

Pages of tokens_per_page positions hold K and V of every layer; each slot's page table maps its
runs of positions to pool pages and the attention kernels read the cache through it.  These tests
scatter a sequence's pages over the pool (small pages, slots grown in turn), check the batched
decode against the reference CPU runtime's per-sequence goldens, check that a prefix hit maps the
cached pages instead of copying them, and serve more requests than a small pool holds at once."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, cuda_available
from test_batch_gpu import MAX_CTX, _executor, _forced, _prompts, _row_ok

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


@pytest.mark.parametrize("fixture", ["tiny_llama_q8_0", "tiny_llama_q4_0"])
def test_scattered_pages_follow_reference_per_sequence(fixture):
    """Pages of 4 positions, handed out to the six slots in turn (slot k's pages are every sixth
    page of the pool, in no order the slot could assume), then each prompt is prefilled into its
    slot and the six sequences decode together, teacher-forced with the reference's tokens: every
    logits row is within the model bar of the reference's own run of that sequence."""
    gold = np.load(GOLDEN / f"{fixture}_batch.npz")
    lengths = [int(n) for n in gold["lengths"]]
    offs = np.concatenate([[0], np.cumsum(lengths)])
    prompts = [gold["prompts"][offs[k]:offs[k + 1]] for k in range(len(lengths))]
    toks, ref = gold["tokens"], gold["logits"]
    K, n_rows = len(prompts), toks.shape[1]
    g, ex = _executor(fixture)
    ex.set_tokens_per_page(4)
    ex.init_paged_kv_cache(K, MAX_CTX)
    ex.set_logits_last_only(True)
    T = ex.tokens_per_page
    assert T == 4
    pool = ex.kv_pool_pages
    for slot in range(K):
        ex.paged_kv_alloc_slot(slot)
    # grow the slots one page at a time, round robin, in reverse slot order on odd rounds
    need = [len(p) + n_rows for p in prompts]
    rounds = max((n + T - 1) // T for n in need)
    for r in range(rounds):
        order = range(K) if r % 2 == 0 else reversed(range(K))
        for slot in order:
            ex.paged_kv_ensure_tokens(slot, min(need[slot], (r + 1) * T))
    held = sum((n + T - 1) // T for n in need)
    assert pool - ex.kv_free_pages == held
    per_page = ex.get_paged_active_vram_bytes() // held
    assert ex.get_paged_active_vram_bytes() == held * per_page
    sym = g.symbol_table
    in_id, out_id = g.inputs[0], g.outputs[0]
    for slot, p in enumerate(prompts):
        ex.prepare({"s": len(p), "pos": 0, "slot": slot, **{s: len(p) for s in sym}})
        ex.set_input_by_id(in_id, np.asarray(p, np.int32))
        ex.run()
        c, ok = _row_ok(ex.get_output_array(out_id).reshape(-1), ref[slot][0])
        assert c >= 0.9998 and ok, f"prefill of sequence {slot}: cosine {c}, argmax {ok}"
    worst = 1.0
    for i in range(n_rows - 1):
        ex.prepare_batch(np.array([lengths[k] + i for k in range(K)], np.int32),
                         np.arange(K, dtype=np.int32))
        ex.set_input_by_id(in_id, np.array([toks[k][i] for k in range(K)], np.int32))
        ex.run()
        out = ex.get_output_array(out_id).reshape(K, -1)
        for k in range(K):
            c, ok = _row_ok(out[k], ref[k][i + 1])
            worst = min(worst, c)
            assert c >= 0.9998 and ok, f"sequence {k} step {i}: cosine {c}, argmax {ok}"
    for slot in range(K):
        ex.paged_kv_free_slot(slot)
    assert ex.kv_free_pages == pool and ex.get_paged_active_vram_bytes() == 0
    print(f"{fixture}: worst cosine {worst:.6f} over pages of {T} positions")


def test_pages_follow_tokens_and_positions_need_pages():
    g, ex = _executor("tiny_llama_q8_0")
    ex.set_tokens_per_page(16)
    ex.init_paged_kv_cache(2, MAX_CTX)
    pool = ex.kv_pool_pages
    ex.paged_kv_alloc_slot(0)
    assert ex.get_paged_active_vram_bytes() == 0
    ex.paged_kv_ensure_tokens(0, 1)
    one = ex.get_paged_active_vram_bytes()
    assert one > 0 and ex.kv_free_pages == pool - 1
    ex.paged_kv_ensure_tokens(0, 16)
    assert ex.get_paged_active_vram_bytes() == one
    ex.paged_kv_ensure_tokens(0, 17)
    assert ex.get_paged_active_vram_bytes() == 2 * one
    # a prefill past the slot's pages is refused before any launch
    sym = g.symbol_table
    with pytest.raises(RuntimeError, match="no pages"):
        ex.prepare({"s": 40, "pos": 0, "slot": 0, **{s: 40 for s in sym}})
    with pytest.raises(RuntimeError, match="no page"):
        ex.prepare_batch(np.array([32], np.int32), np.array([0], np.int32))
    with pytest.raises(RuntimeError):
        ex.set_tokens_per_page(24)  # not a power of two
    with pytest.raises(RuntimeError, match="in use"):
        ex.set_tokens_per_page(32)  # slot 0 holds pages
    ex.paged_kv_free_slot(0)
    assert ex.kv_free_pages == pool and ex.get_paged_active_vram_bytes() == 0
    ex.set_tokens_per_page(32)  # an idle pool is laid out again
    assert ex.tokens_per_page == 32


def test_prefix_hit_maps_cached_pages():
    """Three requests sharing a cold request's two whole prompt pages take one new page each:
    the two cached pages are mapped into their page tables, not copied (6 pages in use, not
    12).  A prompt cached whole gets a private copy of its last page before re-evaluating its
    last token, so the cached page keeps the cold request's rows."""
    from ggmlc_b200 import _runtime as R

    fixture = "tiny_llama_q8_0"
    rng = np.random.default_rng(21)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    g, ex = _executor(fixture)
    ex.set_tokens_per_page(16)
    sched = R.ContinuousBatchScheduler(ex, max_batch_size=4, eos_token_id=-1)
    ex.init_paged_kv_cache(4, MAX_CTX)
    pool = ex.kv_pool_pages
    shared = list(rng.integers(1, vocab, size=32))
    prompts = [shared + list(rng.integers(1, vocab, size=3)) for _ in range(4)]
    ids = [sched.add_request(prompts[0], max_new_tokens=6, temperature=0.0)]
    sched.step()
    assert pool - ex.kv_free_pages == 3  # 35 tokens of 16-position pages
    per_page = ex.get_paged_active_vram_bytes() // 3
    ids += [sched.add_request(p, max_new_tokens=6, temperature=0.0) for p in prompts[1:]]
    sched.step()
    assert sched.active_count() == 4 and sched.total_prefix_cache_hits == 3
    assert pool - ex.kv_free_pages == 6
    assert ex.get_paged_active_vram_bytes() == 6 * per_page
    while sched.has_work():
        sched.step()
    # the finished requests returned their own pages; the tree keeps the two shared ones
    assert pool - ex.kv_free_pages == 2 and ex.get_paged_active_vram_bytes() == 0
    whole = sched.add_request(shared, max_new_tokens=6, temperature=0.0)
    sched.step()
    # the shared first page, a private copy of the second, nothing else
    assert ex.get_paged_active_vram_bytes() == 2 * per_page
    assert pool - ex.kv_free_pages == 3
    while sched.has_work():
        sched.step()
    for rid, p in zip(ids + [whole], prompts + [shared]):
        req = sched.get_request(rid)
        lg = _forced(fixture, p, req.generated_tokens)
        srt = np.sort(lg, axis=1)
        clear = (srt[:, -1] - srt[:, -2]) > 0.01 * (srt[:, -1] - srt[:, 0])
        same = np.argmax(lg, axis=1) == np.asarray(req.generated_tokens)
        assert np.all(same[clear]), f"request {rid}: {np.flatnonzero(~same)}"
    # a later request over the same prefix still reads the cold request's rows (the prompt cached
    # whole wrote only into its private copy)
    hits = sched.total_prefix_cache_hits
    again = sched.add_request(prompts[1], max_new_tokens=6, temperature=0.0)
    while sched.has_work():
        sched.step()
    assert sched.total_prefix_cache_hits == hits + 1
    req = sched.get_request(again)
    lg = _forced(fixture, prompts[1], req.generated_tokens)
    srt = np.sort(lg, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 0.01 * (srt[:, -1] - srt[:, 0])
    same = np.argmax(lg, axis=1) == np.asarray(req.generated_tokens)
    assert np.all(same[clear]), f"repeat request: {np.flatnonzero(~same)}"


def test_small_pool_admits_requests_as_pages_allow():
    """A pool of 6 pages of 16 positions serves ten requests that need 1-4 pages each (20 in
    all) with up to four slots: a request waits until the running ones return enough pages,
    prefix pages are evicted to make room, and every request's tokens follow its own decode
    alone wherever the top-2 gap is clear."""
    from ggmlc_b200 import _runtime as R

    fixture = "tiny_llama_q8_0"
    rng = np.random.default_rng(12)
    vocab = int(np.load(GOLDEN / f"{fixture}.npz")["full_logits"].shape[1])
    prompts = _prompts(rng, [5, 17, 33, 9, 40, 3, 21, 12, 7, 30], vocab)
    n_new = 10
    g, ex = _executor(fixture)
    ex.set_tokens_per_page(16)
    ex.configure_kv_pool_pages(6)
    sched = R.ContinuousBatchScheduler(ex, max_batch_size=4, eos_token_id=-1)
    assert ex.kv_pool_pages == 6
    with pytest.raises(RuntimeError, match="pages"):
        sched.add_request(list(range(1, 91)), max_new_tokens=10)  # 7 pages
    ids = [sched.add_request(p, max_new_tokens=n_new, temperature=0.0) for p in prompts]
    steps = 0
    waited = False
    while sched.has_work():
        sched.step()
        waited |= sched.pending_count() > 0 and sched.active_count() < 4
        assert 6 - ex.kv_free_pages <= 6
        steps += 1
        assert steps < 500
    assert waited  # some request waited for pages, not for a slot
    assert ex.get_paged_active_vram_bytes() == 0
    n_clear = 0
    for rid, p in zip(ids, prompts):
        req = sched.get_request(rid)
        assert req.finished and len(req.generated_tokens) == n_new
        lg = _forced(fixture, p, req.generated_tokens)
        srt = np.sort(lg, axis=1)
        clear = (srt[:, -1] - srt[:, -2]) > 0.01 * (srt[:, -1] - srt[:, 0])
        same = np.argmax(lg, axis=1) == np.asarray(req.generated_tokens)
        assert np.all(same[clear]), f"prompt {len(p)}: {np.flatnonzero(~same)}"
        n_clear += int(clear.sum())
    assert n_clear >= 50
