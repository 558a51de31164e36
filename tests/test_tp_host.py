"""Tensor-parallel partition (ggmlc_b200/csrc/tp.cpp) checked on the host: two gloo ranks each
take their plan from the engine's planner (no device touched), slice the GGUF weights of a
reference-compiled fixture as the executor does at upload, run their shard of every layer's
projections with the oracle's CPU matmul, and exchange partial sums / logits over gloo.

Column-parallel outputs (q / k / v heads, gate / up halves, vocabulary rows) must be bit-exact
slices of the unsharded results; row-parallel outputs (O, down) after the all-reduce must match
the unsharded matmul to fp32 summation order (1e-5 of the output range)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN

torch = pytest.importorskip("torch")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _close(y, ref, rel=1e-5):
    return np.max(np.abs(y - ref)) <= rel * max(np.max(np.abs(ref)), 1e-30)


def _weights(fixture):
    from oracle import oracle as O

    kv, infos, data = O.read_gguf(GOLDEN / f"{fixture}.gguf")
    return infos, data


def _slice(data, dims, wtype, sl):
    """The executor's upload slicing (slice_payload in executor.cpp) on GGUF block bytes."""
    from oracle import oracle as O

    K, N = int(dims[0]), int(np.prod(dims[1:]))
    rows = data.reshape(N, O.row_bytes(wtype, K))
    if "cols" in sl:
        c0, c1 = sl["cols"]
        bb = O.row_bytes(wtype, 32)
        part = rows.reshape(N, K // 32, bb)[:, c0 // 32:c1 // 32].reshape(N, -1)
        return np.ascontiguousarray(part), N, c1 - c0
    part = np.concatenate([rows[a:b] for a, b in sl["rows"]])
    return np.ascontiguousarray(part), part.shape[0], K


def _rank_main(rank, world, port, fixture, q):
    try:
        import torch.distributed as dist

        from ggmlc_b200 import _runtime as R
        from oracle import oracle as O

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = R.ModelLoader.load_from_file(str(GOLDEN / f"{fixture}.gguf"))
        plan = R.tensor_parallel_plan(g, rank, world)
        infos, data = _weights(fixture)
        rng = np.random.default_rng(3)
        checked = 0
        for name, sl in sorted(plan["slices"].items()):
            dims, wtype, _ = infos[name]
            K, N = int(dims[0]), int(np.prod(dims[1:]))
            part, Np, Kp = _slice(data[name], dims, wtype, sl)
            x = rng.standard_normal((3, K)).astype(np.float32)
            if "rows" in sl:  # column-parallel: this rank's output columns, bit-exact
                full = O.mul_mat(wtype, data[name], N, K, x)
                mine = O.mul_mat(wtype, part, Np, Kp, x)
                cols = np.concatenate([np.arange(a, b) for a, b in sl["rows"]])
                assert np.array_equal(mine, full[:, cols]), name
                if ".mlp." in name:  # SwiGLU stays local: gate / up halves of the same units
                    assert np.array_equal(O.swiglu(mine), O.swiglu(full)[:, cols[: Np // 2]])
            else:  # row-parallel: partial sums over this rank's K range, all-reduced
                c0, c1 = sl["cols"]
                y = torch.from_numpy(O.mul_mat(wtype, part, Np, Kp, np.ascontiguousarray(x[:, c0:c1])))
                dist.all_reduce(y)
                assert _close(y.numpy(), O.mul_mat(wtype, data[name], N, K, x)), name
            checked += 1
        # vocabulary-split output projection: logits all-gathered in rank order
        w = plan["vocab_weight"]
        if w:
            dims, wtype, _ = infos[w]
            K, V = int(dims[0]), int(dims[1])
            Vr = plan["vocab_rows"]
            x = rng.standard_normal((2, K)).astype(np.float32)
            rows = data[w].reshape(V, -1)[rank * Vr:(rank + 1) * Vr]
            mine = torch.from_numpy(O.mul_mat(wtype, np.ascontiguousarray(rows), Vr, K, x))
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            assert np.array_equal(torch.cat(parts, 1).numpy(), O.mul_mat(wtype, data[w], V, K, x))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, checked, plan["n_attention"], plan["n_mlp"], None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, 0, 0, 0, repr(e)))


@pytest.mark.parametrize("fixture,world", [("tiny_llama_q8_0", 2), ("tiny_llama_q4_0", 2),
                                           ("tiny_llama_kv8_q4_0", 4), ("tiny_llama_kv8_q4_0", 8)])
def test_tensor_parallel_shards_recombine_over_gloo(fixture, world):
    """world ranks (the eight-KV-head fixture keeps whole heads on 4 and 8 ranks)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, fixture, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, checked, n_att, n_mlp, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert n_att == 2 and n_mlp == 2
        assert checked == 8  # QKV, O, gate_up, down of both layers


def test_tensor_parallel_plan_shapes_and_partition():
    """Each rank's slices tile the weights exactly; head / FFN dimensions are divided; the
    planner refuses head counts that do not divide; blocks it does not shard stay replicated."""
    from ggmlc_b200 import _runtime as R

    g = R.ModelLoader.load_from_file(str(GOLDEN / "tiny_llama_q8_0.gguf"))
    infos, _ = _weights("tiny_llama_q8_0")
    plans = [R.tensor_parallel_plan(g, r, 2) for r in range(2)]
    for name in plans[0]["slices"]:
        dims = infos[name][0]
        K, N = int(dims[0]), int(np.prod(dims[1:]))
        if "cols" in plans[0]["slices"][name]:
            spans = sorted(p["slices"][name]["cols"] for p in plans)
            assert spans[0][0] == 0 and spans[-1][1] == K and spans[0][1] == spans[1][0]
            assert all((b - a) % 32 == 0 for a, b in spans)
        else:
            rows = sorted(r for p in plans for r in p["slices"][name]["rows"])
            assert rows[0][0] == 0 and rows[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
        assert plans[0]["shapes"][name] != [K, N, 1, 1]  # rewritten for the rank
    assert plans[0]["partial"] == plans[1]["partial"] and len(plans[0]["partial"]) == 4
    with pytest.raises(RuntimeError, match="do not divide"):
        R.tensor_parallel_plan(g, 0, 3)
    with pytest.raises(RuntimeError, match="do not divide"):
        R.tensor_parallel_plan(g, 0, 4)  # two KV heads over four ranks
    # eight KV heads: 8 ranks each take one q head and one KV head; the FFN splits 8 ways
    g8 = R.ModelLoader.load_from_file(str(GOLDEN / "tiny_llama_kv8_q4_0.gguf"))
    p8 = [R.tensor_parallel_plan(g8, r, 8) for r in range(8)]
    assert all(p["n_attention"] == 2 and p["n_mlp"] == 2 for p in p8)
    for name, sl in p8[0]["slices"].items():
        if "rows" in sl:  # the ranks' row ranges tile the rows
            rows = sorted(r for p in p8 for r in p["slices"][name]["rows"])
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
    # GPT-2: attention sharded (QKV bias sliced with its rows), the bias-GELU MLP replicated
    gp = R.tensor_parallel_plan(R.ModelLoader.load_from_file(str(GOLDEN / "tiny_gpt2_q8_0.gguf")),
                                1, 2)
    assert gp["n_attention"] == 2 and gp["n_mlp"] == 0 and len(gp["partial"]) == 2
    assert any(k.endswith("bias") and "rows" in v for k, v in gp["slices"].items())
