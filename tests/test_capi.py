"""Host-side checks of the C ABI (no GPU needed): the library loads, exports every symbol the
header declares, parses the reference's GGUF containers like the reference loader, and refuses
the CPU device (no CPU fallback)."""

from __future__ import annotations

import ctypes
import json
import re

import numpy as np
import pytest

from conftest import FIXTURES, GOLDEN, ROOT
from oracle import oracle as O


def header_symbols() -> list[str]:
    text = (ROOT / "include" / "ggmlc_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from ggmlc_b200 import _runtime

    lib = ctypes.CDLL(str(_runtime._LIB_PATH))
    syms = header_symbols()
    assert len(syms) > 50
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_available_devices_lists_cpu_first():
    from ggmlc_b200 import _runtime

    devs = _runtime.get_available_devices()
    assert devs[0] == "cpu"
    assert all(d == "cpu" or d.startswith("cuda") for d in devs)


@pytest.mark.parametrize("fixture", FIXTURES)
def test_loader_matches_graph_spec(fixture):
    from ggmlc_b200 import _runtime

    path = GOLDEN / f"{fixture}.gguf"
    g = _runtime.ModelLoader.load_from_file(str(path))
    kv, infos, data = O.read_gguf(path)
    spec = json.loads(kv["ggmlc.graph_spec"])
    assert g.name == spec["name"]
    assert g.symbol_table == spec["symbol_table"]
    assert g.inputs == spec["inputs"] and g.outputs == spec["outputs"]
    assert g.parameters == spec["parameters"]
    assert sorted(g.tensors) == sorted(int(k) for k in spec["tensors"])
    assert [op.opcode for op in g.ops] == [n["opcode"] for n in spec["nodes"]]
    for tid, t in g.tensors.items():
        st = spec["tensors"][str(tid)]
        assert t.name == st["name"] and t.type == st["type"] and t.storage == st["storage"]
        if t.name in data:
            assert t.data_size == data[t.name].size
    # the token input's ne[0] is the sequence symbol
    t0 = g.tensors[g.inputs[0]]
    assert t0.symbol_index(0) == 0 and t0.symbol_index(1) == -1
    # bytes loader agrees with the file loader
    g2 = _runtime.ModelLoader.load_from_bytes(path.read_bytes())
    assert sorted(g2.tensors) == sorted(g.tensors) and len(g2.ops) == len(g.ops)


def test_loader_rejects_bad_files(tmp_path):
    from ggmlc_b200 import _runtime

    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(RuntimeError, match="bad magic"):
        _runtime.ModelLoader.load_from_file(str(bad))
    with pytest.raises(RuntimeError, match="cannot open"):
        _runtime.ModelLoader.load_from_file(str(tmp_path / "missing.gguf"))
    good = (GOLDEN / "tiny_llama_q8_0.gguf").read_bytes()
    with pytest.raises(RuntimeError):
        _runtime.ModelLoader.load_from_bytes(good[: len(good) // 2])


def test_executor_refuses_cpu_device():
    from ggmlc_b200 import _runtime

    g = _runtime.ModelLoader.load_from_file(str(GOLDEN / "tiny_llama_q8_0.gguf"))
    with pytest.raises(RuntimeError, match="not served by the B200 engine"):
        _runtime.ModelExecutor(g, "cpu")


def test_rope_table_fill_matches_oracle():
    from ggmlc_b200 import _runtime

    lib = _runtime.lib()
    lib.gb_rope_table_fill.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float]
    lib.gb_rope_table_fill.restype = ctypes.c_float
    n_pos, nd = 64, 64
    tab = np.empty((n_pos, nd // 2, 2), np.float32)
    lib.gb_rope_table_fill(tab.ctypes.data, n_pos, nd, 10000.0)
    # rotate a unit vector pair through the oracle: y0 = cos, y1 = sin for x = (1, 0)
    x = np.zeros((n_pos, 1, nd), np.float32)
    x[:, 0, : nd // 2] = 1.0
    y = O.rope_neox(x, np.arange(n_pos, dtype=np.int32), nd, np.float32(10000.0))
    assert np.array_equal(tab[:, :, 0], y[:, 0, : nd // 2])
    assert np.array_equal(tab[:, :, 1], y[:, 0, nd // 2:])


def test_kv_row_offsets_tile_contiguous_and_paged_caches():
    """gb_kv_row_offset, the addressing of every attention kernel: contiguous rows at
    (h * ctx + t) * hd; paged rows inside the listed pages only, every (h, t) of a sequence at
    its own offset, and two sequences with disjoint page lists never on the same row."""
    from ggmlc_b200 import _runtime

    lib = _runtime.lib()
    P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.gb_kv_row_offset.argtypes = [P, I, I64, I64, I64, I64, I64]
    lib.gb_kv_row_offset.restype = I64
    H, hd, ctx = 3, 8, 40
    for h, t in [(0, 0), (2, 39), (1, 17)]:
        assert lib.gb_kv_row_offset(None, 0, H, ctx, h, t, hd) == (h * ctx + t) * hd
    assert lib.gb_kv_row_offset(None, 17, H, ctx, 0, 0, hd) == -1
    rng = np.random.default_rng(4)
    shift = 2  # pages of 4 positions
    T = 1 << shift
    pool = rng.permutation(np.arange(1, 21)).astype(np.int32)  # 20 pages, scattered order
    seqs = [pool[:10].copy(), pool[10:].copy()]  # 10 pages = 40 positions each
    seen = {}
    for s, pages in enumerate(seqs):
        for h in range(H):
            for t in range(len(pages) * T):
                off = lib.gb_kv_row_offset(pages.ctypes.data, shift, H, ctx, h, t, hd)
                page = off // (H * T * hd)
                assert page == pages[t >> shift]  # inside the page the list names
                assert off % hd == 0
                assert off == ((int(pages[t >> shift]) * H + h) * T + (t & (T - 1))) * hd
                assert off not in seen, (s, h, t, seen.get(off))
                seen[off] = (s, h, t)
    assert len(seen) == 2 * H * 10 * T
