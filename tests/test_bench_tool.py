"""ggmlc-bench for this engine (ggmlc_b200/ggmlc-bench): the reference's benchmark CLI
(runtime/tools/ggmlc_bench.cpp) with the same flags and output records, so the reference's
comparison scripts (examples/benchmarks/compare_ggmlc_vs_llama_cpp.py) can run it.  The
argument handling is checked on the host; a GPU run on a golden tiny model checks the JSON
records and the CSV / markdown forms."""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest

from conftest import GOLDEN, cuda_available

ROOT = Path(__file__).resolve().parent.parent
TOOL = ROOT / "ggmlc_b200" / "ggmlc-bench"
# the record keys of the reference's JSON output (ggmlc_bench.cpp:708-744)
KEYS = ["engine", "model_filename", "model_type", "model_size", "model_n_params", "device",
        "n_threads", "n_prompt", "n_gen", "n_depth", "test", "avg_ns", "stddev_ns", "avg_ts",
        "stddev_ts", "avg_ms", "ttft_ms", "decode_ms"]


@pytest.fixture(scope="module")
def tool():
    from ggmlc_b200 import build

    build.build_bench_tool()
    assert TOOL.exists()
    return str(TOOL)


def _run(args, timeout=300):
    return subprocess.run(args, capture_output=True, text=True, timeout=timeout)


def test_cli_help_and_errors(tool):
    r = _run([tool, "--help"])
    assert r.returncode == 0 and "--n-prompt" in r.stdout and "-pg" in r.stdout
    r = _run([tool])
    assert r.returncode == 1  # no arguments: usage, failure (as the reference)
    r = _run([tool, "-m", str(ROOT / "no_such_model.gguf")])
    assert r.returncode == 1 and "Cannot open model file" in r.stderr
    r = _run([tool, "-m", str(GOLDEN / "tiny_llama_q8_0.gguf"), "-pg", "1,2,3"])
    assert r.returncode == 1 and "-pg expects exactly two ints" in r.stderr
    r = _run([tool, "-p", "8"])
    assert r.returncode == 1 and "No model file specified" in r.stderr


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
def test_json_records_on_a_tiny_model(tool):
    model = str(GOLDEN / "tiny_llama_q8_0.gguf")
    r = _run([tool, model, "-m", model, "-p", "16,40", "-n", "8", "-r", "2", "-t", "4",
              "-ub", "16", "--device", "cuda", "-o", "json", "-pg", "24,6", "--cuda-graph"])
    assert r.returncode == 0, r.stderr
    out = r.stdout.strip()
    recs = json.loads(out[out.find("["): out.rfind("]") + 1])
    by_test = {rec["test"]: rec for rec in recs}
    assert sorted(by_test) == ["pp16", "pp24+tg6", "pp40", "tg8"]
    for rec in recs:
        assert list(rec) == KEYS
        assert rec["engine"] == "ggmlc_b200" and rec["device"] == "cuda" and rec["n_threads"] == 4
        assert rec["avg_ts"] > 0 and rec["avg_ns"] > 0 and rec["model_n_params"] > 0
    assert by_test["pp40"]["n_prompt"] == 40 and by_test["pp40"]["ttft_ms"] > 0
    assert by_test["tg8"]["n_gen"] == 8 and by_test["tg8"]["decode_ms"] > 0
    pg = by_test["pp24+tg6"]
    assert pg["ttft_ms"] > 0 and pg["decode_ms"] > 0
    assert pg["avg_ms"] == pytest.approx(pg["ttft_ms"] + pg["decode_ms"], rel=0.05, abs=0.05)
    for fmt, head in (("csv", "engine,model_filename"), ("md", "| model | size")):
        r = _run([tool, "-m", model, "-p", "16", "-n", "4", "-r", "1", "-o", fmt])
        assert r.returncode == 0, r.stderr
        lines = r.stdout.strip().splitlines()
        assert lines[0].startswith(head) and len(lines) == (3 if fmt == "csv" else 4)
