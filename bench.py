"""Benchmark of the ggmlc decoder hot path on B200: pp512 + tg128 on the Llama-3-8B-shaped Q4_0
model (batch 1), prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one sequence: prefill of 512 prompt tokens (one ubatch, logits of the last token) then
128 decode tokens through the KV cache — the reference harness's pp/tg loop
(runtime/tools/ggmlc_bench.cpp:297-565).  `value` is decode tokens/s with inputs resident in HBM
(dummy token ids as the reference harness uses, ggmlc_bench.cpp:303,431), timed with CUDA events
on the executor's stream; `e2e` is the same decode metric through the public API with host
buffers (token H2D and the greedy token D2H every step, its argmax taken on the device by
`output_argmax`).  N > 1 follows the BASELINE
configuration of the model: the Llama-3-70B shape (configs[4], "tensor-parallel over 2/4/8 B200")
runs tensor-parallel over the N GPUs (one sequence; strong scaling: QKV / gate_up / O / down /
output projection sharded, two all-reduces per layer); the shapes that one GPU serves (configs[0],
[2], [3]) run N independent replicas, one sequence each (weak scaling).  --tp / --replicas force
either; device time is the max over ranks.

--impl reference times the reference's own CPU runtime (oracle/_ref/ggmlc-bench, built from the
reference sources) on the same synthesized GGUF with all host threads: its `-pg 512,128` test,
prefill then 128 decode tokens at positions 512..639, the workload of this arm's `value`.  This
arm's `cpu_baseline` is one repetition of the same, and `parity` compares this engine with that
reference run on the same GGUF and prompt (logits cosine, greedy tokens).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "tokens/s pp512 & tg128 (Q4_0/Q8_0) per GPU and TP; % of HBM/INT8 roofline"
FALLBACK_HBM_GBS = 6650.0
BENCH_DIR = Path(os.environ.get("GGMLC_B200_BENCH_DIR", "/tmp/ggmlc_b200_bench"))
REF_BENCH_AVX2 = ROOT / "oracle" / "_ref" / "ggmlc-bench"
REF_BENCH_NATIVE = ROOT / "oracle" / "_ref" / "native" / "ggmlc-bench"
# the ISA of the native build (-march=sapphirerapids); it runs only where the host has all of it
NATIVE_FLAGS = ("avx512f", "avx512bw", "avx512vl", "avx512_vnni", "avx512_bf16", "avx512_fp16",
                "amx_int8", "amx_tile", "avx_vnni")


def ref_bench() -> tuple[Path, str]:
    """The reference's ggmlc-bench for the CPU baseline: the native build (what the reference's
    default cmake build, GGML_NATIVE, compiles on a Sapphire-Rapids-class host) when this host
    can run it, else the portable AVX2 build."""
    try:
        flags = set(Path("/proc/cpuinfo").read_text().split())
    except OSError:
        flags = set()
    if REF_BENCH_NATIVE.exists() and all(f in flags for f in NATIVE_FLAGS):
        return REF_BENCH_NATIVE, ("reference CPU build: oracle/Makefile native, -O3 "
                                  "-march=sapphirerapids (AVX-512 VNNI/BF16/FP16, AMX), the "
                                  "reference's GGML_NATIVE build on this host")
    return REF_BENCH_AVX2, "reference CPU build: oracle/Makefile, -O3 -march=x86-64-v3 (AVX2/FMA/F16C)"


REF_BENCH, REF_BUILD = ref_bench()


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(kernel: str) -> float | None:
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu summary
    profiles/<kernel>_l8_decode.md (line `dram_bytes_per_launch: N`), or None."""
    p = ROOT / "profiles" / f"{kernel}_l8_decode.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


def model_path(model: str, quant: str) -> Path:
    return BENCH_DIR / f"{model}_{quant}.gguf"


def ensure_model(model: str, quant: str, device: str | None) -> Path:
    from ggmlc_b200 import synth

    path = model_path(model, quant)
    if not path.exists():
        BENCH_DIR.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        synth.synth_model(tmp, model, synth.Q4_0 if quant == "q4_0" else synth.Q8_0,
                          device=device, name=f"{model}_{quant}")
        os.replace(tmp, path)
    return path


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    def __init__(self, gpu: int):
        self.proc = None
        self.out = BENCH_DIR / f"clocks_{gpu}_{os.getpid()}.csv"
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.out, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_first(self, timeout_s: float = 5.0) -> None:
        """Block until the sampler has written its first sample: nvidia-smi's start-up (NVML
        initialisation) then falls before the timed region, not inside a short one."""
        t0 = time.time()
        while self.proc and time.time() - t0 < timeout_s:
            try:
                if self.out.read_text().strip():
                    return
            except OSError:
                pass
            time.sleep(0.02)

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in self.out.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def ref_pg(gguf: Path, P: int, G: int, reps: int) -> dict:
    """The reference's own harness (ggmlc-bench, built from the reference sources) on the CPU,
    all host threads, test `-pg P,G`: prefill P tokens, then G decode tokens at positions
    P..P+G-1 (ggmlc_bench.cpp:566-705).  Returns pp tokens/s (P / ttft), tg tokens/s (G /
    decode time, the decode at depth P that `value` measures) and the run's wall time."""
    cores = host_threads()
    cmd = [str(REF_BENCH), "-m", str(gguf), "-d", "cpu", "-t", str(cores), "-p", "0", "-n", "0",
           "-pg", f"{P},{G}", "-r", str(reps), "-o", "json"]
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    wall = time.time() - t0
    if r.returncode != 0:
        raise RuntimeError(f"ggmlc-bench rc={r.returncode}: {r.stderr[-300:]}")
    rows = json.loads(r.stdout[r.stdout.index("["):])
    pg = [x for x in rows if x.get("n_prompt") == P and x.get("n_gen") == G][0]
    return {"tg": G / (float(pg["decode_ms"]) / 1e3), "pp": P / (float(pg["ttft_ms"]) / 1e3),
            "pg": float(pg["avg_ts"]), "cores": cores, "wall_s": wall, "reps": reps,
            "cmd": " ".join(["ggmlc-bench"] + cmd[1:2] + ["<gguf>"] + cmd[3:])}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def cpu_baseline(gguf: Path, P: int, G: int) -> dict | None:
    """The reference CPU runtime on one bounded sample of the same workload (pp P + tg G at
    depth P, one repetition after the harness's own warm-up)."""
    if not REF_BENCH.exists():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": f"unavailable: {REF_BENCH.name} not built"}
    try:
        r = ref_pg(gguf, P, G, 1)
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": host_threads(), "kind": "reference",
                "sample": f"failed: {str(e)[:200]}"}
    return {"value": round(r["tg"], 2), "unit": "tokens/s", "cores": r["cores"],
            "kind": "reference", "pp512_tokens_per_s": round(r["pp"], 1),
            "sample": f"{r['cmd']} (same GGUF, {REF_BUILD}; tg{G} at positions {P}..{P + G - 1}; "
                      f"{r['wall_s']:.0f} s wall incl. load and warm-up)"}


def reference_parity(gguf: Path, ex, in_id: int, out_id: int, sym: str, V: int, P: int,
                     G: int = 16) -> dict:
    """Checker: the reference CPU runtime (oracle/_ref) and this engine on the same GGUF and
    the same seeded prompt of P tokens, then G greedy steps.  Logits cosine per row (the engine
    teacher-forced with the reference's tokens) and whether the free-running greedy tokens are
    identical."""
    from oracle import refrun

    if not refrun.available():
        return {"unavailable": "oracle/_ref not built"}
    prompt = np.random.default_rng(11).integers(0, V, size=P).astype(np.int32)
    t0 = time.time()
    ref = refrun.RefRunner(gguf, V, max_ctx=P + G + 256)
    ref_toks, ref_rows = ref.greedy(prompt, G)
    ref.close()
    t_ref = time.time() - t0

    def run(teacher):
        ex.prepare({"s": P, sym: P, "pos": 0})
        ex.set_input_by_id(in_id, prompt)
        ex.run()
        rows = [np.asarray(ex.get_output_array(out_id), np.float32).reshape(-1)[-V:].copy()]
        toks = [int(np.argmax(rows[0]))]
        for i in range(G):
            feed = toks[-1] if teacher is None else int(teacher[i])
            ex.prepare({"s": 1, sym: 1, "pos": P + i})
            ex.set_input_by_id(in_id, np.array([feed], np.int32))
            ex.run()
            rows.append(np.asarray(ex.get_output_array(out_id), np.float32).reshape(-1)[-V:].copy())
            toks.append(int(np.argmax(rows[-1])))
        return toks, np.stack(rows)

    own, _ = run(None)
    _, tf = run(ref_toks)
    cs = [float(a.astype(np.float64) @ b / np.linalg.norm(a) / np.linalg.norm(b))
          for a, b in zip(tf.astype(np.float64), ref_rows.astype(np.float64))]
    return {"cosine_min": round(min(cs), 7), "tokens_equal": own == ref_toks,
            "prompt": P, "greedy_steps": G, "ref_threads": ref.n_threads,
            "ref_s": round(t_ref, 1)}


def run_reference(args) -> None:
    """The reference's own CPU implementation of the path on this box's host cores: its
    ggmlc-bench on the same synthesized GGUF, test -pg 512,128 (prefill, then 128 decode tokens
    at positions 512..639: the workload of this script's own `value`)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if not REF_BENCH.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ggmlc-bench not built "
                          "(make -C oracle needs the reference sources)"}))
        return
    gguf = ensure_model(args.model, args.quant, None if not _cuda() else "cuda:0")
    P, G = args.prompt, args.gen
    reps = max(1, min(args.steps, args.ref_reps))
    r = ref_pg(gguf, P, G, reps)
    v = round(r["tg"], 2)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round((P / r["pp"] + G / r["tg"]) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"{args.quant} x q8_0 int8 dot, fp32 accumulate (CPU)",
        "data": "synthetic: seeded N(0,0.02) random-init weights, dummy token ids",
        "config": {"workload": f"{args.model} {args.quant} pp{P}+tg{G} B=1 (BASELINE configs[{config_index(args.model)}])",
                   "model": args.model, "quant": args.quant, "prompt": P, "gen": G, "batch": 1,
                   "value_is": f"tg{G} decode tokens/s at positions {P}..{P + G - 1}"},
        "pp512": {"value": round(r["pp"], 1), "unit": "tokens/s"},
        "pg": {"value": round(r["pg"], 1), "unit": "tokens/s", "test": f"pp{P}+tg{G}"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": r["cores"], "kind": "reference",
                         "sample": f"{r['cmd']} ({REF_BUILD}; {r['wall_s']:.0f} s wall; "
                                   f"repetitions = min(steps, {args.ref_reps}))"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def _cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def run_ours(args) -> None:
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    if rank == 0:
        gguf = ensure_model(args.model, args.quant, f"cuda:{local}")
    if dist:
        dist.barrier()
    gguf = model_path(args.model, args.quant)

    from ggmlc_b200 import _runtime as R
    from ggmlc_b200 import synth

    g = R.ModelLoader.load_from_file(str(gguf))
    # tensor parallelism where the model's BASELINE configuration asks for it,
    # replicas where one GPU serves the model (at batch 1 on the 8B shape, tensor parallelism
    # adds two cross-GPU synchronizations a layer and measured slower than one GPU)
    tp = world > 1 and not args.replicas and (args.tp or config_index(args.model) == 4)
    if tp:  # one tensor-parallel group over all ranks; the engine's own NCCL communicator
        box = [R.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ex = R.ModelExecutor(g, f"cuda:{local}", tp_rank=rank, tp_size=world, nccl_id=box[0])
    else:
        ex = R.ModelExecutor(g, f"cuda:{local}")
    seqs = 1 if tp else world  # sequences decoded per step over the whole job
    sym = g.symbol_table[0]
    in_id, out_id = g.inputs[0], g.outputs[0]
    P, G = args.prompt, args.gen
    ex.set_logits_last_only(True)
    P_LONG = 1024  # the second prefill length BASELINE configs[3] names (pp1024)
    ex.init_kv_cache(max(P + G, P_LONG) + 256)
    ex.set_enable_cuda_graph(True)
    stream = torch.cuda.ExternalStream(ex.stream(), device=torch.device("cuda", local))
    rng = np.random.default_rng(rank)
    n_vocab = int(synth.SHAPES[args.model].vocab) if args.model in synth.SHAPES else 128256
    prompt = rng.integers(0, n_vocab, size=P).astype(np.int32)
    dummy = np.ones(1, np.int32)
    # GPT-2 graphs take the token positions as a second input
    pos_id = g.inputs[1] if len(g.inputs) > 1 else None

    def prefill(upload: bool):
        ex.prepare({"s": P, sym: P, "pos": 0})
        if upload:
            ex.set_input_by_id(in_id, prompt)
        if pos_id is not None and upload:
            ex.set_input_by_id(pos_id, np.arange(P, dtype=np.int32))
        ex.run()

    def decode(pos: int, upload_tok=None):
        ex.prepare({"s": 1, sym: 1, "pos": pos})
        # inputs resident for `value` (dummy token and, for GPT-2, dummy position ids, as the
        # reference harness's dummy tokens); e2e uploads the step's token and position
        if upload_tok is not None:
            ex.set_input_by_id(in_id, upload_tok)
            if pos_id is not None:
                ex.set_input_by_id(pos_id, np.array([pos], np.int32))
        ex.run()

    # inputs resident: prompt and decode token uploaded once
    prefill(True)
    decode(P, dummy)
    ex.synchronize()
    ex.prepare({"s": P, sym: P, "pos": 0})
    launches_pp = ex.launches_per_run()
    ex.prepare({"s": 1, sym: 1, "pos": P})
    launches_tg = ex.launches_per_run()

    def one_step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        prefill(False)
        ev[1].record(stream)
        for i in range(G):
            decode(P + i)
        ev[2].record(stream)
        return ev

    # the clock sampler starts before the warm-up (samples under load from then on)
    clocks = Clocks(local) if rank == 0 else None
    if clocks:
        clocks.wait_first()
    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize(local)
    ex.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(local)
    evs = [one_step() for _ in range(args.steps)]
    ex.synchronize()
    torch.cuda.synchronize(local)
    clk = clocks.stop() if clocks else None
    pp_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    tg_ms = sum(e[1].elapsed_time(e[2]) for e in evs)
    tot_ms = sum(e[0].elapsed_time(e[2]) for e in evs)
    if dist:
        t = torch.tensor([pp_ms, tg_ms, tot_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pp_ms, tg_ms, tot_ms = [float(x) for x in t.cpu()]
    tg_tps = seqs * args.steps * G / (tg_ms / 1e3)
    pp_tps = seqs * args.steps * P / (pp_ms / 1e3)

    # e2e: public API with host buffers — prompt H2D, per-token H2D + device argmax (token D2H)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    e2e_tg_ms = e2e_pp_ms = 0.0
    h2d = d2h = 0
    for _ in range(args.steps):
        e0.record(stream)
        prefill(True)
        tok = int(ex.output_argmax(out_id)[0])  # greedy token on the device, 4 bytes back
        e1.record(stream)
        for i in range(G):
            decode(P + i, np.array([tok], np.int32))
            tok = int(ex.output_argmax(out_id)[0])
        e2.record(stream)
        e2.synchronize()
        e2e_pp_ms += e0.elapsed_time(e1)
        e2e_tg_ms += e1.elapsed_time(e2)
    h2d = P * 4 + G * 4 + (P + G) * 4 * (pos_id is not None)
    d2h = (G + 1) * 4
    if dist:
        t = torch.tensor([e2e_pp_ms, e2e_tg_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_pp_ms, e2e_tg_ms = [float(x) for x in t.cpu()]
    e2e_tg = seqs * args.steps * G / (e2e_tg_ms / 1e3)

    # pp1024: a 1024-token prefill from position 0, device time, after one untimed run
    long_prompt = rng.integers(0, n_vocab, size=P_LONG).astype(np.int32)

    def prefill_long():
        ex.prepare({"s": P_LONG, sym: P_LONG, "pos": 0})
        ex.set_input_by_id(in_id, long_prompt)
        if pos_id is not None:
            ex.set_input_by_id(pos_id, np.arange(P_LONG, dtype=np.int32))
        ex.run()

    prefill_long()
    ex.synchronize()
    el = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    el[0].record(stream)
    for _ in range(args.steps):
        prefill_long()
    el[1].record(stream)
    ex.synchronize()
    pp_long_ms = el[0].elapsed_time(el[1]) / args.steps
    if dist:
        t = torch.tensor([pp_long_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pp_long_ms = float(t.item())

    # prefill kernels by device time: events around every launch of one prefill (launches of
    # 0.1-1 ms, where the events cost little)
    ex.set_kernel_timing(True)
    ex.reset_kernel_times()
    prefill(False)
    kt_pp = ex.kernel_times()
    ex.set_kernel_timing(False)
    pp_mm = [sum(v[i] for k, v in kt_pp.items() if k in ("gemm_q", "gemm_swiglu", "gemm_tc",
                                                            "gemm_tc_swiglu")) for i in range(3)]
    # decode kernels of one token by device time, events around every launch (each launch then
    # runs alone, without the programmatic-dependent-launch overlap of the timed run: an upper
    # bound per kernel, for the breakdown)
    ex.set_kernel_timing(True)
    ex.reset_kernel_times()
    decode(P)
    kt_tg = ex.kernel_times()
    ex.set_kernel_timing(False)
    tp_err = ex.tp_allreduce_error() if tp else 0
    if tp_err:
        raise RuntimeError("tensor-parallel all-reduce reported a timed-out peer wait: the timed "
                           "run's sums are not valid")
    # the dominant decode kernel (the fused RMSNorm + gate_up + SwiGLU GEMV, half of a token's
    # weight bytes) timed without per-launch events: back-to-back launches over 16 distinct
    # weight matrices of its shape (1.06 GB, far above L2), chained by programmatic dependent
    # launch as in the decode graph, one event pair around each pass
    roof = gemv_roofline(local) if rank == 0 else None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            parity = reference_parity(gguf, ex, in_id, out_id, sym, vocab_of(g, ex, out_id), P)
        except Exception as e:  # noqa: BLE001 - reported in the line
            parity = {"error": str(e)[:300]}

    sweep = None
    if rank == 0 and world == 1 and not args.no_sweep:
        try:
            sweep = operator_sweep(local)
        except Exception as e:  # noqa: BLE001 - reported in the line
            sweep = {"error": str(e)[:300]}

    cb_line = None
    if not args.no_cb and not tp:
        del ex  # free the single-sequence caches before the batched runs
        try:
            cb_line = run_cb(g, gguf, local)
        except Exception as e:  # noqa: BLE001 - reported in the line, the main metric stands
            cb_line = {"error": str(e)[:300]}
    if rank == 0:
        cb = cpu_baseline(gguf, P, G) if (world == 1 and not args.no_cpu_baseline) else None
        weights_gb = ex_weight_gb(g)
        line = {
            "metric": METRIC, "value": round(tg_tps, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tot_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "q4_0 x q8_0 int8 dot, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) random-init weights (ggmlc Q4_0 quantizer), "
                    "dummy token ids for value, random prompt ids for e2e",
            "config": {"workload": f"{args.model} {args.quant} pp{P}+tg{G} B=1 (BASELINE configs[{config_index(args.model)}])",
                       "model": args.model, "quant": args.quant, "prompt": P, "gen": G,
                       "batch": 1,
                       "parallelism": (f"tp{world}" if tp else f"replicas x{world}") if world > 1
                       else "single",
                       "l2": f"inputs larger than L2: {weights_gb:.2f} GB of weights streamed per "
                             "decode token",
                       "value_is": f"tg{G} decode tokens/s at positions {P}..{P + G - 1}"},
            "pp512": {"value": round(pp_tps, 1), "unit": "tokens/s",
                      "ms": round(pp_ms / args.steps, 3),
                      "matmul_ms": round(pp_mm[0], 3),
                      "kernel_ms": {k: round(v[0], 3) for k, v in
                                    sorted(kt_pp.items(), key=lambda x: -x[1][0])},
                      "matmul_int8_tops": round(pp_flops(args.model, P) / (pp_mm[0] / 1e3) / 1e12, 1)
                      if pp_mm[0] else None},
            "pp1024": {"value": round(seqs * P_LONG / (pp_long_ms / 1e3), 1), "unit": "tokens/s",
                       "ms": round(pp_long_ms, 3)},
            "tg_kernels": {k: {"us": round(v[0] * 1e3, 1), "launches": int(v[1]),
                               "gbs": round(v[2] / (v[0] * 1e6), 1) if v[0] and v[2] else None}
                           for k, v in sorted(kt_tg.items(), key=lambda x: -x[1][0])},
            "pg": {"value": round(seqs * args.steps * (P + G) / (tot_ms / 1e3), 1),
                   "unit": "tokens/s", "test": f"pp{P}+tg{G}"},
            "e2e": {"value": round(e2e_tg, 2), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "pp512_tokens_per_s": round(seqs * args.steps * P / (e2e_pp_ms / 1e3), 1)},
            "roofline": roof,
            "parity": parity,
            "cpu_baseline": cb,
            "continuous_batching": cb_line,
            "operator_sweep": sweep,
            "clocks": clk,
            "gpu_launches": int(args.steps * (launches_pp + G * launches_tg)),
        }
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_cb(g, gguf, local: int, steps: int = 256, buckets=(1, 2, 4, 8, 16)) -> dict:
    """BASELINE configs[3] continuous batching: B sequences with prompt lengths uniform in
    [64, 1024] (seeded) and `steps` greedy decode tokens each, through the scheduler on the
    paged KV cache.  Per B: decode tokens/s (all sequences decoding together) and overall
    tokens/s including the one-at-a-time admissions (prefill)."""
    import time

    from ggmlc_b200 import _runtime as R

    out = {}
    ex = R.ModelExecutor(g, f"cuda:{local}")
    ex.set_enable_cuda_graph(True)
    for B in buckets:
        sched = R.ContinuousBatchScheduler(ex, max_batch_size=B, eos_token_id=-1)
        rng = np.random.default_rng(100 + B)
        lens = rng.integers(64, 1025, size=B)
        for n in lens:
            sched.add_request(rng.integers(0, 128256, size=int(n)).astype(np.int32),
                              max_new_tokens=steps, temperature=0.0)
        t_admit = t_dec = 0.0
        n_dec_tokens = 0
        peak_pages = peak_bytes = 0  # paged KV in use, read between steps (host-side counters)
        while sched.has_work():
            admitting = sched.pending_count() > 0
            t0 = time.perf_counter()
            res = sched.step()
            dt = time.perf_counter() - t0
            if admitting:
                t_admit += dt
            else:
                t_dec += dt
                n_dec_tokens += len(res.new_tokens)
            peak_pages = max(peak_pages, ex.kv_pool_pages - ex.kv_free_pages)
            peak_bytes = max(peak_bytes, ex.get_paged_active_vram_bytes())
        total = B * steps
        out[f"B{B}"] = {"decode_tokens_per_s": round(n_dec_tokens / t_dec, 1) if t_dec else None,
                        "tokens_per_s": round(total / (t_admit + t_dec), 1),
                        "prompt_tokens": int(lens.sum()), "admit_s": round(t_admit, 3),
                        "decode_s": round(t_dec, 3),
                        "kv_pages": {"pool": int(ex.kv_pool_pages),
                                     "tokens_per_page": int(ex.tokens_per_page),
                                     "peak_in_use": int(peak_pages),
                                     "peak_mapped_gb": round(peak_bytes / 1e9, 3)}}
        del sched
    out["prefix_cache"] = run_prefix(ex)
    return out


def run_prefix(ex, n_req: int = 8, shared_len: int = 512, tail: int = 64) -> dict:
    """Prefix caching (prompt pages reused across requests): n_req requests sharing a shared_len-token prompt prefix
    (two 256-token pages) with distinct tails, admitted in one scheduler step after a first
    request with the same prefix has been served; that admission step's time with the cache off
    and on."""
    import time

    from ggmlc_b200 import _runtime as R

    rng = np.random.default_rng(7)
    shared = rng.integers(0, 128256, size=shared_len).astype(np.int32)
    tails = [rng.integers(0, 128256, size=tail).astype(np.int32) for _ in range(n_req + 1)]
    res = {"requests": n_req, "shared_tokens": shared_len, "tail_tokens": tail,
           "tokens_per_page": int(ex.tokens_per_page)}
    for on in (False, True):
        sched = R.ContinuousBatchScheduler(ex, max_batch_size=n_req, eos_token_id=-1)
        sched.enable_prefix_caching(on)
        sched.add_request(np.concatenate([shared, tails[-1]]), max_new_tokens=1, temperature=0.0)
        while sched.has_work():
            sched.step()
        for t in tails[:n_req]:
            sched.add_request(np.concatenate([shared, t]), max_new_tokens=1, temperature=0.0)
        t0 = time.perf_counter()
        sched.step()  # admits all n_req (prefill + first token each)
        dt = time.perf_counter() - t0
        while sched.has_work():
            sched.step()
        res["on" if on else "off"] = {
            "admit_s": round(dt, 4),
            "prompt_tokens_per_s": round(n_req * (shared_len + tail) / dt, 1),
            "hits": sched.total_prefix_cache_hits,
            "tokens_saved": sched.total_prefix_tokens_saved}
        del sched
    return res


def ex_weight_gb(g) -> float:
    return sum(t.data_size for t in g.tensors.values()) / 1e9


def pp_flops(model: str, P: int) -> float:
    """Prefill matmul ops: 2*P*(body linear params) + 2*V*d for the last-token lm_head."""
    from ggmlc_b200.synth import SHAPES

    c = SHAPES[model]
    if not hasattr(c, "n_kv_heads"):  # GPT-2: fused QKV d -> 3d, O, up d -> ffn, down
        per_layer = c.d_model * 3 * c.d_model + c.d_model * c.d_model + 2 * c.d_model * c.ffn
        return 2.0 * P * c.n_layers * per_layer + 2.0 * c.vocab * c.d_model
    per_layer = c.d_model * ((c.n_heads + 2 * c.n_kv_heads) * c.head_dim) + \
        c.n_heads * c.head_dim * c.d_model + c.d_model * 2 * c.ffn + c.ffn * c.d_model
    return 2.0 * P * c.n_layers * per_layer + 2.0 * c.vocab * c.d_model


def config_index(model: str) -> int:
    """BASELINE.json configs entry a model shape belongs to."""
    return {"gpt2-small": 0, "smollm2-135m": 2, "llama3-8b": 3, "llama3-70b": 4}.get(model, 3)


def vocab_of(g, ex, out_id) -> int:
    return int(ex.get_tensor_shape(out_id)[0])


def _q4_weights(L, dev, N: int, K: int, R: int, seed: int = 0):
    """R distinct repacked Q4_0 [N, K] weight matrices of random valid blocks (device)."""
    import ctypes

    import torch

    rng = np.random.default_rng(seed)
    nb = K // 32
    L.gb_weight_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
    L.gb_weight_row_bytes.restype = ctypes.c_int64
    L.gb_repack_blocks.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_void_p]
    out = []
    for _ in range(R):
        blocks = torch.randint(0, 256, (N, nb, 18), dtype=torch.uint8, device=dev)
        sc = (torch.randn((N, nb), device=dev) * 0.001).half().view(torch.uint8).reshape(N, nb, 2)
        blocks[:, :, 0:2] = sc
        wq = torch.empty(N * L.gb_weight_row_bytes(2, K), dtype=torch.uint8, device=dev)
        rc = L.gb_repack_blocks(blocks.data_ptr(), 2, N, K, wq.data_ptr(), None)
        if rc != 0:
            raise RuntimeError(L.gb_last_error().decode())
        out.append(wq)
    del blocks
    torch.cuda.synchronize()
    return out


def gemv_roofline(local: int, N: int = 28672, K: int = 4096, R: int = 16, reps: int = 4) -> dict:
    """HBM roofline of the decode gate_up GEMV as the engine runs it at batch 1 (Llama-3-8B
    shape: RMSNorm prologue, Q4_0 weights [2 x 14336, 4096], SwiGLU epilogue to f32; the down
    GEMV quantizes that row in its own prologue) through gb_gemv.  Algorithmic bytes per launch:
    weights N*K*18/32 + the f32 input row K*4 + the f32 output N/2*4.  Timed with one event pair
    around R launches on distinct weights (no event between launches), after one untimed pass;
    the mean over `reps` passes."""
    import ctypes

    import torch

    from ggmlc_b200 import _runtime as R_

    L = R_.lib()
    dev = torch.device("cuda", local)
    P_, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    L.gb_gemv.argtypes = [I, P_, I64, I64, I64, P_, P_, P_, F, P_, I, P_, P_, P_, P_, P_, P_]
    ws = _q4_weights(L, dev, N, K, R)
    x = torch.randn(K, device=dev)
    h = torch.empty(N // 2, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev)

    def one_pass():
        for w in ws:
            rc = L.gb_gemv(2, w.data_ptr(), N, K, 1, None, None, x.data_ptr(), 1e-5, None, 1,
                           h.data_ptr(), None, None, None, None, ctypes.c_void_p(st.cuda_stream))
            if rc != 0:
                raise RuntimeError(L.gb_last_error().decode())

    one_pass()
    evs = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        one_pass()
        e1.record(st)
        evs.append((e0, e1))
    torch.cuda.synchronize(dev)
    ms = sum(a.elapsed_time(b) for a, b in evs) / (reps * R)
    bytes_ = N * K * 18 / 32 + K * 4 + (N // 2) * 4
    peak, kind = peaks()
    achieved = bytes_ / (ms / 1e3) / 1e9
    del ws
    torch.cuda.empty_cache()
    return {"bound": "hbm", "kernel": "k_dgemv (RMSNorm + gate_up Q4_0 + SwiGLU)",
            "shape": f"N={N} K={K} M=1", "achieved": round(achieved, 1), "peak": peak,
            "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": kind,
            "traffic": profiled_traffic("dgemv_gate_up"),
            "bytes_per_launch": int(bytes_), "launch_us": round(ms * 1e3, 2),
            "timing": f"{R} back-to-back launches on distinct weights per event pair, "
                      f"mean of {reps} passes"}


SWEEP_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
SWEEP_M = [1, 8, 64, 512]


def measured_int8_tops() -> tuple[float, str]:
    """Dense INT8 tensor peak: twice the measured dense bf16 GEMM rate (the B200's int8 and
    bf16 tensor paths differ by 2x in dense throughput), else the nominal 4500 TOP/s."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return 2.0 * float(json.loads(p.read_text())["bf16_tflops"]), "2 x measured bf16"
        except Exception:
            pass
    return 4500.0, "nominal"


def operator_sweep(local: int, reps: int = 5) -> dict:
    """Q8_0 / Q4_0 weights N x K in {4096x4096, 14336x4096, 4096x14336,
    128256x4096} times fp32 activations N(0,1) with M in {1, 8, 64, 512}, the activations
    quantized to Q8_0 (gb_quantize_q8_0) and multiplied (gb_mul_mat_q, the dispatching entry).
    Per cell: microseconds per call (quantize + matmul, and the matmul alone), algorithmic
    TOP/s (2 M N K) and GB/s (weights + Q8_0 activations + f32 output), and the fraction of the
    cell's own bound: max(bytes / HBM peak, ops / INT8 peak) over the measured time.  Weights
    rotate over copies totalling more than L2 (126 MB), so every call streams them from HBM."""
    import ctypes

    import torch

    from ggmlc_b200 import _runtime as R_

    L = R_.lib()
    dev = torch.device("cuda", local)
    P_, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    L.gb_quantize_q8_0.argtypes = [P_, I64, I64, I64, P_, P_, P_]
    L.gb_mul_mat_q.argtypes = [I, P_, I64, I64, P_, P_, I64, P_, P_, P_, P_]
    hbm, _ = peaks()
    tops, tops_kind = measured_int8_tops()
    st = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(st.cuda_stream)
    out = {"peaks": {"hbm_gbs": hbm, "int8_tops": tops, "int8_kind": tops_kind}, "cells": {}}
    for qt, name, bpb in ((8, "q8_0", 34), (2, "q4_0", 18)):
        for (N, K) in SWEEP_SHAPES:
            wbytes = N * K // 32 * bpb
            copies = max(1, min(16, -(-(256 << 20) // wbytes)))
            nb = K // 32
            g = torch.Generator(device=dev)
            g.manual_seed(N + K + qt)
            ws = []
            for _ in range(copies):
                blocks = torch.randint(0, 256, (N, nb, bpb), dtype=torch.uint8, device=dev,
                                       generator=g)
                blocks[:, :, 0:2] = (torch.randn((N, nb), device=dev, generator=g) * 1e-3).half() \
                    .view(torch.uint8).reshape(N, nb, 2)
                L.gb_weight_row_bytes.argtypes = [I, I64]
                L.gb_weight_row_bytes.restype = I64
                wq = torch.empty(N * L.gb_weight_row_bytes(qt, K), dtype=torch.uint8, device=dev)
                L.gb_repack_blocks.argtypes = [P_, I, I64, I64, P_, P_]
                if L.gb_repack_blocks(blocks.data_ptr(), qt, N, K, wq.data_ptr(), None) != 0:
                    raise RuntimeError(L.gb_last_error().decode())
                ws.append(wq)
                del blocks
            for M in SWEEP_M:
                x = torch.randn((M, K), device=dev, generator=g)
                xq = torch.empty((M, K), dtype=torch.int8, device=dev)
                xd = torch.empty((M, nb), dtype=torch.float32, device=dev)
                y = torch.empty((M, N), dtype=torch.float32, device=dev)

                def call(w, quant=True):
                    if quant and L.gb_quantize_q8_0(x.data_ptr(), K, M, K, xq.data_ptr(),
                                                    xd.data_ptr(), sp) != 0:
                        raise RuntimeError(L.gb_last_error().decode())
                    if L.gb_mul_mat_q(qt, w.data_ptr(), N, K, xq.data_ptr(), xd.data_ptr(), M,
                                      y.data_ptr(), None, None, sp) != 0:
                        raise RuntimeError(L.gb_last_error().decode())

                n = max(reps, copies)
                for w in ws:
                    call(w)
                times = {}
                for quant in (True, False):
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    for i in range(n):
                        call(ws[i % copies], quant)
                    e1.record(st)
                    e1.synchronize()
                    times[quant] = e0.elapsed_time(e1) * 1e3 / n
                # prefill rows: the matmul alone on each GEMM path (GGMLC_B200_GEMM)
                paths = {}
                if M > 16:
                    saved = os.environ.get("GGMLC_B200_GEMM")
                    try:
                        for path in ("tc", "mma"):
                            os.environ["GGMLC_B200_GEMM"] = path
                            call(ws[0], False)
                            e0 = torch.cuda.Event(enable_timing=True)
                            e1 = torch.cuda.Event(enable_timing=True)
                            e0.record(st)
                            for i in range(n):
                                call(ws[i % copies], False)
                            e1.record(st)
                            e1.synchronize()
                            paths[path] = round(e0.elapsed_time(e1) * 1e3 / n, 2)
                    finally:
                        if saved is None:
                            os.environ.pop("GGMLC_B200_GEMM", None)
                        else:
                            os.environ["GGMLC_B200_GEMM"] = saved
                ops = 2.0 * M * N * K
                byts = wbytes + M * K * 34 / 32 + M * N * 4
                bound_us = max(byts / (hbm * 1e9), ops / (tops * 1e12)) * 1e6
                us = times[True]
                out["cells"][f"{name} {N}x{K} M={M}"] = {
                    "us": round(us, 2), "matmul_us": round(times[False], 2),
                    "tops": round(ops / (us * 1e-6) / 1e12, 1),
                    "gbs": round(byts / (us * 1e-6) / 1e9, 1),
                    "bound": "hbm" if byts / (hbm * 1e9) >= ops / (tops * 1e12) else "int8",
                    "frac": round(bound_us / us, 3)}
                if paths:
                    out["cells"][f"{name} {N}x{K} M={M}"]["matmul_us_by_path"] = paths
                del x, xq, xd, y
            del ws
            torch.cuda.empty_cache()
    return out


# single-kernel cases at the L8 decode shapes, for ncu captures of one launch (--case NAME)
CASES = {
    "gemv_rms_swiglu": dict(N=28672, K=4096, mode="rms_swiglu"),  # gate_up + RMSNorm + SwiGLU
    "gemv_rms": dict(N=6144, K=4096, mode="rms"),                 # qkv + RMSNorm prologue
    "gemv_res": dict(N=4096, K=14336, mode="res"),                # down + residual
    "attn_decode": dict(Hq=32, Hkv=8, hd=128, ctx=1024, pos=640),
    "gemm_prefill": dict(N=28672, K=4096, M=512, mode="gemm"),    # gate_up at pp512
    "gemm_prefill_tc": dict(N=28672, K=4096, M=512, mode="gemm_tc"),  # the same on tcgen05
    "mmv_swiglu_b16": dict(N=28672, K=4096, M=16, mode="rows_swiglu"),  # gate_up, 16 sequences
    "mmv_res_b16": dict(N=4096, K=14336, M=16, mode="rows_res"),        # down, 16 sequences
}


def run_case(name: str, reps: int) -> None:
    """Launch one decode kernel of the Llama-3-8B shapes `reps` times through the C ABI."""
    import ctypes

    import torch

    from ggmlc_b200 import _runtime as R

    L = R.lib()
    P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    c = CASES[name]
    rng = np.random.default_rng(0)
    dev = torch.device("cuda", 0)
    ptr = lambda t: 0 if t is None else int(t.data_ptr())  # noqa: E731

    def check(rc):
        if rc != 0:
            raise RuntimeError(L.gb_last_error().decode())

    if name.startswith(("gemv", "gemm", "mmv")):
        N, K = c["N"], c["K"]
        nb = K // 32
        blocks = rng.integers(0, 256, size=(N, nb, 18), dtype=np.uint8)
        blocks[:, :, 0:2] = (rng.standard_normal((N, nb)) * 0.001).astype(np.float16) \
            .view(np.uint8).reshape(N, nb, 2)
        L.gb_weight_row_bytes.argtypes = [I, I64]
        L.gb_weight_row_bytes.restype = I64
        src = torch.from_numpy(blocks.reshape(-1)).to(dev)
        wq = torch.empty(N * L.gb_weight_row_bytes(2, K), dtype=torch.uint8, device=dev)
        L.gb_repack_blocks.argtypes = [P, I, I64, I64, P, P]
        check(L.gb_repack_blocks(ptr(src), 2, N, K, ptr(wq), None))
        x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).to(dev)
        xq = torch.empty(K, dtype=torch.int8, device=dev)
        xd = torch.empty(K // 32, dtype=torch.float32, device=dev)
        L.gb_quantize_q8_0.argtypes = [P, I64, I64, I64, P, P, P]
        check(L.gb_quantize_q8_0(ptr(x), K, 1, K, ptr(xq), ptr(xd), None))
        res = torch.zeros(N, dtype=torch.float32, device=dev)
        y = torch.empty(N, dtype=torch.float32, device=dev)
        yq = torch.empty(N // 2, dtype=torch.int8, device=dev)
        yd = torch.empty(N // 64, dtype=torch.float32, device=dev)
        L.gb_gemv.argtypes = [I, P, I64, I64, I64, P, P, P, F, P, I, P, P, P, P, P, P]
        mode = c["mode"]
        if mode in ("gemm", "gemm_tc", "rows_swiglu", "rows_res"):
            M = c["M"]
            xm = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dev)
            xq = torch.empty((M, K), dtype=torch.int8, device=dev)
            xd = torch.empty((M, K // 32), dtype=torch.float32, device=dev)
            check(L.gb_quantize_q8_0(ptr(xm), K, M, K, ptr(xq), ptr(xd), None))
            ym = torch.empty((M, N), dtype=torch.float32, device=dev)
            resm = torch.zeros((M, N), dtype=torch.float32, device=dev)
            yqm = torch.empty((M, N // 2), dtype=torch.int8, device=dev)
            ydm = torch.empty((M, N // 64), dtype=torch.float32, device=dev)
            L.gb_mul_mat_q.argtypes = [I, P, I64, I64, P, P, I64, P, P, P, P]
            L.gb_gemm_tc.argtypes = [I, P, I64, I64, P, P, I64, P, P, P, P]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            if mode == "gemm_tc":
                rc = L.gb_gemm_tc(2, ptr(wq), N, K, ptr(xq), ptr(xd), M, ptr(ym), None, None, None)
            elif mode == "rows_swiglu":
                rc = L.gb_gemv(2, ptr(wq), N, K, M, ptr(xq), ptr(xd), None, 0.0, None, 1, None,
                               ptr(yqm), ptr(ydm), None, None, None)
            elif mode == "rows_res":
                rc = L.gb_gemv(2, ptr(wq), N, K, M, ptr(xq), ptr(xd), None, 0.0, None, 0, ptr(ym),
                               None, None, None, ptr(resm), None)
            elif mode == "gemm":
                rc = L.gb_mul_mat_q(2, ptr(wq), N, K, ptr(xq), ptr(xd), M, ptr(ym), None, None,
                                    None)
            elif mode == "rms_swiglu":  # as the engine runs it at batch 1: SwiGLU to f32
                rc = L.gb_gemv(2, ptr(wq), N, K, 1, None, None, ptr(x), 1e-5, None, 1, ptr(y),
                               None, None, None, None, None)
            elif mode == "rms":
                rc = L.gb_gemv(2, ptr(wq), N, K, 1, None, None, ptr(x), 1e-5, None, 0, ptr(y),
                               None, None, None, None, None)
            else:
                rc = L.gb_gemv(2, ptr(wq), N, K, 1, ptr(xq), ptr(xd), None, 0.0, None, 0, ptr(y),
                               None, None, None, ptr(res), None)
            check(rc)
        e1.record()
    else:
        Hq, Hkv, hd, ctx, pos = c["Hq"], c["Hkv"], c["hd"], c["ctx"], c["pos"]
        n_pos = 4096
        tab = np.empty((n_pos, hd // 2, 2), np.float32)
        L.gb_rope_table_fill.argtypes = [P, I64, I, F]
        L.gb_rope_table_fill.restype = F
        L.gb_rope_table_fill(tab.ctypes.data, n_pos, hd, 500000.0)
        t_d = torch.from_numpy(tab).to(dev)
        qkv = torch.from_numpy(rng.standard_normal((Hq + 2 * Hkv) * hd).astype(np.float32)).to(dev)
        k = torch.randn(Hkv, ctx, hd, device=dev).half()
        v = torch.randn(Hkv, ctx, hd, device=dev).half()
        L.gb_attn_decode_workspace_bytes.argtypes = [I64, I64, I64, I64]
        L.gb_attn_decode_workspace_bytes.restype = ctypes.c_size_t
        work = torch.empty(int(L.gb_attn_decode_workspace_bytes(Hq, Hkv, hd, ctx)),
                           dtype=torch.uint8, device=dev)
        oq = torch.empty(Hq * hd, dtype=torch.int8, device=dev)
        od = torch.empty(Hq * hd // 32, dtype=torch.float32, device=dev)
        L.gb_attn_decode.argtypes = [P, I64, I64, I64, P, P, I64, I64, I, F, P, I64, F, P, P, P,
                                     P, P]
        for _ in range(reps):
            check(L.gb_attn_decode(ptr(qkv), Hq, Hkv, hd, ptr(k), ptr(v), ctx, pos, hd, 500000.0,
                                   ptr(t_d), n_pos, float(hd) ** -0.5, None, ptr(oq), ptr(od),
                                   ptr(work), None))
    torch.cuda.synchronize()
    extra = {}
    if name.startswith(("gemv", "gemm", "mmv")):
        extra["us_per_launch"] = round(e0.elapsed_time(e1) * 1e3 / reps, 2)  # includes the first
    print(json.dumps({"case": name, "launches": reps, **c, **extra}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--quant", default="q4_0", choices=["q4_0", "q8_0"])
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=128)
    ap.add_argument("--ref-reps", type=int, default=3,
                    help="--impl reference: repetitions of the reference's -pg test (<= steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cb", action="store_true", help="skip the continuous-batching leg")
    ap.add_argument("--no-sweep", action="store_true", help="skip the operator-sweep leg")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent replicas instead of one tensor-parallel group")
    ap.add_argument("--tp", action="store_true",
                    help="N > 1: one tensor-parallel group for any model (default: the 70B shape)")
    ap.add_argument("--case", choices=sorted(CASES), help="launch one decode kernel of the L8 "
                    "shapes (a small case for ncu) instead of the benchmark")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    if args.case:
        run_case(args.case, args.reps)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
