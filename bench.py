"""Benchmark of the ggmlc decoder hot path on B200: pp512 + tg128 on the Llama-3-8B-shaped Q4_0
model (batch 1), prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one sequence: prefill of 512 prompt tokens (one ubatch, logits of the last token) then
128 decode tokens through the KV cache — the reference harness's pp/tg loop
(runtime/tools/ggmlc_bench.cpp:297-565).  `value` is decode tokens/s with inputs resident in HBM
(dummy token ids as the reference harness uses, ggmlc_bench.cpp:303,431), timed with CUDA events
on the executor's stream; `e2e` is the same decode metric through the public API with host
buffers (token H2D, logits D2H and a host argmax every step).  N > 1 runs independent replicas
(weak scaling), timed as the max over ranks.

--impl reference times the reference's own CPU runtime (oracle/_ref/ggmlc-bench, built from the
reference sources) on the same synthesized GGUF, all host threads, a bounded tg sample per step.
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
REF_BENCH = ROOT / "oracle" / "_ref" / "ggmlc-bench"


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def model_path(model: str, quant: str) -> Path:
    return BENCH_DIR / f"{model}_{quant}.gguf"


def ensure_model(model: str, quant: str, device: str | None) -> Path:
    from ggmlc_b200 import synth

    path = model_path(model, quant)
    if not path.exists():
        BENCH_DIR.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp")
        synth.synth_llama(tmp, model, synth.Q4_0 if quant == "q4_0" else synth.Q8_0,
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


def cpu_baseline(gguf: Path, n_gen: int = 8) -> dict | None:
    """The reference CPU runtime (ggmlc-bench built from the reference sources) on a bounded
    tg sample of the same model."""
    if not REF_BENCH.exists():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": f"unavailable: {REF_BENCH.name} not built"}
    cores = os.cpu_count() or 1
    cmd = [str(REF_BENCH), "-m", str(gguf), "-d", "cpu", "-t", str(cores), "-p", "0", "-n",
           str(n_gen), "-r", "1", "-o", "json", "--no-warmup"]
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    wall = time.time() - t0
    try:
        rows = json.loads(r.stdout[r.stdout.index("["):])
        tg = [x for x in rows if x.get("n_gen", 0) > 0][0]
        return {"value": float(tg["avg_ts"]), "unit": "tokens/s", "cores": cores,
                "kind": "reference",
                "sample": f"ggmlc-bench -d cpu -t {cores} tg{n_gen} after one untimed token "
                          f"(same GGUF; {wall:.0f} s wall incl. load)"}
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": cores, "kind": "reference",
                "sample": f"failed: {e}; {r.stderr[-200:]}"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gguf = ensure_model(args.model, args.quant, None if not _cuda() else "cuda:0")
    cores = os.cpu_count() or 1
    n_gen = args.ref_gen
    cmd = [str(REF_BENCH), "-m", str(gguf), "-d", "cpu", "-t", str(cores), "-p", "0", "-n",
           str(n_gen), "-r", str(args.steps), "-o", "json"]
    if not REF_BENCH.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ggmlc-bench not built "
                          "(make -C oracle needs the reference sources)"}))
        return
    t0 = time.time()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    wall = time.time() - t0
    rows = json.loads(r.stdout[r.stdout.index("["):])
    tg = [x for x in rows if x.get("n_gen", 0) > 0][0]
    v = float(tg["avg_ts"])
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": float(tg["avg_ms"]),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_0 x q8_0 int8 dot, fp32 accumulate (CPU)",
        "data": "synthetic: seeded N(0,0.02) random-init weights, dummy token ids",
        "config": {"workload": f"{args.model} {args.quant} tg (decode) B=1, reference CPU runtime",
                   "model": args.model, "quant": args.quant, "gen_per_step": n_gen, "batch": 1},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "reference",
                         "sample": f"ggmlc-bench -d cpu -t {cores} -p 0 -n {n_gen} -r {args.steps} "
                                   f"({wall:.0f} s wall)"},
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

    g = R.ModelLoader.load_from_file(str(gguf))
    ex = R.ModelExecutor(g, f"cuda:{local}")
    sym = g.symbol_table[0]
    in_id, out_id = g.inputs[0], g.outputs[0]
    P, G = args.prompt, args.gen
    ex.set_logits_last_only(True)
    ex.init_kv_cache(P + G + 256)
    ex.set_enable_cuda_graph(True)
    stream = torch.cuda.ExternalStream(ex.stream(), device=torch.device("cuda", local))
    rng = np.random.default_rng(rank)
    prompt = rng.integers(0, 128256, size=P).astype(np.int32)
    dummy = np.ones(1, np.int32)

    def prefill(upload: bool):
        ex.prepare({"s": P, sym: P, "pos": 0})
        if upload:
            ex.set_input_by_id(in_id, prompt)
        ex.run()

    def decode(pos: int, upload_tok=None):
        ex.prepare({"s": 1, sym: 1, "pos": pos})
        if upload_tok is not None:
            ex.set_input_by_id(in_id, upload_tok)
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

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize(local)
    ex.synchronize()
    if dist:
        dist.barrier()
    clocks = Clocks(local) if rank == 0 else None
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
    tg_tps = world * args.steps * G / (tg_ms / 1e3)
    pp_tps = world * args.steps * P / (pp_ms / 1e3)

    # e2e: public API with host buffers — prompt H2D, per-token H2D + logits D2H + host argmax
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    e2e_tg_ms = e2e_pp_ms = 0.0
    h2d = d2h = 0
    for _ in range(args.steps):
        e0.record(stream)
        prefill(True)
        logits = ex.get_output_array(out_id)
        e1.record(stream)
        tok = int(np.argmax(logits))
        for i in range(G):
            decode(P + i, np.array([tok], np.int32))
            logits = ex.get_output_array(out_id)
            tok = int(np.argmax(logits))
        e2.record(stream)
        e2.synchronize()
        e2e_pp_ms += e0.elapsed_time(e1)
        e2e_tg_ms += e1.elapsed_time(e2)
    h2d = P * 4 + G * 4
    d2h = (G + 1) * logits.nbytes
    if dist:
        t = torch.tensor([e2e_pp_ms, e2e_tg_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_pp_ms, e2e_tg_ms = [float(x) for x in t.cpu()]
    e2e_tg = world * args.steps * G / (e2e_tg_ms / 1e3)

    # roofline of the dominant decode kernel (Q4_0 GEMV): per-launch events over one sequence
    ex.set_kernel_timing(True)
    ex.reset_kernel_times()
    for i in range(G):
        decode(P + i)
    kt = ex.kernel_times()
    ex.set_kernel_timing(False)
    ex.reset_kernel_times()
    prefill(False)
    ex.set_kernel_timing(True)
    prefill(False)
    kt_pp = ex.kernel_times()
    ex.set_kernel_timing(False)
    peak, peak_kind = peaks()
    mm = kt.get("matmul_q", [0, 1, 0])
    achieved = mm[2] / (mm[0] / 1e3) / 1e9 if mm[0] > 0 else 0.0
    dec_total = sum(v[0] for v in kt.values())
    shares = {k: round(v[0] / dec_total, 4) for k, v in sorted(kt.items(), key=lambda x: -x[1][0])}
    pp_mm = kt_pp.get("matmul_q", [0, 1, 0])

    if rank == 0:
        cb = cpu_baseline(gguf) if (world == 1 and not args.no_cpu_baseline) else None
        weights_gb = ex_weight_gb(g)
        line = {
            "metric": METRIC, "value": round(tg_tps, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tot_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_0 x q8_0 int8 dot, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) random-init weights (ggmlc Q4_0 quantizer), "
                    "dummy token ids for value, random prompt ids for e2e",
            "config": {"workload": f"{args.model} {args.quant} pp{P}+tg{G} B=1 (BASELINE configs[3])",
                       "model": args.model, "quant": args.quant, "prompt": P, "gen": G,
                       "batch": 1, "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": f"inputs larger than L2: {weights_gb:.2f} GB of weights streamed per "
                             "decode token", "value_is": f"tg{G} decode tokens/s"},
            "pp512": {"value": round(pp_tps, 1), "unit": "tokens/s",
                      "ms": round(pp_ms / args.steps, 3),
                      "matmul_ms": round(pp_mm[0], 3),
                      "matmul_int8_tops": round(pp_flops(args.model, P) / (pp_mm[0] / 1e3) / 1e12, 1)
                      if pp_mm[0] else None},
            "e2e": {"value": round(e2e_tg, 2), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "pp512_tokens_per_s": round(world * args.steps * P / (e2e_pp_ms / 1e3), 1)},
            "roofline": {"bound": "hbm", "kernel": "matmul_q (decode GEMV, Q4_0 x Q8_0)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None,
                         "bytes_per_launch": round(mm[2] / max(mm[1], 1)),
                         "launch_ms": round(mm[0] / max(mm[1], 1), 5),
                         "decode_share": shares},
            "cpu_baseline": cb,
            "clocks": clk,
            "gpu_launches": int(args.steps * (launches_pp + G * launches_tg)),
        }
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def ex_weight_gb(g) -> float:
    return sum(t.data_size for t in g.tensors.values()) / 1e9


def pp_flops(model: str, P: int) -> float:
    """Prefill matmul ops: 2*P*(body linear params) + 2*V*d for the last-token lm_head."""
    from ggmlc_b200.synth import SHAPES

    c = SHAPES[model]
    per_layer = c.d_model * ((c.n_heads + 2 * c.n_kv_heads) * c.head_dim) + \
        c.n_heads * c.head_dim * c.d_model + c.d_model * 2 * c.ffn + c.ffn * c.d_model
    return 2.0 * P * c.n_layers * per_layer + 2.0 * c.vocab * c.d_model


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
    ap.add_argument("--ref-gen", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
