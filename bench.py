"""Benchmark of the packed prefill read path (the driver's contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dan|reference] [--config 3]

A step is one packed batch (<= 8192 tokens, drawn with configuration 3's
trunk / branch / label distributions) through the hot path: embedding, 32
Llama-3-8B layers (norm, qkv GEMM, RoPE, tree attention, o GEMM + residual,
norm, gate/up GEMM + SwiGLU, down GEMM + residual) and the fused label
readout. Weights are random N(0, 0.02) bf16 generated on the GPU; token ids
and lengths are seeded synthetic data (no dataset or checkpoint is used).

``value`` is prefill tokens/s over all ranks with the batch already resident
in HBM (device timing with CUDA events, max over ranks). ``e2e`` is the same
metric through the public API ``Runner.read_stream`` (``read_many`` per batch,
with the next batch packed while the device runs the current one) from host
plans: packing, pinned host->device upload of ids / positions / tables, the
forward, and the device->host copy of every question's logits and
probabilities, every step.
Each rank runs an independent replica on its own batches (weak scaling, no
collective on the data path).

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle port, fp32, all host threads) on the same configuration and metric:
each step is a bounded sample (a 1-layer slice of the model over one request,
scaled to 32 layers).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "prefill tokens/s & answers/s per B200 at Llama-3-8B bf16; attn TC % of peak"
WORKLOADS = {3: "cfg3: Llama-3-8B bf16 packed prefill + label readout, <=8192-token batches",
             4: "cfg4: Qwen3.5-4B-style hybrid bf16 (3 DeltaNet : 1 gated attention), <=8192-token batches",
             5: "cfg5: Llama-3-8B FP8 e4m3 + shared 1024-token prefix in the prefix pool, <=8192-token batches"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """Samples nvidia-smi every 200 ms while running (SM clock, max, throttle reasons)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=5)
        return False

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = [n for i, n in enumerate(names) if any(r[3 + i].lower() == "active" for r in self.rows)]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return world, rank, local


def reduce(value, op, world, device):
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.item()


def barrier(world, device):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index] if device.type == "cuda" else None)


# ---------------------------------------------------------------------- CPU arm
SAMPLE_LAYERS = 1
_cpu_state = {}


def cpu_sample(layers=SAMPLE_LAYERS, seed=0):
    """The oracle (fp32 CPU restatement of the reference) over a ``layers``-layer slice of
    Llama-3-8B on one configuration-3 request; returns (seconds, tokens, questions, threads)."""
    from dan_b200 import synthetic
    from dan_b200.loader import llama3_8b_config
    from oracle import llama as OL
    from oracle import runner as OR
    from oracle import weights as OW

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = dict(llama3_8b_config(), num_hidden_layers=layers, vocab_size=1024)
    if layers not in _cpu_state:
        _cpu_state[layers] = OW.random_state(cfg, 0)
    state = _cpu_state[layers]
    import random

    plan = synthetic.request(3, random.Random(seed), 1024)
    ids, pos, segs, reads, _ = OR.pack([plan])
    t0 = time.perf_counter()
    h = OL.hidden(state, cfg, ids, pos, segs)
    for r, labels in reads:
        OL.label_logits(state, h[r], labels)
    dt = time.perf_counter() - t0
    return dt, len(ids), len(reads), torch.get_num_threads()


def run_reference(args, world, rank):
    if rank != 0:
        return
    full_layers = 32
    vals, answers = [], []
    for step in range(args.warmup + args.steps):
        dt, tokens, questions, threads = cpu_sample(seed=step)
        scale = full_layers / SAMPLE_LAYERS
        if step >= args.warmup:
            vals.append(tokens / (dt * scale))
            answers.append(questions / (dt * scale))
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * tokens / v,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "answers_per_s": statistics.median(answers),
            "config": {"workload": "cfg3: Llama-3-8B packed prefill + label readout (1-layer slice x32, 1 request/step)",
                       "global_batch": tokens, "seq_len": tokens, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"oracle fp32, {SAMPLE_LAYERS} of 32 layers of Llama-3-8B over one "
                                       f"request ({tokens} tokens), time x{32 // SAMPLE_LAYERS}"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- GPU arm
def prepare(runner, plans, use_cache=False):
    """Pack and upload one batch (outside the timed region for ``value``)."""
    import numpy as np

    from dan_b200.attention import layout_of

    ids, pos, segs, reads, _ = runner.pack(plans, use_cache=use_cache)
    dev = runner.device
    labels = [list(l) for _, l in reads]
    off = np.zeros(len(labels) + 1, dtype=np.int32)
    off[1:] = np.cumsum([len(l) for l in labels])
    t = lambda xs, dt: torch.as_tensor(np.asarray(xs), dtype=dt).to(dev)
    b = {"ids": t(ids, torch.int64), "pos": t(pos, torch.int64), "segs": segs,
         "rows": t([r for r, _ in reads], torch.int32), "labels": t([x for l in labels for x in l], torch.int32),
         "off": t(off, torch.int32), "max_labels": max(len(l) for l in labels), "tokens": len(ids),
         "questions": len(reads)}
    layout_of(segs, len(ids), dev)
    return b


def step_device(model, b):
    x = model.hidden(b["ids"], b["pos"], b["segs"])
    return model.readout(x, b["rows"], b["labels"], b["off"], b["max_labels"])


def run_dan(args, world, rank, local):
    from dan_b200 import profiling, synthetic
    from dan_b200.loader import llama3_8b_config, random_model
    from dan_b200.runner import Runner

    from dan_b200.loader import qwen35_4b_config

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cid = args.config
    cfg = qwen35_4b_config() if cid == 4 else llama3_8b_config()
    quant = "fp8" if cid == 5 else None
    model = random_model(cfg, seed=0, device=device, quantization=quant)
    runner = Runner(model, device, cache_bytes=(4 << 30) if cid == 5 else 0)
    n = args.warmup + args.steps
    batches = synthetic.batches(cid, n + 1, seed=1000 + rank, vocab=cfg["vocab_size"])
    if cid == 5:  # the shared 1024-token prefix enters the prefix pool once, as in serving
        runner.read_many(batches[0][:1])
    batches = batches[1:]
    prepared = [prepare(runner, p, use_cache=(cid == 5)) for p in batches]
    torch.cuda.synchronize()

    for b in prepared[:args.warmup]:
        step_device(model, b)
    torch.cuda.synchronize()
    timed = prepared[args.warmup:]
    tokens = sum(b["tokens"] for b in timed)
    questions = sum(b["questions"] for b in timed)
    # requests and prompt tokens as dan's usage counts them (cached prefix tokens included,
    # engine.py:74-76), over the same timed batches
    requests = sum(len(p) for p in batches[args.warmup:])
    prompt_tokens = sum(len(pl.prefix) + sum(len(br.suffix) for br in pl.branches)
                        for p in batches[args.warmup:] for pl in p)
    pairs = sum(b["segs"].layout.pairs for b in timed)

    hbm, pk_burst, pk_sust, pk_kind = peaks()
    launches0 = profiling.total_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Per-launch events of the roofline kernels, created before the timed region: creating them
    # inside it cost ~1% (configuration 3) to ~3.5% (configuration 5) of the step; recording
    # pre-created ones ~0% / ~1.4%.
    timer = profiling.KernelTimer({"dan_gemm_bf16", "dan_gemm_bf16_rope", "dan_gemm_e4m3", "dan_gemm_e4m3_rope",
                                   "dan_tree_attention", "dan_gated_delta_scan"})
    timer.reserve(2 * 8 * cfg["num_hidden_layers"] * len(timed))
    with Clocks(local) as clocks:
        barrier(world, device)
        torch.cuda.synchronize()
        ev0.record()
        with timer:
            for b in timed:
                step_device(model, b)
        ev1.record()
        torch.cuda.synchronize()
        barrier(world, device)
    ms = ev0.elapsed_time(ev1)
    launches = profiling.total_launches() - launches0
    kern = timer.summary()
    kern["gemm"] = timer.total("gemm_")
    ms_max = reduce(ms, "max", world, device)
    tok_all = reduce(tokens, "sum", world, device)
    q_all = reduce(questions, "sum", world, device)
    req_all = reduce(requests, "sum", world, device)
    prompt_all = reduce(prompt_tokens, "sum", world, device)

    # end to end through the public API: host plans -> read_many -> host logits
    h2d = d2h = 0
    for plans in batches[args.warmup:]:
        ids, pos, segs, reads, _ = runner.pack(plans, use_cache=False)
        nl = sum(len(l) for _, l in reads)
        h2d += 8 * len(ids) * 2 + 4 * (len(reads) + nl + len(reads) + 1)
        h2d += 4 * 12 * sum(-(-(s.end - s.start) // 128) for s in segs) + 4 * len(ids) + 4
        d2h += 2 * 4 * nl
    for plans in batches[:1]:
        runner.read_many(plans)
    barrier(world, device)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record()
    for _ in runner.read_stream(batches[args.warmup:]):  # one batch queued while the next is packed
        pass
    e1.record()
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ms = reduce(max(e0.elapsed_time(e1), 1000 * t_wall), "max", world, device)

    if rank != 0:
        return
    g = kern.get("gemm", {})
    attn_kind = f"{pk_kind} burst"  # attention stays bf16 in every configuration
    if cid == 5:  # e4m3 GEMMs: the library's measured e4m3 burst rate is the denominator
        try:
            with open(os.path.join(ROOT, "profiles", "fp8_peak.md")) as f:
                for line in f:
                    if line.startswith("fp8_tflops_burst:"):
                        pk_sust = float(line.split(":")[1])
                        pk_kind = "measured fp8 (torch._scaled_mm burst, profiles/fp8_peak.md)"
        except (OSError, ValueError):
            pass
    a = kern.get("dan_tree_attention", {})
    gemm_tflops = g["work_total"] / (g["ms_total"] * 1e-3) / 1e12 if g and g["ms_total"] else None
    attn_tflops = a["work_total"] / (a["ms_total"] * 1e-3) / 1e12 if a and a["ms_total"] else None
    traffic = None  # DRAM bytes per GEMM launch from the committed ncu summary (configuration 3)
    try:
        with open(os.path.join(ROOT, "profiles", "gemm_bf16_cfg3_shapes.md")) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:") and cid == 3:
                    traffic = int(line.split(":")[1])
    except (OSError, ValueError):
        pass
    line = {
        "metric": METRIC, "value": tok_all / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3" if cid == 5 else "bf16", "data": "synthetic",
        "answers_per_s": q_all / (ms_max * 1e-3),
        "requests_per_s": req_all / (ms_max * 1e-3),
        "prompt_tokens_per_s": prompt_all / (ms_max * 1e-3),
        "config": {"workload": WORKLOADS[cid], "model": "qwen3.5-4b-style (random init)" if cid == 4 else
                   "llama-3-8b (random init)", "global_batch": int(tok_all / args.steps),
                   "seq_len": 8192, "parallelism": f"replicas x{world}",
                   "l2": "weights (15 GB) streamed every step exceed the 126 MB L2"},
        "roofline": {"bound": "tensor", "kernel": f"dan_gemm_{'e4m3' if cid == 5 else 'bf16'} (all decoder projections)",
                     "achieved": gemm_tflops,
                     "peak": pk_sust, "unit": "TFLOP/s", "frac": gemm_tflops / pk_sust if gemm_tflops else None,
                     "peak_kind": pk_kind if cid == 5 else f"{pk_kind} sustained (kernel timed inside a long step)",
                     "traffic": traffic, "share_of_step": g.get("ms_total", 0) / ms if g else None},
        "roofline_attention": {"bound": "tensor", "kernel": "dan_tree_attention", "achieved": attn_tflops,
                               "peak": pk_burst, "unit": "TFLOP/s",
                               "frac": attn_tflops / pk_burst if attn_tflops else None,
                               "peak_kind": attn_kind, "useful_pairs_per_step": pairs / args.steps,
                               "share_of_step": a.get("ms_total", 0) / ms if a else None},
        "e2e": {"value": tok_all / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        "gpu_launches": launches,
        "kernels": {k: {"launches": v["launches"], "ms_per_step": v["ms_total"] / args.steps,
                        ("gbs" if k == "dan_gated_delta_scan" else "tflops"):
                            v["work_total"] / max(v["ms_total"], 1e-9) / (1e6 if k == "dan_gated_delta_scan" else 1e9)}
                    for k, v in kern.items() if v["launches"]},
        "clocks": clocks.summary(),
    }
    sc = kern.get("dan_gated_delta_scan")
    if sc and sc["ms_total"]:  # configuration 4: the recurrent scan, HBM-bound by definition
        n_lin = sum(1 for t in cfg.get("layer_types", []) if t == "linear_attention")
        flops = tokens * n_lin * 4 * cfg["linear_num_value_heads"] * cfg["linear_key_head_dim"] * \
            cfg["linear_value_head_dim"]
        gbs = sc["work_total"] / (sc["ms_total"] * 1e-3) / 1e9
        line["roofline_scan"] = {"bound": "hbm", "kernel": "dan_gated_delta_scan", "achieved": gbs, "peak": hbm,
                                 "unit": "GB/s", "frac": gbs / hbm if hbm else None, "peak_kind": "measured",
                                 "tflops": flops / (sc["ms_total"] * 1e-3) / 1e12,
                                 "share_of_step": sc["ms_total"] / ms}
    if world == 1 and not args.no_cpu and cid == 3:
        dt, ctok, cq, threads = cpu_sample()
        v = ctok / (dt * 32 / SAMPLE_LAYERS)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"oracle fp32, {SAMPLE_LAYERS} of 32 layers of Llama-3-8B over one "
                                          f"request ({ctok} tokens), time x{32 // SAMPLE_LAYERS}"}
    print(json.dumps(line), flush=True)
    if args.breakdown:  # every entry point over the same batches again, to stderr
        full = profiling.KernelTimer().reserve(2 * 16 * cfg["num_hidden_layers"] * len(timed))
        with full:
            for b in timed:
                step_device(model, b)
        rows = sorted(full.summary().items(), key=lambda kv: -kv[1]["ms_total"])
        total = sum(v["ms_total"] for _, v in rows)
        n = len(timed)
        print(f"# configuration {cid}: device time per entry point over {n} steps (CUDA events around each "
              f"launch; sum {total / n:.3f} ms/step)", file=sys.stderr)
        for k, v in rows:
            print(f"#   {k:44s} {v['launches'] / n:6.1f}/step {v['ms_total'] / n:8.3f} ms/step "
                  f"{1000 * v['ms_total'] / max(v['launches'], 1):9.1f} us/launch {100 * v['ms_total'] / total:5.1f}%",
                  file=sys.stderr)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="dan", choices=["dan", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--breakdown", action="store_true",
                    help="after the JSON line, time every kernel entry point over the timed batches (stderr)")
    ap.add_argument("--config", type=int, default=3, choices=[3, 4, 5],
                    help="3 (default): Llama-3-8B bf16; 4: Qwen3.5-4B-style hybrid; 5: Llama-3-8B FP8 + prefix pool")
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_dan(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
