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

All ranks draw one seeded stream of batches and deal them so each rank times
``steps`` batches with near-equal token totals; ``per_rank`` lists every
rank's tokens and device time. ``attention_cfg2`` times the tree-attention
kernel alone on a configuration-2 batch, before the warm-up steps (at the
unthrottled clock, as the burst peak is measured; the SM clock read before
and after it is reported); ``cpu_baseline`` is dan's own CPU
path on one of the timed batches (configuration 3, one GPU).

``--impl reference`` runs dan itself: its unmodified ``Runner`` (fp32, all
host threads, dense masked attention) from the offline install under
baseline/_ref, on the same configuration-3 batches and metric. Each step reads
one whole batch through a 1-layer Llama-3-8B-shaped checkpoint (full vocab);
``ms_per_step`` is that measured time, and ``value`` counts the other 31
layers at the hook-timed time of the one layer.
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


# ---------------------------------------------------------------------- reference arm
# dan itself (its unmodified ``dan.runner.Runner``, fp32 on the host cores: the dense masked
# attention path, attention.py:244-270) from the offline install under baseline/_ref.
REF_SITE = os.path.join(ROOT, "baseline", "_ref")
REF_LAYERS = 1  # decoder layers in the reference's checkpoint; the other 31 are counted from its time
FULL_LAYERS = 32


def dan_reference():
    """(dan.runner, None) from the offline install of the reference, or (None, why not)."""
    if os.path.isdir(os.path.join(REF_SITE, "dan")) and REF_SITE not in sys.path:
        sys.path.append(REF_SITE)
    try:
        import dan.runner as ref_runner
    except Exception as e:  # noqa: BLE001 - any import failure makes the arm unavailable
        return None, f"dan is not importable from baseline/_ref ({type(e).__name__}: {e})"
    return ref_runner, None


def reference_checkpoint(path, layers=REF_LAYERS, seed=0):
    """A Llama-3-8B-shaped Hugging Face checkpoint with ``layers`` decoder layers and the full
    128,256-token vocabulary, weights bf16 N(0, 0.02), seeded. The vocabulary matrix repeats one
    seeded 8192-row block and lm_head is tied to it: writing and loading 2 x 1 GB of vocabulary
    rows took most of a minute on a host, and the forward reads only the embedding rows of the
    batch's tokens and the label rows, the same work tied or untied."""
    from safetensors.torch import save_file

    from dan_b200.loader import llama3_8b_config

    cfg = dict(llama3_8b_config(), num_hidden_layers=layers, architectures=["LlamaForCausalLM"],
               tie_word_embeddings=True, torch_dtype="bfloat16", max_position_embeddings=131072,
               hidden_act="silu", attention_bias=False, mlp_bias=False)
    gen = torch.Generator().manual_seed(seed)
    hd, inter, vocab = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    q, kv = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]

    def w(rows, cols):
        return (torch.randn(rows, cols, generator=gen) * 0.02).bfloat16()

    def vocab_rows():
        blk = w(8192, hd)
        return blk.repeat(-(-vocab // 8192), 1)[:vocab].contiguous()

    state = {"model.embed_tokens.weight": vocab_rows(),
             "model.norm.weight": (1 + 0.1 * torch.randn(hd, generator=gen)).bfloat16()}
    for i in range(layers):
        p = f"model.layers.{i}."
        state.update({p + "input_layernorm.weight": (1 + 0.1 * torch.randn(hd, generator=gen)).bfloat16(),
                      p + "post_attention_layernorm.weight": (1 + 0.1 * torch.randn(hd, generator=gen)).bfloat16(),
                      p + "self_attn.q_proj.weight": w(q, hd), p + "self_attn.k_proj.weight": w(kv, hd),
                      p + "self_attn.v_proj.weight": w(kv, hd), p + "self_attn.o_proj.weight": w(hd, q),
                      p + "mlp.gate_proj.weight": w(inter, hd), p + "mlp.up_proj.weight": w(inter, hd),
                      p + "mlp.down_proj.weight": w(hd, inter)})
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    save_file(state, os.path.join(path, "model.safetensors"))
    return cfg


class ReferenceRun:
    """dan's ``Runner`` (fp32, CPU, all host threads) on a ``REF_LAYERS``-layer Llama-3-8B-shaped
    checkpoint. ``step(plans)`` reads one packed batch through ``Runner.read_many`` and returns
    (measured seconds, seconds scaled to 32 layers): the decoder layer is timed by forward hooks
    (pre / post on ``model.model.layers[0]``) and the other 31 layers are counted at its time;
    embedding, final norm, label logits and packing are measured once, as they run."""

    def __init__(self, ref_runner):
        import tempfile

        torch.set_num_threads(os.cpu_count() or 1)
        self.threads = torch.get_num_threads()
        shm = "/dev/shm" if os.path.isdir("/dev/shm") and os.access("/dev/shm", os.W_OK) else None
        with tempfile.TemporaryDirectory(dir=shm) as tmp:
            reference_checkpoint(tmp)
            self.runner = ref_runner.Runner(tmp, device="cpu", dtype=torch.float32, cache_bytes=0)
        self.layer_s = []
        layer = self.runner.model.model.layers[0]
        layer.register_forward_pre_hook(lambda m, a: self.layer_s.append(-time.perf_counter()))
        layer.register_forward_hook(lambda m, a, o: self.layer_s.append(self.layer_s.pop() + time.perf_counter()))

    def step(self, plans):
        self.layer_s.clear()
        t0 = time.perf_counter()
        self.runner.read_many(plans)
        dt = time.perf_counter() - t0
        layers = sum(self.layer_s)
        return dt, dt + (FULL_LAYERS / REF_LAYERS - 1) * layers


def plan_tokens(plans):
    return sum(len(p.prefix) + sum(len(b.suffix) for b in p.branches) for p in plans)


def run_reference(args, world, rank):
    if rank != 0:
        return
    from dan_b200 import synthetic

    ref_runner, why = dan_reference()
    if ref_runner is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    ref = ReferenceRun(ref_runner)
    # the GPU arm's batches (rank 0's stream): warm-up batches first, then the timed ones
    batches = synthetic.batches(3, args.warmup + args.steps + 1, seed=1000, vocab=128256)[1:]
    measured, scaled, tokens, questions = [], [], 0, 0
    for i, plans in enumerate(batches):
        dt, full = ref.step(plans)
        if i >= args.warmup:
            measured.append(dt)
            scaled.append(full)
            tokens += plan_tokens(plans)
            questions += sum(len(p.branches) for p in plans)
    v = tokens / sum(scaled)
    sample = (f"dan.runner.Runner (unmodified, fp32 CPU, dense masked attention) on a {REF_LAYERS}-layer "
              f"Llama-3-8B-shaped checkpoint (vocab 128256, tied) over the GPU arm's configuration-3 batches; "
              f"the layer's hook-timed seconds counted x{FULL_LAYERS // REF_LAYERS}")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(measured) / len(measured),
            "ms_per_step_32_layers": 1000.0 * sum(scaled) / len(scaled),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "answers_per_s": questions / sum(scaled),
            "config": {"workload": WORKLOADS[3] + f" (dan's CPU path; {REF_LAYERS}-layer slice timed per step, "
                                                  f"value counts 32 layers from the slice's layer time)",
                       "global_batch": tokens // len(measured), "seq_len": 8192, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
                             "sample": sample},
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
    x = model.residual(b["ids"], b["pos"], b["segs"])
    return model.readout(x, b["rows"], b["labels"], b["off"], b["max_labels"])


def deal(batches, world, steps):
    """Deal ``world * steps`` batches so every rank gets ``steps`` of them with token totals as
    even as possible: largest first, each to the rank with the fewest tokens among those with
    room (the engine's least-loaded dispatch). Each rank keeps its batches in draw order; with
    one rank this is the batches as drawn."""
    cost = [plan_tokens(p) for p in batches]
    load, got = [0] * world, [[] for _ in range(world)]
    for i in sorted(range(len(batches)), key=lambda i: -cost[i]):
        r = min((r for r in range(world) if len(got[r]) < steps), key=lambda r: (load[r], r))
        got[r].append(i)
        load[r] += cost[i]
    return [[batches[i] for i in sorted(g)] for g in got]


def per_rank(values, world, rank, device):
    """Every rank's ``values`` (a list of floats), gathered by one all-reduce: [world][len]."""
    if world == 1:
        return [list(values)]
    import torch.distributed as dist

    t = torch.zeros(world, len(values), dtype=torch.float64, device=device)
    t[rank] = torch.tensor(values, dtype=torch.float64)
    dist.all_reduce(t)
    return t.tolist()


def flush_l2(buf):
    buf.add_(1)  # writes 256 MB: more than the 126 MB L2


def sm_clock_mhz(index):
    """The GPU's current SM clock by one NVML query (a read; nothing is set), or None."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            return pynvml.nvmlDeviceGetClockInfo(pynvml.nvmlDeviceGetHandleByIndex(index), pynvml.NVML_CLOCK_SM)
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # no NVML on this host
        return None


def attention_cfg2(device, hbm_peak, burst_peak, iters=10, seed=0):
    """dan_tree_attention alone on one configuration-2 batch (<= 8192 tokens, Llama-3-8B heads
    32 / 8 x 128, q / k / v ~ N(0, 1) bf16), timed per launch with CUDA events around the launch
    and L2 flushed between launches. Useful work counts only the (query, key) pairs the tree mask
    allows; the tile table's computed area (key blocks visited x 128 x 128) is reported beside it."""
    from dan_b200 import synthetic
    from dan_b200.attention import TreeLayout, tree_attention
    from dan_b200.runner import Runner

    r = Runner.__new__(Runner)
    r.device, r.cache = device, None
    ids, pos, segs, reads, _ = r.pack(synthetic.batch(2, seed=seed, vocab=128256), use_cache=False)
    n, h, hkv, d = len(ids), 32, 8, 128
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(n, h, d, device=device, generator=g).bfloat16()
    k = torch.randn(n, hkv, d, device=device, generator=g).bfloat16()
    v = torch.randn(n, hkv, d, device=device, generator=g).bfloat16()
    out = torch.empty_like(q)
    lay = TreeLayout.build(segs, n, device)
    buf = torch.empty(64 << 20, dtype=torch.float32, device=device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters + 3)]
    torch.cuda.synchronize()
    mhz_before = sm_clock_mhz(device.index or 0)
    for s, e in ev:
        flush_l2(buf)
        s.record()
        tree_attention(q, k, v, lay, out=out)
        e.record()
    torch.cuda.synchronize()
    mhz_after = sm_clock_mhz(device.index or 0)
    ms = [s.elapsed_time(e) for s, e in ev[3:]]
    med = statistics.median(ms)
    tflops = 4 * h * d * lay.pairs / (med * 1e-3) / 1e12
    computed = lay.blocks * 128 * 128
    return {"bound": "tensor", "kernel": "dan_tree_attention", "workload": "cfg2a: one <=8192-token batch "
            f"({n} tokens, {len(segs)} requests, {len(reads)} branches), 32/8 heads x 128, bf16",
            "achieved": tflops, "peak": burst_peak, "unit": "TFLOP/s", "frac": tflops / burst_peak,
            "peak_kind": "measured burst", "ms_median": med, "ms_min": min(ms), "launches": len(ms),
            "useful_pairs": lay.pairs, "computed_pairs": computed, "useful_frac_of_computed": lay.pairs / computed,
            "l2": "flushed (256 MB write) before every launch", "sm_mhz_before": mhz_before,
            "sm_mhz_after": mhz_after,
            "when": "before the warm-up steps, so at the unthrottled clock the burst peak is measured at"}


def fp8_library_peak(device, iters=5):
    """The FP8 denominator, measured in this run: torch._scaled_mm (cuBLASLt) e4m3 8192^3 with
    row-wise scales, bf16 out; the fastest of ``iters`` launches (burst), CUDA-event timed."""
    n = 8192
    a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    sa, sb = torch.ones(n, 1, device=device), torch.ones(1, n, device=device)
    best = None
    for i in range(iters + 2):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._scaled_mm(a, b.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
        e.record()
        e.synchronize()
        if i >= 2:
            best = s.elapsed_time(e) if best is None else min(best, s.elapsed_time(e))
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def cpu_baseline_sample(plans):
    """dan's own CPU path on one of the timed batches (the reference arm's measurement, bounded
    to one batch): its line's ``cpu_baseline``; None with the reason when dan is unavailable."""
    ref_runner, why = dan_reference()
    if ref_runner is None:
        return {"unavailable": why}
    ref = ReferenceRun(ref_runner)
    ref.step(plans)  # warm-up (thread pools, first-touch of the weights)
    dt, full = ref.step(plans)
    tokens = plan_tokens(plans)
    return {"value": tokens / full, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
            "sample": f"dan.runner.Runner (unmodified, fp32 CPU) on one timed batch ({tokens} tokens), "
                      f"{REF_LAYERS}-layer Llama-3-8B-shaped checkpoint, layer time counted "
                      f"x{FULL_LAYERS // REF_LAYERS}; measured {dt:.2f} s"}


def run_dan(args, world, rank, local):
    from dan_b200 import profiling, synthetic
    from dan_b200.loader import llama3_8b_config, qwen35_4b_config, random_model
    from dan_b200.runner import Runner

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cid = args.config
    cfg = qwen35_4b_config() if cid == 4 else llama3_8b_config()
    quant = "fp8" if cid == 5 else None
    model = random_model(cfg, seed=0, device=device, quantization=quant)
    runner = Runner(model, device, cache_bytes=(4 << 30) if cid == 5 else 0)
    # One seeded request stream for all ranks: batch 0 warms the prefix pool (configuration 5),
    # the next ``warmup`` batches are every rank's warm-up, and the following world x steps
    # batches are dealt so each rank times ``steps`` of them with near-equal token totals.
    drawn = synthetic.batches(cid, 1 + args.warmup + world * args.steps, seed=1000, vocab=cfg["vocab_size"])
    if cid == 5:  # the shared 1024-token prefix enters the prefix pool once, as in serving
        runner.read_many(drawn[0][:1])
    # the configuration-2 attention case runs first, before any step has heated the GPU: the
    # burst peak it is set against was measured the same way (a kernel alone, unthrottled)
    attn_case = None
    if rank == 0 and not args.no_attention_case:
        attn_case = attention_cfg2(device, *peaks()[:2])
    warm_plans = drawn[1:1 + args.warmup]
    timed_plans = deal(drawn[1 + args.warmup:], world, args.steps)[rank]
    use_cache = cid == 5
    warm = [prepare(runner, p, use_cache=use_cache) for p in warm_plans]
    timed = [prepare(runner, p, use_cache=use_cache) for p in timed_plans]
    torch.cuda.synchronize()

    for b in warm:
        step_device(model, b)
    torch.cuda.synchronize()
    tokens = sum(b["tokens"] for b in timed)
    questions = sum(b["questions"] for b in timed)
    # requests and prompt tokens as dan's usage counts them (cached prefix tokens included,
    # engine.py:74-76), over the same timed batches
    requests = sum(len(p) for p in timed_plans)
    prompt_tokens = sum(plan_tokens(p) for p in timed_plans)
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
    ranks = per_rank([tokens, ms, questions, requests, prompt_tokens], world, rank, device)
    ms_max = max(r[1] for r in ranks)
    tok_all, q_all, req_all, prompt_all = (sum(r[i] for r in ranks) for i in (0, 2, 3, 4))

    # end to end through the public API: host plans -> read_stream -> host logits
    h2d = d2h = 0
    for plans in timed_plans:
        ids, pos, segs, reads, _ = runner.pack(plans, use_cache=False)
        nl = sum(len(l) for _, l in reads)
        h2d += 8 * len(ids) * 2 + 4 * (len(reads) + nl + len(reads) + 1)
        h2d += 4 * 12 * sum(-(-(s.end - s.start) // 128) for s in segs) + 4 * len(ids) + 4
        d2h += 2 * 4 * nl
    runner.read_many(warm_plans[0] if warm_plans else timed_plans[0])
    barrier(world, device)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record()
    for _ in runner.read_stream(timed_plans):  # one batch queued while the next is packed
        pass
    e1.record()
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ranks = per_rank([max(e0.elapsed_time(e1), 1000 * t_wall)], world, rank, device)
    e2e_ms = max(r[0] for r in e2e_ranks)

    if rank != 0:
        return
    g = kern.get("gemm", {})
    gemm_peak, gemm_kind = pk_sust, f"{pk_kind} bf16 sustained (kernels timed inside a long step)"
    if cid == 5:  # e4m3 GEMMs: the library's e4m3 burst rate, measured now, is the denominator
        gemm_peak = fp8_library_peak(device)
        gemm_kind = "torch._scaled_mm e4m3 8192^3 burst, measured in this run"
    a = kern.get("dan_tree_attention", {})
    gemm_tflops = g["work_total"] / (g["ms_total"] * 1e-3) / 1e12 if g and g["ms_total"] else None
    attn_tflops = a["work_total"] / (a["ms_total"] * 1e-3) / 1e12 if a and a["ms_total"] else None
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
                   "batches": "one seeded stream; world x steps batches dealt largest-first to the least-loaded "
                              "rank, steps per rank",
                   "l2": "weights (15 GB) streamed every step exceed the 126 MB L2"},
        "per_rank": {"tokens": [int(r[0]) for r in ranks], "ms": [round(r[1], 3) for r in ranks],
                     "tokens_per_s": [r[0] / (r[1] * 1e-3) for r in ranks],
                     "e2e_ms": [round(r[0], 3) for r in e2e_ranks]},
        "roofline": {"bound": "tensor", "kernel": f"dan_gemm_{'e4m3' if cid == 5 else 'bf16'} (all decoder projections)",
                     "achieved": gemm_tflops, "peak": gemm_peak, "unit": "TFLOP/s",
                     "frac": gemm_tflops / gemm_peak if gemm_tflops else None, "peak_kind": gemm_kind,
                     "traffic": None, "share_of_step": g.get("ms_total", 0) / ms if g else None},
        "roofline_attention": {"bound": "tensor", "kernel": "dan_tree_attention", "achieved": attn_tflops,
                               "peak": pk_sust, "unit": "TFLOP/s",
                               "frac": attn_tflops / pk_sust if attn_tflops else None,
                               "peak_kind": f"{pk_kind} bf16 sustained (kernels timed inside a long step)",
                               "frac_of_burst": attn_tflops / pk_burst if attn_tflops else None,
                               "burst_peak": pk_burst, "useful_pairs_per_step": pairs / args.steps,
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
    if attn_case is not None:
        line["attention_cfg2"] = attn_case
    if world == 1 and not args.no_cpu and cid == 3:
        line["cpu_baseline"] = cpu_baseline_sample(timed_plans[0])
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
    ap.add_argument("--no-attention-case", action="store_true", help="skip the configuration-2 attention timing")
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
