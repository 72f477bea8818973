"""Benchmark: batch-1 decode tokens/s of Gemma3-1B and achieved HBM GB/s.

Workload (one "step"): with a 512-token random prompt already in the KV
cache, decode 256 tokens at batch 1 with temperature 0.7 / top-k 64, each
drawn on the device and fed back (positions 512..767).  Weights are seeded
random-init (N(0, 0.02)) in the reference dtype (fp32); no checkpoint or
dataset is reachable offline, so the data is synthetic.

value: decode tokens/s with everything resident in HBM (CUDA events on the
model's stream around K steps, max over ranks).  e2e: the same decode through
the C ABI call a plugin makes per token (mg_step with a host token id in and
the sampled host id out).  roofline: algorithmic bytes of one decode-kernel
launch (weights + KV read/write + logits write) / its average duration,
against the measured HBM copy bandwidth.  cpu_baseline: the oracle (C port of
the reference engine, 1 thread like the reference) on a bounded sample.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG = "gemma3-1b"
PROMPT = 512
DECODE = 256
TEMPERATURE, TOP_K, TOP_P = 0.7, 64, 1.0
METRIC = "batch-1 decode tokens/s (Gemma3-1B) and achieved HBM GB/s vs 8 TB/s peak"
UNIT = "tokens/s"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int) -> None:
        self.gpu = gpu
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def algorithmic_bytes(info, pos0: int, n: int, rows: int = 1, bf16_copies: bool = False) -> float:
    """Average bytes one decode step (of one rank) must move for positions pos0..pos0+n-1 of `rows` rows.

    The weights count once per step whatever the number of row groups.  On the batched tensor-core path
    (`bf16_copies`) the step streams bf16 copies of the weights and writes and reads back [rows, vocab]
    logits."""
    tp = max(1, int(info.tp_size))
    kv_heads = info.num_kv_heads // tp if info.num_kv_heads % tp == 0 else 1  # this rank's kv heads
    kv_row = 2 * kv_heads * info.head_dim * 4  # K+V fp32, one layer, one position
    ctx_avg = pos0 + (n + 1) / 2.0
    kv_read = info.num_layers * kv_row * ctx_avg
    kv_write = info.num_layers * kv_row
    logits = info.vocab_size // tp * 4
    emb_row = info.hidden_size * (4 if info.weight_dtype == 0 else 2)
    weights = float(info.weight_bytes_per_step)
    if bf16_copies:
        weights = weights / (4 if info.weight_dtype == 0 else 2) * 2
        logits *= 2
    return weights + rows * (kv_read + kv_write + logits + emb_row)


# DRAM bytes (read + write) per decode launch over its algorithmic bytes, from
# one ncu capture of this kernel on the Gemma3-270M shape (the full Gemma3-1B
# workload is too large to capture).  Traffic is almost all weight reads, so
# it scales with the algorithmic bytes.
TRAFFIC_RATIO = {("gemma3-1b", "f32"): 1.0046, ("gemma3-270m", "f32"): 1.0046}


def cpu_baseline(weights: dict, threads: int, n_tokens: int) -> dict:
    """Oracle port on the host: n_tokens decode steps from an empty cache."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # noqa: PLC0415

    oracle.set_threads(threads)
    ref = oracle.RefModel(weights, max_seq_len=PROMPT + DECODE)
    toks = [int(t) for t in np.random.default_rng(1).integers(0, 262144, n_tokens)]
    ref.step(toks[0])  # warm the caches
    t0 = time.perf_counter()
    for t in toks[1:]:
        ref.step(t)
    dt = time.perf_counter() - t0
    oracle.set_threads(1)
    ref.close()
    return {"value": (n_tokens - 1) / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_tokens - 1} Gemma3-1B decode steps (fp32, full 262144-vocab lm_head) from an empty cache "
                      f"on {threads} host thread(s); attention is <2% of bytes per token at pos<=768"}


def run_prefill(args, world: int, rank: int, local: int) -> None:
    """Prompt tokens/s of the batched prefill (tcgen05 GEMMs), with the
    token-at-a-time path (the reference's arithmetic) timed beside it."""
    import torch  # noqa: PLC0415

    from mogemma_b200 import _core, synth  # noqa: PLC0415

    d = synth.CONFIGS[CONFIG]
    weights = synth.make_weights(d, seed=0, bf16=args.weight_dtype == "bf16")
    meta = synth.metadata_of(weights)
    prompt = [int(t) for t in synth.prompt_ids(PROMPT, d.vocab, seed=1)]

    def timed(llm, reps: int) -> float:
        h = llm["_handle"]
        stream = torch.cuda.ExternalStream(h.stream, device=torch.device("cuda", local))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(reps):
            h.set_pos(0)
            llm["pos"] = 0
            _core.prefill(llm, prompt)
        ev1.record(stream)
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1) / reps

    llm = _core.init_model(meta, device=local, capacity=PROMPT + 8, weight_dtype=args.weight_dtype, prefill_path=1)
    for _ in range(args.warmup):
        timed(llm, 1)
    ms = timed(llm, args.steps)
    info = llm["_handle"].info
    llm["_handle"].close()
    base = _core.init_model(meta, device=local, capacity=PROMPT + 8, weight_dtype=args.weight_dtype, prefill_path=0)
    ms_tok = timed(base, 1)
    base["_handle"].close()
    params = info.weight_bytes_per_step / (2 if args.weight_dtype == "bf16" else 4) - d.vocab * d.hidden
    flops = 2.0 * params * PROMPT  # projections; attention adds 4 L Hq hd sum(ctx), small at this length
    pk = peaks()
    tf = flops / (ms / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({
            "metric": f"prefill tokens/s ({CONFIG}, {PROMPT}-token prompt)", "value": PROMPT / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (tcgen05, fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) random-init weights, uniform random prompt ids)",
            "config": {"workload": f"{CONFIG} batched prefill of {PROMPT} tokens, batch 1, "
                                   f"{args.weight_dtype} weights (bf16 copies for the tensor cores)"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": pk.get("bf16_tflops", 1590.0), "unit": "TFLOP/s",
                         "frac": tf / pk.get("bf16_tflops", 1590.0), "flops_per_step": flops},
            "token_at_a_time_ms": ms_tok,
        }), flush=True)


EMBED_BATCH, EMBED_LEN, EMBED_DENSE = 256, (16, 512), 3072


NANO_VOCAB = 32768  # the 262k-row per-layer table alone would be 8 GB of host and device memory


def run_nano(args, world: int, rank: int, local: int) -> None:
    """Gemma 3n decode tokens/s (mg_nano_*): a Gemma 3n E2B-like shape (hidden 2048, 30 layers, 8/2 heads of
    256, FFN 8192, per-layer dim 256, Laurel rank 64, 4 AltUp streams, KV sharing from layer 20) with a
    32,768-token vocabulary; fp32 weights tiled from one seeded random block (throughput does not depend on
    the values).  --prompt tokens are prefilled, then --decode steps each return fp32 logits to the host (the
    reference's step contract) and are timed by the host clock; every step synchronises.  Replicas for N > 1."""
    from mogemma_b200 import _core, synth  # noqa: PLC0415

    d = synth.NanoDims("gemma3n-e2b-shape", 2048, 30, 8, 2, 256, 8192, 256, 64, 4, NANO_VOCAB, kv_share_start=20)
    block = (np.random.default_rng(0).standard_normal(1 << 20).astype(np.float32) * np.float32(0.02))
    weights: dict[str, np.ndarray] = {}
    for name, shape in synth.nano_tensor_shapes(d).items():
        a = np.resize(block, shape)
        if name.endswith("norm.weight") or name.endswith("output_scale"):
            a = a + np.float32(1.0)
        layer = int(name.split(".")[2]) if name.startswith("model.layers.") else -1
        if layer >= 20 and (name.endswith("k_proj.weight") or name.endswith("v_proj.weight")):
            a = np.zeros(shape, np.float32)
        weights[name] = np.ascontiguousarray(a, np.float32)
    weights["lm_head.weight"] = weights["model.embed_tokens.weight"]
    # bytes one step reads: every tensor, except one row of the embedding and of the per-layer table, and no
    # k/v projections of the layers that share an earlier layer's cache
    step_bytes = 0
    for name, a in weights.items():
        if name == "model.embed_tokens.weight":
            step_bytes += d.hidden * 4
        elif name == "model.per_layer_embed.weight":
            step_bytes += d.layers * d.per_layer_dim * 4
        elif not ((name.endswith("k_proj.weight") or name.endswith("v_proj.weight")) and not a.any()):
            step_bytes += a.nbytes
    llm = _core.init_model(synth.metadata_of(weights), device=local, capacity=PROMPT + DECODE)
    prompt = [int(t) for t in synth.prompt_ids(PROMPT, d.vocab, seed=1)]

    def run() -> float:
        llm["pos"] = 0
        _core.prefill(llm, prompt[:-1])
        cur = prompt[-1]
        t0 = time.perf_counter()
        for _ in range(DECODE):
            logits = _core.step(llm, cur, 0.0, 0, 1.0)
            cur = int(np.argmax(logits))
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        run()
    barrier(world)
    with ClockSampler(local) as clocks:
        dt = min(run() for _ in range(args.steps))
    dt = dist_max(dt, world)
    ms_tok = dt * 1e3 / DECODE
    achieved = step_bytes / (ms_tok / 1e3) / 1e9
    pk = peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "Gemma 3n decode tokens/s (E2B-like shape, 32k vocabulary)", "value": world * DECODE / dt,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (weights tiled from one seeded N(0,0.02) block; random prompt ids)",
            "config": {"workload": f"gemma3n E2B-like shape, {PROMPT}-token prompt then {DECODE} greedy tokens, "
                                   "logits to the host every step (host clock)",
                       "model": d.name, "global_batch": world, "seq_len": PROMPT + DECODE,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "e2e": {"value": world * DECODE / dt, "unit": "tokens/s", "h2d_bytes_per_step": 8 * DECODE,
                    "d2h_bytes_per_step": 4 * d.vocab * DECODE},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "traffic": None, "peak_source": pk["source"],
                         "kernel": "nano step graph (one warp per GEMV row, single-CTA norms and AltUp)",
                         "algorithmic_bytes_per_launch": step_bytes},
            "cpu_baseline": None, "clocks": clocks.summary(),
            "gpu_launches": DECODE * args.steps, "ms_per_token": ms_tok}), flush=True)
    llm["_handle"].close()


def run_embed(args, world: int, rank: int, local: int) -> None:
    """Sequences/s of the bidirectional encoder (mg_encode): EmbeddingGemma-style
    shape, 256 sequences with lengths uniform in [16, 512], dense 768->3072->768
    head, L2-normalised rows.  Every N>1 rank encodes its own 256 sequences."""
    import torch  # noqa: PLC0415

    from mogemma_b200 import _core, synth  # noqa: PLC0415

    d = synth.CONFIGS["embedding-300m"]
    weights = synth.make_weights(d, seed=0)
    rng = np.random.default_rng(7)
    weights["embed_head.dense0.weight"] = (rng.standard_normal((EMBED_DENSE, d.hidden)) * 0.02).astype(np.float32)
    weights["embed_head.dense1.weight"] = (rng.standard_normal((d.hidden, EMBED_DENSE)) * 0.02).astype(np.float32)
    nseq = args.embed_batch
    lens = rng.integers(EMBED_LEN[0], EMBED_LEN[1] + 1, EMBED_BATCH)[:nseq]
    max_len = int(lens.max())
    ids = np.zeros((nseq, max_len), np.int32)
    for b, n in enumerate(lens):
        ids[b, :n] = synth.prompt_ids(int(n), d.vocab, seed=100 + b)
    lens32 = lens.astype(np.int32)
    out = np.zeros((nseq, d.hidden), np.float32)
    rows = 64  # sequences per group (the model's max_batch)
    llm = _core.init_model(synth.metadata_of(weights), device=local, capacity=EMBED_LEN[1], max_batch=rows,
                           prefill_path=1, mode="gemma3", sliding_window=d.window)
    h = llm["_handle"]
    lib = _core.lib()

    def step() -> None:
        _core._check(lib.mg_encode(h.ptr, ids.ctypes.data_as(_core._I32P), lens32.ctypes.data_as(_core._I32P),
                                   nseq, max_len, out.ctypes.data_as(_core._F32P)))

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.ExternalStream(h.stream, device=torch.device("cuda", local))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        barrier(world)
    ms = dist_max(ev0.elapsed_time(ev1), world) / args.steps
    wall = dist_max(wall, world) / args.steps
    tokens = int(lens.sum())
    # tensor-core work: the projections of every token; attention (CUDA cores) and the head are listed apart
    proj_params = d.layers * d.hidden * ((d.heads + 2 * d.kv_heads) * d.head_dim + d.heads * d.head_dim
                                         + 3 * d.intermediate)
    gemm_flops = 2.0 * proj_params * tokens
    att_flops = 4.0 * d.layers * d.heads * d.head_dim * float((lens.astype(np.float64) ** 2).sum())
    pk = peaks()
    tf = gemm_flops / (ms / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle  # noqa: PLC0415

        ref = oracle.RefModel(weights, max_seq_len=EMBED_LEN[1], mode=1, sliding_window=d.window)
        sample = [ids[b, : lens[b]] for b in range(2)]
        t0 = time.perf_counter()
        for s in sample:
            ref.encode(s, weights["embed_head.dense0.weight"], weights["embed_head.dense1.weight"])
        dt = time.perf_counter() - t0
        ref.close()
        cpu = {"value": len(sample) / dt, "unit": "sequences/s", "cores": 1, "kind": "port",
               "sample": f"2 sequences of the batch ({int(lens[0])} and {int(lens[1])} tokens) through the oracle's "
                         "encoder on 1 host thread"}
    if rank == 0:
        print(json.dumps({
            "metric": "embedding encoder sequences/s (EmbeddingGemma-style 300M, 256 sequences, lengths U[16,512])",
            "value": world * nseq / (ms / 1e3), "unit": "sequences/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 (tcgen05, fp32 accumulate); attention and head fp32",
            "data": "synthetic (seeded N(0,0.02) random-init weights, uniform random ids and lengths)",
            "config": {"workload": f"embedding-300m encoder, {nseq} sequences ({tokens} tokens), lengths "
                                   f"U[{EMBED_LEN[0]},{EMBED_LEN[1]}], dense {d.hidden}->{EMBED_DENSE}->{d.hidden}, "
                                   f"groups of {rows} sequences", "model": "embedding-300m",
                       "global_batch": world * nseq, "seq_len": EMBED_LEN[1],
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "per-step activations and weights (>1.2 GB) larger than L2"},
            "e2e": {"value": world * nseq / wall, "unit": "sequences/s",
                    "h2d_bytes_per_step": 4 * (tokens * 4 + nseq * 2),
                    "d2h_bytes_per_step": 4 * nseq * d.hidden},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / pk["bf16_tflops"], "peak_source": pk["source"],
                         "kernel": "whole encoder step (projection GEMM FLOPs over the step time)",
                         "gemm_flops_per_step": gemm_flops, "attention_flops_per_step": att_flops,
                         "traffic": None},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            # per group: embedding + first norm; per layer q/k/v GEMM, QK-norm/RoPE, V transpose, attention,
            # o_proj GEMM, norm, gate/up GEMM (GeGLU fused), down GEMM, norm; head: 1/rms, pool, 2 dense, L2
            "gpu_launches": args.steps * ((nseq + rows - 1) // rows) * (2 + 9 * d.layers + 5),
        }), flush=True)
    h.close()
    if world > 1:
        import torch.distributed as dist  # noqa: PLC0415

        dist.destroy_process_group()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime  # noqa: PLC0415

        import torch  # noqa: PLC0415
        import torch.distributed as dist  # noqa: PLC0415

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch  # noqa: PLC0415
    import torch.distributed as dist  # noqa: PLC0415

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist  # noqa: PLC0415

        dist.barrier()


def run_reference(args, world: int, rank: int) -> None:
    """The reference's CPU engine (its C restatement in oracle/, all host threads)
    on the benchmark's workload: the 512-token prompt's first 511 tokens are
    prefilled once, untimed, then each step decodes a bounded sample of the
    benchmarked positions (511 onwards, continuing across steps)."""
    if rank != 0:
        return
    from mogemma_b200 import synth  # noqa: PLC0415

    threads = len(os.sched_getaffinity(0))
    d = synth.CONFIGS[CONFIG]
    w = synth.make_weights(d, seed=0)
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # noqa: PLC0415

    oracle.set_threads(threads)
    ref = oracle.RefModel(w, max_seq_len=PROMPT + DECODE)
    prompt = [int(t) for t in synth.prompt_ids(PROMPT, d.vocab, seed=1)]
    for t in prompt[:-1]:  # positions 0..PROMPT-2, outside the timed region
        ref.step_no_logits(t)
    per_step = 4
    rng = np.random.default_rng(3)
    state = {"pos": PROMPT - 1, "cur": prompt[-1]}

    def step() -> None:
        for _ in range(per_step):
            if state["pos"] >= PROMPT + DECODE:  # wrap to the first benchmarked position
                state["pos"] = PROMPT - 1
            ref.pos = state["pos"]
            lg = ref.step(state["cur"])  # logits to the host, then the reference's NumPy draw
            state["cur"] = oracle.sample_next_token(lg, temperature=TEMPERATURE, top_k=TOP_K, top_p=TOP_P,
                                                    u=float(rng.random()))
            state["pos"] += 1

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    n = args.steps * per_step
    v = n / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) random-init weights, uniform random prompt ids)",
        "config": bench_config(1, 1, False),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} decode steps per step at positions {PROMPT - 1}+ (511-token prompt "
                                   f"prefilled untimed) on {threads} host threads (OpenMP over output rows; "
                                   "per-row arithmetic identical to the single-threaded reference engine)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def metric_name(B: int, tp: int) -> str:
    """METRIC for the default workload; the same wording with the batch, model and TP degree otherwise."""
    m = METRIC if B == 1 else METRIC.replace("batch-1", f"batch-{B}")
    if CONFIG != "gemma3-1b":
        m = m.replace("Gemma3-1B", CONFIG.replace("gemma3", "Gemma3").replace("b", "B"))
    return m if tp <= 1 else m.replace(") and", f", tensor-parallel x{tp}) and")


def bench_config(world: int, B: int, tp: bool, weight_dtype: str = "f32") -> dict:
    """The workload description shared by the CUDA arm and the reference arm."""
    streams = 1 if tp else world
    return {"workload": f"{CONFIG} batch-{B} decode: {PROMPT}-token prompt then {DECODE} tokens "
                        f"(T={TEMPERATURE}, top-k {TOP_K}), {weight_dtype} weights",
            "model": CONFIG, "global_batch": streams * B, "seq_len": PROMPT + DECODE,
            "parallelism": (f"tp{world}" if tp else f"replicas x{world}") if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (the weights streamed every token exceed 126 MB)"}


def main() -> None:
    global CONFIG, PROMPT, DECODE  # noqa: PLW0603
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--weight-dtype", default="f32", choices=["f32", "bf16"])
    ap.add_argument("--cpu-sample", type=int, default=25)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", default=CONFIG, help="synthetic config (gemma3-270m for small profiling runs)")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens prefilled before the timed decode")
    ap.add_argument("--decode", type=int, default=DECODE, help="tokens decoded per step")
    ap.add_argument("--batch", type=int, default=1,
                    help="decode rows (beyond the rows one persistent launch holds: one launch per row group, "
                         "or the batched tensor-core steps with --batched-tc)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "embed", "nano"],
                    help="prefill: the batched tensor-core prefill of --prompt tokens; embed: the bidirectional "
                         "encoder on 256 sequences")
    ap.add_argument("--embed-batch", type=int, default=EMBED_BATCH,
                    help="embed: sequences per step (the workload is 256; fewer for small profiling captures)")
    ap.add_argument("--parallel", default="replicas", choices=["replicas", "tp"],
                    help="N>1: independent replicas (weak scaling) or one tensor-parallel model over the N GPUs")
    ap.add_argument("--device-weights", action="store_true",
                    help="generate the seeded random weights on each GPU (Gemma3-4B/27B: larger than host memory)")
    ap.add_argument("--mode", default="ref", choices=["ref", "gemma3"],
                    help="gemma3: sliding window on 5 of 6 layers and dual RoPE theta (the 4B/27B configurations)")
    ap.add_argument("--e2e-passes", type=int, default=10, help="decode passes timed end to end (at least)")
    ap.add_argument("--batched-tc", action="store_true",
                    help="prompt and more than 8 rows on the tensor-core path (bf16 weight copies)")
    args = ap.parse_args()
    CONFIG, PROMPT, DECODE = args.model, args.prompt, args.decode
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.workload == "prefill":
        run_prefill(args, world, rank, local)
        return
    if args.workload == "embed":
        run_embed(args, world, rank, local)
        return
    if args.workload == "nano":
        run_nano(args, world, rank, local)
        return

    import ctypes  # noqa: PLC0415

    import torch  # noqa: PLC0415

    from mogemma_b200 import _core, synth  # noqa: PLC0415

    d = synth.CONFIGS[CONFIG]
    tp = args.parallel == "tp" and world > 1
    B = args.batch
    # more rows than the persistent kernel holds: one launch per row group in fp32 (prefill_path 0), or with
    # --batched-tc the tensor-core path on bf16 weight copies (prefill_path 1)
    opts = dict(device=local, capacity=PROMPT + DECODE, max_batch=B, weight_dtype=args.weight_dtype,
                prefill_path=1 if args.batched_tc and not tp else 0)
    if args.device_weights:
        # seeded N(0, 0.02) weights generated on each device (models larger than host memory);
        # every rank generates the same full tensors and keeps its shard
        meta = {k: (0, v, "F32") for k, v in synth.tensor_shapes(d).items()}
        meta["lm_head.weight"] = (0, (d.vocab, d.hidden), "F32")
        opts.update(synthetic_std=0.02, synthetic_seed=1)
    else:
        weights = synth.make_weights(d, seed=0, bf16=args.weight_dtype == "bf16")
        meta = synth.metadata_of(weights)
    if args.mode == "gemma3":
        opts.update(mode="gemma3", sliding_window=d.window, global_every=6)
    if tp:  # every rank holds its shard; the same seed on every rank draws the same tokens
        llm = _core.init_model_tp(meta, seed=1234, **opts)
    else:
        llm = _core.init_model(meta, seed=1234 + rank, **opts)
    h = llm["_handle"]
    info = h.info
    lib = _core.lib()
    prompts = [[int(t) for t in synth.prompt_ids(PROMPT, d.vocab, seed=1 + b)] for b in range(B)]
    prompt = prompts[0]
    if B == 1:
        _core.prefill(llm, prompt[:-1])
    else:
        _core.prefill_rows(llm, [p[:-1] for p in prompts])
    s, _keep = _core._sampling(TEMPERATURE, TOP_K, TOP_P)
    first = np.array([p[-1] for p in prompts], np.int32)
    stream = torch.cuda.ExternalStream(h.stream, device=torch.device("cuda", local))

    def device_step() -> None:
        # positions 511.. : feed the last prompt token, then 255 sampled tokens (every row)
        _core._check(lib.mg_set_pos(h.ptr, -1, PROMPT - 1))
        _core._check(lib.mg_set_tokens(h.ptr, first.ctypes.data_as(_core._I32P), B))
        _core._check(lib.mg_generate(h.ptr, DECODE, B, ctypes.byref(s), None))

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        ev0.record(stream)
        for _ in range(args.steps):
            device_step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
    ms = ev0.elapsed_time(ev1)
    ms = dist_max(ms, world)
    streams = 1 if tp else world
    tokens = args.steps * DECODE * streams * B
    value = tokens / (ms / 1000.0)
    ms_launch = ms / (args.steps * DECODE)
    rows = h.rows_per_launch  # rows one decode launch holds (5 for Gemma3-1B fp32: the down_proj input stage)
    tc_path = B > rows and args.batched_tc and not tp
    groups = -(-B // rows)  # decode-kernel launches per token (equal groups of at most `rows`)
    bytes_launch = algorithmic_bytes(info, PROMPT - 1, DECODE, B, bf16_copies=tc_path)
    achieved = bytes_launch / (ms_launch / 1000.0) / 1e9
    pk = peaks()

    # e2e: per-token C-ABI call with host buffers (token id in, sampled id out)
    ids = np.zeros(B, np.int32)
    out = np.zeros(B, np.int32)
    idp, outp = ids.ctypes.data_as(_core._I32P), out.ctypes.data_as(_core._I32P)

    def e2e_step() -> None:
        _core._check(lib.mg_set_pos(h.ptr, -1, PROMPT - 1))
        ids[:] = first
        for _ in range(DECODE):
            _core._check(lib.mg_step(h.ptr, idp, B, None, outp, ctypes.byref(s)))
            ids[:] = out

    e2e_step()
    barrier(world)
    t0 = time.perf_counter()
    e2e_steps = max(args.e2e_passes, args.steps)
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = dist_max(time.perf_counter() - t0, world)
    e2e_value = e2e_steps * DECODE * streams * B / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.device_weights:
        cpu = cpu_baseline(weights, 1, args.cpu_sample)
    if rank == 0:
        line = {
            "metric": metric_name(B, world if tp else 1), "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            # more rows than the persistent kernel holds run the batched tensor-core path on bf16 weight copies
            "dtype": args.weight_dtype if not tc_path else "bf16 (tcgen05 on bf16 weight copies, fp32 accumulate)",
            "data": "synthetic (seeded N(0,0.02) random-init weights, uniform random prompt ids)",
            "config": bench_config(world, B, tp, args.weight_dtype),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4 * DECODE,
                    "d2h_bytes_per_step": 4 * DECODE},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"],
                         "traffic": (bytes_launch * TRAFFIC_RATIO[(CONFIG, args.weight_dtype)]
                                     if (CONFIG, args.weight_dtype) in TRAFFIC_RATIO and B <= rows else None),
                         "traffic_source": "ncu dram__bytes_read+write of a Gemma3-270M launch, scaled by bytes",
                         "peak_source": pk["source"],
                         "kernel": ("batched step: tcgen05 GEMMs + prefill kernels per layer, lm_head GEMM, sampler"
                                    if tc_path else "decode_kernel (one launch per token)" if B <= rows else
                                    f"decode_kernel ({groups} launches of up to {rows} rows per token)"),
                         "algorithmic_bytes_per_launch": bytes_launch},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * DECODE * (9 * d.layers + 4 if tc_path else groups),
            "rows_per_launch": rows,
            "ms_per_token": ms_launch,
        }
        print(json.dumps(line), flush=True)
    if tp:
        _core.close_tp(llm)
    else:
        h.close()
    if world > 1:
        import torch.distributed as dist  # noqa: PLC0415

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
