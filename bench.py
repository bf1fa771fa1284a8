#!/usr/bin/env python
"""Benchmark of the CUDA encoder forward on B200: sequences/sec of a ragged throughput run.

Workload (the configuration its "seqs/sec at 1/2/4/8 B200" metric is quoted
on): a multilingual MiniLM-L12 cross-encoder (XLM-R shape: 12 layers, hidden 384, 12 heads, FFN
1536, vocab 250002), random-init weights, f16, 1-logit rerank head, over 65,536 synthetic
query/passage pairs (query length U[4, 32], passage lognormal median 90 sigma 0.8, the pair with
its 4 specials <= 512 tokens). One step = one forward of every pair; the pairs are split across
the ranks (strong scaling, balanced by token count), no collective on the data path; the host
gathers the logits in input order.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--pairs P] [--impl reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)
  python bench.py --workload c2-512-bulk|c3-512-bulk   (sequence length 512 throughput, one GPU)
  python bench.py --workload c1|c2-128|c2-512|c3|c4    (ms/call, one GPU)

value: pairs/sec of the whole job with the packed inputs already resident in HBM, device time
(CUDA events on the library's stream) max over ranks. e2e: the same metric through the public
bulk API with host buffers every step (pinned H2D of the token ids, device-side word-row gather,
forward, D2H of the logits, gather of every rank's logits into input order on rank 0).
cpu_baseline: the C++ restatement of the reference's WASM-SIMD executor (oracle/) on a bounded
sample of the same pairs, B = 1 calls on the 512-token bucket plan (runIds). parity: the GPU's
logits of the sampled pairs against the oracle's; the run fails when they disagree.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from kleinhirn_b200.dp import OutputGather, chunk_size, shard_sequences  # noqa: E402

BUCKET = 512

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one GEMM launch on a 262,144-row
# chunk, mean of the four GEMM launches of a C5 layer (qkv 0.753 GB, FFN-in 0.951 GB, attnOut +
# LayerNorm 0.571 GB, FFN-out + LayerNorm 1.200 GB), from one ncu capture each (the LayerNorm
# launches captured on a 288,315-row chunk and scaled); every term is rows x a per-row byte
# count, so a launch over another chunk size scales with its rows.
GEMM_TRAFFIC_BYTES = 868.8e6
GEMM_TRAFFIC_ROWS = 262144
GEMM_TRAFFIC_SOURCE = "ncu, profiles/gemm_pair_c5.md and profiles/gemm_addln_c5.md"

# f16 parity of the C5 logits against the oracle (f32 on the same f16 weights): the reference's
# own gate is |run - f64| <= 3 * delta_sim, delta_sim the deviation of its f16 simulation of the
# engine (convert/k28_f16_sim.py:9-11); at full depth on this configuration delta_sim = 2.94e-4
# (tests/golden/depth_golden.json), so the bound is 8.8e-4; the oracle is within 1e-5 of f64.
C5_PARITY_ABS = 3 * 2.94e-4 + 1e-5
# N ranks against one: the same pairs packed with other neighbours round the online softmax in
# another order (f16 P), so equality holds to the f16 storage precision.
RANKS_VS_ONE = 2e-3

# throughput workloads: model, sequence lengths (None: the C5 pair distribution)
BULK_WORKLOADS = {
    "c5": ("mminilm-l12-xlmr", None, "pairs"),
    "c2-512-bulk": ("roberta-base", 512, "seqs"),
    "c3-512-bulk": ("deberta-v3-base", 512, "seqs"),
}
# BASELINE configs 1-4 as latency workloads: (configuration, sequence length or None, f16)
CONFIG_WORKLOADS = {
    "c1": ("minilm-l6", 128, False),
    "c2-128": ("roberta-base", 128, True),
    "c2-512": ("roberta-base", 512, True),
    "c3": ("deberta-v3-base", 512, True),
    "c4": ("modernbert-base", None, True),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--pairs", type=int, default=0,
                    help="sequences of a throughput workload (0: 65,536 for c5, 4,096 / 2,048 at L512)")
    ap.add_argument("--chunk-tokens", type=int, default=0,
                    help="packed rows per bulk chunk (0: even chunks of at most 1,048,576 rows)")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-out", default="", help="write the per-launch profile of one forward here")
    ap.add_argument("--workload", default="c5", choices=list(BULK_WORKLOADS) + list(CONFIG_WORKLOADS),
                    help="c5: the headline (BASELINE config 5); c2-512-bulk / c3-512-bulk: sequence length "
                         "512 throughput; c1-c4: ms/call (B = 1 plan calls) or seqs/s (c4) of BASELINE configs 1-4")
    return ap.parse_args()


def host_info(threads: int) -> dict:
    model = platform.processor() or "?"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count() or 1, "cpu_model": model, "threads": threads}


def read_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "tflops": d.get("bf16_tflops_sustained", 1400.0),
                "tflops_burst": d.get("bf16_tflops", 1590.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "tflops_burst": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                s, m = float(f[1]), float(f[2])
            except ValueError:
                continue
            sm.append(s)
            mx = max(mx, m)
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_inputs(name: str, length, count: int, seed: int):
    from kleinhirn_b200 import synthetic
    spec, head = synthetic.model(name)
    if length is None:
        lens = synthetic.seq_lengths(name, count, seed)
    else:
        lens = np.full(count, length, dtype=np.int32)
    ids = synthetic.token_ids(name, lens, seed)
    return spec, head, lens, ids


def model_flops(spec: dict, lens: np.ndarray) -> tuple[float, float]:
    """Algorithmic FLOPs (2 per MAC) of the encoder layers: (GEMM part, attention part). Per layer
    and sequence of n rows: 2 n (3H^2 + H^2) for qkv + attnOut, 4 n H I for the MLP (2 n 3 I H for
    GeGLU), 4 n k H for QK^T and PV over k = n keys (k = min(n, 2 window + 1) on windowed layers),
    and for DeBERTa 4 n P H for the c2p / p2c tables over P relative positions."""
    H, I, layers = spec["hidden"], spec["intermediate"], spec["layers"]
    n = lens.astype(np.float64)
    att = spec["attention"]
    mlp = 2 * n * 3 * I * H if spec.get("ffn", {}).get("kind") == "geglu" else 4 * n * H * I
    gemm = layers * (2 * n * 4 * H * H + mlp).sum()
    attn = 0.0
    for l in range(layers):
        k = n
        win = att.get("window")
        if win and l % win["globalEvery"] != 0:
            k = np.minimum(n, 2 * win["half"] + 1)
        attn += (4 * n * k * H).sum()
        if att["kind"] == "deberta-relative":
            attn += (4 * n * 2 * att["rel"]["buckets"] * H).sum()
    return float(gemm), float(attn)


def cpu_sample(spec, head, w16, ids_all, budget_s: float, threads: int, max_items: int | None = None) -> dict:
    """The oracle on host cores: B = 1 calls (runIds) on the 512-token bucket, f32 on the f16 weights'
    values, sequences in input order until the time budget is used (at least 4)."""
    from kleinhirn_b200.encoder import mask_and_types, word_rows
    from kleinhirn_b200.plan import build_plan
    from oracle import host
    w32 = {k: v.astype(np.float32) for k, v in w16.items()}
    plan = build_plan(spec, head, BUCKET, 1, 0, False)
    rt = host.Runtime(threads=threads)
    try:
        host.load_weights(rt, w32, [plan])
        p = rt.plan(plan)
        table = w32["embeddings.word.weight"]
        cols = plan["output"]["cols"]
        done, t0 = 0, time.perf_counter()
        outs = []
        limit = len(ids_all) if max_items is None else min(max_items, len(ids_all))
        while done < limit:
            ids = ids_all[done]
            inputs = [{"inputIds": list(ids)}]
            mask, types = mask_and_types(spec, inputs, BUCKET)
            p.upload(word_rows(table, inputs, BUCKET), mask, types)
            p.run(len(ids))
            outs.append(p.read_output()[:cols])
            done += 1
            if time.perf_counter() - t0 > budget_s and done >= 4:
                break
        dt = time.perf_counter() - t0
    finally:
        rt.close()
    return {"done": done, "seconds": dt, "outputs": np.array(outs)}


def parity_block(gpu: np.ndarray, cpu: np.ndarray, tol: float) -> dict:
    g = np.asarray(gpu, dtype=np.float64).reshape(len(gpu), -1)
    c = np.asarray(cpu, dtype=np.float64).reshape(len(cpu), -1)[:, :g.shape[1]]
    if g.shape[1] == 1:  # one logit per sequence: the cosine of the logit vector
        cos = float(g.ravel() @ c.ravel() / (np.linalg.norm(g) * np.linalg.norm(c) + 1e-30))
    else:
        cos = float(((g * c).sum(1) / (np.linalg.norm(g, axis=1) * np.linalg.norm(c, axis=1) + 1e-30)).min())
    err = float(np.abs(g - c).max())
    ok = cos >= 0.999 and err <= tol
    return {"n": int(len(g)), "against": "oracle (C++ restatement of the reference WASM executor, f32)",
            "cos_min": cos, "max_abs": err, "tol": tol, "pass": bool(ok)}


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's WASM executor with every host
    thread; each step is a bounded sample of the same workload (rank 0 only)."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    from kleinhirn_b200 import synthetic
    if args.workload not in BULK_WORKLOADS:
        args.workload = "c5"
    name, length, unit = BULK_WORKLOADS[args.workload]
    count = args.pairs or default_count(args.workload)
    spec, head, lens, ids_all = workload_inputs(name, length, count, args.seed)
    w16 = synthetic.to_f16(synthetic.random_weights(spec, head, seed=args.seed))
    threads = os.cpu_count() or 1
    budget = max(2.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    rates, secs, done = [], [], 0
    for step in range(args.warmup + args.steps):
        r = cpu_sample(spec, head, w16, ids_all, budget, threads)
        if step >= args.warmup:
            rates.append(r["done"] / r["seconds"])
            secs.append(r["seconds"])
            done = r["done"]
    value = float(np.mean(rates))
    sample = (f"first {done} of the {count} {unit} in input order per step, B=1 runIds calls on the "
              f"{BUCKET}-token bucket plan, {np.mean(secs):.1f} s per step")
    line = {"metric": metric_name(args.workload), "value": value, "unit": f"{unit}/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * float(np.mean(secs)), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": bulk_config(args.workload, spec, lens, count, world=max(1, args.gpus)),
            "sample": sample,
            "cpu_baseline": {"value": value, "unit": f"{unit}/s", "cores": threads, "kind": "port", "sample": sample,
                             **host_info(threads)},
            "e2e": {"value": value, "unit": f"{unit}/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def default_count(workload: str) -> int:
    return {"c5": 65536, "c2-512-bulk": 4096, "c3-512-bulk": 2048}[workload]


def metric_name(workload: str) -> str:
    if workload == "c5":
        return "encoder pairs/sec (f16 cross-encoder rerank, ragged)"
    name = BULK_WORKLOADS[workload][0]
    return f"encoder seqs/sec ({name} f16, sequence length 512)"


def bulk_config(workload: str, spec: dict, lens: np.ndarray, count: int, world: int) -> dict:
    name = BULK_WORKLOADS[workload][0]
    what = {"c5": f"{name} {count}-pair rerank (BASELINE config 5)",
            "c2-512-bulk": f"{name} {count} sequences of 512 tokens (BASELINE config 2 shape, throughput)",
            "c3-512-bulk": f"{name} {count} sequences of 512 tokens (BASELINE config 3 shape, throughput)"}[workload]
    return {"workload": what, "sequences": int(count), "tokens": int(lens.sum()), "mean_len": float(lens.mean()),
            "bucket": BUCKET, "layers": spec["layers"], "hidden": spec["hidden"], "parallelism": f"dp{world}",
            "l2": "inputs larger than L2 (word rows of every sequence resident, read once per step)"}


def run_config(args):
    """Latency of BASELINE configs 1-3 (B = 1 through the PlanRunner: upload, run, read every call;
    20 warm-up calls, then at least 300 measured, median and p95 as bench/metrics.ts:27-40), and
    seqs/s of config 4 (64 ragged sequences through the bulk API), on one GPU, with the device time
    of the same calls beside it."""
    import torch

    from kleinhirn_b200 import synthetic
    from kleinhirn_b200.backend import CudaBackend
    from kleinhirn_b200.encoder import mask_and_types, packed_inputs, word_rows
    from kleinhirn_b200.plan import build_plan
    name, length, f16 = CONFIG_WORKLOADS[args.workload]
    spec, head = synthetic.model(name)
    w = synthetic.random_weights(spec, head, seed=args.seed)
    if f16:
        w = synthetic.to_f16(w)
    table = w["embeddings.word.weight"]
    be = CudaBackend(w)
    stream = torch.cuda.ExternalStream(be.stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    warm, calls = max(20, args.warmup), max(300, args.steps)
    with ClockSampler(0) as clocks:
        if length is not None:
            ids = synthetic.token_ids(name, np.array([length]), args.seed)[0]
            plan = build_plan(spec, head, length, 1, 0, f16)
            r = be.runner(plan)
            inputs = [{"inputIds": list(ids)}]
            mask, types = mask_and_types(spec, inputs, length)
            rows = word_rows(table, inputs, length)
            tt = types if "typeIds" in plan["inputs"] else None

            def call():
                r.upload(rows, mask, tt)
                r.run(length)
                return r.read_output()

            def device_call():
                r.run(length)
            unit, per_call = "ms", None
            launches = len(r.launches())
        else:
            lens = synthetic.seq_lengths(name, 64, args.seed)
            ids = synthetic.token_ids(name, lens, args.seed)
            emb, types, lens = packed_inputs(spec, table, ids)
            plan = build_plan(spec, head, 512, 1, 0, f16)
            r = be.runner(plan)
            bulk = be.bulk(r, int(lens.sum()), len(lens), chunk_size(int(lens.sum()), args.chunk_tokens))
            tt = types if "typeIds" in plan["inputs"] else None

            def call():
                return bulk.run_batch(lens, emb, tt)

            def device_call():
                bulk.run()
            unit, per_call = "seqs/s", len(lens)
            call()
            launches = bulk.last_timing()[1]
        for _ in range(warm):
            call()
        times = []
        for _ in range(calls):
            t0 = time.perf_counter()
            call()
            times.append((time.perf_counter() - t0) * 1000.0)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(calls):
            device_call()
        ev1.record(stream)
        torch.cuda.synchronize()
        dev_ms = ev0.elapsed_time(ev1) / calls
    times = np.array(times)
    med, p95 = float(np.median(times)), float(np.percentile(times, 95))
    gemm, attn = model_flops(spec, np.array([length]) if length else lens)
    peaks = read_peaks()
    if per_call is None:
        line = {"metric": f"ms/call B=1 L={length} ({name})", "value": med, "unit": "ms", "higher_is_better": False,
                "p95_ms": p95, "device_ms": dev_ms}
    else:
        line = {"metric": f"seqs/sec, 64 ragged sequences ({name})", "value": per_call / (med / 1e3),
                "unit": "seqs/s", "higher_is_better": True, "median_ms": med, "p95_ms": p95,
                "device_seqs_per_s": per_call / (dev_ms / 1e3), "device_ms": dev_ms, "tokens": int(lens.sum())}
    line.update({"n_gpus": 1, "warmup_calls": warm, "calls": calls, "dtype": "f16" if f16 else "f32",
                 "data": "synthetic", "protocol": "20 warm-up calls, then >= 300 measured: median and p95 of the "
                                                  "host wall time from host arrays to the f32 outputs",
                 "config": {"workload": f"{name} (BASELINE config {args.workload[1]})", "layers": spec["layers"],
                            "hidden": spec["hidden"]},
                 "model_tflops_device": (gemm + attn) / (dev_ms / 1e3) / 1e12,
                 "frac_of_peak_device": (gemm + attn) / (dev_ms / 1e3) / 1e12 / peaks["tflops"],
                 "gpu_launches_per_call": launches, "clocks": clocks.summary()})
    if per_call is not None:
        bulk.close()
    r.destroy()
    be.dispose()
    print(json.dumps(line), flush=True)


def run_bulk(args):
    world, rank, local = dist_setup()
    import torch
    torch.cuda.set_device(local)
    dist = gloo = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
        gloo = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=180))
    from kleinhirn_b200 import synthetic
    from kleinhirn_b200.backend import CudaBackend
    from kleinhirn_b200.encoder import packed_inputs
    from kleinhirn_b200.plan import build_plan

    name, length, unit = BULK_WORKLOADS[args.workload]
    count = args.pairs or default_count(args.workload)
    spec, head, lens, ids_all = workload_inputs(name, length, count, args.seed)
    w16 = synthetic.to_f16(synthetic.random_weights(spec, head, seed=args.seed))
    shards = [shard_sequences(lens, world, r) for r in range(world)]
    mine = shards[rank]
    my_ids = [ids_all[i] for i in mine]
    my_lens = lens[mine].astype(np.int32)
    tokens = int(my_lens.sum())

    be = CudaBackend(w16, device=local)
    plan = build_plan(spec, head, BUCKET, 1, 0, True)
    runner = be.runner(plan)
    chunk_rows = chunk_size(tokens, args.chunk_tokens)
    n_chunks = max(1, -(-tokens // chunk_rows))
    launch_rows = tokens / n_chunks  # mean packed rows of one GEMM launch
    bulk = be.bulk(runner, tokens, len(my_lens), chunk_rows)
    stream = torch.cuda.ExternalStream(be.stream, device=torch.device("cuda", local))
    has_types = "typeIds" in plan["inputs"]
    cols = runner.out_cols

    # resident inputs of the device-time run: host-gathered word rows, uploaded once
    emb, types, _ = packed_inputs(spec, w16["embeddings.word.weight"], my_ids)
    bulk.set_lengths(my_lens)
    bulk.upload(emb, types if has_types else None)
    del emb
    # pinned host buffers of the e2e path: packed token ids (the word table lives on the device)
    be.add_tensor("embeddings.word.weight", w16["embeddings.word.weight"])
    bulk.set_word_table("embeddings.word.weight")
    flat_ids = np.concatenate([np.asarray(x, dtype=np.int32) for x in my_ids])
    h_ids = torch.empty(flat_ids.size, dtype=torch.int32, pin_memory=True)
    h_ids.numpy()[:] = flat_ids
    h_types = torch.empty(max(1, types.size), dtype=torch.int32, pin_memory=True)
    h_types.numpy()[:types.size] = types.view(np.int32)
    gather = OutputGather(dist, gloo, rank, shards, cols, pin=True)
    h_out = gather.local
    out_all = None
    torch.cuda.synchronize()

    def barrier():
        if dist:
            dist.barrier(group=gloo)

    def over_ranks(x: float) -> list[float]:
        if not dist:
            return [x]
        t = torch.tensor([x], dtype=torch.float64)
        out = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(out, t, group=gloo)
        return [float(o.item()) for o in out]

    # warm-up, then K timed device-resident forwards (inputs already in HBM)
    for _ in range(args.warmup):
        bulk.run()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            bulk.run()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    rank_ms = over_ranks(ev0.elapsed_time(ev1))
    dev_ms = max(rank_ms)
    per_run_launches = bulk.last_timing()[1]
    launches = per_run_launches * args.steps
    ms_per_step = dev_ms / args.steps
    value = count / (ms_per_step / 1000.0)

    # e2e through the public bulk API, every step: sequence lengths, pinned H2D of the packed token
    # ids (and typeIds), device-side word-row gather, forward, D2H of the logits, and the gather of
    # every rank's logits into input order on rank 0 (the host gather of the data-parallel run)
    def e2e_step():
        bulk.set_lengths(my_lens)
        bulk.upload_ids_ptr(h_ids.data_ptr(), flat_ids.size, h_types.data_ptr() if has_types else None,
                            types.size if has_types else 0)
        bulk.run()
        bulk.read_ptr(h_out.data_ptr(), len(mine) * cols)
        return gather.gather()

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out_all = e2e_step()
    torch.cuda.synchronize()
    e2e_s = max(over_ranks(time.perf_counter() - t0))
    e2e_value = count / (e2e_s / args.steps)
    h2d = flat_ids.nbytes + (types.nbytes if has_types else 0) + my_lens.nbytes
    d2h = len(mine) * cols * 4
    h2d_all = sum(over_ranks(float(h2d)))
    d2h_all = sum(over_ranks(float(d2h)))

    # per-launch profile of one forward (separate pass): the roofline of the GEMM and attention
    # kernel families
    prof = bulk.profile()
    gemm_flops, attn_flops = model_flops(spec, my_lens)
    by_label: dict[str, float] = {}
    for step, ms in prof:
        by_label[step["label"]] = by_label.get(step["label"], 0.0) + ms
    total_prof = sum(by_label.values())
    peaks = read_peaks()

    def family(label: str, flops: float) -> dict:
        ms = by_label.get(label, 0.0)
        ach = flops / (ms / 1000.0) / 1e12 if ms > 0 else 0.0
        return {"achieved": ach, "peak": peaks["tflops"], "unit": "TFLOP/s",
                "frac": ach / peaks["tflops"] if peaks["tflops"] else None,
                "share_of_forward": ms / total_prof if total_prof else None, "ms_per_forward": ms}

    kernels = {"gemm": family("gemm", gemm_flops), "attention": family("attention", attn_flops)}
    top = max(kernels, key=lambda k: kernels[k]["share_of_forward"] or 0.0)
    if args.profile_out and rank == 0:
        Path(args.profile_out).write_text(json.dumps(
            {"steps": [{"label": s["label"], "ops": s["ops"], "ms": ms} for s, ms in prof],
             "by_label_ms": by_label, "tokens": tokens, "sequences": int(len(my_lens)),
             "gemm_flops": gemm_flops, "attn_flops": attn_flops}, indent=1))
    rank_info = [{"rank": r, "device_ms_per_step": ms / args.steps, "tokens": t, "sequences": int(len(shards[r])),
                  "chunks": int(c)}
                 for r, (ms, t, c) in enumerate(zip(rank_ms, over_ranks(float(tokens)), over_ranks(float(n_chunks))))]

    # parity of the logits the e2e steps gathered (input order on rank 0)
    cpu = parity = ranks_vs_one = None
    if rank == 0:
        threads = min(os.cpu_count() or 1, 8)
        budget = args.cpu_seconds if (world == 1 and not args.no_cpu_baseline) else 2.0
        s = cpu_sample(spec, head, w16, ids_all, budget, threads, max_items=None if world == 1 else 16)
        tol = C5_PARITY_ABS if args.workload == "c5" else 2e-2 * max(1.0, float(np.abs(s["outputs"]).max()))
        parity = parity_block(out_all[:s["done"]], s["outputs"], tol)
        if world == 1 and not args.no_cpu_baseline:
            cpu = {"value": s["done"] / s["seconds"], "unit": f"{unit}/s", "cores": threads, "kind": "port",
                   "sample": f"first {s['done']} of the {unit} in input order, B=1 runIds calls on the {BUCKET}-token "
                             f"bucket plan, {s['seconds']:.1f} s", **host_info(threads)}
        if world > 1:
            # every sequence again on this GPU alone, packed as a one-rank run packs it
            one = shard_sequences(lens, 1, 0)
            o_emb, o_types, o_lens = packed_inputs(spec, w16["embeddings.word.weight"], [ids_all[i] for i in one])
            b1 = be.bulk(runner, int(o_lens.sum()), len(o_lens), chunk_size(int(o_lens.sum()), args.chunk_tokens))
            ref1 = np.zeros_like(out_all)
            ref1[one] = b1.run_batch(o_lens, o_emb, o_types if has_types else None).reshape(-1, cols)
            b1.close()
            diff = float(np.abs(ref1 - out_all).max())
            ranks_vs_one = {"n": int(count), "max_abs": diff, "tol": RANKS_VS_ONE, "pass": diff <= RANKS_VS_ONE}
    barrier()

    if rank == 0:
        fam = kernels[top]
        line = {
            "metric": metric_name(args.workload), "value": value, "unit": f"{unit}/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": bulk_config(args.workload, spec, lens, count, world),
            "model_tflops": (gemm_flops + attn_flops) * world / (ms_per_step / 1000.0) / 1e12,
            "gpu_launches": int(launches),
            "e2e": {"value": e2e_value, "unit": f"{unit}/s", "h2d_bytes_per_step": int(h2d_all),
                    "d2h_bytes_per_step": int(d2h_all),
                    "includes": "ids H2D, device gather, forward, logits D2H, host gather in input order"},
            "roofline": {"bound": "tensor", "kernel": top, "achieved": fam["achieved"], "peak": fam["peak"],
                         "unit": "TFLOP/s", "frac": fam["frac"],
                         "peak_source": peaks["source"] + " bf16_tflops_sustained",
                         "traffic": GEMM_TRAFFIC_BYTES * launch_rows / GEMM_TRAFFIC_ROWS if top == "gemm" else None,
                         "traffic_unit": "bytes per launch (mean over the GEMM launches)",
                         "traffic_source": GEMM_TRAFFIC_SOURCE if top == "gemm" else None,
                         "share_of_forward": fam["share_of_forward"]},
            "kernels": kernels,
            "ranks": rank_info,
            "parity": parity,
            "clocks": clocks.summary(),
        }
        if ranks_vs_one:
            line["ranks_vs_one_gpu"] = ranks_vs_one
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    bulk.close()
    runner.destroy()
    be.dispose()
    failed = rank == 0 and (not parity["pass"] or (ranks_vs_one is not None and not ranks_vs_one["pass"]))
    if dist:
        dist.destroy_process_group()
    if failed:
        print("parity check failed", file=sys.stderr, flush=True)
        sys.exit(3)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload in CONFIG_WORKLOADS:
        run_config(args)
        return
    run_bulk(args)


if __name__ == "__main__":
    main()
