#!/usr/bin/env python
"""Benchmark of the CUDA encoder forward on B200: sequences/sec of a ragged throughput run.

Workload (the configuration its "seqs/sec at 1/2/4/8 B200" metric is quoted
on): a multilingual MiniLM-L12 cross-encoder (XLM-R shape: 12 layers, hidden 384, 12 heads, FFN
1536, vocab 250002), random-init weights, f16, 1-logit rerank head, over 65,536 synthetic
query/passage pairs (query length U[4, 32], passage lognormal median 90 sigma 0.8, the pair with
its 4 specials <= 512 tokens). One step = one forward of every pair; the pairs are split across
the ranks (strong scaling, balanced by token count), no collective on the data path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--pairs P] [--impl reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

value: pairs/sec of the whole job with the packed inputs already resident in HBM, device time
(CUDA events on the library's stream) max over ranks. e2e: the same metric through the public
bulk API with host buffers (pinned H2D of the word rows and type ids, D2H of the logits) every
step. cpu_baseline: the C++ restatement of the reference's WASM-SIMD executor (oracle/) on a
bounded sample of the same pairs, B = 1 calls on the 512-token bucket plan (runIds).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOAD = "mminilm-l12-xlmr"
BUCKET = 512


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one GEMM launch on a 262,144-row
# chunk, mean of the four GEMM launches of a layer (qkv 0.753 GB, FFN-in 0.951 GB, attnOut +
# LayerNorm 0.568 GB, FFN-out + LayerNorm 1.195 GB), from one ncu capture each; every term is
# rows x a per-row byte count, so a launch over another chunk size scales with its rows.
GEMM_TRAFFIC_BYTES = 866.2e6
GEMM_TRAFFIC_ROWS = 262144
GEMM_TRAFFIC_SOURCE = "ncu, profiles/gemm_pair_c5.md and profiles/gemm_addln_c5.md"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--pairs", type=int, default=65536)
    ap.add_argument("--chunk-tokens", type=int, default=0,
                    help="packed rows per bulk chunk (0: even chunks of at most 524,288 rows)")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-out", default="", help="write the per-launch profile of one forward here")
    ap.add_argument("--workload", default="c5", choices=["c5", "c1", "c2-128", "c2-512", "c3", "c4"],
                    help="c5: the headline (BASELINE config 5); the others print ms/call (c1-c3, B = 1 plan "
                         "calls) or seqs/s (c4, 64 ragged sequences) of BASELINE configs 1-4, one GPU")
    return ap.parse_args()


# (synthetic configuration, sequence length or None for ragged, f16)
CONFIG_WORKLOADS = {
    "c1": ("minilm-l6", 128, False),
    "c2-128": ("roberta-base", 128, True),
    "c2-512": ("roberta-base", 512, True),
    "c3": ("deberta-v3-base", 512, True),
    "c4": ("modernbert-base", None, True),
}


def run_config(args):
    """ms per call (B = 1 through the PlanRunner: upload, run, read every call) of configs 1-3, and
    seqs/s of config 4 (64 ragged sequences through the bulk API), on one GPU, with the device
    time of the same calls beside it."""
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
            for _ in range(max(3, args.warmup)):
                call()
            calls = max(20, args.steps)
            t0 = time.perf_counter()
            for _ in range(calls):
                call()
            e2e_ms = (time.perf_counter() - t0) * 1000.0 / calls
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(calls):
                r.run(length)
            ev1.record(stream)
            torch.cuda.synchronize()
            dev_ms = ev0.elapsed_time(ev1) / calls
            launches = len(r.launches())
            r.destroy()
            line = {"metric": f"ms/call B=1 L={length} ({name})", "value": e2e_ms, "unit": "ms",
                    "higher_is_better": False, "device_ms": dev_ms, "calls": calls}
        else:
            lens = synthetic.seq_lengths(name, 64, args.seed)
            ids = synthetic.token_ids(name, lens, args.seed)
            emb, types, lens = packed_inputs(spec, table, ids)
            plan = build_plan(spec, head, 512, 1, 0, f16)
            r = be.runner(plan)
            bulk = be.bulk(r, int(lens.sum()), len(lens), chunk_size(int(lens.sum()), args.chunk_tokens))
            tt = types if "typeIds" in plan["inputs"] else None
            for _ in range(max(3, args.warmup)):
                bulk.run_batch(lens, emb, tt)
            calls = max(20, args.steps)
            t0 = time.perf_counter()
            for _ in range(calls):
                bulk.run_batch(lens, emb, tt)
            e2e_s = (time.perf_counter() - t0) / calls
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(calls):
                bulk.run()
            ev1.record(stream)
            torch.cuda.synchronize()
            dev_ms = ev0.elapsed_time(ev1) / calls
            launches = bulk.last_timing()[1]
            bulk.close()
            r.destroy()
            line = {"metric": f"seqs/sec, 64 ragged sequences ({name})", "value": len(lens) / e2e_s,
                    "unit": "seqs/s", "higher_is_better": True, "device_seqs_per_s": len(lens) / (dev_ms / 1e3),
                    "device_ms": dev_ms, "tokens": int(lens.sum()), "calls": calls}
    line.update({"n_gpus": 1, "dtype": "f16" if f16 else "f32", "data": "synthetic",
                 "config": {"workload": f"{name} (BASELINE config {args.workload[1]})", "layers": spec["layers"],
                            "hidden": spec["hidden"]},
                 "gpu_launches_per_call": launches, "clocks": clocks.summary()})
    be.dispose()
    print(json.dumps(line), flush=True)


def model_flops(spec: dict, lens: np.ndarray) -> tuple[float, float]:
    """Algorithmic FLOPs (2 per MAC) of the encoder layers: (GEMM part, attention part). Per layer
    and sequence of n rows: 2 n (3H^2 + H^2) for qkv + attnOut, 4 n H I for the MLP, 4 n n H for
    QK^T and PV (all keys: global attention)."""
    H, I, layers = spec["hidden"], spec["intermediate"], spec["layers"]
    n = lens.astype(np.float64)
    gemm = layers * (2 * n * 4 * H * H + 4 * n * H * I).sum()
    attn = layers * (4 * n * n * H).sum()
    return float(gemm), float(attn)


def read_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "tflops": d.get("bf16_tflops_sustained", 1394.8),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "source": "fallback"}


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


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def shard_pairs(lens: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Indices of this rank's pairs: longest first onto the least-loaded rank (token count), so
    every rank gets about the same work; deterministic on every rank."""
    order = np.argsort(-lens, kind="stable")
    load = np.zeros(world, dtype=np.int64)
    owner = np.empty(len(lens), dtype=np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += int(lens[i])
    mine = np.nonzero(owner == rank)[0]
    return mine[np.argsort(lens[mine], kind="stable")]


def chunk_size(tokens: int, requested: int) -> int:
    """Packed rows per bulk chunk: as asked, or the rank's rows in even chunks of at most
    524,288 (long launches keep the tail waves of the GEMMs small; even chunks avoid a short last
    one), plus room for the sequence that does not fit exactly."""
    if requested > 0:
        return requested
    n = max(1, -(-tokens // 524288))
    return max(BUCKET, -(-tokens // n) + BUCKET)


def make_workload(args):
    from kleinhirn_b200 import synthetic
    spec, head = synthetic.model(WORKLOAD)
    lens = synthetic.seq_lengths(WORKLOAD, args.pairs, args.seed)
    return spec, head, lens


def cpu_baseline(spec, head, w16, ids_all, budget_s: float, threads: int) -> dict:
    """The oracle on host cores: B = 1 calls (runIds) on the 512-token bucket, f32 on the f16 weights'
    values, pairs in input order until the time budget is used."""
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
        done, t0 = 0, time.perf_counter()
        outs = []
        while done < len(ids_all):
            ids = ids_all[done]
            inputs = [{"inputIds": list(ids)}]
            mask, types = mask_and_types(spec, inputs, BUCKET)
            p.upload(word_rows(table, inputs, BUCKET), mask, types)
            p.run(len(ids))
            outs.append(p.read_output()[0])
            done += 1
            if time.perf_counter() - t0 > budget_s and done >= 4:
                break
        dt = time.perf_counter() - t0
    finally:
        rt.close()
    return {"value": done / dt, "unit": "pairs/s", "cores": threads, "kind": "port",
            "sample": f"first {done} of the pairs, B=1 runIds calls on the {BUCKET}-token bucket plan, "
                      f"{dt:.1f} s", "outputs": np.array(outs)}


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's WASM executor with every host
    thread, on bounded samples of the same pairs; rank 0 only."""
    world, rank, local = dist_setup(args)
    if rank != 0:
        return
    from kleinhirn_b200 import synthetic
    spec, head, lens = make_workload(args)
    w16 = synthetic.to_f16(synthetic.random_weights(spec, head, seed=args.seed))
    ids_all = synthetic.token_ids(WORKLOAD, lens, args.seed)
    threads = os.cpu_count() or 1
    budget = max(2.0, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    res = None
    times = []
    for step in range(args.warmup + args.steps):
        r = cpu_baseline(spec, head, w16, ids_all, budget, threads)
        if step >= args.warmup:
            times.append(r["value"])
            res = r
    value = float(np.mean(times))
    line = {"metric": "encoder pairs/sec (f16 cross-encoder rerank, ragged)", "value": value, "unit": "pairs/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * args.pairs / value, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{WORKLOAD} {args.pairs}-pair rerank (BASELINE config 5)", "pairs": args.pairs,
                       "bucket": BUCKET},
            "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": threads, "kind": "port",
                             "sample": res["sample"] if res else ""},
            "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload != "c5":
        run_config(args)
        return
    world, rank, local = dist_setup(args)
    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    from kleinhirn_b200 import synthetic
    from kleinhirn_b200.backend import CudaBackend
    from kleinhirn_b200.encoder import packed_inputs
    from kleinhirn_b200.plan import build_plan

    spec, head, lens = make_workload(args)
    w16 = synthetic.to_f16(synthetic.random_weights(spec, head, seed=args.seed))
    ids_all = synthetic.token_ids(WORKLOAD, lens, args.seed)
    mine = shard_pairs(lens, world, rank)
    my_ids = [ids_all[i] for i in mine]
    emb, types, my_lens = packed_inputs(spec, w16["embeddings.word.weight"], my_ids)
    tokens = int(my_lens.sum())

    be = CudaBackend(w16, device=local)
    plan = build_plan(spec, head, BUCKET, 1, 0, True)
    runner = be.runner(plan)
    chunk_rows = chunk_size(tokens, args.chunk_tokens)
    launch_rows = tokens / max(1, -(-tokens // chunk_rows))  # mean packed rows of one GEMM launch
    bulk = be.bulk(runner, tokens, len(my_lens), chunk_rows)
    stream = torch.cuda.ExternalStream(be.stream, device=torch.device("cuda", local))

    # pinned host buffers of the e2e path: packed token ids (the word table lives on the device)
    be.add_tensor("embeddings.word.weight", w16["embeddings.word.weight"])
    bulk.set_word_table("embeddings.word.weight")
    flat_ids = np.concatenate([np.asarray(x, dtype=np.int32) for x in my_ids])
    h_ids = torch.empty(flat_ids.size, dtype=torch.int32, pin_memory=True)
    h_ids.numpy()[:] = flat_ids
    h_emb = torch.empty(emb.size, dtype=torch.float16, pin_memory=True)
    h_emb.numpy()[:] = emb.reshape(-1)
    h_types = torch.empty(types.size, dtype=torch.int32, pin_memory=True)
    h_types.numpy()[:] = types.view(np.int32)
    h_out = torch.empty(len(my_lens), dtype=torch.float32, pin_memory=True)
    has_types = "typeIds" in plan["inputs"]

    bulk.set_lengths(my_lens)
    bulk.upload_ptr(h_emb.data_ptr(), emb.nbytes, h_types.data_ptr() if has_types else None,
                    types.size if has_types else 0)
    torch.cuda.synchronize()

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up, then K timed device-resident forwards (inputs already in HBM)
    for _ in range(args.warmup):
        bulk.run()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    launches = 0
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            bulk.run()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    dev_ms = ev0.elapsed_time(ev1)
    per_run_launches = bulk.last_timing()[1]
    launches = per_run_launches * args.steps
    dev_ms = max_over_ranks(dev_ms)
    ms_per_step = dev_ms / args.steps
    value = args.pairs / (ms_per_step / 1000.0)

    # e2e through the public bulk API, every step: sequence lengths, pinned H2D of the packed token
    # ids (and typeIds), device-side word-row gather, forward, D2H of the logits
    def e2e_step():
        bulk.set_lengths(my_lens)
        bulk.upload_ids_ptr(h_ids.data_ptr(), flat_ids.size, h_types.data_ptr() if has_types else None,
                            types.size if has_types else 0)
        bulk.run()
        bulk.read_ptr(h_out.data_ptr(), h_out.numel())

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = args.pairs / (e2e_s / args.steps)
    h2d = flat_ids.nbytes + (types.nbytes if has_types else 0) + my_lens.nbytes
    d2h = h_out.numel() * 4

    # per-launch profile of one forward (separate pass): the dominant kernel's roofline
    prof = bulk.profile()
    gemm_flops, attn_flops = model_flops(spec, my_lens)
    by_label: dict[str, float] = {}
    for step, ms in prof:
        by_label[step["label"]] = by_label.get(step["label"], 0.0) + ms
    total_prof = sum(by_label.values())
    gemm_ms = by_label.get("gemm", 0.0)
    peaks = read_peaks()
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else 0.0
    if args.profile_out and rank == 0:
        Path(args.profile_out).write_text(json.dumps(
            {"steps": [{"label": s["label"], "ops": s["ops"], "ms": ms} for s, ms in prof],
             "by_label_ms": by_label, "tokens": tokens, "pairs": int(len(my_lens)),
             "gemm_flops": gemm_flops, "attn_flops": attn_flops}, indent=1))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(spec, head, w16, ids_all, args.cpu_seconds, min(os.cpu_count() or 1, 8))
        cpu_out = cpu.pop("outputs")

    if rank == 0:
        line = {
            "metric": "encoder pairs/sec (f16 cross-encoder rerank, ragged)", "value": value, "unit": "pairs/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": f"{WORKLOAD} {args.pairs}-pair rerank (BASELINE config 5)", "pairs": args.pairs,
                       "tokens": int(lens.sum()), "mean_len": float(lens.mean()), "bucket": BUCKET,
                       "layers": spec["layers"], "hidden": spec["hidden"], "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2 (word rows of every pair resident, read once per step)"},
            "model_tflops": (gemm_flops + attn_flops) * world / (ms_per_step / 1000.0) / 1e12,
            "gpu_launches": int(launches),
            "e2e": {"value": e2e_value, "unit": "pairs/s", "h2d_bytes_per_step": int(h2d) * world,
                    "d2h_bytes_per_step": int(d2h) * world},
            "roofline": {"bound": "tensor", "kernel": "gemm", "achieved": achieved, "peak": peaks["tflops"],
                         "unit": "TFLOP/s", "frac": achieved / peaks["tflops"] if peaks["tflops"] else None,
                         "peak_source": peaks["source"] + " bf16_tflops_sustained",
                         "traffic": GEMM_TRAFFIC_BYTES * launch_rows / GEMM_TRAFFIC_ROWS,
                         "traffic_unit": "bytes per launch (mean over the GEMM launches)",
                         "traffic_source": GEMM_TRAFFIC_SOURCE,
                         "share_of_forward": gemm_ms / total_prof if total_prof else None},
            "clocks": clocks.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    bulk.close()
    runner.destroy()
    be.dispose()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
