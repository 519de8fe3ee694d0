"""Benchmark of the B200 cascade decode-attention path.

Default workload (N=1): the MCTS-shaped Llama-3-8B tree — 32 query / 8 KV
heads, head_dim 128, bf16 KV, an 8192-token root, shared nodes of 128-1024
tokens at depths 1-3 (fan-out 8/4/4), 512 leaves with U[16, 256]-token
private suffixes — one decode query per leaf. A step is one cascade decode of
the whole batch (all 512 queries, every KV head) through dd_cascade_decode.

With N GPUs (torchrun, one process per GPU) every rank decodes its own
independent tree (trees are partitioned across GPUs; no collective on the data
path), so scaling is weak and `value` = all ranks' queries / max-over-ranks
time.

Output: one JSON line (rank 0). `--impl reference` times the reference's CPU
algorithm (the C restatement of ReferenceBackend::decode_batch in oracle/) on
the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn queries/s + HBM GB/s (% of peak) at 1/2/4/8 B200, vs CPU reference"
FALLBACK_HBM_GBS = 6650.0
SEED = 0xD3D1


FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    """(HBM GB/s, dense bf16 TFLOP/s burst, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


WORKLOADS = {
    "mcts8b": dict(kv="bf16", desc="config 3: Llama-3-8B heads, 8192 root, depths 1-3, 512 leaves"),
    "mcts8b-e4m3": dict(kv="e4m3", desc="config 4: config 3 with per-head E4M3 KV pages"),
    "mcts8b-mxfp8": dict(kv="mxfp8", desc="config 4: config 3 with MXFP8 KV pages"),
}


def make_tree(name: str, seed: int):
    from dendrite_b200 import workloads as wl

    return wl.mcts_llama3_8b(seed)


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    def __init__(self, device_index: int, out: Path | None):
        self.proc = None
        self.path = out
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(out, "w") if out else subprocess.DEVNULL
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={device_index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            text, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            text, _ = self.proc.communicate()
        rows = [r.split(", ") for r in text.strip().splitlines() if r.count(",") >= 8]
        if self.path:
            self.path.write_text(text)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


def cpu_sample_rate(tb, pool_bits, q_f32, budget_s: float, threads: int):
    """Reference CPU algorithm (oracle restatement of ReferenceBackend::decode_batch)
    on the first queries of the batch; returns (queries/s, n queries, seconds)."""
    import oracle

    def run(n):
        ip = tb.indptr[: n + 1]
        ids = tb.block_ids[: ip[-1]]
        t0 = time.perf_counter()
        oracle.decode_batch(q_f32[:n], pool_bits, ip, ids, tb.num_tokens[:n], tb.num_kv_heads,
                            threads=threads)
        return time.perf_counter() - t0

    n = min(threads, tb.batch_size)
    t = run(n)
    per = t / n
    n2 = int(max(n, min(tb.batch_size, budget_s / max(per, 1e-6))))
    n2 = max(threads, (n2 // threads) * threads) if n2 >= threads else n2
    t2 = run(n2)
    return n2 / t2, n2, t2


def oracle_threads(tb) -> int:
    """Host threads for the CPU reference: all cores, capped by the memory its
    per-thread gather/repeat copies need."""
    cores = os.cpu_count() or 1
    try:
        import psutil

        avail = psutil.virtual_memory().available
    except Exception:
        avail = 64 << 30
    T = int((np.diff(tb.indptr).max()) * 16)
    per = (tb.num_kv_heads + tb.num_qo_heads) * T * tb.head_dim * 4 * 2
    return int(max(1, min(cores, avail * 0.5 // max(per, 1))))


def host_workload(args, rank):
    tb = make_tree(args.workload, SEED + rank)
    rng = np.random.default_rng(SEED + rank)
    import oracle

    pool = oracle.f32_to_bf16_bits(
        rng.standard_normal((tb.num_pages, 2, tb.num_kv_heads, 16, tb.head_dim), dtype=np.float32))
    q = oracle.f32_to_bf16_bits(
        rng.standard_normal((tb.batch_size, tb.num_qo_heads, tb.head_dim), dtype=np.float32))
    return tb, pool, q


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle

    kv = WORKLOADS[args.workload]["kv"]
    tb, pool, qbits = host_workload(args, 0)
    if kv != "bf16":
        codes, sc = (oracle.quantize_per_head(pool) if kv == "e4m3" else oracle.quantize_mx(pool))
        pool = oracle.dequantize(codes, sc, kv)
    q = oracle.bf16_bits_to_f32(qbits)
    threads = oracle_threads(tb)
    n = min(tb.batch_size, threads)
    ip = tb.indptr[: n + 1]

    def step():
        oracle.decode_batch(q[:n], pool, ip, tb.block_ids[: ip[-1]], tb.num_tokens[:n],
                            tb.num_kv_heads, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    val = n * args.steps / dt
    sample = f"first {n} of {tb.batch_size} queries per step ({threads} threads), {args.steps} steps"
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": args.workload, "desc": WORKLOADS[args.workload]["desc"]},
        "cpu_baseline": {"value": val, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import dendrite_b200 as dd
    from dendrite_b200 import _lib
    from dendrite_b200 import workloads as wl

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    kv = WORKLOADS[args.workload]["kv"]
    hbm_peak, tc_peak, peak_kind = peaks()

    tb = make_tree(args.workload, SEED + rank)
    Hq, Hkv, D, B = tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.batch_size
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + rank)
    pool = torch.randn((tb.num_pages, 2, Hkv, 16, D), generator=gen, device=dev,
                       dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((B, Hq, D), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    scales = None
    kv_dtype, elem, scale_bytes = _lib.DTYPE_BF16, 2.0, 0.0
    if kv != "bf16":
        codes, scales = dd.quantize_kv_pages(pool, kv)
        kv_pages = codes
        kv_dtype = _lib.DTYPE_E4M3 if kv == "e4m3" else _lib.DTYPE_MXFP8
        elem = 1.0
        scale_bytes = D / 32 if kv == "mxfp8" else 0.0
    else:
        kv_pages = pool
    cfg = dd.make_config(Hq, Hkv, D, tb.num_pages, kv_dtype=kv_dtype)
    plan = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
    plan.upload(dev)
    info = plan.info()
    ws = torch.empty(max(int(info.workspace_bytes), 256), dtype=torch.uint8, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    stream = torch.cuda.current_stream()

    def step():
        dd.cascade_decode(cfg, plan, q, kv_pages, scales, out, lse, ws)

    for _ in range(args.warmup):
        step()
        flush.zero_()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local, ROOT / "gpurun_out" / f"clocks_rank{rank}.csv"
                    if (ROOT / "gpurun_out").is_dir() else None)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    n0 = _lib.launch_count()
    for a, b in ev:
        a.record(stream)
        step()
        b.record(stream)
        flush.zero_()  # L2 flush between steps, outside the timed intervals
    torch.cuda.synchronize()
    launches = _lib.launch_count() - n0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_step = ms_max / args.steps

    # Per-kernel durations (CUDA events on the launching stream), separate pass.
    _lib.profile_enable(True)
    prof_steps = min(args.steps, 20)
    for _ in range(prof_steps):
        step()
        flush.zero_()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)

    kv_bytes = info.kv_tokens * 2 * Hkv * (D * elem + scale_bytes)
    if kv == "e4m3":
        kv_bytes += 2 * Hkv * 4
    qo_bytes = B * Hq * D * 4
    eff_bytes = kv_bytes + qo_bytes
    # Roofline of the dominant attention kernel: bytes (streaming kernels) or
    # FLOPs (tcgen05 kernel) it is given by the plan, over its average launch.
    kt = list(info.kv_tokens_by_kernel)
    per_tok = 2 * Hkv * (D * elem + scale_bytes)
    kernels = {}
    for idx, name in ((0, "attn_simple"), (1, "attn_mma")):
        if prof[name][1]:
            ms_l = prof[name][0] / prof[name][1]
            byts = kt[idx] * per_tok + (B * Hq * D * 2 if idx == 1 or not kt[1] else 0)
            kernels[name] = {"bound": "hbm", "algorithmic": byts, "unit": "GB/s", "launch_ms": ms_l,
                             "achieved": byts / (ms_l * 1e-3) / 1e9, "peak": hbm_peak}
    if prof["attn_tc"][1]:
        ms_l = prof["attn_tc"][0] / prof["attn_tc"][1]
        flops = 4.0 * D * info.tc_row_tokens
        kernels["attn_tc"] = {"bound": "tensor", "algorithmic": flops, "unit": "TFLOP/s",
                              "launch_ms": ms_l, "achieved": flops / (ms_l * 1e-3) / 1e12,
                              "peak": tc_peak}
    for k in kernels.values():
        k["frac"] = k["achieved"] / k["peak"]
    attn_kind = max(kernels, key=lambda k: kernels[k]["launch_ms"] * prof[k][1])
    dom = kernels[attn_kind]
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"{args.workload}:{attn_kind}")

    # End-to-end through the public API with host buffers: plan from the host
    # block tables, H2D of the plan and the queries, decode, D2H of the output.
    q_host = q.cpu().pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    q_dev2 = torch.empty_like(q)

    def e2e_step():
        p2 = dd.CascadePlan(cfg, tb.indptr, tb.block_ids, tb.num_tokens)
        p2.device_buffer = plan.device_buffer
        p2.upload(dev)
        q_dev2.copy_(q_host, non_blocking=True)
        dd.cascade_decode(cfg, p2, q_dev2, kv_pages, scales, out, lse, ws)
        out_host.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        return p2.info().device_bytes

    for _ in range(3):
        e2e_step()
    e2e_n = max(5, min(args.steps, 30))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    plan_bytes = 0
    for _ in range(e2e_n):
        plan_bytes = e2e_step()
    e2e_s = torch.tensor([(time.perf_counter() - t0) / e2e_n], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_step_s = float(e2e_s.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        pool_bits = pool.view(torch.int16).cpu().numpy().view(np.uint16)
        if kv != "bf16":
            cc = kv_pages.cpu().numpy()
            ss = scales.cpu().numpy()
            pool_bits = oracle.dequantize(cc, ss, kv)
        qf = q.float().cpu().numpy()
        threads = oracle_threads(tb)
        rate, n, secs = cpu_sample_rate(tb, pool_bits, qf, args.cpu_budget, threads)
        cpu = {"value": rate, "unit": "queries/s", "cores": threads, "kind": "port",
               "sample": f"first {n} of {B} queries ({secs:.1f} s, {threads} threads)"}

    if rank == 0:
        value = B * world / (ms_step * 1e-3)
        gbs = eff_bytes / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if kv == "bf16" else f"{kv} KV / bf16 compute", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": args.workload, "desc": WORKLOADS[args.workload]["desc"],
                       "heads": [Hq, Hkv, D], "batch": B, "pages": tb.num_pages,
                       "unique_kv_tokens": info.kv_tokens, "flat_kv_tokens": info.kv_tokens_flat,
                       "plan_nodes": info.num_nodes, "l2": "flushed between steps (256 MiB write, untimed)",
                       "parallelism": f"tree-partitioned x{world}"},
            "effective_gbs": gbs, "hbm_frac": gbs / hbm_peak,
            "roofline": {"bound": dom["bound"], "kernel": attn_kind, "achieved": dom["achieved"],
                         "peak": dom["peak"], "unit": dom["unit"], "frac": dom["frac"],
                         "traffic": traffic, "peak_source": peak_kind + " (of measured)"
                         if peak_kind == "measured" else "of fallback",
                         "launch_ms": dom["launch_ms"], "algorithmic": dom["algorithmic"]},
            "kernel_rooflines": kernels,
            "kernel_ms_per_step": {k: v[0] / max(prof_steps, 1) for k, v in prof.items() if v[1]},
            "cpu_baseline": cpu,
            "e2e": {"value": B * world / e2e_step_s, "unit": "queries/s",
                    "h2d_bytes_per_step": int(q.numel() * 2 + plan_bytes),
                    "d2h_bytes_per_step": int(out.numel() * 2), "ms_per_step": e2e_step_s * 1e3},
            "clocks": clk, "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mcts8b")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
