"""Benchmark of the B200 cascade decode-attention path.

Default workload (N=1): the MCTS-shaped Llama-3-8B tree (config 3) — 32 query
/ 8 KV heads, head_dim 128, bf16 KV, an 8192-token root, shared nodes of
128-1024 tokens at depths 1-3 (fan-out 8/4/4), 512 leaves with U[16, 256]-token
private suffixes — one decode query per leaf. A step is one cascade decode of
the whole batch (all 512 queries, every KV head) through dd_cascade_decode.

Other workloads (--workload):
  mcts8b-e4m3, mcts8b-mxfp8   config 4: config 3 over FP8 pages
  forest70b                   config 5a: Llama-3-70B heads, 64 trees of a
                              32768-token prefix + 64 x 256-token branches,
                              trees partitioned across the ranks
  long70b                     config 5b: one tree, 131072-token prefix + 256 x
                              256-token branches, split by KV-head group across
                              the ranks; the head outputs are joined inside the
                              merge by NVLink stores into every rank's output
                              (--join p2p; the default up to 2 ranks) or by an
                              NCCL all-gather + reorder (--join nccl; the
                              default beyond)
  quant-e4m3, quant-mxfp8     config 2: quantize a 4096-page x [2][4][16][64]
                              bf16 pool (67.1 MB) with 0.1% x50 outliers

Multi-GPU (torchrun, one process per GPU): mcts8b* give every rank its own
tree (no collective; weak scaling); forest70b splits the 64 trees over the
ranks (strong scaling, no collective); long70b splits the KV heads (strong
scaling; the join and a cross-rank barrier, or an NCCL all-gather, inside
the timed region of every step). `value` is
the whole job's queries (or bytes) per second over the max-over-ranks time.

Output: one JSON line (rank 0). `--impl reference` times the reference's CPU
algorithm (the C restatement of ReferenceBackend::decode_batch, or of the FP8
quantizer, in oracle/) on the host cores instead.
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
QUANT_METRIC = "KV-page quantize HBM GB/s (config 2), vs CPU reference"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
SEED = 0xD3D1

WORKLOADS = {
    "mcts8b": dict(kind="tree", kv="bf16", tree="mcts", split="trees-per-rank",
                   desc="config 3: Llama-3-8B heads, 8192 root, depths 1-3, 512 leaves"),
    "mcts8b-e4m3": dict(kind="tree", kv="e4m3", tree="mcts", split="trees-per-rank",
                        desc="config 4: config 3 with per-head E4M3 KV pages"),
    "mcts8b-mxfp8": dict(kind="tree", kv="mxfp8", tree="mcts", split="trees-per-rank",
                         desc="config 4: config 3 with MXFP8 KV pages"),
    "forest70b": dict(kind="tree", kv="bf16", tree="forest", split="forest",
                      desc="config 5a: Llama-3-70B heads, 64 trees x (32768 prefix + 64 x 256)"),
    "long70b": dict(kind="tree", kv="bf16", tree="long", split="kv-heads",
                    desc="config 5b: Llama-3-70B heads, one tree 131072 prefix + 256 x 256, "
                         "KV-head split + all-gather"),
    "prefill8b": dict(kind="tree", kv="bf16", tree="prefill", split="trees-per-rank",
                      desc="chunked prefill of branch suffixes: Llama-3-8B heads, 8192-token shared "
                           "prefix, 16 branches x 64 new tokens (queries = new tokens)"),
    "quant-e4m3": dict(kind="quant", fmt="e4m3",
                       desc="config 2: per-head E4M3 quantize of 4096 x [2][4][16][64] bf16 pages"),
    "quant-mxfp8": dict(kind="quant", fmt="mxfp8",
                        desc="config 2: MXFP8 quantize of 4096 x [2][4][16][64] bf16 pages"),
}
QUANT_PAGES, QUANT_HKV, QUANT_D = 4096, 4, 64
E2E_MAX_STEPS = 3 + 30  # warm-up + timed steps of the end-to-end loop (e2e_time)


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


def _workloads():
    """dendrite_b200/workloads.py (pure numpy), loaded by path: importing it
    through the package would load libdendrite_b200.so, which the reference
    arm must not map."""
    import importlib.util

    name = "dendrite_b200_workloads_host"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "dendrite_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def make_tree(name: str, rank: int, world: int):
    """This rank's tree batch and the job's total query count."""
    wl = _workloads()

    w = WORKLOADS[name]
    if w["tree"] == "prefill":
        # one new token = one query over its sequence's first prefix + i + 1 tokens
        tb = wl.prefill_branches_8b(SEED + rank).nested()
        return tb, tb.batch_size * world
    if w["tree"] == "mcts":
        tb = wl.mcts_llama3_8b(SEED + rank)
        return tb, tb.batch_size * world
    if w["tree"] == "forest":
        if 64 % world:
            raise SystemExit("forest70b splits 64 trees: world size must divide 64")
        tb = wl.llama3_70b_forest(num_trees=64 // world, seed=SEED + rank)
        return tb, tb.batch_size * world
    tb = wl.llama3_70b_long(SEED)  # the same tree on every rank; heads are split
    return tb, tb.batch_size


class Clocks:
    """nvidia-smi sampler (200 ms period) around the timed region, one process
    for all of the job's GPUs (named by UUID, so CUDA_VISIBLE_DEVICES
    remapping cannot point it at another GPU; rank 0 only, so N samplers do
    not stall the ranks of a collective in turn). A reader thread collects
    the samples; `ready()` returns once the first one is in, so the timed
    steps start with the sampler running, and `stop()` waits for one sample
    taken after them (a step loop can be shorter than the period)."""

    def __init__(self, gpu_ids: str | None, out: Path | None):
        import threading

        self.proc = None
        self.path = out
        self.lines: list[str] = []
        self.t_mark = 0
        self.n_gpus = len(gpu_ids.split(",")) if gpu_ids else 1
        if gpu_ids is None:
            return
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_ids}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            if line.count(",") >= 8:
                self.lines.append(line.strip())

    def _wait_rows(self, n: int, timeout: float):
        t0 = time.time()
        while len(self.lines) < n and time.time() - t0 < timeout and self.proc.poll() is None:
            time.sleep(0.01)

    def ready(self, timeout: float = 5.0):
        """Block until the sampler has produced its first sample (one row per GPU)."""
        if self.proc:
            self._wait_rows(self.n_gpus, timeout)
            self.t_mark = len(self.lines)

    def stop(self):
        if not self.proc:
            return None
        self._wait_rows(self.t_mark + self.n_gpus, 2.0)  # a sample taken after the timed steps
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        text = "\n".join(self.lines) + "\n"
        rows = [r.split(", ") for r in self.lines]
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


# ------------------------------------------------------------ CPU baselines
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


def cpu_sample_rate(tb, pool, q_f32, budget_s: float, threads: int):
    """Reference CPU algorithm (oracle restatement of ReferenceBackend::decode_batch)
    on the first queries of the batch, its per-thread scratch allocated and
    touched before the timed calls; returns (queries/s, n queries, seconds)."""
    import oracle

    scratch = oracle.DecodeScratch(threads, tb.num_qo_heads, tb.num_kv_heads, tb.head_dim,
                                   int(np.diff(tb.indptr).max()) * 16)

    def run(n):
        ip = tb.indptr[: n + 1]
        ids = tb.block_ids[: ip[-1]]
        t0 = time.perf_counter()
        oracle.decode_batch(q_f32[:n], pool, ip, ids, tb.num_tokens[:n], tb.num_kv_heads,
                            scratch=scratch)
        return time.perf_counter() - t0

    n = min(threads, tb.batch_size)
    t = run(n)
    per = t / n
    n2 = int(max(n, min(tb.batch_size, budget_s / max(per, 1e-6))))
    n2 = max(threads, (n2 // threads) * threads) if n2 >= threads else n2
    if n2 > n:
        t = run(n2)
    else:
        n2 = n
    return n2 / t, n2, t


def host_tree_workload(name, rank, world):
    import oracle

    tb, _ = make_tree(name, rank, world)
    rng = np.random.default_rng(SEED + rank)
    pool = oracle.f32_to_bf16_bits(
        rng.standard_normal((tb.num_pages, 2, tb.num_kv_heads, 16, tb.head_dim), dtype=np.float32))
    q = oracle.f32_to_bf16_bits(
        rng.standard_normal((tb.batch_size, tb.num_qo_heads, tb.head_dim), dtype=np.float32))
    return tb, pool, q


def quant_pool_host(rank: int):
    """Config 2 pool as bf16 bits: N(0,1) with 0.1% of the elements x50."""
    import oracle

    rng = np.random.default_rng(SEED + rank)
    x = rng.standard_normal((QUANT_PAGES, 2, QUANT_HKV, 16, QUANT_D), dtype=np.float32)
    x[rng.random(x.shape) < 1e-3] *= 50.0
    return oracle.f32_to_bf16_bits(x)


def quant_bytes(fmt: str) -> int:
    """Algorithmic bytes of one config-2 quantize: bf16 pool read once, codes
    written, E8M0 exponents (MXFP8) or 2 x Hkv scales (E4M3) written."""
    n = QUANT_PAGES * 2 * QUANT_HKV * 16 * QUANT_D
    return n * 2 + n + (n // 32 if fmt == "mxfp8" else 2 * QUANT_HKV * 4)


def time_quant_cpu(pool_bits, fmt: str, budget_s: float):
    import oracle

    f = (lambda: oracle.quantize_per_head(pool_bits)) if fmt == "e4m3" else (lambda: oracle.quantize_mx(pool_bits))
    t0 = time.perf_counter()
    n = 0
    while True:
        f()
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 20:
            break
    return (time.perf_counter() - t0) / n, n


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle

    w = WORKLOADS[args.workload]
    base = {"impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "scaling": "weak", "vs_baseline": None, "data": "synthetic (seeded N(0,1))",
            "config": {"workload": args.workload, "desc": w["desc"]}}
    if w["kind"] == "quant":
        pool = quant_pool_host(0)
        for _ in range(min(args.warmup, 1)):
            time_quant_cpu(pool, w["fmt"], 0.0)
        per, n = time_quant_cpu(pool, w["fmt"], max(1.0, args.steps * 0.5))
        gbs = quant_bytes(w["fmt"]) / per / 1e9
        line = dict(base, metric=QUANT_METRIC, value=gbs, unit="GB/s", ms_per_step=per * 1e3,
                    higher_is_better=True, dtype="bf16 -> e4m3",
                    cpu_baseline={"value": gbs, "unit": "GB/s", "cores": 1, "kind": "port",
                                  "sample": f"the whole config-2 pool, {n} runs (single-threaded C oracle)"},
                    e2e={"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return
    tb, pool, qbits = host_tree_workload(args.workload, 0, 1)
    if w["kv"] != "bf16":
        codes, sc = (oracle.quantize_per_head(pool) if w["kv"] == "e4m3" else oracle.quantize_mx(pool))
        pool = oracle.dequantize(codes, sc, w["kv"])
    q = oracle.bf16_bits_to_f32(qbits)
    threads = oracle_threads(tb)
    # Each step is a bounded sample of the batch: 8 queries per thread (all
    # of them when the batch is smaller), with every worker's gather / repeat
    # scratch allocated and touched before the timed steps.
    n = min(tb.batch_size, 8 * threads)
    ip = tb.indptr[: n + 1]
    scratch = oracle.DecodeScratch(threads, tb.num_qo_heads, tb.num_kv_heads, tb.head_dim,
                                   int(np.diff(ip).max()) * 16)

    def step():
        oracle.decode_batch(q[:n], pool, ip, tb.block_ids[: ip[-1]], tb.num_tokens[:n],
                            tb.num_kv_heads, scratch=scratch)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    val = n * args.steps / dt
    sample = (f"first {n} of {tb.batch_size} queries per step ({threads} threads, scratch "
              f"preallocated), {args.steps} steps")
    line = dict(base, metric=METRIC, value=val, unit="queries/s", ms_per_step=dt / args.steps * 1e3,
                higher_is_better=True, dtype="f32",
                cpu_baseline={"value": val, "unit": "queries/s", "cores": threads, "kind": "port",
                              "sample": sample},
                e2e={"value": val, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ timing
def timed_steps(step, flush, args, world, rank, local, dev):
    """W warm-up steps, then K steps each bracketed by CUDA events on the
    current stream with an untimed L2 flush between them; barrier + sync on
    both sides; max over ranks. Returns (ms per step, launches, clocks)."""
    import torch
    import torch.distributed as dist

    from dendrite_b200 import _lib

    for _ in range(args.warmup):
        step()
        flush.zero_()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    uuid = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    uuids = [uuid]
    if world > 1:
        uuids = [None] * world
        dist.all_gather_object(uuids, uuid)
    clocks = Clocks(",".join(uuids) if rank == 0 else None,
                    Path(args.clocks_csv) if args.clocks_csv else None)
    clocks.ready()
    if world > 1:
        dist.barrier()  # rank 0 waited for the sampler: start the timed steps together
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
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
    return float(t.item()) / args.steps, int(launches), clk


def profile_kernels(step, flush, steps):
    """Per-kernel CUDA-event durations; launches run one at a time in this mode."""
    import torch

    from dendrite_b200 import _lib

    _lib.profile_enable(True)
    for _ in range(steps):
        step()
        flush.zero_()
    torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    return prof


def e2e_time(e2e_step, args, world, dev):
    import torch
    import torch.distributed as dist

    for _ in range(3):
        e2e_step()
    n = max(5, min(args.steps, 30))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(n):
        e2e_step()
    t = torch.tensor([(time.perf_counter() - t0) / n], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def pool_pages(tb) -> int:
    """Pages of the timed pool: the tree's, plus spare pages for the
    end-to-end loop, whose leaves grow a token a step."""
    return tb.num_pages + tb.batch_size * (E2E_MAX_STEPS // 16 + 2)


def device_inputs(tb, num_pages: int, seed: int, dev):
    """Seeded N(0,1) bf16 page pool [num_pages][2][Hkv][16][D] and queries
    [B][Hq][D] on the device (the parity tests of the timed configs rebuild
    them with this function)."""
    import torch

    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    pool = torch.randn((num_pages, 2, tb.num_kv_heads, 16, tb.head_dim), generator=gen, device=dev,
                       dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((tb.batch_size, tb.num_qo_heads, tb.head_dim), generator=gen, device=dev,
                    dtype=torch.float32).to(torch.bfloat16)
    return pool, q


def run_tree(args, world, rank, local, dev):
    import torch
    import torch.distributed as dist

    import dendrite_b200 as dd
    from dendrite_b200 import _lib
    from dendrite_b200 import head_split as hs
    from dendrite_b200 import workloads as wl

    w = WORKLOADS[args.workload]
    kv = w["kv"]
    heads = w["split"] == "kv-heads"
    hbm_peak, tc_peak, peak_kind = peaks()

    tb, total_queries = make_tree(args.workload, rank, world)
    Hq, Hkv, D, B = tb.num_qo_heads, tb.num_kv_heads, tb.head_dim, tb.batch_size
    num_pages = pool_pages(tb)
    pool, q = device_inputs(tb, num_pages, SEED if heads else SEED + rank, dev)
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
    cfg = dd.make_config(Hq, Hkv, D, num_pages, kv_dtype=kv_dtype)
    if heads:
        lcfg = hs.shard_config(cfg, world)
        kv_local = hs.shard_pages(kv_pages, rank, world)
        sc_local = hs.shard_scales(scales, kv_dtype, rank, world, Hkv)
        q_local = hs.shard_queries(q, cfg, rank, world)
        del pool
    else:
        lcfg, kv_local, sc_local, q_local = cfg, kv_pages, scales, q
    pb = wl.prefill_branches_8b(SEED + rank) if w["tree"] == "prefill" else None

    def make_plan():
        if pb is not None:
            return dd.CascadePlan.prefill(lcfg, pb.indptr, pb.block_ids, pb.prefix_len, pb.num_new)
        return dd.CascadePlan(lcfg, tb.indptr, tb.block_ids, tb.num_tokens, tc_sms=args.tc_sms)

    plan = make_plan()
    plan.upload(dev)
    info = plan.info()
    ws = torch.empty(max(int(info.workspace_bytes), 256), dtype=torch.uint8, device=dev)
    out_local = torch.empty_like(q_local)
    lse = torch.empty(B, lcfg.num_qo_heads, dtype=torch.float32, device=dev)
    out = torch.empty_like(q)
    gathered = torch.empty((world,) + tuple(q_local.shape), dtype=q.dtype, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    del q

    coll_ev = []  # (start, end) events around the all-gather + reorder of each step

    join = args.join if args.join != "auto" else ("p2p" if world <= 2 else "nccl")
    fused = hs.FusedHeadSplit(cfg, world, rank, B, dev) if heads and join == "p2p" else None

    def decode(plan_, q_in, evs=None):
        if fused is not None:
            # The join fused into the merge (NVLink stores into every rank's
            # output); the events bracket the cross-rank barrier after it.
            if plan_.device_buffer is None:
                plan_.upload(dev)
            from dendrite_b200.backend import _ptr, _stream
            import ctypes as C
            h = fused.handles[fused.step % 2]
            _lib.check(_lib.lib.dd_cascade_decode_shards(
                C.byref(lcfg), plan_._h, _ptr(q_in), _ptr(kv_local), _ptr(sc_local),
                C.c_void_p(int(h.buffer_ptrs_dev)), world, rank, cfg.num_qo_heads, cfg.num_kv_heads,
                _ptr(lse), _ptr(ws), ws.numel(), _stream(None)), "dd_cascade_decode_shards")
            if evs is not None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            h.barrier(channel=0)
            if evs is not None:
                e1.record()
                evs.append((e0, e1))
            r = fused.bufs[fused.step % 2]
            fused.step += 1
            return r
        dd.cascade_decode(lcfg, plan_, q_in, kv_local, sc_local, out_local, lse, ws)
        if heads:
            if evs is not None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            if world > 1:
                dist.all_gather_into_tensor(gathered, out_local)
            else:
                gathered[0].copy_(out_local)
            dd.scatter_head_shards(cfg, world, gathered, out)
            if evs is not None:
                e1.record()
                evs.append((e0, e1))
            return out
        return out_local

    def step():
        decode(plan, q_local, coll_ev if heads else None)

    ms_step, launches, clk = timed_steps(step, flush, args, world, rank, local, dev)
    coll_ms = None
    if heads:
        # All-gather + head reorder per timed step (includes waiting for the
        # slowest rank's attention), max over ranks.
        timed = coll_ev[-args.steps:]
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in timed) / max(len(timed), 1)],
                         dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        coll_ms = float(t.item())
    prof_steps = min(args.steps, 20)
    prof = profile_kernels(step, flush, prof_steps)

    # Roofline of the dominant attention kernel: bytes (streaming kernels) or
    # FLOPs (tcgen05 kernel) the plan gives it, over its average launch.
    kt = list(info.kv_tokens_by_kernel)
    Hkv_l, Hq_l = lcfg.num_kv_heads, lcfg.num_qo_heads
    per_tok = 2 * Hkv_l * (D * elem + scale_bytes)
    kernels = {}
    # Times are per step (a family may launch more than once per step: the
    # tcgen05 family is one launch per CTA size).
    for idx, name in ((0, "attn_simple"), (1, "attn_mma")):
        if prof[name][1]:
            ms_l = prof[name][0] / prof_steps
            byts = kt[idx] * per_tok + (B * Hq_l * D * 2 if idx == 1 or not kt[1] else 0)
            kernels[name] = {"bound": "hbm", "algorithmic": byts, "unit": "GB/s", "launch_ms": ms_l,
                             "achieved": byts / (ms_l * 1e-3) / 1e9, "peak": hbm_peak}
    if prof["attn_tc"][1]:
        ms_l = prof["attn_tc"][0] / prof_steps
        flops = 4.0 * D * info.tc_row_tokens
        kernels["attn_tc"] = {"bound": "tensor", "algorithmic": flops, "unit": "TFLOP/s",
                              "launch_ms": ms_l, "achieved": flops / (ms_l * 1e-3) / 1e12,
                              "peak": tc_peak}
    for k in kernels.values():
        k["frac"] = k["achieved"] / k["peak"]
    attn_kind = max(kernels, key=lambda k: kernels[k]["launch_ms"])
    dom = kernels[attn_kind]
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"{args.workload}:{attn_kind}")

    # End-to-end through the public API with host buffers: plan from the host
    # block tables (dd_plan_rebuild), H2D of the plan and the queries, decode
    # (and, for the head split, the all-gather), D2H of the output.
    q_host = q_local.cpu().pin_memory()
    res = out if heads else out_local
    out_host = torch.empty(res.shape, dtype=res.dtype).pin_memory()
    q_dev2 = torch.empty_like(q_local)
    # The engine keeps one plan object across decode steps: every leaf grows
    # by one token a step (a new block from the spare pages when its last one
    # is full) and the plan is advanced in place (dd_plan_advance), re-planned
    # from the grown tables only when that is refused. A prefill plan is
    # built anew each step.
    p2 = make_plan()
    p2.device_buffer = plan.device_buffer
    ntok_e = tb.num_tokens.astype(np.int64).copy()
    appended = [[] for _ in range(B)]
    next_spare = [tb.num_pages]
    ones = np.ones(B, np.int32)

    def grown_tables():
        lens = np.diff(tb.indptr) + np.array([len(a) for a in appended])
        ids = [np.concatenate([tb.block_ids[tb.indptr[b]:tb.indptr[b + 1]],
                               np.array(appended[b], np.uint32)]) for b in range(B)]
        return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), np.concatenate(ids), ntok_e

    # Where an end-to-end step's time goes: device intervals between events on
    # the stream (query copy, plan upload, decode, output copy) and the host's
    # planning time, summed over the steps.
    brk = {"h2d_queries": 0.0, "plan_upload": 0.0, "decode": 0.0, "d2h_output": 0.0,
           "host_plan": 0.0, "steps": 0}

    def plan_next():
        """The tree grows one token per leaf: the plan of the next step (the
        engine knows it before this step's outputs exist)."""
        nonlocal p2
        if pb is not None:
            buf = p2.device_buffer
            p2 = make_plan()
            p2.device_buffer = buf
        else:
            full = np.nonzero(ntok_e % 16 == 0)[0]
            new_block = np.zeros(B, np.uint32)
            new_block[full] = np.arange(next_spare[0], next_spare[0] + len(full))
            next_spare[0] += len(full)
            for b in full:
                appended[b].append(int(new_block[b]))
            ntok_e[:] += 1
            if not p2.advance(ones, new_block):
                p2.rebuild(*grown_tables())

    def e2e_step():
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        evs[0].record()
        q_dev2.copy_(q_host, non_blocking=True)
        evs[1].record()
        p2.upload(dev)  # asynchronous, from the plan's pinned staging copy
        evs[2].record()
        r = decode(p2, q_dev2)
        evs[3].record()
        out_host.copy_(r, non_blocking=True)
        evs[4].record()
        # The next step's plan is made on the host while this step runs on
        # the device (its upload waits for this step's copy to finish).
        th = time.perf_counter()
        plan_next()
        brk["host_plan"] += time.perf_counter() - th
        torch.cuda.synchronize()
        for k, (a, b) in zip(("h2d_queries", "plan_upload", "decode", "d2h_output"), zip(evs, evs[1:])):
            brk[k] += a.elapsed_time(b) * 1e-3
        brk["steps"] += 1
        return p2.info().device_bytes

    e2e_step_s = e2e_time(e2e_step, args, world, dev)
    plan_bytes = int(info.device_bytes)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        pool_np = kv_pages.view(torch.int16).cpu().numpy().view(np.uint16) if kv == "bf16" else \
            oracle.dequantize(kv_pages.cpu().numpy(), scales.cpu().numpy(), kv)
        qf = q_local.float().cpu().numpy()
        threads = oracle_threads(tb)
        rate, n, secs = cpu_sample_rate(tb, pool_np, qf, args.cpu_budget, threads)
        cpu = {"value": rate, "unit": "queries/s", "cores": threads, "kind": "port",
               "sample": f"first {n} of {B} queries ({secs:.1f} s, {threads} threads)"}

    if rank == 0:
        kv_bytes = info.kv_tokens * per_tok + (2 * Hkv_l * 4 if kv == "e4m3" else 0)
        eff_bytes = (kv_bytes + B * Hq_l * D * 4) * world  # every rank's share of the job
        value = total_queries / (ms_step * 1e-3)
        gbs = eff_bytes / (ms_step * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak" if w["split"] == "trees-per-rank" else "strong",
            "vs_baseline": None,
            "dtype": "bf16" if kv == "bf16" else f"{kv} KV / bf16 compute", "data": "synthetic (seeded N(0,1))",
            "config": {"workload": args.workload, "desc": w["desc"], "heads": [Hq, Hkv, D],
                       "queries": total_queries, "pages_per_rank": tb.num_pages,
                       "unique_kv_tokens_per_rank": info.kv_tokens,
                       "flat_kv_tokens_per_rank": info.kv_tokens_flat, "plan_nodes": info.num_nodes, "tc_ctas": info.tc_ctas,
                       "l2": "flushed between steps (256 MiB write, untimed)",
                       "parallelism": f"{w['split']} x{world}" + (f", join {join}" if heads else "")},
            "effective_gbs": gbs, "hbm_frac": gbs / (hbm_peak * world),
            "roofline": {"bound": dom["bound"], "kernel": attn_kind, "achieved": dom["achieved"],
                         "peak": dom["peak"], "unit": dom["unit"], "frac": dom["frac"],
                         "traffic": traffic, "peak_source": peak_kind + " (of measured)"
                         if peak_kind == "measured" else "of fallback",
                         "launch_ms": dom["launch_ms"], "algorithmic": dom["algorithmic"]},
            "kernel_rooflines": kernels,
            "kernel_ms_per_step": {k: v[0] / max(prof_steps, 1) for k, v in prof.items() if v[1]},
            "allgather_ms_per_step": coll_ms,
            "cpu_baseline": cpu,
            "e2e": {"value": total_queries / e2e_step_s, "unit": "queries/s",
                    "h2d_bytes_per_step": int(q_local.numel() * 2 + plan_bytes),
                    "d2h_bytes_per_step": int(res.numel() * 2), "ms_per_step": e2e_step_s * 1e3,
                    "breakdown_ms": {k: round(v / max(brk["steps"], 1) * 1e3, 4) for k, v in brk.items()
                                     if k != "steps"}},
            "clocks": clk, "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)


def run_quant(args, world, rank, local, dev):
    import torch

    import dendrite_b200 as dd
    from dendrite_b200 import _lib

    fmt = WORKLOADS[args.workload]["fmt"]
    hbm_peak, _, peak_kind = peaks()
    bits = quant_pool_host(rank)
    host = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).pin_memory()
    pool = host.to(dev)
    codes, scales = dd.quantize_kv_pages(pool, fmt)
    qws = torch.empty(1 << 20, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        dd.quantize_kv_pages(pool, fmt, codes=codes, scales=scales, workspace=qws)

    ms_step, launches, clk = timed_steps(step, flush, args, world, rank, local, dev)
    prof = profile_kernels(step, flush, min(args.steps, 20))
    nbytes = quant_bytes(fmt)
    qms = prof["quant"][0] / max(prof["quant"][1], 1)
    codes_host = torch.empty(codes.shape, dtype=torch.uint8).pin_memory()
    scales_host = torch.empty(scales.shape, dtype=scales.dtype).pin_memory()

    def e2e_step():
        pool.copy_(host, non_blocking=True)
        step()
        codes_host.copy_(codes, non_blocking=True)
        scales_host.copy_(scales, non_blocking=True)
        torch.cuda.synchronize()

    e2e_s = e2e_time(e2e_step, args, world, dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        per, n = time_quant_cpu(bits, fmt, args.cpu_budget)
        cpu = {"value": nbytes / per / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"the whole config-2 pool, {n} runs (single-threaded C oracle)"}
    if rank == 0:
        gbs = nbytes * world / (ms_step * 1e-3) / 1e9
        qlaunches = prof["quant"][1] / max(min(args.steps, 20), 1)
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get(f"{args.workload}:quant")
        line = {
            "metric": QUANT_METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"bf16 -> {fmt}", "data": "synthetic (seeded N(0,1), 0.1% x50 outliers)",
            "config": {"workload": args.workload, "desc": WORKLOADS[args.workload]["desc"],
                       "algorithmic_bytes": nbytes, "l2": "flushed between steps (256 MiB write, untimed)"},
            # Per step: the algorithmic bytes over all quantize launches of the
            # step (E4M3: the amax pass and the codes pass), and their DRAM
            # traffic summed (profiles/traffic.json).
            "roofline": {"bound": "hbm", "kernel": "quant", "achieved": nbytes / (qms * qlaunches * 1e-3) / 1e9,
                         "peak": hbm_peak, "unit": "GB/s",
                         "frac": nbytes / (qms * qlaunches * 1e-3) / 1e9 / hbm_peak,
                         "traffic": traffic, "per": "step (all quantize launches)",
                         "peak_source": peak_kind, "launch_ms": qms, "launches_per_step": qlaunches},
            "cpu_baseline": cpu,
            "e2e": {"value": nbytes * world / e2e_s / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": int(host.numel() * 2),
                    "d2h_bytes_per_step": int(codes.numel() + scales.numel() * scales.element_size()),
                    "ms_per_step": e2e_s * 1e3},
            "clocks": clk, "gpu_launches": launches,
        }
        print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    try:
        if WORKLOADS[args.workload]["kind"] == "quant":
            run_quant(args, world, rank, local, dev)
        else:
            run_tree(args, world, rank, local, dev)
    finally:
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
    ap.add_argument("--join", choices=["auto", "nccl", "p2p"], default="auto",
                    help="long70b: join the head shards by NCCL all-gather + reorder, or inside "
                         "the merge by NVLink stores into symmetric memory (dd_cascade_decode_shards); "
                         "auto: p2p up to 2 ranks, NCCL beyond (measured faster at 8)")
    ap.add_argument("--tc-sms", type=int, default=0,
                    help="CTAs of the tcgen05 kernel (plan option tc_sms: 0 = one per SM, "
                         "-1 = one CTA per work item)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--clocks-csv", default=None,
                    help="also write the raw nvidia-smi clock samples of the timed region here")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
