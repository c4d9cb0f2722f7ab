#!/usr/bin/env python3
"""k-NN search throughput (queries/sec) of the B200 backend, and of the
reference's CPU path on this host.

Default workload (N=1 and the scaling runs): exact cosine search, fp16 rows,
base N=2,000,000 x d=768 drawn from a Gaussian mixture (1,024 centroids
~N(0, I), per-point noise sigma=0.1, L2-normalised), Q=10,000 queries from the
same mixture, k=100. With N GPUs the base is row-sharded (contiguous ranges,
as GpuDistributedIndex's split_ids) and the per-rank top-k lists are merged by
an NCCL all-gather plus the library's merge kernel: total work is fixed, so
the scaling is strong. One step = one search of all Q queries.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl reference]

Inputs are seeded synthetic data with the configuration's shapes and value
distributions; the base (>= 2 GB) is larger than L2, so no flush is needed
between steps for the default workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "exact_fp16_cosine": dict(
        workload="exact cosine fp16, N=2,000,000 x d=768 Gaussian mixture (1,024 centroids, sigma=0.1, "
                 "L2-normalised), Q=10,000, k=100",
        n=2_000_000, d=768, q=10_000, k=100, metric="cosine", precision="fp16", data="mixture",
        centroids=1024, sigma=0.1, normalized=True, dtype="f16 (fp32 accumulate)"),
    "exact_fp32_l2": dict(
        workload="exact L2 fp32 (3xTF32), N=100,000 x d=128 N(0,1), Q=1,000, k=10",
        n=100_000, d=128, q=1_000, k=10, metric="euclidean", precision="fp32", data="gaussian",
        dtype="f32 (3xTF32)"),
    "int8_ip": dict(
        workload="int8 inner product, N=5,000,000 x d=1,024 uniform int8 [-127,127], Q=4,096, k=50, int32 accumulate",
        n=5_000_000, d=1024, q=4096, k=50, metric="dot_product", precision="int8", data="int8",
        dtype="s8 (int32 accumulate)"),
    "filtered_bf16_l2": dict(
        workload="filtered exact L2 bf16, N=1,000,000 x d=384 N(0,1), Bernoulli(0.1) row filter, query batches "
                 "of 1, 8 and 64, k=20",
        n=1_000_000, d=384, q=64, k=20, metric="euclidean", precision="bf16", data="gaussian",
        mask_p=0.1, batches=[1, 8, 64], dtype="bf16 (fp32 accumulate)"),
    "ivfpq": dict(
        workload="IVF-PQ, N=10,000,000 x d=128 Gaussian mixture (4,096 centroids, sigma=0.2, fp32), nlist=4,096 "
                 "(k-means), PQ 16 x 8 bits on residuals, nprobe=32, Q=10,000, k=10",
        n=10_000_000, d=128, q=10_000, k=10, metric="euclidean", precision="fp32", data="mixture",
        centroids=4096, sigma=0.2, normalized=False, nlist=4096, pq_dim=16, pq_bits=8, nprobe=32,
        kmeans_iters=4, dtype="f32 (u8 PQ codes)"),
    "ivf_build": dict(
        workload="IVF-PQ model build as GpuIVFPQIndex::build_from_batch (IVF k-means 4 rounds + final "
                 "assignment, PQ 16 x 8 bits trained 10 rounds on all residuals, residual codes), N=10,000,000 x "
                 "d=128 Gaussian mixture (4,096 centroids, sigma=0.2, fp32), nlist=4,096",
        n=10_000_000, d=128, q=0, k=0, metric="euclidean", precision="fp32", data="mixture",
        centroids=4096, sigma=0.2, normalized=False, nlist=4096, pq_dim=16, pq_bits=8, nprobe=32,
        kmeans_iters=4, dtype="f32 (sequential sums, no FMA)"),
    "batcher": dict(
        workload="DynamicBatcher: 64 concurrent callers of single-query exact L2 bf16 search, N=1,000,000 x "
                 "d=384 N(0,1), k=20, window 200 us, max batch 256",
        n=1_000_000, d=384, q=4096, k=20, metric="euclidean", precision="bf16", data="gaussian",
        callers=64, window_us=200, max_batch=256, dtype="bf16 (fp32 accumulate)"),
}
for _name, _c in CONFIGS.items():
    _c["name"] = _name
DEFAULT_CONFIG = "exact_fp16_cosine"
# The other configurations the default run also times, each reported under
# `workloads` in the same JSON line (with its own roofline, e2e, clocks, CPU
# baseline and parity), the headline staying the top-level value.
DEFAULT_WORKLOADS = ["exact_fp32_l2", "ivfpq", "int8_ip", "filtered_bf16_l2"]
# Queries checked against the oracle per configuration (seeded, the first of
# the batch): at least 1,000 for the large ones, every query for the small.
PARITY_QUERIES = {"exact_fp16_cosine": 1000, "ivfpq": 1000, "int8_ip": 1000, "exact_fp32_l2": 1000,
                  "filtered_bf16_l2": 64}
METRIC_NAME = "k-NN queries/sec (exact d=768 N=2M k=100; IVF-PQ) at 1/2/4/8 B200, % roofline"
CHUNK = 1 << 16
SEED = 20261201


# ----------------------------------------------------------------- data

def _centroids(cfg, device="cpu"):
    import torch
    g = torch.Generator().manual_seed(SEED)
    return torch.randn(cfg["centroids"], cfg["d"], generator=g).to(device)


def _gen_chunk(cfg, c, stream_seed, total, cents, device):
    import torch
    g = torch.Generator(device=device).manual_seed(stream_seed * 1_000_003 + c)
    rows = min(CHUNK, total - c * CHUNK)
    if cfg["data"] == "mixture":
        u = torch.randint(0, cents.shape[0], (rows,), generator=g, device=device)
        x = cents[u] + cfg["sigma"] * torch.randn(rows, cfg["d"], generator=g, device=device)
        if cfg.get("normalized"):
            x = x / x.norm(dim=1, keepdim=True)
    elif cfg["data"] == "gaussian":
        x = torch.randn(rows, cfg["d"], generator=g, device=device)
    else:
        x = torch.randint(-127, 128, (rows, cfg["d"]), generator=g, dtype=torch.int8, device=device)
    if cfg["precision"] == "fp16":
        x = x.half().float()
    elif cfg["precision"] == "bf16":
        x = x.bfloat16().float()
    return x


def gen_rows(cfg, start: int, count: int, stream_seed: int, total: int, cents=None, device="cpu"):
    """Rows [start, start+count) of a seeded table of `total` rows, generated in
    fixed 65,536-row chunks so any rank can produce any range (float32, or int8
    for the int8 configuration), on `device`. Values are rounded to the
    configuration's storage precision (fp16 / bf16) and widened back."""
    import torch
    from concurrent.futures import ThreadPoolExecutor
    c0, c1 = start // CHUNK, (start + count - 1) // CHUNK
    chunks = list(range(c0, c1 + 1))
    if str(device) == "cpu" and len(chunks) > 1:
        with ThreadPoolExecutor(max_workers=min(len(chunks), os.cpu_count() or 1)) as ex:
            parts = list(ex.map(lambda c: _gen_chunk(cfg, c, stream_seed, total, cents, device), chunks))
    else:
        parts = [_gen_chunk(cfg, c, stream_seed, total, cents, device) for c in chunks]
    out = []
    for c, x in zip(chunks, parts):
        lo = max(start, c * CHUNK) - c * CHUNK
        hi = min(start + count, c * CHUNK + x.shape[0]) - c * CHUNK
        out.append(x[lo:hi])
    return torch.cat(out).contiguous()


def gen_mask_words(cfg, total: int):
    import torch
    g = torch.Generator().manual_seed(SEED + 7)
    bits = (torch.rand(total, generator=g) < cfg["mask_p"]).numpy()
    words = np.zeros((total + 31) // 32, np.uint32)
    idx = np.nonzero(bits)[0]
    np.bitwise_or.at(words, idx >> 5, (np.uint32(1) << (idx & 31).astype(np.uint32)))
    return words


# --------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock, max clock and clock-event reasons of one GPU through
    NVML (what nvidia-smi reports) every 100 ms while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch_device: int):
        self.samples = []
        self.active = False
        self._stop = threading.Event()
        self._handle = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(torch_device).uuid)
            self._handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - depends on the box
            self.error = f"nvml unavailable: {e}"
            self.max_mhz = None

    def _run(self):
        p = self._nvml
        while not self._stop.is_set():
            try:
                sm = p.nvmlDeviceGetClockInfo(self._handle, p.NVML_CLOCK_SM)
                try:
                    reasons = p.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                except Exception:
                    reasons = p.nvmlDeviceGetCurrentClocksThrottleReasons(self._handle)
                self.samples.append((time.perf_counter(), sm, reasons, self.active))
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        if self._handle is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._handle is not None:
            self._t.join()

    def summary(self):
        if self._handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "error", "")}
        load = [s for s in self.samples if s[3]] or self.samples
        mhz = [s[1] for s in load]
        mask = 0
        for s in load:
            mask |= s[2]
        reasons = sorted(name for bit, name in self.REASONS.items() if mask & bit)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(load)}


# ------------------------------------------------------------ helpers

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic(config: str, n_shard: int):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary,
    scaled to this shard's rows when the capture was taken on a smaller case."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text()).get(config)
    if not d:
        return None
    return d["dram_bytes_per_launch"] * n_shard / d["rows"]


# ------------------------------------------------- IVF-PQ model (setup)

def _nearest_k(x, c, k):
    cn = (c * c).sum(1)
    return (cn[None, :] - 2.0 * (x @ c.T)).topk(k, dim=1, largest=False).indices


def train_ivfpq_model(cfg, base):
    """The IVF-PQ model of the base rows, built on their GPU by
    elips_b200_ivfpq_train: bit-identical to what the reference's
    GpuIVFPQIndex::build_from_batch computes (IvfIndexState::train_centroids
    with kmeans_n_iters rounds and the final assignment, then rebuild_codes:
    a 10-round PQ codebook on all residuals and the residual codes).
    Returns (centroids [nlist, d], assignments int32 [n], codebook
    [m, ksub, d/m], codes uint8 [n, m], build seconds)."""
    import torch
    from elips_b200 import train
    if not base.is_cuda:
        raise RuntimeError("the IVF-PQ model is built on a CUDA device")
    torch.cuda.synchronize(base.device)
    t = time.perf_counter()
    cent, assign, cb, codes = train.ivfpq_train_device(cfg["metric"], base, cfg["nlist"], cfg["kmeans_iters"],
                                                       cfg["pq_dim"], cfg["pq_bits"])
    torch.cuda.synchronize(base.device)
    return cent, assign, cb, codes, time.perf_counter() - t


def ivf_base_rows(cfg, dev, cents=None):
    """The seeded base rows of an IVF workload, [n, d] float32 on `dev`."""
    import torch
    n, d = cfg["n"], cfg["d"]
    cents = _centroids(cfg, dev) if cents is None else cents
    base = torch.empty((n, d), dtype=torch.float32, device=dev)
    for r0 in range(0, n, 1 << 20):
        cnt = min(1 << 20, n - r0)
        base[r0:r0 + cnt] = gen_rows(cfg, r0, cnt, SEED + 1, n, cents, device=dev)
    return base


def ivfpq_inputs(cfg, dev, train=True):
    """Seeded base rows and queries of the IVF-PQ workload and its trained
    model, all on `dev`: (base, queries, centroids, assignments, codebook,
    codes, build seconds); the model entries are None when train is False."""
    cents = _centroids(cfg, dev)
    base = ivf_base_rows(cfg, dev, cents)
    queries = gen_rows(cfg, 0, cfg["q"], SEED + 2, cfg["q"], cents, device=dev)
    if not train:
        return base, queries, None, None, None, None, None
    return (base, queries) + train_ivfpq_model(cfg, base)


def _num_sms(device):
    import torch
    return torch.cuda.get_device_properties(device).multi_processor_count


def scanned_bytes(cfg, centroids, queries, assign, lists=None):
    """Algorithmic bytes of one IVF-PQ scan: for every (query, probed list),
    each member's code (pq_dim bytes) and slot id (4 bytes); only the lists
    where `lists` (bool per list) is true when given (one GPU's share)."""
    import torch
    nprobe = min(cfg["nprobe"], centroids.shape[0])
    probes = _nearest_k(queries, centroids, nprobe)
    sizes = torch.bincount(assign.long(), minlength=centroids.shape[0])
    if lists is not None:
        sizes = sizes * torch.as_tensor(lists, device=sizes.device).to(sizes.dtype)
    return int(sizes[probes].sum().item()) * (cfg["pq_dim"] + 4)


# ------------------------------------------------------------ b200 arm

def run_b200_ivfpq(args, cfg, world, rank, local, parity_q=None):
    """IVF-PQ on one GPU, or list-sharded over N (ShardedIvfPqIndex: rank 0
    trains the model and broadcasts it with the assignments; every rank keeps
    the rows of its own lists)."""
    import torch
    from elips_b200 import _capi
    from elips_b200.distributed import ShardedIvfPqIndex, balanced_lists
    from elips_b200.ivfpq import IvfPqIndex

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, d, nq, k = cfg["n"], cfg["d"], cfg["q"], cfg["k"]
    t0 = time.perf_counter()
    base, q_dev, centroids, assign, codebook, all_codes, model_s = ivfpq_inputs(cfg, dev, train=(rank == 0))
    parity_q = 0 if args.no_parity else min(nq, parity_q if parity_q is not None else nq)
    if world > 1:
        import torch.distributed as dist
        if rank != 0:
            centroids = torch.empty((cfg["nlist"], d), dtype=torch.float32, device=dev)
            codebook = torch.empty((cfg["pq_dim"], 1 << cfg["pq_bits"], d // cfg["pq_dim"]), dtype=torch.float32,
                                   device=dev)
            assign = torch.empty((n,), dtype=torch.int32, device=dev)
        for t in (centroids, codebook, assign):
            dist.broadcast(t, src=0)
    cent_np, cb_np = centroids.cpu().numpy(), codebook.cpu().numpy()
    if world == 1:
        index = IvfPqIndex(cfg["metric"], d, cent_np, cb_np, nprobe=cfg["nprobe"], pq_bits=cfg["pq_bits"],
                           device=local)
        for r0 in range(0, n, 1 << 21):
            index.add_device(base[r0:r0 + (1 << 21)], assign[r0:r0 + (1 << 21)])
        lists = None
    else:
        # Scan cost per list = size x how often queries probe it, estimated
        # from a separate seeded sample of queries of the same distribution.
        sample = gen_rows(cfg, 0, cfg["q"], SEED + 3, cfg["q"], _centroids(cfg, dev), device=dev)
        counts = torch.bincount(_nearest_k(sample, centroids, min(cfg["nprobe"], cfg["nlist"])).flatten(),
                                minlength=cfg["nlist"])
        # 8 queries per scan item: the scan's group size at ~78 queries per list
        owner = balanced_lists(torch.bincount(assign.long(), minlength=cfg["nlist"]).cpu().numpy(), world,
                               counts.cpu().numpy(), queries_per_item=8)
        index = ShardedIvfPqIndex(cfg["metric"], d, cent_np, cb_np, cfg["nprobe"], pq_bits=cfg["pq_bits"],
                                  rank=rank, world=world, device=local, owner=owner,
                                  peer=False if args.exchange == "allgather" else None)
        for r0 in range(0, n, 1 << 21):
            index.add_device(base[r0:r0 + (1 << 21)], assign[r0:r0 + (1 << 21)], r0)
        lists = owner == rank
    alg_bytes = scanned_bytes(cfg, centroids, q_dev, assign, lists)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_r = torch.empty((nq, k), dtype=torch.int64, device=dev)
    last = [None]

    def step():
        if world == 1:
            index.search_device(q_dev, k, out_dist=out_d, out_rows=out_r)
            last[0] = (out_d, out_r)
        else:
            last[0] = index.search_device(q_dev, k)

    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        # the clock sampler's first reading, then the warm-up steps, then the
        # ranks enter the timed steps together (barrier right before them)
        time.sleep(0.25)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        _capi.profiler_reset()
        _capi.profiler_enable(True)
        launches0 = _capi.launch_count()
        sampler.active = True
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        sampler.active = False
    barrier(world)
    launches = _capi.launch_count() - launches0
    _capi.profiler_enable(False)
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    scan = _capi.profiler_stats("ivfpq_scan")
    scan_ms_max = max_over_ranks(scan["total_ms"] / max(1, scan["launches"]), world)
    allk = _capi.profiler_stats(None)
    per_kernel = {name: round(_capi.profiler_stats(name)["total_ms"] / args.steps, 4)
                  for name in ("distances", "topk_rows", "ivfpq_plan", "ivfpq_scan", "merge_topk", "ivfpq_rerank")}
    value = nq * args.steps / (ms / 1e3)
    timed = None
    if rank == 0 and parity_q and last[0] is not None and last[0][0] is not None:
        timed = (last[0][0][:parity_q].cpu().numpy(), last[0][1][:parity_q].cpu().numpy())

    q_pin = q_dev.cpu().pin_memory()
    q_np = q_pin.numpy()
    od_t = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    or_t = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    od, orr = od_t.numpy(), or_t.numpy()

    def e2e_step():
        if world == 1:
            index.search_batch(q_np, k, out_dist=od, out_rows=orr)
            return
        dd, rr = index.search_device(q_pin.to(dev, non_blocking=True), k)
        if rank == 0:
            od_t.copy_(dd, non_blocking=True)
            or_t.copy_(rr, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(world)
    t = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t, world)
    barrier(world)
    e2e = {"value": round(nq * args.steps / e2e_s, 2), "unit": "queries/s",
           "h2d_bytes_per_step": int(q_np.nbytes) * world, "d2h_bytes_per_step": int(nq * k * 12),
           "api": "elips_b200_ivfpq_search (host buffers)" if world == 1 else
                  "ShardedIvfPqIndex.search_device from pinned host queries (probe and candidate all-gathers, "
                  + ("peer-memory bounds and hand-off to the root" if index.peer is not None else
                     "NCCL all-gather of the k best") + ", merge kernels)"}

    peaks, peak_src = load_peaks()
    scan_ms = scan["total_ms"] / max(1, scan["launches"])
    achieved = alg_bytes / (scan_ms / 1e3) / 1e9
    # The lookup floor: every (query, member of a probed list) pair sums pq_dim
    # table entries read from shared memory; this layout costs 0.0655
    # wavefronts per entry (bank-conflict simulation; ncu measures 0.065-0.068)
    # at one wavefront per clock per SM.
    clk = sampler.summary()
    pairs = alg_bytes // (cfg["pq_dim"] + 4)
    lookups = pairs * cfg["pq_dim"]
    sm_hz = (clk["sm_mhz"] or 1965) * 1e6
    floor_ms = lookups * 0.0655 / (_num_sms(local) * sm_hz) * 1e3
    probed_pairs = nq * min(cfg["nprobe"], cfg["nlist"])
    lookup_floor = {"lookups": int(lookups), "wavefronts_per_lookup": 0.0655, "sm_mhz": clk["sm_mhz"],
                    "floor_ms": round(floor_ms, 3), "frac": round(floor_ms / scan_ms, 4),
                    "mean_list_rows": round(n / cfg["nlist"], 1),
                    "mean_probed_list_rows": round(pairs / max(1, probed_pairs), 1),
                    "note": "the scan's real bound: shared-memory table lookups (codes stay in L2); probed lists are "
                            "larger than the mean list (queries probe where the rows are)"}
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(peaks["hbm_gbs"], 1), "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": load_traffic(cfg["name"], n if world == 1 else index.local.size()),
                "kernel": "ivfpq_scan_kernel", "kernel_ms_avg": round(scan_ms, 4),
                "kernel_ms_max_over_ranks": round(scan_ms_max, 4),
                "kernel_share_of_step": round(scan["total_ms"] / max(1e-9, allk["total_ms"]), 4),
                "algorithmic_bytes_per_launch": alg_bytes, "per_kernel_ms_per_step": per_kernel,
                "peak_source": f"{peak_src} HBM copy bandwidth", "lookup_floor": lookup_floor}
    result = {
        "metric": METRIC_NAME, "value": round(value, 2), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": cfg["name"], "base_rows": n, "dim": d,
                   "queries_per_step": nq, "k": k, "nlist": cfg["nlist"], "nprobe": cfg["nprobe"],
                   "pq": f"{cfg['pq_dim']}x{cfg['pq_bits']}",
                   "l2": "inputs larger than L2 (codes 160 MB, vectors 5.1 GB); no flush"},
        "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline, "clocks": sampler.summary(),
        "build_s": round(build_s, 2),
        "model_build": {"s": round(model_s, 3) if model_s is not None else None, "rows": n, "nlist": cfg["nlist"],
                        "kmeans_rounds": cfg["kmeans_iters"], "pq_rounds": 10,
                        "api": "elips_b200_ivfpq_train (bit-identical to GpuIVFPQIndex::build_from_batch)"}}
    if world > 1:
        result["config"]["parallelism"] = (f"lists sharded over {world} GPUs (balanced by size x sampled probe "
                                           f"count), exchange: {'peer' if index.peer is not None else 'allgather'}")
        index.close()  # collective: unmap, then the root frees its exchange buffers
    if rank == 0 and ((not args.no_cpu_baseline and world == 1) or timed is not None):
        import oracle
        from oracle import parity
        host_base = base.cpu().numpy()
        codes = all_codes.cpu().numpy()
        a_np = assign.cpu().numpy().view(np.uint32)
        cent_np, cb_np = centroids.cpu().numpy(), codebook.cpu().numpy()
        threads = os.cpu_count() or 1
        qh = q_dev.cpu().numpy()
        del index, base
        torch.cuda.empty_cache()
        ref_answers, sample, ref_kind = None, 0, None
        if not args.no_cpu_baseline and world == 1:
            try:
                ref = oracle.RefIvfPqIndex(cfg["metric"], cent_np, a_np, cb_np, codes, host_base, cfg["nprobe"],
                                           pq_bits=cfg["pq_bits"])
                ref_kind, what = "reference", \
                    "reference GpuIVFPQIndex::search on a CPU GpuPort (import_snapshot of this model)"
                search = lambda qq, kk, tt: ref.search(qq, kk, tt)
            except Exception:
                ref_kind, what = "port", "C restatement of GpuIVFPQIndex::search"
                search = lambda qq, kk, tt: oracle.ivfpq_search(cfg["metric"], cent_np, cb_np, codes, host_base,
                                                                a_np, qq, cfg["nprobe"], kk, tt)
            sample = _calibrated_sample(search, cfg, qh, threads, target_s=10.0)
            t = time.perf_counter()
            ref_answers = search(qh[:sample], k, threads)
            dt = time.perf_counter() - t
            result["cpu_baseline"] = {"value": round(sample / dt, 3), "unit": "queries/s",
                                      "cores": min(threads, sample), "kind": ref_kind,
                                      "sample": f"{sample} of the {nq} queries over the full {n}-row "
                                      f"index ({what}), {dt:.2f} s wall"}
        if timed is not None:
            t = time.perf_counter()
            od_, or_ = oracle.ivfpq_search(cfg["metric"], cent_np, cb_np, codes, host_base, a_np, qh[:parity_q],
                                           cfg["nprobe"], k, threads, order="device")
            par = parity.bit_exact(timed[0], timed[1], od_, or_)
            par["oracle"] = ("oracle.c GpuIVFPQIndex::search restatement in the device's documented order "
                             "(approximate terms grouped per subspace, rerank-set ties by slot)")
            par["oracle_s"] = round(time.perf_counter() - t, 2)
            if ref_answers is not None and ref_kind == "reference":
                m = min(sample, parity_q)
                _, _, gap = oracle.ivfpq_search(cfg["metric"], cent_np, cb_np, codes, host_base, a_np, qh[:m],
                                                cfg["nprobe"], k, threads, order="reference", with_gap=True)
                par["vs_reference_sample"] = parity.against_reference_with_ties(
                    timed[0][:m], timed[1][:m], ref_answers[0][:m], ref_answers[1][:m], gap)
                par["pass"] = bool(par["pass"] and par["vs_reference_sample"]["pass"])
            par["what"] = "the last timed step's answers for the first queries of the batch"
            result["parity"] = par
    barrier(world)
    return result


def _peak_for(cfg, peaks, peak_src, capped, long_timed):
    """Tensor peak for this configuration's operand type: the measured bf16
    burst figure for a kernel timed alone in a short region (the regime it was
    measured in), with the sustained figure reported beside it."""
    if cfg["precision"] == "int8":
        return 2.0 * peaks["bf16_tflops"], 2.0 * peaks["bf16_tflops_sustained"], \
            f"int8 dense = 2 x {peak_src} bf16 burst"
    if cfg["precision"] == "fp32":
        return peaks["bf16_tflops"] / 2.0, peaks["bf16_tflops_sustained"] / 2.0, \
            f"tf32 dense = {peak_src} bf16 burst / 2 (3xTF32 issues 3 MMAs per counted flop)"
    note = f"{peak_src} bf16 burst" + (" (sw_power_cap was active in the timed region; the sustained "
                                        "fraction is given beside it)" if capped else "")
    return peaks["bf16_tflops"], peaks["bf16_tflops_sustained"], note


def _full_base_host(cfg, dev, cents):
    """The whole seeded base on the host (float32, int8 for the int8 codec),
    generated on `dev` in chunks: what the oracle searches."""
    n = cfg["n"]
    out = np.empty((n, cfg["d"]), np.int8 if cfg["precision"] == "int8" else np.float32)
    for r0 in range(0, n, 1 << 18):
        cnt = min(1 << 18, n - r0)
        out[r0:r0 + cnt] = gen_rows(cfg, r0, cnt, SEED + 1, n, cents, device=dev).cpu().numpy()
    return out


def exact_parity(cfg, base, queries, dist, rows, mask_words, ref_answers=None, ref_sample=0):
    """Parity of an exact search's results (dist, rows: host arrays of the
    first len(dist) queries) with the oracle (oracle.c's arithmetic, pinned to
    the reference's ExactIndex::search), plus, when given, with the
    reference's own answers for the first ref_sample queries (the CPU
    baseline's sample)."""
    import oracle
    from oracle import parity
    nq = dist.shape[0]
    q = queries[:nq]
    threads = os.cpu_count() or 1
    t = time.perf_counter()
    if cfg["precision"] == "int8":
        rd, rr = oracle.int8_ip_search_fast(base, q, cfg["k"], threads)
        out = parity.bit_exact(dist, rows, rd, rr)
        out["oracle"] = "integer restatement of the int8 inner-product codec (oracle_fast.c)"
    else:
        rd, rr = oracle.exact_search_fast(cfg["metric"], base, q, cfg["k"], threads, mask=mask_words)
        if cfg["precision"] == "fp32":
            atol = 1e-5 if cfg["metric"] == "cosine" else 0.0
            out = parity.fp32_exact(dist, rows, rd, rr,
                                    lambda qi, r: oracle.distance(cfg["metric"], q[qi], base[r]), atol=atol)
        else:
            out = parity.low_precision(dist, rows, rd, rr)
        out["oracle"] = "oracle.c ExactIndex::search arithmetic (blocked form, oracle_fast.c) on the stored " \
                        "(rounded) values"
    out["oracle_s"] = round(time.perf_counter() - t, 2)
    if ref_answers is not None and ref_sample:
        d_ref, r_ref, kind = ref_answers
        m = min(ref_sample, nq)
        out["vs_cpu_baseline_sample"] = {
            "queries": m, "recall": round(parity.recall(rows[:m], r_ref[:m]), 6),
            "max_abs_dist_err": parity._dist_err(dist[:m], d_ref[:m])[0],
            "source": ("the reference's own answers (oracle/_ref)" if kind == "reference" else
                       "the CPU restatement's answers") + " for the cpu_baseline sample"}
    return out


def run_b200(args, cfg, world, rank, local, parity_q=None):
    import torch
    from elips_b200 import ExactIndex, _capi
    from elips_b200.distributed import ReplicatedIndex, ShardedExactIndex, query_range, shard_range, slice_mask

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, d, nq, k = cfg["n"], cfg["d"], cfg["q"], cfg["k"]
    replicate = args.distributed == "replicate" and world > 1
    lo, hi = (0, n) if replicate else shard_range(n, rank, world)
    cents = _centroids(cfg, dev) if cfg["data"] == "mixture" else None
    parity_q = 0 if args.no_parity else min(nq, parity_q if parity_q is not None else nq)
    want_cpu = world == 1 and not args.no_cpu_baseline

    # ---- build: this rank's shard (or whole replica), generated on the device in chunks
    t0 = time.perf_counter()
    if replicate:
        index = ReplicatedIndex(ExactIndex(cfg["metric"], d, precision=cfg["precision"], device=local))
    else:
        index = ShardedExactIndex(cfg["metric"], d, n, precision=cfg["precision"], device=local,
                                  exchange=args.exchange)
    host_base = np.empty((hi - lo, d), np.int8 if cfg["precision"] == "int8" else np.float32) \
        if (world == 1 and (want_cpu or parity_q)) else None
    step_rows = 1 << 18
    for r0 in range(lo, hi, step_rows):
        cnt = min(step_rows, hi - r0)
        rows = gen_rows(cfg, r0, cnt, SEED + 1, n, cents, device=dev)
        if host_base is not None:
            host_base[r0 - lo:r0 - lo + cnt] = rows.cpu().numpy()
        index.add_device(rows)
        del rows
    q_dev = gen_rows(cfg, 0, nq, SEED + 2, nq, cents, device=dev)
    queries = q_dev.cpu()
    mask_words = None
    mask_dev = None
    global_mask = None
    if cfg.get("mask_p"):
        global_mask = gen_mask_words(cfg, n)
        words = global_mask
        if world > 1 and not replicate:
            words = slice_mask(words, lo, hi)  # this rank's rows, starting at bit 0
        mask_words = words
        mask_dev = torch.from_numpy(words.view(np.int32)).to(dev)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0

    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_r = torch.empty((nq, k), dtype=torch.int64, device=dev)
    last = [None]

    def step():
        if world == 1:
            index.local.search_device(q_dev, k, mask=mask_dev, out_dist=out_d, out_rows=out_r)
            last[0] = (out_d, out_r)
        else:
            last[0] = index.search_device(q_dev, k, mask=mask_dev)

    # ---- device-resident throughput (value), with the kernel profiler live
    stream = torch.cuda.current_stream(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        # the clock sampler's first reading, then the warm-up steps, then the
        # ranks enter the timed steps together (barrier right before them)
        time.sleep(0.25)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        _capi.profiler_reset()
        _capi.profiler_enable(True)
        launches0 = _capi.launch_count()
        sampler.active = True
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        sampler.active = False
    barrier(world)
    launches = _capi.launch_count() - launches0
    _capi.profiler_enable(False)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, world)
    kstats = _capi.profiler_stats("exact_topk")
    allstats = _capi.profiler_stats(None)
    ms_per_step = ms_max / args.steps
    value = nq * args.steps / (ms_max / 1e3)
    # the last timed step's answers (root rank): what the parity leg checks
    timed = None
    if last[0] is not None and last[0][0] is not None and parity_q:
        timed = (last[0][0][:parity_q].cpu().numpy(), last[0][1][:parity_q].cpu().numpy())

    # ---- end to end through the public API, host (pinned) buffers
    q_pin = queries.pin_memory()
    if world == 1:
        q_np = q_pin.numpy()
        od = torch.empty((nq, k), dtype=torch.float32).pin_memory()
        orr = torch.empty((nq, k), dtype=torch.int64).pin_memory()
        od_np, or_np = od.numpy(), orr.numpy()

        def e2e_step():
            index.local.search_batch(q_np, k, mask=mask_words, out_dist=od_np, out_rows=or_np)
    else:
        def e2e_step():
            index.search_batch(q_pin, k)
    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier(world)
    t = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t, world)
    barrier(world)
    if getattr(index, "peer", None) is not None:
        index.peer.close()  # collective: unmap, then the root frees its exchange buffers
    # sharded: every rank uploads the whole batch; replicas: each its own slice
    in_bytes = queries.numel() * queries.element_size() * (1 if replicate else world)
    if mask_words is not None:
        in_bytes += mask_words.nbytes
    e2e = {"value": round(nq * args.steps / e2e_s, 2), "unit": "queries/s",
           "h2d_bytes_per_step": int(in_bytes), "d2h_bytes_per_step": int(nq * k * (4 + 8)),
           "api": "elips_b200_exact_search (host buffers)" if world == 1 else
                  ("ReplicatedIndex.search_batch (host buffers, query slices, NCCL all-gather of the results)"
                   if replicate else
                   ("ShardedExactIndex.search_batch (host buffers; bounds shared and candidates handed to the "
                    "root over NVLink peer memory, merge kernel)" if getattr(index, "exchange", "") == "peer" else
                    "ShardedExactIndex.search_batch (host buffers, NCCL all-gather, merge kernel)"))}

    # ---- roofline of the dominant kernel (fused GEMM + top-k)
    peaks, peak_src = load_peaks()
    n_shard = hi - lo
    # queries one launch on this rank answers: the whole batch, or its slice
    nq_rank = (lambda r: r[1] - r[0])(query_range(nq, rank, world)) if replicate else nq
    clocks = sampler.summary()
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    flops = 2.0 * nq_rank * n_shard * d
    peak, peak_sus, peak_note = _peak_for(cfg, peaks, peak_src, capped, ms_max > 2000)
    avg_kernel_ms = kstats["total_ms"] / max(1, kstats["launches"])
    achieved = flops / (avg_kernel_ms / 1e3) / 1e12
    bytes_alg = n_shard * d * (2 if cfg["precision"] in ("fp16", "bf16") else (1 if cfg["precision"] == "int8" else 4))
    # The roofline is the slower of the GEMM at tensor peak and one read of
    # the base at HBM bandwidth; small query batches are bound by the latter.
    t_tensor = flops / (peak * 1e12)
    t_hbm = bytes_alg / (peaks["hbm_gbs"] * 1e9)
    if t_hbm > t_tensor:
        bound, ach, pk, unit = "hbm", bytes_alg / (avg_kernel_ms / 1e3) / 1e9, peaks["hbm_gbs"], "GB/s"
        peak_note = f"{peak_src} HBM copy bandwidth (base bytes / HBM exceeds FLOPs / tensor peak here)"
        frac_sus = None
    else:
        bound, ach, pk, unit = "tensor", achieved, peak, "TFLOP/s"
        frac_sus = round(achieved / peak_sus, 4)
    roofline = {
        "bound": bound, "achieved": round(ach, 1), "peak": round(pk, 1), "unit": unit,
        "frac": round(ach / pk, 4), "traffic": load_traffic(cfg["name"], n_shard),
        "kernel": "exact_topk_kernel", "kernel_ms_avg": round(avg_kernel_ms, 4),
        "kernel_share_of_step": round(kstats["total_ms"] / max(1e-9, allstats["total_ms"]), 4),
        "per_kernel_ms_per_step": {name: round(_capi.profiler_stats(name)["total_ms"] / args.steps, 4)
                                   for name in ("exact_topk", "merge_topk", "prep_rows")},
        "algorithmic_flops_per_launch": flops, "algorithmic_bytes_per_launch": bytes_alg,
        "hbm_time_ms_at_peak": round(bytes_alg / (peaks["hbm_gbs"] * 1e9) * 1e3, 4),
        "peak_source": peak_note}
    if frac_sus is not None:
        roofline["frac_of_sustained"] = frac_sus
        roofline["peak_sustained"] = round(peak_sus, 1)
    if world > 1:
        # where a step goes on this rank: the fused kernel, the merges, and
        # the rest (NCCL exchange, waiting for the slowest rank, glue)
        kern = kstats["total_ms"] / args.steps
        merge = _capi.profiler_stats("merge_topk")["total_ms"] / args.steps
        roofline["step_breakdown_ms"] = {
            "kernel": round(kern, 4), "kernel_max_over_ranks": round(max_over_ranks(kern, world), 4),
            "merges": round(merge, 4), "exchange_and_skew": round(ms_per_step - kern - merge, 4)}

    result = {
        "metric": METRIC_NAME, "value": round(value, 2), "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": cfg["name"], "base_rows": n, "dim": d,
                   "queries_per_step": nq, "k": k, "metric": cfg["metric"], "precision": cfg["precision"],
                   "sharding": (f"replicas: whole base on each of {world} GPUs, query batch split {world} ways"
                                if replicate else f"rows split {world} ways (contiguous ranges)")
                               if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (base >= 2 GB); no flush"
                         if n * d * 2 > 126e6 else "L2-resident base; steps back to back"},
        "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline, "clocks": clocks,
        "build_s": round(build_s, 2),
    }
    if rank == 0 and (want_cpu or parity_q):
        del index
        torch.cuda.empty_cache()
        base_np = host_base if host_base is not None else _full_base_host(cfg, dev, cents)
        ref_answers, ref_sample = None, 0
        if want_cpu:
            result["cpu_baseline"], ref_answers, ref_sample = cpu_baseline(cfg, base_np, queries.numpy(),
                                                                           global_mask)
        if timed is not None:
            result["parity"] = exact_parity(cfg, base_np, queries.numpy(), timed[0], timed[1], global_mask,
                                            ref_answers, ref_sample)
            result["parity"]["what"] = "the last timed step's answers for the first queries of the batch"
    barrier(world)
    return result


def run_b200_filtered(args, cfg, world, rank, local, parity_q=None):
    """Filtered exact search at small batches (1, 8 and 64 queries): per-call
    latency (p50 / p99, CUDA events on the launching stream) and queries/s
    for each batch, on device-resident queries, and end to end from host
    buffers (queries and the row filter copied in, results copied out)."""
    import torch
    from elips_b200 import ExactIndex, _capi
    from elips_b200.distributed import ShardedExactIndex, shard_range, slice_mask

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, d, k = cfg["n"], cfg["d"], cfg["k"]
    pool = max(cfg["batches"])
    lo, hi = shard_range(n, rank, world)
    t0 = time.perf_counter()
    index = ShardedExactIndex(cfg["metric"], d, n, precision=cfg["precision"], device=local, exchange=args.exchange)
    host_base = [] if rank == 0 and world == 1 else None
    for r0 in range(lo, hi, 1 << 18):
        rows = gen_rows(cfg, r0, min(1 << 18, hi - r0), SEED + 1, n, None, device=dev)
        if host_base is not None:
            host_base.append(rows.cpu().numpy())
        index.add_device(rows)
    q_dev = gen_rows(cfg, 0, pool, SEED + 2, pool, None, device=dev)
    queries = q_dev.cpu().numpy()
    global_mask = gen_mask_words(cfg, n)
    words = slice_mask(global_mask, lo, hi) if world > 1 else global_mask
    mask_dev = torch.from_numpy(words.view(np.int32)).to(dev)
    sel_local = int(np.unpackbits(words.view(np.uint8)).sum())
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream(dev)
    iters = max(50, 10 * args.steps)
    per_batch = {}
    answers = {}
    sampler = ClockSampler(local)
    peaks, peak_src = load_peaks()
    launches = 0
    with sampler:
        for b in cfg["batches"]:
            nbat = pool // b
            qs = [q_dev[i * b:(i + 1) * b] for i in range(nbat)]
            outs = []
            for i in range(nbat):   # warm-up, and every query of the pool answered once
                outs.append(index.search_device(qs[i], k, mask=mask_dev))
            torch.cuda.synchronize()
            if rank == 0:
                answers[b] = (torch.cat([o[0] for o in outs]).cpu().numpy(),
                              torch.cat([o[1] for o in outs]).cpu().numpy())
            barrier(world)
            _capi.profiler_reset()
            _capi.profiler_enable(True)
            l0 = _capi.launch_count()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(iters)]
            sampler.active = True
            for i in range(iters):
                evs[i][0].record(stream)
                index.search_device(qs[i % nbat], k, mask=mask_dev)
                evs[i][1].record(stream)
            torch.cuda.synchronize()
            sampler.active = False
            launches += _capi.launch_count() - l0
            _capi.profiler_enable(False)
            lat = np.array([a.elapsed_time(z) for a, z in evs])   # ms, this rank
            tot_ms = max_over_ranks(float(evs[0][0].elapsed_time(evs[-1][1])), world)
            kst = _capi.profiler_stats("exact_topk")
            kms = kst["total_ms"] / max(1, kst["launches"])
            breakdown = {name: round(_capi.profiler_stats(name)["total_ms"] / iters * 1e3, 2)
                         for name in ("mask_select", "mask_gather", "prep_rows", "exact_topk", "merge_topk")}
            # end to end from host buffers: the queries and the filter in, the results out
            qh = np.ascontiguousarray(queries[:b])
            if world == 1:
                od = torch.empty((b, k), dtype=torch.float32).pin_memory().numpy()
                orr = torch.empty((b, k), dtype=torch.int64).pin_memory().numpy()
            e2e_lat = []
            barrier(world)
            for i in range(iters):
                qh = np.ascontiguousarray(queries[(i % nbat) * b:(i % nbat + 1) * b])
                t = time.perf_counter()
                if world == 1:
                    index.local.search_batch(qh, k, mask=words, out_dist=od, out_rows=orr)
                else:
                    index.search_batch(torch.from_numpy(qh).pin_memory(), k, mask=words)
                e2e_lat.append((time.perf_counter() - t) * 1e3)
            e2e_lat = np.array(e2e_lat)
            sel_bytes = sel_local * d * 2 + words.nbytes
            full_bytes = (hi - lo) * d * 2
            per_batch[str(b)] = {
                "queries_per_s": round(b * iters / (tot_ms / 1e3), 1),
                "latency_us_p50": round(float(np.percentile(lat, 50)) * 1e3, 1),
                "latency_us_p99": round(float(np.percentile(lat, 99)) * 1e3, 1),
                "e2e_latency_us_p50": round(float(np.percentile(e2e_lat, 50)) * 1e3, 1),
                "e2e_latency_us_p99": round(float(np.percentile(e2e_lat, 99)) * 1e3, 1),
                "e2e_queries_per_s": round(b * iters / (max_over_ranks(float(e2e_lat.sum()), world) / 1e3), 1),
                "kernel_us_avg": round(kms * 1e3, 2), "device_us_per_call": breakdown,
                "hbm_frac_selected_rows": round(sel_bytes / (kms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                "hbm_frac_full_scan": round(full_bytes / (kms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                "calls": iters}
    if getattr(index, "peer", None) is not None:
        index.peer.close()
    top = per_batch[str(max(cfg["batches"]))]
    sel_rows = int(_mask_rows(global_mask, n).shape[0])
    kms_top = top["kernel_us_avg"] / 1e3
    full_b = (hi - lo) * d * 2
    result = {
        "metric": "filtered k-NN queries/sec and latency at batches 1/8/64", "value": top["queries_per_s"],
        "unit": "queries/s", "n_gpus": world, "steps": iters, "warmup": 1,
        "ms_per_step": round(1e3 * max(cfg["batches"]) / top["queries_per_s"], 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": cfg["name"], "base_rows": n, "dim": d, "k": k,
                   "batches": cfg["batches"], "selected_rows": sel_rows,
                   "sharding": f"rows split {world} ways, filter sliced per range" if world > 1 else "single GPU",
                   "l2": "base 768 MB > L2, read by every call; no flush"},
        "per_batch": per_batch,
        "e2e": {"value": per_batch[str(max(cfg["batches"]))]["e2e_queries_per_s"], "unit": "queries/s",
                "h2d_bytes_per_step": int(max(cfg["batches"]) * d * 4 + words.nbytes),
                "d2h_bytes_per_step": int(max(cfg["batches"]) * k * 12),
                "api": "elips_b200_exact_search (host buffers, row filter passed per call)" if world == 1 else
                       "ShardedExactIndex.search_batch (host buffers)"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(full_b / kms_top / 1e6, 1), "peak": round(peaks["hbm_gbs"], 1),
                     "unit": "GB/s", "frac": round(full_b / kms_top / 1e6 / peaks["hbm_gbs"], 4), "traffic": None,
                     "kernel": "exact_topk_kernel", "kernel_ms_avg": round(kms_top, 4),
                     "algorithmic_bytes_per_launch": full_b,
                     "selected_row_bytes_per_launch": int(sel_local * d * 2 + words.nbytes),
                     "frac_vs_selected_row_bytes": top["hbm_frac_selected_rows"],
                     "peak_source": f"{peak_src} HBM copy bandwidth; batch {max(cfg['batches'])}"},
        "clocks": sampler.summary(), "build_s": round(build_s, 2)}
    if rank == 0:
        del index
        torch.cuda.empty_cache()
        base_np = np.concatenate(host_base) if host_base is not None else _full_base_host(cfg, dev, None)
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"], _, _ = cpu_baseline(cfg, base_np, queries, global_mask, target_s=5.0)
        if not args.no_parity:
            par = {}
            ok = True
            for b, (dd, rr) in answers.items():
                par[str(b)] = exact_parity(cfg, base_np, queries, dd, rr, global_mask)
                bits_ok = bool(((global_mask[rr[rr >= 0] >> 5] >> (rr[rr >= 0] & 31).astype(np.uint32)) & 1).all())
                par[str(b)]["masked_rows_returned"] = not bits_ok
                ok = ok and par[str(b)]["pass"] and bits_ok
            result["parity"] = {"per_batch": par, "queries": pool, "pass": ok,
                                "what": "every query of the pool answered at each batch size"}
    barrier(world)
    return result


# ------------------------------------------------------- CPU reference

def _ref_or_port():
    import oracle
    try:
        oracle.ref()
        return oracle, "reference"
    except Exception:
        return oracle, "port"


# ------------------------------------------------------------ index build

def _build_flops(n, d, nlist, m, ksub, iters):
    """Lane operations of the assignment passes of one IVF-PQ build: 3 per
    (row, centroid, dimension) (subtract, multiply, add): max(1, iters) + 1
    IVF passes, 10 PQ rounds plus the encode pass over every subspace."""
    ivf = (max(1, iters) + 1) * n * nlist * d
    pq = 11 * n * ksub * d
    return 3.0 * (ivf + pq), 3.0 * n * nlist * d


def _reference_build_rate(cfg, base_np):
    """The reference's own build (IvfIndexState::train_centroids through
    GpuIVFFlatIndex::build_from_batch, single-threaded as it is) on a bounded
    sample at the workload's nlist and dimension: seconds per row per IVF
    assignment pass, extrapolated to the workload's build. Returns
    (rows/s, description, cores, kind)."""
    oracle, kind = _ref_or_port()
    ns = max(cfg["nlist"] * 2, 8192)
    sample = np.ascontiguousarray(base_np[:ns])
    t = time.perf_counter()
    if kind == "reference":
        oracle.ref_ivf_train(cfg["metric"], sample, cfg["nlist"], 1)
    else:
        oracle.ivf_train(cfg["metric"], sample, cfg["nlist"], 1)
    dt = time.perf_counter() - t
    per_row_pass = dt / (ns * 2)
    total, per_pass = _build_flops(cfg["n"], cfg["d"], cfg["nlist"], cfg["pq_dim"], 1 << cfg["pq_bits"],
                                   cfg["kmeans_iters"])
    passes = total / per_pass
    rate = 1.0 / (per_row_pass * passes)
    what = (f"{'reference GpuIVFFlatIndex::build_from_batch' if kind == 'reference' else 'C restatement'} "
            f"on {ns} rows, nlist {cfg['nlist']}, 1 round (2 assignment passes) in {dt:.2f} s; extrapolated to "
            f"{passes:.2f} pass-equivalents per row for the full build (PQ rounds counted by their lane "
            f"operations)")
    return rate, what, 1, kind


def run_b200_build(args, cfg):
    """Rows/s of the whole IVF-PQ model build on one GPU (device-resident rows)."""
    import torch
    from elips_b200 import _capi, train
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, d = cfg["n"], cfg["d"]
    base = ivf_base_rows(cfg, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return train.ivfpq_train_device(cfg["metric"], base, cfg["nlist"], cfg["kmeans_iters"], cfg["pq_dim"],
                                        cfg["pq_bits"])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _capi.profiler_reset()
    _capi.profiler_enable(True)
    launches0 = _capi.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(0)
    with sampler:
        time.sleep(0.25)
        sampler.active = True
        ev0.record(stream)
        for _ in range(args.steps):
            out = step()
        ev1.record(stream)
        torch.cuda.synchronize()
        sampler.active = False
    launches = _capi.launch_count() - launches0
    ms = ev0.elapsed_time(ev1)
    near = _capi.profiler_stats("nearest_centroid")
    _capi.profiler_enable(False)
    cent, asg, cb, codes = (t.cpu().numpy() for t in out)
    # e2e: the host-buffer entry point, rows copied in and the model copied out.
    host = base.cpu().numpy()
    t = time.perf_counter()
    train.ivfpq_train("euclidean", host, cfg["nlist"], cfg["kmeans_iters"], cfg["pq_dim"], cfg["pq_bits"])
    e2e_s = time.perf_counter() - t
    total, _ = _build_flops(n, d, cfg["nlist"], cfg["pq_dim"], 1 << cfg["pq_bits"], cfg["kmeans_iters"])
    near_ms = near["total_ms"] / max(1, args.steps)
    achieved = total / (near_ms / 1e3) / 1e12
    sm_max = load_peaks()[0].get("sm_max_mhz", 1965.0)
    peak = 148 * 128 * sm_max * 1e6 / 1e12
    result = {
        "metric": "IVF-PQ model build rows/s (build_from_batch semantics, bit-identical)", "value": round(n * args.steps / (ms / 1e3), 1),
        "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": args.config, "rows": n, "dim": d, "nlist": cfg["nlist"],
                   "pq": f"{cfg['pq_dim']}x{cfg['pq_bits']}", "l2": "inputs larger than L2 (rows 5.1 GB); no flush"},
        "e2e": {"value": round(n / e2e_s, 1), "unit": "rows/s", "h2d_bytes_per_step": int(host.nbytes),
                "d2h_bytes_per_step": int(cent.nbytes + asg.nbytes + cb.nbytes + codes.nbytes),
                "api": "elips_b200_ivfpq_train (host buffers)"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "fp32-simt", "achieved": round(achieved, 2), "peak": round(peak, 2),
                     "unit": "T lane-ops/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "kernel": "nearest_centroid_kernel", "kernel_ms_per_step": round(near_ms, 2),
                     "kernel_share_of_step": round(near["total_ms"] / max(1e-9, ms), 4),
                     "algorithmic_lane_ops_per_step": total,
                     "peak_source": "nominal FP32 issue rate (148 SMs x 128 lanes x max SM clock): the exact "
                                    "sequential sums cannot use FMA or tensor cores; no measured figure exists"},
        "clocks": sampler.summary()}
    if not args.no_cpu_baseline:
        rate, what, cores, kind = _reference_build_rate(cfg, host)
        result["cpu_baseline"] = {"value": round(rate, 3), "unit": "rows/s", "cores": cores, "kind": kind,
                                  "sample": what}
    return result


# ------------------------------------------------------ dynamic batching

def run_b200_batcher(args, cfg):
    """Queries/s of `callers` host threads, each issuing single-query searches
    through DynamicBatcher (host buffers in and out: the value is end to end)."""
    import threading
    import torch
    from elips_b200 import DynamicBatcher, ExactIndex, _capi
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, d, k, callers = cfg["n"], cfg["d"], cfg["k"], cfg["callers"]
    ix = ExactIndex(cfg["metric"], d, precision=cfg["precision"])
    for r0 in range(0, n, CHUNK):
        ix.add_device(gen_rows(cfg, r0, min(CHUNK, n - r0), SEED + 1, n, None, device=dev))
    queries = gen_rows(cfg, 0, cfg["q"], SEED + 2, cfg["q"], None, device=dev).cpu().numpy()
    b = DynamicBatcher(ix, window_us=cfg["window_us"], max_batch=cfg["max_batch"])
    per = max(1, args.steps)

    def drive(count):
        lat = []
        def work(t):
            for i in range(count):
                x = queries[(t * count + i) % len(queries)]
                t0 = time.perf_counter()
                b.search(x, k)
                lat.append(time.perf_counter() - t0)
        ts = [threading.Thread(target=work, args=(t,)) for t in range(callers)]
        t0 = time.perf_counter()
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return time.perf_counter() - t0, np.array(lat)

    drive(max(1, args.warmup))
    _capi.profiler_reset()
    _capi.profiler_enable(True)
    launches0 = _capi.launch_count()
    st0 = b.stats()
    sampler = ClockSampler(0)
    with sampler:
        sampler.active = True
        wall, lat = drive(per)
        sampler.active = False
    st1 = b.stats()
    kern = _capi.profiler_stats("exact_topk")
    launches = _capi.launch_count() - launches0
    _capi.profiler_enable(False)
    b.close()
    total = callers * per
    batches = st1["kernel_launches"] - st0["kernel_launches"]
    kms = kern["total_ms"] / max(1, kern["launches"])
    bytes_per_launch = n * d * 2
    achieved = bytes_per_launch / (kms / 1e3) / 1e9
    peaks, peak_src = load_peaks()
    result = {
        "metric": "k-NN queries/sec through DynamicBatcher (concurrent single-query callers)",
        "value": round(total / wall, 1), "unit": "queries/s", "n_gpus": 1, "steps": per, "warmup": args.warmup,
        "ms_per_step": round(wall / per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": args.config, "base_rows": n, "dim": d, "k": k,
                   "callers": callers, "queries_per_caller_per_run": per,
                   "l2": "base 768 MB > L2, read by every launch; no flush"},
        "e2e": {"value": round(total / wall, 1), "unit": "queries/s", "h2d_bytes_per_step": callers * d * 4,
                "d2h_bytes_per_step": callers * k * 12,
                "api": "elips_b200_batcher_search from host buffers (the value itself is end to end)",
                "latency_us_p50": round(float(np.percentile(lat, 50)) * 1e6, 1),
                "latency_us_p99": round(float(np.percentile(lat, 99)) * 1e6, 1),
                "avg_batch": round(total / max(1, batches), 2)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(peaks["hbm_gbs"], 1),
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "kernel": "exact_topk_kernel", "kernel_ms_avg": round(kms, 4),
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "peak_source": f"{peak_src} HBM copy bandwidth (small batches: the base read bounds a launch)"},
        "clocks": sampler.summary()}
    if not args.no_cpu_baseline:
        base = np.concatenate([gen_rows(cfg, r0, min(1 << 18, n - r0), SEED + 1, n, None, device=dev).cpu().numpy()
                               for r0 in range(0, n, 1 << 18)])
        result["cpu_baseline"], _, _ = cpu_baseline(cfg, base, queries, None)
    return result


def _cpu_searcher(cfg, base, mask_words):
    """Returns (search(queries, k, threads), kind, description) for the reference's
    CPU path on this configuration."""
    oracle, kind = _ref_or_port()
    metric = cfg["metric"]
    if cfg["precision"] == "int8":
        # The reference ships no int8 x int8 codec: its CPU counterpart is the
        # C restatement of the codec's definition (scalar loops, exact int32).
        return (lambda q, k, t: oracle.int8_ip_search(base, q, k, t)), "port", \
            "C restatement of the symmetric int8 inner-product codec (no reference counterpart), scalar loops"
    if mask_words is not None:
        if kind == "reference":
            sel = _mask_rows(mask_words, base.shape[0])
            idx = oracle.RefExactIndex(metric, base[sel])
            return (lambda q, k, t: idx.search(q, k, t)), kind, \
                "reference ExactIndex over the MetadataIndex::exact_candidates subset"
        return (lambda q, k, t: oracle.exact_search(metric, base, q, k, t, mask=mask_words)), kind, \
            "C restatement, masked scan"
    if kind == "reference":
        idx = oracle.RefExactIndex(metric, base)
        return (lambda q, k, t: idx.search(q, k, t)), kind, "reference ExactIndex::search (src/ExactIndex.cpp:55-87)"
    return (lambda q, k, t: oracle.exact_search(metric, base, q, k, t)), kind, "C restatement of ExactIndex::search"


def _calibrated_sample(search, cfg, queries, threads, target_s):
    """Query count (a multiple of the thread count) whose search takes about
    target_s seconds on this host."""
    first = min(queries.shape[0], threads)
    t = time.perf_counter()
    search(queries[:first], cfg["k"], threads)
    dt = max(time.perf_counter() - t, 1e-6)
    rounds = max(1, int(target_s / dt))
    return min(queries.shape[0], first * rounds)


def cpu_baseline(cfg, base, queries, mask_words, target_s=10.0):
    """The reference's CPU path timed on this host over a calibrated sample of
    the queries. Returns (cpu_baseline object, (dist, rows) of the sample,
    sample size, answers comparable with the device's); the answers are in
    the base's row numbering."""
    threads = os.cpu_count() or 1
    search, kind, what = _cpu_searcher(cfg, base, mask_words)
    sample = _calibrated_sample(search, cfg, queries, threads, target_s=target_s)
    t = time.perf_counter()
    dist, rows = search(queries[:sample], cfg["k"], threads)
    dt = time.perf_counter() - t
    if mask_words is not None and kind == "reference":
        sel = _mask_rows(mask_words, base.shape[0])
        rows = np.where(rows >= 0, sel[np.maximum(rows, 0)], -1)
    obj = {"value": round(sample / dt, 3), "unit": "queries/s", "cores": min(threads, sample), "kind": kind,
           "sample": f"{sample} of the {queries.shape[0]} queries over the full {base.shape[0]}-row base "
                     f"({what}), {dt:.2f} s wall"}
    obj_kind = kind
    return obj, (dist, rows, obj_kind), sample


def _mask_rows(mask_words, n):
    idx = np.arange(n)
    return np.nonzero((mask_words[idx >> 5] >> (idx & 31).astype(np.uint32)) & 1)[0].astype(np.int64)


def _reference_ivfpq(cfg):
    """(search, kind, description, base rows, queries) for the reference's
    GpuIVFPQIndex::search on a CPU GpuPort, the trained model imported as a
    snapshot. The rows are generated and the model built on the GPU (the
    build equals the reference's own build_from_batch bit for bit, which on
    the CPU would take hours at this size); only the search is timed."""
    import torch
    oracle, kind = _ref_or_port()
    base, q, cent, assign, cb, codes, _ = ivfpq_inputs(cfg, "cuda")
    codes = codes.cpu().numpy()
    base_np, q_np = base.cpu().numpy(), q.cpu().numpy()
    cent_np, cb_np, a_np = cent.cpu().numpy(), cb.cpu().numpy(), assign.cpu().numpy().view(np.uint32)
    del base, q, cent, assign, cb
    torch.cuda.empty_cache()
    if kind == "reference":
        idx = oracle.RefIvfPqIndex(cfg["metric"], cent_np, a_np, cb_np, codes, base_np, cfg["nprobe"],
                                   pq_bits=cfg["pq_bits"])
        return (lambda qq, kk, tt: idx.search(qq, kk, tt)), kind, \
            "reference GpuIVFPQIndex::search on a CPU GpuPort (import_snapshot of the trained model)", base_np, q_np
    return (lambda qq, kk, tt: oracle.ivfpq_search(cfg["metric"], cent_np, cb_np, codes, base_np, a_np, qq,
                                                   cfg["nprobe"], kk, tt)), kind, \
        "C restatement of GpuIVFPQIndex::search", base_np, q_np


def run_reference(args, cfg):
    """The reference's CPU implementation of the path, all host threads, one
    bounded query sample per step."""
    import torch
    if args.config == "ivfpq":
        threads = os.cpu_count() or 1
        search, kind, what, base, queries = _reference_ivfpq(cfg)
        return _time_reference(args, cfg, search, kind, what, base, queries, threads)
    if args.config == "ivf_build":
        gdev = "cuda" if torch.cuda.is_available() else "cpu"
        cents = _centroids(cfg, gdev)
        ns = max(cfg["nlist"] * 2, 8192)
        base = gen_rows(cfg, 0, ns, SEED + 1, cfg["n"], cents, device=gdev).cpu().numpy()
        rate, what, cores, kind = _reference_build_rate(cfg, base)
        return {"metric": "IVF-PQ model build rows/s (build_from_batch semantics, bit-identical)",
                "value": round(rate, 3), "unit": "rows/s", "n_gpus": args.gpus, "steps": 1, "warmup": 0,
                "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded; shapes and distributions of the configuration)",
                "config": {"workload": cfg["workload"], "config": args.config}, "impl": "reference",
                "cpu_baseline": {"value": round(rate, 3), "unit": "rows/s", "cores": cores, "kind": kind, "sample": what},
                "e2e": {"value": round(rate, 3), "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    # Data generation only (untimed): on the GPU when one is visible, else CPU.
    gdev = "cuda" if torch.cuda.is_available() else "cpu"
    cents = _centroids(cfg, gdev) if cfg["data"] == "mixture" else None
    base = np.concatenate([gen_rows(cfg, r0, min(1 << 18, cfg["n"] - r0), SEED + 1, cfg["n"], cents,
                                    device=gdev).cpu().numpy() for r0 in range(0, cfg["n"], 1 << 18)])
    queries = gen_rows(cfg, 0, cfg["q"], SEED + 2, cfg["q"], cents, device=gdev).cpu().numpy()
    if gdev == "cuda":
        torch.cuda.empty_cache()
    mask_words = gen_mask_words(cfg, cfg["n"]) if cfg.get("mask_p") else None
    threads = os.cpu_count() or 1
    search, kind, what = _cpu_searcher(cfg, base, mask_words)
    return _time_reference(args, cfg, search, kind, what, base, queries, threads)


def _time_reference(args, cfg, search, kind, what, base, queries, threads):
    sample = _calibrated_sample(search, cfg, queries, threads, target_s=1.0)
    for i in range(args.warmup):
        search(queries[:sample], cfg["k"], threads)
    t = time.perf_counter()
    for i in range(args.steps):
        j = (i * sample) % max(1, queries.shape[0] - sample + 1)
        search(queries[j:j + sample], cfg["k"], threads)
    dt = time.perf_counter() - t
    value = sample * args.steps / dt
    return {
        "metric": METRIC_NAME, "value": round(value, 3), "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; shapes and distributions of the configuration)",
        "config": {"workload": cfg["workload"], "config": args.config},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 3), "unit": "queries/s", "cores": threads, "kind": kind,
                         "sample": f"{sample} queries per step over the full {base.shape[0]}-row base ({what})"},
        "e2e": {"value": round(value, 3), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _trim(r: dict) -> dict:
    """A workload's result without the keys the enclosing line already holds."""
    drop = ("metric", "n_gpus", "steps", "warmup", "higher_is_better", "vs_baseline", "data")
    out = {"metric": r.get("metric")} if r.get("metric") != METRIC_NAME else {}
    out.update({key: v for key, v in r.items() if key not in drop})
    return out


def run_config(args, name, cfg, world, rank, local):
    if world > 1 and args.distributed == "replicate" and name in ("ivfpq", "ivf_build", "batcher",
                                                                   "filtered_bf16_l2"):
        raise SystemExit("--distributed replicate applies to the exact configurations")
    pq = args.parity_queries if args.parity_queries is not None else PARITY_QUERIES.get(name, 256)
    if world > 1:
        pq = min(pq, 256)   # rank 0 checks a smaller sample while the other ranks wait
    if name == "ivfpq":
        return run_b200_ivfpq(args, cfg, world, rank, local, pq)
    if name == "filtered_bf16_l2":
        return run_b200_filtered(args, cfg, world, rank, local, pq)
    if name in ("ivf_build", "batcher"):
        if world > 1:
            raise SystemExit(f"--config {name} runs on one GPU")
        return (run_b200_build if name == "ivf_build" else run_b200_batcher)(args, cfg)
    return run_b200(args, cfg, world, rank, local, pq)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=None, choices=sorted(CONFIGS),
                    help="time one configuration alone (default: the headline configuration, "
                         f"{DEFAULT_CONFIG}, then the workloads)")
    ap.add_argument("--workloads", default="all",
                    help="default run only: 'all', 'none', or a comma-separated list of configurations timed "
                         "after the headline and reported under `workloads`")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle comparison of the timed answers")
    ap.add_argument("--parity-queries", type=int, default=None,
                    help="queries of each timed batch checked against the oracle (default per configuration)")
    ap.add_argument("--distributed", default="shard", choices=["shard", "replicate"],
                    help="exact configurations at N>1: rows split across the GPUs (shard) or the whole base on "
                         "every GPU with the query batch split (replicate)")
    ap.add_argument("--exchange", default=None, choices=["peer", "allgather"],
                    help="row-sharded exact search at N>1: shared bounds and candidates over NVLink peer memory "
                         "(peer, the default with NCCL) or private bounds and an NCCL all-gather (allgather)")
    ap.add_argument("--base-rows", type=int, default=None,
                    help="smaller base of the same configuration (profiling captures)")
    ap.add_argument("--queries", type=int, default=None,
                    help="smaller query batch of the same configuration (profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    explicit = args.config is not None
    name = args.config or DEFAULT_CONFIG
    cfg = dict(CONFIGS[name])
    if args.base_rows:
        cfg["n"] = args.base_rows
        cfg["workload"] += f" [reduced: N={args.base_rows:,}]"
    if args.queries:
        cfg["q"] = args.queries
        cfg["workload"] += f" [reduced: Q={args.queries:,}]"
    args.config = name
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        print(json.dumps(run_reference(args, cfg)), flush=True)
        return
    if explicit:
        workloads = []
    elif args.workloads == "all":
        workloads = list(DEFAULT_WORKLOADS)
    elif args.workloads == "none":
        workloads = []
    else:
        workloads = [w for w in args.workloads.split(",") if w]
        for w in workloads:
            if w not in CONFIGS:
                raise SystemExit(f"unknown workload {w!r}")
    world, rank, local = dist_setup(args)
    try:
        result = run_config(args, name, cfg, world, rank, local)
        if workloads:
            import gc
            import torch
            result["workloads"] = {}
            for w in workloads:
                gc.collect()
                torch.cuda.empty_cache()
                t = time.perf_counter()
                try:
                    r = _trim(run_config(args, w, dict(CONFIGS[w]), world, rank, local))
                except Exception as e:  # one GPU: report it and go on; N GPUs: every rank fails alike
                    if world > 1:
                        raise
                    r = {"error": f"{type(e).__name__}: {e}"}
                r["wall_s"] = round(time.perf_counter() - t, 1)
                result["workloads"][w] = r
        if rank == 0:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
