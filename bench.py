"""Benchmark: flat PQ search queries/s on B200 (BASELINE.json metric), one JSON line on stdout (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1] [--m 16] [--impl ours|reference]

Default workload: config 1 (1M SIFT-shaped mixture vectors, d=128, PQ m=16, nq=1,000, k=10), the configuration
the reference's headline number is quoted on. With N > 1 (torchrun, one process per GPU) the database is sharded
contiguously by id: each rank searches its shard (global ids), the per-rank top-k lists are all-gathered over
NCCL and merged on the GPU by the same warp-merge kernel (strong scaling: total work fixed).

A step = one search of all nq queries: LUT build -> fused scan + top-k -> merge.
  value  device-resident: queries already in HBM, results left in HBM; CUDA events on the launching stream,
         L2 flushed (256 MB write) before every timed step, outside the events.
  e2e    the reference-facing call (vk_search: host queries in pinned memory -> host results), host<->device
         copies inside; its stage timings (CUDA events on the index's stream) give the scan kernel's duration
         for the roofline.
--impl reference: the reference's own CPU path (adc_search, built from its sources into oracle/_ref) timed on
this box's host cores on a bounded query sample of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="c1")
    p.add_argument("--m", type=int, default=None)
    p.add_argument("--n", type=int, default=None)
    p.add_argument("--nq", type=int, default=None)
    p.add_argument("--k", type=int, default=None)
    p.add_argument("--qpb", type=int, default=8, help="queries per block (Q; reduced when the LUTs do not fit)")
    p.add_argument("--ilp", type=int, default=2, help="32-row groups per warp step")
    p.add_argument("--bpq", type=int, default=0, help="vector chunks per query group (0: planned by the library)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU-baseline sample duration")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--skip-full", action="store_true", help="skip the full-scan (early_abandon=0) comparison loops")
    p.add_argument("--skip-h16", action="store_true", help="skip the half-precision LUT (lut_f16) loops")
    p.add_argument("--skip-pq4", action="store_true",
                   help="skip the 4-bit PQ block (one GPU, configs 0-2: the same rows with 16-centroid codebooks)")
    p.add_argument("--ivf-nprobe", type=int, default=16,
                   help="one GPU, configs 0-2: also an IVF search with 256 lists probing this many (0: skip)")
    p.add_argument("--no-verify", action="store_true",
                   help="N > 1: skip rank 0's search of the whole database on its GPU, which checks the merged results "
                        "bit-exactly (done by default)")
    p.add_argument("--no-coop", action="store_true",
                   help="N > 1: shards prune with their own bounds only (no bound exchange between the GPUs)")
    p.add_argument("--sharded", default="c3",
                   help="generated configuration (c3 or c4) also measured sharded by id over the run's GPUs, reported "
                        "under 'sharded'; 'none' to skip")
    p.add_argument("--sharded-steps", type=int, default=2)
    p.add_argument("--sharded-warmup", type=int, default=3)
    p.add_argument("--rerank", type=int, default=0,
                   help="one GPU: each step is the PQ search for k candidates followed by the exact re-rank of them to "
                        "this many neighbours (the reference's --rerank); reports recall@R with and without it")
    return p.parse_args()


# ------------------------------------------------------------------------------------------------ helpers
def rank_info():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled every 5 ms during the timed region.

    Reads NVML in a background thread (read-only queries); the device is found by its UUID, so the sample follows
    the CUDA device whatever CUDA_VISIBLE_DEVICES says. Without NVML it falls back to `nvidia-smi -lms 100`."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int, period_s: float = 0.005):
        self.device = device
        self.period = period_s
        self.rows = []  # (sm_mhz, max_mhz, power_w, reasons)
        self.proc = None
        self.thread = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"vk_clocks_{os.getpid()}.csv"

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            bits = {name: getattr(nv, "nvmlClocksEventReason" + key, getattr(nv, "nvmlClocksThrottleReason" + key))
                    for name, key in zip(self.NAMES, ("HwSlowdown", "HwThermalSlowdown", "SwThermalSlowdown",
                                                      "SwPowerCap"))}
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                                 getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
            max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._stop = threading.Event()

            def sample():
                mask = reasons_fn(h)
                self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), max_mhz,
                                  nv.nvmlDeviceGetPowerUsage(h) / 1e3, [n for n, b in bits.items() if mask & b]))

            def loop():
                while not self._stop.is_set():
                    try:
                        sample()
                    except Exception:
                        pass
                    self._stop.wait(self.period)

            sample()  # fail here, not in the thread, if NVML cannot be read
            self.rows.clear()
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            rows = self.rows
            source = "nvml"
        elif self.proc is not None:
            self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            rows = []
            for line in self.path.read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].replace(".", "").isdigit():
                    rows.append((float(f[1]), float(f[2]) if f[2].replace(".", "").isdigit() else float("nan"),
                                 float(f[3]) if f[3].replace(".", "").isdigit() else float("nan"),
                                 [self.NAMES[i] for i in range(4) if f[5 + i].lower() == "active"]))
            self.path.unlink(missing_ok=True)
            source = "nvidia-smi"
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source (NVML, nvidia-smi)"]}
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted({x for r in rows for x in r[3]}), "samples": len(rows), "source": source,
                "power_w_max": round(max(r[2] for r in rows), 1)}


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the default scan kernel, from ncu
# captures of these workloads on one B200 (1-pass dram and duration metrics of the scan kernel). Keyed by
# (config, rows scanned per GPU, m, nq, k); a run whose shard matches no capture reports the bytes scaled from the
# capture of the same config by rows (codes and placement bytes grow with rows, LUT bytes with nq), marked scaled.
NCU_TRAFFIC = {
    ("c1", 1_000_000, 16, 1000, 10): {"dram_bytes_per_launch": 33_659_136, "kernel": "scan_kernel<8,16,2,1,16,1>"},
    ("c3", 10_000_000, 16, 1000, 10): {"dram_bytes_per_launch": 196_180_000, "kernel": "scan_kernel<8,16,2,1,16,1>"},
    # ncu prints this capture in GB / MB with two decimals (windowed item order: 16.75 GB read + 188.51 MB written)
    ("c3", 100_000_000, 16, 10_000, 10): {"dram_bytes_per_launch": 16_938_510_000, "kernel": "scan_kernel<8,16,2,1,16,1>"},
}


def ncu_traffic(config, rows, m, nq, k):
    hit = NCU_TRAFFIC.get((config, rows, m, nq, k))
    if hit:
        return dict(hit, captured=True)
    for (c, r, mm, q, kk), v in NCU_TRAFFIC.items():
        if c == config and mm == m and q == nq and kk == k:
            lut = nq * m * 256 * 4
            per_row = (v["dram_bytes_per_launch"] - lut) / r
            return {"dram_bytes_per_launch": int(lut + per_row * rows), "kernel": v["kernel"], "captured": False,
                    "scaled_from_rows": r}
    return None


def lookup_wavefront_model(codes: np.ndarray, Q: int, sample_rows: int = 1 << 17) -> float:
    """Mean shared-memory wavefronts per warp-wide LUT fetch for these codes under the scan kernel's layout
    ([s][c][Q] entries: LDS.32 / .64 / .128 for Q = 1 / 2 / 4 and 8; 32 consecutive rows per warp instruction):
    per phase of 32 / 16 / 8 lanes, the max over 128-byte bank groups of distinct entries addressed."""
    n, m = codes.shape
    rows = min(n, sample_rows) // 32 * 32
    c = codes[:rows].reshape(-1, 32, m).astype(np.int64)  # [warps, lanes, m]
    lanes_per_phase = {1: 32, 2: 16, 4: 8, 8: 8}[Q]
    entry_banks = {1: 1, 2: 2, 4: 4, 8: 4}[Q]
    groups = 32 // entry_banks
    total = 0.0
    for ph in range(32 // lanes_per_phase):
        cc = c[:, ph * lanes_per_phase:(ph + 1) * lanes_per_phase, :]  # [warps, lanes, m]
        bank = cc % groups
        # distinct entries per bank group: count unique codes per (warp, s, bank)
        key = (cc * groups + bank)  # unique code implies unique key
        w, l, s = key.shape
        k2 = np.sort(key.transpose(0, 2, 1).reshape(-1, l), axis=1)
        distinct = np.ones_like(k2, dtype=bool)
        distinct[:, 1:] = k2[:, 1:] != k2[:, :-1]
        b2 = k2 % groups
        load = np.zeros((k2.shape[0], groups), np.int64)
        np.add.at(load, (np.repeat(np.arange(k2.shape[0]), l), b2.ravel()), distinct.ravel())
        total += load.max(axis=1).mean()
    return total  # wavefronts per warp instruction (all phases)


# ------------------------------------------------------------------------------------------------ workload
def build_workload(args, rank: int, world: int):
    """This rank's shard of the configuration (generated row range only; same codebooks on every rank)."""
    from veckern_b200 import configs
    from veckern_b200.shard import shard_of

    spec = configs.spec(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k)
    sh = shard_of(spec["n"], world, rank)
    w = configs.make(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k, encode=gpu_encoder(),
                     train=gpu_trainer(), rows=(sh.lo, sh.hi))
    return spec, w, sh


def gpu_encoder():
    from veckern_b200.data import gpu_encoder as enc
    return enc()


def gpu_trainer():
    from veckern_b200.data import gpu_trainer as tr
    return tr()


# ------------------------------------------------------------------------------------------------ reference arm
def usable_cores() -> int:
    """Host threads this process may run on (its CPU affinity), the reference CPU path's thread count."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference's own CPU search (adc_search, oracle/_ref) with every usable host thread, on a bounded query
    sample per step. The workload is built without this repository's libraries: inputs by the numpy restatement of
    the configuration's generators (oracle/inputs.py), codebook and codes by the reference's own ProductQuantizer.
    At N = 1 it also runs the reference's own GPU kernel (v8, FusedWarp, compiled for sm_100a from its sources) on
    the same inputs over its tuning sweep (key reference_gpu_v8)."""
    rank, world, _ = rank_info()
    if rank != 0:
        return
    cores = usable_cores()
    # torchrun exports OMP_NUM_THREADS=1; libgomp reads the variable when it loads, which happens below
    os.environ["OMP_NUM_THREADS"] = str(cores)
    import oracle
    from veckern_b200.configs import spec as config_spec  # a plain dict: loads no library

    s = config_spec(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k)
    kind = "reference" if oracle.ref_available() else "port"
    t_setup = time.perf_counter()
    pq = None
    if kind == "reference" and s["kind"] in ("normal", "mixture"):
        from oracle import inputs
        R = oracle.ref()
        threads = R.set_threads(cores)
        pq, codes, queries = inputs.reference_workload(s, R)
        centroids = pq.centroids
        inputs_by = "numpy generators (oracle/inputs.py) + the reference's ProductQuantizer train/encode"
        run = lambda q: R.adc_search(pq, codes, q, s["k"])  # noqa: E731
    else:
        from veckern_b200 import configs
        w = configs.make(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k)
        if w.codes is None:
            from veckern_b200 import data
            w.codes = data.gen_codes(s["code_seed"], w.cdf, 0, s["n"])
        centroids, codes, queries = w.centroids, w.codes, w.queries
        inputs_by = "the package's host generators"
        if kind == "reference":
            R = oracle.ref()
            threads = R.set_threads(cores)
            pq = R.pq(s["d"], s["m"])
            pq.centroids = centroids
            run = lambda q: R.adc_search(pq, codes, q, s["k"])  # noqa: E731
        else:
            P = oracle.port()
            threads = cores
            run = lambda q: P.adc_search(centroids, codes, q, s["k"], cores)  # noqa: E731
    setup_s = time.perf_counter() - t_setup
    nq = s["nq"]
    probe_n = max(1, min(cores, nq))
    t0 = time.perf_counter()
    run(queries[:probe_n])
    per_q = (time.perf_counter() - t0) / probe_n
    per_step = 60.0 / max(1, args.steps + args.warmup)  # the whole reference run stays near one minute
    sample = int(max(1, min(nq, per_step / max(per_q, 1e-9))))
    for i in range(args.warmup):
        run(queries[:sample])
    times, counts = [], []
    cpu_res = None
    for i in range(args.steps):
        q0 = (i * sample) % nq
        qs = queries[q0:q0 + sample]
        t0 = time.perf_counter()
        res = run(qs)
        times.append(time.perf_counter() - t0)
        counts.append(qs.shape[0])
        if i == 0:
            cpu_res = (q0, res)
    qps = float(np.sum(counts)) / float(np.sum(times)) if times else 0.0
    line = {"impl": "reference", "metric": "queries/s", "value": round(qps, 3), "unit": "queries/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * float(np.mean(times)), 3) if times else None, "higher_is_better": True,
            "config": {"workload": workload_name(s, args.config), "n": s["n"], "m": s["m"], "nq_sample": sample,
                       "k": s["k"]},
            "dtype": "f32", "data": "synthetic",
            "cpu_baseline": {"value": round(qps, 3), "unit": "queries/s", "cores": threads, "kind": kind,
                             "sample": f"{sample} of {nq} queries per step, full database of {s['n']} rows",
                             "inputs": inputs_by, "setup_s": round(setup_s, 1)},
            "e2e": {"value": round(qps, 3), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if world == 1 and pq is not None:
        line["reference_gpu_v8"] = reference_gpu_v8(centroids, codes, queries, s, cpu_res)
    print(json.dumps(finite(line)), flush=True)


def reference_gpu_v8(centroids, codes, queries, s, cpu_res):
    """The reference's final kernel (FusedWarp through its own PQSearcher, searcher.cu compiled for sm_100a) on the
    same inputs: its default tuning and the best point of its own queries_per_block x ilp sweep
    (scripts/run_all.sh:87-91), each the median of 5 searches after a warm-up (bench/bench_main.cpp:191-214).
    q/s = nq / (transfer + lut + scan + select), the reference's own definition. ids_equal_cpu: share of the
    (query, rank) ids equal to the reference CPU path on the timed CPU sample (its v8 regroups additions)."""
    import oracle
    if not oracle.refgpu_available():
        return {"unavailable": "oracle/_ref/libveckern_refgpu.so not built (needs the reference sources)"}
    if s["m"] % 16 != 0:
        return {"unavailable": "the reference's v8 requires m % 16 == 0"}
    try:
        import torch
        if not torch.cuda.is_available():
            return {"unavailable": "no GPU"}
        name = torch.cuda.get_device_name(0)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"torch: {e}"}
    points = [(2, 4)] + [(q, ilp) for q in (1, 2, 4, 8) for ilp in (1, 2, 4)]
    try:
        rows, (vd, vi) = oracle.refgpu_sweep(centroids, codes, queries, s["k"], points, reps=5)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": str(e)}
    nq = queries.shape[0]

    def summary(r):
        return {"queries/s": round(nq / (r["total_ms"] / 1e3), 1), "total_ms": round(r["total_ms"], 4),
                "scan_ms": round(r["scan_ms"], 4), "lut_ms": round(r["lut_ms"], 4),
                "select_ms": round(r["select_ms"], 4), "transfer_ms": round(r["transfer_ms"], 4),
                "queries_per_block": int(r["queries_per_block"]), "ilp": int(r["vectors_per_step"]),
                "blocks_x": int(r["blocks_x"]), "grid_y": int(r["grid_y"])}
    best = min(rows[1:], key=lambda r: r["total_ms"])
    out = {"device": name, "default_tuning": summary(rows[0]), "best_of_sweep": summary(best),
           "sweep_points": len(points) - 1}
    if cpu_res is not None:
        q0, (cd, ci) = cpu_res
        out["ids_equal_cpu"] = round(float(np.mean(vi[q0:q0 + ci.shape[0]] == ci)), 6)
        out["ids_equal_cpu_queries"] = int(ci.shape[0])
    return out


def finite(x):
    """NaN / inf (e.g. full-scan figures under --skip-full) become null, so the line is strict JSON."""
    if isinstance(x, dict):
        return {k: finite(v) for k, v in x.items()}
    if isinstance(x, list):
        return [finite(v) for v in x]
    if isinstance(x, float) and not np.isfinite(x):
        return None
    return x


def workload_name(s, cfg):
    return f"{cfg}: flat PQ search n={s['n']:,} d={s['d']} m={s['m']} nq={s['nq']:,} k={s['k']}"


# ------------------------------------------------------------------------------------------------ our arm
def wavefront_floor(codes_sample: np.ndarray, perm: np.ndarray, Q: int, lookups: float, sm_count: int,
                    sm_mhz: float):
    """(wavefronts per fetch in the index's placement, the same in row order, floor ms) of a full scan: the
    conflict-inclusive shared-memory wavefronts of `lookups` lookup-adds at one wavefront per clock per SM."""
    full = codes_sample.shape[0] // 64 * 64
    placed = np.concatenate([codes_sample[(np.arange(full) & ~63) + perm[:full]], codes_sample[full:]])
    wf = lookup_wavefront_model(placed, Q)
    wf_rows = lookup_wavefront_model(codes_sample, Q)
    per_fetch = 4 if Q >= 4 else Q  # lookups served per warp LUT fetch per lane
    floor_ms = lookups / 32.0 / per_fetch * wf / (sm_count * sm_mhz * 1e6) * 1e3
    return wf, wf_rows, floor_ms


class ShardExchange:
    """This rank's side of a cooperative sharded search (N > 1 unless --no-coop): the shards' scans lower each
    other's pruning bounds with posted atomics over NVLink (vk_search_device_coop), exchange arrays mapped across
    the rank processes with CUDA IPC handles (all-gathered once). Every rank calls search() in the same order, so
    the epochs agree. close() only after all ranks have synchronised: no rank's kernel may still write into this
    rank's memory."""

    def __init__(self, args, world: int, local: int, nq: int):
        self.coop = None
        self.active = False
        self.epoch = 0
        if world > 1 and not args.no_coop:
            import torch.distributed as dist

            from veckern_b200 import CoopSearch, VkError
            self.coop = CoopSearch(local, nq)
            handles = [None] * world
            dist.all_gather_object(handles, self.coop.ipc_handle())
            try:
                self.coop.attach_ipc(handles)
                self.active = True
            except VkError as e:  # e.g. GPUs without a link that carries atomics: search this shard alone
                print(f"bound exchange unavailable: {e}", file=sys.stderr, flush=True)

    def search(self, s, d_q, k, d_out, stream, tuning=None):
        if not self.active:
            s.search_device(d_q, k, d_out, stream, tuning=tuning)
        else:
            self.epoch += 1
            s.search_device_coop(self.coop, self.epoch, d_q, k, d_out, stream, tuning=tuning)

    def close(self):
        if self.coop is not None:
            self.coop.close()
            self.coop = None
            self.active = False


def run_sharded(args, rank: int, world: int, local: int, stream, flush):
    """A generated configuration (default c3: 100M rows, m 16, nq 10,000, k 10) sharded contiguously by id over the
    run's ranks, each shard's codes generated on its GPU: every rank searches its shard, the per-shard top-k lists are
    all-gathered over NCCL and merged on the GPU. Every rank takes the same collective steps; rank 0 returns the
    block of the JSON line (None elsewhere). Steps are timed with CUDA events on the launching stream, L2 flushed
    before each, max over ranks."""
    import torch
    import torch.distributed as dist

    from veckern_b200 import PQSearcher, Tuning, configs, data, device_info, merge_topk_device
    from veckern_b200.shard import gather_and_merge, shard_of

    name = args.sharded
    w = configs.make(name)
    spec = w.spec
    n, m, nq, k = spec["n"], spec["m"], spec["nq"], spec["k"]
    sh = shard_of(n, world, rank)
    tuning = Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp)
    s = PQSearcher.generated(w.centroids, spec["code_seed"], w.cdf, sh.lo, sh.rows, device=local, id_base=sh.lo)
    s.set_tuning(tuning)
    d_q = torch.from_numpy(w.queries).cuda()
    d_local = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    d_gather = torch.empty((world, nq, k), dtype=torch.int64, device="cuda") if world > 1 else None
    d_final = torch.empty((nq, k), dtype=torch.int64, device="cuda") if world > 1 else d_local
    shx = ShardExchange(args, world, local, nq)

    def exchange():
        def merge(buf, lay):
            merge_topk_device(local, buf, nq, lay["lists"], lay["k_in"], lay["query_stride"], lay["list_stride"], k,
                              d_final, stream)
        gather_and_merge(d_local, d_gather, nq, k, lambda buf, x: dist.all_gather_into_tensor(buf, x), merge)

    for _ in range(args.sharded_warmup):
        shx.search(s, d_q, k, d_local, stream)
        if world > 1:
            exchange()
    s.sync(stream)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.sharded_steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for e in evs:
        flush.zero_()
        e[0].record(stream)
        shx.search(s, d_q, k, d_local, stream)
        e[1].record(stream)
        if world > 1:
            exchange()
        e[2].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s.sync(stream)
    clk = clocks.stop()
    total = sum(a.elapsed_time(c) for a, b, c in evs)
    search = sum(a.elapsed_time(b) for a, b, c in evs)
    t = torch.tensor([total, search, -search], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_max, search_max, search_min = t[0].item(), t[1].item(), -t[2].item()

    verified = None
    if world > 1 and not args.no_verify:
        if rank == 0:  # one GPU over the whole database: the merged result must be identical
            with PQSearcher.generated(w.centroids, spec["code_seed"], w.cdf, 0, n, device=local) as one:
                one.set_tuning(tuning)
                ref = torch.empty((nq, k), dtype=torch.int64, device="cuda")
                one.search_device(d_q, k, ref, stream)
                one.sync(stream)
            verified = bool(torch.equal(ref, d_final))
        dist.barrier()
        if rank == 0 and not verified:
            raise SystemExit(f"{name}: multi-GPU merged result differs from the single-GPU search")

    out = None
    if rank == 0:
        K = max(1, args.sharded_steps)
        info = device_info(local)
        sm_mhz = clk.get("sm_mhz") or info.clock_mhz
        search_ms = search_max / K
        Q = min(args.qpb, 8)
        sample = data.gen_codes(spec["code_seed"], w.cdf, sh.lo, min(1 << 17, sh.rows))
        wf, wf_rows, floor_ms = wavefront_floor(sample, s.get_placement(sample.shape[0]), Q,
                                                float(nq) * sh.rows * m, info.sm_count, sm_mhz)
        out = {"workload": workload_name(spec, name) + f", sharded by id over {world} GPU(s)",
               "metric": "queries/s", "value": round(nq / (total_max / K / 1e3), 2), "unit": "queries/s",
               "ms_per_step": round(total_max / K, 3), "steps": args.sharded_steps, "warmup": args.sharded_warmup,
               "shards": world, "rows_per_gpu": sh.rows, "queries_per_block": tuning.queries_per_block,
               "search_ms_per_gpu": {"max": round(search_max / K, 3), "min": round(search_min / K, 3)},
               "exchange_ms": round((total_max - search_max) / K, 3) if world > 1 else 0.0,
               "lookup_floor": {"wavefronts_per_fetch": round(wf, 3), "wavefronts_per_fetch_row_order": round(wf_rows, 3),
                                "floor_ms_per_gpu": round(floor_ms, 3),
                                "frac": round(floor_ms / search_ms, 4),
                                "note": "full scan's conflict-inclusive shared-memory wavefronts of this shard at one "
                                        "per clock per SM, against the per-GPU search time (LUT + pruned scan + "
                                        "list merge)"},
               "hbm": {"code_bytes_per_gpu": int(sh.rows * m),
                       "traffic": ncu_traffic(name, sh.rows, m, nq, k), "peak_gbs_measured": _peak("hbm_gbs")},
               "bound_exchange": shx.active,
               "verified_against_single_gpu": verified, "clocks": clk,
               "l2": "flushed (256 MB write) before every timed step"}
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # no rank's scan may still write into this rank's exchange array
    shx.close()
    s.close()
    del d_q, d_local, d_gather, d_final
    torch.cuda.empty_cache()
    return out


def run_pq4(args, spec, exact_ids, stream, flush, local, sm_mhz):
    """4-bit PQ over the same database rows (one GPU): 16 centroids per sub-space at twice the sub-spaces (m = 32
    for config 1: the 8-bit index's 16 code bytes per row), trained by the same steps on the same sample. Device-
    resident steps timed like the headline, pruned (default) and full scan; the scan kernel's time from the stage
    events. A 4-bit LUT fetch never conflicts (one 128-byte table per query pair and sub-space, one LDS.64 serves
    64 lookups in 2 wavefronts), so its lookup floor is the shared-memory bandwidth itself. Recall@k of both
    indexes against exact L2 neighbours on a query sample."""
    import torch

    from veckern_b200 import PQSearcher, Tuning, configs, device_info, device_result_split
    m4 = 2 * spec["m"]
    t0 = time.perf_counter()
    w4 = configs.make_pq4(args.config, m=m4, n=args.n, nq=args.nq, k=args.k, keep_base=True)
    build_s = time.perf_counter() - t0
    nq, k, n = spec["nq"], spec["k"], spec["n"]
    res = {}
    with PQSearcher(w4.centroids, w4.codes, device=local) as s4:
        d_q = torch.from_numpy(w4.queries).cuda()
        out = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        h_q = np.ascontiguousarray(w4.queries)
        for name, prune in (("pruned", True), ("full", False)):
            s4.set_tuning(Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp, early_abandon=prune))
            for _ in range(args.warmup):
                s4.search_device(d_q, k, out, stream)
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps)]
            for e in ev:
                flush.zero_()
                e[0].record(stream)
                s4.search_device(d_q, k, out, stream)
                e[1].record(stream)
            torch.cuda.synchronize()
            s4.sync(stream)
            ms = sum(a.elapsed_time(b) for a, b in ev) / max(1, args.steps)
            scan = []
            for i in range(args.warmup + args.steps):
                flush.zero_()
                _, t = s4.search(h_q, k)
                if i >= args.warmup:
                    scan.append(t.scan_ms)
            res[name] = (ms, float(np.mean(scan)))
            if prune:
                ids4 = device_result_split(out)[1].cpu().numpy()
                Q = s4.last_launch().queries_per_block
    info = device_info(local)
    lookups = float(nq) * n * m4
    peak = 128.0 * info.sm_count * sm_mhz * 1e6
    sample = min(nq, 100)
    truth = exact_topk(torch.from_numpy(w4.base).cuda(), torch.from_numpy(w4.queries[:sample]).cuda(), k)
    ids8 = device_result_split(exact_ids)[1].cpu().numpy()
    recall = lambda ids: float(np.mean([len(set(a) & set(b)) / k for a, b in zip(ids[:sample], truth)]))  # noqa: E731
    ms, scan_ms = res["pruned"]
    full_ms, full_scan_ms = res["full"]
    return {"value": round(nq / (ms / 1e3), 1), "unit": "queries/s", "ms_per_step": round(ms, 4),
            "scan_kernel_ms": round(scan_ms, 4), "m": m4, "code_bytes_per_row": m4 // 2, "queries_per_block": Q,
            "full_scan": {"value": round(nq / (full_ms / 1e3), 1), "ms_per_step": round(full_ms, 4),
                          "scan_kernel_ms": round(full_scan_ms, 4)},
            "roofline": {"bound": "smem", "unit": "GB/s", "peak": round(peak / 1e9, 1),
                         "achieved": round(lookups * 4 / (scan_ms / 1e3) / 1e9, 1),
                         "frac": round(lookups * 4 / (scan_ms / 1e3) / peak, 4),
                         "full_scan_frac": round(lookups * 4 / (full_scan_ms / 1e3) / peak, 4)},
            "recall_at_k_vs_exact_l2": {"k": k, "queries": sample, "pq4": round(recall(ids4), 4),
                                        "pq8_headline_index": round(recall(ids8), 4)},
            "build_s": round(build_s, 2),
            "note": "4-bit PQ (vk_index_create_pq4): 16 centroids per sub-space, two sub-codes per byte, fp32 LUTs, "
                    "bit-exact against its CPU restatement; achieved = 4 B x nq*n*m lookups / scan-kernel time, "
                    "peak = 128 B/clk/SM x SMs x median SM clock (conflict-free fetches: the floor is the peak)"}


def run_ivf(args, w, spec, exact_ids, stream, flush, local):
    """IVF search over the same database (one GPU): 256 lists whose coarse centroids are trained by the device PQ
    trainer with m = 1 (the reference's Lloyd iterations over whole vectors) on the configuration's training
    sample, rows assigned to the nearest; each query probes --ivf-nprobe lists. Device-resident steps timed like
    the headline; recall = share of the exact flat search's top-k ids it returns."""
    import torch

    from veckern_b200 import IVFSearcher, Tuning, assign_lists, data, device_result_split
    n, d, nq, k = spec["n"], spec["d"], spec["nq"], spec["k"]
    t0 = time.perf_counter()
    train = data.gen_mixture(spec["mix_seed"], spec["mix_seed"], min(spec.get("train_rows", n), n), d) \
        if spec["kind"] == "mixture" else data.gen_normal(spec["data_seed"], min(n, 100_000), d)
    coarse = data.pq_train_gpu(train, 1, 10, spec.get("pq_seed", 1)).reshape(256, d)
    lists = np.empty(n, np.int32)
    step = 1 << 20
    for a in range(0, n, step):
        b = min(n, a + step)
        x = data.gen_mixture(spec["mix_seed"], spec["mix_seed"], b - a, d, row0=a) if spec["kind"] == "mixture" \
            else data.gen_normal(spec["data_seed"], b - a, d, row0=a)
        lists[a:b] = assign_lists(x, coarse, local)
    nprobe = args.ivf_nprobe
    with IVFSearcher(w.centroids, w.codes, coarse, lists, device=local) as ivf:
        build_s = time.perf_counter() - t0
        ivf.set_tuning(Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp))
        d_q = torch.from_numpy(w.queries).cuda()
        out = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        for _ in range(args.warmup):
            ivf.search_device(d_q, k, nprobe, out, stream)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e in ev:
            flush.zero_()
            e[0].record(stream)
            ivf.search_device(d_q, k, nprobe, out, stream)
            e[1].record(stream)
        torch.cuda.synchronize()
        ivf.sync(stream)
        ms = sum(a.elapsed_time(b) for a, b in ev) / max(1, args.steps)
        ids = device_result_split(out)[1].cpu().numpy()
    ids_x = device_result_split(exact_ids)[1].cpu().numpy()
    recall = float(np.mean([len(set(a) & set(b)) / k for a, b in zip(ids, ids_x)]))
    sizes = np.bincount(lists, minlength=256)
    return {"value": round(nq / (ms / 1e3), 1), "unit": "queries/s", "ms_per_step": round(ms, 4), "nlist": 256,
            "nprobe": nprobe, "recall_vs_flat": round(recall, 5),
            "list_rows": {"min": int(sizes.min()), "median": int(np.median(sizes)), "max": int(sizes.max())},
            "build_s": round(build_s, 2),
            "note": "IVF search (vk_ivf_*): the flat search restricted to the rows of each query's nprobe nearest "
                    "lists, bit-exact against its CPU restatement; recall_vs_flat = share of the exact flat "
                    "search's top-k ids it returns"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from veckern_b200 import PQSearcher, Tuning, device_info, merge_topk_device

    rank, world, local = rank_info()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    spec, w, sh = build_workload(args, rank, world)
    n, m, nq, k = spec["n"], spec["m"], spec["nq"], spec["k"]
    lo, hi = sh.lo, sh.hi
    tuning = Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp, blocks_per_query=args.bpq)
    if w.codes is not None:
        s = PQSearcher(w.centroids, w.codes, device=local, id_base=lo)
    else:
        s = PQSearcher.generated(w.centroids, spec["code_seed"], w.cdf, lo, hi - lo, device=local, id_base=lo)
    s.set_tuning(tuning)

    stream = torch.cuda.current_stream()
    d_q = torch.from_numpy(w.queries).cuda()
    d_local = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    d_gather = torch.empty((world, nq, k), dtype=torch.int64, device="cuda") if world > 1 else None
    d_final = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    from veckern_b200.shard import gather_and_merge
    shx = ShardExchange(args, world, local, nq)

    def exchange():
        """One all-gather of the per-shard lists over NCCL, then the GPU merge into d_final."""
        def merge(buf, lay):
            merge_topk_device(local, buf, nq, lay["lists"], lay["k_in"], lay["query_stride"], lay["list_stride"], k,
                              d_final, stream)
        gather_and_merge(d_local, d_gather, nq, k, lambda buf, x: dist.all_gather_into_tensor(buf, x), merge)

    def step_device(tun=None):
        shx.search(s, d_q, k, d_local, stream, tuning=tun)
        if world > 1:
            exchange()

    for _ in range(args.warmup):
        step_device()
    s.sync(stream)
    torch.cuda.synchronize()

    # ---- value: device-resident steps
    clocks = ClockSampler(local)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        step_device()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s.sync(stream)
    dev_ms = sum(a.elapsed_time(b) for a, b in ev)
    exact_ids = (d_final if world > 1 else d_local).clone()

    # ---- the same steps with early abandoning off (full scan of every (query, row, sub-space) lookup)
    full_tuning = Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp, blocks_per_query=args.bpq,
                         early_abandon=False)
    for _ in range(0 if args.skip_full else args.warmup):
        step_device(full_tuning)
    torch.cuda.synchronize()
    ev_full = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    for i in range(0 if args.skip_full else args.steps):
        flush.zero_()
        ev_full[i][0].record(stream)
        step_device(full_tuning)
        ev_full[i][1].record(stream)
    torch.cuda.synchronize()
    s.sync(stream)
    full_ms = float("nan") if args.skip_full else sum(a.elapsed_time(b) for a, b in ev_full)

    # ---- the same steps with half-precision LUTs (VK_LUT_F16: approximate, exactly defined; recall reported)
    h16_tuning = Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp, blocks_per_query=args.bpq,
                        lut_f16=True)
    h16_ok = m in (16, 32, 64) and not args.skip_h16
    for _ in range(args.warmup if h16_ok else 0):
        step_device(h16_tuning)
    torch.cuda.synchronize()
    ev_h16 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    for i in range(args.steps if h16_ok else 0):
        flush.zero_()
        ev_h16[i][0].record(stream)
        step_device(h16_tuning)
        ev_h16[i][1].record(stream)
    torch.cuda.synchronize()
    s.sync(stream)
    h16_ms = sum(a.elapsed_time(b) for a, b in ev_h16) if h16_ok else float("nan")
    h16_ids = (d_final if world > 1 else d_local).clone() if h16_ok else None

    # ---- e2e. N = 1: the host-buffer C-ABI call (vk_search: H2D, LUT, scan, merge, D2H), its stage events giving
    # the scan kernel's time. N > 1: the pinned host queries copied to the device, this rank's shard search (with
    # the bound exchange), the all-gather + merge, and the merged result copied back to pinned host memory.
    h_q_t = torch.from_numpy(w.queries).pin_memory()
    h_q = h_q_t.numpy()
    from veckern_b200 import NEIGHBOR_DTYPE
    h_out = torch.empty((nq, k), dtype=torch.int64).pin_memory().numpy().view(NEIGHBOR_DTYPE)
    h_final = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    d_q2 = torch.empty_like(d_q)
    e2e_ms, scan_ms, lut_ms, sel_ms = [], [], [], []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        if world == 1:
            t0.record(stream)
            _, t = s.search(h_q, k, out=h_out)  # synchronous: H2D, LUT, scan, merge, D2H
            t1.record(stream)
        else:
            ta = torch.cuda.Event(enable_timing=True)
            tb = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            d_q2.copy_(h_q_t, non_blocking=True)
            ta.record(stream)
            shx.search(s, d_q2, k, d_local, stream)
            tb.record(stream)
            exchange()
            h_final.copy_(d_final, non_blocking=True)
            t1.record(stream)
        torch.cuda.synchronize()
        total = t0.elapsed_time(t1)
        if i >= args.warmup:
            e2e_ms.append(total)
            if world == 1:
                scan_ms.append(t.scan_ms)
                lut_ms.append(t.lut_ms)
                sel_ms.append(t.select_ms)
            else:  # LUT + scan + merge of the shard: its scan dominates
                scan_ms.append(ta.elapsed_time(tb))
                lut_ms.append(float("nan"))
                sel_ms.append(float("nan"))
    # scan-kernel duration of the full scan, from the same stage events (one GPU)
    s.set_tuning(full_tuning)
    full_scan_ms = [float("nan")] if args.skip_full or world > 1 else []
    for i in range(0 if args.skip_full or world > 1 else args.warmup + args.steps):
        flush.zero_()
        _, t = s.search(h_q, k, out=h_out)
        if i >= args.warmup:
            full_scan_ms.append(t.scan_ms)
    h16_scan_ms = [float("nan")]
    if h16_ok and world == 1:
        s.set_tuning(h16_tuning)
        h16_scan_ms = []
        for i in range(args.warmup + args.steps):
            flush.zero_()
            _, t = s.search(h_q, k, out=h_out)
            if i >= args.warmup:
                h16_scan_ms.append(t.scan_ms)
    s.set_tuning(tuning)
    clk = clocks.stop()

    verified = None
    if not args.no_verify and world > 1:
        # the gathered + merged result of the last device step against one GPU over the whole database
        shx.search(s, d_q, k, d_local, stream)
        exchange()
        torch.cuda.synchronize()
        if rank == 0:
            from veckern_b200 import configs
            full = configs.make(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k, encode=gpu_encoder(),
                                train=gpu_trainer())
            one = (PQSearcher(full.centroids, full.codes, device=local) if full.codes is not None else
                   PQSearcher.generated(full.centroids, spec["code_seed"], full.cdf, 0, n, device=local))
            with one:
                one.set_tuning(tuning)
                ref = torch.empty((nq, k), dtype=torch.int64, device="cuda")
                one.search_device(d_q, k, ref, stream)
                one.sync(stream)
            verified = bool(torch.equal(ref, d_final))
            if not verified:
                raise SystemExit("multi-GPU merged result differs from the single-GPU search")
        dist.barrier()

    dev_ms_t = torch.tensor([dev_ms, float(np.sum(e2e_ms)), float(np.mean(scan_ms)), full_ms,
                             float(np.mean(full_scan_ms)), h16_ms, float(np.mean(h16_scan_ms))], device="cuda")
    if world > 1:
        dist.all_reduce(dev_ms_t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_total, scan_mean, full_ms, full_scan_mean, h16_ms, h16_scan_mean = dev_ms_t.tolist()
    h16_block = None
    ivf_block = None
    if world == 1 and args.ivf_nprobe > 0 and spec["kind"] in ("mixture", "normal") and m in (16, 32):
        ivf_block = run_ivf(args, w, spec, exact_ids, stream, flush, local)
    pq4_block = None
    if world == 1 and not args.skip_pq4 and spec["kind"] in ("mixture", "normal") and 2 * m in (16, 32, 64):
        pq4_block = run_pq4(args, spec, exact_ids, stream, flush, local, clk.get("sm_mhz") or 1965.0)
    if h16_ok and rank == 0:
        from veckern_b200 import device_result_split
        ids_h = device_result_split(h16_ids)[1].cpu().numpy()
        ids_x = device_result_split(exact_ids)[1].cpu().numpy()
        recall = float(np.mean([len(set(a) & set(b)) / k for a, b in zip(ids_h, ids_x)]))
        h16_block = {"value": round(nq / (h16_ms / args.steps / 1e3), 1), "unit": "queries/s",
                     "ms_per_step": round(h16_ms / args.steps, 4), "scan_kernel_ms": round(h16_scan_mean, 4),
                     "recall_vs_fp32": round(recall, 5),
                     "note": "half-precision LUTs (lut_precision = VK_LUT_F16): per-query power-of-two scale, "
                             "entries rounded to half, fp32 sums; bit-exact against its CPU restatement; "
                             "recall_vs_fp32 = share of the exact search's top-k ids it returns"}

    if rank == 0:
        ms_step = dev_ms / args.steps
        value = nq / (ms_step / 1e3)
        e2e_value = nq / (e2e_total / args.steps / 1e3)
        info = device_info(local)
        sm_mhz = clk.get("sm_mhz") or info.clock_mhz
        lookups = float(nq) * (hi - lo) * m  # per rank (rank 0's shard) per launch
        achieved = lookups / (scan_mean / 1e3)
        smem_peak_bytes = 128.0 * info.sm_count * sm_mhz * 1e6
        if world > 1:  # the shard searches above ran on the device path: one untimed host call records the plan
            s.search(np.ascontiguousarray(w.queries), k)
        Q = s.last_launch().queries_per_block
        sample = 1 << 17
        if w.codes is not None:
            rows_codes = w.codes[:sample]
        else:  # generated configs: the shard's first rows, regenerated on the host
            from veckern_b200 import data as vkdata
            rows_codes = vkdata.gen_codes(spec["code_seed"], w.cdf, lo, min(sample, hi - lo))
        # the device layout: rows of whole 64-row windows in the index's lane placement
        wf, wf_rows, floor_ms = wavefront_floor(rows_codes, s.get_placement(rows_codes.shape[0]), Q, lookups,
                                                info.sm_count, sm_mhz)
        roofline = {
            "bound": "smem",
            "achieved": round(achieved * 4 / 1e9, 1), "peak": round(smem_peak_bytes / 1e9, 1), "unit": "GB/s",
            "frac": round(achieved * 4 / smem_peak_bytes, 4),
            "traffic": ncu_traffic(args.config, hi - lo, m, nq, k),
            "note": ("achieved = algorithmic LUT bytes (4 B per (query, row, sub-space) lookup, nq*n*m per launch) / "
                     "scan-kernel event time; peak = shared-memory bandwidth 128 B/clk/SM x SMs x median SM clock "
                     "sampled under load. lookup_floor: time the full scan's conflict-inclusive LDS wavefronts need "
                     "(bank-conflict model of these codes in the index's lane placement, one wavefront per clock "
                     "per SM; wavefronts_per_fetch_row_order: the same codes in row order); the default kernel "
                     "abandons most pairs early, so it can beat that floor"),
            "lookup_floor": {"wavefronts_per_fetch": round(wf, 3) if wf else None,
                             "wavefronts_per_fetch_row_order": round(wf_rows, 3) if wf_rows else None,
                             "floor_ms": round(floor_ms, 4) if floor_ms else None,
                             "kernel_ms": round(scan_mean, 4),
                             "frac": round(floor_ms / scan_mean, 4) if floor_ms else None,
                             "full_scan_kernel_ms": round(full_scan_mean, 4),
                             "full_scan_frac": round(floor_ms / full_scan_mean, 4) if floor_ms else None},
            "hbm": {"code_bytes_per_launch": int((hi - lo) * m), "peak_gbs_measured": _peak("hbm_gbs")},
        }
        cpu = None if args.no_cpu_baseline else cpu_baseline(args, w, spec)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # no rank's scan may still write into this rank's exchange array
    bound_exchange = shx.active
    shx.close()
    sharded = None
    if args.sharded not in ("none", args.config):
        s.close()
        sharded = run_sharded(args, rank, world, local, stream, flush)
    if rank == 0:
        line = {
            "metric": "queries/s", "value": round(value, 1), "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name(spec, args.config), "n": n, "d": spec["d"], "m": m, "nq": nq,
                       "k": k, "queries_per_block": Q, "vectors_per_step": s.last_launch().vectors_per_step,
                       "shards": world, "l2": "flushed (256 MB write) before every timed step",
                       "bound_exchange": bound_exchange,
                       "parallelism": f"id-sharded x{world}" if world > 1 else "single GPU"},
            "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                    "h2d_bytes_per_step": int(w.queries.nbytes), "d2h_bytes_per_step": int(nq * k * 8),
                    "stages_ms": {"lut": round(float(np.mean(lut_ms)), 4), "scan": round(scan_mean, 4),
                                  "select": round(float(np.mean(sel_ms)), 4)}},
            "lut_f16": h16_block,
            "ivf": ivf_block,
            "pq4": pq4_block,
            "full_scan": {"value": round(nq / (full_ms / args.steps / 1e3), 1), "unit": "queries/s",
                          "ms_per_step": round(full_ms / args.steps, 4), "scan_kernel_ms": round(full_scan_mean, 4),
                          "note": "early abandoning off: every (query, row, sub-space) lookup executed"},
            "gpu_launches": args.steps * (3 + (1 if world > 1 else 0)),
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "verified_against_single_gpu": verified,
            "sharded": sharded,
        }
        print(json.dumps(finite(line)), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _peak(key):
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()).get(key)
    except Exception:
        return None


def cpu_baseline(args, w, spec):
    """The reference's adc_search on this host, bounded to about --cpu-seconds of work (rank 0, N = 1 only)."""
    import oracle

    if int(os.environ.get("WORLD_SIZE", 1)) > 1:
        return None
    cores = usable_cores()
    if w.codes is None:  # generated database: the C port streams host-regenerated codes for one query
        from veckern_b200 import data
        P = oracle.port()
        lut = P.compute_lut(w.centroids, w.queries[:1])
        n = spec["n"]
        rows = min(n, int(args.cpu_seconds * 4e6))  # bounded sample of the database (~args.cpu_seconds)
        block = 1 << 22
        t0 = time.perf_counter()
        P.stream_search(lut, ((data.gen_codes(spec["code_seed"], w.cdf, a, min(block, rows - a)), a)
                              for a in range(0, rows, block)), spec["k"], cores)
        dt = time.perf_counter() - t0
        return {"value": round(rows / n / dt, 4), "unit": "queries/s", "cores": cores, "kind": "port",
                "sample": f"1 query over the first {rows:,} of {n:,} rows (codes regenerated on the host, "
                          f"{dt:.1f} s), scaled to the full database"}
    kind = "reference" if oracle.ref_available() else "port"
    if kind == "reference":
        R = oracle.ref()
        cores = R.set_threads(cores)
        pq = R.pq(spec["d"], spec["m"])
        pq.centroids = w.centroids
        run = lambda q: R.adc_search(pq, w.codes, q, spec["k"])  # noqa: E731
    else:
        P = oracle.port()
        run = lambda q: P.adc_search(w.centroids, w.codes, q, spec["k"], cores)  # noqa: E731
    t0 = time.perf_counter()
    run(w.queries[:cores])
    per_q = (time.perf_counter() - t0) / cores
    sample = int(max(cores, min(spec["nq"], args.cpu_seconds / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    run(w.queries[:sample])
    dt = time.perf_counter() - t0
    return {"value": round(sample / dt, 2), "unit": "queries/s", "cores": cores, "kind": kind,
            "sample": f"{sample} of {spec['nq']} queries over the full {spec['n']:,}-row database ({dt:.1f} s)"}


def exact_topk(base, queries, k, chunk=1 << 20):
    """Ground truth for recall: exact squared L2 in float64 on the GPU (torch), k smallest ids per query."""
    import torch
    q = queries.double()
    qn = (q * q).sum(1, keepdim=True)
    best_d = torch.full((q.shape[0], k), float("inf"), dtype=torch.float64, device=q.device)
    best_i = torch.full((q.shape[0], k), -1, dtype=torch.int64, device=q.device)
    for a in range(0, base.shape[0], chunk):
        xb = base[a:a + chunk].double()
        dist = qn - 2.0 * q @ xb.T + (xb * xb).sum(1)[None, :]
        d2 = torch.cat([best_d, dist], 1)
        i2 = torch.cat([best_i, torch.arange(a, a + xb.shape[0], device=q.device).expand(q.shape[0], -1)], 1)
        best_d, idx = torch.topk(d2, k, dim=1, largest=False)
        best_i = torch.gather(i2, 1, idx)
    return best_i.cpu().numpy()


def run_rerank(args):
    """PQ search for spec k candidates + exact GPU re-rank to args.rerank neighbours, on one GPU (config 2 is the
    reference's re-ranking candidate pass, bench_main.cpp:146-153)."""
    import torch

    from veckern_b200 import PQSearcher, Tuning, device_result_split, rerank_device
    from veckern_b200 import configs

    torch.cuda.set_device(0)
    spec = configs.spec(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k)
    w = configs.make(args.config, n=args.n, m=args.m, nq=args.nq, k=args.k, keep_base=True, encode=gpu_encoder(),
                     train=gpu_trainer())
    nq, r, k = spec["nq"], spec["k"], args.rerank
    s = PQSearcher(w.centroids, w.codes, device=0)
    s.set_tuning(Tuning(queries_per_block=args.qpb, vectors_per_step=args.ilp))
    d_base = torch.from_numpy(w.base).cuda()
    d_q = torch.from_numpy(w.queries).cuda()
    d_cand = torch.empty((nq, r), dtype=torch.int64, device="cuda")
    d_out = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        s.search_device(d_q, r, d_cand, stream)
        rerank_device(0, d_base, d_q, d_cand, k, d_out, stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    s.sync(stream)
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    sample = min(nq, 100)
    truth = exact_topk(d_base, d_q[:sample], k)
    pq_ids = device_result_split(d_cand)[1][:sample, :k].cpu().numpy()
    rr_ids = device_result_split(d_out)[1][:sample].cpu().numpy()
    recall = lambda ids: float(np.mean([len(set(a) & set(b)) / k for a, b in zip(ids, truth)]))  # noqa: E731
    line = {"metric": "queries/s", "value": round(nq / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload_name(spec, args.config) + f" + exact re-rank of {r} candidates to {k}",
                       "l2": "flushed (256 MB write) before every timed step"},
            "recall_at_k": {"k": k, "queries": sample, "pq_only": round(recall(pq_ids), 4),
                            "with_rerank": round(recall(rr_ids), 4),
                            "truth": "exact squared L2 in float64 over all rows"}}
    print(json.dumps(finite(line)), flush=True)
    s.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.rerank:
        run_rerank(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
