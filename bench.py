"""Benchmark of the paged MLA decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload sharded|mla32]

Workload "sharded" (default; the configuration the headline metric is quoted
on at 1/2/4/8 GPUs): 1024 sequences with context lengths log-uniform in
512..65536 (seed 4), a bf16 MLA latent cache of 576-value entries (512 latent
+ 64 rope) in 64-token pages whose physical order is a random permutation,
128 absorbed query heads, softmax scale 1/sqrt(192).  Sequences are sharded
over the N ranks by longest-processing-time on their lengths; each rank holds
only its sequences.  One step = append one new token to every sequence
(quantise/convert on append) + paged MLA decode over all its tokens (split
across the SMs, with the split-KV combine).  Total work is fixed as N grows
("strong" scaling).  Workload "mla32": 32 sequences x 4096 tokens, seed 1.

value: KV tokens attended per second over all ranks, inputs resident in HBM,
timed with CUDA events on the launching stream (max over ranks).  e2e: the
same step through ct_attn_mla_decode_step_host with the queries and new
tokens in pinned host memory and the outputs copied back every step.
roofline: the decode launch (MLA kernel + split-KV combine) against the
measured HBM copy bandwidth; algorithmic bytes = 1152 B per attended token +
queries + outputs.  cpu_baseline / --impl reference: the reference's own
ct_attn_forward (oracle/_ref, compiled from the reference sources) over the
same pages gathered to fp32, on a bounded sample of the workload, all host
threads.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

E, DV, H, PAGE = 576, 512, 128, 64
SCALE = float(1.0 / np.sqrt(192.0))
BYTES_PER_TOKEN = E * 2
METRIC = "decode KV tokens/s and achieved HBM GB/s vs ~8 TB/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def workload(name):
    """(lengths as stored in the cache before the step, description)."""
    if name == "mla32":
        lens = np.full(32, 4096 - 1, np.int64)
        desc = "MLA paged decode, 32 seqs x 4096 tokens (after the appended token), seed 1"
        seed = 1
    else:
        lens = lengths_loguniform(1024, 512, 65536, seed=4)
        desc = ("sequence-sharded MLA serving: 1024 seqs, context log-uniform 512..65536 (seed 4), "
                "one append + decode per seq")
        seed = 4
    return lens, desc, seed


GOLDEN = 0x9E3779B97F4A7C15
MASK64 = (1 << 64) - 1


def synth_key(seed, stream):
    """Key of the seeded synthetic stream (seed, stream): the library's
    ct_synth_key rule (csrc/synth.cu) restated in Python, so that the workload
    can be derived without loading any native library (the reference arm
    must not load this repository's)."""
    return splitmix((seed * GOLDEN + splitmix(stream + 0x632BE59BD9B4E019)) & MASK64)


def lengths_loguniform(n, lo, hi, seed):
    """Same rule as the oracle's generator (ct_oracle.c: floor(lo*(hi/lo)^u))."""
    key = synth_key(seed, 0)
    out = np.empty(n, np.int64)
    for s in range(n):
        z = splitmix(key + (s + 1) * 0x9E3779B97F4A7C15)
        u = (z >> 11) * (1.0 / 9007199254740992.0)
        t = np.floor(lo * np.exp(u * np.log(hi / lo)))
        out[s] = int(min(max(t, lo), hi))
    return out


def splitmix(z):
    m = (1 << 64) - 1
    z &= m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def physical_gpu(dev):
    """nvidia-smi index of CUDA device `dev` (CUDA_VISIBLE_DEVICES remaps)."""
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        ids = [x.strip() for x in cvd.split(",") if x.strip()]
        if dev < len(ids) and ids[dev].isdigit():
            return int(ids[dev])
    return dev


def measured_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(workload_name):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "mla_decode_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload_name)
    except Exception:
        return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of one GPU, read through
    NVML every 5 ms by a thread that runs across the timed region (reads
    only; no setting is changed).  Falls back to `nvidia-smi -lms` when NVML
    cannot be loaded."""

    NAMES = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []          # (sm MHz, reason bits)
        self.smax = None
        self.stop_flag = threading.Event()
        self.t = None

    def start(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self.nvml = N
            self.handle = N.nvmlDeviceGetHandleByIndex(self.gpu)
            self.smax = float(N.nvmlDeviceGetMaxClockInfo(self.handle, N.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:      # live before the timed region starts
                time.sleep(0.001)
            return
        except Exception:
            self.nvml = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _poll(self):
        N = self.nvml
        get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            N.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag.is_set():
            try:
                self.samples.append((float(N.nvmlDeviceGetClockInfo(self.handle, N.NVML_CLOCK_SM)),
                                     int(get_reasons(self.handle))))
            except Exception:
                return
            time.sleep(0.005)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            n0 = len(self.samples)
            t0 = time.time()
            while len(self.samples) == n0 and time.time() - t0 < 1.0:  # one sample after the region
                time.sleep(0.001)
            self.stop_flag.set()
            self.t.join(timeout=2)
            sm = [c for c, _ in self.samples]
            bits = 0
            for _, b in self.samples:
                bits |= b
            reasons = sorted(n for n, m in self.NAMES.items() if bits & m)
            return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.smax, "reasons": reasons,
                    "samples": len(sm), "source": "nvml, 5 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = list(self.NAMES)
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 100 ms"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import cautreo_b200 as ct

    torch.cuda.set_device(local_rank)
    dev = local_rank
    L = ct.lib()
    lens_all, desc, seed = workload(args.workload)
    n_all = len(lens_all)
    rank_of = ct.lpt_shard(lens_all.astype(np.uint32), world) if world > 1 else np.zeros(n_all, np.int32)
    mine = np.nonzero(rank_of == rank)[0]
    lens = lens_all[mine]                               # tokens cached before the step
    n = len(mine)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    # ---- cache: pages for len+1 tokens, physical order permuted ----
    pages = ((lens + 1) + PAGE - 1) // PAGE
    n_pages = int(pages.sum())
    max_pages = int(pages.max())
    kv = ct.PagedKV(n, max_pages, n_pages, PAGE, E, 0, ct.CT_KV_BF16, dev, sp)
    perm = np.random.default_rng(seed * 1000 + rank).permutation(n_pages).astype(np.int32)
    kv.set_free_order(perm)
    kv.append(list(range(n)), (lens + 1).tolist(), None)          # reserve slots for len + 1 tokens
    rows = torch.arange(n, dtype=torch.int32, device="cuda")
    lens_dev = torch.from_numpy(lens.astype(np.int32)).cuda()
    ct.check(L.ct_synth_fill_paged(kv.pool, None, ct.CT_KV_BF16, kv.block_table_dev, max_pages, rows.data_ptr(),
                                   lens_dev.data_ptr(), n, int(lens.max()), PAGE, E, ct.synth_key(seed, 10), 0, 1.0,
                                   sp), "fill")
    bt = kv.block_table()
    dest = np.array([bt[i, lens[i] // PAGE] * PAGE + lens[i] % PAGE for i in range(n)], np.int32)
    dest_dev = torch.from_numpy(dest).cuda()
    # ---- step inputs ----
    q = torch.empty(n * H * E, dtype=torch.int16, device="cuda")
    new_tok = torch.empty(n * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(q.data_ptr(), 0, ct.synth_key(seed, 11), rank << 40, n * H * E, 0, 1.0, sp))
    ct.check(L.ct_synth_fill(new_tok.data_ptr(), 0, ct.synth_key(seed, 13), rank << 40, n * E, 0, 1.0, sp))
    out = torch.empty(n * H * DV, dtype=torch.int16, device="cuda")
    att = (lens + 1).astype(np.int64)
    plan = ct.MlaPlan(att.astype(np.int32), n_pages, max_pages_per_seq=max_pages, device=dev)
    torch.cuda.synchronize()

    def step():
        ct.check(L.ct_kv_paged_write_slots(kv.pool, None, ct.CT_KV_BF16, new_tok.data_ptr(), ct.CT_KV_BF16,
                                           dest_dev.data_ptr(), n, E, sp))
        ct.check(L.ct_attn_mla_decode_paged(plan.h, q.data_ptr(), kv.pool, None, kv.block_table_dev,
                                            kv.seq_lens_dev, out.data_ptr(), None, sp))

    group = dist.group.WORLD if world > 1 else None

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def append_call():
        ct.check(L.ct_kv_paged_write_slots(kv.pool, None, ct.CT_KV_BF16, new_tok.data_ptr(), ct.CT_KV_BF16,
                                           dest_dev.data_ptr(), n, E, sp))

    def decode_call():
        ct.check(L.ct_attn_mla_decode_paged(plan.h, q.data_ptr(), kv.pool, None, kv.block_table_dev,
                                            kv.seq_lens_dev, out.data_ptr(), None, sp))

    for _ in range(args.warmup):
        step()
    barrier()
    # A serving loop replays the step as CUDA graphs (one for the append, one
    # for the decode + combine): the same kernels and arguments as the calls
    # above, without a host enqueue per launch.  Launches are counted at
    # capture and multiplied by the replays.
    graphs = None
    launches_per_step = 0
    if not args.no_graph:
        try:
            g = (torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph())
            l0 = ct.launch_count()
            with torch.cuda.graph(g[0], stream=stream, capture_error_mode="thread_local"):
                append_call()
            with torch.cuda.graph(g[1], stream=stream, capture_error_mode="thread_local"):
                decode_call()
            launches_per_step = ct.launch_count() - l0
            graphs = g
        except Exception as exc:                        # keep measuring, from the host loop
            print(f"rank {rank}: CUDA graph capture failed ({exc}); enqueueing from the host", file=sys.stderr)
            torch.cuda.synchronize()
        if graphs:
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    graphs[0].replay()
                    graphs[1].replay()
        barrier()
    launch_mode = ("each step replays two CUDA graphs (append; decode + combine)" if graphs
                   else "each step enqueues its launches from the host")
    clocks = ClockSampler(physical_gpu(dev))
    clocks.start()
    launches0 = ct.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    t_start.record(stream)
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            ev[i][0].record(stream)
            graphs[0].replay() if graphs else append_call()
            ev[i][1].record(stream)
            graphs[1].replay() if graphs else decode_call()
            ev[i][2].record(stream)
    t_end.record(stream)
    barrier()
    launches = ct.launch_count() - launches0 + launches_per_step * args.steps
    graphs = None                                       # released before the process group goes away
    # a bounded wait that ran out leaves the kernel's outputs invalid: read its error word
    tc_error = int(L.ct_mla_tc_error(1))
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end)
    dec_ms = float(np.mean([e[1].elapsed_time(e[2]) for e in ev]))
    app_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    tokens = float(att.sum())

    # ---- e2e through the host-buffer C-ABI call ----
    import ctypes as C
    qh = ct.lib().ct_hal_cuda_alloc_host(n * H * E * 2)
    eh = ct.lib().ct_hal_cuda_alloc_host(n * E * 2)
    oh = ct.lib().ct_hal_cuda_alloc_host(n * H * DV * 2)
    q_host, tok_host = q.cpu().numpy(), new_tok.cpu().numpy()
    C.memmove(qh, q_host.ctypes.data, n * H * E * 2)
    C.memmove(eh, tok_host.ctypes.data, n * E * 2)

    def step_host():
        ct.check(L.ct_attn_mla_decode_step_host(plan.h, qh, eh, dest_dev.data_ptr(), kv.pool, None,
                                                kv.block_table_dev, kv.seq_lens_dev, oh, sp))

    for _ in range(max(1, args.warmup)):
        step_host()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_host()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    for p_ in (qh, eh, oh):
        ct.lib().ct_hal_cuda_free_host(p_)

    # ---- reduce over ranks ----
    import torch.distributed as dist
    # this GPU's decode: algorithmic bytes over its own mean launch time
    my_bytes = tokens * BYTES_PER_TOKEN + n * H * E * 2 + n * H * DV * 2
    my_gbs = my_bytes / (dec_ms * 1e-3) / 1e9
    tc_error = max(tc_error, int(L.ct_mla_tc_error(1)))
    vals = torch.tensor([ms, e2e_ms, dec_ms, app_ms, tokens, float(launches), float(n), my_gbs, float(tc_error != 0)],
                        dtype=torch.float64, device="cuda")
    if world > 1:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    else:
        mx = sm = vals
    ms_max, e2e_max, dec_max = float(mx[0]), float(mx[1]), float(mx[2])
    tok_total = float(sm[4])
    launches_total = int(sm[5])
    gbs_mean = float(sm[7]) / world                     # per-GPU achieved GB/s, mean over ranks
    tok_rank0 = tokens

    # ---- the one exchange: outputs and statistics gathered to rank 0 by the
    # library's NCCL backend (ct_dist_gather_rows / ct_dist_gather_stats),
    # timed separately with events on the stream the gather runs after ----
    gather_ms = None
    per_rank = None
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(ct.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)                         # the launcher's process group carries the id
        nctx = ct.NcclContext(rank, world, bytes(uid.cpu().numpy()), dev)
        full = torch.empty((n_all, H * DV), dtype=torch.int16, device="cuda") if rank == 0 else None
        ids = mine.astype(np.uint32)
        row_bytes = H * DV * 2

        def gather():
            nctx.gather_rows(out.data_ptr(), n, row_bytes, ids, n_all, full.data_ptr() if full is not None else None,
                             sp)

        gather()                                       # first call sizes the staging buffers
        gms = []
        for _ in range(3):
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            gather()
            g1.record(stream)
            torch.cuda.synchronize()
            gms.append(g0.elapsed_time(g1))
        gt = torch.tensor([float(np.median(gms))], dtype=torch.float64, device="cuda")
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gather_ms = float(gt[0])
        mine_stats = ct.DistStats(int(tokens), int(my_bytes), float(dec_ms * 1e3), int(tc_error), int(n))
        allst = nctx.gather_stats(mine_stats)
        if rank == 0:
            per_rank = [{"kv_tokens": int(x.kv_tokens), "bytes": int(x.bytes), "decode_us": float(x.decode_us),
                         "error": int(x.error), "n_seqs": int(x.n_seqs)} for x in allst]
        nctx.close()

    if rank != 0:
        return None
    hbm, hbm_kind = measured_hbm()
    achieved = gbs_mean             # per GPU: its own bytes over its own decode time, averaged over ranks
    traffic = committed_traffic(args.workload)
    if traffic is not None and world > 1:
        traffic = traffic * tok_rank0 / tok_total      # rank 0's launch: the one-GPU capture scaled by its tokens
    value = tok_total * args.steps / (ms_max * 1e-3)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "KV tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded SplitMix64/Box-Muller latents and queries, generated on the device)",
        "config": {"workload": desc, "n_seqs": int(n_all), "heads": H, "entry_dim": E, "v_dim": DV,
                   "page_tokens": PAGE, "kv_dtype": "bf16", "softmax_scale": "1/sqrt(192)",
                   "kv_tokens_per_step": int(tok_total), "sharding": "LPT by length" if world > 1 else "none",
                   "parallelism": f"sequence-sharded x{world}",
                   "launch": launch_mode,
                   "l2": f"inputs larger than L2 (KV of rank 0: {tok_rank0 * BYTES_PER_TOKEN / 1e6:.0f} MB vs "
                         "126 MB L2, read once per step); no flush"},
        "hbm_gbs": tok_total * args.steps * BYTES_PER_TOKEN / (ms_max * 1e-3) / 1e9,
        "gpu_launches": launches_total,
        "e2e": {"value": tok_total * args.steps / (e2e_max * 1e-3), "unit": "KV tokens/s",
                "h2d_bytes_per_step": int(n_all * H * E * 2 + n_all * E * 2),
                "d2h_bytes_per_step": int(n_all * H * DV * 2),
                "path": "ct_attn_mla_decode_step_host (pinned host q/new tokens in, outputs out)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": traffic, "peak_kind": hbm_kind, "per": "GPU (mean over ranks)",
                     "kernel": "MLA decode + split-KV combine (one ct_attn_mla_decode_paged call)",
                     "decode_ms": dec_max, "append_ms": float(mx[3])},
        "clocks": clk,
    }
    if gather_ms is not None:
        line["gather_ms"] = gather_ms                 # outputs of every rank to rank 0 (C-ABI NCCL gather)
        line["value_with_gather"] = tok_total / ((ms_max / args.steps + gather_ms) * 1e-3)
        line["per_rank"] = per_rank
    if float(mx[8]) != 0.0:
        line["invalid"] = "a bounded wait of the MLA decode kernel expired on some rank (ct_mla_tc_error != 0)"
    return line


# ---------------------------------------------------------------------------
# CPU arms: the reference's own ct_attn_forward on gathered pages
# ---------------------------------------------------------------------------

CPU_TOKEN_CAP = 8192


def cpu_sample(lens, seed, budget_s, threads):
    """Decode sequences of the workload (64 stratified over the lengths, in a
    seeded order) with the reference ct_attn_forward on all host threads until
    ~budget_s of decode time; each sequence is decoded over its first
    min(len, 8192) tokens so one call stays a few seconds (per-token cost
    still grows past that length, so the sample reads slightly fast).
    Input generation is outside the timed calls.  Returns (tokens/s, tokens,
    seconds): tokens over the busiest thread's decode time."""
    import concurrent.futures as cf
    import oracle
    R = oracle.ref()
    order = np.argsort(lens)
    strat = order[np.linspace(0, len(order) - 1, min(len(order), 64)).astype(int)]
    rng = np.random.default_rng(seed)
    rng.shuffle(strat)
    O = oracle.port()
    key_kv = O.orc_key(seed, 10)
    key_q = O.orc_key(seed, 11)
    busy = {}
    lock = threading.Lock()
    stop = threading.Event()

    def one(s):
        if stop.is_set():
            return 0
        n = min(int(lens[s]) + 1, CPU_TOKEN_CAP)
        kv = oracle.bf16_to_f32(oracle.normal_bf16(key_kv, (int(s) << 24) * E, n * E))
        q = oracle.bf16_to_f32(oracle.normal_bf16(key_q, int(s) * H * E, H * E))
        o = np.empty(H * E, np.float32)
        t0 = time.perf_counter()
        R.ct_attn_forward(q.ctypes.data, kv.ctypes.data, kv.ctypes.data, n, H, E, SCALE, o.ctypes.data)
        dt = time.perf_counter() - t0
        tid = threading.get_ident()
        with lock:
            busy[tid] = busy.get(tid, 0.0) + dt
            if max(busy.values()) > budget_s:
                stop.set()
        return n

    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        tok = sum(ex.map(one, strat))
    t = max(busy.values()) if busy else 1e-9
    return tok / t, tok, t


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    try:
        import oracle
        if not oracle.ref_available():
            return {"impl": "reference", "unavailable": "reference objects (oracle/_ref/libctref.so) not built"}
    except Exception as e:  # pragma: no cover
        return {"impl": "reference", "unavailable": f"oracle import failed: {e}"}
    lens, desc, seed = workload(args.workload)
    threads = os.cpu_count() or 1
    per_step = max(3.0, 60.0 / max(1, args.steps + args.warmup))
    rates = []
    for i in range(args.warmup + args.steps):
        r, tok, el = cpu_sample(lens, seed + i, per_step, threads)
        if i >= args.warmup:
            rates.append(r)
    value = float(np.mean(rates))
    total = int((lens + 1).sum())
    sample = (f"each step: up to 64 sequences stratified over the workload's lengths, each decoded over its first "
              f"<= {CPU_TOKEN_CAP} tokens through the reference ct_attn_forward (all 128 heads share the gathered "
              f"fp32 [n][576] entries), ~{per_step:.0f} s of decode on {threads} threads; value = sampled KV tokens "
              f"over the busiest thread's decode time.  Extrapolation to the full step ({total} KV tokens): "
              f"{total / value:.0f} s at this rate, taking the reference's cost per KV token as independent of the "
              f"sequence length (each head's pass over n x 576 fp32 entries leaves the host caches beyond ~1k "
              f"tokens, so longer sequences cost the same per token)")
    return {"metric": METRIC, "value": value, "unit": "KV tokens/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64 accumulate (f32 in/out)", "data": "synthetic",
            "config": {"workload": desc}, "impl": "reference",
            "full_step_s_extrapolated": total / value,
            "cpu_baseline": {"value": value, "unit": "KV tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "KV tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# secondary workloads (one JSON line each; the default line above is the
# headline): plain decode, quantised pools, eviction + compaction
# ---------------------------------------------------------------------------

def _events(torch, n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def run_plain(args):
    """4 layers x 8 heads x 64 fp32 contiguous cache, batch 1: 256 steps of
    (append one token to every layer, attend over the whole cache), captured
    in one CUDA graph.  The cache (4 MiB) stays in L2."""
    import torch
    import cautreo_b200 as ct
    L_, Hh, D, steps = 4, 8, 64, 256
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    n = steps * L_ * Hh * D
    q, k, v = (torch.empty(n, dtype=torch.float32, device="cuda") for _ in range(3))
    for i, t in enumerate((q, k, v)):
        ct.check(L.ct_synth_fill(t.data_ptr(), 1, ct.synth_key(0, i), 0, n, 0, 1.0, sp))
    kc = torch.zeros(L_ * steps * Hh * D, dtype=torch.float32, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    row = L_ * Hh * D

    def run_all():
        for s in range(steps):
            ct.check(L.ct_attn_decode_step_contig(q.data_ptr() + 4 * s * row, k.data_ptr() + 4 * s * row,
                                                  v.data_ptr() + 4 * s * row, kc.data_ptr(), vc.data_ptr(), L_,
                                                  steps, Hh, Hh, D, s, 0.0, out.data_ptr() + 4 * s * row, sp))

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        run_all()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        run_all()
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = _events(torch, 2)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps                  # one 256-step run
    tokens = L_ * steps * (steps + 1) // 2                  # KV positions read (all heads), per run
    kv_bytes = tokens * Hh * D * 4 * 2
    line = {"metric": "plain decode KV tokens/s (4 layers x 8 heads x 64 fp32, batch 1, 256 steps)",
            "value": tokens / (ms * 1e-3), "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "us_per_decode_step": ms * 1e3 / steps,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic (seed 0)",
            "config": {"workload": "plain contiguous KV decode: 4 layers, 8 heads, head_dim 64, fp32, batch 1, "
                                   "256 append+attend steps in one CUDA graph (a bench step = the 256-step run)"},
            "gpu_launches": steps * args.steps,
            "roofline": {"bound": "l2", "achieved": kv_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
                         "note": "the whole cache (4 MiB) is L2-resident; an HBM fraction is not meaningful"}}
    if not args.no_cpu_baseline:
        try:
            import oracle
            if oracle.ref_available():
                line["cpu_baseline"] = _plain_reference(oracle, q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(),
                                                        L_, Hh, D, steps, tokens)
        except Exception as e:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "error": str(e)}
    return line


def _plain_reference(oracle, q, k, v, L_, Hh, D, steps, tokens):
    """The reference CPU path timed on this host: ct_kv_append for every
    layer, then per layer and head ct_kv_get of that head's rows and
    ct_attn_forward (the engine's loop), one thread."""
    import ctypes as C
    R = oracle.ref()
    row = L_ * Hh * D
    q, k, v = q.reshape(steps, L_, Hh * D), k.reshape(steps, L_, Hh * D), v.reshape(steps, L_, Hh * D)
    cfg = oracle.KvConfig(L_, Hh, D, steps, 1.0)
    c = R.ct_kv_create(C.byref(cfg))
    krow = np.empty(Hh * D, np.float32)
    vrow = np.empty(Hh * D, np.float32)
    kh = np.empty((steps, D), np.float32)
    vh = np.empty((steps, D), np.float32)
    out = np.empty(D, np.float32)
    t0 = time.perf_counter()
    try:
        for s in range(steps):
            for l in range(L_):
                R.ct_kv_append(c, l, s, k[s, l].ctypes.data, v[s, l].ctypes.data)
            for l in range(L_):
                for t in range(s + 1):
                    R.ct_kv_get(c, l, t, krow.ctypes.data, vrow.ctypes.data)
                    kh[t] = krow.reshape(Hh, D)[0]
                    vh[t] = vrow.reshape(Hh, D)[0]
                for h in range(Hh):
                    R.ct_attn_forward(q[s, l, h * D:(h + 1) * D].ctypes.data, kh.ctypes.data, vh.ctypes.data,
                                      s + 1, 1, D, 0.0, out.ctypes.data)
    finally:
        R.ct_kv_destroy(c)
    el = time.perf_counter() - t0
    return {"value": tokens / el, "unit": "KV tokens/s", "cores": 1, "kind": "reference",
            "sample": "the whole 256-step run through the reference ct_kv_append / ct_kv_get / ct_attn_forward "
                      "(head 0's rows gathered once per layer and step and reused for every head)"}


def run_quant(args):
    """64 sequences x 8192 tokens of MLA entries (N(0,1), 1 % x20 outliers) in
    int8 and fp8-e4m3 pools with one fp32 scale per token (and, for
    comparison, a bf16 pool): quantise-on-append, dequantise-on-gather and
    decode over the quantised pages; then the block-codec pools."""
    import torch
    import cautreo_b200 as ct
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    B, T = 64, 8192
    n_tok = B * T
    pages_per = T // PAGE
    n_pages = B * pages_per
    src = torch.empty(n_tok * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(src.data_ptr(), 0, ct.synth_key(2, 10), 0, n_tok * E, 100, 20.0, sp))
    perm = np.random.default_rng(2).permutation(n_pages).astype(np.int32)
    q = torch.empty(B * H * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(q.data_ptr(), 0, ct.synth_key(2, 11), 0, B * H * E, 0, 1.0, sp))
    out = torch.empty(B * H * DV, dtype=torch.int16, device="cuda")
    gat = torch.empty(n_tok * E, dtype=torch.int16, device="cuda")
    hbm, hbm_kind = measured_hbm()
    res = {}
    tensor_peak, _ = measured_tensor()
    dec_flops = n_tok * H * 2 * (E + DV)                   # q.k over 576 values, p.v over 512, per head
    for name, dt in (("bf16", ct.CT_KV_BF16), ("int8", ct.CT_KV_INT8), ("e4m3", ct.CT_KV_E4M3)):
        kv = ct.PagedKV(B, pages_per, n_pages, PAGE, E, 0, dt, 0, sp)
        kv.set_free_order(perm)
        kv.append(list(range(B)), [T] * B, None)             # every slot reserved, pages permuted
        bt = kv.block_table()
        dest = (bt[:, :, None] * PAGE + np.arange(PAGE)[None, None, :]).reshape(-1).astype(np.int32)
        dest_dev = torch.from_numpy(dest).cuda()

        def append():
            ct.check(L.ct_kv_paged_write_slots(kv.pool, kv.scales, dt, src.data_ptr(), ct.CT_KV_BF16,
                                               dest_dev.data_ptr(), n_tok, E, sp))

        g_seqs = np.arange(B, dtype=np.uint32)
        g_starts = np.zeros(B, np.uint32)
        g_counts = np.full(B, T, np.uint32)

        def gather():                                     # every sequence, one launch
            ct.check(L.ct_kv_paged_gather_batch(kv.h, g_seqs.ctypes.data, g_starts.ctypes.data, g_counts.ctypes.data,
                                                B, gat.data_ptr(), ct.CT_KV_BF16))

        plan = ct.MlaPlan(np.full(B, T, np.int32), n_pages, kv_dtype=dt, max_pages_per_seq=pages_per)

        def decode():
            plan.decode(q.data_ptr(), kv.pool, kv.scales, kv.block_table_dev, kv.seq_lens_dev, out.data_ptr(), None,
                        sp)

        r = {}
        for what, fn, reps in (("append", append, args.steps), ("gather", gather, args.steps),
                               ("decode", decode, max(1, args.steps // 4))):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = _events(torch, 2)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            r[what] = e0.elapsed_time(e1) / reps
        code_bytes = n_tok * (E * 2 if dt == ct.CT_KV_BF16 else E + 4)
        dec_bytes = code_bytes + B * H * (E + DV) * 2          # pages + bf16 q + bf16 out
        res[name] = {
            "append_ms": r["append"], "append_gbs": (n_tok * E * 2 + code_bytes) / (r["append"] * 1e-3) / 1e9,
            "gather_ms": r["gather"], "gather_gbs": (code_bytes + n_tok * E * 2) / (r["gather"] * 1e-3) / 1e9,
            "decode_ms": r["decode"], "decode_tokens_s": n_tok / (r["decode"] * 1e-3),
            "decode_hbm_frac": dec_bytes / (r["decode"] * 1e-3) / 1e9 / hbm,
            "decode_tensor_frac": dec_flops / (r["decode"] * 1e-3) / 1e12 / tensor_peak,
            "decode_kernel": "tensor cores" if plan.tensor_cores else "CUDA cores",
        }
        res[name]["append_frac"] = res[name]["append_gbs"] / hbm
        res[name]["gather_frac"] = res[name]["gather_gbs"] / hbm
        if L.ct_mla_tc_error(1) != 0:
            res[name]["invalid"] = "a bounded wait of the MLA decode kernel expired (ct_mla_tc_error != 0)"
        plan.close()
        kv.close()
    # cold-tier block codecs (quant.h Q8_0 / Q4_0 / Q2_0 / Q1_0): append and gather only
    for name, dt in (("q8_0", ct.CT_KV_Q8_0), ("q4_0", ct.CT_KV_Q4_0), ("q2_0", ct.CT_KV_Q2_0),
                     ("q1_0", ct.CT_KV_Q1_0)):
        kv = ct.PagedKV(B, pages_per, n_pages, PAGE, E, 0, dt, 0, sp)
        kv.set_free_order(perm)
        kv.append(list(range(B)), [T] * B, None)
        bt = kv.block_table()
        dest = (bt[:, :, None] * PAGE + np.arange(PAGE)[None, None, :]).reshape(-1).astype(np.int32)
        dest_dev = torch.from_numpy(dest).cuda()
        g_seqs = np.arange(B, dtype=np.uint32)
        g_starts = np.zeros(B, np.uint32)
        g_counts = np.full(B, T, np.uint32)

        def append_b():
            ct.check(L.ct_kv_paged_write_slots(kv.pool, None, dt, src.data_ptr(), ct.CT_KV_BF16,
                                               dest_dev.data_ptr(), n_tok, E, sp))

        def gather_b():
            ct.check(L.ct_kv_paged_gather_batch(kv.h, g_seqs.ctypes.data, g_starts.ctypes.data, g_counts.ctypes.data,
                                                B, gat.data_ptr(), ct.CT_KV_BF16))

        r = {}
        for what, fn in (("append", append_b), ("gather", gather_b)):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = _events(torch, 2)
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            r[what] = e0.elapsed_time(e1) / args.steps
        code_bytes = n_tok * ct.entry_bytes(dt, E)
        res[name] = {"append_ms": r["append"], "append_gbs": (n_tok * E * 2 + code_bytes) / (r["append"] * 1e-3) / 1e9,
                     "gather_ms": r["gather"], "gather_gbs": (code_bytes + n_tok * E * 2) / (r["gather"] * 1e-3) / 1e9,
                     "bytes_per_token": ct.entry_bytes(dt, E)}
        res[name]["append_frac"] = res[name]["append_gbs"] / hbm
        res[name]["gather_frac"] = res[name]["gather_gbs"] / hbm
        kv.close()
    line = {"metric": "quantised paged KV: append / gather GB/s and decode KV tokens/s", "value": res["int8"]["append_gbs"],
            "unit": "GB/s (int8 quantise-on-append)", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "int8 / e4m3 codes + fp32 per-token scale", "data": "synthetic (seed 2)",
            "config": {"workload": "64 seqs x 8192 tokens, 576-value MLA entries N(0,1) with 1 % x20 outliers, "
                                   "64-token pages randomly permuted; append = one write of every token from bf16, "
                                   "gather = every sequence to contiguous bf16, decode = 128 heads over all pages",
                       "l2": "inputs larger than L2 (302 MB codes, 604 MB bf16); no flush"},
            "roofline": {"bound": "hbm", "achieved": res["int8"]["append_gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": res["int8"]["append_frac"], "peak_kind": hbm_kind,
                         "kernel": "k_write_slots (bf16 -> int8 + scale)"},
            "paths": res}
    return line


def measured_tensor():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def run_produce(args):
    """The producer side: each new token's 576-value entry = W . x (hidden 7168,
    bf16 weights [576][7168]) on the tensor cores, appended into an int8 pool
    (quantise-on-append in the same call): a decode batch of 1024 tokens (one
    per sequence) and a prefill chunk of 8192 tokens."""
    import torch
    import cautreo_b200 as ct
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    n_in = 7168
    w = torch.empty(E * n_in, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(w.data_ptr(), 0, ct.synth_key(6, 1), 0, E * n_in, 0, 0.02, sp))
    peak, peak_kind = measured_tensor()
    hbm, hbm_kind = measured_hbm()
    res = {}
    for n in (1024, 8192):
        x = torch.empty(n * n_in, dtype=torch.int16, device="cuda")
        ct.check(L.ct_synth_fill(x.data_ptr(), 0, ct.synth_key(6, 2), 0, n * n_in, 0, 1.0, sp))
        pages = (n + PAGE - 1) // PAGE
        pool = torch.empty(pages * PAGE * E, dtype=torch.uint8, device="cuda")
        scales = torch.empty(pages * PAGE, dtype=torch.float32, device="cuda")
        dest = torch.from_numpy(np.random.default_rng(6).permutation(pages * PAGE)[:n].astype(np.int32)).cuda()

        def step():
            ct.check(L.ct_kv_project_write_slots(x.data_ptr(), w.data_ptr(), None, 1e-6, 0, n, n_in, E, pool.data_ptr(),
                                                 scales.data_ptr(), ct.CT_KV_INT8, dest.data_ptr(), sp))

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        e0, e1 = _events(torch, 2)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        flops = 2.0 * n * n_in * E
        bytes_ = n * n_in * 2 + E * n_in * 2 + n * (E + 4)
        res[str(n)] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "tensor_frac": flops / (ms * 1e-3) / 1e12 / peak,
                       "gbs": bytes_ / (ms * 1e-3) / 1e9, "hbm_frac": bytes_ / (ms * 1e-3) / 1e9 / hbm,
                       "tokens_s": n / (ms * 1e-3)}
    assert L.ct_kv_project_error(1) == 0
    top = res["8192"]
    return {"metric": "fused latent projection + quantise-on-append: TFLOP/s and tokens/s", "value": top["tflops"],
            "unit": "TFLOP/s (8192-token chunk)", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "bf16 x bf16 -> fp32, int8 pool", "data": "synthetic (seed 6)",
            "config": {"workload": "entries = W[576][7168] . x for 1024 (decode batch) and 8192 (prefill chunk) "
                                   "tokens, appended into an int8 pool at permuted slots",
                       "l2": "weights (8.3 MB) stay L2-resident across steps; x is 14.7 / 117 MB"},
            "roofline": {"bound": "tensor", "achieved": top["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": top["tensor_frac"], "peak_kind": peak_kind, "kernel": "k_proj_tc + k_proj_finish + "
                         "k_write_slots"},
            "paths": res}


def run_aux(args):
    """The library's secondary kernels, each on inputs larger than L2 (one
    launch per step, CUDA events on the launching stream), for the launch
    list and DRAM bytes of every kernel that the other workloads do not
    reach: entries longer than 768 values appended (k_write_slots), gathers
    from an fp32 pool (k_gather, k_gather_batch), the CUDA-core MLA decode of
    a 16-head shape (k_mla_simt), the reference block and per-token codecs
    on device buffers (k_quant_blocks, k_dequant_blocks, k_quant_tokens,
    k_dequant_tokens), the reference attention and softmax contracts
    (k_attn_shared, k_softmax), ct_kv_compress (k_compress_*) and the row
    scatter of the multi-GPU gather (k_scatter_rows, through a one-rank NCCL
    context)."""
    import torch
    import cautreo_b200 as ct
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    res = {}

    def timed(name, fn, nbytes, reps=None):
        reps = reps or args.steps
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = _events(torch, 2)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}

    # entries of 1024 values, bf16 -> int8 + scale (one warp per token), 131,072 tokens
    n, D = 131072, 1024
    src = torch.zeros(n * D, dtype=torch.int16, device="cuda")
    codes = torch.empty(n * D, dtype=torch.int8, device="cuda")
    scl = torch.empty(n, dtype=torch.float32, device="cuda")
    dest = torch.arange(n, dtype=torch.int32, device="cuda")
    timed("k_write_slots bf16 -> int8, 1024 values x 131072", lambda: ct.check(L.ct_kv_paged_write_slots(
        codes.data_ptr(), scl.data_ptr(), ct.CT_KV_INT8, src.data_ptr(), ct.CT_KV_BF16, dest.data_ptr(), n, D, sp)),
        n * (2 * D + D + 4))
    del src, codes, scl, dest
    # fp32 pool gathers: 65,536 tokens of 576 values
    n = 65536
    kv = ct.PagedKV(2, n // PAGE, n // PAGE, PAGE, E, 0, ct.CT_KV_F32, 0, sp)
    kv.append([0, 1], [n // 2, n // 2], None)
    out = torch.empty(n * E, dtype=torch.float32, device="cuda")
    timed("k_gather f32 pool -> f32, 32768 tokens", lambda: ct.check(L.ct_kv_paged_gather(
        kv.h, 0, 0, n // 2, out.data_ptr(), ct.CT_KV_F32)), (n // 2) * E * 8)
    g_seqs, g_starts, g_counts = np.array([0, 1], np.uint32), np.zeros(2, np.uint32), np.full(2, n // 2, np.uint32)
    timed("k_gather_batch f32 pool -> f32, 2 x 32768 tokens", lambda: ct.check(L.ct_kv_paged_gather_batch(
        kv.h, g_seqs.ctypes.data, g_starts.ctypes.data, g_counts.ctypes.data, 2, out.data_ptr(), ct.CT_KV_F32)),
        n * E * 8)
    kv.close()
    del out
    # CUDA-core MLA decode, 16 heads (a shape the tensor-core kernel does not take): 32 x 4096 tokens
    S, T, Hs = 32, 4096, 16
    pages = S * T // PAGE
    pool = torch.zeros(pages * PAGE * E, dtype=torch.int16, device="cuda")
    bt = torch.arange(pages, dtype=torch.int32, device="cuda")
    lens = torch.full((S,), T, dtype=torch.int32, device="cuda")
    q = torch.zeros(S * Hs * E, dtype=torch.int16, device="cuda")
    o = torch.empty(S * Hs * DV, dtype=torch.int16, device="cuda")
    plan = ct.MlaPlan(np.full(S, T, np.int32), pages, n_heads=Hs, max_pages_per_seq=T // PAGE)
    timed("k_mla_simt 16 heads, 32 x 4096 tokens", lambda: plan.decode(
        q.data_ptr(), pool.data_ptr(), None, bt.data_ptr(), lens.data_ptr(), o.data_ptr(), None, sp),
        S * T * E * 2 + S * Hs * (E + DV) * 2, reps=max(1, args.steps // 4))
    plan.close()
    del pool, bt, lens, q, o
    # reference block codec Q8_0 and per-token int8 codec on device buffers, 32 M values
    nv = 32 * 1024 * 1024
    x = torch.zeros(nv, dtype=torch.float32, device="cuda")
    blk = torch.empty(nv // 32 * 34, dtype=torch.uint8, device="cuda")
    timed("k_quant_blocks Q8_0, 32 M values", lambda: ct.check(L.ct_quant_q8_0_dev(x.data_ptr(), blk.data_ptr(), nv, sp)),
          nv * 4 + nv // 32 * 34)
    timed("k_dequant_blocks Q8_0, 32 M values", lambda: ct.check(L.ct_dequant_q8_0_dev(blk.data_ptr(), x.data_ptr(), nv,
                                                                                         sp)), nv * 4 + nv // 32 * 34)
    del blk
    n_tok = nv // E
    c8 = torch.empty(n_tok * E, dtype=torch.int8, device="cuda")
    sc = torch.empty(n_tok, dtype=torch.float32, device="cuda")
    timed("k_quant_tokens int8 from fp32, 58254 x 576", lambda: ct.check(L.ct_quant_kv_int8(
        x.data_ptr(), 0, n_tok, E, c8.data_ptr(), sc.data_ptr(), sp)), n_tok * (E * 4 + E + 4))
    timed("k_dequant_tokens int8 to fp32, 58254 x 576", lambda: ct.check(L.ct_dequant_kv_int8(
        c8.data_ptr(), sc.data_ptr(), n_tok, E, x.data_ptr(), sp)), n_tok * (E * 4 + E + 4))
    del x, c8, sc
    # the reference attention contract (host buffers in and out; the kernel reads K and V once)
    nt, hh, hd = 262144, 8, 128
    qh = np.zeros(hh * hd, np.float32)
    kh = np.zeros(nt * hd, np.float32)
    vh = np.zeros(nt * hd, np.float32)
    oh = np.zeros(hh * hd, np.float32)
    for _ in range(2):
        if not L.ct_attn_forward(qh.ctypes.data, kh.ctypes.data, vh.ctypes.data, nt, hh, hd, 0.0, oh.ctypes.data):
            raise RuntimeError("ct_attn_forward")
    sm = np.zeros(16 * 1024 * 1024, np.float32)
    for _ in range(2):
        L.ct_attn_softmax(sm.ctypes.data, sm.size)
    res["k_attn_shared, k_softmax"] = {"note": "host-buffer reference contracts (ct_attn_forward 262144 tokens x 8 "
                                                "heads x 128, ct_attn_softmax 16 M values); see the launch list"}
    del kh, vh, sm
    # ct_kv_compress: 4 layers x 4096 tokens x 1024 values, every second token kept
    cache = ct.KvCache(4, 8, 128, 4096)
    row = np.zeros(1024, np.float32)
    for layer in range(4):
        for pos in range(4096):
            cache.append(layer, pos, row, row)
    if not L.ct_kv_compress(cache.h, 2.0):
        raise RuntimeError("ct_kv_compress")
    res["k_compress_*"] = {"note": "ct_kv_compress, 4 layers x 4096 tokens x 1024 fp32 values (K and V), step 2; "
                                   "see the launch list"}
    cache.close()
    # row scatter of the multi-GPU gather, one rank: 1024 rows of 128 KB
    ctx = ct.NcclContext(0, 1, ct.nccl_unique_id(), 0)
    nr, rb = 1024, H * DV * 2
    rows = torch.zeros(nr * rb // 2, dtype=torch.int16, device="cuda")
    dst = torch.empty(nr * rb // 2, dtype=torch.int16, device="cuda")
    ids = np.arange(nr, dtype=np.uint32)[::-1].copy()
    timed("k_scatter_rows 1024 x 128 KB (one-rank gather)", lambda: ctx.gather_rows(
        rows.data_ptr(), nr, rb, ids, nr, dst.data_ptr(), sp), 2 * nr * rb)
    ctx.close()
    hbm, hbm_kind = measured_hbm()
    for v in res.values():
        if "gbs" in v:
            v["frac"] = v["gbs"] / hbm
    return {"metric": "secondary kernels: GB/s each", "value": None, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "mixed",
            "data": "zeros (timing and traffic only; parity is in tests/)",
            "config": {"workload": "one launch per step of each secondary kernel, inputs larger than L2",
                       "peak": hbm, "peak_kind": hbm_kind},
            "kernels": res}


def run_serve(args):
    """A serving loop whose sequences grow: the sequence-sharded workload's
    1024 sequences (512..65536 tokens, seed 4) take one new token each per
    step through the paged allocator (ct_kv_paged_append: host bookkeeping,
    pages opened as lengths cross page boundaries, block-table and length
    updates scattered to the device, the token written), then one decode
    over all their tokens with a plan created once (the work split is
    recomputed on the device from the current lengths at every decode).
    Timed per step on the device (events around the step on the launching
    stream) and on the host (wall clock, which includes the allocator)."""
    import torch
    import cautreo_b200 as ct
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    lens0 = lengths_loguniform(1024, 512, 65536, seed=4)
    n = len(lens0)
    grow = args.warmup + args.steps + 1
    cap = lens0 + grow
    pages_cap = (cap + PAGE - 1) // PAGE
    n_pages, max_pages = int(pages_cap.sum()), int(pages_cap.max())
    kv = ct.PagedKV(n, max_pages, n_pages, PAGE, E, 0, ct.CT_KV_BF16, 0, sp)
    kv.set_free_order(np.random.default_rng(4000).permutation(n_pages).astype(np.int32))
    kv.append(list(range(n)), lens0.tolist(), None)              # the cached context, slots reserved
    rows = torch.arange(n, dtype=torch.int32, device="cuda")
    ct.check(L.ct_synth_fill_paged(kv.pool, None, ct.CT_KV_BF16, kv.block_table_dev, max_pages, rows.data_ptr(),
                                   kv.seq_lens_dev, n, int(lens0.max()), PAGE, E, ct.synth_key(4, 10), 0, 1.0, sp), "fill")
    q = torch.empty(n * H * E, dtype=torch.int16, device="cuda")
    new_tok = torch.empty(n * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(q.data_ptr(), 0, ct.synth_key(4, 11), 0, n * H * E, 0, 1.0, sp))
    ct.check(L.ct_synth_fill(new_tok.data_ptr(), 0, ct.synth_key(4, 13), 0, n * E, 0, 1.0, sp))
    out = torch.empty(n * H * DV, dtype=torch.int16, device="cuda")
    plan = ct.MlaPlan(lens0.astype(np.int32), n_pages, max_pages_per_seq=max_pages)
    seqs = np.arange(n, dtype=np.uint32)
    ones = np.ones(n, np.uint32)
    torch.cuda.synchronize()

    def step():
        ct.check(L.ct_kv_paged_append(kv.h, seqs.ctypes.data, ones.ctypes.data, n, new_tok.data_ptr(),
                                      ct.CT_KV_BF16), "append")
        ct.check(L.ct_attn_mla_decode_paged(plan.h, q.data_ptr(), kv.pool, None, kv.block_table_dev, kv.seq_lens_dev,
                                            out.data_ptr(), None, sp), "decode")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    opened0 = kv.stats().n_pages_live
    tok0 = int(kv.seq_lens().astype(np.int64).sum())
    e0, e1 = _events(torch, 2)
    launches0 = ct.launch_count()
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / args.steps
    launches = ct.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    assert L.ct_mla_tc_error(1) == 0
    st = kv.stats()
    attended = tok0 + n * (args.steps + 1) / 2.0      # mean KV tokens a timed step attends (each adds n)
    hbm, hbm_kind = measured_hbm()
    gbs = (attended * BYTES_PER_TOKEN + n * H * (E + DV) * 2) / (ms * 1e-3) / 1e9
    line = {"metric": "serving loop with growing sequences: KV tokens/s per decode step including the allocator",
            "value": attended / (ms * 1e-3), "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "host_ms_per_step": wall, "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic (seed 4)",
            "config": {"workload": "1024 seqs, 512..65536 tokens (seed 4), +1 token per sequence per step through "
                                   "ct_kv_paged_append, decode with one plan (device-side work split)",
                       "l2": "inputs larger than L2; no flush"},
            "pages_opened_in_timed_steps": int(st.n_pages_live - opened0),
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_kind": hbm_kind, "kernel": "whole step (append + plan + decode + combine)"}}
    plan.close()
    kv.close()
    return line


def run_evict(args):
    """256 sequences, lengths log-uniform 512..32768 (seed 3), 64-token bf16
    MLA pages in a pool of 60 % of the demand, 4096-token sliding window with
    LRU eviction under pressure: every token appended in rounds through the
    allocator, then a defragmenting compaction."""
    import torch
    import cautreo_b200 as ct
    L = ct.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    lens = lengths_loguniform(256, 512, 32768, seed=3)
    demand = int(((lens + PAGE - 1) // PAGE).sum())
    n_pages = int(0.6 * demand)
    max_pages = int((lens.max() + PAGE - 1) // PAGE)
    n_tok = int(lens.sum())
    src = torch.empty(n_tok * E, dtype=torch.int16, device="cuda")
    ct.check(L.ct_synth_fill(src.data_ptr(), 0, ct.synth_key(3, 10), 0, n_tok * E, 0, 1.0, sp))
    torch.cuda.synchronize()
    app, comp, whole, moved = [], [], [], []
    warm, reps = 1, max(2, args.steps // 5)            # each repetition rebuilds the cache from scratch
    for it in range(warm + reps):
        kv = ct.PagedKV(256, max_pages, n_pages, PAGE, E, 4096, ct.CT_KV_BF16, 0, sp)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        kv.append(list(range(256)), lens.tolist(), src.data_ptr())
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        # the compaction gather alone: live pages in (seq, lpage) order into a spare buffer
        bt = kv.block_table()
        live = bt[bt >= 0].astype(np.int32)               # row-major = (seq, lpage) order
        map_dev = torch.from_numpy(live).cuda()
        spare = torch.empty(len(live) * PAGE * E, dtype=torch.int16, device="cuda")
        e0, e1 = _events(torch, 2)
        e0.record(stream)
        ct.check(L.ct_kv_paged_move_pages(kv.pool, None, spare.data_ptr(), None, map_dev.data_ptr(), len(live),
                                          PAGE * E * 2, PAGE, sp))
        e1.record(stream)
        torch.cuda.synchronize()
        del spare
        # the whole call: renumbering, upload, gather into a fresh pool, table update
        t2 = time.perf_counter()
        ct.check(L.ct_kv_paged_compact(kv.h))
        torch.cuda.synchronize()
        t3 = time.perf_counter()
        st = kv.stats()
        if it >= warm:
            app.append(t1 - t0)
            comp.append(e0.elapsed_time(e1))
            whole.append((t3 - t2) * 1e3)
            moved.append(st.bytes_compacted)
        stats = st
        kv.close()
    hbm, hbm_kind = measured_hbm()
    comp_ms = float(np.mean(comp))
    comp_gbs = float(np.mean(moved)) / (comp_ms * 1e-3) / 1e9     # bytes_compacted counts read + write
    return {"metric": "eviction + compaction: compaction GB/s and append tokens/s through the allocator",
            "value": comp_gbs, "unit": "GB/s (compaction, read + write)", "n_gpus": 1, "steps": reps,
            "warmup": warm, "higher_is_better": True, "dtype": "bf16 pages", "data": "synthetic (seed 3)",
            "config": {"workload": f"256 seqs, lengths log-uniform 512..32768 (seed 3, {n_tok} tokens, {demand} pages "
                                   f"demanded), pool {n_pages} pages (60 %), window 4096, LRU under pressure, then "
                                   f"compaction"},
            "append_s": float(np.mean(app)), "append_tokens_s": n_tok / float(np.mean(app)),
            "compact_kernel_ms": comp_ms, "compact_call_ms": float(np.mean(whole)),
            "bytes_compacted": int(np.mean(moved)),
            "evictions": {"window": int(stats.n_evict_window), "lru": int(stats.n_evict_lru),
                          "live_pages": int(stats.n_pages_live)},
            "roofline": {"bound": "hbm", "achieved": comp_gbs, "peak": hbm, "unit": "GB/s", "frac": comp_gbs / hbm,
                         "peak_kind": hbm_kind, "kernel": "k_move_pages (compaction gather)"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="sharded",
                    choices=["sharded", "mla32", "plain", "quant", "evict", "produce", "serve", "aux"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="enqueue each step's launches from the host")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.workload in ("plain", "quant", "evict", "produce", "serve", "aux"):
        if int(os.environ.get("RANK", "0")) != 0 or args.impl == "reference":
            return 0          # one-GPU measurements of the other configurations
        line = {"plain": run_plain, "quant": run_quant, "evict": run_evict, "produce": run_produce,
                "serve": run_serve, "aux": run_aux}[args.workload](args)
        print(json.dumps(line), flush=True)
        return 0

    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if line is not None and world == 1 and not args.no_cpu_baseline:
            lens, desc, seed = workload(args.workload)
            try:
                import oracle
                if oracle.ref_available():
                    r, tok, el = cpu_sample(lens, seed, args.cpu_seconds, os.cpu_count() or 1)
                    line["cpu_baseline"] = {"value": r, "unit": "KV tokens/s", "cores": os.cpu_count() or 1,
                                            "kind": "reference",
                                            "sample": f"{tok} KV tokens of stratified sequences (first <= "
                                                      f"{CPU_TOKEN_CAP} tokens each) in {el:.1f} s of decode through "
                                                      f"the reference ct_attn_forward on gathered fp32 pages"}
            except Exception as e:  # pragma: no cover
                line["cpu_baseline"] = {"value": None, "error": str(e)}
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
