"""Benchmark of the fused LoRA-on-lm_head CE fwd+bwd+AdamW step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per GPU (weak scaling): the isolated fused op, h [8192 x 576] bf16,
W [49152 x 576] f16, LoRA rank 4 (alpha 8), Zipf(1.1) targets, one
fwd + bwd + AdamW (lr 1e-3, wd 0.01) step per iteration; for N > 1 every
rank takes its own 8192 positions and the dA/dB gradients are summed by one
NCCL all-reduce inside the step.  Inputs are seeded synthetic data.  The
working set (W 56.6 MB + h 9.4 MB) fits in L2, so L2 is flushed (a 256 MB
write) before every timed step; each step is timed alone with CUDA events
on the library's stream.

Prints one JSON line (rank 0).  `value` is the device-resident step
throughput (tokens/s over all ranks); `e2e` is the same step through the
public C ABI call with pinned host buffers (h and targets copied in, loss
read back, all inside the timed region), with a breakdown of where a
host-input step's time goes (host enqueue and wait, the chunked copies).
`roofline` describes the dominant kernel, `cpu_baseline` the reference CPU
path timed on this host's cores.  The default line also carries `strong`:
the rank-16 workload with 65,536 positions split over the N GPUs (strong
scaling), with its per-rank all-reduce and pass times.

Other modes: --config 3/4/5 (the rank-16, Q4_K and rank-64 workloads as the
main line), --tokens T (positions per rank), --op merge / q4k (the merge and
dequantisation kernels), --kernel-run (only the device steps, the command
to capture under ncu; --rank R runs them at another adapter rank, e.g. 128
for the wide-rank path), --impl reference (the reference's CPU path).
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "smollm2.c_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

V, D, R, ALPHA = 49152, 576, 4, 8
T_PER_GPU = 8192
LR, WD = 1e-3, 0.01
METRIC = "LoRA lm_head CE fwd+bwd tokens/s"
UNIT = "tokens/s"
# The workloads (--config): 2 is the default bench line; 3, 4 and 5 are the
# rank-16 strong-scaling, the Q4_K (QLoRA) lm_head and the rank-64
# long-context configurations.
CONFIGS = {
    2: dict(rank=4, alpha=8, tokens=8192, scaling="weak", q4k=False,
            desc="isolated fused LoRA lm_head CE fwd+bwd+AdamW step: h [8192x576] bf16 per GPU, "
                 "W [49152x576] f16, r 4, alpha 8"),
    3: dict(rank=16, alpha=32, tokens=65536, scaling="strong", q4k=False,
            desc="rank 16, 65536 positions split evenly over the GPUs, W [49152x576] f16, "
                 "alpha 32, dA/dB all-reduce before AdamW"),
    5: dict(rank=64, alpha=128, tokens=65536, scaling="weak", q4k=False, clip=1.0,
            desc="long-context batch: 32 x 2048 positions per GPU, r 64, alpha 128, W "
                 "[49152x576] f16, AdamW with grad-clip 1.0"),
    4: dict(rank=8, alpha=16, tokens=32768, scaling="weak", q4k=True,
            desc="QLoRA lm_head: W [49152x576] as Q4_K super-blocks (dequantised once into the "
                 "f16 GEMM operand), r 8, alpha 16, h [32768x576] bf16 per GPU"),
}
CONFIG = CONFIGS[2]


def flops(rank):
    """(whole step, one GEMM pass) FLOPs per predicted token:
    4*V*d + 8*V*r + 4*d*r and 2*V*d (tensor) + 4*V*r (rank terms)."""
    return 4 * V * D + 8 * V * rank + 4 * D * rank, 2 * V * D + 4 * V * rank


F_TOK, F_PASS = flops(R)


def step_tokens(world: int) -> int:
    """Predicted positions one step processes over all ranks."""
    return CONFIG["tokens"] if CONFIG["scaling"] == "strong" else CONFIG["tokens"] * world


def apply_config(n: int) -> None:
    global CONFIG, R, ALPHA, T_PER_GPU, F_TOK, F_PASS
    CONFIG = CONFIGS[n]
    R, ALPHA, T_PER_GPU = CONFIG["rank"], CONFIG["alpha"], CONFIG["tokens"]
    F_TOK, F_PASS = flops(R)


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def bind_near_gpu(local: int):
    """Run this process on the CPUs of the GPU's own NUMA node (from sysfs),
    so the pinned host buffers of the end-to-end leg are allocated there and
    host-device copies do not cross the socket link.  Returns the CPU list
    or None when the topology is not visible."""
    try:
        import torch
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return spec
    except (OSError, ValueError, AttributeError):
        pass
    return None


class L2Flush:
    """Cold L2 before a timed launch: write a 256 MB buffer (twice the L2),
    then read a second one, so that the written lines' write-back to HBM
    happens here, outside the timed region, and not inside the next
    HBM-bound kernel."""

    def __init__(self, torch, dev):
        n = 256 * 1024 * 1024 // 4
        self.w = torch.empty(n, dtype=torch.float32, device=dev)
        self.r = torch.ones(n, dtype=torch.float32, device=dev)
        self.acc = torch.empty((), dtype=torch.float32, device=dev)
        self.torch = torch

    def __call__(self):
        self.w.fill_(1.0)
        self.torch.sum(self.r, 0, out=self.acc)


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["bf16_tflops"]), float(j["hbm_gbs"]), "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """SM clocks, power and throttle reasons during the timed region: an
    NVML polling thread (every 2 ms, so that a region of a few tens of ms
    still gets many samples), or nvidia-smi -lms 200 when NVML is not
    importable."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.rows = []
        self.thread = None
        self.stop = False

    def _poll(self, nv, hdl):
        clk = nv.NVML_CLOCK_SM
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        mx = nv.nvmlDeviceGetMaxClockInfo(hdl, clk)
        while not self.stop:
            try:
                self.rows.append((float(nv.nvmlDeviceGetClockInfo(hdl, clk)), float(mx),
                                  nv.nvmlDeviceGetPowerUsage(hdl) / 1000.0, int(fn(hdl))))
            except Exception:  # noqa: BLE001 - a failed read only loses a sample
                pass
            time.sleep(0.002)

    def __enter__(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            busid = None
            try:
                import torch
                p = torch.cuda.get_device_properties(self.gpu)
                busid = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            except Exception:  # noqa: BLE001
                pass
            hdl = (nv.nvmlDeviceGetHandleByPciBusId(busid) if busid
                   else nv.nvmlDeviceGetHandleByIndex(self.gpu))
            self.thread = threading.Thread(target=self._poll, args=(nv, hdl), daemon=True)
            self.thread.start()
            time.sleep(0.01)
            return self
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.thread is not None:
            self.stop = True
            self.thread.join(timeout=2)
            return
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out = ""
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in (self.out or "").strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    bits = sum(self.REASONS[n] for n, v in zip(names, f[5:9]) if v.lower() == "active")
                    self.rows.append((float(f[1]), float(f[2]), float(f[3]), bits))
                except ValueError:
                    continue

    def summary(self):
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({n for r in rows for n, b in self.REASONS.items() if r[3] & b})
        loaded = [r[0] for r in rows if r[2] > 200.0] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows),
                "source": "nvml" if self.thread is not None else "nvidia-smi"}


# ----------------------------------------------------------------- CPU leg
def _ref_worker_init(lib_path):
    global _REF
    import oracle as orc
    _REF = orc.RefHarness()


def _ref_worker(args):
    """The reference's train_step (oracle/_ref) on one shard of positions;
    returns its own wall time."""
    import numpy as np
    import workload as wl
    seed, T, r, alpha = args
    W = wl.make_weight(1, V, D)
    h, tgt, A, B = wl.make_step_inputs(seed, T, V, D, r)
    H = wl.oracle_hidden(h)
    tokens = np.concatenate([[1], tgt]).astype(np.int32)
    t0 = time.perf_counter()
    _REF.train_steps(W, H, tokens, r, alpha, LR, 1 << 30, n_steps=1, A_dr=A, B_rv=B)
    return time.perf_counter() - t0


def _oracle_worker(args):
    import numpy as np
    import oracle as orc
    import workload as wl
    seed, T, threads, r, alpha = args
    W = wl.make_weight(1, V, D)
    h, tgt, A, B = wl.make_step_inputs(seed, T, V, D, r)
    H = wl.oracle_hidden(h)
    o = orc.Oracle()
    t0 = time.perf_counter()
    o.step(W, A, B, H, tgt, alpha / r, LR, wd=WD, nthreads=threads)
    return time.perf_counter() - t0


class CpuReference:
    """Tokens/s of the reference CPU path on this host: the reference's own
    train.c (oracle/_ref, single-threaded by design) run as one process per
    core, each on its own shard of positions (the data-parallel split the
    GPU path uses); the oracle port on all cores when oracle/_ref is absent.
    The pool is spawned (never forked), so it is safe to start after GPU work."""

    def __init__(self):
        import oracle as orc
        self.cores = os.cpu_count() or 1
        self.kind = "reference" if orc.ref_available() else "port"
        self.procs = min(self.cores, 128) if self.kind == "reference" else 1
        ctx = mp.get_context("spawn")
        if self.kind == "reference":
            self.pool = ctx.Pool(self.procs, initializer=_ref_worker_init, initargs=(None,))
            t_cal = max(self.pool.map(_ref_worker,
                                      [(100 + i, 2, R, ALPHA) for i in range(self.procs)]))
            self.per_tok = max(t_cal / 2, 1e-3)
        else:
            self.pool = ctx.Pool(1)
            self.per_tok = 0.05 / self.cores

    def sample(self, target_seconds: float):
        if self.kind == "reference":
            n_tok = max(2, int(target_seconds / self.per_tok))
            # the slowest worker's own train_step time (input generation excluded)
            wall = max(self.pool.map(_ref_worker,
                                     [(200 + i, n_tok, R, ALPHA) for i in range(self.procs)]))
            total, used = n_tok * self.procs, self.procs
            sample = (f"{self.procs} processes x {n_tok} positions (V {V}, d {D}, r {R}, f16 W); "
                      "the reference train_step in each")
        else:
            n_tok = max(self.cores, int(target_seconds / self.per_tok))
            wall = max(self.pool.map(_oracle_worker, [(300, n_tok, self.cores, R, ALPHA)]))
            total, used = n_tok, self.cores
            sample = f"{n_tok} positions on {self.cores} threads (oracle port)"
        return {"value": total / wall, "unit": UNIT, "cores": used, "kind": self.kind,
                "sample": sample}

    def close(self):
        self.pool.close()
        self.pool.join()


def run_reference_arm(args):
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    if rank != 0:
        return
    ref = CpuReference()
    per_step = max(2.0, min(8.0, 150.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        ref.sample(per_step / 2)
    steps = [ref.sample(per_step) for _ in range(args.steps)]
    ref.close()
    value = statistics.mean(s["value"] for s in steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * step_tokens(world) / value,
        "higher_is_better": True, "scaling": CONFIG["scaling"], "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; bf16 h, f16 W, Zipf(1.1) targets)",
        "config": dict(config_dict(args.config, world, step_tokens(world) // world),
                       tokens_per_step=step_tokens(world),
                       sample="each step a bounded sample of positions on the reference's CPU "
                              "path (f16 W: the reference has no Q4_K)"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": steps[0]["cores"],
                         "kind": steps[0]["kind"], "sample": steps[0]["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- merge
def run_merge(args):
    """Merge of the adapter into the tied lm_head (train_merge's
    lora_patched_weight): W [49152x576] f16 in, patched f16 out.  HBM-bound;
    algorithmic bytes per launch = 2*V*d (read W) + 2*V*d (write out) +
    4*(d+V)*r (A, B).  The CPU leg times the oracle restatement of the same
    merge (single thread) on the same inputs."""
    import ctypes as C
    import numpy as np
    import torch
    import lora_ce
    import workload as wl

    args.warmup = max(args.warmup, 3)
    args.steps = max(args.steps, 200)  # a timed region long enough for the clock sampler
    r = args.merge_rank
    cpu = None
    if not args.no_cpu_baseline:
        import oracle as orc
        o = orc.Oracle()
        Wc = wl.make_weight(1, V, D)
        rng = np.random.default_rng(5)
        Ac = rng.standard_normal((D, r), dtype=np.float32)
        Bc = rng.standard_normal((r, V), dtype=np.float32) * np.float32(1e-2)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 10.0:
            o.merge(Wc, Ac, Bc, ALPHA / r)
            n += 1
        dt = time.perf_counter() - t0
        cpu = {"value": n * 4.0 * V * D / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{n} full merges of W [49152x576], r {r} (oracle restatement of "
                         "lora_patched_weight, one thread)"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = lora_ce.load_library()
    W = torch.from_numpy(wl.make_weight(1, V, D).view(np.int16)).to(dev)
    g = torch.Generator(device="cpu").manual_seed(5)
    A = torch.randn(D, r, generator=g).to(dev)
    B = (torch.randn(r, V, generator=g) * 1e-2).to(dev)
    out = torch.empty_like(W)
    flush = L2Flush(torch, dev)
    st = torch.cuda.current_stream(dev)

    def launch():
        rc = lib.lora_ce_merge_weight_device(C.c_void_p(W.data_ptr()), C.c_void_p(A.data_ptr()),
                                             C.c_void_p(B.data_ptr()), D, r, V,
                                             float(ALPHA / r), C.c_void_p(out.data_ptr()),
                                             C.c_void_p(st.cuda_stream))
        if rc != 0:
            raise RuntimeError(lib.lora_ce_merge_last_error().decode())

    for _ in range(args.warmup):
        flush()
        launch()
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for s_, e_ in evs:
            flush()
            s_.record(st)
            launch()
            e_.record(st)
        torch.cuda.synchronize(dev)
    ms = [s_.elapsed_time(e_) for s_, e_ in evs]
    t_ms = sum(ms) / len(ms)
    alg = 4.0 * V * D + 4.0 * (D + V) * r
    gbs = alg / (t_ms * 1e-3) / 1e9
    # end to end through lora_ce_merge_weight (host buffers, copies inside)
    Wh = wl.make_weight(1, V, D)
    Ah, Bh = A.cpu().numpy(), B.cpu().numpy()
    lora_ce.merge_weight(Wh, Ah, Bh, ALPHA / r)
    n_e2e = min(args.steps, 20)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        lora_ce.merge_weight(Wh, Ah, Bh, ALPHA / r)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    _, hbm, peak_kind = peaks()
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(f"merge_r{r}")
    line = {
        "metric": "LoRA merge into lm_head GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms,
        "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; W f16 N(0,0.02), A N(0,1), B N(0,1e-2))",
        "config": {"workload": f"merge W [49152x576] f16 + (alpha/r) A B, r {r}, alpha 8",
                   "rank": r, "l2": "flushed before every launch (256 MB write, then 256 MB read so the write-back is done)"},
        "roofline": {"kernel": "lce_merge", "bound": "hbm", "achieved": gbs, "peak": hbm,
                     "unit": "GB/s", "frac": gbs / hbm, "peak_kind": f"{peak_kind} copy",
                     "bytes_per_launch": alg, "traffic": traffic},
        "cpu_baseline": cpu,
        "e2e": {"value": alg / e2e_s / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": int(2 * V * D + 4 * (D + V) * r),
                "d2h_bytes_per_step": int(2 * V * D), "timer": "host wall clock"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- Q4_K
def run_q4k(args):
    """Dequantisation of the Q4_K lm_head (config 4's weight: 110,592
    super-blocks) into the f16 GEMM operand.  HBM-bound; algorithmic bytes
    per launch = 144 in + 512 out per super-block.  The CPU leg times the
    oracle restatement (f32 output, one thread) on the same blocks."""
    import ctypes as C
    import numpy as np
    import torch
    import lora_ce
    import workload as wl

    args.warmup = max(args.warmup, 3)
    args.steps = max(args.steps, 200)  # a timed region long enough for the clock sampler
    blocks_h = wl.make_weight_q4k(1, V, D)
    n = blocks_h.shape[0]
    alg = n * (144.0 + 512.0)
    cpu = None
    if not args.no_cpu_baseline:
        import oracle as orc
        o = orc.Oracle()
        t0 = time.perf_counter()
        k = 0
        while time.perf_counter() - t0 < 10.0:
            o.q4k_dequant(blocks_h)
            k += 1
        dt = time.perf_counter() - t0
        cpu = {"value": k * n * (144.0 + 1024.0) / dt / 1e9, "unit": "GB/s", "cores": 1,
               "kind": "port", "sample": f"{k} dequantisations of the {n}-block lm_head to f32 "
                                         "(oracle restatement, one thread; no reference "
                                         "implementation exists)"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = lora_ce.load_library()
    blocks = torch.from_numpy(blocks_h).to(dev)
    out = torch.empty(n * 256, dtype=torch.int16, device=dev)
    flush = L2Flush(torch, dev)
    st = torch.cuda.current_stream(dev)

    def launch():
        rc = lib.lora_ce_q4k_dequant_device(C.c_void_p(blocks.data_ptr()), n,
                                            C.c_void_p(out.data_ptr()), lora_ce.F16,
                                            C.c_void_p(st.cuda_stream))
        if rc != 0:
            raise RuntimeError(lib.lora_ce_q4k_last_error().decode())

    for _ in range(args.warmup):
        flush()
        launch()
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for s_, e_ in evs:
            flush()
            s_.record(st)
            launch()
            e_.record(st)
        torch.cuda.synchronize(dev)
    t_ms = sum(s_.elapsed_time(e_) for s_, e_ in evs) / args.steps
    gbs = alg / (t_ms * 1e-3) / 1e9
    # The dequantisation work a GEMM producer that dequantises W itself
    # would repeat per pass at 32,768 positions: pass 1 streams W once per
    # block of 256 resident positions, 128 times, with the Q4_K blocks warm
    # in L2 (back-to-back launches, no flush in between).
    reps = 32768 // 256
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        launch()
    e1.record(st)
    torch.cuda.synchronize(dev)
    repeat_ms = e0.elapsed_time(e1)
    lora_ce.q4k_dequant(blocks_h, lora_ce.F16)
    n_e2e = min(args.steps, 20)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        lora_ce.q4k_dequant(blocks_h, lora_ce.F16)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    _, hbm, peak_kind = peaks()
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get("q4k_dequant")
    line = {
        "metric": "Q4_K lm_head dequantisation GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms,
        "higher_is_better": True, "scaling": "replicas only", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic (seeded Q4_K super-blocks: uniform quant and scale "
                               "bytes, d/dmin f16 in [4e-5, 1.2e-4])",
        "config": {"workload": f"Q4_K W [49152x576] ({n} super-blocks) -> f16",
                   "l2": "flushed before every launch (256 MB write, then 256 MB read so the write-back is done)"},
        "roofline": {"kernel": "lce_q4k_dequant", "bound": "hbm", "achieved": gbs, "peak": hbm,
                     "unit": "GB/s", "frac": gbs / hbm, "peak_kind": f"{peak_kind} copy",
                     "bytes_per_launch": alg, "traffic": traffic},
        "cpu_baseline": cpu,
        "e2e": {"value": alg / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(n * 144),
                "d2h_bytes_per_step": int(n * 512), "timer": "host wall clock"},
        "gpu_launches": args.steps + reps,
        "clocks": clk.summary(),
        "in_producer_equivalent": {"launches": reps, "ms": repeat_ms,
                                   "what": "W dequantised once per 256-position block of a "
                                           "32,768-position pass, L2 warm"},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- config 1
BODY_LAYERS, BODY_SEQ = 30, 256


def _write_body_model(path: str):
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import studio_fixtures as sf
    return sf.write_smollm_gguf(path, seed=1, n_layers=BODY_LAYERS, norm_spread=0.2,
                                return_tensors=True)


def run_config1(args):
    """The CPU-body training workload (30-layer SmolLM2-135M shape, packed
    sequences of 256, rank 4, alpha 8, lr 1e-3): the whole training step
    with its body forward.  GPU: lora_body_train_step (body forward of the
    sample's positions, then the LoRA step), one sample (255 predicted
    positions) per step as the reference trains, and the packed variant
    with 4 samples per step.  CPU: the reference's own body forward and
    train_step's body forward, as processes over the host cores, on a
    bounded sample of positions."""
    import tempfile
    import numpy as np
    import torch
    import lora_ce
    import workload as wl

    args.warmup = max(args.warmup, 3)
    tmp = tempfile.mkdtemp(prefix="bench_body_")
    model = os.path.join(tmp, "m30.gguf")
    embd, out_norm, layers = _write_body_model(model)
    note("config 1: model written")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(1)
    seqs = [wl.zipf_targets(rng, BODY_SEQ, V).astype(np.int32) for _ in range(4)]
    body = lora_ce.LoraBody(BODY_LAYERS, max_seq=BODY_SEQ, max_tokens=4 * BODY_SEQ)
    body.set_embedding(embd, out_norm)
    for L, t in enumerate(layers):
        body.set_layer(L, t)
    A = np.asarray(wl.make_step_inputs(1000, 8, V, D, 4)[2])
    res = {}
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.ExternalStream(body.stream, device=dev)
    clk_out = None
    for pack in (1, 4):
        T = pack * (BODY_SEQ - 1)
        ce = lora_ce.LoraCE(lora_ce.default_config(D, V, 4, T, scale=2.0, lr=LR))
        ce.set_weight(embd)
        ce.set_adapter(A, np.zeros((4, V), np.float32), 0)
        tok = np.concatenate([s[:-1] for s in seqs[:pack]])
        tgt = np.concatenate([s[1:] for s in seqs[:pack]])
        off = np.arange(pack + 1, dtype=np.int32) * (BODY_SEQ - 1)
        for _ in range(args.warmup):
            body.train_step(ce, tok, off, tgt)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        clk = ClockSampler(0)
        with clk:
            for s_, e_ in evs:
                with torch.cuda.stream(st):
                    flush.fill_(1.0)
                s_.record(st)
                body.train_step(ce, tok, off, tgt)
                e_.record(st)
            torch.cuda.synchronize(dev)
        ms = [s_.elapsed_time(e_) for s_, e_ in evs]
        # the body alone (device tokens -> device hidden rows)
        dT = torch.from_numpy(tok).to(dev)
        dH = torch.empty((T, D), dtype=torch.float32, device=dev)
        bev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for s_, e_ in bev:
            with torch.cuda.stream(st):
                flush.fill_(1.0)
            s_.record(st)
            body.hidden_device(dT.data_ptr(), off, dH.data_ptr(), lora_ce.F32)
            e_.record(st)
        torch.cuda.synchronize(dev)
        body_ms = sum(s_.elapsed_time(e_) for s_, e_ in bev) / args.steps
        ce.close()
        res[pack] = dict(T=T, ms=sum(ms) / len(ms), body_ms=body_ms,
                         tokens_s=T * len(ms) / (sum(ms) / 1e3))
        if clk_out is None:
            clk_out = clk.summary()
    body.close()
    note("config 1: GPU legs done")
    # MACs of the body per position: 30 layers x (q,k,v,o,gate,up,down) int8
    kv = 192
    macs = BODY_LAYERS * (D * (D + 2 * kv) + D * D + 3 * D * 1536)
    cpu = None
    if not args.no_cpu_baseline:
        note("config 1: CPU reference")
        procs = max(1, min(os.cpu_count() or 1, 16))
        n = 24
        ctx = mp.get_context("spawn")
        with ctx.Pool(procs) as pool:
            out = pool.map(_ref_body_step, [(model, 50 + i, n) for i in range(procs)])
        wall = max(out)
        cpu = {"value": procs * n / wall, "unit": UNIT, "cores": procs, "kind": "reference",
               "sample": f"{procs} processes x {n} positions of a 30-layer sequence: the "
                         "reference's body forward position by position (its forward_decode, "
                         "base logits included); the step's lora_accum and Adam, about 1% of "
                         "it, are not counted, so this rate is an upper bound of the "
                         "reference's"}
    peak_tf, _, peak_kind = peaks()
    one = res[1]
    line = {
        "metric": "LoRA training step with the body forward, tokens/s", "value": one["tokens_s"],
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": one["ms"], "higher_is_better": True, "scaling": "replicas only",
        "vs_baseline": None, "dtype": "int8 body, f16 lm_head",
        "data": "synthetic (seeded 30-layer SmolLM2-135M-shaped model file, norms 1+U(-0.2,0.2); "
                "Zipf(1.1) token ids)",
        "config": {"workload": "CPU-body training workload: 30 layers, d 576, 9/3 heads, FFN "
                               "1536, V 49152, sequences of 256, rank 4, alpha 8, lr 1e-3; "
                               "one sample (255 predicted positions) per step as the reference "
                               "trains", "config": 1,
                   "l2": "flushed (256 MB write) before every timed step"},
        "body_ms_per_step": one["body_ms"],
        "body": {"kernel": "body forward (int8 dp4a GEMMs, attention, norms)",
                 "int8_tops": 2.0 * macs * one["T"] / (one["body_ms"] * 1e-3) / 1e12,
                 "macs_per_position": macs},
        "packed4": {"tokens_per_step": res[4]["T"], "ms_per_step": res[4]["ms"],
                    "value": res[4]["tokens_s"], "body_ms_per_step": res[4]["body_ms"]},
        "cpu_baseline": cpu,
        "e2e": {"value": one["tokens_s"], "unit": UNIT, "h2d_bytes_per_step": 8 * one["T"],
                "d2h_bytes_per_step": 4,
                "note": "lora_body_train_step takes host tokens and targets and returns the loss: "
                        "the device-timed step is already end to end"},
        "gpu_launches": None, "clocks": clk_out,
    }
    print(json.dumps(line), flush=True)


def body_kernel_run(args):
    """Only the body forward of the 30-layer model on --tokens positions
    (one sequence, default 255), --warmup + --steps times: the command for
    an ncu capture of the body's kernels."""
    import tempfile
    import numpy as np
    import lora_ce
    import workload as wl

    T = args.tokens or BODY_SEQ - 1
    tmp = tempfile.mkdtemp(prefix="bench_body_")
    embd, out_norm, layers = _write_body_model(os.path.join(tmp, "m30.gguf"))
    body = lora_ce.LoraBody(BODY_LAYERS, max_seq=T, max_tokens=T)
    body.set_embedding(embd, out_norm)
    for L, t in enumerate(layers):
        body.set_layer(L, t)
    tok = wl.zipf_targets(np.random.default_rng(1), T, V).astype(np.int32)
    for _ in range(args.warmup + args.steps):
        body.hidden(tok, [0, T])
    body.close()
    print(f"body kernel run ok: {BODY_LAYERS} layers, T {T}", flush=True)


def _ref_body_step(args):
    """Seconds of the reference's own body forward (src/forward.c, position
    by position as train_step runs it) over one sample of n positions of the
    30-layer model."""
    import numpy as np
    import oracle as orc
    import workload as wl
    model, seed, n = args
    rng = np.random.default_rng(seed)
    tokens = wl.zipf_targets(rng, n, V).astype(np.int32)
    rb = orc.RefBody(model, n)
    _, body_s = rb.hidden(tokens, D)
    rb.close()
    return body_s


# ----------------------------------------------------------------- GPU leg
def note(msg: str) -> None:
    """Progress on stderr (the JSON line is the only stdout)."""
    print(f"[bench] {msg}", file=sys.stderr, flush=True)


def cfg_workload(n: int, world: int, tokens: int | None = None):
    """(rank, alpha, positions per rank, clip, q4k) of workload n at world ranks."""
    c = CONFIGS[n]
    T = tokens or c["tokens"]
    T_rank = T // world if c["scaling"] == "strong" else T
    return c["rank"], c["alpha"], T_rank, c.get("clip", 0.0), c["q4k"]


def make_handle(n, world, rank, local, tokens=None, seed=1000):
    """A handle and its device / host inputs for workload n on this rank."""
    import numpy as np
    import torch
    import lora_ce
    import workload as wl

    r, alpha, T, clip, q4k = cfg_workload(n, world, tokens)
    h, tgt, _, _ = wl.make_step_inputs(seed + rank, T, V, D, r)
    _, _, A, B = wl.make_step_inputs(seed, 8, V, D, r)  # same adapter on every rank
    cfg = lora_ce.default_config(D, V, r, T, scale=alpha / r, lr=LR, weight_decay=WD,
                                 clip_norm=clip, device=local)
    m = lora_ce.LoraCE(cfg)
    if q4k:
        m.set_weight_q4k(wl.make_weight_q4k(1, V, D))
    else:
        m.set_weight(wl.make_weight(1, V, D))
    m.set_adapter(A, B, 0)
    dev = torch.device("cuda", local)
    dH = torch.from_numpy(h.view(np.int16)).to(dev)
    dT = torch.from_numpy(tgt).to(dev)
    return m, h, tgt, dH, dT, T


class Rig:
    """The per-process measurement set-up: device, L2 flush buffer, barrier
    and max-over-ranks reductions."""

    def __init__(self, torch, dist, local):
        self.torch, self.dist = torch, dist
        self.dev = torch.device("cuda", local)
        self.flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=self.dev)

    def barrier(self):
        self.torch.cuda.synchronize(self.dev)
        if self.dist is not None:
            self.dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        if self.dist is not None:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, obj):
        if self.dist is None:
            return [obj]
        out = [None] * self.dist.get_world_size()
        self.dist.all_gather_object(out, obj)
        return out

    def timed(self, st, fn, n):
        """n calls of fn, each bracketed by CUDA events on stream st with an
        L2 flush (256 MB write) before it; per-call ms."""
        torch = self.torch
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(n)]
        for s, e in evs:
            with torch.cuda.stream(st):
                self.flush_buf.fill_(1.0)
            s.record(st)
            fn()
            e.record(st)
        torch.cuda.synchronize(self.dev)
        return [s.elapsed_time(e) for s, e in evs]


def measure(rig, m, h, tgt, dH, dT, T, world, steps, warmup, clocks=None, breakdown=True):
    """Device-resident and end-to-end throughput of one workload's step on
    this rank's handle; max over ranks for the timed totals."""
    import numpy as np
    import torch
    import lora_ce

    st = torch.cuda.ExternalStream(m.stream, device=rig.dev)
    dLoss = torch.zeros(2, dtype=torch.float32, device=rig.dev)
    note("device-resident steps")

    def dev_step():
        m.step_device(dH.data_ptr(), lora_ce.BF16, T, dT.data_ptr(), dLoss.data_ptr())

    for _ in range(warmup):
        dev_step()
    m.sync()
    rig.barrier()
    if clocks is not None:
        with clocks:
            ms = rig.timed(st, dev_step, steps)
    else:
        ms = rig.timed(st, dev_step, steps)
    m.sync()
    launches = m.last_launches
    rig.barrier()
    total_ms = rig.max_over_ranks(sum(ms))
    out = {"T": T, "ms": ms, "total_ms": total_ms, "launches": launches,
           "value": world * T * steps / (total_ms / 1e3)}
    if clocks is not None:
        out["clocks"] = clocks.summary()

    # per-kernel durations (same stream), for the roofline and the breakdown
    m.set_profiling(True)
    phase = {}
    for _ in range(max(3, steps // 2)):
        with torch.cuda.stream(st):
            rig.flush_buf.fill_(1.0)
        dev_step()
        for k, v in m.phase_times().items():
            phase.setdefault(k, []).append(v)
    m.set_profiling(False)
    out["phase_ms"] = {k: sum(v) / len(v) for k, v in phase.items()}

    # end to end through the public API with pinned host buffers
    note("end-to-end steps")
    hH = torch.from_numpy(h.view(np.int16)).pin_memory()
    hT = torch.from_numpy(tgt).pin_memory()
    hHn, hTn = hH.numpy().view(np.uint16), hT.numpy()
    for _ in range(2):
        m.step(hHn, hTn)
    rig.barrier()
    host = []

    def e2e_step():
        m.step(hHn, hTn)
        host.append(m.copy_times())  # the graph replay's host enqueue / wait

    e2e_ms = rig.timed(st, e2e_step, steps)
    out["e2e_host_us"] = {"enqueue_median": round(statistics.median(x["host_us"] for x in host), 1),
                          "wait_median": round(statistics.median(x["wait_us"] for x in host), 1)}
    out["e2e_ms"] = e2e_ms
    out["e2e_value"] = world * T * steps / (rig.max_over_ranks(sum(e2e_ms)) / 1e3)
    out["h2d_bytes"] = int(hH.numel() * 2 + hT.numel() * 4)
    if breakdown:
        # the same end-to-end steps again with event nodes in the graph: where
        # each step's time goes (host enqueue, host wait, the chunk copies)
        note("end-to-end breakdown")
        m.set_copy_timing(True)
        for _ in range(2):
            m.step(hHn, hTn)
        rows = []
        for _ in range(steps):
            with torch.cuda.stream(st):
                rig.flush_buf.fill_(1.0)
            m.step(hHn, hTn)
            rows.append(m.copy_times())
        m.set_copy_timing(False)
        med = statistics.median
        nch = len(rows[0]["chunk_ms"])
        out["e2e_breakdown"] = {
            "steps": len(rows),
            "host_enqueue_us": {"min": round(min(r["host_us"] for r in rows), 1),
                                "median": round(med(r["host_us"] for r in rows), 1),
                                "max": round(max(r["host_us"] for r in rows), 1)},
            "host_wait_us": {"min": round(min(r["wait_us"] for r in rows), 1),
                             "median": round(med(r["wait_us"] for r in rows), 1),
                             "max": round(max(r["wait_us"] for r in rows), 1)},
            "copy_start_ms_median": round(med(r["copy_wait_ms"] for r in rows), 4),
            "chunk_copy_ms_median": [round(med(r["chunk_ms"][c] for r in rows), 4)
                                     for c in range(nch)],
            "h2d_GBps_median": round(out["h2d_bytes"] / 1e6 /
                                     med(sum(r["chunk_ms"]) for r in rows), 2),
            "graph_step_ms": {"min": round(min(r["step_ms"] for r in rows), 4),
                              "median": round(med(r["step_ms"] for r in rows), 4),
                              "max": round(max(r["step_ms"] for r in rows), 4)},
        }
    return out


def kernel_run(args):
    """Only the device step of the chosen workload, `--steps` times after
    `--warmup` untimed steps, nothing else: the command to run under ncu for
    a kernel capture (small --tokens keep the capture short)."""
    import torch
    import lora_ce

    torch.cuda.set_device(0)
    if args.rank:
        CONFIGS[args.config] = dict(CONFIGS[args.config], rank=args.rank, alpha=2 * args.rank)
    m, h, tgt, dH, dT, T = make_handle(args.config, 1, 0, 0, args.tokens)
    for _ in range(args.warmup + args.steps):
        m.step_device(dH.data_ptr(), lora_ce.BF16, T, dT.data_ptr(), 0)
    m.sync()
    m.close()
    print(f"kernel run ok: config {args.config}, rank {CONFIGS[args.config]['rank']}, T {T}, "
          f"{args.warmup + args.steps} steps", flush=True)


def main():
    import faulthandler
    # a run that stalls prints every thread's stack and exits instead of
    # holding the GPUs until an outer limit kills it
    faulthandler.dump_traceback_later(float(os.environ.get("BENCH_WATCHDOG_S", "1200")), exit=True)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--op", default="step", choices=["step", "merge", "q4k"])
    ap.add_argument("--config", type=int, default=2, choices=[1] + sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=None,
                    help="positions per step (per rank for weak scaling) instead of the "
                         "workload's own")
    ap.add_argument("--no-strong", action="store_true",
                    help="leave out the rank-16 strong-scaling object of the default line")
    ap.add_argument("--kernel-run", action="store_true",
                    help="run only the device steps (the command for an ncu capture)")
    ap.add_argument("--rank", type=int, default=None,
                    help="with --kernel-run: this adapter rank (alpha 2 x rank) instead of the "
                         "workload's, e.g. 128 for the wide-rank path")
    ap.add_argument("--merge-rank", type=int, default=R)
    args = ap.parse_args()
    if args.config == 1:
        if args.kernel_run:
            body_kernel_run(args)
        else:
            run_config1(args)
        return
    apply_config(args.config)
    if args.tokens:
        CONFIG["tokens"] = args.tokens
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.op == "merge":
        run_merge(args)
        return
    if args.op == "q4k":
        run_q4k(args)
        return
    if args.kernel_run:
        kernel_run(args)
        return
    args.warmup = max(args.warmup, 3)

    import torch

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group(backend="cpu:gloo,cuda:nccl",
                                timeout=datetime.timedelta(seconds=120))

    numa_cpus = bind_near_gpu(local)
    rig = Rig(torch, dist, local)

    def with_comm(m):
        if world > 1:
            uid = [m.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            m.comm_init(world, rank, uid[0])
        return m

    m, h, tgt, dH, dT, T = make_handle(args.config, world, rank, local, CONFIG["tokens"])
    with_comm(m)
    note(f"workload {args.config}: T {T} per rank, rank {R}")
    res = measure(rig, m, h, tgt, dH, dT, T, world, args.steps, args.warmup,
                  clocks=ClockSampler(local), breakdown=args.config == 2)
    clk = res.pop("clocks", None)
    m.close()
    phase_ms = res["phase_ms"]
    dom = max(("pass1_lse", "pass2_grad"), key=lambda k: phase_ms[k])
    peak_tf, hbm, peak_kind = peaks()
    achieved = F_PASS * T / (phase_ms[dom] * 1e-3) / 1e12
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp) and not args.tokens:
        with open(tp) as f:  # per workload: the GEMM passes' DRAM bytes per launch
            traffic = json.load(f).get(f"config{args.config}", {}).get(dom)

    # the rank-16 strong-scaling workload (65,536 positions split over the
    # ranks) at this world size, beside the default line
    strong = None
    if args.config == 2 and not args.no_strong:
        note("strong-scaling workload")
        r3 = CONFIGS[3]["rank"]
        m3, h3, tgt3, dH3, dT3, T3 = make_handle(3, world, rank, local, None, seed=3000)
        with_comm(m3)
        s3 = measure(rig, m3, h3, tgt3, dH3, dT3, T3, world, args.steps, args.warmup,
                     breakdown=False)
        m3.close()
        per_rank = rig.gather({"rank": rank, "phase_ms": {k: round(v, 4)
                                                          for k, v in s3["phase_ms"].items()}})
        f3 = flops(r3)[0]
        strong = {
            "workload": CONFIGS[3]["desc"], "config": 3, "scaling": "strong",
            "tokens_per_step": CONFIGS[3]["tokens"], "T_per_gpu": T3, "rank": r3,
            "value": s3["value"], "unit": UNIT, "ms_per_step": s3["total_ms"] / args.steps,
            "frac_step_of_peak": f3 * s3["value"] / world / 1e12 / peak_tf,
            "e2e": {"value": s3["e2e_value"], "unit": UNIT,
                    "h2d_bytes_per_step": s3["h2d_bytes"] * world, "d2h_bytes_per_step": 8},
            "allreduce_us_per_rank": [round(1e3 * p["phase_ms"].get("allreduce", 0.0), 1)
                                      for p in per_rank],
            "pass_ms_per_rank": [{"pass1": p["phase_ms"]["pass1_lse"],
                                  "pass2": p["phase_ms"]["pass2_grad"]} for p in per_rank],
            "phase_ms_rank0": per_rank[0]["phase_ms"],
            "gpu_launches": s3["launches"] * args.steps,
        }

    # The CPU reference last: its pool (spawned, all host cores) runs after
    # the GPU legs, so that the host-memory churn of its processes cannot
    # affect the pinned buffers of the end-to-end leg.
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        note("CPU reference")
        ref = CpuReference()
        cpu = ref.sample(15.0)
        ref.close()

    if rank == 0:
        e2e_ms = res["e2e_ms"]
        line = {
            "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["total_ms"] / args.steps,
            "higher_is_better": True, "scaling": CONFIG["scaling"], "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded; h bf16 N(0,1), W " +
                    ("Q4_K blocks" if CONFIG["q4k"] else "f16 N(0,0.02)") + ", Zipf(1.1) targets)",
            "config": config_dict(args.config, world, T),
            "tflops_step": F_TOK * T * world / (res["total_ms"] / args.steps * 1e-3) / 1e12 / world,
            "frac_step_of_peak": F_TOK * T / (res["total_ms"] / args.steps * 1e-3) / 1e12 / peak_tf,
            "phase_ms": {k: round(v, 4) for k, v in phase_ms.items()},
            "roofline": {"kernel": dom, "bound": "tensor", "achieved": achieved,
                         "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                         "peak_kind": f"{peak_kind} bf16 dense burst",
                         "flops_per_launch": F_PASS * T, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": res["e2e_value"], "unit": UNIT,
                    "h2d_bytes_per_step": res["h2d_bytes"], "d2h_bytes_per_step": 8,
                    "host_cpus": numa_cpus,
                    "ms_per_step": {"min": round(min(e2e_ms), 4),
                                    "median": round(statistics.median(e2e_ms), 4),
                                    "max": round(max(e2e_ms), 4)},
                    "graph_host_us": res.get("e2e_host_us"),
                    "breakdown": res.get("e2e_breakdown")},
            "gpu_launches": res["launches"] * args.steps,
            "clocks": clk,
        }
        if strong is not None:
            line["strong"] = strong
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def config_dict(n: int, world: int, T: int) -> dict:
    """The `config` object of a line (the same keys in both arms)."""
    return {"workload": CONFIGS[n]["desc"], "config": n, "T_per_gpu": T, "vocab": V, "dim": D,
            "rank": CONFIGS[n]["rank"], "lr": LR, "weight_decay": WD,
            "parallelism": f"dp{world}",
            "l2": "flushed (256 MB write) before every timed step"}


if __name__ == "__main__":
    main()
