"""Benchmark of the KERNIX-B200 .knx forward path (one JSON line on rank 0).

Workload: config c2 -- the int8-quantised MLP 1024-4096-4096-1024 with GELU hidden layers (I8_COL weights), batch
4096 per GPU, seeded synthetic inputs ~N(0,1) and random-init weights ~N(0,0.02). A step is one forward pass over
one batch. With N GPUs (torchrun, one process per GPU) every rank runs its own replica on its own 4096 samples:
the path has no cross-sample exchange, so there is no collective in the data path ("scaling": "weak").

  value        samples/s over all ranks with inputs already in HBM (kernix_model_forward_device), each step
               timed with CUDA events on the launching stream after an L2 flush, max over ranks
  e2e          samples/s through the public C ABI kernix_capi_forward with page-locked host input and output
               (host->device copy of the inputs and device->host copy of the outputs inside the timed region)
  roofline     the dominant kernel (tcgen05 kind::i8 GEMM, all three layers), algorithmic int8 ops / CUDA-event time
  cpu_baseline the reference's own CPU forward (oracle/_ref, compiled from the reference sources) on a bounded
               sample, all host threads (one model instance per thread; the reference's forward is per-model serial)
  per_config   (N = 1) every other configuration at its benchmark batch -- c1 256, c2 32, c3 1024, c4 512, c5 1 and
               256 -- device-resident samples/s with the achieved rate and its fraction of the bound at that batch
  strong_scaling  c5 at batch 1 / 64 / 256 with every layer's output columns split over all N GPUs (the runtime's
               own ncclAllGather per layer), ms per forward, max over ranks: the strong-scaling companion of value

  --impl reference times the reference's CPU forward on the same 4096-sample c2 batch per step, all host threads.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kernix|reference]
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = "c2"
BATCH = 4096
DIMS = [1024, 4096, 4096, 1024]
METRIC = "samples/s, int8 MLP 1024-4096-4096-1024 (config c2), batch 4096 per GPU"
WORKLOAD = "c2: int8-quantised MLP 1024-4096-4096-1024, GELU hidden, I8_COL per-output-channel weights, batch 4096"
L2_FLUSH_BYTES = 256 << 20
# DRAM bytes (read + write) of one k_i8_chain launch at M = 4096 from an ncu capture (dram__bytes_read.sum 29.80 MB +
# dram__bytes_write.sum 11.80 MB): the weights and the layer-0 rows are read once, the output written once, the hidden
# int8 rows stay in L2
CHAIN_DRAM_BYTES = 41.60e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["kernix", "reference"], default="kernix")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="time box of the CPU-baseline sample (0: none)")
    ap.add_argument("--kernel-case", type=int, default=0, metavar="M",
                    help="profiling case: only run the int8 GEMM of c2's 4096x4096 layer with M rows, 3 launches, then exit")
    ap.add_argument("--kernel-k", type=int, default=4096, help="K of the profiling case (1024: c2's first layer)")
    ap.add_argument("--kernel-act", type=int, default=1, help="activation of the profiling case (1 GELU, -1 none)")
    ap.add_argument("--kernel-dtype", choices=["i8", "f32", "attn", "chain"], default="i8",
                    help="kernel of the profiling case: int8 or 3xTF32 GEMM, (attn) the attention core on c4's shape "
                         "(M samples x 128 positions, 8 heads of 64), or (chain) c2's three int8 layers as the forward "
                         "runs them, one k_i8_chain launch over M rows")
    ap.add_argument("--workload", choices=["c2", "c5-rows", "c1", "c3", "c4", "c5"], default="c2",
                    help="c5-rows: config c5 with its wide layers split by output columns over the torchrun ranks "
                         "(one NCCL all-gather per layer; every rank runs the same batch: strong scaling). c1, c3, c4, "
                         "c5: the device-resident forward of that configuration at --batch samples per GPU")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong_scaling object (c5 column-sharded over all ranks at batch 1 / 64 / 256)")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per_config object (the other configurations at their benchmark batch sizes)")
    ap.add_argument("--batch", type=int, default=0,
                    help="samples per step: global batch of c5-rows (default 64), per-GPU batch of c1/c3/c4/c5 "
                         "(default: the configuration's own, 256 / 1024 / 512 / 256)")
    return ap.parse_args()


class ChainCase:
    """c2's three int8 layers (1024-4096-4096-1024, GELU hidden) as one kx_i8_chain launch over m rows, the forward's
    dominant kernel: seeded int8 rows and weights (timing does not depend on the values), the quantised hidden rows
    in scratch, control words cleared before every launch as the forward's quantiser clears them."""

    def __init__(self, L, torch, np, m):
        import ctypes
        rng = np.random.default_rng(3)
        self.L, self.torch, self.m = L, torch, m
        self.ctypes = ctypes
        d = DIMS
        self.keep = []
        dev = lambda a: self._k(torch.from_numpy(np.ascontiguousarray(a)).cuda())  # noqa: E731
        self.a = [dev(rng.integers(-127, 128, (m, d[0]), dtype=np.int8))] + \
            [self._k(torch.zeros((m, d[l + 1]), dtype=torch.int8, device="cuda")) for l in range(2)]
        self.sx = [self._k(torch.full((m,), 0.01, device="cuda")) for _ in range(3)]
        self.wq = [dev(rng.integers(-127, 128, (d[l + 1], d[l]), dtype=np.int8)) for l in range(3)]
        self.sc = [self._k(torch.full((d[l + 1],), 0.002, device="cuda")) for l in range(3)]
        self.bi = [self._k(torch.zeros(d[l + 1], device="cuda")) for l in range(3)]
        rgs = (m + 127) // 128
        self.ctl = self._k(torch.zeros(2 * (m + 2 * rgs), dtype=torch.int32, device="cuda"))
        self.y = self._k(torch.empty((m, d[-1]), device="cuda"))
        self.status = self._k(torch.zeros(1, dtype=torch.int32, device="cuda"))
        P = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])  # noqa: E731
        I = lambda v: (ctypes.c_int * len(v))(*v)  # noqa: E731, E741
        self.args = [P(self.a), I(d[:3]), P(self.sx), P(self.wq), I(d[:3]), P(self.sc), P(self.bi), I(d[:3]), I(d[1:]),
                     I([1, 1, -1]), (ctypes.c_float * 3)(0.0, 0.0, 0.0), P(self.sx[1:])]

    def _k(self, t):
        self.keep.append(t)
        return t

    def clear(self):
        self.ctl.zero_()

    def launch(self, stream):
        vp = self.ctypes.c_void_p
        if self.L.kx_i8_chain(3, self.m, *self.args, vp(self.ctl.data_ptr()), vp(self.y.data_ptr()),
                              vp(self.status.data_ptr()), vp(stream.cuda_stream)) != 0:
            raise RuntimeError("kx_i8_chain failed")

    def check(self):
        if int(self.status.item()) != 0:
            raise RuntimeError("the int8 chain reported a timeout")


def kernel_case(m_rows, k=4096, act=1, dtype="i8"):
    """Three launches of the int8 GEMM (GELU epilogue by default), or with dtype "f32" of the 3xTF32 GEMM, on an
    M x K x 4096 problem -- for an ncu capture of one kernel on a case larger than L2 (M = 8192, K = 4096: 32 MB A
    + 16 MB B + 128 MB C for int8)."""
    import numpy as np
    import torch

    from kernix_b200 import build, kx_abi
    build.build()
    L = kx_abi.lib()
    n = 4096
    rng = np.random.default_rng(0)
    if dtype == "chain":
        case = ChainCase(L, torch, np, m_rows)
        st = torch.cuda.current_stream()
        for _ in range(3):
            case.clear()
            case.launch(st)
        torch.cuda.synchronize()
        case.check()
        print(json.dumps({"kernel_case": "k_i8_chain", "m": m_rows, "dims": DIMS, "launches": 3}))
        return
    if dtype == "attn":  # c4's attention core: S = 128, 8 heads, d = 64, Q / K / V packed in one row as the model does
        S, H, d = 128, 8, 64
        qkv = torch.from_numpy(rng.standard_normal((m_rows * S, 3 * H * d)).astype(np.float32)).cuda()
        ctx = torch.empty((m_rows * S, H * d), device="cuda")
        ld, base = 3 * H * d, qkv.data_ptr()
        for _ in range(3):
            kx_abi.call("kx_attention", base, ld, base + 4 * H * d, ld, base + 8 * H * d, ld, ctx.data_ptr(), H * d, m_rows, S, S,
                        H, d, d, 0, None, None)
        torch.cuda.synchronize()
        print(json.dumps({"kernel_case": "k_attention_tc", "samples": m_rows, "seq": S, "heads": H, "head_dim": d,
                          "launches": 3}))
        return
    if dtype == "f32":
        ldw = (k + 31) // 32 * 32
        w = torch.from_numpy((rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)).cuda()
        hi = torch.empty((n, ldw), device="cuda")
        lo = torch.empty((n, ldw), device="cuda")
        kx_abi.call("kx_prep_f32_weight", w.data_ptr(), k, n, hi.data_ptr(), lo.data_ptr(), ldw, None)
        x = torch.from_numpy(rng.standard_normal((m_rows, k)).astype(np.float32)).cuda()
        b = torch.zeros(n, device="cuda")
        y = torch.empty((m_rows, n), device="cuda")
        for _ in range(3):
            kx_abi.call("kx_gemm_f32", x.data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, b.data_ptr(), y.data_ptr(), n,
                        m_rows, n, k, act, 0.0, None, None)
        torch.cuda.synchronize()
        print(json.dumps({"kernel_case": "k_gemm_tf32x3", "m": m_rows, "n": n, "k": k, "act": act, "launches": 3}))
        return
    xq = torch.from_numpy(rng.integers(-127, 128, (m_rows, k), dtype=np.int8)).cuda()
    wq = torch.from_numpy(rng.integers(-127, 128, (n, k), dtype=np.int8)).cuda()
    sx = torch.full((m_rows,), 0.01, device="cuda")
    sc = torch.full((n,), 0.001, device="cuda")
    b = torch.zeros(n, device="cuda")
    y = torch.empty((m_rows, n), device="cuda")
    for _ in range(3):
        if L.kx_gemm_i8(xq.data_ptr(), k, sx.data_ptr(), wq.data_ptr(), k, sc.data_ptr(), b.data_ptr(), y.data_ptr(), n, m_rows,
                        n, k, act, 0.0, None, None) != 0:
            raise RuntimeError("kx_gemm_i8 failed")
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": "k_gemm_i8", "m": m_rows, "n": n, "k": k, "act": act, "launches": 3}))


def model_file(rank):
    from kernix_b200 import configs
    return configs.model_path(CFG, os.environ.get("KERNIX_MODEL_DIR", f"/tmp/kernix_models_r{rank}"))


# ------------------------------------------------------------------------------ reference CPU forward
def reference_throughput(path, seconds, samples_per_call=8, threads=None):
    """The reference's own forward (oracle/_ref: include/kernix_model.h compiled from source) on host cores: one
    model per thread (kernix_model_forward is not reentrant per model; different models may run concurrently),
    default workspace limit, so the int8 layers run the reference's kernix_qmatmul (x86: its scalar loop).
    Returns (samples/s, threads, samples processed, seconds)."""
    import numpy as np

    from kernix_b200 import configs
    from oracle import ref_lib

    threads = threads or os.cpu_count() or 1
    models = [ref_lib.RefModel(path) for _ in range(threads)]
    x = configs.inputs(CFG, samples_per_call, seed=7)
    models[0].forward(x)  # warm
    counts = [0] * threads
    stop = time.perf_counter() + seconds

    def work(i):
        m = models[i]
        while time.perf_counter() < stop:
            m.forward(x)
            counts[i] += samples_per_call

    t0 = time.perf_counter()
    ts = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    dt = time.perf_counter() - t0
    n = sum(counts)
    for m in models:
        m.close()
    del np
    return n / dt, threads, n, dt


def cpu_model():
    """The host CPU's model name (first 'model name' of /proc/cpuinfo), or the platform's processor string."""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.lower().startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def run_reference(args):
    """The reference arm: the reference's own CPU forward (oracle/_ref, include/kernix_model.h compiled from its
    sources) on the same workload as the GPU arm -- config c2, 4096 samples per step -- with every host thread:
    the 4096 samples are split over one reference model per thread (kernix_model_forward is serial per model and
    models may run concurrently), each at the reference's default workspace limit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import ref_lib
    if not ref_lib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libkernix_ref.so was not built (make -C oracle/ref)"}))
        return
    path = model_file(0)
    threads = os.cpu_count() or 1
    per_step = BATCH  # the GPU arm's batch: same configuration, same samples per step
    from oracle import ref_lib as rl
    from kernix_b200 import configs
    models = [rl.RefModel(path) for _ in range(threads)]
    x = configs.inputs(CFG, per_step, seed=100)
    bounds = [per_step * i // threads for i in range(threads + 1)]
    chunks = [x[bounds[i]:bounds[i + 1]] for i in range(threads)]

    def step():
        ts = [threading.Thread(target=models[i].forward, args=(chunks[i],)) for i in range(threads) if len(chunks[i])]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    v = per_step * args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic: inputs ~N(0,1) seed 100, random-init weights ~N(0,0.02)",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH, "global_batch": per_step,
                       "parallelism": f"{threads} host threads, one reference model each"},
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "cpu": cpu_model(), "kind": "reference",
                             "sample": f"the full {per_step}-sample batch per step, split over {threads} threads with one "
                                       "reference model each (default workspace: the int8 layers run the reference's "
                                       "kernix_qmatmul scalar loop on x86)"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    for m in models:
        m.close()
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi samples (200 ms) of this GPU's SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        import tempfile
        self.path = tempfile.mktemp(prefix="kx_clocks_", suffix=".csv")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            try:
                self.lines = [ln for ln in open(self.path).read().splitlines() if ln.strip()]
                os.remove(self.path)
            except OSError:
                pass

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------------- GPU bench
def reduce_max(dist, v, device):
    """The maximum of v over all ranks (v itself without a process group): every rank's timed region is
    reported as the slowest rank's."""
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_batch(rank):
    """The seeded synthetic input rows of one rank: every rank runs its own BATCH samples (weak scaling)."""
    from kernix_b200 import configs
    return configs.inputs(CFG, BATCH, seed=100 + rank)


def run_kernix(args):
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        return reduce_max(dist, v, "cuda")

    from kernix_b200 import Model, build, configs, kx_abi
    build.build()
    L = kx_abi.lib()
    L.kernix_model_forward_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    L.kernix_model_forward_device.restype = ctypes.c_int
    L.kernix_model_check.argtypes = [ctypes.c_void_p]
    L.kernix_model_check.restype = ctypes.c_int

    os.environ["KERNIX_DEVICE"] = str(local)
    path = model_file(rank)
    m = Model(path)
    x_np = rank_batch(rank)
    x_pin = torch.from_numpy(x_np).pin_memory()
    out_pin = torch.empty((BATCH, DIMS[-1]), dtype=torch.float32).pin_memory()
    x_dev = x_pin.cuda()
    y_dev = torch.empty((BATCH, DIMS[-1]), dtype=torch.float32, device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()  # every launch and event of the timed regions goes on this one stream
    torch.cuda.set_stream(stream)

    def fwd_device():
        if L.kernix_model_forward_device(m._h, x_dev.data_ptr(), BATCH, y_dev.data_ptr(), stream.cuda_stream) != 0:
            raise RuntimeError("forward_device failed")

    # ---- value: device-resident forward, events per step, L2 flushed before each step
    for _ in range(args.warmup):
        fwd_device()
    torch.cuda.synchronize()
    if L.kernix_model_check(m._h) != 0:
        raise RuntimeError("a kernel reported a failure")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    with Clocks(local) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            fwd_device()
            e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    if L.kernix_model_check(m._h) != 0:
        raise RuntimeError("a kernel reported a failure")
    t_dev = sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3
    t_dev = max_over_ranks(t_dev)
    ms_step = t_dev / args.steps * 1e3
    value = world * BATCH * args.steps / t_dev

    # ---- e2e: public C ABI with page-locked host buffers (H2D + forward + D2H inside the timed region)
    def fwd_host():
        if L.kernix_capi_forward(m._h, x_pin.data_ptr(), BATCH, out_pin.data_ptr()) != 0:
            raise RuntimeError("kernix_capi_forward failed")

    # untimed: the host forward tries its piece counts over its first 7 calls at a batch size and keeps the fastest
    for _ in range(max(args.warmup, 8)):
        fwd_host()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fwd_host()
    torch.cuda.synchronize()
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e = world * BATCH * args.steps / t_e2e
    y_e2e = out_pin.numpy().copy()
    if not np.array_equal(y_e2e, y_dev.cpu().numpy()):
        raise RuntimeError("host-memory and device-memory forward disagree")

    # ---- roofline of the dominant kernel: the int8 GEMM of each layer, CUDA events on the launching stream
    roof = None
    if rank == 0:
        roof = gemm_roofline(L, torch, np, args.steps, flush)

    # ---- CPU baseline: the reference's own forward on this host (rank 0 at N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle import ref_lib
        if ref_lib.available():
            v, thr, n, dt = reference_throughput(path, args.cpu_seconds)
            cpu = {"value": v, "unit": "samples/s", "cores": thr, "cpu": cpu_model(), "kind": "reference",
                   "sample": f"{n} samples of the c2 workload in {dt:.1f} s, {thr} threads with one reference model each "
                             "(default workspace: int8 layers run the reference's kernix_qmatmul scalar loop on x86)"}
        else:
            cpu = {"value": None, "unit": "samples/s", "cores": 0, "kind": "reference", "sample": "oracle/_ref not built"}

    # ---- strong scaling beside the weak-scaling value: c5 column-sharded over all ranks (every N, every rank)
    strong = None
    if not args.no_strong:
        strong = c5_sharded_times(L, torch, dist, rank, world, local, [1, 64, 256], max(5, args.steps // 2), 3)

    # ---- the other configurations at their benchmark batch sizes (rank 0 at N = 1 only)
    per_config = None
    if rank == 0 and world == 1 and not args.no_per_config:
        per_config = measure_configs(L, torch, flush, stream, max(5, args.steps // 2), 3)

    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except (OSError, ValueError):
            pass
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic: inputs ~N(0,1) seeded per rank, random-init weights ~N(0,0.02) quantised per output column",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH, "global_batch": BATCH * world,
                       "parallelism": f"dp{world} (independent replicas, batch sharded)",
                       "l2": "flushed (256 MB write) before every timed device step, flush not timed; weights 25 MB"},
            "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": BATCH * DIMS[0] * 4,
                    "d2h_bytes_per_step": BATCH * DIMS[-1] * 4, "api": "kernix_capi_forward, page-locked host buffers"},
            "roofline": roof,
            "cpu_baseline": cpu,
            "per_config": per_config,
            "strong_scaling": strong,
            "clocks": clk.summary(),
            "gpu_launches": 2 * args.steps,  # per forward: the row quantiser, then the one-launch int8 chain
            "peaks_file": bool(peaks),
        }
        print(json.dumps(line), flush=True)
    m.close()
    if dist is not None:
        dist.destroy_process_group()


def layer_gemm_times(L, torch, np, steps, flush):
    """Each c2 layer shape as its own kx_gemm_i8 launch (M = 4096, fp32 output, GELU), CUDA events around each
    launch, L2 flushed before each: the per-layer context of the roofline."""
    rng = np.random.default_rng(3)
    st = torch.cuda.current_stream()
    per = []
    for k, n in zip(DIMS[:-1], DIMS[1:]):
        xq = torch.from_numpy(rng.integers(-127, 128, (BATCH, k), dtype=np.int8)).cuda()
        wq = torch.from_numpy(rng.integers(-127, 128, (n, k), dtype=np.int8)).cuda()
        sx = torch.full((BATCH,), 0.01, device="cuda")
        sc = torch.full((n,), 0.001, device="cuda")
        b = torch.zeros(n, device="cuda")
        y = torch.empty((BATCH, n), device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")

        def launch():
            if L.kx_gemm_i8(xq.data_ptr(), k, sx.data_ptr(), wq.data_ptr(), k, sc.data_ptr(), b.data_ptr(), y.data_ptr(), n,
                            BATCH, n, k, 1, 0.0, status.data_ptr(), st.cuda_stream) != 0:
                raise RuntimeError("kx_gemm_i8 failed")

        for _ in range(3):
            launch()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(st)
            launch()
            e1.record(st)
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError("GEMM reported a timeout")
        t = sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3 / steps
        per.append({"m": BATCH, "k": k, "n": n, "us": t * 1e6, "tops": 2.0 * BATCH * k * n / t / 1e12})
    return per


def gemm_roofline(L, torch, np, steps, flush):
    """Roofline of the forward's dominant kernel, k_i8_chain (c2's three int8 layers in one persistent launch; the
    quantiser that feeds it is the rest of the forward), timed alone on c2's M = 4096 as the forward runs it: CUDA
    events on the launching stream around each launch, L2 flushed and the chain's control words cleared before each.
    Achieved = 206.16 GOP per launch / mean launch time; peak = 2 x the measured dense bf16 burst."""
    st = torch.cuda.current_stream()
    case = ChainCase(L, torch, np, BATCH)
    for _ in range(3):
        case.clear()
        case.launch(st)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in evs:
        flush.zero_()
        case.clear()
        e0.record(st)
        case.launch(st)
        e1.record(st)
    torch.cuda.synchronize()
    case.check()
    t = sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3 / steps
    ops = 2.0 * BATCH * sum(k * n for k, n in zip(DIMS[:-1], DIMS[1:]))
    achieved = ops / t / 1e12
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak = 2.0 * float(peaks["bf16_tflops"])
        basis = "2 x measured dense bf16 burst (MEASURED_PEAKS.json); the int8 tensor rate is twice bf16 on B200"
    except (OSError, ValueError, KeyError):
        peak = 2.0 * 1590.0
        basis = "2 x fallback dense bf16 1.59 PFLOP/s"
    per = layer_gemm_times(L, torch, np, steps, flush)
    return {"kernel": "k_i8_chain (tcgen05 kind::i8, cta_group::2, 256x256 tiles of all three layers in one persistent "
                      "launch; hidden layers quantise their own output rows)",
            "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s (int8, 2 ops per MAC)",
            "frac": achieved / peak, "peak_basis": basis, "us_per_launch": t * 1e6, "traffic": CHAIN_DRAM_BYTES,
            "traffic_note": "dram read + write bytes of one k_i8_chain launch at M = 4096 from an ncu capture (profiles/)",
            "algorithmic_ops_per_launch": ops, "per_layer_standalone": per}


def c5_sharded_times(L, torch, dist, rank, world, local, batches, steps, warmup):
    """Strong scaling of config c5 (fp32 MLP 8192-16384-16384-8192): its layers split by output columns over all
    `world` ranks (kernix_model_load_sharded_nccl; the runtime calls ncclAllGather per layer on the model's stream;
    one rank = the whole model), each batch timed as `steps` back-to-back device-resident forwards with CUDA events
    on the model's stream, max over ranks. The weights (2.15 GB / world per rank) stream from HBM every forward."""
    from kernix_b200 import Model, configs, shard
    model_dir = os.environ.get("KERNIX_MODEL_DIR_SHARED", "/tmp/kernix_models_shared")
    if rank == 0:
        configs.model_path("c5", model_dir)
    if dist is not None:
        dist.barrier()
    path = configs.model_path("c5", model_dir)
    uid = shard.share_nccl_id() if world > 1 else None
    m = Model(path, workspace_mb=0, shard=(rank, world, uid) if world > 1 else None)
    stream = torch.cuda.current_stream()
    out = {}
    for B in batches:
        x = torch.from_numpy(configs.inputs("c5", B, seed=100)).cuda()
        y = torch.empty((B, 8192), dtype=torch.float32, device="cuda")

        def step():
            if L.kernix_model_forward_device(m._h, x.data_ptr(), B, y.data_ptr(), stream.cuda_stream) != 0:
                raise RuntimeError("forward_device failed (c5 sharded)")

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        if L.kernix_model_check(m._h) != 0:
            raise RuntimeError("a kernel reported a failure (c5 sharded)")
        t = reduce_max(dist, e0.elapsed_time(e1) / 1e3 / steps, "cuda")
        out[str(B)] = {"ms_per_forward": t * 1e3, "samples_per_s": B / t, "achieved_tflops": 2.0 * 536870912 * B / t / 1e12}
    m.close()
    return {"workload": "c5 fp32 MLP 8192-16384-16384-8192, every layer's output columns split over all GPUs",
            "scaling": "strong", "n_gpus": world, "by_batch": out,
            "collective": "ncclAllGather per layer, called by the runtime on the model's stream" if world > 1 else "none (1 GPU)"}


def _peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured (MEASURED_PEAKS.json)"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# (configuration, batch) of the per_config object: every configuration at the batch its benchmark names
PER_CONFIG = [("c1", 256), ("c2", 32), ("c3", 1024), ("c4", 512), ("c5", 1), ("c5", 256)]
# algorithmic bytes one forward must move when it is bound by weight streaming: c2's int8 weights (+ scales and
# biases), c5's fp32 weights (+ biases)
WEIGHT_BYTES = {"c2": 1024 * 4096 + 4096 * 4096 + 4096 * 1024 + 8 * (4096 + 4096 + 1024),
                "c5": 4 * (8192 * 16384 + 16384 * 16384 + 16384 * 8192) + 4 * (16384 + 16384 + 8192)}
DOMINANT = {"c1": "k_mlp_chain (the three layers and the softmax in one cooperative launch, CUDA cores)",
            "c2": "k_gemm_i8 with K ranges + k_i8_rows (split-K int8 layers: tcgen05 kind::i8 over every SM)",
            "c3": "k_conv_tf32x3_cmt (3xTF32 tcgen05 implicit-GEMM convolution fed by TMA)",
            "c4": "k_gemm_tf32x3_pp / k_gemm_tf32x3_pair (3xTF32 tcgen05 GEMMs)",
            "c5@1": "k_skinny (fp32 weight streaming on the CUDA cores)",
            "c5@256": "k_gemm_tf32x3_pair (3xTF32 tcgen05, drained long reductions)"}


def measure_configs(L, torch, flush, stream, steps, warmup):
    """Device-resident forward (kernix_model_forward_device, inputs in HBM) of every configuration at its benchmark
    batch: CUDA events on the launching stream per step, L2 flushed (256 MB write) before each, the mean over the
    steps. Each entry gives samples/s, the achieved algorithmic rate and its fraction of the bound the
    configuration has at that batch: the 3xTF32 rate (measured dense bf16 burst / 2 for tf32, / 3 for the three
    products) for the tensor-bound ones, measured HBM bandwidth on the weight bytes for the weight-streaming ones
    (c2 at 32 rows, c5 at 1 row). The fraction is of the whole forward, so it bounds its dominant kernel's from below."""
    from kernix_b200 import Model, configs
    peaks, basis = _peaks()
    tf32x3 = float(peaks["bf16_tflops"]) / 2 / 3
    hbm = float(peaks["hbm_gbs"])
    out = {}
    model_dir = os.environ.get("KERNIX_MODEL_DIR_SHARED", "/tmp/kernix_models_shared")
    for cfg, B in PER_CONFIG:
        m = Model(configs.model_path(cfg, model_dir), workspace_mb=0)
        x = torch.from_numpy(configs.inputs(cfg, B, seed=100)).cuda()
        y = torch.empty((B, m.out_dim), dtype=torch.float32, device="cuda")

        def step():
            if L.kernix_model_forward_device(m._h, x.data_ptr(), x.shape[0], y.data_ptr(), stream.cuda_stream) != 0:
                raise RuntimeError(f"forward_device failed on {cfg}")

        for _ in range(warmup):
            step()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
        if L.kernix_model_check(m._h) != 0:
            raise RuntimeError(f"a kernel reported a failure on {cfg}")
        t = sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3 / steps
        m.close()
        del x, y
        key = f"{cfg}@{B}"
        e = {"batch": B, "samples_per_s": B / t, "ms_per_forward": t * 1e3,
             "dominant_kernel": DOMINANT.get(key, DOMINANT.get(cfg))}
        if cfg == "c2":  # 32 rows: weight streaming (the 25 MB of int8 weights leave L2 with the flush)
            gbs = WEIGHT_BYTES["c2"] / t / 1e9
            e.update(bound="hbm", achieved=gbs, unit="GB/s", frac=gbs / hbm, achieved_tops=2 * 25165824 * B / t / 1e12)
        elif cfg == "c5" and B <= 16:
            gbs = WEIGHT_BYTES["c5"] / t / 1e9
            e.update(bound="hbm", achieved=gbs, unit="GB/s", frac=gbs / hbm, achieved_tflops=CONFIG_FLOPS[cfg] * B / t / 1e12)
        else:
            tf = CONFIG_FLOPS[cfg] * B / t / 1e12
            e.update(bound="tensor (3xTF32)", achieved=tf, unit="TFLOP/s", frac=tf / tf32x3)
        out[key] = e
    out["peaks"] = {"basis": basis, "hbm_gbs": hbm, "tf32x3_tflops": tf32x3}
    return out


# algorithmic FLOPs per sample (2 per MAC) of the configurations, and their default batch
CONFIG_FLOPS = {"c1": 2 * 535040, "c3": 2 * 115018240, "c4": 2 * 2516582400, "c5": 2 * 536870912}
CONFIG_BATCH = {"c1": 256, "c3": 1024, "c4": 512, "c5": 256}


def run_config(args):
    """Device-resident forward of configuration c1, c3, c4 or c5 (kernix_model_forward_device; inputs already in
    HBM): each step is one forward of --batch samples per GPU after a 256 MB L2 flush, timed with CUDA events on the
    model's stream; value = samples of all ranks / max over ranks of the timed steps (weak scaling)."""
    import datetime

    import torch

    cfg = args.workload
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    from kernix_b200 import Model, build, configs, kx_abi
    build.build()
    L = kx_abi.lib()
    L.kernix_model_forward_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    L.kernix_model_forward_device.restype = ctypes.c_int
    L.kernix_model_check.argtypes = [ctypes.c_void_p]
    L.kernix_model_check.restype = ctypes.c_int
    model_dir = os.environ.get("KERNIX_MODEL_DIR", f"/tmp/kernix_models_r{rank}")
    os.environ["KERNIX_DEVICE"] = str(local)
    m = Model(configs.model_path(cfg, model_dir), workspace_mb=0)
    B = args.batch or CONFIG_BATCH[cfg]
    x = torch.from_numpy(configs.inputs(cfg, B, seed=100 + rank)).cuda()
    rows = x.shape[0]
    y = torch.empty((B, m.out_dim), dtype=torch.float32, device="cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB, larger than L2
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)

    def step():
        if L.kernix_model_forward_device(m._h, x.data_ptr(), rows, y.data_ptr(), stream.cuda_stream) != 0:
            raise RuntimeError("forward_device failed")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize()
    if L.kernix_model_check(m._h) != 0:
        raise RuntimeError("a kernel reported a failure")
    t = reduce_max(dist, sum(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3, "cuda")
    if rank == 0:
        line = {
            "metric": f"samples/s, configuration {cfg}, device-resident forward", "value": world * B * args.steps / t,
            "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (CUDA-core fp32 FMA)" if cfg == "c1" else "f32 (3xTF32 tensor cores)",
            "data": "synthetic: the configuration's seeded inputs and weights",
            "config": {"workload": cfg, "batch_per_gpu": B, "global_batch": B * world, "parallelism": f"dp{world}",
                       "l2": "flushed (256 MB write) before every step"},
            "achieved_tflops": CONFIG_FLOPS[cfg] * B * world * args.steps / t / 1e12,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    m.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_c5_rows(args):
    """Config c5 (fp32 MLP 8192-16384-16384-8192, ReLU) at a small batch, its three layers split by output columns
    over the ranks (kernix_model_load_sharded_nccl: the runtime calls ncclAllGather on the model's stream). value: batch * steps / (max
    over ranks of the CUDA-event time of the timed steps); the weights (2.15 GB, 1/N per rank) stream from HBM every
    step, larger than L2, so no flush is needed. e2e: kernix_capi_forward with page-locked host buffers."""
    import datetime

    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    from kernix_b200 import Model, build, configs, kx_abi, shard
    build.build()
    L = kx_abi.lib()
    L.kernix_model_forward_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    L.kernix_model_forward_device.restype = ctypes.c_int
    L.kernix_model_check.argtypes = [ctypes.c_void_p]
    L.kernix_model_check.restype = ctypes.c_int
    if rank == 0:
        configs.model_path("c5")
    if dist is not None:
        dist.barrier()
    path = configs.model_path("c5")
    os.environ["KERNIX_DEVICE"] = str(local)
    m = Model(path, workspace_mb=0, shard=(rank, world, shard.share_nccl_id()) if world > 1 else None)
    B = args.batch or 64
    x_pin = torch.from_numpy(configs.inputs("c5", B, seed=100)).pin_memory()
    out_pin = torch.empty((B, 8192), dtype=torch.float32).pin_memory()
    x_dev = x_pin.cuda()
    y_dev = torch.empty((B, 8192), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)

    def step():
        if L.kernix_model_forward_device(m._h, x_dev.data_ptr(), B, y_dev.data_ptr(), stream.cuda_stream) != 0:
            raise RuntimeError("forward_device failed")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    if L.kernix_model_check(m._h) != 0:
        raise RuntimeError("a kernel reported a failure")
    t = reduce_max(dist, e0.elapsed_time(e1) / 1e3, "cuda")
    value = B * args.steps / t
    # e2e through the C ABI with page-locked host buffers (untimed calls first: the piece-count tuning)
    for _ in range(8):
        L.kernix_capi_forward(m._h, x_pin.data_ptr(), B, out_pin.data_ptr())
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        if L.kernix_capi_forward(m._h, x_pin.data_ptr(), B, out_pin.data_ptr()) != 0:
            raise RuntimeError("kernix_capi_forward failed")
    t_e2e = reduce_max(dist, time.perf_counter() - t0, "cuda")
    if not np.array_equal(out_pin.numpy(), y_dev.cpu().numpy()):
        raise RuntimeError("host-memory and device-memory forward disagree")
    if rank == 0:
        flops = 2.0 * 536870912 * B  # 536,870,912 MACs per sample
        line = {
            "metric": f"samples/s, fp32 MLP 8192-16384-16384-8192 (config c5), batch {B}, layers split by output columns",
            "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (3xTF32 tensor cores)", "data": "synthetic: inputs U[-1,1) seed 100, weights N(0, sqrt(2/fan_in)), b = 0.01",
            "config": {"workload": f"c5-rows: c5 at batch {B}, every layer's output columns split over {world} GPU(s)",
                       "global_batch": B, "parallelism": f"column-parallel x{world}, ncclAllGather per layer from the runtime",
                       "l2": "no flush: 2.15 GB of weights stream from HBM every step"},
            "e2e": {"value": B * args.steps / t_e2e, "unit": "samples/s", "h2d_bytes_per_step": B * 8192 * 4,
                    "d2h_bytes_per_step": B * 8192 * 4, "api": "kernix_capi_forward, page-locked host buffers"},
            "achieved_tflops": flops * args.steps / t / 1e12,
            # weight bytes streamed per step per GPU: the fp32 copy on the skinny path (<= 16 rows), else tf32 hi + lo
            "weight_stream_gbs_per_gpu": (1 if B <= 16 else 2) * 2.147e9 / world * args.steps / t / 1e9,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    m.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.kernel_case:
        kernel_case(a.kernel_case, a.kernel_k, a.kernel_act, a.kernel_dtype)
    elif a.workload == "c5-rows":
        run_c5_rows(a)
    elif a.workload in CONFIG_FLOPS and a.impl != "reference":
        run_config(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_kernix(a)
