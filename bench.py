"""Benchmark of the RAC rotation-accumulate hot path on B200.

Default workload (the headline metric): rac_matmul, fp32 row-major
M = N = K = 4096, A and B i.i.d. U[-1, 1), CORDIC mode, 16 iterations; the
same JSON line carries the metric's second half under "llama":
RACLlamaBlock tokens/s (d 4096, 32 heads, ff 11008 SwiGLU, x [4, 2048, 4096],
CORDIC 16, tensor-parallel over the ranks).
Metric: MAC-equivalent GOP/s = 2*M*N*K / t, summed over all ranks.  With N
GPUs the columns of B and C are sharded across ranks (no collective on the
data path; strong scaling of the fixed 4096^3 problem).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload matmul|rotate|rope|softmax|rmsnorm|layernorm|llama]

`--impl reference` times the reference's own CPU implementation of
rac_matmul (lib/c rac_hal_sgemm, AVX2, all host threads) built from its
sources into oracle/_ref, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")
FALLBACK_HBM_GBS = 6650.0
# ~0.5 ms device spin queued ahead of each timed launch, so that the host's
# launch latency (Python + ctypes) is not inside the CUDA-event interval.
SPIN_CYCLES = 1_000_000


def load_peaks() -> dict:
    try:
        with open(PEAKS_PATH) as f:
            return json.load(f)
    except OSError:
        return {}


def load_traffic() -> dict:
    try:
        with open(TRAFFIC_PATH) as f:
            return json.load(f)
    except OSError:
        return {}


# ── distributed plumbing ──────────────────────────────────────────────────

def dist_init():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
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
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ── clocks ────────────────────────────────────────────────────────────────

class ClockSampler:
    """Samples nvidia-smi every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        mhz, maxm, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                maxm = max(maxm, float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": maxm or None,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ── CPU baselines (oracle/, the reference's lib/c built from its sources) ─

def cpu_matmul_baseline(M: int, N: int, K: int, iters: int, reps: int = 3, warm: int = 1) -> dict:
    """Times the reference's CPU rac_matmul (lib/c rac_hal_sgemm, AVX2 + OpenMP)
    on the full problem, plus the CORDIC GEMM composed from the reference's
    rac_project_n on a row sample (information only)."""
    import numpy as np
    import oracle as O
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    cores = os.cpu_count() or 1
    out = {"cores": cores}
    if O.ref_available():
        for _ in range(warm):
            O.ref_sgemm(A, B)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            O.ref_sgemm(A, B)
            ts.append(time.perf_counter() - t0)
        t = statistics.mean(ts)
        out.update(kind="reference", value=2.0 * M * N * K / t / 1e9,
                   sample=f"full {M}x{N}x{K} rac_hal_sgemm (lib/c AVX2 FMA path), mean of {reps}")
        rows = 16
        t0 = time.perf_counter()
        O.gemm_composed_ref(A[:rows], B, iters)
        tc = time.perf_counter() - t0
        out["cordic_composed"] = {"value": 2.0 * rows * N * K / tc / 1e9, "unit": "GOP/s",
                                  "sample": f"{rows} rows of C, sum_k rac_project_n(.., {iters}) * |b|"}
    else:
        rows = 64
        t0 = time.perf_counter()
        O.gemm(A[:rows], B, "nn", 1, iters)
        t = time.perf_counter() - t0
        out.update(kind="port", value=2.0 * rows * N * K / t / 1e9,
                   sample=f"{rows} rows of C through oracle.gemm (CORDIC, {iters} iterations)")
    out["unit"] = "GOP/s"
    return out


def cpu_stream_baseline(w: str, iters: int) -> dict | None:
    """The reference lib/c op on the host cores, on a bounded sample of the workload."""
    import numpy as np
    import oracle as O
    if not O.ref_available():
        return None
    rng = np.random.default_rng(3)
    cores = os.cpu_count() or 1
    if w == "rotate":
        n = 1 << 22
        v = rng.standard_normal((n, 2)).astype(np.float32)
        th = rng.uniform(-np.pi, np.pi, n).astype(np.float32)
        if iters == 16:
            f = lambda: O.ref_rotate_batch(v, th)                  # noqa: E731
            kind, sample = "reference", "2^22 vectors, lib/c rac_rotate_batch (16 iterations, OpenMP)"
        else:   # lib/c has only the scalar rac_rotate_n: time the OpenMP restatement of it
            f = lambda: O.rotate_batch(v, th, iters, literal_kinv=False)   # noqa: E731
            kind, sample = "port", f"2^22 vectors, rac_rotate_n restated (oracle, {iters} iterations, OpenMP)"
        units, unit = n, "Gvec/s"
    elif w == "rope":
        x = rng.standard_normal((1, 32, 4096, 128)).astype(np.float32)
        c, s_ = O.ref_rope_cache(4096, 128, 10000.0)
        f = lambda: O.ref_rope_apply(x, c, s_)                    # noqa: E731
        units, unit, sample = x.size, "Gelem/s", "[1,32,4096,128], lib/c rac_rope_apply (incl. one copy)"
        kind = "reference"
    elif w == "attention":
        q, k, v = (rng.standard_normal((1, 8, 2048, 128)).astype(np.float32) for _ in range(3))
        f = lambda: O.ref_attention(q, k, v, None, True)          # noqa: E731
        units, unit = 2 * 8 * 2048 * 2048 * 128 * 1e-3, "TFLOP/s"   # /1e9 below -> TFLOP/s
        sample = "[1,8,2048,128] causal, lib/c rac_scaled_dot_attention (OpenMP)"
        kind = "reference"
    elif w == "softmax":
        x = (rng.standard_normal((4096, 4096)) * 3).astype(np.float32)
        f = lambda: O.ref_softmax(x)                              # noqa: E731
        units, unit, sample = x.size, "Gelem/s", "4096 rows x 4096, lib/c rac_softmax_batch"
        kind = "reference"
    else:
        x = rng.standard_normal((4096, 4096)).astype(np.float32)
        g = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
        b = (rng.standard_normal(4096) * 0.1).astype(np.float32)
        f = (lambda: O.ref_rmsnorm(x, g, 1e-6)) if w == "rmsnorm" else (lambda: O.ref_layernorm(x, g, b, 1e-6))
        units, unit, sample = x.size, "Gelem/s", f"4096 rows x 4096, lib/c rac_{w}"
        kind = "reference"
    f()
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        f()
    t = (time.perf_counter() - t0) / reps
    return {"value": units / t / 1e9, "unit": unit, "cores": cores, "kind": kind, "sample": sample}


class _RefSwiGLU:
    """Built lazily around the reference module: down(silu(gate(x)) * up(x)) from
    three reference RACLinear layers -- the SwiGLU of
    bench/bench_rac_transformer.c:441-453, which the reference module lacks."""

    @staticmethod
    def make(ref, d, ff):
        import torch.nn as nn
        import torch.nn.functional as F

        class RefSwiGLU(nn.Module):
            def __init__(self):
                super().__init__()
                self.gate = ref.RACLinear(d, ff, bias=False)
                self.up = ref.RACLinear(d, ff, bias=False)
                self.down = ref.RACLinear(ff, d, bias=False)

            def forward(self, x):
                return self.down(F.silu(self.gate(x)) * self.up(x))
        return RefSwiGLU()


def _load_reference_module():
    """The reference's rac_torch.py (copied into oracle/_ref/py by oracle.build()),
    imported WITHOUT an extension so that it runs its own CPU path."""
    import importlib.util
    import warnings
    import oracle as O
    path = os.path.join(O.REF_PY_DIR, "rac_torch_ref.py")
    if not os.path.exists(path) or "rac_cuda_ext" in sys.modules:
        return None
    spec = importlib.util.spec_from_file_location("rac_torch_ref_cpu", path)
    mod = importlib.util.module_from_spec(spec)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        spec.loader.exec_module(mod)
    return mod


def cpu_llama_baseline(sample: dict) -> dict:
    """The reference RACLlamaBlock module on the host cores (every thread), on a
    bounded sample: batch 0's first T tokens through the full-width block with
    the benchmark's weights.  Off the GPU the reference module runs its own
    torch fallback (F.linear / matmul, rac_torch.py:183, :232).  The FFN is the
    gated one the benchmark runs, built from the reference's RACLinear.

    Also checks the GPU output on that sample: causal attention makes the first
    T outputs depend on the first T inputs only, so y_gpu[0, :T] must match the
    CPU oracle (oracle/torch_block.py with the CORDIC operand map, the CORDIC
    GEMM's exact identity) within 1e-4 of the output's rms."""
    import numpy as np
    import torch
    import oracle as O
    from oracle import torch_block as TB
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    p, x, y_gpu, H = sample["params"], sample["x"], sample["y"], sample["heads"]
    T, d = x.shape[1], x.shape[2]
    ff = p["up"].shape[0]
    iters = sample["iters"]
    with torch.no_grad():
        cos, sin = TB.rope_cache(d // H, T)
        op = (lambda t: torch.from_numpy(O.cordic_operand(t.contiguous().numpy(), iters))) \
            if sample["mode"] == "cordic" else None
        want = TB.block_forward(p, x, H, cos=cos, sin=sin, operand=op).numpy()
    err = float(np.abs(y_gpu.numpy() - want).max() / np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    assert err <= 1e-4, f"RACLlamaBlock output differs from the CPU oracle: {err:.3e}"
    check = {"max_abs_over_rms": err, "bar": 1e-4,
             "vs": f"oracle/torch_block.py ({sample['mode']}), batch 0 tokens 0..{T - 1}"}
    ref = _load_reference_module()
    with torch.no_grad():
        if ref is not None:
            blk = ref.RACLlamaBlock(d, H, ff_dim=ff, max_seq_len=T)
            blk.ffn = _RefSwiGLU.make(ref, d, ff)
            blk.norm1.weight.copy_(p["norm1"])
            blk.norm2.weight.copy_(p["norm2"])
            blk.attn.qkv.weight.copy_(p["qkv"])
            blk.attn.out_proj.weight.copy_(p["out"])
            for k in ("gate", "up", "down"):
                getattr(blk.ffn, k).weight.copy_(p[k])
            f = lambda: blk(x, is_causal=True)                 # noqa: E731
            kind = "reference"
            what = "the reference RACLlamaBlock module (rac_torch.py:1348-1383) on its CPU torch path"
        else:
            f = lambda: TB.block_forward(p, x, H, cos=cos, sin=sin)   # noqa: E731
            kind = "port"
            what = "oracle/torch_block.py, the restatement of the reference module's CPU path"
        f()
        reps = 3
        t0 = time.perf_counter()
        for _ in range(reps):
            f()
        t = (time.perf_counter() - t0) / reps
    return {"value": T / t, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"x [1,{T},{d}] through {what}, SwiGLU FFN, fp32 FMA (not CORDIC), mean of {reps}",
            "parity_check": check}


def run_reference(args) -> None:
    """--impl reference: the reference's own CPU rac_matmul on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M = N = K = 4096
    cores = os.cpu_count() or 1
    # torchrun sets OMP_NUM_THREADS=1 per process; the reference arm uses every
    # host thread (OpenMP reads the variable when the library is loaded).
    os.environ["OMP_NUM_THREADS"] = str(cores)
    import numpy as np
    import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/librac_ref.so not built"}))
        return
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    for _ in range(args.warmup):
        O.ref_sgemm(A, B)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.ref_sgemm(A, B)
        ts.append(time.perf_counter() - t0)
    t = statistics.mean(ts)
    v = 2.0 * M * N * K / t / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "rac_matmul MAC-equiv GOP/s at 4096^3", "value": v,
        "unit": "GOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "rac_matmul 4096x4096x4096 fp32 U[-1,1) (reference lib/c CPU path)"},
        "cpu_baseline": {"value": v, "unit": "GOP/s", "cores": cores, "kind": "reference",
                         "sample": "full 4096^3 per step: lib/c rac_hal_sgemm -> rac_sgemm_avx2 "
                                   "(the reference's CPU rac_matmul; FMA, lib/c has no CORDIC GEMM)"},
        "e2e": {"value": v, "unit": "GOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ── GPU workloads ─────────────────────────────────────────────────────────

def roofline_fp32(achieved_gops: float, iters: int, peaks: dict, sms: int, dur_ms: float,
                  traffic, mode: int = 1) -> dict:
    """FP32-issue roofline of the GEMM at SMs x 128 lanes x max SM clock:
    CORDIC costs (2n+2) FP32 instructions per MAC (the cost model stated for
    the path), FAST one FFMA per MAC."""
    mhz = float(peaks.get("sm_max_mhz", 1965.0))
    instr_peak = sms * 128 * mhz * 1e6
    per_mac = (2 * iters + 2) if mode else 1
    peak_gops = 2.0 * instr_peak / per_mac / 1e9
    return {"bound": "fp32_issue", "achieved": achieved_gops, "peak": peak_gops,
            "unit": "GOP/s (MAC-equiv)", "frac": achieved_gops / peak_gops,
            "peak_basis": f"{sms} SMs x 128 FP32 lanes x {mhz:.0f} MHz / {per_mac} instr per MAC "
                          "(of measured sm_max_mhz)",
            "kernel_ms": dur_ms, "traffic": traffic}


def run_matmul(args, world, rank, local) -> dict | None:
    import torch
    from rac_b200 import _lib, ext
    M = N = K = args.size
    if args.shape:
        M, N, K = (int(v) for v in args.shape.split(","))
    iters = args.iters
    mode = 0 if args.mode == "fast" else 1
    n0, n1 = N * rank // world, N * (rank + 1) // world
    Nl = n1 - n0
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(1234)
    A = torch.rand((M, K), device=dev, generator=g) * 2 - 1
    g.manual_seed(4321 + rank)
    B = torch.rand((K, Nl), device=dev, generator=g) * 2 - 1
    C = torch.empty((M, Nl), device=dev)
    flush = torch.empty(256 << 20 >> 2, device=dev)    # 256 MiB > 126 MB L2
    s = torch.cuda.current_stream()

    def step():
        ext.gemm(A, B, _lib.LAYOUT_NN, iters, mode, out=C, variant=args.variant)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()                              # between steps, outside the events
            torch.cuda._sleep(SPIN_CYCLES)
            starts[i].record(s)
            step()
            ends[i].record(s)
        torch.cuda.synchronize()
    barrier(world)
    per = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    t_local = statistics.mean(per)
    t = max_over_ranks(t_local, world)
    value = 2.0 * M * N * K / (t * 1e-3) / 1e9
    achieved_local = 2.0 * M * Nl * K / (t_local * 1e-3) / 1e9

    # e2e through the C ABI (rac_matmul_ex) with pinned host buffers.
    Ah = A.cpu().pin_memory()
    Bh = B.cpu().pin_memory()
    Ch = torch.empty((M, Nl)).pin_memory()
    L = _lib.lib()
    e2e_steps = max(1, min(args.steps, 5))
    L.rac_matmul_ex(Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr(), M, Nl, K, iters, mode)
    _lib.check()
    barrier(world)
    ts = []
    for _ in range(e2e_steps):
        t0 = time.perf_counter()
        L.rac_matmul_ex(Ah.data_ptr(), Bh.data_ptr(), Ch.data_ptr(), M, Nl, K, iters, mode)
        ts.append(time.perf_counter() - t0)
    _lib.check()
    te = max_over_ranks(statistics.mean(ts), world)
    assert torch.equal(Ch, C.cpu()), "e2e result differs from the device-resident run"
    te_abi = te
    # With N > 1 ranks the replicated A need not cross every rank's PCIe link:
    # through rac_b200.tp each rank uploads 1/N of A's rows and its B block, NCCL
    # all-gathers A over NVLink, and each rank downloads its C block.
    te_dist = None
    if world > 1 and M % world == 0:
        import torch.distributed as dist
        from rac_b200 import tp
        a0, a1 = M * rank // world, M * (rank + 1) // world
        Ash = A[a0:a1].cpu().pin_memory()
        Afull = torch.empty((M, K), device=dev)
        Cd = torch.empty((M, Nl), device=dev)
        ts = []
        for it_ in range(e2e_steps + 1):
            torch.cuda.synchronize()
            barrier(world)
            t0 = time.perf_counter()
            dist.all_gather_into_tensor(Afull, Ash.to(dev, non_blocking=True))
            tp.sharded_matmul(Afull, Bh.to(dev, non_blocking=True), iters, mode, out=Cd)
            Ch.copy_(Cd, non_blocking=True)
            torch.cuda.synchronize()
            if it_:
                ts.append(time.perf_counter() - t0)
        te_dist = max_over_ranks(statistics.mean(ts), world)
        assert torch.equal(Ch, C.cpu()), "distributed e2e result differs from the device-resident run"
        te = min(te, te_dist)

    # Context: cuBLAS SGEMM (torch.matmul, fp32, TF32 off) on the same operands.
    torch.backends.cuda.matmul.allow_tf32 = False
    for _ in range(3):
        torch.matmul(A, B)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record()
    for _ in range(reps):
        torch.matmul(A, B)
    e1.record()
    torch.cuda.synchronize()
    t_cublas = e0.elapsed_time(e1) / reps
    if rank != 0:
        return None
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peaks = load_peaks()
    traffic = load_traffic().get(f"gemm_cordic{iters}_{M}") if mode and M == N == K else None
    out = {
        "metric": "rac_matmul MAC-equiv GOP/s at 4096^3" if M == N == K == 4096
                  else f"rac_matmul MAC-equiv GOP/s at {M}x{N}x{K}",
        "value": value, "unit": "GOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"rac_matmul {M}x{N}x{K} fp32 U[-1,1), "
                               f"{'CORDIC ' + str(iters) + ' iterations' if mode else 'FAST'}",
                   "sharding": f"N-columns over {world} rank(s), no collective",
                   "l2": "flushed between steps (256 MiB write outside the timed events)"},
        "roofline": roofline_fp32(achieved_local, iters, peaks, sms, t_local, traffic, mode),
        "e2e": {"value": 2.0 * M * N * K / te / 1e9, "unit": "GOP/s",
                "h2d_bytes_per_step": 4 * (M * K + K * Nl) if te_dist is None or te_abi <= te_dist
                else 4 * (M * K // world + K * Nl),
                "d2h_bytes_per_step": 4 * M * Nl,
                "api": "rac_matmul_ex (C ABI), pinned host buffers, blocking"
                       if te_dist is None or te_abi <= te_dist else
                       "rac_b200.tp: 1/N of A's rows and this rank's B block uploaded from pinned host "
                       "buffers, A all-gathered over NVLink (NCCL), sharded_matmul, C block downloaded",
                "c_abi_value": 2.0 * M * N * K / te_abi / 1e9,
                "nccl_gather_value": None if te_dist is None else 2.0 * M * N * K / te_dist / 1e9,
                "bytes_note": "per rank"},
        "context": {"cublas_sgemm": {"value": 2.0 * M * Nl * K / (t_cublas * 1e-3) / 1e9,
                                     "unit": "GFLOP/s", "ms": t_cublas,
                                     "note": "torch.matmul fp32 (TF32 off) on this rank's operands; "
                                             "plain FMA SGEMM, not the CORDIC arithmetic"}},
        "gpu_launches": args.steps * (2 if _splits(M, N // world, K, sms) > 1 else 1),
        "clocks": clk.summary(),
    }
    return out


def _splits(M: int, N: int, K: int, sms: int) -> int:
    """Mirror of the library's tile and split-K rules (gemm_dispatch.cu)."""
    if M <= 32:
        tiles = -(-M // 16) * -(-N // 128)
    else:
        cands = [(-(-M // bm) * -(-N // bn), bm * bn) for bm, bn in ((64, 64), (32, 64))]
        tiles = min(cands, key=lambda c: (-(-c[0] // sms)) * c[1])[0]
    if tiles >= sms or K < 1024:
        return 1
    best, S = 1.0, 1
    for c in range(2, K // 256 + 1):
        share = -(-tiles * c // sms) / c
        if share < best - 1e-9:
            best, S = share, c
    return S


def stream_e2e(w: str, args, v: dict, world: int) -> dict:
    """The workload through the blocking rac.h entry point with pinned HOST
    buffers (host->device copies, kernel, device->host copies all inside the
    wall-clock timed call), max over ranks."""
    import ctypes

    import torch
    from rac_b200 import _lib
    L = _lib.lib()
    pin = lambda t: t.cpu().pin_memory()                      # noqa: E731
    p = lambda t: t.data_ptr()                                # noqa: E731
    f32 = ctypes.c_float
    if w == "rotate":
        vh, thh = pin(v["v"]), pin(v["th"])
        oh = torch.empty_like(vh).pin_memory()
        n = vh.shape[0]
        call = lambda: L.rac_rotate_batch_n(p(vh), p(thh), p(oh), n, args.iters)  # noqa: E731
        hin, hout = 12 * n, 8 * n
    elif w == "rope":
        qh, kh, ch, sh = pin(v["q"]), pin(v["kk"]), pin(v["ctab"]), pin(v["stab"])

        def call():
            L.rac_rope_apply(p(qh), p(ch), p(sh), *qh.shape)
            L.rac_rope_apply(p(kh), p(ch), p(sh), *kh.shape)
        hin = 4 * (qh.numel() + kh.numel()) + 2 * 4 * (ch.numel() + sh.numel())
        hout = 4 * (qh.numel() + kh.numel())
    elif w == "attention":
        qh, kh, vh = pin(v["qa"]), pin(v["ka"]), pin(v["va"])
        oh = torch.empty_like(qh).pin_memory()
        B, H, T, D = qh.shape
        call = lambda: L.rac_attention(p(qh), p(kh), p(vh), None, 1, p(oh), B, H, T, D)  # noqa: E731
        hin, hout = 3 * 4 * qh.numel(), 4 * qh.numel()
    else:
        xh = pin(v["x"])
        yh = torch.empty_like(xh).pin_memory()
        rows, d = xh.shape
        if w == "softmax":
            call = lambda: L.rac_softmax_batch(p(xh), p(yh), rows, d)  # noqa: E731
            hin = 4 * xh.numel()
        elif w == "rmsnorm":
            gh = pin(v["gam"])
            call = lambda: L.rac_rmsnorm(p(xh), p(yh), p(gh), f32(1e-6), rows, d)  # noqa: E731
            hin = 4 * (xh.numel() + d)
        else:
            gh, bh = pin(v["gam"]), pin(v["bet"])
            call = lambda: L.rac_layernorm(p(xh), p(yh), p(gh), p(bh), f32(1e-6), rows, d)  # noqa: E731
            hin = 4 * (xh.numel() + 2 * d)
        hout = 4 * xh.numel()
    call()
    _lib.check()
    ts = []
    for _ in range(max(1, min(args.steps, 3))):
        barrier(world)
        t0 = time.perf_counter()
        call()
        ts.append(time.perf_counter() - t0)
    _lib.check()
    te = max_over_ranks(statistics.mean(ts), world)
    units = v["units"]
    val = units * world / te / (1e12 if w == "attention" else 1e9)
    return {"value": val, "unit": v["unit_name"], "h2d_bytes_per_step": hin, "d2h_bytes_per_step": hout,
            "api": "blocking rac.h call on pinned host buffers (C ABI)"}


def run_stream(args, world, rank, local) -> dict | None:
    """HBM-bound ops of the path (replicas across ranks: rows are independent)."""
    import torch
    from rac_b200 import ext
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    w = args.workload
    launches_per_step = 2 if w == "rope" else 1
    if w == "rotate":
        n = 1 << args.log2n
        v = torch.randn((n, 2), device=dev, generator=g)
        th = (torch.rand(n, device=dev, generator=g) * 2 - 1) * 3.14159265
        ro = torch.empty_like(v)
        fn = lambda: ext.rotate_batch(v, th, args.iters, out=ro)  # noqa: E731
        bytes_, units, unit_name = 20 * n, n, "Gvec/s"
        cfg = f"rac_rotate_batch_n 2^{args.log2n} float2 ~N(0,1), theta U[-pi,pi), {args.iters} iterations"
    elif w == "rope":
        q = torch.randn((8, 32, 4096, 128), device=dev, generator=g)
        kk = torch.randn((8, 32, 4096, 128), device=dev, generator=g)
        ctab, stab = ext.rope_cache(4096, 128, 10000.0, device=dev)

        def fn():
            ext.rope_apply_(q, ctab, stab)
            ext.rope_apply_(kk, ctab, stab)
        bytes_, units, unit_name = 2 * 8 * q.numel(), 2 * q.numel(), "Gelem/s"
        cfg = "rac_rope_apply Q and K [8,32,4096,128] fp32 in place, base 1e4"
    elif w == "attention":
        qa, ka, va = [torch.randn((4, 32, 2048, 128), device=dev, generator=g) for _ in range(3)]
        ao = torch.empty_like(qa)
        fn = lambda: ext.attention(qa, ka, va, None, True, out=ao)  # noqa: E731
        # causal: QK^T and PV each B*H*T*(T/2)*hd MACs, 2 FLOP per MAC
        bytes_, units, unit_name = 4 * 4 * qa.numel(), 2 * 4 * 32 * 2048 * 2048 * 128, "TFLOP/s"
        cfg = "rac_attention [4,32,2048,128] fp32 causal (the RACLlamaBlock attention core)"
    elif w == "softmax":
        x = torch.randn((32768, 4096), device=dev, generator=g) * 3
        y = torch.empty_like(x)
        fn = lambda: ext.softmax(x, out=y)                        # noqa: E731
        bytes_, units, unit_name = 8 * x.numel(), x.numel(), "Gelem/s"
        cfg = "rac_softmax [32768, 4096] fp32 ~N(0,9)"
    else:
        x = torch.randn((args.rows, 4096), device=dev, generator=g)
        gam = torch.rand(4096, device=dev, generator=g) + 0.5
        bet = torch.randn(4096, device=dev, generator=g) * 0.1
        y = torch.empty_like(x)
        if w == "rmsnorm":
            fn = lambda: ext.rmsnorm(x, gam, 1e-6, out=y)         # noqa: E731
        else:
            fn = lambda: ext.layernorm(x, gam, bet, 1e-6, out=y)  # noqa: E731
        bytes_, units, unit_name = 8 * x.numel(), x.numel(), "Gelem/s"
        cfg = f"rac_{w} [{args.rows}, 4096] fp32, eps 1e-6"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    flush = torch.empty(256 << 20 >> 2, device=dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    s = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(SPIN_CYCLES)          # keeps the GPU busy while the host enqueues
            starts[i].record(s)
            fn()
            ends[i].record(s)
        torch.cuda.synchronize()
    barrier(world)
    t_local = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends))
    t = max_over_ranks(t_local, world)
    e2e = stream_e2e(w, args, locals(), world)
    if rank != 0:
        return None
    peaks = load_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    ach = bytes_ / (t_local * 1e-3) / 1e9
    if w == "attention":
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        fp32 = sms * 128 * 2 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12
        flops = units / (t_local * 1e-3) / 1e12
        return {"metric": "rac_attention FP32 TFLOP/s (causal, algorithmic)", "value": flops * world,
                "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": {"workload": cfg, "sharding": "replicas"},
                "roofline": {"bound": "fp32", "achieved": flops, "peak": fp32, "unit": "TFLOP/s",
                             "frac": flops / fp32, "peak_basis": "SMs x 128 lanes x 2 x sm_max_mhz",
                             "note": "causal diagonal tiles are computed in full (about 1/32 extra work)"},
                "e2e": e2e, "gpu_launches": args.steps, "clocks": clk.summary(),
                "cpu_baseline": cpu_stream_baseline(w, args.iters)
                if (world == 1 and not args.no_cpu_baseline) else None}
    cpu = cpu_stream_baseline(w, args.iters) if (world == 1 and not args.no_cpu_baseline) else None
    return {
        "cpu_baseline": cpu,
        "metric": f"{w} throughput", "value": units * world / (t * 1e-3) / 1e9, "unit": unit_name,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": cfg, "sharding": "replicas",
                                        "l2": "flushed between steps"},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "peak_basis": "of measured" if "hbm_gbs" in peaks else "of fallback",
                     "frac_of_8TBs": ach / 8000.0, "kernel_ms": t_local,
                     "traffic": load_traffic().get(f"rotate_{args.iters}" if w == "rotate" else w)},
        "e2e": e2e, "gpu_launches": args.steps * launches_per_step, "clocks": clk.summary(),
    }


def _all_host_threads() -> None:
    """The CPU baselines use every host core; set before oracle/ is loaded."""
    if int(os.environ.get("WORLD_SIZE", "1")) == 1:
        os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="matmul",
                    choices=["matmul", "rotate", "rope", "softmax", "rmsnorm", "layernorm", "llama",
                             "attention"])
    ap.add_argument("--size", type=int, default=4096)
    ap.add_argument("--shape", default=None, help="M,N,K for the matmul workload (e.g. 16,11008,4096)")
    ap.add_argument("--iters", type=int, default=16)
    ap.add_argument("--mode", choices=["cordic", "fast"], default="cordic")
    ap.add_argument("--variant", type=int, default=0)
    ap.add_argument("--rows", type=int, default=16384, help="norm workloads: row count")
    ap.add_argument("--log2n", type=int, default=26, help="rotate workload: log2 of the vector count")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp-chunks", type=int, default=None,
                    help="llama: batch pieces per tensor-parallel forward, each piece's all-reduce "
                         "overlapping the next piece's GEMMs (default 1)")
    ap.add_argument("--no-llama", action="store_true",
                    help="matmul workload: skip the RACLlamaBlock measurement in the same line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return
    _all_host_threads()
    # stdout carries rank 0's JSON line only: with several ranks, whatever the
    # communication libraries print at start-up (NCCL's version banner) goes to
    # stderr, and the line is written to the saved stdout descriptor.
    json_fd = 1
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        sys.stdout.flush()
        json_fd = os.dup(1)
        os.dup2(2, 1)
    world, rank, local = dist_init()
    from rac_b200 import tp
    llama = None
    if args.workload == "matmul":
        out = run_matmul(args, world, rank, local)
        if not args.no_llama and args.size == 4096 and not args.shape:
            llama = tp.bench_llama(args, world, rank, local, barrier, max_over_ranks, ClockSampler)
    elif args.workload == "llama":
        out = llama = tp.bench_llama(args, world, rank, local, barrier, max_over_ranks, ClockSampler)
    else:
        out = run_stream(args, world, rank, local)
    if rank == 0 and out is not None:
        if world == 1 and not args.no_cpu_baseline and args.workload == "matmul":
            if args.shape:
                M, N, K = (int(v) for v in args.shape.split(","))
            else:
                M = N = K = args.size
            out["cpu_baseline"] = cpu_matmul_baseline(M, N, K, args.iters)
        if llama is not None:
            sample = llama.pop("_sample", None)
            if world == 1 and not args.no_cpu_baseline and sample is not None:
                llama["cpu_baseline"] = cpu_llama_baseline(sample)
            if llama is not out:
                out["llama"] = llama
        os.write(json_fd, (json.dumps(out) + "\n").encode())
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
