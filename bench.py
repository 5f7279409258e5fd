#!/usr/bin/env python3
"""Benchmark of the quantized-MatMul hot path (and the GDN chunk inverse) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload gemm|gdn|decode]

Headline workload: W4A16 LPBQ GEMM, M=4096, K=4096, N=14336, LPBQ block 64, u16
activations from N(0,1), int4 weights from N(0,0.02), int32 bias, u16 output.  A "step" is one
quantized GEMM over one batch of synthetic input.  Metric: logical TOPS = 2*M*N*K / step time.

Multi-GPU (torchrun): the GEMM shards over N -- every rank owns a 14336-wide slab of output
channels (its own weights), so per-GPU work is fixed ("weak" scaling) and no collective touches
the data path; ``--allgather`` additionally gathers the outputs with NCCL and reports that time
separately.  Timing: CUDA events on the launching stream, per step, L2 flushed between steps (a
256 MB write, then a 256 MB read of another buffer so the write-back happens before the timed
window), max over ranks.

The default line also carries the GDN C=256 inverse ("secondary", 4096 chunks) and the BASELINE
decode/prefill rows of the W4A16 LPBQ GEMM ("decode": M in {1, 16, 128}, N in {4096, 14336}, GB/s
against the HBM peak), and the per-group W4 schema at the headline shape ("per_group": float32
scale per 64 weights of K, float32 bias).  ``--workload gdn``, ``--workload decode --m M --n N`` and
``--workload per_group --m M --n N`` run one of those alone (the commands the committed ncu
summaries were taken with).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from one
# `ncu --set full` capture of this script's own workload (bench.py --steps 1 --warmup 3 ...); the
# GDN figure is a 1024-chunk capture scaled by the chunk count to the 4096-chunk launch
NCU_TRAFFIC_BYTES = {
    ("qgemm", 4096, 4096, 14336): 152_121_856 + 98_887_424,           # full-size capture
    ("gdn", 4096): 4 * (100_822_016 + 208_797_696),                    # 1024-chunk capture x 4 chunks
    ("gdn_fused", 4096): 4 * (69_339_904 + 208_701_952),               # 1024-chunk capture x 4 chunks
    ("qdecode", 16, 4096, 14336): 118_091_264 + 4_662_784,             # full-size capture
    ("qdecode", 1, 4096, 4096): 33_753_344 + 0,                        # full-size capture
}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ----------------------------------------------------------------------------------------------
# synthetic inputs (generated on the device; BASELINE.json distributions)
# ----------------------------------------------------------------------------------------------
def synth_w4a16_lpbq(m: int, k: int, n: int, block: int, seed: int, device) -> dict:
    """u16 activations (asymmetric, fixed zp 32768) and LPBQ int4 weights, quantized with the
    reference generator's rules: symmetric int4 per (channel, K-block) group scales, factorised as
    per-channel base x integer factor in [1,16] (generate_qnn_matmul_python_cases.py:189-200,320-361)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=device)
    w = torch.randn((n, k), generator=g, device=device) * 0.02
    b = torch.randn((n,), generator=g, device=device) * 0.1
    s_a = max(-float(x.min()) / 32768.0, float(x.max()) / 32767.0, 1e-12)
    act = torch.clamp(torch.round(x.double() / s_a + 32768), 0, 65535).to(torch.int32).to(torch.uint16)
    wb = w.double().reshape(n, k // block, block)
    gs = (wb.abs().amax(dim=2).clamp_min(1e-12) / 7.0).float().double()
    base = torch.maximum(gs.amin(dim=1).clamp_min(1e-12), gs.amax(dim=1).clamp_min(1e-12) / 16.0)
    f = torch.clamp(torch.ceil(gs / base[:, None] - 1e-9), 1, 16)
    q = torch.clamp(torch.round(wb / (base[:, None, None] * f[:, :, None])), -7, 7).to(torch.int8).reshape(n, k)
    scale = base.float()
    bias_q = torch.clamp(torch.round(b.double() / (s_a * scale.double())), -2 ** 31, 2 ** 31 - 1).to(torch.int32)
    # output scale from the float output of the first 256 rows
    y = x[:256].double() @ w.double().t() + b.double()
    s_o = max(-float(y.min()) / 32768.0, float(y.max()) / 32767.0, 1e-12)
    nib = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).t().contiguous()
    return dict(act=act, w_packed=packed, q=q, factor=f.to(torch.uint8).contiguous(), scale=scale.contiguous(),
                bias_q=bias_q.contiguous(), s_a=s_a, s_o=s_o, m=m, k=k, n=n, block=block)


def synth_w4a16_per_group(m: int, k: int, n: int, seed: int, device) -> dict:
    """u16 activations as above and per-group int4 weights with the reference generator's rules:
    symmetric float32 scale per (channel, 64 weights of K), float32 bias kept unquantized
    (generate_qnn_matmul_python_cases.py:392-423, 460-470)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=device)
    w = torch.randn((n, k), generator=g, device=device) * 0.02
    b = torch.randn((n,), generator=g, device=device) * 0.1
    s_a = max(-float(x.min()) / 32768.0, float(x.max()) / 32767.0, 1e-12)
    act = torch.clamp(torch.round(x.double() / s_a + 32768), 0, 65535).to(torch.int32).to(torch.uint16)
    wb = w.double().reshape(n, k // 64, 64)
    gs = (wb.abs().amax(dim=2).clamp_min(1e-12) / 7.0).float()
    q = torch.clamp(torch.round(wb / gs.double()[:, :, None]), -7, 7).to(torch.int8).reshape(n, k)
    y = x[:256].double() @ w.double().t() + b.double()
    s_o = max(-float(y.min()) / 32768.0, float(y.max()) / 32767.0, 1e-12)
    nib = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).t().contiguous()
    return dict(act=act, w_packed=packed, q=q, scale=gs.contiguous(), bias=b.float().contiguous(), s_a=s_a,
                s_o=s_o, k=k, n=n)


def synth_gdn_A(n_chunks: int, C: int, dk: int, seed: int, device) -> torch.Tensor:
    """A = -strict_tril(beta_i (k_i.k_j) exp(g_i - g_j)), k L2-normalised, beta = sigmoid(N(0,1)),
    g = cumsum(logsigmoid(0.5 N(0,1) - 2)) per chunk; bf16 (BASELINE.json GDN config)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = torch.empty((n_chunks, C, C), dtype=torch.bfloat16, device=device)
    tril = torch.tril(torch.ones(C, C, dtype=torch.bool, device=device), -1)
    for s in range(0, n_chunks, 256):
        e = min(n_chunks, s + 256)
        kk = torch.randn((e - s, C, dk), generator=g, device=device)
        kk = kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6)
        beta = torch.sigmoid(torch.randn((e - s, C), generator=g, device=device))
        gg = torch.cumsum(torch.nn.functional.logsigmoid(0.5 * torch.randn((e - s, C), generator=g, device=device)
                                                         - 2.0), dim=-1)
        diff = gg[:, :, None] - gg[:, None, :]
        A = -(beta[:, :, None] * (kk @ kk.transpose(1, 2)) * torch.exp(torch.where(tril, diff, -torch.inf)))
        out[s:e] = torch.where(tril, A, 0.0).to(torch.bfloat16)
    return out


# ----------------------------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock, max clock and clock-event reasons through NVML (read-only) every ~2 ms in a
    background thread; summary() reports the samples taken inside the marked timed window."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples = []          # (t, sm_mhz, max_mhz, reason_bits)
        self.window = None
        self.err = None

    def _handle(self, nv):
        try:
            props = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def _run(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.bits = {name: getattr(nv, attr) for name, attr in self.REASONS}
            while not self._stop.is_set():
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((time.perf_counter(), sm, rs))
                self._stop.wait(0.002)
        except Exception as e:  # NVML missing or not permitted: report it
            self.err = repr(e)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        time.sleep(0.01)
        return self

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=5)

    def summary(self) -> dict:
        if self.err or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"nvml unavailable: {self.err}"]}
        sel = self.samples
        if self.window:
            inside = [x for x in self.samples if self.window[0] <= x[0] <= self.window[1]]
            sel = inside or sel
        reasons = sorted({n for _, _, rs in sel for n, b in self.bits.items() if rs & b})
        return {"sm_mhz": statistics.median(x[1] for x in sel), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sel), "source": "NVML, 2 ms, timed window"}


# ----------------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------------
def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class L2Flush:
    """Evicts L2 between timed steps: writes a 256 MB buffer (the flush proper), then reads a second
    256 MB buffer so that the dirty lines of the write are written back here, outside the timed
    window, and the timed kernel starts from a cold, clean L2 (126 MB)."""

    def __init__(self, device):
        self.w = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.sink = torch.zeros((), dtype=torch.float32, device=device)

    def __call__(self):
        self.w.add_(1)
        torch.amax(self.r, dim=0, out=self.sink)


def timed_steps(fn, steps: int, warmup: int, flush, world: int, stream, clk=None) -> list[float]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t_host0 = time.perf_counter()
    times = []
    for _ in range(steps):
        flush()                            # evict L2 outside the timed window
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    torch.cuda.synchronize()
    if clk is not None:
        clk.mark(t_host0, time.perf_counter())
    barrier(world)
    return times


# ----------------------------------------------------------------------------------------------
# CPU baseline: the reference's float64 oracle path (quantize_case core), on a row sample
# ----------------------------------------------------------------------------------------------
def cpu_gemm_baseline(d: dict, budget_s: float = 12.0) -> dict:
    from oracle import mm_oracle as O   # the checker; timed here as the reference CPU implementation
    try:
        from threadpoolctl import threadpool_info
        threads = max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"),
                      default=os.cpu_count())
    except Exception:
        threads = os.cpu_count()
    k, n = d["k"], d["n"]
    q = d["q"].cpu().numpy()
    f = d["factor"].cpu().numpy()
    scale = d["scale"].cpu().numpy()
    expanded = (q.astype(np.int16).reshape(n, k // d["block"], d["block"]) *
                f.astype(np.int16)[:, :, None]).reshape(n, k)
    w_deq = (expanded.astype(np.float32) * scale[:, None]).astype(np.float64)   # prepared once
    bias_deq = d["bias_q"].cpu().numpy().astype(np.float64) * (d["s_a"] * scale.astype(np.float64))
    act = d["act"].cpu().numpy()
    rows, elapsed = 8, 0.0
    while True:
        xs = act[:rows]
        t0 = time.perf_counter()
        x_deq = (xs.astype(np.float64) - 32768) * d["s_a"]
        y = x_deq @ w_deq.T + bias_deq
        O.quantize_affine(y, d["s_o"], -32768, 65535, np.uint16)
        elapsed = time.perf_counter() - t0
        if elapsed * 2 > budget_s or rows * 2 > act.shape[0]:
            break
        rows *= 2
    tops = 2.0 * rows * n * k / elapsed / 1e12
    return {"value": tops, "unit": "TFLOP/s", "cores": int(threads), "kind": "port",
            "sample": f"{rows} of {act.shape[0]} rows, full K={k}, N={n}: float64 x_deq @ w_deq.T + bias, "
                      f"requant (generate_qnn_matmul_python_cases.py:472-481 restated); {elapsed:.2f} s",
            "seconds": elapsed}


def cpu_per_group_baseline(d: dict, budget_s: float = 8.0) -> dict:
    """The reference's float64 path for the per-group schema on a row sample:
    y = x_deq @ w_deq.T + bias with w_deq = float32(q * s[n, k/64]) (generate_qnn_matmul_python_cases.py
    :392-423, 460-481), then the affine requant."""
    from oracle import mm_oracle as O   # the checker; timed here as the reference CPU implementation
    try:
        from threadpoolctl import threadpool_info
        threads = max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"),
                      default=os.cpu_count())
    except Exception:
        threads = os.cpu_count()
    k, n = d["k"], d["n"]
    q = d["q"].cpu().numpy()
    scale = d["scale"].cpu().numpy()
    w_deq = (q.astype(np.float32) * np.repeat(scale, 64, axis=1)).astype(np.float64)   # prepared once
    bias = d["bias"].cpu().numpy().astype(np.float64)
    act = d["act"].cpu().numpy()
    rows, elapsed = 8, 0.0
    while True:
        xs = act[:rows]
        t0 = time.perf_counter()
        x_deq = (xs.astype(np.float64) - 32768) * d["s_a"]
        y = x_deq @ w_deq.T + bias
        O.quantize_affine(y, d["s_o"], -32768, 65535, np.uint16)
        elapsed = time.perf_counter() - t0
        if elapsed * 2 > budget_s or rows * 2 > act.shape[0]:
            break
        rows *= 2
    return {"value": 2.0 * rows * n * k / elapsed / 1e12, "unit": "TFLOP/s", "cores": int(threads), "kind": "port",
            "sample": f"{rows} of {act.shape[0]} rows, full K={k}, N={n}: float64 x_deq @ w_deq.T + bias, "
                      f"requant (generate_qnn_matmul_python_cases.py:460-481 restated); {elapsed:.2f} s",
            "seconds": elapsed}


def cpu_gdn_baseline(A: torch.Tensor, budget_s: float = 10.0) -> dict:
    from oracle import gdn_oracle as G
    import ctypes
    lib_path = ROOT / "oracle" / "libgdn_block_ref.so"
    a = A.float().cpu().numpy()
    C = a.shape[-1]
    threads = os.cpu_count()
    n, el = 4, 0.0
    while True:
        sub = a[:n]
        sA = float(np.abs(sub).max() / 32767.0)
        Aq = np.clip(np.rint(sub / sA), -32767, 32767).astype(np.int16)
        T = np.zeros(sub.shape, np.float64)
        sAv = np.full(n, sA, np.float32)
        t0 = time.perf_counter()
        if lib_path.exists():
            lib = ctypes.CDLL(str(lib_path))
            lib.gdn_block_ref_solve(Aq.ctypes.data_as(ctypes.c_void_p), sAv.ctypes.data_as(ctypes.c_void_p),
                                    ctypes.c_float(2.0 / 32767.0), n, C, T.ctypes.data_as(ctypes.c_void_p),
                                    threads)
            kind = "port"
        else:
            G.inverse_fp64(sub)
            kind = "port"
        el = time.perf_counter() - t0
        if el * 2 > budget_s or n * 2 > a.shape[0]:
            break
        n *= 2
    return {"value": n / el, "unit": "chunks/s", "cores": threads, "kind": kind,
            "sample": f"{n} chunks of C={C}: BL=16 int16-code forward substitution + fp64 block merge "
                      f"(gdn_solve_ref.c restated, OpenMP over chunks); {el:.2f} s"}


# ----------------------------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------------------------
def run_gemm(args, world, rank, local, stream) -> dict:
    from qcom_htp_b200 import QuantMatMul
    dev = torch.device("cuda", local)
    m, k, n, blk = args.m, args.k, args.n, 64
    d = synth_w4a16_lpbq(m, k, n, blk, seed=1234 + rank, device=dev)
    op = QuantMatMul("w4a16", d["w_packed"], d["scale"], d["bias_q"], act_scale=d["s_a"], out_scale=d["s_o"],
                     schema="lpbq", lpbq_block_scale=d["factor"], lpbq_block=blk)
    act, out = d["act"], torch.empty((m, n), dtype=torch.uint16, device=dev)
    flush = L2Flush(dev)
    fn = lambda: op(act, out)
    with ClockSampler(local) as clk:
        times = timed_steps(fn, args.steps, args.warmup, flush, world, stream, clk)
    op.check_device(m)
    t_step = max_over_ranks(statistics.mean(times), world)
    ops = 2.0 * m * n * k
    value = ops * world / t_step / 1e12
    # end to end through the public API with host buffers (qhtp_matmul_run_host): pinned H2D of the
    # activation, GEMM, D2H of the output, every step, in row chunks whose copies overlap the GEMMs
    act_h = act.cpu().pin_memory()
    out_h = torch.empty((m, n), dtype=torch.uint16).pin_memory()

    def e2e():
        op.run_host(act_h, out_h, stream=stream)

    t_e2e = max_over_ranks(statistics.mean(timed_steps(e2e, max(3, args.steps // 2), 2, flush, world, stream)),
                           world)
    pk = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]      # dense int8 rate is 2x dense bf16 on B200
    achieved = ops / statistics.mean(times) / 1e12
    executed = achieved * 4                   # 2 activation byte planes x (q, e') weight planes
    res = {
        "metric": "w4a16_lpbq_gemm_tops", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u16xint4->u16 (int8 tensor ops, int64 combine)",
        "data": "synthetic (BASELINE.json distributions, generated on device)",
        "config": {"workload": "W4A16 LPBQ GEMM (BASELINE configs[2]/[4] shape)", "m": m, "k": k,
                   "n_per_gpu": n, "lpbq_block": blk, "parallelism": f"N-shard x{world}, no data-path collective",
                   "l2": "flushed between steps: 256 MB write, then 256 MB read of another buffer (cold, clean L2)", "bit_exact": True},
        "e2e": {"value": ops * world / t_e2e / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": m * k * 2,
                "d2h_bytes_per_step": m * n * 2},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                     "frac": achieved / int8_peak, "op_kind": "int8 MAC x2, logical",
                     "traffic": NCU_TRAFFIC_BYTES.get(("qgemm", m, k, n)),
                     "executed_tflops": executed, "frac_executed": executed / int8_peak,
                     "peak_src": f"2 x bf16_tflops ({pk['src']}, burst)",
                     "kernel": "split_u16_planes + qgemm_kernel<2,F32> (one qhtp_matmul_run)"},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if args.allgather and world > 1:
        import torch.distributed as dist
        gathered = torch.empty((world, m, n), dtype=torch.uint16, device=dev)
        # moved as bytes: NCCL has no 16-bit integer type, and a gather does no arithmetic
        ag = lambda: dist.all_gather_into_tensor(gathered.view(torch.uint8), out.view(torch.uint8))
        t_ag = max_over_ranks(statistics.mean(timed_steps(ag, max(3, args.steps // 2), 2, flush, world, stream)),
                              world)
        res["allgather"] = {"ms": t_ag * 1e3, "bytes": world * m * n * 2,
                            "tops_incl_allgather": ops * world / (t_step + t_ag) / 1e12}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_gemm_baseline(d)
    if not args.no_gdn:
        res["secondary"] = run_gdn(args, world, rank, local, stream, secondary=True)
    if not args.no_decode:
        res["decode"] = {"workload": "W4A16 LPBQ decode/prefill rows (BASELINE configs[2])",
                         "peak_gbs": peaks()["hbm_gbs"], "rows": run_decode(args, world, rank, local, stream)}
    if not args.no_per_group:
        res["per_group"] = run_per_group(args, world, rank, local, stream)
    return res


def run_per_group(args, world, rank, local, stream) -> dict:
    """The per-group W4 schema (float32 scale per 64 weights of K) at the headline GEMM shape: the
    same timing rules and int8 roofline denominator as the LPBQ line."""
    from qcom_htp_b200 import QuantMatMul
    dev = torch.device("cuda", local)
    m, k, n = args.m, args.k, args.n
    d = synth_w4a16_per_group(m, k, n, seed=777 + rank, device=dev)
    op = QuantMatMul("w4a16", d["w_packed"], d["scale"], None, schema="per_group", bias_float=d["bias"],
                     act_scale=d["s_a"], out_scale=d["s_o"])
    act, out = d["act"], torch.empty((m, n), dtype=torch.uint16, device=dev)
    flush = L2Flush(dev)
    times = timed_steps(lambda: op(act, out), max(5, args.steps // 2), args.warmup, flush, world, stream)
    op.check_device(m)
    t = max_over_ranks(statistics.mean(times), world)
    ops = 2.0 * m * n * k
    pk = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]
    achieved = ops / statistics.mean(times) / 1e12
    res = {"metric": "w4a16_per_group_gemm_tops", "value": ops * world / t / 1e12, "unit": "TFLOP/s",
            "ms_per_step": t * 1e3, "m": m, "k": k, "n_per_gpu": n, "group": 64,
            "kernel": "split_u16_planes + qgemm_group_kernel<2> (channel-major, float64 group accumulation)",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                         "frac": achieved / int8_peak, "executed_tflops": achieved * 4,
                         "frac_executed": achieved * 4 / int8_peak,
                         "note": "per 64-K group the accumulators are drained from TMEM and folded into float64"},
            "gpu_launches": 2 * max(5, args.steps // 2)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_per_group_baseline(d)
    return res


def run_decode(args, world, rank, local, stream, shapes=None) -> list:
    """BASELINE decode/prefill rows of the W4A16 LPBQ GEMM (M in {1, 16, 128}, K = 4096,
    N in {4096, 14336}): HBM-bound.  Reports GB/s on the algorithmic bytes (int4 weights, block
    factors, scales, bias, u16 activation and output) and on the bytes the kernel reads (the
    prepared byte planes: q and the float32-dequant residual e', 2 bytes per weight)."""
    from qcom_htp_b200 import QuantMatMul
    dev = torch.device("cuda", local)
    pk = peaks()
    flush = L2Flush(dev)
    rows = []
    k, blk = 4096, 64
    shapes = shapes or [(m, n) for n in (4096, 14336) for m in (1, 16, 128)]
    for m, n in shapes:
        if True:
            d = synth_w4a16_lpbq(m, k, n, blk, seed=4321 + m + n, device=dev)
            op = QuantMatMul("w4a16", d["w_packed"], d["scale"], d["bias_q"], act_scale=d["s_a"],
                             out_scale=d["s_o"], schema="lpbq", lpbq_block_scale=d["factor"], lpbq_block=blk)
            act, out = d["act"], torch.empty((m, n), dtype=torch.uint16, device=dev)
            times = timed_steps(lambda: op(act, out), max(5, args.steps // 2), args.warmup, flush, world, stream)
            op.check_device(m)
            t = max_over_ranks(statistics.mean(times), world)   # the event clock ticks in ~1 us steps
            alg = m * k * 2 + n * k // 2 + n * (k // blk) + n * 8 + m * n * 2
            read = int(op.plan.plane_bytes) + n * 32 + m * k * 2 + m * n * 2
            # the library's dispatch: the channel-major decode kernel up to 64 rows, and up to 128 rows
            # when the channel tiles leave room for a K split; else the row-tiled GEMM
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            row_tiled = m > 64 and 2 * ((n + 127) // 128) > sms
            rows.append({"m": m, "k": k, "n": n, "us": round(t * 1e6, 2),
                         "kernel": "split_u16_planes + " + ("qgemm_kernel (row tiles)" if row_tiled else
                                                            "qdecode_kernel (channel-major, cluster split-K)"),
                         "alg_bytes": alg, "alg_gbs": round(alg / t / 1e9, 1),
                         "alg_frac": round(alg / t / 1e9 / pk["hbm_gbs"], 3),
                         "read_bytes": read, "read_gbs": round(read / t / 1e9, 1),
                         "read_frac": round(read / t / 1e9 / pk["hbm_gbs"], 3)})
            del op, d, act, out
    return rows


def run_gdn(args, world, rank, local, stream, secondary=False) -> dict:
    from qcom_htp_b200 import gdn_inverse
    dev = torch.device("cuda", local)
    C = 256
    n_chunks = args.gdn_chunks
    A = synth_gdn_A(n_chunks, C, 128, seed=99 + rank, device=dev)
    T = torch.empty((n_chunks, C, C), dtype=torch.float32, device=dev)
    flush = L2Flush(dev)
    fn = lambda: gdn_inverse(A, T)
    steps = args.steps
    with ClockSampler(local) as clk:
        times = timed_steps(fn, steps, args.warmup, flush, world, stream, clk)
    t = max_over_ranks(statistics.mean(times), world)
    pk = peaks()
    bytes_alg = n_chunks * (C * C * 2 + C * C * 4)       # read A (bf16), write T (fp32)
    achieved = bytes_alg / statistics.mean(times) / 1e9
    res = {"metric": "gdn_inverse_chunks_per_s", "value": n_chunks * world / t, "unit": "chunks/s",
           "ms_per_step": t * 1e3, "config": {"workload": "GDN C=256 inverse", "chunks_per_gpu": n_chunks,
                                             "note": "batch 8 x 32 heads x 16 chunks per GPU"},
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / pk["hbm_gbs"], "traffic": NCU_TRAFFIC_BYTES.get(("gdn", n_chunks)),
                        "peak_src": f"hbm_gbs ({pk['src']})"},
           "gpu_launches": steps, "clocks": clk.summary()}
    # the reference's production carrier (GdnSolve / gdnbm_solve): u16 codes in and out, scales of
    # gdn_solve_oc_check.py:20-23, same chunks
    from qcom_htp_b200 import gdn_solve_u16
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    Ac = torch.clamp(torch.round(A.float() / sA) + zp, 0, 65535).to(torch.int32).to(torch.uint16)
    Tc = torch.empty_like(Ac)
    fn16 = lambda: gdn_solve_u16(Ac, zpA=zp, sA=sA, zpT=zp, sT=sT, out=Tc)
    t16 = max_over_ranks(statistics.mean(timed_steps(fn16, steps, args.warmup, flush, world, stream)), world)
    b16 = n_chunks * (C * C * 2 + C * C * 2)
    res["u16_carrier"] = {"metric": "gdn_solve_u16_chunks_per_s", "value": n_chunks * world / t16,
                          "ms_per_step": t16 * 1e3, "hbm_gbs": b16 / t16 / 1e9, "hbm_frac": b16 / t16 / 1e9 / pk["hbm_gbs"],
                          "note": "u16 codes A -> u16 codes T (zp 32768), algorithmic bytes 2C^2 + 2C^2 per chunk"}
    del Ac, Tc
    # the step on the input side fused in: A built on the SM from raw keys, beta and per-token log
    # gates (gdn_chunk Stage A, scripts/gdn_ref_kernel.py:66-82), then inverted; same chunk count
    from qcom_htp_b200 import gdn_chunk_inverse
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    kk = torch.randn((n_chunks, C, 128), generator=gen, device=dev).to(torch.bfloat16)
    bb = torch.sigmoid(torch.randn((n_chunks, C), generator=gen, device=dev))
    gg = torch.nn.functional.logsigmoid(0.5 * torch.randn((n_chunks, C), generator=gen, device=dev) - 2.0)
    fnf = lambda: gdn_chunk_inverse(kk, bb, gg, T)
    tf = max_over_ranks(statistics.mean(timed_steps(fnf, steps, args.warmup, flush, world, stream)), world)
    bf = n_chunks * (C * 128 * 2 + C * 4 * 2 + C * C * 4)
    res["fused_A"] = {"metric": "gdn_chunk_inverse_chunks_per_s", "value": n_chunks * world / tf,
                      "ms_per_step": tf * 1e3, "hbm_gbs": bf / tf / 1e9, "hbm_frac": bf / tf / 1e9 / pk["hbm_gbs"],
                      "traffic": NCU_TRAFFIC_BYTES.get(("gdn_fused", n_chunks)),
                      "kernel": "gdn256f_kernel (Gram MMAs + A epilogue + the C=256 inverse)",
                      "note": "k bf16 [C,128], beta and log gates f32 [C] -> T f32: algorithmic bytes 256C + 8C + 4C^2 "
                              "per chunk; A (bf16 [C,C]) never written or read"}
    del kk, bb, gg
    if args.allgather and world > 1:
        import torch.distributed as dist
        # every rank ends with all ranks' T ([world * chunks, C, C]); the only collective of the path
        gathered = torch.empty((world,) + tuple(T.shape), dtype=T.dtype, device=dev)
        ag = lambda: dist.all_gather_into_tensor(gathered, T)
        t_ag = max_over_ranks(statistics.mean(timed_steps(ag, max(3, steps // 2), 2, flush, world, stream)), world)
        res["allgather"] = {"ms": t_ag * 1e3, "bytes": world * T.numel() * T.element_size(),
                            "chunks_per_s_incl_allgather": n_chunks * world / (t + t_ag)}
        del gathered
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_gdn_baseline(A)
    if not secondary:
        res.update({"n_gpus": world, "steps": steps, "warmup": args.warmup, "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "dtype": "bf16 in / fp32 out (tf: bf16 MMA, fp32 acc)",
                    "data": "synthetic (BASELINE.json GDN distribution, generated on device)",
                    "e2e": None})
    return res


# ----------------------------------------------------------------------------------------------
# reference arm: the reference's own CPU implementation of the path, on the host cores
# ----------------------------------------------------------------------------------------------
def run_reference(args, world, rank) -> None:
    if rank != 0:
        return
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    m, k, n = args.m, args.k, args.n
    d = synth_w4a16_lpbq(m, k, n, 64, seed=1234, device=dev)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_gemm_baseline(d, budget_s=max(2.0, 60.0 / max(1, args.steps + args.warmup)))
        if i >= args.warmup:
            vals.append(r)
    v = statistics.mean(x["value"] for x in vals)
    out = {"impl": "reference", "metric": "w4a16_lpbq_gemm_tops", "value": v, "unit": "TFLOP/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
           "config": {"workload": "W4A16 LPBQ GEMM (BASELINE configs[2]/[4] shape)", "m": m, "k": k, "n_per_gpu": n,
                      "lpbq_block": 64},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": vals[-1]["cores"], "kind": "port",
                            "sample": vals[-1]["sample"]},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference has no GPU path; its CPU oracle (float64 numpy) is timed on the host cores"}
    print(json.dumps(out))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "gdn", "decode", "per_group"], default="gemm")
    # --gemm-m / --gemm-n: the same options under names that torchrun's own parser does not take for
    # abbreviations of its --master-*/--nnodes/--nproc-per-node (a bare --m or --n under torchrun errors)
    ap.add_argument("--m", "--gemm-m", dest="m", type=int, default=4096)
    ap.add_argument("--k", "--gemm-k", dest="k", type=int, default=4096)
    ap.add_argument("--n", "--gemm-n", dest="n", type=int, default=14336)
    ap.add_argument("--gdn-chunks", type=int, default=4096)
    ap.add_argument("--allgather", action="store_true")
    ap.add_argument("--no-gdn", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-per-group", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        # rank 0 alone times the CPU implementation; other ranks exit without work
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return 0
    world, rank, local = dist_init()
    stream = torch.cuda.current_stream()
    if args.workload == "gemm":
        res = run_gemm(args, world, rank, local, stream)
    elif args.workload == "gdn":
        res = run_gdn(args, world, rank, local, stream)
    elif args.workload == "per_group":
        # the per-group W4A16 GEMM alone at --m / --k / --n (the command its ncu summary was taken with)
        row = run_per_group(args, world, rank, local, stream)
        res = {"metric": row["metric"], "value": row["value"], "unit": row["unit"], "n_gpus": world,
               "steps": max(5, args.steps // 2), "warmup": args.warmup, "ms_per_step": row["ms_per_step"],
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "u16xint4->u16 (int8 tensor ops, float64 group fold)",
               "data": "synthetic (BASELINE.json distributions, generated on device)",
               "config": {"workload": f"W4A16 per-group GEMM {args.m}x{args.k}x{args.n}", "m": args.m, "k": args.k,
                          "n": args.n, "group": 64, "l2": "flushed between steps (256 MB write + 256 MB read)"},
               "roofline": row["roofline"], "gpu_launches": row["gpu_launches"], "e2e": None}
        if "cpu_baseline" in row:
            res["cpu_baseline"] = row["cpu_baseline"]
    else:
        # one decode-shaped GEMM (the --m / --n shape, K = 4096), HBM roofline
        row = run_decode(args, world, rank, local, stream, shapes=[(args.m, args.n)])[0]
        pk = peaks()
        res = {"metric": "w4a16_lpbq_decode_gbs", "value": row["alg_gbs"] * world, "unit": "GB/s",
               "n_gpus": world, "steps": max(5, args.steps // 2), "warmup": args.warmup,
               "ms_per_step": row["us"] * 1e-3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "u16xint4->u16 (int8 tensor ops, int64 combine)", "data": "synthetic (BASELINE.json distributions)",
               "config": {"workload": f"W4A16 LPBQ decode M={args.m} K=4096 N={args.n}", "m": args.m, "k": 4096,
                          "n": args.n, "l2": "flushed between steps (256 MB write + 256 MB read)"},
               "roofline": {"bound": "hbm", "achieved": row["alg_gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": row["alg_frac"], "traffic": NCU_TRAFFIC_BYTES.get(("qdecode", args.m, 4096, args.n)),
                            "read_gbs": row["read_gbs"],
                            "read_frac": row["read_frac"], "kernel": row["kernel"]},
               "gpu_launches": 2 * max(5, args.steps // 2), "e2e": None}
    if rank == 0:
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
