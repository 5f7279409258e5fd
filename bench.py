#!/usr/bin/env python3
"""Benchmark of the quantized-MatMul hot path (and the GDN chunk inverse) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemm|gdn|decode|per_group|family|peak]

Headline workload (BASELINE.json configs[2]/[4]): W4A16 LPBQ GEMM, M=4096, K=4096, N=14336, LPBQ
block 64, u16 activations from N(0,1), int4 weights from N(0,0.02), int32 bias, u16 output.  A "step"
is one quantized GEMM over one batch of synthetic input.  Metric: logical TOPS = 2*M*N*K / step time.

Multi-GPU (torchrun, one process per GPU; BASELINE configs[4], the sharded sweep): ONE global weight
set of N = 14336 output channels is cut into per-rank channel slabs by qcom_htp_b200.shard
(shard_matmul_weights), the activation is replicated, and every rank runs its slab -- the total work
is fixed ("strong" scaling) and `value` is the whole problem's logical TOPS over the max-over-ranks
step time of the sharded GEMM (the outputs stay in each rank's HBM as [M, N/P] slabs).  The NCCL
all-gather of the outputs is timed beside it (`allgather`: one gather after the GEMM, and the GEMM in
row chunks with each chunk's gather on a second stream overlapping the next chunk's GEMM).  The W4A8
per-channel GEMM of configs[4] is a second row cut the same way, and GDN's 64 x 32 x 64 = 131072
chunks are split over batch x heads (`secondary`).

Timing: CUDA events on the launching stream, per step, L2 flushed between steps (a 256 MB write, then
a 256 MB read of another buffer so the write-back happens before the timed window), max over ranks.
Claims in the line are computed: `bit_exact` compares a row x channel sample of the timed output with
the exact oracle, `oc` is the GDN gate metric on a chunk sample of the timed output.

At one GPU the line also carries the GDN configs[3] workload (4096 chunks), one row per MatMul family
at the headline shape (W16A16 also at the configs[2] decode/prefill shapes), the W4A16 LPBQ
decode/prefill rows, the per-group W4 schema, and the measured tcgen05 kind::i8 tensor-pipe rate that
the GEMM rooflines are quoted against.
"""
from __future__ import annotations

import os
import sys

# The reference arm times numpy's float64 BLAS on the host cores.  torchrun sets OMP_NUM_THREADS=1 for
# its workers; the CPU arm must use every core, so the BLAS thread count is set before numpy loads.
if "--impl" in sys.argv and "reference" in sys.argv:
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = str(os.cpu_count() or 1)

import argparse
import json
import statistics
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from one ncu capture
# of this script's own workload (the command is in the profiles/ summary of each kernel); the GDN
# figures are 1024-chunk captures scaled by the chunk count (traffic grows with the chunks)
NCU_TRAFFIC_BYTES = {
    ("qgemm", 4096, 4096, 14336): 153_400_832 + 100_256_768,          # full-size capture (LO3 variant)
    ("gdn_per_chunk",): (100_822_016 + 208_797_696) / 1024,            # 1024-chunk capture
    ("gdn_fused_per_chunk",): (69_339_904 + 208_701_952) / 1024,       # 1024-chunk capture
    ("qdecode", 16, 4096, 14336): 118_091_264 + 4_662_784,             # full-size capture
    ("qdecode", 1, 4096, 4096): 33_753_344 + 0,                        # full-size capture
}

FAMILY_BITS = {"u8i8": (8, 8, 8), "w4a8": (8, 4, 8), "w8a16": (16, 8, 16), "w4a16": (16, 4, 16),
               "w16a16": (16, 16, 16)}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def blas_threads() -> int:
    """Pin the host BLAS to every core (torchrun workers start with one) and report the count."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n, user_api="blas")
        return max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"), default=n)
    except Exception:
        return n


# ----------------------------------------------------------------------------------------------
# synthetic inputs (generated on the device; BASELINE.json distributions, the reference generator's
# quantization rules: generate_qnn_matmul_python_cases.py:174-218, 288-423, 426-481)
# ----------------------------------------------------------------------------------------------
def _affine_fixed(vmin: float, vmax: float, qmax: int, zp: int) -> float:
    s = 1.0e-12
    if vmin < 0 and zp > 0:
        s = max(s, -vmin / zp)
    if vmax > 0 and qmax > zp:
        s = max(s, vmax / (qmax - zp))
    return s


def _affine_free(vmin: float, vmax: float, qmax: int) -> tuple[float, int]:
    lo, hi = min(vmin, 0.0), max(vmax, 0.0)
    s = max((hi - lo) / qmax, 1.0e-12)
    return s, int(min(max(-round(lo / s), 0), qmax))


def synth_gemm(family: str, schema: str, m: int, k: int, n: int, seed: int, device, block: int = 64,
               free_offsets: bool = False) -> dict:
    """Activations X ~ N(0,1), weights W ~ N(0, 0.02) (int4) or N(0, 0.05) (int8 / int16), bias ~ N(0, 0.1).

    Activations: asymmetric with the family's fixed zero point (A8 128, A16 32768), or -- free_offsets,
    BASELINE configs[0] -- scale (max-min)/255 and zero point -round(min/scale), output likewise.
    Weights: symmetric per output channel; LPBQ: per (channel, K block) scales factorised as a
    per-channel base x integer factor in [1, 16]; free_offsets: one per-tensor int8 scale.  Output
    scale from the float output of the first 256 rows."""
    a_bits, w_bits, o_bits = FAMILY_BITS[family]
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=device)
    sigma = 0.02 if w_bits == 4 else 0.05
    w = torch.randn((n, k), generator=g, device=device) * sigma
    b = torch.randn((n,), generator=g, device=device) * 0.1
    a_qmax, o_qmax = (1 << a_bits) - 1, (1 << o_bits) - 1
    if free_offsets:
        s_a, a_zp = _affine_free(float(x.min()), float(x.max()), a_qmax)
    else:
        a_zp = 1 << (a_bits - 1)
        s_a = _affine_fixed(float(x.min()), float(x.max()), a_qmax, a_zp)
    act = torch.clamp(torch.round(x.double() / s_a + a_zp), 0, a_qmax).to(torch.int32)
    act = act.to(torch.uint16 if a_bits == 16 else torch.uint8)
    qmax = (1 << (w_bits - 1)) - 1
    wd = w.double()
    factor = None
    if schema == "lpbq":
        wb = wd.reshape(n, k // block, block)
        gs = (wb.abs().amax(dim=2).clamp_min(1e-12) / qmax).float().double()
        base = torch.maximum(gs.amin(dim=1).clamp_min(1e-12), gs.amax(dim=1).clamp_min(1e-12) / 16.0)
        f = torch.clamp(torch.ceil(gs / base[:, None] - 1e-9), 1, 16)
        q = torch.clamp(torch.round(wb / (base[:, None, None] * f[:, :, None])), -qmax, qmax).reshape(n, k)
        scale = base.float()
        factor = f.to(torch.uint8).contiguous()
    elif free_offsets:
        s_t = torch.tensor(max(float(w.abs().max()), 1e-12) / qmax, dtype=torch.float32, device=device)
        q = torch.clamp(torch.round(wd / s_t.double()), -qmax, qmax)
        scale = s_t.expand(n).contiguous()
    else:
        s = wd.abs().amax(dim=1).clamp_min(1e-12) / qmax
        q = torch.clamp(torch.round(wd / s[:, None]), -qmax, qmax)
        scale = s.float()
    q = q.to(torch.int16 if w_bits == 16 else torch.int8).contiguous()
    scale = scale.contiguous()
    bias_q = torch.clamp(torch.round(b.double() / (s_a * scale.double())), -2 ** 31, 2 ** 31 - 1).to(torch.int32)
    y = x[:256].double() @ wd.t() + b.double()
    if free_offsets:
        s_o, o_zp = _affine_free(float(y.min()), float(y.max()), o_qmax)
    else:
        o_zp = 32768 if o_bits == 16 else 0
        s_o = _affine_fixed(float(y.min()), float(y.max()), o_qmax, o_zp)
    if w_bits == 4:
        nib = (q.to(torch.int16) & 0xF).to(torch.uint8)
        carrier = (nib[:, 0::2] | (nib[:, 1::2] << 4)).t().contiguous()     # K-pair [K/2, N]
    else:
        carrier = q
    return dict(family=family, schema=schema, act=act, weight=carrier, q=q, factor=factor, scale=scale,
                bias_q=bias_q.contiguous(), s_a=s_a, s_o=s_o, a_zp=a_zp, o_zp=o_zp, m=m, k=k, n=n, block=block)


def shard_gemm(d: dict, world: int, rank: int) -> dict:
    """Rank's channel slab of a global weight set (qcom_htp_b200.shard.shard_matmul_weights)."""
    from qcom_htp_b200.shard import shard_matmul_weights
    w_bits = FAMILY_BITS[d["family"]][1]
    sh = shard_matmul_weights(d["weight"], d["scale"], d["bias_q"], weight_bits=w_bits, world=world, rank=rank,
                              lpbq_block_scale=d["factor"])
    out = dict(d)
    out.update(weight=sh.weight, scale=sh.weight_scale, bias_q=sh.bias_q, factor=sh.lpbq_block_scale,
               q=d["q"][sh.n0:sh.n1], n=sh.n1 - sh.n0, n0=sh.n0, n1=sh.n1, n_total=d["n"])
    return out


def make_op(d: dict):
    from qcom_htp_b200 import QuantMatMul
    kw = {}
    if d["schema"] == "lpbq":
        kw = dict(schema="lpbq", lpbq_block_scale=d["factor"], lpbq_block=d["block"])
    return QuantMatMul(d["family"], d["weight"], d["scale"], d["bias_q"], act_scale=d["s_a"], out_scale=d["s_o"],
                       act_offset=-d["a_zp"], out_offset=-d["o_zp"], **kw)


def synth_w4a16_per_group(m: int, k: int, n: int, seed: int, device) -> dict:
    """u16 activations and per-group int4 weights with the reference generator's rules: symmetric
    float32 scale per (channel, 64 weights of K), float32 bias kept unquantized
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
# the checker: exact oracle on a sample of the timed outputs (outside every timed region)
# ----------------------------------------------------------------------------------------------
ORACLE_FAMILY = {("u8i8", "per_channel"): "u8i8", ("w4a8", "per_channel"): "w4a8_per_channel",
                 ("w4a8", "lpbq"): "w4a8_lpbq", ("w8a16", "per_channel"): "w8a16",
                 ("w4a16", "per_channel"): "w4a16_per_channel", ("w4a16", "lpbq"): "w4a16_lpbq",
                 ("w16a16", "per_channel"): "w16a16"}


def sample_rows(m: int, count: int = 24) -> np.ndarray:
    """Rows spread over every 128-row tile region, first and last included."""
    return np.unique(np.r_[0, m - 1, np.linspace(0, m - 1, min(count, m)).astype(np.int64)])


def sample_channels(n: int) -> np.ndarray:
    """Four channels of every 128-channel tile (its edges and interior)."""
    cols = [t * 128 + c for t in range((n + 127) // 128) for c in (0, 37, 90, 127) if t * 128 + c < n]
    return np.unique(np.r_[cols, n - 1])


def check_gemm_sample(d: dict, out: torch.Tensor) -> dict:
    """Compare a row x channel sample of the timed output with oracle.mm_oracle.exact_output (the
    checker; every output channel is independent, so a channel subset is checked exactly)."""
    from oracle import mm_oracle as O
    fam = O.FAMILIES[ORACLE_FAMILY[(d["family"], d["schema"])]]
    if d["schema"] == "lpbq":
        fam = fam.with_block(d["block"])
    rows, cols = sample_rows(d["m"]), sample_channels(d["n"])
    r_t, c_t = torch.from_numpy(rows).to(out.device), torch.from_numpy(cols).to(out.device)
    q = d["q"].index_select(0, c_t).cpu().numpy()
    f = d["factor"].index_select(0, c_t).cpu().numpy() if d["factor"] is not None else None
    expanded = None
    if f is not None:
        expanded = (q.astype(np.int16).reshape(len(cols), -1, d["block"]) *
                    f.astype(np.int16)[:, :, None]).reshape(len(cols), -1)
    case = O.QuantCase(fam, d["act"].index_select(0, r_t).cpu().numpy(), q,
                       d["scale"].index_select(0, c_t).cpu().numpy(), d["bias_q"].index_select(0, c_t).cpu().numpy(),
                       d["s_a"], d["s_o"], f, expanded, act_zp_free=d["a_zp"], out_zp_free=d["o_zp"])
    want = O.exact_output(case, dequant="exact" if d["family"] == "w16a16" else "f32")
    got = out.index_select(0, r_t).index_select(1, c_t).cpu().numpy()
    bad = int((got != want).sum())
    return {"bit_exact": bad == 0, "mismatches": bad, "checked": int(want.size),
            "sample": f"{len(rows)} rows x {len(cols)} channels (4 per 128-channel tile) vs oracle exact_output"}


def gdn_oc_sample(T: torch.Tensor, A: torch.Tensor, count: int = 16) -> dict:
    """oc (gdn_solve_oc_check.py:31) of T on a chunk sample against the fp64 inverse of the same A."""
    from oracle import gdn_oracle as G
    idx = torch.from_numpy(np.unique(np.linspace(0, T.shape[0] - 1, count).astype(np.int64))).to(T.device)
    t = T.index_select(0, idx).double().cpu().numpy()
    ref = G.inverse_fp64(A.index_select(0, idx).double().cpu().numpy())
    return {"oc": G.oc(t, ref), "gate": G.OC_GATE, "chunks": int(idx.numel())}


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
        self.samples = []          # (t, sm_mhz, reason_bits)
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
# distributed plumbing and timing
# ----------------------------------------------------------------------------------------------
def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
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


def all_ranks_true(v: bool, world: int) -> bool:
    if world == 1:
        return bool(v)
    import torch.distributed as dist
    t = torch.tensor([0 if v else 1], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item()) == 0


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
# the measured tensor-pipe peak (tcgen05 kind::i8 and kind::f16 issue loops, qhtp_selftest_mma_rate)
# ----------------------------------------------------------------------------------------------
def measure_mma_peak(device, iters: int = 20000, reps: int = 5) -> dict:
    from qcom_htp_b200 import _lib as L
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    err = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream()
    res = {}
    for kind, name, kbytes in ((0, "i8_tops", 32), (1, "bf16_tflops", 16)):
        ts = []
        for r in range(reps + 1):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            L.check("qhtp_selftest_mma_rate", L.lib.qhtp_selftest_mma_rate(kind, iters, sms, err.data_ptr(),
                                                                            stream.cuda_stream))
            e1.record(stream)
            e1.synchronize()
            if r:                       # first launch is the warm-up
                ts.append(e0.elapsed_time(e1) * 1e-3)
        ops = sms * iters * 4 * 2.0 * 128 * 256 * kbytes
        res[name] = ops / min(ts) / 1e12
    if int(err.item()) != 0:
        raise RuntimeError(f"tensor-pipe probe recorded device error {int(err.item())}")
    res.update(sms=sms, iters=iters, note="best of 5 launches; one CTA per SM issuing M=128 N=256 MMAs "
                                          "back to back from shared memory (no memory traffic)")
    return res


def int8_peak(pk: dict, probe: dict | None) -> tuple[float, str]:
    if probe:
        return probe["i8_tops"], "measured: tcgen05.mma kind::i8 issue loop (qhtp_selftest_mma_rate), burst"
    return 2.0 * pk["bf16_tflops"], f"2 x bf16_tflops ({pk['src']}, burst)"


# ----------------------------------------------------------------------------------------------
# CPU baseline: the reference's float64 oracle path (quantize_case core), on a row sample
# ----------------------------------------------------------------------------------------------
def cpu_gemm_baseline(d: dict, budget_s: float = 12.0) -> dict:
    """The reference's float64 path (generate_qnn_matmul_python_cases.py:472-481):
    y = x_deq @ w_deq.T + bias_deq with w_deq = float32(q * s), then the affine requant; weights
    dequantized once (not timed), the GEMM + requant timed on a doubling row sample."""
    from oracle import mm_oracle as O   # the checker; timed here as the reference CPU implementation
    threads = blas_threads()
    k, n = d["k"], d["n"]
    q = d["q"].cpu().numpy()
    scale = d["scale"].cpu().numpy()
    if d["factor"] is not None:
        f = d["factor"].cpu().numpy()
        q = (q.astype(np.int16).reshape(n, k // d["block"], d["block"]) * f.astype(np.int16)[:, :, None]).reshape(n, k)
    w_deq = (q.astype(np.float32) * scale[:, None]).astype(np.float64)       # prepared once
    bias_deq = d["bias_q"].cpu().numpy().astype(np.float64) * (d["s_a"] * scale.astype(np.float64))
    act = d["act"].cpu().numpy()
    o_bits = FAMILY_BITS[d["family"]][2]
    o_dt = np.uint16 if o_bits == 16 else np.uint8
    rows, elapsed = 8, 0.0
    while True:
        xs = act[:rows]
        t0 = time.perf_counter()
        x_deq = (xs.astype(np.float64) - d["a_zp"]) * d["s_a"]
        y = x_deq @ w_deq.T + bias_deq
        O.quantize_affine(y, d["s_o"], -d["o_zp"], (1 << o_bits) - 1, o_dt)
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
    threads = blas_threads()
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
    """The reference's BL=16 GDN solve (gdn_solve_ref.c, restated in oracle/gdn_block_ref.c and
    checked bit for bit against the reference's own compiled solver), OpenMP over chunks."""
    from oracle import gdn_oracle as G
    import ctypes
    lib_path = ROOT / "oracle" / "libgdn_block_ref.so"
    threads = os.cpu_count() or 1
    C = A.shape[-1]
    n, el = 4, 0.0
    while True:
        sub = A[:n].float().cpu().numpy()
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
        else:
            G.block_model(Aq, sA, 2.0 / 32767.0)
        el = time.perf_counter() - t0
        if el * 2 > budget_s or n * 2 > A.shape[0]:
            break
        n *= 2
    return {"value": n / el, "unit": "chunks/s", "cores": threads, "kind": "port",
            "sample": f"{n} chunks of C={C}: BL=16 int16-code forward substitution + fp64 block merge "
                      f"(gdn_solve_ref.c restated, OpenMP over chunks); {el:.2f} s"}


# ----------------------------------------------------------------------------------------------
# GEMM rows
# ----------------------------------------------------------------------------------------------
def executed_multiplier(op, m: int) -> int:
    """Tensor-pipe work per logical op: activation byte planes x weight planes ([q | e'] in the
    float32-dequant mode, [hi | lo] for int16 weights; one plane in the exact mode).  Where the launch
    uses the lo-plane residual bound (QuantMatMul.lo_residual_launch) the lo activation plane
    multiplies the q rows only: 3."""
    planes_w = 2 if int(op.plan.mode) in (0, 2) else 1
    if int(op.plan.mode) == 0 and int(op.plan.a_planes) == 2 and op.lo_residual_launch(m):
        return 3
    return int(op.plan.a_planes) * planes_w


def gemm_alg_bytes(d: dict, n: int) -> int:
    a_bits, w_bits, o_bits = FAMILY_BITS[d["family"]]
    m, k = d["m"], d["k"]
    lp = n * (k // d["block"]) if d["schema"] == "lpbq" else 0
    return m * k * a_bits // 8 + n * k * w_bits // 8 + n * 8 + lp + m * n * o_bits // 8


def gemm_row(d: dict, args, world: int, rank: int, stream, flush, *, steps: int, probe: dict | None,
             clk_local: int | None = None, cpu: bool = False, cpu_budget: float = 12.0) -> tuple[dict, object]:
    """Time one (sharded) quantized GEMM: this rank's slab of d.  Returns the row and the op."""
    op = make_op(d)
    m, k, n_r = d["m"], d["k"], d["n"]
    n_total = d.get("n_total", n_r)
    act = d["act"]
    out = torch.empty((m, n_r), dtype=torch.uint16 if FAMILY_BITS[d["family"]][2] == 16 else torch.uint8,
                      device=act.device)
    fn = lambda: op(act, out)
    clk = None
    if clk_local is not None:
        with ClockSampler(clk_local) as clk:
            times = timed_steps(fn, steps, args.warmup, flush, world, stream, clk)
    else:
        times = timed_steps(fn, steps, args.warmup, flush, world, stream)
    op.check_device(m)
    t_local = statistics.mean(times)
    t_step = max_over_ranks(t_local, world)
    ops_total = 2.0 * m * n_total * k
    chk = check_gemm_sample(d, out)
    chk["bit_exact"] = all_ranks_true(chk["bit_exact"], world)
    pk = peaks()
    row = {"ms_per_step": t_step * 1e3, "tops": ops_total / t_step / 1e12, "check": chk}
    if m > 128:
        i8, i8_src = int8_peak(pk, probe)
        achieved = 2.0 * m * n_r * k / t_local / 1e12
        mult = executed_multiplier(op, m)
        row["roofline"] = {"bound": "tensor", "achieved": achieved, "peak": i8, "unit": "TFLOP/s",
                           "frac": achieved / i8, "op_kind": "int8 MAC x2, logical (2*M*N*K)",
                           "executed_tflops": achieved * mult, "frac_executed": achieved * mult / i8,
                           "executed_per_logical": mult, "peak_src": i8_src}
    else:
        alg = gemm_alg_bytes(d, n_r)
        read = int(op.plan.plane_bytes) + n_r * 32 + m * k * FAMILY_BITS[d["family"]][0] // 8
        row["roofline"] = {"bound": "hbm", "achieved": alg / t_local / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                           "frac": alg / t_local / 1e9 / pk["hbm_gbs"], "alg_bytes": alg,
                           "read_bytes": read, "read_frac": read / t_local / 1e9 / pk["hbm_gbs"],
                           "peak_src": f"hbm_gbs ({pk['src']})"}
    if clk is not None:
        row["clocks"] = clk.summary()
    if cpu and rank == 0 and world == 1 and not args.no_cpu_baseline:
        row["cpu_baseline"] = cpu_gemm_baseline(d, cpu_budget)
    row["_out"] = out
    return row, op


def gemm_allgather(op, d: dict, out: torch.Tensor, args, world: int, stream, flush, ops_total: float,
                   t_step: float, chunks: int = 4) -> dict:
    """The configs[4] output exchange: every rank ends with every rank's [M, N/P] slab.  (a) one NCCL
    all-gather after the GEMM; (b) the GEMM in `chunks` row chunks, chunk i's all-gather issued on a
    second stream as soon as chunk i is done, overlapping chunk i+1's GEMM.  The persistent GEMM holds
    every SM it is given, so in (b) it runs on all but `reserve` SMs (qhtp_matmul_run_ctas) and the
    NCCL kernel of the previous chunk's gather runs on the rest; measured for a few reserves.  NCCL
    moves local buffers only (bytes: NCCL has no 16-bit integer type)."""
    import torch.distributed as dist
    m = d["m"]
    act = d["act"]
    sms = torch.cuda.get_device_properties(out.device).multi_processor_count
    gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=out.device)
    ag = lambda: dist.all_gather_into_tensor(gathered.view(torch.uint8), out.view(torch.uint8))
    t_ag = max_over_ranks(statistics.mean(timed_steps(ag, max(3, args.steps // 2), 2, flush, world, stream)),
                          world)
    rows = (m + chunks - 1) // chunks
    bounds = [(r0, min(m, r0 + rows)) for r0 in range(0, m, rows)]
    parts = [torch.empty((world, r1 - r0, out.shape[1]), dtype=out.dtype, device=out.device) for r0, r1 in bounds]
    comm = torch.cuda.Stream(device=out.device)
    evs = [torch.cuda.Event() for _ in bounds]

    def overlapped(reserve: int):
        works = []
        for (r0, r1), part, ev in zip(bounds, parts, evs):
            op(act[r0:r1], out[r0:r1], max_ctas=sms - reserve)
            ev.record(stream)
            with torch.cuda.stream(comm):
                comm.wait_event(ev)
                works.append(dist.all_gather_into_tensor(part.view(torch.uint8), out[r0:r1].view(torch.uint8),
                                                         async_op=True))
        for w in works:
            w.wait()          # the launching stream waits for every gather

    sweep = {}
    for reserve in (8, 16, 32):
        t = max_over_ranks(statistics.mean(timed_steps(lambda: overlapped(reserve), max(3, args.steps // 2), 2,
                                                       flush, world, stream)), world)
        sweep[reserve] = t
    best = min(sweep, key=sweep.get)
    t_ov = sweep[best]
    op.check_device(rows)
    ok = all(torch.equal(parts[i][dist.get_rank()], out[r0:r1]) for i, (r0, r1) in enumerate(bounds))
    return {"bytes_received_per_rank": (world - 1) * out.numel() * out.element_size(),
            "serial": {"allgather_ms": t_ag * 1e3, "total_ms": (t_step + t_ag) * 1e3,
                       "tops_incl_allgather": ops_total / (t_step + t_ag) / 1e12},
            "overlapped": {"row_chunks": chunks, "reserved_sms": best, "total_ms": t_ov * 1e3,
                           "tops_incl_allgather": ops_total / t_ov / 1e12,
                           "vs_max_compute_gather": t_ov / max(t_step, t_ag), "own_slab_roundtrip_ok": ok,
                           "ms_by_reserved_sms": {str(k): v * 1e3 for k, v in sweep.items()}}}


def run_gemm(args, world, rank, local, stream) -> dict:
    dev = torch.device("cuda", local)
    flush = L2Flush(dev)
    probe = measure_mma_peak(dev) if not args.no_probe else None
    args._probe = probe
    m, k, n = args.m, args.k, args.n
    full = synth_gemm("w4a16", "lpbq", m, k, n, seed=1234, device=dev)        # one global weight set
    d = shard_gemm(full, world, rank)
    del full
    row, op = gemm_row(d, args, world, rank, stream, flush, steps=args.steps, probe=probe, clk_local=local,
                       cpu=True)
    out = row.pop("_out")
    t_step = row["ms_per_step"] * 1e-3
    ops_total = 2.0 * m * n * k
    # end to end through the public API with host buffers (qhtp_matmul_run_host): pinned H2D of the
    # activation, GEMM, D2H of this rank's output slab, every step, in row chunks whose copies overlap
    act_h = d["act"].cpu().pin_memory()
    out_h = torch.empty(tuple(out.shape), dtype=out.dtype).pin_memory()
    t_e2e = max_over_ranks(statistics.mean(timed_steps(lambda: op.run_host(act_h, out_h, stream=stream),
                                                       max(3, args.steps // 2), 2, flush, world, stream)), world)
    op.check_host()
    e2e_ok = torch.equal(out_h, out.cpu())
    rf = row["roofline"]
    rf["traffic"] = NCU_TRAFFIC_BYTES.get(("qgemm", m, k, d["n"]))
    rf["kernel"] = ("split_u16_planes + qgemm_kernel<2,F32" + (",LO3" if op.lo_residual_launch(m) else "") +
                  "> (one qhtp_matmul_run)")
    res = {
        "metric": "w4a16_lpbq_gemm_tops", "value": ops_total / t_step / 1e12, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": row["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u16xint4->u16 (int8 tensor ops, int64 combine)",
        "data": "synthetic (BASELINE.json distributions, generated on device)",
        "config": {"workload": "W4A16 LPBQ GEMM 4096x4096x14336 (BASELINE configs[2]/[4]), output channels "
                               "sharded over the ranks", "m": m, "k": k, "n_total": n, "n_per_rank": d["n"],
                   "lpbq_block": 64,
                   "parallelism": f"N-shard x{world} of one weight set (qcom_htp_b200.shard), activation replicated",
                   "value_scope": "sharded GEMM; outputs stay in each rank's HBM as [M, N/P] slabs "
                                  "(the all-gather is timed in `allgather`)",
                   "l2": "flushed between steps: 256 MB write, then 256 MB read of another buffer (cold, clean L2)",
                   "bit_exact": row["check"]["bit_exact"], "bit_exact_check": row["check"]},
        "e2e": {"value": ops_total / t_e2e / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": m * k * 2,
                "d2h_bytes_per_step": m * d["n"] * 2, "ms_per_step": t_e2e * 1e3,
                "api": "QuantMatMul.run_host -> qhtp_matmul_run_host (pinned host buffers)",
                "output_equals_device_run": bool(all_ranks_true(e2e_ok, world))},
        "roofline": rf,
        "gpu_launches": 2 * args.steps,
        "clocks": row["clocks"],
    }
    if probe:
        res["tensor_peak_probe"] = probe
    if "cpu_baseline" in row:
        res["cpu_baseline"] = row["cpu_baseline"]
    if world > 1:
        res["allgather"] = gemm_allgather(op, d, out, args, world, stream, flush, ops_total, t_step)
    del op, out, act_h, out_h, d
    torch.cuda.empty_cache()
    if not args.no_w4a8:
        res["w4a8_per_channel"] = run_sharded_w4a8(args, world, rank, local, stream, flush, probe)
    if not args.no_gdn:
        res["secondary"] = run_gdn(args, world, rank, local, stream, secondary=True)
    if world == 1:
        if not args.no_families:
            res["families"] = run_families(args, world, rank, local, stream, flush, probe)
        if not args.no_decode:
            res["decode"] = {"workload": "W4A16 LPBQ decode/prefill rows (BASELINE configs[2])",
                             "peak_gbs": peaks()["hbm_gbs"], "rows": run_decode(args, world, rank, local, stream)}
        if not args.no_per_group:
            res["per_group"] = run_per_group(args, world, rank, local, stream)
        if not args.no_chain:
            res["chain"] = {"workload": "CHAIN=8 at M=K=N=256 per family (gen_quant_chain.py:1612-1613)",
                            "rows": run_chain(args, world, rank, local, stream, L2Flush(torch.device("cuda", local)))}
    return res


def run_sharded_w4a8(args, world, rank, local, stream, flush, probe) -> dict:
    """BASELINE configs[4]'s second GEMM: W4A8 per-channel 4096x4096x14336, sharded like the headline."""
    dev = torch.device("cuda", local)
    m, k, n = args.m, args.k, args.n
    full = synth_gemm("w4a8", "per_channel", m, k, n, seed=4848, device=dev)
    d = shard_gemm(full, world, rank)
    del full
    row, op = gemm_row(d, args, world, rank, stream, flush, steps=max(5, args.steps // 2), probe=probe, cpu=True,
                       cpu_budget=4.0)
    out = row.pop("_out")
    res = {"metric": "w4a8_per_channel_gemm_tops", "value": row["tops"], "unit": "TFLOP/s",
           "ms_per_step": row["ms_per_step"], "m": m, "k": k, "n_total": n, "n_per_rank": d["n"],
           "scaling": "strong", "kernel": "qgemm_kernel<1,F32> (u8 activation, [q | e'] weight planes)",
           "bit_exact": row["check"]["bit_exact"], "bit_exact_check": row["check"], "roofline": row["roofline"]}
    if "cpu_baseline" in row:
        res["cpu_baseline"] = row["cpu_baseline"]
    if world > 1:
        res["allgather"] = gemm_allgather(op, d, out, args, world, stream, flush, 2.0 * m * n * k,
                                          row["ms_per_step"] * 1e-3)
    del op, out, d
    torch.cuda.empty_cache()
    return res


FAMILY_ROWS = [  # (name, family, schema, free_offsets)
    ("u8i8", "u8i8", "per_channel", True),
    ("w4a8_per_channel", "w4a8", "per_channel", False),
    ("w4a8_lpbq", "w4a8", "lpbq", False),
    ("w8a16", "w8a16", "per_channel", False),
    ("w4a16_per_channel", "w4a16", "per_channel", False),
    ("w16a16", "w16a16", "per_channel", False),
]


def run_families(args, world, rank, local, stream, flush, probe, only: str | None = None,
                 shapes: list | None = None) -> list:
    """One row per MatMul family at the headline shape (u8i8 with BASELINE configs[0]'s free-offset
    encodings and per-tensor weights), plus W16A16 at BASELINE configs[2]'s decode/prefill shapes.
    Each row: time, logical TOPS, roofline, the oracle check of a sample of the timed output, and the
    reference's float64 CPU path on a row sample."""
    dev = torch.device("cuda", local)
    rows = []
    todo = [(nm, f, s, fo, args.m, args.k, args.n) for nm, f, s, fo in FAMILY_ROWS]
    todo += [("w16a16", "w16a16", "per_channel", False, mm, 4096, nn) for nn in (4096, 14336) for mm in (1, 16, 128)]
    if only is not None:
        todo = [t for t in todo if t[0] == only]
        if shapes:
            todo = [(t[0], t[1], t[2], t[3], mm, args.k, nn) for t in todo[:1] for mm, nn in shapes]
    for i, (name, fam, schema, free, m, k, n) in enumerate(todo):
        d = synth_gemm(fam, schema, m, k, n, seed=500 + i, device=dev, free_offsets=free)
        row, op = gemm_row(d, args, world, rank, stream, flush, steps=max(5, args.steps // 2), probe=probe,
                           cpu=True, cpu_budget=2.0)
        row.pop("_out")
        rows.append({"family": name, "m": m, "k": k, "n": n, "us": row["ms_per_step"] * 1e3,
                     "tops": row["tops"], "kernel": ("qdecode_kernel" if m <= 128 else "qgemm_kernel") +
                     f" (mode {int(op.plan.mode)}, {int(op.plan.a_planes)} activation plane(s))",
                     "encodings": "free activation/output zero points, per-tensor int8 weights (configs[0])"
                     if free else "fixed zero points, per-channel weights",
                     "act_zp": d["a_zp"], "out_zp": d["o_zp"],
                     "bit_exact": row["check"]["bit_exact"], "bit_exact_check": row["check"],
                     "roofline": row["roofline"], "cpu_baseline": row.get("cpu_baseline")})
        del op, d
        torch.cuda.empty_cache()
    return rows


CHAIN_ROWS = [("u8i8", "u8i8", "per_channel"), ("w4a8_per_channel", "w4a8", "per_channel"),
              ("w4a8_lpbq", "w4a8", "lpbq"), ("w8a16", "w8a16", "per_channel"),
              ("w4a16_per_channel", "w4a16", "per_channel"), ("w4a16_lpbq", "w4a16", "lpbq"),
              ("w16a16", "w16a16", "per_channel")]


def cpu_chain_baseline(d: dict, chain: int, budget_s: float = 2.0) -> dict:
    """The reference's chain reference (gen_quant_chain.py:1542-1545): its float64 step applied
    `chain` times, each step's requantized codes the next step's activation codes."""
    from oracle import mm_oracle as O   # the checker; timed here as the reference CPU implementation
    threads = blas_threads()
    k, n = d["k"], d["n"]
    q = d["q"].cpu().numpy()
    scale = d["scale"].cpu().numpy()
    if d["factor"] is not None:
        f = d["factor"].cpu().numpy()
        q = (q.astype(np.int16).reshape(n, k // d["block"], d["block"]) * f.astype(np.int16)[:, :, None]).reshape(n, k)
    w_deq = (q.astype(np.float32) * scale[:, None]).astype(np.float64)
    bias_deq = d["bias_q"].cpu().numpy().astype(np.float64) * (d["s_a"] * scale.astype(np.float64))
    o_bits = FAMILY_BITS[d["family"]][2]
    o_dt = np.uint16 if o_bits == 16 else np.uint8
    act = d["act"].cpu().numpy()
    reps, elapsed = 0, 0.0
    t0 = time.perf_counter()
    while elapsed < budget_s or reps == 0:
        x = act
        for _ in range(chain):
            y = ((x.astype(np.float64) - d["a_zp"]) * d["s_a"]) @ w_deq.T + bias_deq
            x = O.quantize_affine(y, d["s_o"], -d["o_zp"], (1 << o_bits) - 1, o_dt)
        reps += 1
        elapsed = time.perf_counter() - t0
    return {"value": reps * chain * 2.0 * act.shape[0] * n * k / elapsed / 1e12, "unit": "TFLOP/s",
            "cores": int(threads), "kind": "port",
            "sample": f"{reps} chains of {chain} float64 steps at {act.shape[0]}x{k}x{n} "
                      f"(gen_quant_chain.py:1542-1545 restated); {elapsed:.2f} s"}


def run_chain(args, world, rank, local, stream, flush, chain: int = 8, mkn: int = 256) -> list:
    """CHAIN=8 at M = K = N = 256 (the reference's chain gates, gen_quant_chain.py:1612-1613) per
    family: one qhtp_<family>_run_prepared call (the fused kernel keeps the intermediate activations in
    shared memory) against the same chain as `chain` separate GEMM calls through HBM.  Both outputs
    are compared with each other and a row sample with the oracle's chained output."""
    from oracle import mm_oracle as O   # the checker
    dev = torch.device("cuda", local)
    rows = []
    steps = max(10, args.steps)
    for i, (name, fam, schema) in enumerate(CHAIN_ROWS):
        d = synth_gemm(fam, schema, mkn, mkn, mkn, seed=900 + i, device=dev, block=64 if schema == "lpbq" else 64)
        op = make_op(d)
        act = d["act"]
        o_dt = torch.uint16 if FAMILY_BITS[fam][2] == 16 else torch.uint8
        out_f = torch.empty((mkn, mkn), dtype=o_dt, device=dev)
        scratch = torch.zeros(op.scratch_bytes(mkn, chain), dtype=torch.uint8, device=dev)
        fused = lambda: op.run_prepared(act, out_f, chain=chain, scratch=scratch)
        t_f = max_over_ranks(statistics.mean(timed_steps(fused, steps, args.warmup, flush, world, stream)), world)
        bufs = [torch.empty((mkn, mkn), dtype=o_dt, device=dev) for _ in range(2)]

        def unfused():
            x = act
            for s in range(chain):
                op(x, bufs[s % 2])
                x = bufs[s % 2]
        t_u = max_over_ranks(statistics.mean(timed_steps(unfused, steps, args.warmup, flush, world, stream)), world)
        op.check_device(mkn)
        out_u = bufs[(chain - 1) % 2]
        same = bool(torch.equal(out_f, out_u))
        # the checker: the oracle's chain on a row sample (rows are independent through the chain)
        fam_o = O.FAMILIES[ORACLE_FAMILY[(fam, schema)]]
        if schema == "lpbq":
            fam_o = fam_o.with_block(d["block"])
        r = torch.from_numpy(sample_rows(mkn, 8)).to(dev)
        q = d["q"].cpu().numpy()
        f = d["factor"].cpu().numpy() if d["factor"] is not None else None
        expanded = None if f is None else (q.astype(np.int16).reshape(mkn, -1, d["block"]) *
                                           f.astype(np.int16)[:, :, None]).reshape(mkn, -1)
        x = d["act"].index_select(0, r).cpu().numpy()
        for _ in range(chain):
            c = O.QuantCase(fam_o, x, q, d["scale"].cpu().numpy(), d["bias_q"].cpu().numpy(), d["s_a"], d["s_o"],
                            f, expanded)
            x = O.exact_output(c, dequant="exact" if fam == "w16a16" else "f32")
        bad = int((out_f.index_select(0, r).cpu().numpy() != x).sum())
        ops = chain * 2.0 * mkn ** 3
        row = {"family": name, "chain": chain, "m": mkn, "k": mkn, "n": mkn,
               "fused_us": t_f * 1e6, "unfused_us": t_u * 1e6, "speedup": t_u / t_f,
               "tops_fused": ops / t_f / 1e12, "tops_unfused": ops / t_u / 1e12,
               "kernel": "qchain_kernel (one launch; + split_u16_planes for u16 activations)",
               "fused_equals_unfused": same, "bit_exact": bad == 0 and same,
               "bit_exact_check": {"mismatches": bad, "checked": int(x.size),
                                   "sample": f"{len(r)} rows through all {chain} steps vs the oracle's chain"}}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            row["cpu_baseline"] = cpu_chain_baseline(d, chain)
        rows.append(row)
        del op, d, scratch, bufs, out_f
    return rows


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
    i8, i8_src = int8_peak(pk, getattr(args, "_probe", None))
    achieved = ops / statistics.mean(times) / 1e12
    # the checker: oracle per_group_output on a row x channel sample
    from oracle import mm_oracle as O
    rows, cols = sample_rows(m), sample_channels(n)
    r_t, c_t = torch.from_numpy(rows).to(dev), torch.from_numpy(cols).to(dev)
    case = O.QuantCase(O.FAMILIES["w4a16_per_group"], act.index_select(0, r_t).cpu().numpy(),
                       d["q"].index_select(0, c_t).cpu().numpy(), d["scale"].index_select(0, c_t).cpu().numpy(),
                       np.zeros(len(cols), np.int32), d["s_a"], d["s_o"],
                       bias_float=d["bias"].index_select(0, c_t).cpu().numpy())
    bad = int((out.index_select(0, r_t).index_select(1, c_t).cpu().numpy() != O.per_group_output(case)).sum())
    res = {"metric": "w4a16_per_group_gemm_tops", "value": ops * world / t / 1e12, "unit": "TFLOP/s",
           "ms_per_step": t * 1e3, "m": m, "k": k, "n_per_gpu": n, "group": 64,
           "kernel": "split_u16_planes + qgemm_group_kernel<2> (channel-major, float64 group accumulation)",
           "bit_exact": bad == 0, "bit_exact_check": {"mismatches": bad, "checked": int(len(rows) * len(cols)),
                                                       "sample": "rows x 4 channels per tile vs oracle per_group_output"},
           "roofline": {"bound": "tensor", "achieved": achieved, "peak": i8, "unit": "TFLOP/s",
                        "frac": achieved / i8, "executed_tflops": achieved * 4,
                        "frac_executed": achieved * 4 / i8, "peak_src": i8_src,
                        "note": "per 64-K group the accumulators are drained from TMEM and folded into float64"},
           "gpu_launches": 2 * max(5, args.steps // 2)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_per_group_baseline(d)
    return res


def run_decode(args, world, rank, local, stream, shapes=None) -> list:
    """BASELINE decode/prefill rows of the W4A16 LPBQ GEMM (M in {1, 16, 128}, K = 4096,
    N in {4096, 14336}): HBM-bound.  Reports GB/s on the algorithmic bytes (int4 weights, block
    factors, scales, bias, u16 activation and output) and on the bytes the kernel reads (the
    prepared byte planes: q and the float32-dequant residual e', 2 bytes per weight; or, for the
    int4 code stream, 0.5 byte per weight plus factors and e' tables)."""
    dev = torch.device("cuda", local)
    pk = peaks()
    flush = L2Flush(dev)
    rows = []
    k, blk = 4096, 64
    shapes = shapes or [(m, n) for n in (4096, 14336) for m in (1, 16, 128)]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for m, n in shapes:
        d = synth_gemm("w4a16", "lpbq", m, k, n, seed=4321 + m + n, device=dev, block=blk)
        op = make_op(d)
        act, out = d["act"], torch.empty((m, n), dtype=torch.uint16, device=dev)
        times = timed_steps(lambda: op(act, out), max(5, args.steps // 2), args.warmup, flush, world, stream)
        op.check_device(m)
        t = max_over_ranks(statistics.mean(times), world)   # the event clock ticks in ~1 us steps
        alg = gemm_alg_bytes(d, n)
        # the library's dispatch: the int4 code stream for one or two rows over a long weight stream
        # (>= 6 stages of 256 K per SM); the channel-major decode kernel up to 64 rows, and up to 128
        # rows when the channel tiles leave room for a K split; else the row-tiled GEMM
        n_tiles = (n + 127) // 128
        code_stream = m <= 2 and bool(op.plan.flags & 2) and n_tiles * (k // 256) >= 6 * sms
        row_tiled = m > 64 and 2 * n_tiles > sms
        if code_stream:  # codes, factors per 32 K, one e' table set per tile, records, activation, output
            read = n_tiles * 128 * k // 2 + n_tiles * (k // 32) * 128 + n_tiles * 16 * 128 * 16 + n * 32 + \
                m * k * 2 + m * n * 2
            kernel = "qgemv4_kernel (int4 code stream, CUDA cores) + dec4_combine_kernel"
        else:
            read = int(op.plan.plane_bytes) + n * 32 + m * k * 2 + m * n * 2
            kernel = "split_u16_planes + " + ("qgemm_kernel (row tiles)" if row_tiled else
                                              "qdecode_kernel (channel-major, cluster split-K)")
        chk = check_gemm_sample(d, out)
        rows.append({"m": m, "k": k, "n": n, "us": round(t * 1e6, 2),
                     "kernel": kernel,
                     "alg_bytes": alg, "alg_gbs": round(alg / t / 1e9, 1),
                     "alg_frac": round(alg / t / 1e9 / pk["hbm_gbs"], 3),
                     "read_bytes": read, "read_gbs": round(read / t / 1e9, 1),
                     "read_frac": round(read / t / 1e9 / pk["hbm_gbs"], 3),
                     "bit_exact": chk["bit_exact"], "bit_exact_checked": chk["checked"]})
        del op, d, act, out
    return rows


def run_gdn(args, world, rank, local, stream, secondary=False) -> dict:
    """GDN C=256 inverse over BASELINE configs[4]'s 64 x 32 x 64 = 131072 chunks (--gdn-chunks),
    split over batch x heads (contiguous chunk ranges, qcom_htp_b200.shard.shard_chunks): the bf16 ->
    f32 inverse, the reference's u16 code carrier, and the fused A construction + inverse, each with
    the achieved oc on a chunk sample; at one GPU also configs[3]'s 4096 chunks."""
    from qcom_htp_b200 import gdn_chunk_inverse, gdn_inverse, gdn_solve_u16
    from qcom_htp_b200.shard import shard_chunks
    dev = torch.device("cuda", local)
    C = 256
    total = args.gdn_chunks
    c0, c1 = shard_chunks(total, world, rank)
    n_chunks = c1 - c0
    pk = peaks()
    flush = L2Flush(dev)
    steps = args.steps
    A = synth_gdn_A(n_chunks, C, 128, seed=99 + rank, device=dev)
    T = torch.empty((n_chunks, C, C), dtype=torch.float32, device=dev)
    fn = lambda: gdn_inverse(A, T)
    with ClockSampler(local) as clk:
        times = timed_steps(fn, steps, args.warmup, flush, world, stream, clk)
    t = max_over_ranks(statistics.mean(times), world)
    bytes_alg = n_chunks * (C * C * 2 + C * C * 4)       # read A (bf16), write T (fp32)
    achieved = bytes_alg / statistics.mean(times) / 1e9
    oc = gdn_oc_sample(T, A)
    oc["oc"] = max_over_ranks(oc["oc"], world)
    per_chunk = NCU_TRAFFIC_BYTES[("gdn_per_chunk",)]
    res = {"metric": "gdn_inverse_chunks_per_s", "value": total / t, "unit": "chunks/s",
           "ms_per_step": t * 1e3, "scaling": "strong",
           "config": {"workload": "GDN C=256 inverse, BASELINE configs[4]: 64 x 32 x 64 chunks split over "
                                  "batch x heads", "chunks_total": total, "chunks_per_rank": n_chunks},
           "oc": oc,
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": achieved / pk["hbm_gbs"], "traffic": int(per_chunk * n_chunks),
                        "peak_src": f"hbm_gbs ({pk['src']})"},
           "gpu_launches": steps, "clocks": clk.summary()}
    A_sample = A[:64].clone()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_gdn_baseline(A_sample)
    if world > 1:
        import torch.distributed as dist
        # every rank ends with all ranks' T ([world * chunks, C, C]); the only collective of the path
        gathered = torch.empty((world,) + tuple(T.shape), dtype=T.dtype, device=dev)
        ag = lambda: dist.all_gather_into_tensor(gathered, T)
        t_ag = max_over_ranks(statistics.mean(timed_steps(ag, max(3, steps // 2), 2, flush, world, stream)), world)
        res["allgather"] = {"ms": t_ag * 1e3, "bytes_received_per_rank": (world - 1) * T.numel() * T.element_size(),
                            "chunks_per_s_incl_allgather": total / (t + t_ag)}
        del gathered
    # the reference's production carrier (GdnSolve / gdnbm_solve): u16 codes in and out, scales of
    # gdn_solve_oc_check.py:20-23, same chunks
    sA, sT, zp = 2.770166930875267e-05, 6.103701895199438e-05, 32768
    Ac = torch.empty((n_chunks, C, C), dtype=torch.uint16, device=dev)
    for s in range(0, n_chunks, 1024):
        Ac[s:s + 1024] = torch.clamp(torch.round(A[s:s + 1024].float() / sA) + zp, 0, 65535).to(torch.int32)
    del A
    torch.cuda.empty_cache()
    Tc = torch.empty_like(Ac)
    fn16 = lambda: gdn_solve_u16(Ac, zpA=zp, sA=sA, zpT=zp, sT=sT, out=Tc)
    t16 = max_over_ranks(statistics.mean(timed_steps(fn16, steps, args.warmup, flush, world, stream)), world)
    b16 = n_chunks * (C * C * 2 + C * C * 2)
    idx = torch.from_numpy(np.linspace(0, n_chunks - 1, 16).astype(np.int64)).to(dev)
    from oracle import gdn_oracle as G   # the checker
    a_deq = (Ac.index_select(0, idx).to(torch.int32) - zp).double().cpu().numpy() * sA
    t_deq = (Tc.index_select(0, idx).to(torch.int32) - zp).double().cpu().numpy() * sT
    oc16 = max_over_ranks(G.oc(t_deq, G.inverse_fp64(a_deq)), world)
    res["u16_carrier"] = {"metric": "gdn_solve_u16_chunks_per_s", "value": total / t16,
                          "ms_per_step": t16 * 1e3, "hbm_gbs": b16 / t16 / 1e9 * world,
                          "hbm_frac": b16 / t16 / 1e9 / pk["hbm_gbs"],
                          "oc": {"oc": oc16, "gate": G.OC_GATE, "chunks": 16},
                          "note": "u16 codes A -> u16 codes T (zp 32768), algorithmic bytes 2C^2 + 2C^2 per chunk"}
    del Ac, Tc
    torch.cuda.empty_cache()
    # the step on the input side fused in: A built on the SM from raw keys, beta and per-token log
    # gates (gdn_chunk Stage A, scripts/gdn_ref_kernel.py:66-82), then inverted; same chunk count
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    kk = torch.randn((n_chunks, C, 128), generator=gen, device=dev).to(torch.bfloat16)
    bb = torch.sigmoid(torch.randn((n_chunks, C), generator=gen, device=dev))
    gg = torch.nn.functional.logsigmoid(0.5 * torch.randn((n_chunks, C), generator=gen, device=dev) - 2.0)
    fnf = lambda: gdn_chunk_inverse(kk, bb, gg, T)
    tf = max_over_ranks(statistics.mean(timed_steps(fnf, steps, args.warmup, flush, world, stream)), world)
    bf = n_chunks * (C * 128 * 2 + C * 4 * 2 + C * C * 4)
    Af = G.chunk_A_from_kbg(kk.index_select(0, idx).float().cpu().numpy(), bb.index_select(0, idx).cpu().numpy(),
                            gg.index_select(0, idx).cpu().numpy())
    ocf = max_over_ranks(G.oc(T.index_select(0, idx).double().cpu().numpy(), G.inverse_fp64(Af)), world)
    per_chunk_f = NCU_TRAFFIC_BYTES[("gdn_fused_per_chunk",)]
    res["fused_A"] = {"metric": "gdn_chunk_inverse_chunks_per_s", "value": total / tf,
                      "ms_per_step": tf * 1e3, "hbm_gbs": bf / tf / 1e9, "hbm_frac": bf / tf / 1e9 / pk["hbm_gbs"],
                      "traffic": int(per_chunk_f * n_chunks),
                      "oc": {"oc": ocf, "gate": G.OC_GATE, "chunks": 16},
                      "kernel": "gdn256f_kernel (Gram MMAs + A epilogue + the C=256 inverse)",
                      "note": "k bf16 [C,128], beta and log gates f32 [C] -> T f32: algorithmic bytes 256C + 8C + 4C^2 "
                              "per chunk; A (bf16 [C,C]) never written or read"}
    del kk, bb, gg, T
    torch.cuda.empty_cache()
    if world == 1 and args.gdn_chunks != 4096:
        # batch 8 x 32 heads x 16 chunks = 4096 chunks
        A3 = synth_gdn_A(4096, C, 128, seed=98, device=dev)
        T3 = torch.empty((4096, C, C), dtype=torch.float32, device=dev)
        t3 = statistics.mean(timed_steps(lambda: gdn_inverse(A3, T3), steps, args.warmup, flush, world, stream))
        b3 = 4096 * (C * C * 6)
        res["config3_4096_chunks"] = {"value": 4096 / t3, "unit": "chunks/s", "ms_per_step": t3 * 1e3,
                                      "hbm_gbs": b3 / t3 / 1e9, "hbm_frac": b3 / t3 / 1e9 / pk["hbm_gbs"],
                                      "oc": gdn_oc_sample(T3, A3),
                                      "workload": "BASELINE configs[3]: batch 8 x 32 heads x 16 chunks of C=256"}
        del A3, T3
    if not secondary:
        res.update({"n_gpus": world, "steps": steps, "warmup": args.warmup, "higher_is_better": True,
                    "vs_baseline": None, "dtype": "bf16 in / fp32 out (tf: bf16 MMA, fp32 acc)",
                    "data": "synthetic (BASELINE.json GDN distribution, generated on device)", "e2e": None})
    return res


# ----------------------------------------------------------------------------------------------
# reference arm: the reference's own CPU implementation of the path, on the host cores
# ----------------------------------------------------------------------------------------------
def run_reference(args, world, rank) -> None:
    if rank != 0:
        return
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    m, k, n = args.m, args.k, args.n
    d = synth_gemm("w4a16", "lpbq", m, k, n, seed=1234, device=dev)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_gemm_baseline(d, budget_s=max(2.0, 60.0 / max(1, args.steps + args.warmup)))
        if i >= args.warmup:
            vals.append(r)
    v = statistics.mean(x["value"] for x in vals)
    out = {"impl": "reference", "metric": "w4a16_lpbq_gemm_tops", "value": v, "unit": "TFLOP/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
           "config": {"workload": "W4A16 LPBQ GEMM 4096x4096x14336 (BASELINE configs[2]/[4]), output channels "
                                  "sharded over the ranks", "m": m, "k": k, "n_total": n, "lpbq_block": 64},
           "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": vals[-1]["cores"], "kind": "port",
                            "sample": vals[-1]["sample"]},
           "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference has no GPU path; its CPU oracle (float64 numpy, BLAS on every host core) "
                   "is timed on the host cores"}
    print(json.dumps(out))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "gdn", "decode", "per_group", "family", "peak", "chain"],
                    default="gemm")
    ap.add_argument("--family", default="w4a8_per_channel", help="--workload family: the row name")
    # --gemm-m / --gemm-n: the same options under names that torchrun's own parser does not take for
    # abbreviations of its --master-*/--nnodes/--nproc-per-node (a bare --m or --n under torchrun errors)
    ap.add_argument("--m", "--gemm-m", dest="m", type=int, default=4096)
    ap.add_argument("--k", "--gemm-k", dest="k", type=int, default=4096)
    ap.add_argument("--n", "--gemm-n", dest="n", type=int, default=14336)
    ap.add_argument("--gdn-chunks", type=int, default=131072)
    ap.add_argument("--no-gdn", action="store_true")
    ap.add_argument("--no-w4a8", action="store_true")
    ap.add_argument("--no-families", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-per-group", action="store_true")
    ap.add_argument("--no-chain", action="store_true")
    ap.add_argument("--no-probe", action="store_true")
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
    dev = torch.device("cuda", local)
    if args.workload == "gemm":
        res = run_gemm(args, world, rank, local, stream)
    elif args.workload == "gdn":
        res = run_gdn(args, world, rank, local, stream)
    elif args.workload == "chain":
        rows = run_chain(args, world, rank, local, stream, L2Flush(dev))
        res = {"metric": "chain8_fused_tops", "n_gpus": world, "steps": max(10, args.steps), "warmup": args.warmup,
               "higher_is_better": True, "rows": rows}
    elif args.workload == "peak":
        res = {"metric": "tcgen05_mma_rate", "n_gpus": world, **measure_mma_peak(dev)}
    elif args.workload == "family":
        # one MatMul family row alone at --m / --k / --n (the command its ncu summary was taken with)
        rows = run_families(args, world, rank, local, stream, L2Flush(dev), None, only=args.family,
                            shapes=[(args.m, args.n)])
        res = {"metric": f"{args.family}_gemm_tops", "value": rows[0]["tops"], "unit": "TFLOP/s", "n_gpus": world,
               "steps": max(5, args.steps // 2), "warmup": args.warmup, "higher_is_better": True, "row": rows[0]}
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
               "roofline": row["roofline"], "gpu_launches": row["gpu_launches"], "e2e": None,
               "bit_exact": row["bit_exact"]}
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
               "gpu_launches": 2 * max(5, args.steps // 2), "e2e": None, "bit_exact": row["bit_exact"]}
    if rank == 0:
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
