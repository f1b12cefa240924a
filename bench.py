#!/usr/bin/env python3
"""Benchmark of the tadma_b200 hot path (achieved HBM GB/s), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1-5] [--impl ours|reference]
    python bench.py --views      # view copies / element-wise calls vs torch, one line per case

Metric: achieved HBM GB/s = algorithmic bytes (every input
read once, every output written once; gathered rows counted per use) / time.
Headline (`value`): config 2, y = gelu(x * 0.5 +
bias), x[8192, 8192] bf16, bias[8192] bf16 -> y bf16, one fused kernel.  The
other configs (1, 3, 4, 5) are timed after it in the same process and
reported under "configs", each with its own roofline parts, restated
reference kernels and CPU baseline.

Multi-GPU (torchrun, one process per GPU): every config's GLOBAL workload is
split on its leading axis (config 2: 8192 / N rows per rank; config 3: 32 / N
batches; config 4: 64 / N LayerNorm and 32 / N softmax batches; config 5:
2048 / N id rows), each shard generated at its global element offset, so the
N ranks together do exactly the 1-GPU job (strong scaling); config 1 runs as
N replicas.  No collective on the data path; the one exchange of the path, a
sum over the sharded axis, is measured separately ("cross_shard_reduce":
config 3's X summed over axis 0, a local reduction per rank plus one NCCL
all-reduce, checked at sampled positions).  Timing: W warm-up steps, then K
steps back to back between two CUDA events on the launching stream, barrier +
synchronize on both sides, the max over ranks reported.  No L2 flush: every
step's inputs are larger than L2 or rotate through sets whose total is
(config 2 keeps at least 252 MB, twice the L2, of x/y sets in rotation).

--impl reference times the reference's algorithm on the host cores: the
reference itself cannot be built here (it needs clang >= 19 / C++23), so this
is the oracle's straightforward host loop (oracle/), all threads, on a
bounded sample of the same workload; only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GB = 1e9
L2_BYTES = 126 << 20
# Steps timed per extra config (the headline takes --steps): enough for a
# timed region of tens of milliseconds each at 1 GPU.
EXTRA_STEPS = {1: 200, 2: 200, 3: 20, 4: 20, 5: 6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-extras", action="store_true",
                    help="time the headline config only (no other configs, no cross-shard reduce)")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's GPU algorithm (baseline/refalgo) beside ours")
    ap.add_argument("--views", action="store_true",
                    help="instead of a config: one JSON line per view-copy / element-wise case of the generated-graph "
                         "calls (permutes, transposes, casts, concat, where), ours and torch, 1 GPU")
    ap.add_argument("--chain-reduce", action="store_true",
                    help="fused chain -> reduction calls (tadma_b200_reduce_chain) on X[32768, 4096], one line per case")
    ap.add_argument("--view-filter", default="",
                    help="with --views: run only the cases whose name contains this text")
    ap.add_argument("--batch", type=int, default=0,
                    help="leading-axis size per GPU (0 = the BASELINE size); smaller values give the small cases "
                         "used for ncu captures")
    return ap.parse_args()


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per
# (config, part label) from `ncu --set full` captures of this script, scaled
# from the captured batch to the full workload by rows processed; the
# summaries and commands are under profiles/.  Writes still dirty in L2 when a
# launch ends are not in its figure (they reach DRAM during the next launch).
NCU_TRAFFIC = {
    (2, "act(x*s + b) rows"): {"bytes": 217880832, "captured": "full size"},
    (3, "sum axis -1"): {"bytes": 8 * 271808512, "captured": "batch 4, x8"},
    (3, "max axis -1"): {"bytes": 8 * 272069632, "captured": "batch 4, x8"},
    (3, "argmax axis -1"): {"bytes": 8 * 272051200, "captured": "batch 4, x8"},
    (3, "mean axis 1 (+ finish kernel when split)"): {"bytes": 8 * 273262592, "captured": "batch 4, x8"},
    (4, "LayerNorm (ONNX) rows of 1024"): {"bytes": 2 * 217847000, "captured": "batch 32, x2"},
    (4, "softmax rows of 2048"): {"bytes": 2 * 4245502000, "captured": "batch 16, x2"},
    (5, "gather + pos add"): {"bytes": 32 * 4077850000, "captured": "batch 64, x32"},
}


# ----------------------------------------------------------------- clocks --

class ClockSampler:
    """Polls NVML (SM clock, clock-event reasons) in a thread during the timed region."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz, self.ok = [], 0, None, False
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            h = None
            try:
                props = torch.cuda.get_device_properties(device_index)
                bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nvml, self.h = pynvml, h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML unavailable: report it, do not fail the bench
            self.err = str(e)
        self._stop = threading.Event()

    def _reasons(self):
        n = self.nvml
        f = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        return f(self.h)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                self.reasons |= int(self._reasons())
            except Exception:
                pass
            time.sleep(0.001)

    def __enter__(self):
        if self.ok:
            self._stop.clear()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def result(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": getattr(self, "err", "no samples")}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": [v for k, v in self.REASONS.items() if self.reasons & k], "samples": len(self.samples)}


# ---------------------------------------------------------------- configs --

class Config1:
    """y = sum_{last}(exp(A + b)), A[64, 128] fp32, b[128] fp32 -> y[64]: a
    launch-bound correctness config.  One step = one tadma_b200_reduce_chain
    call (the chain A + b -> exp reduced in the same kernel), captured once
    into a CUDA graph and replayed; the eager call and the two-call
    composition (eltwise, then reduce with an exp pre-op) are timed beside it."""
    dtype = "f32"

    scaling = "replicas"  # too small to split: every GPU runs the whole workload

    def __init__(self, rank, world, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Compute, Dist, DType, Op, Reduce, instr, make_tensor
        R = batch or 64
        self.name = f"cfg1: y = sum_last(exp(A + b)), A[{R},128] fp32, b[128] fp32 -> [{R}] (one fused kernel, CUDA graph)"
        self.A = torch.empty((R, 128), dtype=torch.float32, device="cuda")
        self.b = torch.empty((128,), dtype=torch.float32, device="cuda")
        tb.fill(self.A, Dist.NORMAL, 0.0, 1.0, 0, 1)
        self.shard = "the whole workload (replica)"
        tb.fill(self.b, Dist.NORMAL, 0.0, 1.0, 0, 2)
        self.t = torch.empty_like(self.A)
        self.y = torch.empty((R,), dtype=torch.float32, device="cuda")
        bv = make_tensor(self.b.data_ptr(), DType.F32, [R, 128], [0, 1])
        self.side = torch.cuda.Stream()

        def fused(st):
            return tb.prepare_reduce_chain(Reduce.SUM, [self.A, bv], [instr(Op.ADD, b=1), instr(Op.EXP)], -1, self.y,
                                           Compute.F32, stream=st)
        self.eager = fused(None)
        self.two = [tb.prepare_eltwise(self.t, [self.A, bv], [instr(Op.ADD, b=1)], Compute.F32),
                    tb.prepare_reduce(Reduce.SUM, self.t, -1, self.y.view(R, 1), Op.EXP)]
        cap = fused(self.side)
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            cap()
        self.side.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.side):
            cap()
        torch.cuda.synchronize()
        self.bytes = R * 128 * 4 + 128 * 4 + R * 4
        self.launches = 1
        self.units = R

    def step(self):
        self.graph.replay()

    def two_calls(self):
        for c in self.two:
            c()

    def parts(self):
        return [("chain_reduce_typed_kernel", "one fused call, CUDA graph replay", self.bytes, self.step),
                ("chain_reduce_typed_kernel", "compare: one fused call, eager", self.bytes, self.eager),
                ("affine_rows_kernel + reduce_row_kernel", "compare: two calls (eltwise, reduce), eager", self.bytes,
                 self.two_calls)]

    def cpu_sample(self, budget_s):
        import numpy as np
        from oracle import oracle as O
        from tadma_b200.abi import Op, Reduce
        A = self.A.cpu().numpy()
        b = self.b.cpu().numpy()
        y = np.zeros((A.shape[0], 1), np.float32)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            t = (A + b).astype(np.float32)
            O.reduce(Reduce.SUM, t, -1, y, Op.EXP)
            done += 1
        el = time.perf_counter() - t0
        return done * self.bytes / el / GB, 1, f"{done} x the whole step (numpy add + oracle exp-sum, 1 thread)"


class Config2:
    """y = gelu(x * 0.5 + bias), x[8192, 8192] bf16, bias[8192] bf16, y bf16;
    a rank owns a contiguous block of x's rows."""
    COLS = 8192
    dtype = "bf16"
    scaling = "strong"

    def __init__(self, rank, world, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Compute, Dist, DType, make_tensor
        from tadma_b200.shard import shard_range
        self.tb = tb
        self.GLOBAL_ROWS = batch or 8192
        sh = shard_range(self.GLOBAL_ROWS, rank, world)
        self.ROWS = R = sh.size
        C = self.COLS
        self.name = f"cfg2: y = gelu(x*0.5 + bias), x[{self.GLOBAL_ROWS},8192] bf16, bias[8192] bf16 -> bf16"
        self.shard = f"rows {sh.start}:{sh.stop} of {self.GLOBAL_ROWS}"
        self.bias = torch.empty((C,), dtype=torch.bfloat16, device="cuda")
        tb.fill(self.bias, Dist.NORMAL, 0.0, 0.1, seed=0, stream_id=2)
        self.bview = make_tensor(self.bias.data_ptr(), DType.BF16, [R, C], [0, 1])
        self.prog = self.program()
        # The rank's rows of x, plus copies at other addresses: the step rotates
        # through them so that no step finds its input (or output) in L2; the
        # sets in rotation hold at least twice the L2 size.
        set_bytes = 2 * R * C * 2
        self.nbuf = max(4, min(64, -(-2 * L2_BYTES // set_bytes)))
        self.xs, self.ys, self.calls = [], [], []
        for k in range(self.nbuf):
            x = torch.empty((R, C), dtype=torch.bfloat16, device="cuda")
            if k == 0:
                tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=1, offset=sh.start * C)
            else:
                x.copy_(self.xs[0])
            y = torch.empty((R, C), dtype=torch.bfloat16, device="cuda")
            self.xs.append(x)
            self.ys.append(y)
            self.calls.append(tb.prepare_eltwise(y, [x, self.bview], self.prog, Compute.F32))
        self.x, self.y, self.i = self.xs[0], self.ys[0], 0
        self.bytes = 2 * R * C * 2 + C * 2
        self.launches = 1
        self.units = R * C
        self.l2_note = f"{self.nbuf} x/y sets of {set_bytes / 1e6:.0f} MB in rotation"
        # One pass over the sets (nbuf launches) captured in a CUDA graph: at
        # 8 GPUs a rank's step is 34 MB, a few microseconds of kernel, and a
        # ctypes call per launch would leave the GPU waiting on the host.
        self.side = torch.cuda.Stream()
        cap = [tb.prepare_eltwise(y, [x, self.bview], self.prog, Compute.F32, stream=self.side)
               for x, y in zip(self.xs, self.ys)]
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            for c in cap:
                c()
        self.side.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.side):
            for c in cap:
                c()
        torch.cuda.synchronize()
        self.timing_note = f"launches replayed from a CUDA graph of one pass over the {self.nbuf} sets"

    @staticmethod
    def program():
        from tadma_b200.abi import SRC_IMM, DType, Op, instr
        return [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
                instr(Op.GELU, round_dtype=DType.F32)]

    def step(self):
        self.calls[self.i % self.nbuf]()
        self.i += 1

    def run_steps(self, k):
        """k steps: whole passes over the sets from the graph, then single calls."""
        full, rem = divmod(k, self.nbuf)
        for _ in range(full):
            self.graph.replay()
        for _ in range(rem):
            self.step()

    def parts(self):
        return [("affine_rows_kernel", "act(x*s + b) rows", self.bytes, self.step)]

    def e2e(self, steps, stream):
        """Same op through the public API with host buffers: every step uploads
        x and bias from pinned host memory and downloads y, inside the timed
        region; tadma_b200.pipeline.RowPipeline overlaps the upload, the
        per-chunk C-ABI calls and the download across 8 row chunks."""
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Compute, DType, make_tensor
        from tadma_b200.pipeline import RowPipeline
        xh = torch.empty_like(self.x, device="cpu").pin_memory()
        bh = torch.empty_like(self.bias, device="cpu").pin_memory()
        yh = torch.empty_like(self.y, device="cpu").pin_memory()
        xh.copy_(self.x)
        bh.copy_(self.bias)
        C = self.COLS

        def make_call(lo, hi, st):
            bv = make_tensor(self.bias.data_ptr(), DType.BF16, [hi - lo, C], [0, 1])
            return tb.prepare_eltwise(self.y[lo:hi], [self.x[lo:hi], bv], self.prog, Compute.F32, stream=st)

        pipe = RowPipeline(self.ROWS, 8, uploads=[(xh, self.x)], downloads=[(self.y, yh)], make_call=make_call,
                           once=[(bh, self.bias)])
        pipe(stream)
        stream.synchronize()
        times = []
        for _ in range(steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            pipe(stream)
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e) / 1e3)
        h2d = xh.numel() * 2 + bh.numel() * 2
        d2h = yh.numel() * 2
        return statistics.mean(times), h2d, d2h

    # CPU legs (oracle host loop: test infrastructure, timed as the baseline only)
    def cpu_sample(self, budget_s):
        import numpy as np
        from oracle import oracle as O
        rows = 1024
        x = self.x[:rows].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
        b = self.bias.view(torch_int16()).cpu().numpy().view(np.uint16)
        y = np.zeros_like(x)
        L = O.lib()
        done, t0 = 0, time.perf_counter()
        while True:
            L.or_cfg2_gelu_affine_bf16(O.ptr(x), O.ptr(b), 0.5, O.ptr(y), rows, self.COLS)
            done += 1
            el = time.perf_counter() - t0
            if el >= budget_s:
                break
        bytes_ = done * (2 * rows * self.COLS * 2 + self.COLS * 2)
        return bytes_ / el / GB, L.or_num_threads(), f"{done} x {rows} rows of [8192, 8192] ({rows * self.COLS} elements per call)"


def torch_int16():
    import torch
    return torch.int16


class Config3:
    """sum / max / argmax over the last axis and mean over the middle axis of X[32, 4096, 4096] fp32."""
    dtype = "f32"

    scaling = "strong"

    def __init__(self, rank, world, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, Reduce
        from tadma_b200.shard import shard_range
        self.tb = tb
        GB_, R, C = batch or 32, 4096, 4096
        sh = shard_range(GB_, rank, world)
        B = sh.size
        self.name = f"cfg3: sum/max/argmax over axis -1 + mean over axis 1 of X[{GB_},4096,4096] fp32"
        self.shard = f"batches {sh.start}:{sh.stop} of {GB_}"
        self.global_batch, self.batch0 = GB_, sh.start
        self.x = torch.empty((B, R, C), dtype=torch.float32, device="cuda")
        tb.fill(self.x, Dist.UNIFORM, -1.0, 1.0, seed=0, stream_id=1, offset=sh.start * R * C)
        self.s = torch.empty((B, R, 1), dtype=torch.float32, device="cuda")
        self.m = torch.empty((B, R, 1), dtype=torch.float32, device="cuda")
        self.a = torch.empty((B, R), dtype=torch.int64, device="cuda")
        self.mean = torch.empty((B, 1, C), dtype=torch.float32, device="cuda")
        xin = B * R * C * 4
        self.bytes = 4 * xin + B * R * 4 * 2 + B * R * 8 + B * C * 4
        self.launches = 4
        self.units = 4 * B * R * C
        self.calls = [tb.prepare_reduce(Reduce.SUM, self.x, -1, self.s), tb.prepare_reduce(Reduce.MAX, self.x, -1, self.m),
                      tb.prepare_reduce(Reduce.ARGMAX, self.x, -1, self.a),
                      tb.prepare_reduce(Reduce.MEAN, self.x, 1, self.mean)]

    def step(self):
        for c in self.calls:
            c()

    def parts(self):
        B, R, C = self.x.shape
        xin = self.x.numel() * 4
        return [("reduce_row_kernel", "sum axis -1", xin + B * R * 4, self.calls[0]),
                ("reduce_row_kernel", "max axis -1", xin + B * R * 4, self.calls[1]),
                ("reduce_row_kernel", "argmax axis -1", xin + B * R * 8, self.calls[2]),
                ("reduce_col_kernel", "mean axis 1 (+ finish kernel when split)", xin + B * C * 4, self.calls[3])]

    def cpu_sample(self, budget_s):
        import numpy as np
        from oracle import oracle as O
        x = self.x[0, :1024].contiguous().cpu().numpy()
        L = O.lib()
        s, a = np.zeros(1024, np.float32), np.zeros(1024, np.int64)
        mean = np.zeros(4096, np.float32)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            L.or_cfg3_sum_lastaxis_f32(O.ptr(x), O.ptr(s), 1024, 4096)
            L.or_cfg3_max_lastaxis_f32(O.ptr(x), O.ptr(s), 1024, 4096)
            L.or_cfg3_argmax_lastaxis_f32(O.ptr(x), O.ptr(a), 1024, 4096)
            L.or_cfg3_mean_midaxis_f32(O.ptr(x), O.ptr(mean), 1, 1024, 4096)
            done += 1
        el = time.perf_counter() - t0
        return done * 4 * x.nbytes / el / GB, L.or_num_threads(), f"{done} x X[0, :1024, :] for all four ops"


class Config4:
    """LayerNorm over the last axis of [64, 2048, 1024] fp16 + softmax over the last axis of [32, 16, 2048, 2048] fp16."""
    dtype = "f16"

    scaling = "strong"

    def __init__(self, rank, world, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, LNMode
        from tadma_b200.shard import shard_range
        self.tb = tb
        glb = batch or 64
        gsb = max(1, glb // 2)
        ls, ss = shard_range(glb, rank, world), shard_range(gsb, rank, world)
        lb, sb = ls.size, ss.size
        self.name = f"cfg4: LayerNorm [{glb},2048,1024] fp16 + softmax [{gsb},16,2048,2048] fp16 (last axis)"
        self.shard = f"LayerNorm batches {ls.start}:{ls.stop}, softmax batches {ss.start}:{ss.stop}"
        self.x = torch.empty((lb, 2048, 1024), dtype=torch.float16, device="cuda")
        self.g = torch.empty((1024,), dtype=torch.float16, device="cuda")
        self.b = torch.empty((1024,), dtype=torch.float16, device="cuda")
        tb.fill(self.x, Dist.NORMAL, 0.0, 1.0, 0, 1, offset=ls.start * 2048 * 1024)
        tb.fill(self.g, Dist.NORMAL, 1.0, 0.02, 0, 2)
        tb.fill(self.b, Dist.NORMAL, 0.0, 0.02, 0, 3)
        self.y = torch.empty_like(self.x)
        self.s = torch.empty((sb, 16, 2048, 2048), dtype=torch.float16, device="cuda")
        tb.fill(self.s, Dist.NORMAL, 0.0, 3.0, 0, 4, offset=ss.start * 16 * 2048 * 2048)
        self.sy = torch.empty_like(self.s)
        self.bytes = (2 * self.x.numel() * 2 + 2 * 1024 * 2) + 2 * self.s.numel() * 2
        self.launches = 2
        self.units = self.x.numel() + self.s.numel()
        self.calls = [tb.prepare_layer_norm(self.x, -1, self.g, self.b, 1e-5, self.y, LNMode.ONNX),
                      tb.prepare_softmax(self.s, -1, self.sy)]

    def step(self):
        for c in self.calls:
            c()

    def parts(self):
        return [("rownorm_warp_kernel", "LayerNorm (ONNX) rows of 1024", 2 * self.x.numel() * 2 + 2 * 1024 * 2,
                 self.calls[0]),
                ("rownorm_warp_kernel", "softmax rows of 2048", 2 * self.s.numel() * 2, self.calls[1])]

    def cpu_sample(self, budget_s):
        import numpy as np
        from oracle import oracle as O
        L = O.lib()
        xs = self.x.view(-1, 1024)[:4096].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
        g = self.g.view(torch_int16()).cpu().numpy().view(np.uint16)
        b = self.b.view(torch_int16()).cpu().numpy().view(np.uint16)
        ss = self.s.view(-1, 2048)[:2048].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
        y1, y2 = np.zeros_like(xs), np.zeros_like(ss)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            L.or_cfg4_layer_norm_f16(O.ptr(xs), O.ptr(g), O.ptr(b), 1e-5, O.ptr(y1), 4096, 1024)
            L.or_cfg4_softmax_f16(O.ptr(ss), O.ptr(y2), 2048, 2048)
            done += 1
        el = time.perf_counter() - t0
        return done * 2 * (xs.nbytes + ss.nbytes) / el / GB, L.or_num_threads(), f"{done} x (4096 LN rows + 2048 softmax rows)"


class Config5:
    """Embedding gather: table [50257, 4096] fp16, ids [2048, 4096] int64, + pos [4096, 4096] bf16 -> bf16."""
    dtype = "f16/bf16"
    V, B, S, D = 50257, 2048, 4096, 4096

    scaling = "strong"

    def __init__(self, rank, world, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, DType, make_tensor
        from tadma_b200.shard import shard_range
        self.tb = tb
        gb = batch or Config5.B
        sh = shard_range(gb, rank, world)
        self.B = sh.size
        V, B, S, D = self.V, self.B, self.S, self.D
        self.name = f"cfg5: gather table[50257,4096] fp16 by ids[{gb},4096] int64 + pos[4096,4096] bf16 -> bf16"
        self.shard = f"id rows {sh.start}:{sh.stop} of {gb} (table and pos replicated)"
        self.table = torch.empty((V, D), dtype=torch.float16, device="cuda")
        self.ids = torch.empty((B, S), dtype=torch.int64, device="cuda")
        self.pos = torch.empty((S, D), dtype=torch.bfloat16, device="cuda")
        tb.fill(self.table, Dist.NORMAL, 0.0, 0.02, 0, 1)
        tb.fill(self.ids, Dist.INDEX, 0, V, 0, 2, offset=sh.start * S)
        tb.fill(self.pos, Dist.NORMAL, 0.0, 0.02, 0, 3)
        self.out = torch.empty((B, S, D), dtype=torch.bfloat16, device="cuda")
        self.addv = make_tensor(self.pos.data_ptr(), DType.BF16, [B, S, D], [0, D, 1])
        n_out = B * S * D
        self.bytes = B * S * 8 + n_out * 2 + S * D * 2 + n_out * 2
        self.compulsory = B * S * 8 + V * D * 2 + S * D * 2 + n_out * 2
        self.launches = 1
        self.units = n_out
        self.call = tb.prepare_gather(self.table, 0, self.ids, self.out, add=self.addv)

    def step(self):
        self.call()

    def parts(self):
        return [("gather_rows_kernel", "gather + pos add", self.bytes, self.call)]

    def cpu_sample(self, budget_s):
        import numpy as np
        from oracle import oracle as O
        L = O.lib()
        rows = 16
        table = self.table.view(torch_int16()).cpu().numpy().view(np.uint16)
        ids = self.ids[:rows].contiguous().cpu().numpy()
        pos = self.pos.view(torch_int16()).cpu().numpy().view(np.uint16)
        out = np.zeros((rows, self.S, self.D), np.uint16)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            L.or_cfg5_gather_add(O.ptr(table), self.V, O.ptr(ids), O.ptr(pos), O.ptr(out), rows, self.S, self.D)
            done += 1
        el = time.perf_counter() - t0
        per = rows * self.S * 8 + rows * self.S * self.D * 2 * 2 + self.S * self.D * 2
        return done * per / el / GB, L.or_num_threads(), f"{done} x {rows} batch rows of ids[2048, 4096]"


CONFIGS = {1: Config1, 2: Config2, 3: Config3, 4: Config4, 5: Config5}

# ------------------------------------------------- reference GPU algorithm --

REFALGO = os.path.join(ROOT, "baseline", "refalgo", "librefalgo.so")


def time_steps(fn, steps, warmup, stream):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / 1e3 / steps


def ref_gpu(cfg, args, stream):
    """TADMA's own GPU kernels restated with their launch geometry
    (baseline/refalgo/refalgo.cu) on the same device inputs, timed like ours
    and reported against the same algorithmic bytes.  Returns the object for
    the JSON line, or an `unavailable` note."""
    import ctypes
    import torch
    if not os.path.exists(REFALGO):
        return {"unavailable": "baseline/refalgo/librefalgo.so not built"}
    L = ctypes.CDLL(REFALGO)
    st = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    steps = max(3, min(args.steps, 20))
    if isinstance(cfg, Config1):
        if cfg.A.shape[0] != 64:
            return {"unavailable": "restated for the A[64, 128] workload only"}
        t = torch.empty_like(cfg.A)
        y = torch.empty((64,), dtype=torch.float32, device="cuda")
        sec = time_steps(lambda: L.ref_cfg1(P(cfg.A), P(cfg.b), P(t), P(y), st), steps, 2, stream)
        nbytes, launches = cfg.bytes, 3
        note = "A + b node, exp<true> node, sum<-1> through ReduceKernel<128>: 3 launches"
    elif isinstance(cfg, Config2):
        if cfg.ROWS != 8192:
            return {"unavailable": "restated for the full [8192, 8192] workload only"}
        t1 = torch.empty((8192, 8192), dtype=torch.float32, device="cuda")
        t2 = torch.empty_like(t1)
        sec = time_steps(lambda: L.ref_cfg2(P(cfg.x), P(cfg.bias), P(t1), P(t2), st), steps, 2, stream)
        nbytes, launches = cfg.bytes, 3
        note = "x*0.5f -> +bias -> gelu<true>: 3 executor launches with fp32 intermediates (the reference's result type)"
    elif isinstance(cfg, Config3):
        if cfg.x.shape[0] != 32:
            return {"unavailable": "restated for the full X[32, 4096, 4096] workload only"}
        o1 = torch.empty((32, 4096), dtype=torch.float32, device="cuda")
        o2, o3 = torch.empty_like(o1), torch.empty_like(o1)
        sec = time_steps(lambda: L.ref_cfg3(P(cfg.x), P(o1), P(o2), P(o3), st), steps, 2, stream)
        nbytes = 3 * cfg.x.numel() * 4 + 3 * o1.numel() * 4
        launches = 3
        note = "sum<2>, max<2>, mean<1> through ReduceKernel<1024> (the reference has no argmax); bytes of those 3 ops"
    elif isinstance(cfg, Config4):
        if cfg.x.shape[0] != 64:
            return {"unavailable": "restated for the full config-4 workload only"}
        m = torch.empty((64 * 2048,), dtype=torch.float16, device="cuda")
        sd = torch.empty_like(m)
        sums = torch.empty((32 * 16 * 2048,), dtype=torch.float16, device="cuda")
        sx = cfg.s.clone()

        def step():
            L.ref_cfg4_ln(P(cfg.x), P(cfg.g), P(cfg.b), P(m), P(sd), P(cfg.y), st)
            L.ref_cfg4_softmax(P(sx), P(sums), ctypes.c_int64(32 * 16 * 2048), st)
        sec = time_steps(step, steps, 2, stream)
        nbytes, launches = cfg.bytes, 6
        note = "LN: mean reduce, sq-diff reduce, normalise node; softmax: exp node, fp16 sum reduce, divide node"
        del sx
    else:
        B = 64
        if cfg.B < B:
            return {"unavailable": "restated at batch 64; this run has fewer batch rows"}
        ids = cfg.ids[:B].contiguous()
        g = torch.empty((B, 4096, 4096), dtype=torch.float16, device="cuda")
        out = torch.empty((B, 4096, 4096), dtype=torch.float32, device="cuda")
        sec = time_steps(lambda: L.ref_cfg5_b64(P(cfg.table), P(ids), P(cfg.pos), P(g), P(out), st), steps, 2, stream)
        n_out = B * 4096 * 4096
        nbytes = B * 4096 * 8 + n_out * 2 + 4096 * 4096 * 2 + n_out * 2
        launches = 2
        note = ("gather node (256 threads, one element per thread) then + pos node, at batch 64: the reference's "
                "32-bit index cannot address the batch-2048 output; GB/s over the batch-64 algorithmic bytes")
        del g, out
    torch.cuda.synchronize()
    return {"value": round(nbytes / sec / GB, 3), "unit": "GB/s", "ms_per_step": round(sec * 1e3, 4),
            "launches_per_step": launches, "kind": "reference algorithm, restated (baseline/refalgo/refalgo.cu)",
            "note": note}



# --------------------------------------------------------------- reference --

def reference_workload(cfg_id):
    """Host inputs and one step of the reference algorithm (the oracle's C
    loops, OpenMP over rows) on a bounded sample of config `cfg_id`'s
    workload, generated with the GPU arm's seeds.  Returns (name, sample
    description, bytes per step, step function)."""
    import numpy as np
    from oracle import oracle as O
    from tadma_b200.abi import Dist, DType
    L = O.lib()
    if cfg_id == 1:
        A = O.fill((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 0, 1)
        b = O.fill((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 0, 2)
        y = np.zeros((64, 1), np.float32)
        from tadma_b200.abi import Op, Reduce

        def step():
            t = (A + b).astype(np.float32)
            O.reduce(Reduce.SUM, t, -1, y, Op.EXP)
        return ("cfg1: y = sum_last(exp(A + b)), A[64,128] fp32, b[128] fp32 -> [64]", "the whole workload per step",
                64 * 128 * 4 + 128 * 4 + 64 * 4, step)
    if cfg_id == 2:
        rows, C = 1024, Config2.COLS
        x = O.fill((rows, C), DType.BF16, Dist.NORMAL, 0.0, 1.0, 0, 1)
        b = O.fill((C,), DType.BF16, Dist.NORMAL, 0.0, 0.1, 0, 2)
        y = np.zeros_like(x)
        return ("cfg2: y = gelu(x*0.5 + bias), x[8192,8192] bf16, bias[8192] bf16 -> bf16",
                f"{rows} rows of x[8192, 8192] per step", 2 * rows * C * 2 + C * 2,
                lambda: L.or_cfg2_gelu_affine_bf16(O.ptr(x), O.ptr(b), 0.5, O.ptr(y), rows, C))
    if cfg_id == 3:
        rows, C = 1024, 4096
        x = O.fill((rows, C), DType.F32, Dist.UNIFORM, -1.0, 1.0, 0, 1)
        s_, a_, m_ = np.zeros(rows, np.float32), np.zeros(rows, np.int64), np.zeros(C, np.float32)

        def step():
            L.or_cfg3_sum_lastaxis_f32(O.ptr(x), O.ptr(s_), rows, C)
            L.or_cfg3_max_lastaxis_f32(O.ptr(x), O.ptr(s_), rows, C)
            L.or_cfg3_argmax_lastaxis_f32(O.ptr(x), O.ptr(a_), rows, C)
            L.or_cfg3_mean_midaxis_f32(O.ptr(x), O.ptr(m_), 1, rows, C)
        return ("cfg3: sum/max/argmax over axis -1 + mean over axis 1 of X[32,4096,4096] fp32",
                f"X[0, :{rows}, :] for all four ops per step", 4 * x.nbytes, step)
    if cfg_id == 4:
        xs = O.fill((4096, 1024), DType.F16, Dist.NORMAL, 0.0, 1.0, 0, 1)
        g = O.fill((1024,), DType.F16, Dist.NORMAL, 1.0, 0.02, 0, 2)
        bb = O.fill((1024,), DType.F16, Dist.NORMAL, 0.0, 0.02, 0, 3)
        ss = O.fill((2048, 2048), DType.F16, Dist.NORMAL, 0.0, 3.0, 0, 4)
        y1, y2 = np.zeros_like(xs), np.zeros_like(ss)

        def step():
            L.or_cfg4_layer_norm_f16(O.ptr(xs), O.ptr(g), O.ptr(bb), 1e-5, O.ptr(y1), 4096, 1024)
            L.or_cfg4_softmax_f16(O.ptr(ss), O.ptr(y2), 2048, 2048)
        return ("cfg4: LayerNorm [64,2048,1024] fp16 + softmax [32,16,2048,2048] fp16 (last axis)",
                "4096 LayerNorm rows + 2048 softmax rows per step", 2 * (xs.nbytes + ss.nbytes), step)
    if cfg_id == 5:
        V, S, D, rows = Config5.V, Config5.S, Config5.D, 4
        table = O.fill((V, D), DType.F16, Dist.NORMAL, 0.0, 0.02, 0, 1)
        ids = O.fill((rows, S), DType.I64, Dist.INDEX, 0, V, 0, 2)
        pos = O.fill((S, D), DType.BF16, Dist.NORMAL, 0.0, 0.02, 0, 3)
        out = np.zeros((rows, S, D), np.uint16)
        return ("cfg5: gather table[50257,4096] fp16 by ids[2048,4096] int64 + pos[4096,4096] bf16 -> bf16",
                f"{rows} batch rows of ids[2048, 4096] per step", rows * S * 8 + rows * S * D * 2 * 2 + S * D * 2,
                lambda: L.or_cfg5_gather_add(O.ptr(table), V, O.ptr(ids), O.ptr(pos), O.ptr(out), rows, S, D))
    return None


def run_reference(args, rank, world):
    """--impl reference: the reference's algorithm on the host cores (the
    reference itself needs clang >= 19 / C++23 and cannot be built here, so
    its algorithm runs as the oracle's C loops), rank 0 only, on the same
    metric and workload as the GPU arm, a bounded sample per step."""
    if rank != 0:
        return
    from oracle import oracle as O
    L = O.lib()
    # torchrun sets OMP_NUM_THREADS=1 for every rank; this arm runs alone on
    # rank 0 and may use every host thread it is allowed to run on.
    L.or_set_num_threads(len(os.sched_getaffinity(0)))
    wl = reference_workload(args.config)
    if wl is None:
        print(json.dumps({"impl": "reference", "unavailable": f"no reference workload for config {args.config}"}))
        return
    name, sample, per, step = wl
    for _ in range(max(1, args.warmup)):
        step()
    # Each timed step repeats the sample so that the K steps take >= 1.5 s
    # (thread start-up and the first-touch of pages do not dominate), capped
    # so the whole arm ends within a couple of minutes.
    t0 = time.perf_counter()
    step()
    one = max(time.perf_counter() - t0, 1e-6)
    reps = max(1, min(int(-(-1.5 // (one * args.steps))), int(120 // (one * args.steps)) or 1))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(reps):
            step()
    el = time.perf_counter() - t0
    v = per * reps * args.steps / el / GB
    sample = f"{sample}, repeated {reps}x per step"
    cores = L.or_num_threads()
    print(json.dumps({
        "impl": "reference", "metric": "achieved HBM GB/s", "value": round(v, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": CONFIGS[args.config].scaling, "vs_baseline": None,
        "dtype": CONFIGS[args.config].dtype, "data": "synthetic", "config": {"workload": name, "sample": sample},
        "region_s": round(el, 3),
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{sample}, {args.steps} steps"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference (OgnianM/TADMA) needs clang>=19/C++23 and cannot be built here; its algorithm runs as the "
                "oracle's host C loop (oracle/tadma_oracle.c, OpenMP)",
    }))


# -------------------------------------------------------------------- main --

def run_views(args):
    """View copies and single element-wise calls of generated graph code
    (contiguous() after transpose<perm>, concat, casts, residual adds, where,
    comparisons, strided slices) through the public API, each with the torch
    call that does the same.  Every case builds as many independent
    input/output sets as it takes to hold at least twice the L2 (252 MB), and
    one pass over all sets is captured in a CUDA graph and replayed, so no
    launch finds its operands in L2 from the launch before: GB/s = bytes of
    the inputs read once + output written once, over the device time."""
    import torch
    import tadma_b200 as tb
    from tadma_b200.abi import Dist, Op, instr

    side = torch.cuda.Stream()

    def graph_time(fns, launches):
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for f in fns:
                f()
        side.synchronize()
        passes = max(1, -(-20 // len(fns)))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(passes):
                for f in fns:
                    f()
        for _ in range(max(3, args.warmup)):
            g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iters = 10
        s.record()
        for _ in range(iters):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        del g
        return s.elapsed_time(e) / iters / (passes * launches) * 1e-3

    def rnd(shape, dt):
        t = torch.empty(shape, dtype=dt, device="cuda")
        tb.fill(t, Dist.NORMAL, 0, 1, 0, 1)
        return t

    def P(out, ins, prog):
        return tb.prepare_eltwise(out, ins, prog, stream=side)

    f16, f32 = torch.float16, torch.float32

    # Each case: (name, bytes per call, builder).  builder() allocates one
    # independent set and returns (our calls, torch calls) on it.
    def head_split():
        x, y = rnd((32, 512, 16, 64), f16), torch.empty((32, 16, 512, 64), dtype=f16, device="cuda")
        xp = x.permute(0, 2, 1, 3)
        return [P(y, [xp], [instr(Op.COPY)])], [lambda: y.copy_(xp)]

    def kt():
        k, o = rnd((32, 16, 512, 64), f16), torch.empty((32, 16, 64, 512), dtype=f16, device="cuda")
        kp = k.permute(0, 1, 3, 2)
        return [P(o, [kp], [instr(Op.COPY)])], [lambda: o.copy_(kp)]

    def perm0231():
        x, o = rnd((32, 512, 16, 64), f16), torch.empty((32, 16, 64, 512), dtype=f16, device="cuda")
        xp = x.permute(0, 2, 3, 1)
        return [P(o, [xp], [instr(Op.COPY)])], [lambda: o.copy_(xp)]

    def transpose(dt):
        def build():
            a, o = rnd((8192, 8192), dt), torch.empty((8192, 8192), dtype=dt, device="cuda")
            return [P(o, [a.t()], [instr(Op.COPY)])], [lambda: o.copy_(a.t())]
        return build

    def cast():
        a, h = rnd((8192, 8192), f32), torch.empty((8192, 8192), dtype=f16, device="cuda")
        return [P(h, [a], [instr(Op.COPY)])], [lambda: h.copy_(a)]

    def add16():
        a, b, o = rnd((8192, 8192), f16), rnd((8192, 8192), f16), torch.empty((8192, 8192), dtype=f16, device="cuda")
        return [P(o, [a, b], [instr(Op.ADD, b=1)])], [lambda: torch.add(a, b, out=o)]

    def copy32():
        a, o = rnd((8192, 8192), f32), torch.empty((8192, 8192), dtype=f32, device="cuda")
        return [P(o, [a], [instr(Op.COPY)])], [lambda: o.copy_(a)]

    def concat():
        c0, c1 = rnd((32, 512, 1024), f16), rnd((32, 512, 1024), f16)
        cc = torch.empty((32, 1024, 1024), dtype=f16, device="cuda")
        return ([P(cc[:, :512], [c0], [instr(Op.COPY)]), P(cc[:, 512:], [c1], [instr(Op.COPY)])],
                [lambda: torch.cat([c0, c1], 1, out=cc)])

    def where():
        cond = torch.rand((8192, 8192), device="cuda") > 0.5
        a, b, w = rnd((8192, 8192), f32), rnd((8192, 8192), f32), torch.empty((8192, 8192), dtype=f32, device="cuda")
        return [P(w, [cond, a, b], [instr(Op.WHERE, b=1, c=2)])], [lambda: torch.where(cond, a, b, out=w)]

    def greater():
        a, b = rnd((8192, 8192), f32), rnd((8192, 8192), f32)
        gt = torch.empty((8192, 8192), dtype=torch.bool, device="cuda")
        return [P(gt, [a, b], [instr(Op.GT, b=1)])], [lambda: torch.gt(a, b, out=gt)]

    def slice2():
        a, sl = rnd((8192, 8192), f32), torch.empty((4096, 8192), dtype=f32, device="cuda")
        return [P(sl, [a[::2]], [instr(Op.COPY)])], [lambda: sl.copy_(a[::2])]

    n = 8192 * 8192
    hs = 32 * 512 * 16 * 64
    cases = [
        ("head split: permute(0,2,1,3).contiguous() f16 [32,512,16,64]", 4 * hs, head_split),
        ("K^T: permute(0,1,3,2).contiguous() f16 [32,16,512,64]", 4 * hs, kt),
        ("permute(0,2,3,1).contiguous() f16 [32,512,16,64]", 4 * hs, perm0231),
        ("transpose f32 [8192,8192]", 8 * n, transpose(f32)),
        ("transpose f16 [8192,8192]", 4 * n, transpose(f16)),
        ("cast f32 -> f16 [8192,8192]", 6 * n, cast),
        ("add f16 [8192,8192]", 6 * n, add16),
        ("copy f32 [8192,8192]", 8 * n, copy32),
        ("concat axis 1 f16 2 x [32,512,1024]", 4 * 32 * 1024 * 1024, concat),
        ("where(bool, f32, f32) [8192,8192]", 13 * n, where),
        ("greater f32 -> bool [8192,8192]", 9 * n, greater),
        ("slice [::2] f32 [8192,8192] -> [4096,8192]", 8 * n // 2, slice2),
    ]
    for name, nbytes, build in cases:
        if args.view_filter not in name:
            continue
        nsets = max(1, -(-2 * L2_BYTES // nbytes))
        sets = [build() for _ in range(nsets)]
        ours = [f for o, _ in sets for f in o]
        theirs = [f for _, t in sets for f in t]
        per_call = len(sets[0][0])
        t_ours = graph_time(ours, nsets) / 1.0
        t_torch = graph_time(theirs, nsets)
        print(json.dumps({"case": name, "us": round(t_ours * 1e6, 2), "GBs": round(nbytes / t_ours / GB, 1),
                          "torch_GBs": round(nbytes / t_torch / GB, 1), "unit": "GB/s", "sets": nsets,
                          "calls_per_set": per_call}), flush=True)
        del sets, ours, theirs
        torch.cuda.empty_cache()


def run_chain_reduce(args):
    """tadma_b200_reduce_chain on rows of X[32768, 4096] (512 MB fp32, larger
    than L2): the row-operand forms that run on the reduction engine's row
    kernel (row variance, softmax denominator) and chains that need the
    general chain interpreter (a per-column operand, two binary steps).
    GB/s = X read once + the per-row / per-column operand + the output, over
    the average of 20 back-to-back launches."""
    import torch
    import tadma_b200 as tb
    from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, Op, Reduce, instr, make_tensor
    R, C = 32768, 4096
    peak, _ = measured_peak()
    stream = torch.cuda.current_stream()
    for dt, tdt in ((DType.F32, torch.float32), (DType.BF16, torch.bfloat16)):
        x = torch.empty((R, C), dtype=tdt, device="cuda")
        tb.fill(x, Dist.NORMAL, 0.0, 1.0, 0, 1)
        m = torch.empty((R, 1), dtype=torch.float32, device="cuda")
        tb.fill(m, Dist.NORMAL, 0.0, 0.1, 0, 2)
        b = torch.empty((C,), dtype=torch.float32, device="cuda")
        tb.fill(b, Dist.NORMAL, 0.0, 0.1, 0, 3)
        mv = make_tensor(m.data_ptr(), DType.F32, [R, C], [1, 0])
        bv = make_tensor(b.data_ptr(), DType.F32, [R, C], [0, 1])
        out = torch.empty((R, 1), dtype=torch.float32, device="cuda")
        xb = x.numel() * x.element_size()
        cases = [
            ("mean((x - m)^2), m per row", Reduce.MEAN, [x, mv], [instr(Op.SUB, b=1), instr(Op.POW, b=SRC_IMM, imm=2.0)],
             xb + R * 4 + R * 4),
            ("sum(exp(x - m)), m per row", Reduce.SUM, [x, mv], [instr(Op.SUB, b=1), instr(Op.EXP)], xb + R * 8),
            ("sum(x * 0.5)", Reduce.SUM, [x], [instr(Op.MUL, b=SRC_IMM, imm=0.5)], xb + R * 4),
            ("sum(exp(x + b)), b per column (general kernel)", Reduce.SUM, [x, bv], [instr(Op.ADD, b=1), instr(Op.EXP)],
             xb + C * 4 + R * 4),
            ("sum((x - m) * 1.5), m per row (general kernel)", Reduce.SUM, [x, mv],
             [instr(Op.SUB, b=1), instr(Op.MUL, b=SRC_IMM, imm=1.5)], xb + R * 8),
        ]
        for name, op, ins, prog, nbytes in cases:
            call = tb.prepare_reduce_chain(op, ins, prog, -1, out, Compute.F32)
            sec = time_steps(call, 20, 3, stream)
            print(json.dumps({"case": f"{name}, X[{R},{C}] {dt.name.lower()}", "us": round(sec * 1e6, 2),
                              "GBs": round(nbytes / sec / GB, 1), "frac": round(nbytes / sec / GB / peak, 4),
                              "unit": "GB/s"}), flush=True)
        del x
        torch.cuda.empty_cache()


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.views:
        run_views(args)
        return
    if args.chain_reduce:
        run_chain_reduce(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        run(args, rank, world, local)
    finally:
        if world > 1:
            dist.destroy_process_group()


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def time_parts(cfg, args, stream):
    """Each launch of the step timed on its own: n back-to-back launches of
    that call on the launching stream between CUDA events (inputs larger than
    L2, so no launch finds its input cached).  Returns [(kernel, label, bytes,
    seconds per launch)]."""
    n = max(3, min(args.steps, 20))
    out = []
    for kernel, label, nbytes, fn in cfg.parts():
        out.append((kernel, label, nbytes, time_steps(fn, n, 2, stream)))
    return out


def roofline(cid, cfg, args, parts, peak, peak_kind, step_s):
    """Roofline of the dominant launch (the part with the largest time per
    step): achieved = its algorithmic bytes / its average launch duration."""
    rows = []
    for kernel, label, nbytes, sec in parts:
        tr = NCU_TRAFFIC.get((cid, label))
        rows.append({"kernel": kernel, "part": label, "ms": round(sec * 1e3, 4),
                     "achieved": round(nbytes / sec / GB, 1), "frac": round(nbytes / sec / GB / peak, 4),
                     "algorithmic_bytes": nbytes, "traffic": tr["bytes"] if tr else None,
                     "share": round(sec / sum(p[3] for p in parts if not p[1].startswith("compare:")), 4)})
    # Parts labelled "compare:" are alternatives timed beside the step, not in it.
    top = max((r for r in rows if not r["part"].startswith("compare:")), key=lambda r: r["ms"])
    tr = NCU_TRAFFIC.get((cid, top["part"]))
    return {"bound": "hbm", "achieved": top["achieved"], "peak": peak, "unit": "GB/s", "frac": top["frac"],
            "traffic": top["traffic"], "kernel": top["kernel"], "part": top["part"],
            "algorithmic_bytes_per_launch": top["algorithmic_bytes"],
            "traffic_note": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, captured at "
                             f"{tr['captured']}" if tr else "no capture for this part"),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "step": {"achieved": round(cfg.bytes / step_s / GB, 1), "frac": round(cfg.bytes / step_s / GB / peak, 4),
                     "algorithmic_bytes_per_step": cfg.bytes},
            "parts": rows}


def timed_region(cfg, steps, warmup, world, stream, sampler=None):
    """W warm-up steps, then `steps` steps back to back between two CUDA events
    on the launching stream, barrier + synchronize on both sides.  Returns
    (max over ranks of the seconds per step, wall seconds of the region)."""
    import torch
    import torch.distributed as dist
    run = getattr(cfg, "run_steps", None)
    if run:
        run(max(warmup, 3) + getattr(cfg, "nbuf", 0))  # the graph's first replay included
    else:
        for _ in range(max(warmup, 3)):
            cfg.step()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    if sampler:
        sampler.__enter__()
    try:
        start.record(stream)
        if run:
            run(steps)
        else:
            for _ in range(steps):
                cfg.step()
        end.record(stream)
        barrier(world)
    finally:
        if sampler:
            sampler.__exit__(None, None, None)
    region = time.perf_counter() - t0
    t = torch.tensor([start.elapsed_time(end) / 1e3 / steps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), region


def job_total(x, world):
    """Sum over ranks of a per-rank quantity (bytes, elements)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def cross_shard_reduce(cfg3, world, rank, stream):
    """The path's one exchange: X[32, 4096, 4096] of config 3, split by batch,
    summed over axis 0 -- each rank reduces its slab (tadma_b200_reduce), then
    one all-reduce of the [4096, 4096] fp32 partial (NCCL over NVLink at N > 1).
    Timed with CUDA events (max over ranks) and checked on rank 0 at 64 sampled
    positions against a float64 sum of the same elements, regenerated on the
    device from the seeded generator at their global offsets."""
    import torch
    import tadma_b200 as tb
    from tadma_b200.abi import Dist
    from tadma_b200.shard import reduce_leading_axis_sharded
    R = C = 4096
    out = torch.empty((R, C), dtype=torch.float32, device="cuda")

    def step():
        reduce_leading_axis_sharded(cfg3.x, out.view(1, R, C))

    class _Step:
        pass
    st = _Step()
    st.step = step
    n = 5
    sec, _ = timed_region(st, n, 3, world, stream)
    step()
    torch.cuda.synchronize()
    res = {"op": "sum over axis 0 of X[32,4096,4096] fp32, batch-sharded", "bytes_allreduced": R * C * 4,
           "collective": "nccl all_reduce (sum)" if world > 1 else "none (one GPU holds every batch)",
           "ms": round(sec * 1e3, 4), "steps": n}
    if rank == 0:
        g = torch.Generator().manual_seed(7)
        pos = torch.randint(0, R * C, (64,), generator=g).tolist()
        err = 0.0
        col = torch.empty((1,), dtype=torch.float64, device="cuda")
        for p in pos:
            acc = 0.0
            for b in range(cfg3.global_batch):
                tb.fill(col, Dist.UNIFORM, -1.0, 1.0, seed=0, stream_id=1, offset=b * R * C + p)
                acc += float(col.item())
            err = max(err, abs(float(out.view(-1)[p].item()) - acc))
        # fp32 partial sums of 32 values in (-1, 1): far below 1e-4.
        res["check"] = {"positions": len(pos), "max_abs_err": err, "ok": err < 1e-4,
                        "against": "float64 sum of the regenerated elements (seeded generator, global offsets)"}
    return res


def measure(cid, args, rank, world, stream, peak, peak_kind, steps, warmup, sampler=None, headline=False):
    """One config: its timed region, per-launch parts (rank 0), the restated
    reference kernels and the CPU baseline (N = 1, rank 0).  Returns (cfg,
    result dict)."""
    cfg = CONFIGS[cid](rank, world, args.batch)
    step_s, region = timed_region(cfg, steps, warmup, world, stream, sampler)
    total = job_total(cfg.bytes, world)
    units = job_total(cfg.units, world)
    value = total / step_s / GB
    res = {"workload": cfg.name, "value": round(value, 3), "unit": "GB/s", "scaling": cfg.scaling,
           "per_gpu": round(value / world, 3), "frac_per_gpu": round(value / world / peak, 4),
           "ms_per_step": round(step_s * 1e3, 5), "steps": steps, "warmup": max(warmup, 3),
           "elements_per_s": round(units / step_s, 1), "launches_per_step": cfg.launches,
           "shard_rank0": cfg.shard if rank == 0 else None, "region_s": round(region, 4)}
    if hasattr(cfg, "compulsory"):
        res["compulsory_bytes_gbs"] = round(job_total(cfg.compulsory, world) / step_s / GB, 3)
    if hasattr(cfg, "l2_note"):
        res["l2"] = cfg.l2_note
    if hasattr(cfg, "timing_note"):
        res["timing"] = cfg.timing_note
    refg = None
    if world == 1 and not args.no_ref_gpu:
        refg = ref_gpu(cfg, args, stream)
    parts = time_parts(cfg, args, stream) if rank == 0 else None
    barrier(world)
    if rank == 0:
        roof = roofline(cid, cfg, args, parts, peak, peak_kind, step_s)
        res["roofline"] = roof
        res["kernel"] = roof["kernel"]
        res["reference_gpu_restated"] = refg
        if world == 1 and args.cpu_seconds > 0:
            budget = args.cpu_seconds if headline else min(args.cpu_seconds, 3.0)
            v, cores, sample = cfg.cpu_sample(budget)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                                   "sample": sample}
    return cfg, res


def run(args, rank, world, local):
    import torch
    stream = torch.cuda.current_stream()
    peak, peak_kind = measured_peak()
    sampler = ClockSampler(local)
    cfg, head = measure(args.config, args, rank, world, stream, peak, peak_kind, args.steps, args.warmup,
                        sampler=sampler, headline=True)
    e2e = None
    if hasattr(cfg, "e2e"):
        e2e_steps = max(1, min(args.e2e_steps, args.steps))
        e_s, h2d, d2h = cfg.e2e(e2e_steps, stream)
        te = torch.tensor([e_s], dtype=torch.float64, device="cuda")
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        total = job_total(cfg.bytes, world)
        e2e = {"value": round(total / float(te.item()) / GB, 3), "unit": "GB/s",
               "h2d_bytes_per_step": int(job_total(h2d, world)), "d2h_bytes_per_step": int(job_total(d2h, world)),
               "ms_per_step": round(float(te.item()) * 1e3, 4), "steps": e2e_steps,
               "path": "public API from pinned host buffers (tadma_b200.pipeline.RowPipeline, 8 row chunks per rank)"}
    launches = cfg.launches * args.steps
    del cfg
    torch.cuda.empty_cache()

    extras, cross = {}, None
    ids = [c for c in (1, 2, 3, 4, 5) if c != args.config] if not args.no_extras else []
    clocks_all = ClockSampler(local)
    for cid in ids:
        c, r = measure(cid, args, rank, world, stream, peak, peak_kind, EXTRA_STEPS[cid], 3, sampler=clocks_all)
        if cid == 3:
            cross = cross_shard_reduce(c, world, rank, stream)
        extras[f"cfg{cid}"] = r
        del c
        torch.cuda.empty_cache()
        barrier(world)
    if rank != 0:
        return
    line = {
        "metric": "achieved HBM GB/s", "value": head["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None, "dtype": CONFIGS[args.config].dtype,
        "data": ("synthetic, BASELINE.json's distributions: N(mu, sigma) by Box-Muller and U(-1, 1) from a seeded "
                 "counter-based generator (bit-identical on the host), ids U[0, 50257); seed 0"),
        "config": {"workload": head["workload"], "global_batch": "the whole config (BASELINE.json sizes) split "
                   "across the N GPUs on its leading axis" if world > 1 else "the whole config on one GPU",
                   "shard_rank0": head["shard_rank0"],
                   "l2": ("inputs larger than L2, no flush, K steps back to back: " + head.get("l2", "")).strip(),
                   "timing": head.get("timing", "one C-ABI call per step"),
                   "parallelism": f"dp{world} (leading-axis shards, no data-path collective)"},
        "roofline": head["roofline"], "cpu_baseline": head.get("cpu_baseline"), "e2e": e2e,
        "reference_gpu_restated": head.get("reference_gpu_restated"),
        "gpu_launches": launches,
        "clocks": sampler.result(),
        "elements_per_s": head["elements_per_s"],
        "region_s": head["region_s"],
        "configs": extras,
        "cross_shard_reduce": cross,
        "clocks_all_configs": clocks_all.result() if extras else None,
    }
    print(json.dumps(line))


if __name__ == "__main__":
    main()
