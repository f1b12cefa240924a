#!/usr/bin/env python3
"""Benchmark of the tadma_b200 hot path (achieved HBM GB/s), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl ours|reference]
    python bench.py --views      # view copies / element-wise calls vs torch, one line per case

Metric: achieved HBM GB/s = algorithmic bytes (every input
read once, every output written once; gathered rows counted per use) / time.
Default workload: config 2, y = gelu(x * 0.5 +
bias), x[8192, 8192] bf16, bias[8192] bf16 -> y bf16, one fused kernel.
Configs 3-5 are selectable for their own lines.

Multi-GPU (torchrun, one process per GPU): every rank processes its own
batch of the config's shape (a shard of an N-times larger global batch,
generated at its global offset), no collective on the data path -> weak
scaling.  Timing: W warm-up steps, then K steps back to back between two CUDA
events on the launching stream, barrier + synchronize on both sides, the max
over ranks reported.  No L2 flush: every step's inputs are larger than L2 and
were not touched by the previous step (config 2 rotates 4 input/output sets).

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
NBUF = 4  # rotating input/output sets of the config-2 workload


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's GPU algorithm (baseline/refalgo) beside ours")
    ap.add_argument("--views", action="store_true",
                    help="instead of a config: one JSON line per view-copy / element-wise case of the generated-graph "
                         "calls (permutes, transposes, casts, concat, where), ours and torch, 1 GPU")
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

    def __init__(self, rank, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Compute, Dist, DType, Op, Reduce, instr, make_tensor
        R = batch or 64
        self.name = f"cfg1: y = sum_last(exp(A + b)), A[{R},128] fp32, b[128] fp32 -> [{R}] (one fused kernel, CUDA graph)"
        self.A = torch.empty((R, 128), dtype=torch.float32, device="cuda")
        self.b = torch.empty((128,), dtype=torch.float32, device="cuda")
        tb.fill(self.A, Dist.NORMAL, 0.0, 1.0, 0, 1, offset=rank * R * 128)
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
        return [("chain_reduce_kernel", "one fused call, CUDA graph replay", self.bytes, self.step),
                ("chain_reduce_kernel", "one fused call, eager", self.bytes, self.eager),
                ("chain_vec_kernel + reduce_row_kernel", "two calls (eltwise, reduce), eager", self.bytes,
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
    """y = gelu(x * 0.5 + bias), x[8192, 8192] bf16, bias[8192] bf16, y bf16."""
    ROWS, COLS = 8192, 8192
    dtype = "bf16"

    def __init__(self, rank, batch=0):
        self.ROWS = batch or Config2.ROWS
        self.name = f"cfg2: y = gelu(x*0.5 + bias), x[{self.ROWS},8192] bf16, bias[8192] bf16 -> bf16"
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, DType, make_tensor
        self.tb = tb
        R, C = self.ROWS, self.COLS
        from tadma_b200.abi import Compute
        self.bias = torch.empty((C,), dtype=torch.bfloat16, device="cuda")
        tb.fill(self.bias, Dist.NORMAL, 0.0, 0.1, seed=0, stream_id=2)
        self.bview = make_tensor(self.bias.data_ptr(), DType.BF16, [R, C], [0, 1])
        self.prog = self.program()
        # NBUF batches (consecutive shards of the global batch) rotate so that
        # no step finds its input in L2: each x is 134 MB > the 126 MB L2.
        self.xs, self.ys, self.calls = [], [], []
        for k in range(NBUF):
            x = torch.empty((R, C), dtype=torch.bfloat16, device="cuda")
            tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=1, offset=(rank * NBUF + k) * R * C)
            y = torch.empty((R, C), dtype=torch.bfloat16, device="cuda")
            self.xs.append(x)
            self.ys.append(y)
            self.calls.append(tb.prepare_eltwise(y, [x, self.bview], self.prog, Compute.F32))
        self.x, self.y, self.i = self.xs[0], self.ys[0], 0
        self.bytes = 2 * R * C * 2 + C * 2
        self.launches = 1
        self.units = R * C

    @staticmethod
    def program():
        from tadma_b200.abi import SRC_IMM, DType, Op, instr
        return [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
                instr(Op.GELU, round_dtype=DType.F32)]

    def step(self):
        self.calls[self.i % NBUF]()
        self.i += 1

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

    def reference_step(self, state):
        from oracle import oracle as O
        x, b, y, rows = state
        O.lib().or_cfg2_gelu_affine_bf16(O.ptr(x), O.ptr(b), 0.5, O.ptr(y), rows, self.COLS)
        return 2 * rows * self.COLS * 2 + self.COLS * 2

    def reference_state(self):
        import numpy as np
        rows = 512
        x = self.x[:rows].contiguous().view(torch_int16()).cpu().numpy().view(np.uint16)
        b = self.bias.view(torch_int16()).cpu().numpy().view(np.uint16)
        return (x, b, np.zeros_like(x), rows), f"512 rows of x[8192, 8192] per step"


def torch_int16():
    import torch
    return torch.int16


class Config3:
    """sum / max / argmax over the last axis and mean over the middle axis of X[32, 4096, 4096] fp32."""
    dtype = "f32"

    def __init__(self, rank, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, Reduce
        self.tb = tb
        B, R, C = batch or 32, 4096, 4096
        self.name = f"cfg3: sum/max/argmax over axis -1 + mean over axis 1 of X[{B},4096,4096] fp32"
        self.x = torch.empty((B, R, C), dtype=torch.float32, device="cuda")
        tb.fill(self.x, Dist.UNIFORM, -1.0, 1.0, seed=0, stream_id=1, offset=rank * B * R * C)
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

    def __init__(self, rank, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, LNMode
        self.tb = tb
        lb = batch or 64
        sb = max(1, lb // 2)
        self.name = f"cfg4: LayerNorm [{lb},2048,1024] fp16 + softmax [{sb},16,2048,2048] fp16 (last axis)"
        self.x = torch.empty((lb, 2048, 1024), dtype=torch.float16, device="cuda")
        self.g = torch.empty((1024,), dtype=torch.float16, device="cuda")
        self.b = torch.empty((1024,), dtype=torch.float16, device="cuda")
        tb.fill(self.x, Dist.NORMAL, 0.0, 1.0, 0, 1, offset=rank * self.x.numel())
        tb.fill(self.g, Dist.NORMAL, 1.0, 0.02, 0, 2)
        tb.fill(self.b, Dist.NORMAL, 0.0, 0.02, 0, 3)
        self.y = torch.empty_like(self.x)
        self.s = torch.empty((sb, 16, 2048, 2048), dtype=torch.float16, device="cuda")
        tb.fill(self.s, Dist.NORMAL, 0.0, 3.0, 0, 4, offset=rank * self.s.numel())
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

    def __init__(self, rank, batch=0):
        import torch
        import tadma_b200 as tb
        from tadma_b200.abi import Dist, DType, make_tensor
        self.tb = tb
        self.B = batch or Config5.B
        V, B, S, D = self.V, self.B, self.S, self.D
        self.name = f"cfg5: gather table[50257,4096] fp16 by ids[{B},4096] int64 + pos[4096,4096] bf16 -> bf16"
        self.table = torch.empty((V, D), dtype=torch.float16, device="cuda")
        self.ids = torch.empty((B, S), dtype=torch.int64, device="cuda")
        self.pos = torch.empty((S, D), dtype=torch.bfloat16, device="cuda")
        tb.fill(self.table, Dist.NORMAL, 0.0, 0.02, 0, 1)
        tb.fill(self.ids, Dist.INDEX, 0, V, 0, 2, offset=rank * B * S)
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
        rows, C = 512, Config2.COLS
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
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    v = per * args.steps / el / GB
    cores = L.or_num_threads()
    print(json.dumps({
        "impl": "reference", "metric": "achieved HBM GB/s", "value": round(v, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": CONFIGS[args.config].dtype,
        "data": "synthetic", "config": {"workload": name, "sample": sample},
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
    call that does the same.  Every call is prepared once and replayed 20x
    from a CUDA graph (no Python in the timed region); GB/s = bytes of the
    inputs read once + output written once, over the device time.  Inputs are
    64-256 MB, some below L2 size: read these as per-launch kernel
    throughput, not as cold-cache figures."""
    import torch
    import tadma_b200 as tb
    from tadma_b200.abi import Dist, Op, instr

    rep, side = 20, torch.cuda.Stream()

    def graph_time(fns, iters=10):
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for f in fns:
                f()
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(rep):
                for f in fns:
                    f()
        for _ in range(max(3, args.warmup)):
            g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        del g
        return s.elapsed_time(e) / iters / rep * 1e-3

    def rnd(shape, dt):
        t = torch.empty(shape, dtype=dt, device="cuda")
        tb.fill(t, Dist.NORMAL, 0, 1, 0, 1)
        return t

    def P(out, ins, prog):
        return tb.prepare_eltwise(out, ins, prog, stream=side)

    f16, f32 = torch.float16, torch.float32
    x = rnd((32, 512, 16, 64), f16)
    y = torch.empty((32, 16, 512, 64), dtype=f16, device="cuda")
    k = rnd((32, 16, 512, 64), f16)
    kt = torch.empty((32, 16, 64, 512), dtype=f16, device="cuda")
    qt = torch.empty((32, 16, 64, 512), dtype=f16, device="cuda")
    a, a16 = rnd((8192, 8192), f32), rnd((8192, 8192), f16)
    at, at16, h = torch.empty_like(a), torch.empty_like(a16), torch.empty_like(a16)
    b16, s16 = rnd((8192, 8192), f16), torch.empty_like(a16)
    c0, c1 = rnd((32, 512, 1024), f16), rnd((32, 512, 1024), f16)
    cc = torch.empty((32, 1024, 1024), dtype=f16, device="cuda")
    cond = torch.rand((8192, 8192), device="cuda") > 0.5
    b2, w, gt = rnd((8192, 8192), f32), torch.empty_like(a), torch.empty_like(cond)
    sl = torch.empty((4096, 8192), dtype=f32, device="cuda")
    xp, kp, qp = x.permute(0, 2, 1, 3), k.permute(0, 1, 3, 2), x.permute(0, 2, 3, 1)
    n = a.numel()
    cases = [
        ("head split: permute(0,2,1,3).contiguous() f16 [32,512,16,64]", 4 * x.numel(),
         [P(y, [xp], [instr(Op.COPY)])], [lambda: y.copy_(xp)]),
        ("K^T: permute(0,1,3,2).contiguous() f16 [32,16,512,64]", 4 * k.numel(),
         [P(kt, [kp], [instr(Op.COPY)])], [lambda: kt.copy_(kp)]),
        ("permute(0,2,3,1).contiguous() f16 [32,512,16,64]", 4 * x.numel(),
         [P(qt, [qp], [instr(Op.COPY)])], [lambda: qt.copy_(qp)]),
        ("transpose f32 [8192,8192]", 8 * n, [P(at, [a.t()], [instr(Op.COPY)])], [lambda: at.copy_(a.t())]),
        ("transpose f16 [8192,8192]", 4 * n, [P(at16, [a16.t()], [instr(Op.COPY)])], [lambda: at16.copy_(a16.t())]),
        ("cast f32 -> f16 [8192,8192]", 6 * n, [P(h, [a], [instr(Op.COPY)])], [lambda: h.copy_(a)]),
        ("add f16 [8192,8192]", 6 * n, [P(s16, [a16, b16], [instr(Op.ADD, b=1)])],
         [lambda: torch.add(a16, b16, out=s16)]),
        ("copy f32 [8192,8192]", 8 * n, [P(at, [a], [instr(Op.COPY)])], [lambda: at.copy_(a)]),
        ("concat axis 1 f16 2 x [32,512,1024]", 4 * cc.numel(),
         [P(cc[:, :512], [c0], [instr(Op.COPY)]), P(cc[:, 512:], [c1], [instr(Op.COPY)])],
         [lambda: torch.cat([c0, c1], 1, out=cc)]),
        ("where(bool, f32, f32) [8192,8192]", 13 * n, [P(w, [cond, a, b2], [instr(Op.WHERE, b=1, c=2)])],
         [lambda: torch.where(cond, a, b2, out=w)]),
        ("greater f32 -> bool [8192,8192]", 9 * n, [P(gt, [a, b2], [instr(Op.GT, b=1)])],
         [lambda: torch.gt(a, b2, out=gt)]),
        ("slice [::2] f32 [8192,8192] -> [4096,8192]", 8 * sl.numel(), [P(sl, [a[::2]], [instr(Op.COPY)])],
         [lambda: sl.copy_(a[::2])]),
    ]
    for name, nbytes, ours, theirs in cases:
        if args.view_filter not in name:
            continue
        t_ours, t_torch = graph_time(ours), graph_time(theirs)
        print(json.dumps({"case": name, "us": round(t_ours * 1e6, 2), "GBs": round(nbytes / t_ours / GB, 1),
                          "torch_GBs": round(nbytes / t_torch / GB, 1), "unit": "GB/s"}), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.views:
        run_views(args)
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


def roofline(cfg, args, parts, peak, peak_kind, step_s):
    """Roofline of the dominant launch (the part with the largest time per
    step): achieved = its algorithmic bytes / its average launch duration."""
    rows = []
    for kernel, label, nbytes, sec in parts:
        tr = NCU_TRAFFIC.get((args.config, label))
        rows.append({"kernel": kernel, "part": label, "ms": round(sec * 1e3, 4),
                     "achieved": round(nbytes / sec / GB, 1), "frac": round(nbytes / sec / GB / peak, 4),
                     "algorithmic_bytes": nbytes, "traffic": tr["bytes"] if tr else None,
                     "share": round(sec / sum(p[3] for p in parts), 4)})
    top = max(rows, key=lambda r: r["ms"])
    tr = NCU_TRAFFIC.get((args.config, top["part"]))
    return {"bound": "hbm", "achieved": top["achieved"], "peak": peak, "unit": "GB/s", "frac": top["frac"],
            "traffic": top["traffic"], "kernel": top["kernel"], "part": top["part"],
            "algorithmic_bytes_per_launch": top["algorithmic_bytes"],
            "traffic_note": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, captured at "
                             f"{tr['captured']}" if tr else "no capture for this part"),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "step": {"achieved": round(cfg.bytes / step_s / GB, 1), "frac": round(cfg.bytes / step_s / GB / peak, 4),
                     "algorithmic_bytes_per_step": cfg.bytes},
            "parts": rows}


def run(args, rank, world, local):
    import torch
    import torch.distributed as dist
    cfg = CONFIGS[args.config](rank, args.batch)
    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        cfg.step()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    t_region = time.perf_counter()
    with sampler:
        start.record(stream)
        for _ in range(args.steps):
            cfg.step()
        end.record(stream)
        barrier(world)
    region_s = time.perf_counter() - t_region
    step_s = start.elapsed_time(end) / 1e3 / args.steps
    t = torch.tensor([step_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_max = float(t.item())
    value = cfg.bytes * world / step_max / GB

    e2e = None
    if hasattr(cfg, "e2e"):
        e2e_steps = max(1, min(args.e2e_steps, args.steps))
        e_s, h2d, d2h = cfg.e2e(e2e_steps, stream)
        te = torch.tensor([e_s], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": round(cfg.bytes * world / float(te.item()) / GB, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(float(te.item()) * 1e3, 4),
               "steps": e2e_steps}
    refg = None
    if world == 1 and not args.no_ref_gpu:
        refg = ref_gpu(cfg, args, stream)
    parts = time_parts(cfg, args, stream) if rank == 0 else None
    barrier(world)
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    roof = roofline(cfg, args, parts, peak, peak_kind, step_s)
    cpu = None
    if world == 1 and args.cpu_seconds > 0:
        v, cores, sample = cfg.cpu_sample(args.cpu_seconds)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
    line = {
        "metric": "achieved HBM GB/s", "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(step_max * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg.dtype,
        "data": "synthetic (seeded counter-based generator, BASELINE.json distributions)",
        "config": {"workload": cfg.name, "per_gpu_batch": "one full config batch per GPU (global batch = N x)",
                   "l2": "inputs larger than L2: every step reads > 126 MB of input not touched by the previous "
                         "step (config 2 rotates 4 x/y sets of 134 MB each); no flush; K steps timed back to back",
                   "parallelism": f"dp{world} (leading-axis shards, no data-path collective)"},
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "reference_gpu_restated": refg,
        "gpu_launches": cfg.launches * args.steps,
        "clocks": sampler.result(),
        "elements_per_s": round(cfg.units * world / step_max, 1),
        "region_s": round(region_s, 4),
    }
    if hasattr(cfg, "compulsory"):
        line["compulsory_bytes_gbs"] = round(cfg.compulsory * world / step_max / GB, 3)
    print(json.dumps(line))


if __name__ == "__main__":
    main()
