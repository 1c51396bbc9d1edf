"""Benchmark of the FP8 QDQ operator path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Default workload (N=1): the FP8 QDQ GEMM of the GEMM sweep at M=N=K=8192 —
one step is QuantizeLinear of the fp32 activation A [M,K] with a dynamic
per-tensor scale (amax(A)/448, computed on the device every step) followed by
the fused FP8 GEMM against the e4m3 weight B [N,K] (DequantizeLinear of both
operands and the output cast folded into the epilogue), bf16 output.
Throughput counts 2*M*N*K FLOP per step. Under torchrun the same 8192^3
problem is split by rows of A across the ranks (strong scaling): a max of
max|A| over the ranks keeps the one-GPU scale, each rank quantizes its rows,
and its GEMM stores its rows of Y into every rank's output over NVLink (the
all-gather fused into the epilogue); a barrier ends the step; time is the
max over ranks. The `tp_gemm` configuration splits the columns instead.

`--impl reference` times the reference algorithm on the host cores instead
(the CPU restatement in oracle/, all threads, bounded sample per step): the
reference's own GPU path needs a graphics API that this machine lacks.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--config", default="gemm8192", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    return p.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name):
    """Per-launch DRAM bytes from the committed ncu summary profiles/<name>.md
    (a line 'traffic_bytes_per_launch: <int>'), or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(path).read())
    return int(m.group(1)) if m else None


class ClockSampler:
    """SM clock and throttle reasons sampled while the timed region runs: an
    NVML polling thread (every 0.5 ms, so even a timed region of a few
    milliseconds gets samples; one sample is taken before the region
    starts), or nvidia-smi -lms 100 when NVML is not importable. Read-only."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.thread = None
        self.lines = []

    def _nvml_index(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if ids and all(v.isdigit() for v in ids) and self.gpu_index < len(ids):
            return int(ids[self.gpu_index])
        return self.gpu_index

    def _poll(self):
        import pynvml
        bits = [("hw_slowdown", pynvml.nvmlClocksEventReasonHwSlowdown),
                ("hw_thermal_slowdown", pynvml.nvmlClocksEventReasonHwThermalSlowdown),
                ("sw_thermal_slowdown", pynvml.nvmlClocksEventReasonSwThermalSlowdown),
                ("sw_power_cap", pynvml.nvmlClocksEventReasonSwPowerCap)]
        while True:
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
                r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            except Exception:
                return
            f = ["Active" if r & b else "Not Active" for _, b in bits]
            self.lines.append(", ".join([str(self.gpu_index), str(sm), str(self.max_sm), "0", hex(r)] + f))
            if self.stop.wait(0.0005):
                return

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self._nvml_index())
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            while not self.lines and self.thread.is_alive():  # first sample before the region starts
                time.sleep(0.0002)
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workloads
class GemmWorkload:
    """QDQ GEMM of the GEMM sweep configuration: each step is the dynamic
    per-tensor QuantizeLinear of the fp32 activation A (s = amax(A) / 448,
    computed on the device every step) and the fused FP8 GEMM against the e4m3
    weight B [N, K] (per-tensor scale), bf16 output.

    Under torchrun (WORLD_SIZE > 1) the same problem is split by rows of A
    (tokens; strong scaling): every rank takes max |A| over its M / N rows,
    one exchange over NVLink (lcml_peer_exchange_max) gives the whole
    tensor's amax, the rank quantizes its rows with the resulting scale (the
    same s as one GPU), and its GEMM against all of B stores each output
    tile into its own full [M, N] output and, over NVLink, into every other
    rank's (the all-gather fused into the epilogue); a barrier exchange after
    the GEMM ends the step. Every rank's Y equals the one-GPU Y bit for bit.
    Splitting rows rather than columns also splits the quantize of A, which
    a column split repeats on every rank. One GPU runs the same kernels with
    no peers."""

    def __init__(self, M, N, K, name):
        self.M, self.N, self.K, self.name = M, N, K, name
        self.ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        # steps of up to 4096^3 are launch-bound: on one GPU their C-ABI calls
        # are replayed as one CUDA graph; 8192^3 and every multi-GPU step run
        # them directly, with the GEMM's events inside the timed step
        self.graph_step = M * N * K <= 4096 ** 3 and self.ws == 1
        self.scaling = "strong" if self.ws > 1 else "weak"
        self.same_input_all_ranks = True
        self.parallelism = (f"M (token) split over {self.ws} ranks: amax exchange, per-rank quantize, GEMM with "
                            "the all-gather of Y fused into its epilogue (P2P stores over NVLink), barrier exchange")

    def describe(self):
        d = {"workload": self.name, "M": self.M, "N": self.N, "K": self.K,
             "a": "fp32 activation; QuantizeLinear with a dynamic per-tensor scale s = amax(A) / 448, amax "
                  "computed on the device every step (two passes over A)",
             "b": "e4m3 weight initializer [N,K] (Gemm transB=1), per-tensor scale", "out": "bf16",
             "l2": "flushed between timed steps (256 MiB write, untimed)",
             "step": ("amax + quantize + GEMM C-ABI calls captured once as a CUDA graph and replayed each step; "
                      "GEMM kernel time from a second loop with CUDA events around the GEMM") if self.graph_step
             else ("amax + quantize + GEMM C-ABI calls each step; GEMM kernel time from a second loop with CUDA "
                   "events around the GEMM")}
        if self.M <= 4:
            d["step"] = ("one kernel (lcml_fp8_gemm_quantize_a: max|A|, QuantizeLinear of A and the GEMV) captured "
                         "once as a CUDA graph and replayed each step; its time from a second loop with CUDA events")
        if self.ws > 1:
            d["rows_per_rank"] = self.rows
            d["step"] = ("amax of the rank's rows, max over the ranks (lcml_peer_exchange_max: one 64-bit NVLink store "
                         "per peer), quantize of the rank's rows, GEMM (rank's rows x all of B) storing into every "
                         "rank's Y; then a barrier (the same exchange without a value) after which every rank holds "
                         "all of Y; GEMM kernel time from a second loop with CUDA events around the GEMM")
        return d

    def setup(self, dev, seed):
        import torch
        import luisaml_b200 as lb
        from luisaml_b200 import tp
        if self.M % self.ws:
            raise SystemExit(f"M = {self.M} rows do not split evenly over {self.ws} ranks")
        self.rows = self.M // self.ws
        self.r0 = self.rank * self.rows
        g = torch.Generator(device=dev).manual_seed(seed)  # the same A on every rank; each uses its rows
        A = torch.randn(self.M, self.K, device=dev, generator=g)
        self.A = A[self.r0:self.r0 + self.rows].clone() if self.ws > 1 else A
        del A
        Bt = tp.column_block_weights(torch, self.K, 0, self.N, dev, seed + 100, 1.0)  # all of B on every rank
        bmax = lb.amax(Bt)
        self.sb = torch.where(bmax > 0, bmax / 448.0, torch.ones_like(bmax))
        self.Bq = lb.quantize(Bt, self.sb)
        del Bt
        self.flops = 2.0 * self.rows * self.N * self.K  # per rank
        self.Aq = torch.empty(self.rows, self.K, dtype=torch.uint8, device=dev)
        self.sa = torch.empty(1, dtype=torch.float32, device=dev)
        self.amax_ws = torch.empty(lb.TENSOR_DYNAMIC_WORKSPACE_BYTES // 4, dtype=torch.float32, device=dev)
        self.peers = None
        if self.ws > 1:
            import torch.distributed as dist
            self.dist = dist
            self.amax_t = torch.zeros(1, dtype=torch.float32, device=dev)  # this rank's rows
            self.amax_g = torch.zeros(1, dtype=torch.float32, device=dev)  # the whole tensor
            self.xchg = tp.PeerExchange(torch, dist, dev)
            self.peers = tp.PeerOutputs(torch, dist, self.M * self.N * 2, dev)
            row_off = self.r0 * self.N * 2  # this rank's rows start here in every rank's Y
            self.peer_rows = (self.peers.peer_array + row_off).contiguous()
            self.barrier_t = torch.zeros(1, device=dev)
            d = lb.GemmDesc()
            d.M, d.N, d.K = self.rows, self.N, self.K
            d.A, d.lda, d.B, d.ldb, d.b_kmajor = self.Aq.data_ptr(), self.K, self.Bq.data_ptr(), self.K, 1
            d.scale_a, d.scale_a_mode = self.sa.data_ptr(), lb.SCALE_TENSOR
            d.scale_b, d.scale_b_mode = self.sb.data_ptr(), lb.SCALE_TENSOR
            d.alpha, d.beta = 1.0, 1.0
            d.Y, d.y_dtype, d.ldy, d.y_col_offset = self.peers.local + row_off, lb.DTYPE_BFLOAT16, self.N, 0
            d.y_peers, d.y_num_peers = self.peer_rows.data_ptr(), self.ws - 1
            self.desc = d
        else:
            self.Y = torch.empty(self.M, self.N, dtype=torch.bfloat16, device=dev)
            self.desc, _ = lb.gemm(self.Aq, self.Bq, self.sa, self.sb, out=self.Y, desc_only=True)
        self.lib = lb.lib()
        self.kernels_per_step = 3

    def step(self, stream, ev=None):
        import ctypes
        import luisaml_b200 as lb
        s = ctypes.c_void_p(stream.cuda_stream)
        if self.ws > 1:  # amax of this rank's rows -> the whole tensor's amax -> s = amax / 448
            lb.check(self.lib.lcml_amax(ctypes.c_void_p(self.A.data_ptr()), self.A.numel(),
                                        ctypes.c_void_p(self.amax_t.data_ptr()), s))
            self.xchg.max(self.amax_t.data_ptr(), self.amax_g.data_ptr(), stream.cuda_stream)
            lb.check(self.lib.lcml_fp8_quantize_from_amax(
                ctypes.c_void_p(self.A.data_ptr()), 1, 1, self.A.numel(), ctypes.c_void_p(self.amax_g.data_ptr()),
                ctypes.c_void_p(self.sa.data_ptr()), ctypes.c_void_p(self.Aq.data_ptr()), s))
        elif self.M <= 4:  # decode: the quantize of A runs inside the GEMV (one kernel per step)
            if ev is not None:
                ev[0].record(stream)
            lb.check(self.lib.lcml_fp8_gemm_quantize_a(
                ctypes.byref(self.desc), ctypes.c_void_p(self.A.data_ptr()), self.K,
                ctypes.c_void_p(self.Aq.data_ptr()), ctypes.c_void_p(self.sa.data_ptr()), None, s))
            if ev is not None:
                ev[1].record(stream)
            return
        else:
            lb.check(self.lib.lcml_fp8_quantize_tensor_dynamic(
                ctypes.c_void_p(self.A.data_ptr()), self.A.numel(), ctypes.c_void_p(self.sa.data_ptr()),
                ctypes.c_void_p(self.Aq.data_ptr()), ctypes.c_void_p(self.amax_ws.data_ptr()), s))
        if ev is not None:
            ev[0].record(stream)
        lb.check(self.lib.lcml_fp8_gemm(ctypes.byref(self.desc), s))
        if ev is not None:
            ev[1].record(stream)
        if self.ws > 1:
            self.xchg.barrier(stream.cuda_stream)  # every rank's rows have landed in every rank's output

    # End to end through the C ABI: every step copies this rank's rows of A in
    # from pinned host memory and its rows of the bf16 Y out to pinned host
    # memory. On one GPU the steps are pipelined over two slots of A and Y:
    # step i's host-to-device copy (one stream) and step i-1's device-to-host
    # copy (another) run while the compute stream quantizes and multiplies,
    # with events keeping each slot's copy, quantize, GEMM and read-back in
    # order (the executor's host-staged I/O does the same for the graphs).
    # Every step still moves all of its bytes; the copies of different steps
    # overlap each other and the compute. Under torchrun, and for steps that
    # copy less than 8 MB, the steps run in sequence on one stream.
    def setup_e2e(self):
        import ctypes
        import torch
        self.A_host = self.A.cpu().pin_memory()  # this rank's rows of A
        self.h2d = self.A_host.numel() * 4
        self.d2h = self.rows * self.N * 2
        # pipelining pays for large copies; a step of a few KB is launch-bound
        # and only gains the extra events and stream waits
        self.pipelined = self.ws == 1 and self.h2d + self.d2h >= (8 << 20)
        if not self.pipelined:
            self.Y_host = torch.empty((self.rows, self.N), dtype=torch.bfloat16).pin_memory()
            return
        dev = self.A.device
        self.e2e_path = ("pinned host A -> H2D (copy stream) -> amax + quantize + GEMM (compute stream) -> D2H of Y "
                         "(second copy stream), two slots, consecutive steps overlapped")
        self.slot_A = [self.A, torch.empty_like(self.A)]
        self.slot_Y = [self.Y, torch.empty_like(self.Y)]
        d2 = type(self.desc)()
        ctypes.memmove(ctypes.byref(d2), ctypes.byref(self.desc), ctypes.sizeof(d2))
        d2.Y = self.slot_Y[1].data_ptr()
        self.slot_desc = [self.desc, d2]
        self.slot_Yh = [torch.empty((self.rows, self.N), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        self.s_in, self.s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev = lambda: [torch.cuda.Event(), torch.cuda.Event()]  # noqa: E731
        self.ev_ready, self.ev_read, self.ev_ydone, self.ev_out = ev(), ev(), ev(), ev()
        self.used = [False, False]
        self.e2e_i = 0

    def e2e_begin(self, stream):
        if getattr(self, "pipelined", False):  # the copy streams start after the timed region's first event
            self.s_in.wait_stream(stream)
            self.s_out.wait_stream(stream)

    def e2e_join(self, stream):
        if getattr(self, "pipelined", False):
            stream.wait_stream(self.s_in)
            stream.wait_stream(self.s_out)

    def step_e2e(self, stream):
        import ctypes
        import luisaml_b200 as lb
        c = lambda p: ctypes.c_void_p(p)  # noqa: E731
        if not self.pipelined:
            self.A.copy_(self.A_host, non_blocking=True)
            self.step(stream)
            ybase = self.peers.local if self.peers is not None else self.Y.data_ptr()
            lb.check(self.lib.lcml_memcpy_async(c(self.Y_host.data_ptr()), c(ybase + self.r0 * self.N * 2),
                                                self.d2h, 2, c(stream.cuda_stream)))
            return
        k = self.e2e_i % 2
        self.e2e_i += 1
        A, desc, Y, Yh = self.slot_A[k], self.slot_desc[k], self.slot_Y[k], self.slot_Yh[k]
        if self.used[k]:  # slot k's A was last read by the quantize of step i-2
            self.s_in.wait_event(self.ev_read[k])
        lb.check(self.lib.lcml_memcpy_async(c(A.data_ptr()), c(self.A_host.data_ptr()), self.h2d, 1,
                                            c(self.s_in.cuda_stream)))
        self.ev_ready[k].record(self.s_in)
        stream.wait_event(self.ev_ready[k])
        s = c(stream.cuda_stream)
        lb.check(self.lib.lcml_fp8_quantize_tensor_dynamic(c(A.data_ptr()), A.numel(), c(self.sa.data_ptr()),
                                                           c(self.Aq.data_ptr()), c(self.amax_ws.data_ptr()), s))
        self.ev_read[k].record(stream)
        if self.used[k]:  # slot k's Y was last read by the device-to-host copy of step i-2
            stream.wait_event(self.ev_out[k])
        lb.check(self.lib.lcml_fp8_gemm(ctypes.byref(desc), s))
        self.ev_ydone[k].record(stream)
        self.s_out.wait_event(self.ev_ydone[k])
        lb.check(self.lib.lcml_memcpy_async(c(Yh.data_ptr()), c(Y.data_ptr()), self.d2h, 2,
                                            c(self.s_out.cuda_stream)))
        self.ev_out[k].record(self.s_out)
        self.used[k] = True

    def close(self):
        if self.peers is not None:
            self.peers.close()
            self.xchg.close()

    def dominant(self):
        if self.M <= 128:  # skinny: streaming B dominates (arithmetic intensity ~2M FLOP/B)
            a_bytes = (4 if self.M <= 4 else 1) * self.M * self.K  # the fused GEMV reads A as fp32
            bytes_ = a_bytes + self.N * self.K + 2 * self.M * self.N
            return {"kernel": "gemv_fp8 (quantize of A fused)" if self.M <= 4 else "gemm_fp8_splitk",
                    "bound": "hbm", "unit": "GB/s",
                    "work": bytes_,
                    "profile": f"gemv_fp8_skinny_{self.M}" if self.M <= 4 else f"gemm_fp8_skinny_{self.M}"}
        # the library's choice (gemm_fp8.cu dispatch): CTA pairs for long K with a 256 x 256 tile for every
        # SM, for every pair when K >= 2048, for every other pair when K >= 4096
        import torch
        pairs = torch.cuda.get_device_properties(self.A.device).multi_processor_count // 2
        pair_tiles = ((self.rows + 255) // 256) * ((self.N + 255) // 256)
        pair = (self.rows >= 256 and self.N >= 256 and self.K >= 1024 and
                (pair_tiles >= 2 * pairs or (self.K >= 2048 and pair_tiles >= pairs) or
                 (self.K >= 4096 and 2 * pair_tiles >= pairs)))
        kern = "gemm_fp8_tc2" if pair else "gemm_fp8_tc"
        if self.ws > 1:
            kern += " (+ fused all-gather)"
        return {"kernel": kern, "bound": "tensor", "unit": "TFLOP/s", "work": self.flops,
                "profile": f"gemm_fp8_tc2_{self.M}"}

    def fp8_anchor(self, dev, steps, flush):
        """The same e4m3 GEMM through the library path torch offers
        (torch._scaled_mm, per-tensor scales, bf16 out), CUDA events per call
        after the same L2 flush: a same-box measure of the dense-FP8 rate."""
        import torch
        try:
            a = self.Aq.view(torch.float8_e4m3fn)
            b = self.Bq.view(torch.float8_e4m3fn).t()
            out = torch._scaled_mm(a, b, scale_a=self.sa, scale_b=self.sb, out_dtype=torch.bfloat16)
        except Exception as e:  # not every torch build has an sm_100 FP8 kernel
            return {"unavailable": f"torch._scaled_mm failed: {type(e).__name__}: {e}"[:200]}
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.fill_(float(i))
            ev[i][0].record()
            torch._scaled_mm(a, b, scale_a=self.sa, scale_b=self.sb, out_dtype=torch.bfloat16, out=out)
            ev[i][1].record()
        torch.cuda.synchronize()
        ms = sum(x.elapsed_time(y) for x, y in ev) / steps
        return {"tflops": 2.0 * self.M * self.N * self.K / (ms / 1e3) / 1e12, "ms": ms,
                "what": "torch._scaled_mm e4m3 x e4m3 -> bf16, per-tensor scales, same operands, CUDA events, "
                        "L2 flushed between calls"}

    # CPU reference: oracle quantize + oracle QDQ GEMM on a bounded row sample
    def cpu_sample(self, budget_s=12.0):
        import numpy as np
        import oracle
        rng = np.random.default_rng(0)
        K, N = self.K, self.N
        if getattr(self, "_cpu_bq", None) is None:
            self._cpu_bq = rng.integers(0, 0x7e, size=(N, K), dtype=np.uint8)
        Bq = self._cpu_bq
        sb = np.float32([0.01])

        def run(rows):
            A = rng.standard_normal((rows, K)).astype(np.float32)
            t0 = time.perf_counter()
            sa = np.float32([oracle.scale_from_amax(oracle.amax(A))])
            Aq = oracle.quantize(A, sa[0])
            oracle.qdq_gemm(Aq, sa, Bq, sb)
            return time.perf_counter() - t0

        t = run(4)
        rows = int(max(4, min(self.M, 4 * budget_s / max(t, 1e-3))))
        t = run(rows)
        return {"value": 2.0 * rows * N * K / t / 1e12, "unit": "TFLOP/s", "cores": oracle.num_threads(),
                "kind": "port",
                "sample": f"{rows} of {self.M} rows of the {self.M}x{self.N}x{self.K} QDQ GEMM "
                          f"(amax + quantize + DQ + K-ordered fp32 fma), {t:.1f} s"}


class GraphWorkload:
    """A benchmark configuration run as an ONNX graph through the C++
    NetworkInstance (lcml_session C ABI): one step = one forward."""

    unit = "TFLOP/s"
    parallelism = "batch split"
    e2e_path = ("pinned host inputs -> NetworkInstance::forward (C ABI) with host-staged I/O: the H2D copy of each "
                "step's input on a second stream (overlapping the previous step once its input readers ran) -> "
                "nodes -> D2H of the outputs on a third stream (overlapping the next step until its writer of the "
                "output runs)")

    def setup_graph(self, dev, text, blob, inputs, outputs):
        import torch
        from luisaml_b200.session import Network
        self.net = Network(text)
        self.blob = torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).to(dev)
        self.net.set_weight_buffer(self.blob)
        self.inputs, self.outputs = inputs, outputs
        for k, t in inputs.items():
            self.net.set_input(k, t)
        for k, t in outputs.items():
            self.net.set_output(k, t)
        self.stream_handle = torch.cuda.current_stream(dev).cuda_stream
        self.net.set_stream(self.stream_handle)
        self.net.forward()  # prepare (weights interleaved, constants uploaded)
        torch.cuda.synchronize()

    def step(self, stream, ev=None):
        if ev is not None:
            ev[0].record(stream)
        self.net.forward()
        if ev is not None:
            ev[1].record(stream)

    def setup_e2e(self):
        import torch
        self.in_host = {k: t.cpu().pin_memory() for k, t in self.inputs.items()}
        self.out_host = {k: torch.empty(t.shape, dtype=t.dtype).pin_memory() for k, t in self.outputs.items()}
        self.h2d = sum(t.numel() * t.element_size() for t in self.in_host.values())
        self.d2h = sum(t.numel() * t.element_size() for t in self.out_host.values())

        for k, t in self.in_host.items():
            self.net.set_input_host(k, t)
        for k, t in self.out_host.items():
            self.net.set_output_host(k, t)
        self.net.set_async_outputs(True)

    def step_e2e(self, stream):
        self.net.forward()  # H2D of the inputs, the nodes, D2H of the outputs

    def e2e_join(self, stream):
        self.net.wait_outputs(stream.cuda_stream)  # the timed region ends after the last output copy


class MlpWorkload(GraphWorkload):
    """the simple MLP graph 784->512->512->10 with QDQ e4m3 weights,
    batch 32 (per rank: replicas)."""
    unit = "inferences/s"

    def __init__(self, batch=32):
        self.batch = batch
        self.flops = 2.0 * batch * (784 * 512 + 512 * 512 + 512 * 10)
        self.work_per_step = batch

    def describe(self):
        return {"workload": "simple_mlp_qdq_784-512-512-10", "batch": self.batch,
                "weights": "e4m3 initializers + DequantizeLinear (per tensor), fp32 activations",
                "path": "LuisaML-JSON graph -> NetworkInstance (DQ of constant weights folded at prepare)",
                "l2": "working set (0.8 MB) stays in L2; L2 flushed between timed steps"}

    def setup(self, dev, seed):
        import torch
        from luisaml_b200 import graphs
        text, blob, _ = graphs.mlp(batch=self.batch)
        x = torch.rand((self.batch, 784), generator=torch.Generator(device=dev).manual_seed(seed), device=dev)
        y = torch.empty((self.batch, 10), dtype=torch.float32, device=dev)
        self.setup_graph(dev, text, blob, {"input": x}, {"output": y})

    def dominant(self):
        return {"kernel": "whole forward (3 kernels)", "bound": "latency", "unit": "TFLOP/s", "work": self.flops,
                "profile": "mlp", "kernel_only": False}

    def cpu_sample(self, budget_s=5.0):
        import oracle
        from luisaml_b200 import graphs
        _, _, meta = graphs.mlp(batch=self.batch)
        x = np.random.default_rng(0).random((self.batch, 784), dtype=np.float32)
        ws = [(oracle.dequantize(L["q"], L["s"][0]), L["bias"]) for L in meta["layers"]]
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s:
            h = x
            for i, (w, bb) in enumerate(ws):
                h = oracle.gemm(h, w, bb, transB=1)
                if i < 2:
                    h = oracle.relu(h)
            n += 1
        t = time.perf_counter() - t0
        return {"value": n * self.batch / t, "unit": "inferences/s", "cores": oracle.num_threads(), "kind": "port",
                "sample": f"{n} forwards of the batch-{self.batch} MLP (fp32 gemm.cpp loop on dequantized weights)"}


class FfnWorkload(GraphWorkload):
    """Llama-style FFN block as an ONNX graph (dynamic per-token QDQ,
    gate/up/down e4m3 weights, SiLU*up, residual, bf16 out). Tokens are split
    across ranks (batch split, no collective)."""

    def __init__(self, tokens=4096, d=4096, f=11008):
        self.T, self.D, self.F = tokens, d, f

    def describe(self):
        return {"workload": f"llama_ffn_qdq_t{self.T}_d{self.D}_f{self.F}",
                "tokens_per_rank": getattr(self, "t_rank", self.T),
                "path": "LuisaML-JSON graph -> NetworkInstance with QDQ fusion (4 kernels per forward)",
                "l2": "inputs larger than L2 (fp32 x and h); L2 flushed between timed steps"}

    def setup(self, dev, seed):
        import torch
        from luisaml_b200 import graphs
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.t_rank = self.T // ws
        self.flops = 2.0 * self.t_rank * self.D * self.F * 3
        text, blob, _ = graphs.ffn(self.t_rank, self.D, self.F)
        x = torch.randn((self.t_rank, self.D), generator=torch.Generator(device=dev).manual_seed(seed), device=dev)
        y = torch.empty((self.t_rank, self.D), dtype=torch.bfloat16, device=dev)
        self.setup_graph(dev, text, blob, {"x": x}, {"y": y})

    def dominant(self):
        return {"kernel": "whole forward (4 kernels)", "bound": "tensor", "unit": "TFLOP/s", "work": self.flops,
                "profile": "ffn", "kernel_only": False}

    def cpu_sample(self, budget_s=12.0):
        import oracle
        rng = np.random.default_rng(0)
        D, F = self.D, self.F
        wg = rng.integers(0, 0x60, size=(F, D), dtype=np.uint8)
        wu = rng.integers(0, 0x60, size=(F, D), dtype=np.uint8)
        wd = rng.integers(0, 0x60, size=(D, F), dtype=np.uint8)
        s = np.full(F, 0.001, np.float32)
        sd = np.full(D, 0.001, np.float32)
        rows = 2
        x = rng.standard_normal((rows, D)).astype(np.float32)
        t0 = time.perf_counter()
        xq, sx = oracle.quantize_dynamic_rows(x)
        h = oracle.silu_mul(oracle.qdq_gemm(xq, sx, wg, s), oracle.qdq_gemm(xq, sx, wu, s))
        hq, sh = oracle.quantize_dynamic_rows(h)
        oracle.qdq_gemm(hq, sh, wd, sd)
        t = time.perf_counter() - t0
        return {"value": 2.0 * rows * D * F * 3 / t / 1e12, "unit": "TFLOP/s", "cores": oracle.num_threads(),
                "kind": "port", "sample": f"{rows} token rows of the FFN (quantize, gate/up, SiLU*up, quantize, down)"}


class TpGemmWorkload:
    """A [16384, 8192] dynamically per-token quantized, B [8192, 28672]
    per-column e4m3, Y bf16 [16384, 28672]. N is split across ranks; each rank's
    GEMM epilogue stores its shard into every rank's output over NVLink
    (fused all-gather, mode "fused") or the shards are all-gathered by NCCL and
    re-laid out (mode "nccl", the library baseline). Strong scaling."""

    unit = "TFLOP/s"
    scaling = "strong"

    def __init__(self, M=16384, K=8192, N=28672, mode=None):
        self.M, self.K, self.N = M, K, N
        self.mode = mode or os.environ.get("LCML_TP_MODE", "fused")
        self.parallelism = ("N split; all-gather fused into the GEMM epilogue (P2P stores over NVLink)"
                            if self.mode == "fused" else "N split; NCCL all-gather + re-layout")
        self.e2e_path = "pinned host A -> H2D -> per-token quantize -> TP GEMM (+ all-gather) -> D2H of this rank's shard"

    def describe(self):
        return {"workload": f"tp_fp8_gemm_{self.M}x{self.N}x{self.K}", "mode": self.mode,
                "shard_columns": self.Nr, "l2": "inputs larger than L2; L2 flushed between timed steps"}

    def setup(self, dev, seed):
        import ctypes
        import torch
        import torch.distributed as dist
        import luisaml_b200 as lb
        from luisaml_b200 import tp
        self.ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.dist = dist
        M, K, N = self.M, self.K, self.N
        start, stop = tp.shard_columns(N, self.ws, self.rank)
        self.start, self.Nr = start, stop - start
        self.flops = 2.0 * M * N * K / self.ws
        self.A = torch.randn((M, K), generator=torch.Generator(device=dev).manual_seed(5000), device=dev)
        Bt = tp.column_block_weights(torch, K, start, stop, dev, 5100, 0.02)
        self.Bq, self.sb = lb.quantize_rows_dynamic(Bt)  # per-column scales of B = per-row of B^T
        del Bt
        self.Aq = torch.empty((M, K), dtype=torch.uint8, device=dev)
        self.sa = torch.empty(M, dtype=torch.float32, device=dev)
        self.peers = None
        if self.ws > 1 and self.mode == "fused":
            self.xchg = tp.PeerExchange(torch, dist, dev)
            self.peers = tp.PeerOutputs(torch, dist, M * N * 2, dev)
            ybase, npeers, peer_arr = self.peers.local, self.ws - 1, self.peers.peer_array.data_ptr()
            ldy, off = N, start
        elif self.ws > 1:
            self.Yr = torch.empty((M, self.Nr), dtype=torch.bfloat16, device=dev)
            self.gathered = torch.empty((self.ws * M * self.Nr,), dtype=torch.bfloat16, device=dev)
            self.Y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            ybase, npeers, peer_arr, ldy, off = self.Yr.data_ptr(), 0, 0, self.Nr, 0
        else:
            self.Y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            ybase, npeers, peer_arr, ldy, off = self.Y.data_ptr(), 0, 0, N, 0
        d = lb.GemmDesc()
        d.M, d.N, d.K = M, self.Nr, K
        d.A, d.lda, d.B, d.ldb, d.b_kmajor = self.Aq.data_ptr(), K, self.Bq.data_ptr(), K, 1
        d.scale_a, d.scale_a_mode, d.scale_b, d.scale_b_mode = self.sa.data_ptr(), lb.SCALE_ROW, self.sb.data_ptr(), lb.SCALE_COL
        d.alpha, d.beta = 1.0, 1.0
        d.Y, d.y_dtype, d.ldy, d.y_col_offset = ybase, lb.DTYPE_BFLOAT16, ldy, off
        d.y_peers, d.y_num_peers = peer_arr, npeers
        self.desc = d
        self.lib = lb.lib()
        self.barrier_t = torch.zeros(1, device=dev)
        self.ctypes = ctypes

    def step(self, stream, ev=None):
        import luisaml_b200 as lb
        c = self.ctypes
        s = c.c_void_p(stream.cuda_stream)
        lb.check(self.lib.lcml_fp8_quantize_rows_dynamic(c.c_void_p(self.A.data_ptr()), self.M, self.K, self.K,
                                                         c.c_void_p(self.sa.data_ptr()), c.c_void_p(self.Aq.data_ptr()), s))
        if ev is not None:
            ev[0].record(stream)
        lb.check(self.lib.lcml_fp8_gemm(c.byref(self.desc), s))
        if ev is not None:
            ev[1].record(stream)
        if self.ws > 1 and self.mode == "fused":
            self.xchg.barrier(stream.cuda_stream)  # every shard has landed in every rank's output
        elif self.ws > 1:
            self.dist.all_gather_into_tensor(self.gathered, self.Yr.reshape(-1))
            self.Y.copy_(self.gathered.view(self.ws, self.M, self.Nr).permute(1, 0, 2).reshape(self.M, self.N))

    def setup_e2e(self):
        import torch
        self.A_host = self.A.cpu().pin_memory()
        self.out_host = torch.empty((self.M, self.Nr), dtype=torch.bfloat16).pin_memory()
        self.h2d = self.A_host.numel() * 4
        self.d2h = self.out_host.numel() * 2

    def step_e2e(self, stream):
        self.A.copy_(self.A_host, non_blocking=True)
        self.step(stream)
        if self.peers is not None:
            import ctypes
            self.lib.lcml_memcpy_async(ctypes.c_void_p(self.out_host.data_ptr()), ctypes.c_void_p(self.peers.local),
                                       self.out_host.numel() * 2, 2, ctypes.c_void_p(stream.cuda_stream))
        else:
            src = self.Y[:, self.start:self.start + self.Nr] if hasattr(self, "Y") else self.Yr
            self.out_host.copy_(src, non_blocking=True)

    def dominant(self):
        return {"kernel": "gemm_fp8_tc2" + (" (+ fused all-gather)" if self.mode == "fused" and self.ws > 1 else ""),
                "bound": "tensor" if self.ws == 1 else "nvlink", "unit": "TFLOP/s", "work": self.flops,
                "profile": "tp_gemm"}

    def cpu_sample(self, budget_s=12.0):
        import oracle
        rng = np.random.default_rng(0)
        K, N = self.K, self.N
        rows = 1
        x = rng.standard_normal((rows, K)).astype(np.float32)
        bq = rng.integers(0, 0x60, size=(N, K), dtype=np.uint8)
        sb = np.full(N, 0.001, np.float32)
        t0 = time.perf_counter()
        xq, sx = oracle.quantize_dynamic_rows(x)
        oracle.qdq_gemm(xq, sx, bq, sb)
        t = time.perf_counter() - t0
        return {"value": 2.0 * rows * N * K / t / 1e12, "unit": "TFLOP/s", "cores": oracle.num_threads(), "kind": "port",
                "sample": f"{rows} row of the {self.M}x{self.N}x{self.K} TP GEMM (quantize + DQ + fma loop)"}

    def close(self):
        if self.peers is not None:
            self.peers.close()
            self.xchg.close()


class ResnetWorkload(GraphWorkload):
    """ResNet-50 v1.5 as a fully quantized QDQ graph at 224x224,
    batch 128 split across the ranks (batch split, no collective): 53 fused
    FP8 conv GEMMs (scales, bias, residual, Relu and requantization in the
    epilogue), e4m3 max pool and global average pool, QDQ classifier."""
    unit = "inferences/s"
    scaling = "strong"
    parallelism = "batch split (no collective)"

    def __init__(self, batch=128, image=224):
        self.total_batch, self.image = batch, image
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.batch = max(1, batch // ws)
        self.work_per_step = self.batch
        self.flop_per_image = None  # known once the graph is built

    def describe(self):
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        return {"workload": f"resnet50_qdq_{self.image}", "batch_per_rank": self.batch,
                "total_batch": self.batch * ws, "flop_per_image": self.flop_per_image,
                "path": "LuisaML-JSON graph -> NetworkInstance: 53 fused FP8 convs, e4m3 pools, QDQ Gemm head",
                "l2": "activations larger than L2; L2 flushed between timed steps"}

    def setup(self, dev, seed):
        import torch
        from luisaml_b200 import graphs
        text, blob, meta = graphs.resnet50(batch=self.batch, image=self.image)
        self.flop_per_image = meta["flop_per_image"]
        self.flops = float(self.flop_per_image) * self.batch
        x = torch.randn((self.batch, 3, self.image, self.image), generator=torch.Generator(device=dev).manual_seed(seed),
                        device=dev)
        y = torch.empty((self.batch, 1000), dtype=torch.float32, device=dev)
        self.setup_graph(dev, text, blob, {"x": x}, {"logits": y})

    def dominant(self):
        return {"kernel": "whole forward", "bound": "tensor", "unit": "TFLOP/s", "work": self.flops,
                "profile": "resnet50", "kernel_only": False}

    def cpu_sample(self, budget_s=15.0):
        import oracle
        from luisaml_b200 import graphs
        _, _, meta = graphs.resnet50(batch=1, image=self.image)
        self.flop_per_image = meta["flop_per_image"]
        x = np.random.default_rng(0).standard_normal((1, 3, self.image, self.image)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s:
            oracle.replay_plan(meta["plan"], x)
            n += 1
        t = time.perf_counter() - t0
        return {"value": n / t, "unit": "inferences/s", "cores": oracle.num_threads(), "kind": "port",
                "sample": f"{n} single-image forwards (QDQ replay: conv.cpp direct loop, pools, gemm.cpp), {t:.1f} s"}


CONFIGS = {
    "resnet50": lambda: ResnetWorkload(),
    "tp_gemm": lambda: TpGemmWorkload(),
    "mlp": lambda: MlpWorkload(),
    "ffn": lambda: FfnWorkload(),
    "gemm8192": lambda: GemmWorkload(8192, 8192, 8192, "qdq_gemm_8192x8192x8192"),
    "gemm4096": lambda: GemmWorkload(4096, 4096, 4096, "qdq_gemm_4096x4096x4096"),
    "gemm2048": lambda: GemmWorkload(2048, 2048, 2048, "qdq_gemm_2048x2048x2048"),
    "gemm1024": lambda: GemmWorkload(1024, 1024, 1024, "qdq_gemm_1024x1024x1024"),
    "skinny1": lambda: GemmWorkload(1, 4096, 4096, "qdq_gemm_1x4096x4096"),
    "skinny16": lambda: GemmWorkload(16, 4096, 4096, "qdq_gemm_16x4096x4096"),
    "skinny128": lambda: GemmWorkload(128, 4096, 4096, "qdq_gemm_128x4096x4096"),
}


# ----------------------------------------------------------------------------- runners
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args, wl):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    samples = []
    budget = max(0.2, 120.0 / (args.steps + args.warmup))  # whole run within a few minutes
    for i in range(args.warmup + args.steps):
        r = wl.cpu_sample(budget_s=budget)
        if i >= args.warmup:
            samples.append(r)
    v = statistics.median(s["value"] for s in samples)
    unit = getattr(wl, "unit", "TFLOP/s")
    metric = METRIC if unit == "TFLOP/s" else f"{wl.describe()['workload']} {unit}"
    line = {"impl": "reference", "metric": metric, "value": v, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 accumulate", "data": "synthetic",
            "config": wl.describe(),
            "cpu_baseline": {"value": v, "unit": unit, "cores": samples[0]["cores"], "kind": "port",
                             "sample": samples[0]["sample"]},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's GPU path (LuisaCompute dx/vk backends) is unavailable on this box; this is "
                    "the reference algorithm restated in C (oracle/) on all host threads"}
    print(json.dumps(line), flush=True)


METRIC = "FP8 QDQ-GEMM TFLOP/s"


def run_ours(args, wl):
    import torch
    import torch.distributed as dist
    import luisaml_b200 as lb

    ws, rank, local = dist_env()
    if ws > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lb.check(lb.lib().lcml_device_check())
    wl.setup(dev, seed=1234 + (0 if getattr(wl, "same_input_all_ranks", False) else rank))
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    for _ in range(args.warmup):
        flush.fill_(1.0)
        wl.step(stream)
    torch.cuda.synchronize()

    # Launch-bound steps (the GEMM sweep) replay the step's C-ABI calls as one
    # CUDA graph: the same kernels on the same buffers, without the host launch
    # latency and the timing events between the kernels. Their dominant-kernel
    # time then comes from a separate loop with events around that kernel.
    graph, graph_launches = None, 0
    if getattr(wl, "graph_step", False):
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        c0 = lb.launch_count()
        with torch.cuda.stream(cs):
            graph.capture_begin()
            wl.step(cs)
            graph.capture_end()
        graph_launches = lb.launch_count() - c0
        stream.wait_stream(cs)
        for _ in range(args.warmup):
            flush.fill_(1.0)
            graph.replay()
        torch.cuda.synchronize()

    n = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lb.launch_count()
    with ClockSampler(local) as clk:
        for i in range(n):
            flush.fill_(float(i))          # evict L2 (untimed: outside the step's events)
            ev[i][0].record(stream)
            if graph is not None:
                graph.replay()
            else:
                wl.step(stream)            # no events inside the step: its kernels overlap as in serving
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        launches = lb.launch_count() - launches0 + graph_launches * n * (graph is not None)
        # dominant-kernel times (not part of `value`): the same steps again with
        # events around the dominant kernel
        for i in range(n):
            flush.fill_(float(i))
            wl.step(stream, kev[i])
        torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    assert lb.device_error() == 0

    unit = getattr(wl, "unit", "TFLOP/s")
    if unit == "TFLOP/s":
        value = wl.flops * n * ws / (total_ms / 1e3) / 1e12
    else:
        value = wl.work_per_step * n * ws / (total_ms / 1e3)
    peaks = measured_peaks()
    dom = wl.dominant()
    kern_avg_s = (sum(kern_ms) / n) / 1e3
    traffic = profile_traffic(dom["profile"])
    if dom["unit"] == "GB/s":
        achieved = dom["work"] / kern_avg_s / 1e9
        peak = peaks["hbm_gbs"]
        peak_source = f"{peaks['source']} HBM copy bandwidth"
    else:
        achieved = dom["work"] / kern_avg_s / 1e12
        peak = 2.0 * peaks["bf16_tflops"]
        peak_source = (f"2 x {peaks['source']} dense bf16 burst ({peaks['bf16_tflops']} TF/s): "
                       "the B200 FP8 dense rate is twice its bf16 rate")
    roofline = {"bound": dom["bound"], "achieved": achieved, "peak": peak, "unit": dom["unit"],
                "frac": achieved / peak, "traffic": traffic, "kernel": dom["kernel"],
                "peak_source": peak_source, "kernel_ms": kern_avg_s * 1e3,
                "timed": "the dominant kernel alone" if dom.get("kernel_only", True) else "the whole step"}

    if ws == 1 and dom["bound"] == "tensor" and hasattr(wl, "fp8_anchor"):
        anchor = wl.fp8_anchor(dev, min(n, 20), flush)
        roofline["fp8_anchor"] = anchor
        if "tflops" in anchor:
            roofline["frac_vs_fp8_anchor"] = achieved / anchor["tflops"]
        roofline["frac_vs_nominal_fp8_dense"] = achieved / 4500.0

    e2e = None
    if not args.no_e2e:
        wl.setup_e2e()
        for _ in range(3):
            wl.step_e2e(stream)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ne = max(10, min(20, n // 10))
        e0.record(stream)
        if hasattr(wl, "e2e_begin"):
            wl.e2e_begin(stream)
        for _ in range(ne):
            wl.step_e2e(stream)
        if hasattr(wl, "e2e_join"):
            wl.e2e_join(stream)
        e1.record(stream)
        torch.cuda.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if ws > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e_t = float(et.item()) / 1e3
        e2e_v = (wl.flops * ne * ws / e2e_t / 1e12) if unit == "TFLOP/s" else (wl.work_per_step * ne * ws / e2e_t)
        e2e = {"value": e2e_v, "unit": unit,
               "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h,
               "path": getattr(wl, "e2e_path", "pinned host inputs -> H2D -> the step's C-ABI calls -> D2H outputs")}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = wl.cpu_sample()

    if rank == 0:
        line = {"metric": METRIC if unit == "TFLOP/s" else f"{wl.describe()['workload']} {unit}", "value": value,
                "unit": unit, "n_gpus": ws, "steps": n,
                "warmup": args.warmup, "ms_per_step": total_ms / n, "higher_is_better": True,
                "scaling": getattr(wl, "scaling", "weak"),
                "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 accumulate, bf16 out", "data": "synthetic",
                "config": wl.describe(), "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches, "clocks": clk.summary(),
                "parallelism": getattr(wl, "parallelism", "replicas") if ws > 1 else "single"}
        print(json.dumps(line), flush=True)
    if hasattr(wl, "close"):
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        wl.close()
    if ws > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    wl = CONFIGS[args.config]()
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
