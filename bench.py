"""Benchmark: emitted sm_100a kernels on the benchmark workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config rowops|sum|bigsum|matmul|attention|pointwise]
    python bench.py --impl reference ...       # the reference's CPU path (bounded sample, <= ~90 s)

A step is one pass of the hot path over one batch of synthetic input:

  rowops  (default) fused row ops on f32 [8192, 4096] N(0,1): row softmax,
          RMSNorm (eps 1e-6, w ~ U[0.5, 1.5)) and row L2-normalise -- three
          kernels compiled by compile.py from IR in emmy's one-row-per-CTA
          schedule, each on its own input matrix (3 x 128 MiB of inputs,
          larger than the 126 MB L2, so no step reads another's data from L2);
          N GPUs each run their own [8192, 4096] matrices (weak scaling).
  sum     r01-style single-kernel sum of f32[1,048,576] U[-1, 1).
  bigsum  f32[2^30] U[-1, 1) split into contiguous slices over N GPUs: one
          two-pass grid-reduction kernel per GPU, then an NCCL all-reduce of
          the per-GPU partials.
  matmul  f16 C = A B (B column-major), f32 out: 4096^3 and 8192x3072x1024 on
          the tcgen05 matmul family; N GPUs run replicas (weak scaling).
  attention  softmax(Q K^T / sqrt(d)) V, f16 [8, 16, 2048, 128] on the tcgen05
          attention family; the 128 (batch, head) units split over N GPUs.
  pointwise  relu(x0) * x1 on f32[2^28] in the p03 schedule (vectorised
          pointwise family); N GPUs run replicas.

value is the whole-job algorithmic HBM bandwidth (bytes the workload must
move / max-over-ranks device time of the K steps, CUDA events on the launch
stream).  e2e is the same metric through the runner's host-buffer C ABI call
(thr_run), host <-> device copies from pinned memory included.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "thompiler-emmy-hackathon_b200"))
sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_traffic(name: str, tag: str = ""):
    """dram bytes per launch from the committed ncu summary of this kernel, if any: the line
    ``dram_bytes_per_launch: B`` (or ``dram_bytes_per_launch[tag]: B`` for one of several shapes)."""
    f = ROOT / "profiles" / f"{name}.md"
    if not f.exists():
        return None
    key = f"dram_bytes_per_launch[{tag}]:" if tag else "dram_bytes_per_launch:"
    for line in f.read_text().splitlines():
        if line.strip().startswith(key):
            return int(line.split(":")[1].strip().replace(",", ""))
    return None


# ---- clocks ---------------------------------------------------------------------

class ClockSampler:
    """SM clock and throttle reasons sampled every 10 ms from NVML on a background
    thread while the timed region runs (``nvidia-smi``'s own polling is too coarse
    for a sub-second region); the first sample is taken before ``start`` returns."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, gpu: int):
        import threading
        self.samples: list[tuple[int, int, int]] = []
        self.stop_flag = threading.Event()
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self._physical(gpu))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._sample()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception as e:  # no NVML: report that instead of clocks
            self.error, self.thread = f"nvml unavailable: {e}", None

    @staticmethod
    def _physical(gpu: int) -> int:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x for x in vis.split(",") if x.strip()]
        return int(ids[gpu]) if gpu < len(ids) and ids[gpu].strip().isdigit() else gpu

    def _sample(self) -> None:
        nv = self.nv
        self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM),
                             nv.nvmlDeviceGetCurrentClocksEventReasons(self.h), 0))

    def _run(self) -> None:
        while not self.stop_flag.wait(0.01):
            try:
                self._sample()
            except Exception:
                break

    def stop(self) -> dict:
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error]}
        self.stop_flag.set()
        self.thread.join(timeout=5)
        self._sample()
        sm = [s[0] for s in self.samples]
        reasons = sorted({n for s in self.samples for n, bit in self.REASONS.items() if s[1] & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml, 10 ms"}


# ---- workloads -----------------------------------------------------------------------

class RowOps:
    name = "rowops"
    metric = "achieved HBM GB/s (fused row ops: softmax + RMSNorm + L2-norm)"
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, rank: int, world: int, dev: int, rows: int = 8192, cols: int = 4096):
        import torch
        from thompiler import synth
        from thompiler.device import DeviceKernel
        self.torch, self.rows, self.cols, self.eps, self.dev, self.world = torch, rows, cols, 1e-6, dev, world
        tmp = Path(tempfile.mkdtemp(prefix=f"bench_rowops_{rank}_"))
        self.kinds = ("softmax", "rmsnorm", "l2norm")
        self.k = {}
        for kind in self.kinds:
            d = synth.row_package(tmp / kind, kind, rows, cols, eps=self.eps)
            meta = json.loads((d / "meta.json").read_text())
            self.k[kind] = DeviceKernel(d / f"{meta['kernels'][0]['entry']}.ir.json", device=dev)
        g = torch.Generator(device=f"cuda:{dev}").manual_seed(1000 + rank)
        self.x = {kind: torch.randn(rows, cols, device=f"cuda:{dev}", generator=g) for kind in self.kinds}
        self.y = {kind: torch.empty(rows, cols, device=f"cuda:{dev}") for kind in self.kinds}
        self.w = torch.rand(cols, device=f"cuda:{dev}", generator=g) + 0.5
        self.c_count = torch.tensor([float(cols)], device=f"cuda:{dev}")
        self.c_eps = torch.tensor([self.eps], device=f"cuda:{dev}")
        self.kbytes = {"softmax": 2 * rows * cols * 4, "l2norm": 2 * rows * cols * 4,
                       "rmsnorm": 2 * rows * cols * 4 + cols * 4}
        self.bytes_per_step = sum(self.kbytes.values())
        self.launches_per_step = 3
        self.dominant = "softmax"

    def ptrs(self, kind: str) -> dict:
        p = {"x": self.x[kind].data_ptr()}
        out = {"softmax": "softmax", "rmsnorm": "mul_1", "l2norm": "div"}[kind]
        p[out] = self.y[kind].data_ptr()
        if kind == "rmsnorm":
            p.update(w=self.w.data_ptr(), mean_count=self.c_count.data_ptr(), add_c1=self.c_eps.data_ptr())
        return p

    def step(self, stream: int, events=None) -> None:
        for i, kind in enumerate(self.kinds):
            if events is not None:
                events[kind][0].record()
            self.k[kind](self.ptrs(kind), stream)
            if events is not None:
                events[kind][1].record()

    def check(self) -> None:
        torch = self.torch
        self.step(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        x, y = self.x["softmax"], self.y["softmax"]
        ref = torch.softmax(x.double(), -1)
        assert torch.allclose(y.double(), ref, rtol=1e-5, atol=1e-6), "softmax mismatch"
        x, y = self.x["rmsnorm"], self.y["rmsnorm"]
        ref = x.double() / torch.sqrt((x.double() ** 2).mean(-1, keepdim=True) + self.eps) * self.w.double()
        assert torch.allclose(y.double(), ref, rtol=1e-5, atol=1e-5), "rmsnorm mismatch"
        x, y = self.x["l2norm"], self.y["l2norm"]
        ref = x.double() / torch.sqrt((x.double() ** 2).sum(-1, keepdim=True))
        assert torch.allclose(y.double(), ref, rtol=1e-5, atol=1e-6), "l2norm mismatch"

    def e2e(self, steps: int) -> dict:
        """Host-buffer path (thr_run): each step copies inputs in and results out."""
        from thompiler import runner
        torch = self.torch
        host = {}
        for kind in self.kinds:
            hx = torch.empty(self.rows, self.cols, pin_memory=True)
            hx.copy_(self.x[kind])
            hy = torch.empty(self.rows, self.cols, pin_memory=True)
            host[kind] = (hx.numpy(), hy.numpy())
        hw = torch.empty(self.cols, pin_memory=True)
        hw.copy_(self.w)
        consts = {"mean_count": torch.tensor([float(self.cols)]).numpy(), "add_c1": torch.tensor([self.eps]).numpy()}

        def args(kind):
            k = self.k[kind]
            out = []
            for n in k.arg_order:
                if n == "x":
                    out.append({"array": host[kind][0]})
                elif n == "w":
                    out.append({"array": hw.numpy()})
                elif n in consts:
                    out.append({"array": consts[n]})
                else:
                    out.append({"array": host[kind][1], "output": True})
            return out

        runs = {kind: args(kind) for kind in self.kinds}
        for kind in self.kinds:                 # warm the runner's buffers
            runner.run(self.k[kind].fn, self.k[kind].plan, runs[kind])
        t = time.perf_counter()
        for _ in range(steps):
            for kind in self.kinds:
                r = runner.run(self.k[kind].fn, self.k[kind].plan, runs[kind])
                if not r["ok"]:
                    raise RuntimeError(r["stderr"])
        sec_single = (time.perf_counter() - t) / steps
        # the three requests of a step as one thr_run_batch: copies in, kernels and copies out overlap
        batch = [(self.k[kind].fn, self.k[kind].plan, runs[kind], self.k[kind].arg_order) for kind in self.kinds]
        r = runner.run_batch(batch)
        if not r["ok"]:
            raise RuntimeError(r["stderr"])
        ref = torch.softmax(torch.from_numpy(host["softmax"][0][:4]).double(), -1)
        assert torch.allclose(torch.from_numpy(host["softmax"][1][:4]).double(), ref, rtol=1e-5, atol=1e-6)
        t = time.perf_counter()
        for _ in range(steps):
            r = runner.run_batch(batch)
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
        sec_three = (time.perf_counter() - t) / steps
        runner.release()
        # the same step as 1024-row requests (the same row kernels compiled for 1024 rows), prepared
        # once: one thr_run_batch of 3 x 8 requests per step, so each direction's copies stream back
        # to back while the kernels run
        chunk = self.E2E_CHUNK_ROWS
        kch = self._chunk_kernels(chunk)
        creqs = []
        for kind in self.kinds:
            for r0 in range(0, self.rows, chunk):
                a = []
                for n in kch[kind].arg_order:
                    if n == "x":
                        a.append({"array": host[kind][0][r0:r0 + chunk]})
                    elif n == "w":
                        a.append({"array": hw.numpy()})
                    elif n in consts:
                        a.append({"array": consts[n]})
                    else:
                        a.append({"array": host[kind][1][r0:r0 + chunk], "output": True})
                creqs.append((kch[kind].fn, kch[kind].plan, a, kch[kind].arg_order))
        for kind in self.kinds:
            host[kind][1][...] = 0
        prepared = runner.PreparedBatch(creqs)
        r = prepared.run()
        if not r["ok"]:
            raise RuntimeError(r["stderr"])
        for kind, fn in (("softmax", lambda x: torch.softmax(x, -1)),
                         ("l2norm", lambda x: x / torch.sqrt((x * x).sum(-1, keepdim=True)))):
            rows = [0, chunk - 1, chunk, self.rows - 1]
            xr = torch.from_numpy(host[kind][0][rows]).double()
            assert torch.allclose(torch.from_numpy(host[kind][1][rows]).double(), fn(xr), rtol=1e-5, atol=1e-6), kind
        t = time.perf_counter()
        for _ in range(steps):
            r = prepared.run()
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
        sec = (time.perf_counter() - t) / steps
        runner.release()
        for k in kch.values():
            k.close()
        h2d = sum(h[0].nbytes for h in host.values()) + hw.numel() * 4 + 8
        d2h = sum(h[1].nbytes for h in host.values())
        # the device-API pipeline for comparison (one GPU only: it pins another 768 MB of host memory)
        streamed = self.e2e_streamed(steps) if self.world == 1 else None
        out = {"value": self.bytes_per_step / sec / 1e9, "unit": "GB/s", "work": self.bytes_per_step,
               "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": sec * 1e3,
               "how": f"one thr_run_batch per step on pinned host buffers (the C-ABI host-buffer call, its "
                      f"descriptors prepared once), the three row ops as {3 * self.rows // chunk} requests of "
                      f"{chunk} rows each: copies in, kernels and copies out overlap on three streams",
               "three_requests": {"value": self.bytes_per_step / sec_three / 1e9, "ms_per_step": sec_three * 1e3},
               "one_thr_run_per_kernel": {"value": self.bytes_per_step / sec_single / 1e9,
                                          "ms_per_step": sec_single * 1e3}}
        if streamed is not None:
            out["streamed_device_api"] = {
                "value": streamed["value"], "ms_per_step": streamed["ms_per_step"],
                "how": "DeviceKernel launches on device buffers; per 1024-row chunk a host->device copy, "
                       "the kernel and a device->host copy on three streams, so both copy directions "
                       "and the kernels overlap"}
        return out

    E2E_CHUNK_ROWS = 1024

    def _chunk_kernels(self, chunk_rows: int) -> dict:
        """The three row kernels compiled for [chunk_rows, cols] (one CTA per row, as the full ones)."""
        from thompiler import synth
        from thompiler.device import DeviceKernel
        tmp = Path(tempfile.mkdtemp(prefix="bench_rowops_chunk_"))
        kch = {}
        for kind in self.kinds:
            d = synth.row_package(tmp / kind, kind, chunk_rows, self.cols, eps=self.eps)
            meta = json.loads((d / "meta.json").read_text())
            kch[kind] = DeviceKernel(d / f"{meta['kernels'][0]['entry']}.ir.json", device=self.dev)
        return kch

    def e2e_streamed(self, steps: int, chunk_rows: int = 1024) -> dict:
        """The same three row ops on host data, chunked by rows and pipelined on three streams
        (copy in, compute, copy out); each step copies every input in and every result out."""
        torch = self.torch
        nch = self.rows // chunk_rows
        kch = self._chunk_kernels(chunk_rows)
        xh = {k: torch.empty(self.rows, self.cols, pin_memory=True) for k in self.kinds}
        yh = {k: torch.empty(self.rows, self.cols, pin_memory=True) for k in self.kinds}
        for k in self.kinds:
            xh[k].copy_(self.x[k])
        wh = torch.empty(self.cols, pin_memory=True)
        wh.copy_(self.w)
        wd = torch.empty_like(self.w)
        outname = {"softmax": "softmax", "rmsnorm": "mul_1", "l2norm": "div"}
        s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev_k, ev_o = {}, {}

        def ptrs(kind, c):
            r0 = c * chunk_rows
            p_ = {"x": self.x[kind][r0].data_ptr(), outname[kind]: self.y[kind][r0].data_ptr()}
            if kind == "rmsnorm":
                p_.update(w=wd.data_ptr(), mean_count=self.c_count.data_ptr(), add_c1=self.c_eps.data_ptr())
            return p_

        def one_step():
            with torch.cuda.stream(s_in):
                wd.copy_(wh, non_blocking=True)
            for kind in self.kinds:
                for c in range(nch):
                    r0, r1, key = c * chunk_rows, (c + 1) * chunk_rows, (kind, c)
                    with torch.cuda.stream(s_in):
                        if key in ev_k:
                            s_in.wait_event(ev_k[key])          # the last kernel on this chunk has read x
                        self.x[kind][r0:r1].copy_(xh[kind][r0:r1], non_blocking=True)
                        e_in = torch.cuda.Event()
                        e_in.record(s_in)
                    s_cmp.wait_event(e_in)
                    if key in ev_o:
                        s_cmp.wait_event(ev_o[key])             # the last copy-out of this chunk is done
                    kch[kind](ptrs(kind, c), s_cmp.cuda_stream)
                    e_k = torch.cuda.Event()
                    e_k.record(s_cmp)
                    ev_k[key] = e_k
                    s_out.wait_event(e_k)
                    with torch.cuda.stream(s_out):
                        yh[kind][r0:r1].copy_(self.y[kind][r0:r1], non_blocking=True)
                        e_o = torch.cuda.Event()
                        e_o.record(s_out)
                        ev_o[key] = e_o

        one_step()
        torch.cuda.synchronize()
        ref = torch.softmax(xh["softmax"][:4].double(), -1)
        assert torch.allclose(yh["softmax"][:4].double(), ref, rtol=1e-5, atol=1e-6), "streamed softmax mismatch"
        t = time.perf_counter()
        for _ in range(steps):
            one_step()
        torch.cuda.synchronize()
        sec = (time.perf_counter() - t) / steps
        for k in kch.values():
            k.close()
        h2d = sum(x.numel() * 4 for x in xh.values()) + wh.numel() * 4
        d2h = sum(y.numel() * 4 for y in yh.values())
        return {"value": self.bytes_per_step / sec / 1e9, "ms_per_step": sec * 1e3, "h2d": h2d, "d2h": d2h}

    def cpu_baseline(self) -> dict:
        from oracle import cpu_baseline
        rows = 1024
        r = cpu_baseline.rowops_sample(rows, self.cols, self.eps)
        bytes_sample = self.bytes_per_step * rows / self.rows
        return {"value": bytes_sample / r["seconds"] / 1e9, "unit": "GB/s", "cores": r["cores"], "kind": "port",
                "sample": f"torch CPU softmax + RMSNorm + L2-norm on f32[{rows}, {self.cols}] (1/8 of a step), "
                          "best of 3"}

    def details(self, world: int) -> dict:
        return {"workload": f"fused row ops f32[{self.rows}, {self.cols}] x3 (softmax, rmsnorm eps=1e-6, l2norm), "
                            "one row per CTA", "rows_per_gpu": self.rows, "cols": self.cols,
                "kernels": {k: self.k[k].family for k in self.kinds},
                "l2": "inputs larger than L2 (3 x 128 MiB distinct input matrices per GPU)",
                "parallelism": f"weak: {world} GPU(s), one matrix set each, no collective"}


class Pointwise:
    """relu(x0) * x1 over f32[2^28] (the p03 schedule: 4 elements per thread, 1 GiB per operand,
    3 GiB per step, larger than L2); N GPUs run replicas."""
    name = "pointwise"
    metric = "achieved HBM GB/s (pointwise relu(x0) * x1, f32)"
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, rank: int, world: int, dev: int, n: int = 0):
        import torch
        from thompiler import synth
        from thompiler.device import DeviceKernel
        self.torch, self.n, self.dev = torch, n or 1 << 28, dev
        d = synth.pointwise_package(Path(tempfile.mkdtemp(prefix=f"bench_pw_{rank}_")) / "pw", self.n, "relu_mul")
        self.k = DeviceKernel(d / "k_mul_pointwise.ir.json", device=dev)
        g = torch.Generator(device=f"cuda:{dev}").manual_seed(4000 + rank)
        self.x0 = torch.randn(self.n, device=f"cuda:{dev}", generator=g)
        self.x1 = torch.randn(self.n, device=f"cuda:{dev}", generator=g)
        self.y = torch.empty(self.n, device=f"cuda:{dev}")
        self.kinds = ("pointwise",)
        self.kbytes = {"pointwise": 12 * self.n}
        self.bytes_per_step = 12 * self.n
        self.launches_per_step = 1
        self.dominant = "pointwise"

    def ptrs(self) -> dict:
        return {"x0": self.x0.data_ptr(), "x1": self.x1.data_ptr(), "mul": self.y.data_ptr()}

    def step(self, stream: int, events=None) -> None:
        if events is not None:
            events["pointwise"][0].record()
        self.k(self.ptrs(), stream)
        if events is not None:
            events["pointwise"][1].record()

    def check(self) -> None:
        torch = self.torch
        self.step(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert torch.equal(self.y, torch.relu(self.x0) * self.x1), "pointwise mismatch"

    def e2e(self, steps: int) -> dict:
        from thompiler import runner
        torch = self.torch
        m = min(self.n, 1 << 26)                   # host copies of 3 x 256 MiB per step
        h = [torch.empty(m, pin_memory=True) for _ in range(3)]
        h[0].copy_(self.x0[:m])
        h[1].copy_(self.x1[:m])
        from thompiler import synth
        d = synth.pointwise_package(Path(tempfile.mkdtemp(prefix="bench_pw_e2e_")) / "pw", m, "relu_mul")
        from thompiler.device import DeviceKernel
        k = DeviceKernel(d / "k_mul_pointwise.ir.json", device=self.dev)
        args = [{"array": h[0].numpy()}, {"array": h[1].numpy()}, {"array": h[2].numpy(), "output": True}]
        runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
        t = time.perf_counter()
        for _ in range(steps):
            r = runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
        sec = (time.perf_counter() - t) / steps
        runner.release()
        k.close()
        return {"value": 12 * m / sec / 1e9, "unit": "GB/s", "work": 12 * m, "h2d_bytes_per_step": 8 * m,
                "d2h_bytes_per_step": 4 * m, "ms_per_step": sec * 1e3, "elements": m}

    def cpu_baseline(self) -> dict:
        from oracle import cpu_baseline
        r = cpu_baseline.pointwise_sample(1 << 24)
        return {"value": 12 * (1 << 24) / r["seconds"] / 1e9, "unit": "GB/s", "cores": r["cores"],
                "kind": "port", "sample": "torch CPU relu(x0) * x1 on f32[2^24], best of 3"}

    def reference_lowering(self) -> dict:
        """The same IR through the statement-by-statement lowering (scalar 4-byte accesses)."""
        from thompiler.device import DeviceKernel
        torch = self.torch
        gk = DeviceKernel(self.k.ir_path, device=self.dev, tuned=False)
        s = torch.cuda.current_stream().cuda_stream
        for _ in range(3):
            gk(self.ptrs(), s)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(20):
            gk(self.ptrs(), s)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 20
        gk.close()
        return {"ms": ms, "gbs": 12 * self.n / ms / 1e6}

    def details(self, world: int) -> dict:
        return {"workload": f"pointwise relu(x0) * x1, f32[{self.n}] N(0,1), p03 schedule (4 per thread)",
                "kernel": self.k.family, "l2": "operands (3 GiB per step) far exceed L2; no flush",
                "parallelism": f"replicas over {world} GPU(s)"}


BIGSUM_METRIC = "achieved HBM GB/s (sharded sum: per-GPU reduction + cross-GPU combine)"


class FullSum:
    name = "sum"
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, rank: int, world: int, dev: int, n_total: int = 1 << 20, sharded: bool = False,
                 collective: str = "peer"):
        import torch
        from thompiler import synth
        from thompiler.device import DeviceKernel
        from thompiler.shard import PeerCombine, slice_bounds
        self.torch, self.rank, self.world, self.sharded = torch, rank, world, sharded
        lo, hi = slice_bounds(n_total, rank, world) if sharded else (0, n_total)
        self.n = hi - lo
        self.n_total = n_total
        self.collective = collective if (sharded and world > 1) else None
        self.metric = (BIGSUM_METRIC if sharded else "achieved HBM GB/s (single-kernel array sum)")
        tmp = Path(tempfile.mkdtemp(prefix=f"bench_sum_{rank}_"))
        d = synth.sum_package(tmp / "sum", self.n)
        self.k = DeviceKernel(d / "k_sum_1_reduce.ir.json", device=dev)
        g = torch.Generator(device=f"cuda:{dev}").manual_seed(7 + rank)
        self.x = torch.rand(self.n, device=f"cuda:{dev}", generator=g) * 2 - 1
        self.out = torch.zeros(1, device=f"cuda:{dev}")
        self.kbytes = {"sum": self.n * 4 + 4}
        self.bytes_per_step = self.n * 4 * (world if sharded else 1) + 4 * world
        self.launches_per_step = 1
        self.dominant = "sum"
        self.kinds = ("sum",)
        self.peer = PeerCombine(self.k.module, rank, world) if self.collective == "peer" else None

    def step(self, stream: int, events=None) -> None:
        if events is not None:
            events["sum"][0].record()
        self.k({"x": self.x.data_ptr(), "sum_1": self.out.data_ptr()}, stream)
        if events is not None:
            events["sum"][1].record()
        if self.collective == "nccl":
            import torch.distributed as dist
            dist.all_reduce(self.out)

    def check(self) -> None:
        from thompiler import runner
        torch = self.torch
        want = self.x.double().sum()
        if self.collective is not None:
            import torch.distributed as dist
            dist.all_reduce(want)
        self.step(self.torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        got = float(self.out.item())
        if self.k.plan.error_word:
            assert runner.read_error_word(self.k.module, self.k.plan) == 0, "peer combine gave up"
        assert abs(got - float(want)) <= 1e-5 * max(1.0, abs(float(want))) + 1e-3, f"sum mismatch {got} vs {want}"

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def e2e(self, steps: int) -> dict:
        from thompiler import runner
        torch = self.torch
        hx = torch.empty(self.n, pin_memory=True)
        hx.copy_(self.x)
        ho = torch.zeros(1)
        args = [{"array": hx.numpy()}, {"array": ho.numpy(), "output": True}]
        def ranks_together():
            # the in-kernel combine waits (bounded) for every rank's kernel: enter each launch together
            if self.collective == "peer":
                import torch.distributed as dist
                dist.barrier()
        ranks_together()
        runner.run(self.k.fn, self.k.plan, args)
        t = time.perf_counter()
        for _ in range(steps):
            ranks_together()
            r = runner.run(self.k.fn, self.k.plan, args)
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
            if self.collective == "nccl":          # the peer combine already left the total in ho
                import torch.distributed as dist
                v = torch.tensor([float(ho[0])], device=self.x.device)
                dist.all_reduce(v)
                float(v.item())
        sec = (time.perf_counter() - t) / steps
        runner.release()
        return {"value": self.bytes_per_step / sec / 1e9, "unit": "GB/s", "work": self.n * 4 + 4,
                "h2d_bytes_per_step": hx.numel() * 4,
                "d2h_bytes_per_step": 4, "ms_per_step": sec * 1e3}

    def cpu_baseline(self) -> dict:
        from oracle import cpu_baseline
        n = min(self.n_total, 1 << 26)
        r = cpu_baseline.sum_sample(n)
        return {"value": n * 4 / r["seconds"] / 1e9, "unit": "GB/s", "cores": r["cores"], "kind": "port",
                "sample": f"torch CPU sum of f32[{n}], best of 3"}

    def details(self, world: int) -> dict:
        how = {"peer": "in-kernel combine over NVLink peer memory (no NCCL in the step)",
               "nccl": "NCCL all-reduce of the per-GPU results", None: "no exchange (one GPU)"}
        c = {"workload": (f"sharded sum f32[2^{self.n_total.bit_length() - 1}] -> per-GPU two-pass reduction "
                          f"+ {how[self.collective]}" if self.sharded else f"array sum f32[{self.n}] U[-1,1)"),
             "elements_per_gpu": self.n, "kernel": self.k.family,
             "launch": {"grid": list(self.k.plan.grid), "block": list(self.k.plan.block)},
             "l2": ("inputs larger than L2" if self.n * 4 > 126e6 else
                    "input (4 MiB) fits in L2: every step after the first reads it from L2")}
        c["parallelism"] = f"{'contiguous slices' if self.sharded else 'replicas'} over {world} GPU(s)"
        return c


class Matmul:
    """The two matmul benchmark shapes, f16 in, f32 accumulate and out, B column-major."""
    name = "matmul"
    metric = "achieved tensor TFLOP/s (f16 matmul, f32 accumulate: 4096^3 + 8192x3072x1024)"
    unit = "TFLOP/s"
    dtype = "f16"
    bound = "tensor"

    SHAPES = {"square": (4096, 4096, 4096), "rect": (8192, 3072, 1024)}

    def __init__(self, rank: int, world: int, dev: int, scale: int = 0, which: tuple = ("square", "rect")):
        import torch
        from thompiler import synth
        from thompiler.device import DeviceKernel
        self.torch = torch
        self.shapes = {k: self.SHAPES[k] for k in which}
        if scale:
            self.shapes = {"square": (scale, scale, scale)}
        if len(self.shapes) == 1:
            self.metric = (f"achieved tensor TFLOP/s (f16 matmul, f32 accumulate: "
                           f"{'x'.join(map(str, next(iter(self.shapes.values()))))})")
        tmp = Path(tempfile.mkdtemp(prefix=f"bench_mm_{rank}_"))
        self.k, self.gen, self.t = {}, {}, {}
        g = torch.Generator(device=f"cuda:{dev}").manual_seed(2000 + rank)
        for name, (m, n, k) in self.shapes.items():
            d = synth.matmul_package(tmp / name, m, n, k, b_layout="col", out_dtype="f32")
            self.k[name] = DeviceKernel(d / "k_matmul_f16.ir.json", device=dev)
            self.gen[name] = DeviceKernel(d / "k_matmul_f16.ir.json", device=dev, tuned=False)
            a = (torch.randn(m, k, device=f"cuda:{dev}", generator=g) * 0.02).half()
            b = (torch.randn(n, k, device=f"cuda:{dev}", generator=g) * 0.02).half()
            c = torch.empty(m, n, device=f"cuda:{dev}")
            self.t[name] = (a, b, c)
        self.kinds = tuple(self.shapes)
        self.flops = {k: 2 * m * n * kk for k, (m, n, kk) in self.shapes.items()}
        self.kbytes = {k: (m * kk + n * kk) * 2 + m * n * 4 for k, (m, n, kk) in self.shapes.items()}
        self.flops_per_step = sum(self.flops.values())
        self.bytes_per_step = self.flops_per_step        # value is flops-based for this workload
        self.launches_per_step = len(self.kinds)
        self.dominant = "square" if "square" in self.shapes else next(iter(self.shapes))

    def ptrs(self, name):
        a, b, c = self.t[name]
        return {"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}

    def step(self, stream: int, events=None) -> None:
        for name in self.kinds:
            if events is not None:
                events[name][0].record()
            self.k[name](self.ptrs(name), stream)
            if events is not None:
                events[name][1].record()

    def check(self) -> None:
        from thompiler import runner
        torch = self.torch
        s = torch.cuda.current_stream().cuda_stream
        for name in self.kinds:
            a, b, c = self.t[name]
            self.k[name](self.ptrs(name), s)
            torch.cuda.synchronize()
            assert runner.read_error_word(self.k[name].module, self.k[name].plan) == 0, "kernel wait gave up"
            ref = a.double() @ b.double().t()
            assert torch.allclose(c.double(), ref, rtol=2e-2, atol=2e-3), f"{name} mismatch against float64"

    def reference_lowering(self) -> dict:
        """The same IR through the statement-by-statement lowering (mma.sync, the
        reference compiler's kernel): ms per launch, for context."""
        torch = self.torch
        s = torch.cuda.current_stream().cuda_stream
        out = {}
        for name in self.kinds:
            a, b, c = self.t[name]
            p = {"x0": a.data_ptr(), "x1": b.data_ptr(), "matmul": c.data_ptr()}
            for _ in range(2):
                self.gen[name](p, s)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                self.gen[name](p, s)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 5
            out[name] = {"ms": ms, "tflops": self.flops[name] / (ms / 1e3) / 1e12}
        return out

    def e2e(self, steps: int) -> dict:
        from thompiler import runner
        torch = self.torch
        runs = {}
        h2d = d2h = 0
        for name in self.kinds:
            a, b, c = self.t[name]
            ha, hb = torch.empty_like(a, device="cpu").pin_memory(), torch.empty_like(b, device="cpu").pin_memory()
            ha.copy_(a)
            hb.copy_(b)
            hc = torch.empty(c.shape, pin_memory=True)
            k = self.k[name]
            arrs = {"x0": ha.numpy(), "x1": hb.numpy(), "matmul": hc.numpy()}
            runs[name] = (k, [{"array": arrs[n], "output": n == "matmul"} for n in k.arg_order])
            h2d += ha.numel() * 2 + hb.numel() * 2
            d2h += hc.numel() * 4
        for name, (k, args) in runs.items():
            runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
        t = time.perf_counter()
        for _ in range(steps):
            for name, (k, args) in runs.items():
                r = runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
                if not r["ok"]:
                    raise RuntimeError(r["stderr"])
        sec = (time.perf_counter() - t) / steps
        runner.release()
        return {"value": self.flops_per_step / sec / 1e12, "unit": "TFLOP/s", "work": self.flops_per_step,
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": sec * 1e3}

    def cpu_baseline(self) -> dict:
        from oracle import cpu_baseline
        r = cpu_baseline.matmul_sample(1024, 1024, 1024)
        return {"value": 2 * 1024 ** 3 / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": r["cores"],
                "kind": "port", "sample": "torch CPU f16 matmul 1024^3 (f32 result), one run"}

    def details(self, world: int) -> dict:
        return {"workload": "f16 matmul, f32 accumulate/out, A row-major, B column-major: "
                            + ", ".join(f"{m}x{n}x{k}" for m, n, k in self.shapes.values()),
                "kernels": {k: self.k[k].family for k in self.kinds},
                "tiles": {k: self.k[k].module.sidecar.get("tile") for k in self.kinds},
                "l2": "operands (56-96 MiB per GEMM incl. output) exceed half of L2; no flush",
                "parallelism": f"replicas over {world} GPU(s)"}


def _attention_ref(torch, q, k, v):
    """float32 softmax(Q K^T / sqrt(d)) V of f16 tensors (CPU or GPU)."""
    s = (q.float() @ k.float().transpose(-1, -2)) / q.shape[-1] ** 0.5
    return torch.softmax(s, -1) @ v.float()


class Attention:
    """softmax(Q K^T / sqrt(d)) V, f16 [8, 16, 2048, 128], non-causal; (batch, head) units
    split over the ranks (strong scaling, no collective)."""
    name = "attention"
    metric = "achieved tensor TFLOP/s (attention f16 [8,16,2048,128], non-causal)"
    unit = "TFLOP/s"
    dtype = "f16"
    bound = "tensor"
    sharded = True

    def __init__(self, rank: int, world: int, dev: int, seq: int = 0):
        import torch
        from thompiler import synth
        from thompiler.device import DeviceKernel
        from thompiler.shard import unit_range
        self.torch, self.dev = torch, dev
        B, H, S, D = 8, 16, seq or 2048, 128
        self.B, self.H, self.S, self.D, self.world = B, H, S, D, world
        u0, u1 = unit_range(B * H, rank, world)          # this rank's (batch, head) units
        Ul = u1 - u0
        tmp = Path(tempfile.mkdtemp(prefix=f"bench_att_{rank}_"))
        d = synth.attention_package(tmp / "att", Ul, 1, S, D)
        self.k = {"attention": DeviceKernel(d / "k_attention.ir.json", device=dev)}
        g = torch.Generator(device=f"cuda:{dev}").manual_seed(3000 + rank)
        self.q, self.kk, self.v = (torch.randn(Ul, 1, S, D, device=f"cuda:{dev}", generator=g).half()
                                   for _ in range(3))
        self.c = torch.tensor([D ** 0.5], device=f"cuda:{dev}")
        self.o = torch.empty(Ul, 1, S, D, device=f"cuda:{dev}", dtype=torch.float16)
        self.kinds = ("attention",)
        self.flops = {"attention": 4 * Ul * S * S * D}
        self.kbytes = {"attention": 4 * Ul * S * D * 2}
        self.flops_per_step = 4 * B * H * S * S * D
        self.bytes_per_step = self.flops_per_step
        self.launches_per_step = 1
        self.dominant = "attention"

    def ptrs(self) -> dict:
        return {"div_c1": self.c.data_ptr(), "q": self.q.data_ptr(), "k": self.kk.data_ptr(),
                "v": self.v.data_ptr(), "attn": self.o.data_ptr()}

    def step(self, stream: int, events=None) -> None:
        if events is not None:
            events["attention"][0].record()
        self.k["attention"](self.ptrs(), stream)
        if events is not None:
            events["attention"][1].record()

    def check(self) -> None:
        from thompiler import runner
        torch = self.torch
        self.step(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        k = self.k["attention"]
        assert runner.read_error_word(k.module, k.plan) == 0, "kernel wait gave up"
        s = (self.q[0].float() @ self.kk[0].float().transpose(-1, -2)) / self.D ** 0.5
        ref = torch.softmax(s, -1) @ self.v[0].float()
        assert torch.allclose(self.o[0].float(), ref, rtol=2e-2, atol=2e-3), "attention mismatch"

    def e2e(self, steps: int) -> dict:
        from thompiler import runner
        torch = self.torch
        k = self.k["attention"]
        host = {n: torch.empty_like(x, device="cpu").pin_memory() for n, x in
                (("q", self.q), ("k", self.kk), ("v", self.v), ("attn", self.o))}
        for n, x in (("q", self.q), ("k", self.kk), ("v", self.v)):
            host[n].copy_(x)
        arrs = {n: h.numpy() for n, h in host.items()}
        arrs["div_c1"] = self.c.cpu().numpy()
        args = [{"array": arrs[n], "output": n == "attn"} for n in k.arg_order]
        runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
        t = time.perf_counter()
        for _ in range(steps):
            r = runner.run(k.fn, k.plan, args, arg_order=k.arg_order)
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
        sec_single = (time.perf_counter() - t) / steps
        runner.release()
        # the same step as requests of `chunk` (batch, head) units each, on one module compiled
        # for that many units, in one thr_run_batch: one request's Q, K, V cross PCIe while
        # another's kernel runs and a third's output comes back
        units = self.q.shape[0]
        chunk = next(c for c in (16, 8, 4, 2, 1) if units % c == 0)
        from thompiler import synth
        from thompiler.device import DeviceKernel
        kc = DeviceKernel(synth.attention_package(Path(tempfile.mkdtemp(prefix="bench_att_e2e_")) / "att", chunk, 1,
                                                  self.S, self.D) / "k_attention.ir.json", device=self.dev)
        reqs = []
        for u0 in range(0, units, chunk):
            a = {n: (arrs[n] if n == "div_c1" else arrs[n][u0:u0 + chunk]) for n in kc.arg_order}
            reqs.append((kc.fn, kc.plan, [{"array": a[n], "output": n == "attn"} for n in kc.arg_order],
                         kc.arg_order))
        batch = runner.PreparedBatch(reqs)
        r = batch.run()
        if not r["ok"]:
            raise RuntimeError(r["stderr"])
        ref = _attention_ref(torch, host["q"][:1], host["k"][:1], host["v"][:1])
        assert torch.allclose(host["attn"][:1].float(), ref, rtol=2e-2, atol=2e-3), "chunked attention mismatch"
        t = time.perf_counter()
        for _ in range(steps):
            r = batch.run()
            if not r["ok"]:
                raise RuntimeError(r["stderr"])
        sec = (time.perf_counter() - t) / steps
        runner.release()
        kc.close()
        return {"value": self.flops["attention"] / sec / 1e12, "unit": "TFLOP/s", "work": self.flops["attention"],
                "h2d_bytes_per_step": 3 * self.q.numel() * 2 + 4, "d2h_bytes_per_step": self.o.numel() * 2,
                "ms_per_step": sec * 1e3,
                "how": f"one thr_run_batch per step on pinned host buffers: {units // chunk} requests of {chunk} "
                       "(batch, head) units on one module, copies in, kernels and copies out overlapped",
                "one_thr_run": {"value": self.flops["attention"] / sec_single / 1e12, "ms_per_step": sec_single * 1e3}}

    def cpu_baseline(self) -> dict:
        from oracle import cpu_baseline
        r = cpu_baseline.attention_sample(2, self.S, self.D)
        fl = 4 * 2 * self.S * self.S * self.D
        return {"value": fl / r["seconds"] / 1e12, "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
                "sample": f"torch CPU f16 attention on 2 of the 128 heads ([2, {self.S}, {self.D}]), one run"}

    def details(self, world: int) -> dict:
        return {"workload": f"attention f16 [{self.B}, {self.H}, {self.S}, {self.D}] non-causal, "
                            "scale 1/sqrt(d), f32 accumulate",
                "kernels": {"attention": self.k["attention"].family},
                "tile": self.k["attention"].module.sidecar.get("tile") if self.k["attention"].module.sidecar else None,
                "l2": "K/V of a head (1 MiB) shared in L2 by its 16 query tiles; no flush",
                "parallelism": f"(batch, head) sharding over {world} GPU(s), no collective"}


# ---- the suite ------------------------------------------------------------------------

# about one second of timed work per workload at one GPU (used with an explicit --config
# when --steps is not given)
DEFAULT_STEPS = {"rowops": 6000, "sum": 20000, "bigsum": 1500, "bigsum_nccl": 1500, "matmul": 5000,
                 "matmul_square": 5000, "matmul_rect": 10000, "attention": 2500, "pointwise": 2000}

CONFIGS = {"rowops": lambda r, w, d, n: RowOps(r, w, d, rows=n or 8192),
           "pointwise": lambda r, w, d, n: Pointwise(r, w, d, n),
           "attention": lambda r, w, d, n: Attention(r, w, d, n),
           "matmul": lambda r, w, d, n: Matmul(r, w, d, n),
           "matmul_square": lambda r, w, d, n: Matmul(r, w, d, n, which=("square",)),
           "matmul_rect": lambda r, w, d, n: Matmul(r, w, d, n, which=("rect",)),
           "sum": lambda r, w, d, n: FullSum(r, w, d, n or 1 << 20),
           "bigsum": lambda r, w, d, n: FullSum(r, w, d, n or 1 << 30, sharded=True, collective="peer"),
           "bigsum_nccl": lambda r, w, d, n: FullSum(r, w, d, n or 1 << 30, sharded=True, collective="nccl")}

# the default run: the row ops are the headline line, every workload is one record of `configs`
SUITE = ("rowops", "sum", "bigsum", "matmul_square", "matmul_rect", "attention", "pointwise")
SUITE_MULTI = ("rowops", "sum", "bigsum", "bigsum_nccl", "matmul_square", "matmul_rect", "attention",
               "pointwise")

SHARDED = {"bigsum", "bigsum_nccl", "attention"}

METRICS = {"rowops": RowOps.metric, "pointwise": Pointwise.metric, "attention": Attention.metric,
           "matmul": Matmul.metric,
           "matmul_square": "achieved tensor TFLOP/s (f16 matmul, f32 accumulate: 4096x4096x4096)",
           "matmul_rect": "achieved tensor TFLOP/s (f16 matmul, f32 accumulate: 8192x3072x1024)",
           "sum": "achieved HBM GB/s (single-kernel array sum)", "bigsum": BIGSUM_METRIC,
           "bigsum_nccl": BIGSUM_METRIC}


def workload_config(name: str, world: int) -> dict:
    """The workload a line measures, identical in both arms (ours and the reference's CPU path)."""
    mm = {"matmul": "4096x4096x4096, 8192x3072x1024", "matmul_square": "4096x4096x4096",
          "matmul_rect": "8192x3072x1024"}
    if name == "rowops":
        c = {"workload": "fused row ops f32[8192, 4096] x3 (softmax, rmsnorm eps=1e-6, l2norm)",
             "l2": "inputs larger than L2 (3 x 128 MiB distinct input matrices per GPU)",
             "parallelism": f"weak: {world} GPU(s), one matrix set each, no collective"}
    elif name == "pointwise":
        c = {"workload": "pointwise relu(x0) * x1, f32[268435456] N(0,1), p03 schedule (4 per thread)",
             "l2": "operands (3 GiB per step) far exceed L2; no flush",
             "parallelism": f"replicas over {world} GPU(s)"}
    elif name in mm:
        c = {"workload": f"f16 matmul, f32 accumulate/out, A row-major, B column-major, N(0,0.02): {mm[name]}",
             "l2": "operands (56-96 MiB per GEMM incl. output) exceed half of L2; no flush",
             "parallelism": f"replicas over {world} GPU(s)"}
    elif name == "attention":
        c = {"workload": "attention f16 [8, 16, 2048, 128] N(0,1) non-causal, scale 1/sqrt(d), f32 accumulate",
             "l2": "K/V of a head (1 MiB) shared in L2 by its 16 query tiles; no flush",
             "parallelism": f"strong: (batch, head) units split over {world} GPU(s), no collective"}
    elif name == "sum":
        c = {"workload": "array sum f32[1048576] U[-1,1), one kernel",
             "l2": "input (4 MiB) fits in L2: every step after the first reads it from L2",
             "parallelism": f"replicas over {world} GPU(s)"}
    else:
        how = ("NCCL all-reduce of the per-GPU results" if name == "bigsum_nccl" else
               "in-kernel combine over NVLink peer memory (no NCCL in the step)")
        c = {"workload": f"sharded sum f32[2^30] U[-1,1): per-GPU two-pass reduction + "
                         f"{how if world > 1 else 'no exchange (one GPU)'}",
             "l2": "inputs larger than L2",
             "parallelism": f"strong: contiguous slices over {world} GPU(s)"}
    return c


def cpu_sample(name: str) -> dict:
    """The reference's CPU path (the torch expression each problem was generated from, on this
    host's cores) over a bounded sample of one step of workload ``name``: the callable, the
    sample's algorithmic work in the metric's unit and what the sample is."""
    from oracle import cpu_baseline as cb
    if name == "rowops":
        rows, cols = 1024, 4096
        return {"run": lambda: cb.rowops_sample(rows, cols), "work": 3 * 2 * rows * cols * 4 + cols * 4,
                "unit": "GB/s", "scale": 1e9, "dtype": "f32",
                "sample": f"torch CPU softmax + RMSNorm + L2-norm on f32[{rows}, {cols}] (1/8 of a step)"}
    if name == "pointwise":
        m = 1 << 24
        return {"run": lambda: cb.pointwise_sample(m), "work": 12 * m, "unit": "GB/s", "scale": 1e9,
                "dtype": "f32", "sample": f"torch CPU relu(x0) * x1 on f32[{m}] (1/16 of a step)"}
    if name in ("matmul", "matmul_square", "matmul_rect"):
        m, n, k = (512, 4096, 4096) if name == "matmul_square" else (1024, 3072, 1024)
        part = "1/8 of the 4096^3 rows" if name == "matmul_square" else "1/8 of the 8192x3072x1024 rows"
        return {"run": lambda: cb.matmul_sample(m, n, k), "work": 2 * m * n * k, "unit": "TFLOP/s",
                "scale": 1e12, "dtype": "f16",
                "sample": f"torch CPU f16 matmul {m}x{n}x{k} (B column-major, f32 result; {part})"}
    if name == "attention":
        bh, sq, d = 2, 2048, 128
        return {"run": lambda: cb.attention_sample(bh, sq, d), "work": 4 * bh * sq * sq * d, "unit": "TFLOP/s",
                "scale": 1e12, "dtype": "f16",
                "sample": f"torch CPU f16 attention on {bh} of the 128 heads ([{bh}, {sq}, {d}])"}
    n = 1 << 20 if name == "sum" else 1 << 26
    return {"run": lambda: cb.sum_sample(n), "work": n * 4, "unit": "GB/s", "scale": 1e9, "dtype": "f32",
            "sample": f"torch CPU sum of f32[{n}]" + ("" if name == "sum" else " (1/16 of the 2^30 array)")}


def time_cpu_sample(name: str, steps: int, warmup: int, budget_s: float) -> dict:
    from oracle import cpu_baseline as cb
    smp = cpu_sample(name)
    for _ in range(min(warmup, 3)):
        smp["run"]()
    samples, t0 = [], time.perf_counter()
    while len(samples) < steps and (not samples or time.perf_counter() - t0 < budget_s):
        samples.append(smp["run"]()["seconds"])
    sec = statistics.median(samples)
    return {"value": smp["work"] / sec / smp["scale"], "unit": smp["unit"], "cores": cb.threads(), "kind": "port",
            "sample": smp["sample"], "seconds": sec, "samples_timed": len(samples), "dtype": smp["dtype"]}


REFERENCE_BUDGET_S = 90.0      # wall-time cap on the reference arm's timed samples (one workload)
SUITE_REFERENCE_BUDGET_S = 15.0    # the same, per workload of the default suite


def reference_record(name: str, args, world: int, budget_s: float) -> dict:
    r = time_cpu_sample(name, args.steps, args.warmup, budget_s)
    value, unit = r["value"], r["unit"]
    return {"impl": "reference", "metric": METRICS[name], "value": value, "unit": unit,
            "ms_per_step": r["seconds"] * 1e3, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong" if name in SHARDED else "weak",
            "dtype": r["dtype"], "config": workload_config(name, world),
            "cpu_baseline": {"value": value, "unit": unit, "cores": r["cores"], "kind": "port",
                             "sample": r["sample"], "samples_timed": r["samples_timed"]},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_arm(args, world: int, out=None) -> None:
    """The reference's CPU path (the torch expression each problem was generated from, evaluated on
    this host's cores, all of its threads) on a bounded sample of the same workload, same metric and
    config as our arm.  Under torchrun rank 0 alone runs and prints; the other ranks exit."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.config != "all":
        line = reference_record(args.config, args, world, REFERENCE_BUDGET_S)
    else:
        suite = SUITE_MULTI if world > 1 else SUITE
        line = reference_record("rowops", args, world, SUITE_REFERENCE_BUDGET_S)
        line["configs"] = {n: reference_record(n, args, world, SUITE_REFERENCE_BUDGET_S) for n in suite}
    line.update(n_gpus=world, vs_baseline=None, data="synthetic")
    print(json.dumps(line), file=out or sys.stdout, flush=True)


def _result_stream():
    """The JSON line is the only thing this program writes to its standard output: native
    libraries (NCCL's version banner, driver JIT messages) print to file descriptor 1 too, so
    that descriptor is pointed at stderr and the line goes to a private copy of the original."""
    out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    return out


PROFILE = {"rowops": ("k_softmax_rows_rowops", ""), "sum": ("k_sum_1_reduce_sum", ""),
           "bigsum": ("k_sum_1_reduce_bigsum", ""), "bigsum_nccl": ("k_sum_1_reduce_bigsum", ""),
           "matmul": ("k_matmul_f16_matmul", "square"), "matmul_square": ("k_matmul_f16_matmul", "square"),
           "matmul_rect": ("k_matmul_f16_matmul", "rect"), "attention": ("k_attention_attention", ""),
           "pointwise": ("k_mul_pointwise_pointwise", "")}


def measure(name: str, w, args, steps: int, world: int, rank: int, local: int) -> dict | None:
    """Check, warm up and time ``steps`` steps of workload ``w``; rank 0 gets its record."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream().cuda_stream
    w.check()
    for _ in range(args.warmup):
        w.step(stream)
    # per-kernel durations: CUDA events around every launch of an untimed pass on the launch stream
    n_ev = min(steps, 200)
    events = {k: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(n_ev)] for k in w.kinds}
    for i in range(n_ev):
        w.step(stream, {k: events[k][i] for k in w.kinds})
    torch.cuda.synchronize()
    per_kernel = {k: statistics.mean(a.elapsed_time(b) for a, b in events[k]) for k in w.kinds}
    # the timed region: the K steps replayed from CUDA graphs of G steps each (no host launch
    # overhead between kernels; a step's NCCL all-reduce is captured with it)
    use_graph = not args.no_graph
    graph, G = None, 1
    if use_graph:
        G = next(g for g in range(min(steps, 500), 0, -1) if steps % g == 0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cap = torch.cuda.current_stream().cuda_stream
            for _ in range(G):
                w.step(cap)
        graph.replay()
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the clock sampler starts before the ranks meet, so they all start the timed region right
    # after the barrier (a combine inside the kernels makes early ranks wait for late ones)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if world > 1:
        # the host barrier releases the ranks some microseconds apart; a one-element all-reduce
        # queued just before the start event lines the GPUs up, so a short region is not
        # lengthened on the early ranks by the late ranks' start
        tick = torch.zeros(1, device=f"cuda:{local}")
        dist.all_reduce(tick)
    # a ~1 ms device-side delay (outside the timed region) before the start event: by the time
    # it ends the host has queued every replay of the region, so a region of a few microseconds
    # per step does not also time the host's submission of its first graph
    torch.cuda._sleep(2_000_000)
    start.record()
    if graph is not None:
        for _ in range(steps // G):
            graph.replay()
    else:
        for _ in range(steps):
            w.step(stream)
    end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    if graph is not None:
        # kernels run back to back inside the graphs: share the timed step among them in the
        # proportions of their event-timed durations (one kernel per step: the step itself)
        tot = sum(per_kernel.values())
        per_kernel = {k: ms * v / tot for k, v in per_kernel.items()}
    del graph
    t = torch.tensor([ms], device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    e2e = None
    if not args.no_e2e:
        e2e = w.e2e(max(1, min(steps, 5)))
        if world > 1:
            # the job's e2e rate: the work every rank did in one step over the slowest rank's step
            v = torch.tensor([e2e["ms_per_step"]], device=f"cuda:{local}", dtype=torch.float64)
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
            wk = torch.tensor([float(e2e["work"])], device=f"cuda:{local}", dtype=torch.float64)
            dist.all_reduce(wk, op=dist.ReduceOp.SUM)
            unit_scale = 1e12 if getattr(w, "bound", "hbm") == "tensor" else 1e9
            e2e["value"] = float(wk.item()) / (float(v.item()) / 1e3) / unit_scale
            e2e["ms_per_step"] = float(v.item())
            e2e["work"] = float(wk.item())
    if rank != 0:
        return None
    pk = peaks()
    dom = w.dominant
    kms = per_kernel[dom]
    kernel_name = f"{w.k[dom].info.name if isinstance(w.k, dict) else w.k.info.name}"
    prof, tag = PROFILE.get(name, (f"{kernel_name}_{name}", ""))
    traffic = profile_traffic(prof, tag)
    total = w.bytes_per_step if getattr(w, "sharded", False) else w.bytes_per_step * world
    if getattr(w, "bound", "hbm") == "tensor":
        long_run = ms_max * steps > 1000.0
        peak = pk.get("bf16_tflops_sustained" if long_run else "bf16_tflops", pk["bf16_tflops"])
        achieved = w.flops[dom] / (kms / 1e3) / 1e12
        value, unit = total / (ms_max / 1e3) / 1e12, "TFLOP/s"
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "peak_kind": "sustained" if long_run else "burst"}
    else:
        achieved = w.kbytes[dom] / (kms / 1e3) / 1e9
        value, unit = total / (ms_max / 1e3) / 1e9, "GB/s"
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "traffic": traffic}
    roof.update(kernel=kernel_name, peak_source=pk["source"], kernel_ms=kms, per_kernel_ms=per_kernel)
    details = w.details(world)
    how = f"{steps // G} replays of a CUDA graph of {G} steps" if use_graph else "steps launched one by one"
    details["timing"] = how + ("; per-kernel times: the timed step shared in the proportions of per-launch "
                               "CUDA events" if use_graph else "; per-kernel times from per-launch CUDA events")
    if hasattr(w, "reference_lowering"):
        details["reference_lowering"] = w.reference_lowering()
    cpu = None
    if world == 1:
        r = time_cpu_sample(name, 3, 1, 10.0)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    return {"metric": w.metric, "value": value, "unit": unit, "ms_per_step": ms_max, "steps": steps,
            "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong" if getattr(w, "sharded", False) else "weak", "dtype": w.dtype,
            "config": workload_config(name, world), "details": details, "roofline": roof,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": w.launches_per_step * steps, "clocks": clk}


def run_workload(name: str, args, steps: int, world: int, rank: int, local: int) -> dict | None:
    import gc

    import torch
    w = CONFIGS[name](rank, world, local, args.size)
    try:
        return measure(name, w, args, steps, world, rank, local)
    finally:
        if hasattr(w, "close"):
            w.close()
        ks = w.k.values() if isinstance(w.k, dict) else [w.k]
        for k in ks:
            k.close()
        for g in getattr(w, "gen", {}).values():
            g.close()
        del w
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def main() -> None:
    out = _result_stream()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0,
                    help="timed steps (default: 20 for the suite; about one second of work for one --config)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="all", choices=["all", *sorted(CONFIGS)],
                    help="all (default): the row ops as the headline line and every workload as a record "
                         "of its `configs` object; otherwise one workload")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the timed steps one by one instead of replaying CUDA graphs")
    ap.add_argument("--size", type=int, default=0,
                    help="override the workload size (rows for rowops, elements for sums); profiling only")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps <= 0:
        args.steps = 20 if args.config == "all" else DEFAULT_STEPS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        reference_arm(args, world, out)
        return

    import torch
    import torch.distributed as dist
    from thompiler import runner

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    runner.init(local)
    if args.config == "all":
        suite = SUITE_MULTI if world > 1 else SUITE
        records = {n: run_workload(n, args, args.steps, world, rank, local) for n in suite}
        line = dict(records["rowops"]) if rank == 0 else None
        if line is not None:
            line["configs"] = records
    else:
        line = run_workload(args.config, args, args.steps, world, rank, local)
    if rank == 0:
        line.update(n_gpus=world, vs_baseline=None, data="synthetic")
        print(json.dumps(line), file=out, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
