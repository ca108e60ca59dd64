#!/usr/bin/env python
"""Benchmark of the NVFP4 hot path on B200s; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload attention|quantize|decode|qkv|prefill|weights|llama|gemm]
                    [--impl ours|reference]

With no --workload the line is the long-context prefill (the headline: a
fixed 70.37 TFLOP job split over the ranks, strong scaling) with the
Llama-3-8B attention, the [4096,4096] quantize and the 70B weight-stack
quantize as sub-objects of the same line, each with its own value, roofline,
e2e and CPU baseline.  For N > 1 launch one rank per GPU with
torch.distributed.run; ranks shard the work with no collective on the data
path and every reported time is the max over ranks.  The dense NVFP4 peak
(the FP4 roofline denominator) is measured at the start of every run.

Workloads (synthetic data with the shapes and distributions of the named
configurations; no dataset is read):

* attention -- NVFP4 attention forward, Llama-3-8B shape: B=1, 32 query /
  8 KV heads, D=128, T=4096, causal, bf16 q/k/v ~ N(0,1) from seed 1.  A
  step quantizes Q/K/V to NVFP4 and runs the FP4 attention kernel.  Metric:
  TFLOP/s with the algorithmic causal count 4*B*Hq*T^2*D/2.
* quantize -- NVFP4 quantize of one bf16 [4096,4096] tensor (N(0,1), seed
  0, 0.1% of entries x50) with a per-tensor scale amax/(448*6).  Metric:
  GB/s of algorithmic traffic, 2.5625 B per element (2 B read, 0.5 B codes,
  1/16 B scales).
* decode -- one decode step over an NVFP4 KV cache: B=8, 32 query / 8 KV
  heads, D=128, 32768 cached tokens (N(0,1) bf16 K/V appended in calls of
  4096 tokens, seed 2 + rank).  Metric: GB/s of cache bytes read per step.
* qkv -- the Q and K projections of one Llama-3-8B layer fused with RoPE and
  the NVFP4 quantizer: T=4096 tokens, hidden 4096, 32 + 8 heads (hidden
  N(0,1), weights N(0,0.02), seed 3 + rank).  Metric: TFLOP/s of the two
  projections, 2*T*hidden*(Hq+Hkv)*128.
* prefill -- long-context prefill: B=4, 64 query / 8 KV heads, D=128,
  T=32768, causal, q/k/v N(0,1)*0.5 with a per-(kv-head, channel) N(0,2)
  bias on k (seed 2).  Strong scaling: the 32 (batch, KV-head) units are
  split over the ranks in contiguous blocks (1, 2, 4 or 8 ranks).  Metric:
  TFLOP/s of the whole job, 70.37 TFLOP per step.
* weights -- per-tensor NVFP4 quantize of the linear weights of a
  Llama-3-70B-shaped stack (q/o 8192x8192, k/v 1024x8192, gate/up
  28672x8192, down 8192x28672; bf16 N(0,0.02), tensor t from seed 4 + t).
  Weak scaling by whole layers: 10 layers per rank, so 8 ranks quantize the
  80-layer stack.  Metric: GB/s of algorithmic traffic (2.5625 B/element).
* llama -- one forward of a Llama-2-7B-shaped model (random bf16 weights
  N(0,0.02), seed 3) with the FP4 attention patch installed, batch 8 x 2048
  token ids; strong scaling over the batch.  Metric: tokens/s.
* gemm -- an FP4 linear layer: 8192 tokens of bf16 activations quantized
  per token and multiplied by layer 0's per-tensor NVFP4 gate weight of the
  70B stack (8192 -> 28672) on tcgen05.  Metric: TFLOP/s, 2*M*N*K.

decode and qkv measure the rows that extend the path (the NVFP4 KV cache,
the fused projection); prefill and weights the long-context and weight
configurations, llama the patched model.

L2 (126 MB) is defeated by rotating through input/output buffer sets larger
than L2 in total, so every step reads HBM.

--impl reference times the reference's own CPU implementation of the path
(its torch ops, restated op for op in oracle/torch_port.py and pinned to its
outputs) on the host cores, for the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

L2_BYTES = 126 * 2**20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["attention", "quantize", "decode", "qkv", "prefill", "weights",
                                                     "llama", "gemm"],
                    default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=10,
                    help="weights workload: layers per rank (10 = the 80-layer stack at 8 ranks)")
    ap.add_argument("--decode-batch", type=int, default=8,
                    help="decode workload: sequences per rank (8 = the headline case; profiles capture 4)")
    return ap.parse_args()


def profile_traffic(name):
    """DRAM bytes per launch of a kernel from its committed ncu summary (profiles/<name>.md), or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1])
    except OSError:
        pass
    return None


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def fp4_peak(peaks, peak_src):
    """(peak TFLOP/s, source) for FP4 contractions: the mxf4nvf4 throughput measured in this run
    (measure_fp4_peak) when present, else 4 x the dense bf16 peak."""
    if peaks.get("fp4_tflops"):
        return peaks["fp4_tflops"], (f"measured mxf4nvf4 (this run, {peaks.get('fp4_mhz')} MHz median); "
                                     f"4 x {peak_src} dense bf16 = {4 * peaks['bf16_tflops']:.0f}; nominal dense FP4 9000")
    return 4 * peaks["bf16_tflops"], f"4 x {peak_src} dense bf16 (no measured FP4 peak); nominal dense FP4 9000"


def measure_fp4_peak(dev, iters=16384, reps=5):
    """Dense NVFP4 tensor throughput of this GPU: fp4_mma_peak_run (one CTA per SM issuing
    back-to-back tcgen05 mxf4nvf4 M128 N128 K64 MMAs), best of `reps` event-timed launches."""
    from fp4_attn_b200 import _lib
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    st = torch.cuda.current_stream(dev)
    for _ in range(3):
        _lib.call("fp4_mma_peak_run", iters, 0, st.cuda_stream)
    torch.cuda.synchronize(dev)
    best = 0.0
    with Clocks(dev) as clk:
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            _lib.call("fp4_mma_peak_run", iters, 0, st.cuda_stream)
            b.record(st)
            b.synchronize()
            best = max(best, sms * iters * 4194304 / (a.elapsed_time(b) / 1e3) / 1e12)
    if _lib.load().fp4attn_device_status(1) != 0:
        raise RuntimeError("mma_peak_kernel: a bounded wait gave up")
    return best, clk.summary().get("sm_mhz")


# ----------------------------------------------------------------- clocks
class Clocks:
    """SM clock and throttle reasons sampled through NVML (a polling thread,
    ~5 ms period) while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, dev):
        self.dev = dev
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = False
        self._thread = None

    def _handle(self):
        import pynvml
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.dev)
        dom, bus, dv = (getattr(props, a, None) for a in ("pci_domain_id", "pci_bus_id", "pci_device_id"))
        if all(isinstance(v, int) for v in (dom, bus, dv)):
            # torch reports the PCI location as integers; NVML wants "dddddddd:bb:dd.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dv:02x}.0")
        return pynvml.nvmlDeviceGetHandleByIndex(self.dev.index or 0)

    def _run(self, h):
        import pynvml
        while not self._stop:
            try:
                self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                self.reasons |= pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        import threading
        try:
            import pynvml
            h = self._handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, args=(h,), daemon=True)
            self._thread.start()
            time.sleep(0.02)
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *a):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        names = sorted(v for k, v in self.REASONS.items() if self.reasons & k)
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples), "source": "nvml"}


# ------------------------------------------------------------- workloads
def quantize_input(rank=0):
    g = torch.Generator().manual_seed(rank)
    x = torch.randn(4096, 4096, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    x.view(-1)[idx] *= 50
    return x.bfloat16()


class E2EPipe:
    """Host-buffer steps overlapped the way a serving loop runs them: step i's H2D
    copy (copy stream), compute (compute stream) and D2H read-back (second copy
    stream) wait only on what they use, so the next step's inputs cross PCIe while
    this step computes.  Every step still moves its own inputs and result."""

    def __init__(self, nslots):
        self.h2d, self.comp, self.d2h = (torch.cuda.Stream() for _ in range(3))
        self.used = [None] * nslots  # compute done with the slot's device buffers
        self.read = [None] * nslots  # D2H done with the slot's result

    def begin(self):
        ev = torch.cuda.Event()
        ev.record()
        for st in (self.h2d, self.comp, self.d2h):
            st.wait_event(ev)

    def step(self, slot, h2d, compute, d2h):
        with torch.cuda.stream(self.h2d):
            if self.used[slot] is not None:
                self.h2d.wait_event(self.used[slot])
            h2d()
            ev_in = torch.cuda.Event()
            ev_in.record()
        with torch.cuda.stream(self.comp):
            self.comp.wait_event(ev_in)
            if self.read[slot] is not None:
                self.comp.wait_event(self.read[slot])
            res = compute()
            ev_c = torch.cuda.Event()
            ev_c.record()
        with torch.cuda.stream(self.d2h):
            self.d2h.wait_event(ev_c)
            d2h(res)
            ev_r = torch.cuda.Event()
            ev_r.record()
        self.used[slot], self.read[slot] = ev_c, ev_r

    def join(self):
        cur = torch.cuda.current_stream()
        for st in (self.h2d, self.comp, self.d2h):
            cur.wait_stream(st)


class QuantizeWorkload:
    name = "quantize"
    metric = "NVFP4 quantize GB/s per B200, % of HBM roofline"
    unit = "GB/s"
    dtype = "bf16->nvfp4 (fp32 arithmetic)"

    def __init__(self, dev, rank=0, world=1):
        from fp4_attn_b200 import _lib
        self.lib = _lib
        self.dev = dev
        x = quantize_input(rank)  # weak scaling: one [4096,4096] tensor per rank, seed r
        self.m, self.n = x.shape
        self.elems = x.numel()
        self.algo_bytes = self.elems * (2 + 0.5 + 1 / 16)
        per_set = self.elems * (2 + 0.5 + 1 / 16)
        self.nsets = max(2, int(2 * L2_BYTES // per_set) + 1)
        self.x_host = x.pin_memory()
        self.xs = [x.to(dev) for _ in range(self.nsets)]
        self.codes = [torch.empty(self.m, self.n // 2, dtype=torch.uint8, device=dev) for _ in range(self.nsets)]
        self.scales = [torch.empty(self.m, self.n // 16, dtype=torch.uint8, device=dev) for _ in range(self.nsets)]
        self.g = [torch.empty(1, dtype=torch.float32, device=dev) for _ in range(self.nsets)]
        self.codes_host = torch.empty(self.m, self.n // 2, dtype=torch.uint8).pin_memory()
        self.scales_host = torch.empty(self.m, self.n // 16, dtype=torch.uint8).pin_memory()
        self.stream = torch.cuda.current_stream(dev).cuda_stream
        self.config = {"workload": "quantize bf16 [4096,4096], per-tensor scale amax/2688, block 16",
                       "elements": self.elems, "l2": f"rotating {self.nsets} input/output sets (> L2)",
                       "global_batch": world, "shard": "tensor r on rank r (seed r)"}

    def _global(self, i):
        self.lib.call("fp4q_global_scale", self.xs[i].data_ptr(), 1, 1, self.m, 1, self.n, 0, self.n, 0,
                      3, 0, 2688.0, self.g[i].data_ptr(), self.stream)

    def _rows(self, i):
        self.lib.call("fp4q_quantize", self.xs[i].data_ptr(), 1, 1, self.m, 1, self.n, 0, self.n, 0, self.m,
                      3 | 0x10, 0, 2688.0, self.codes[i].data_ptr(), self.n // 2, self.scales[i].data_ptr(), 0,
                      self.n // 16, self.g[i].data_ptr(), None, 0, 0, self.stream)

    use_graph = True  # ~25 us steps: timed as CUDA graph replays

    def _full(self, i):
        # per-tensor max and quantize in one call: the library runs its single-pass
        # kernel when the tensor fits on chip, else the max pre-pass + row kernel
        self.lib.call("fp4q_quantize", self.xs[i].data_ptr(), 1, 1, self.m, 1, self.n, 0, self.n, 0, self.m,
                      3, 0, 2688.0, self.codes[i].data_ptr(), self.n // 2, self.scales[i].data_ptr(), 0,
                      self.n // 16, self.g[i].data_ptr(), None, 0, 0, self.stream)

    def step(self, i, ev=None):
        i %= self.nsets
        if ev is not None:
            ev[0].record()
        self._full(i)
        if ev is not None:
            ev[1].record()

    def kernel(self, i):
        self._full(i % self.nsets)

    def e2e_step(self, i):
        """Public API, host buffers: H2D input, quantize, D2H codes + scales (pipelined over steps)."""
        from fp4_attn_b200 import quant
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets

        def d2h(t):
            self.codes_host.copy_(t.codes, non_blocking=True)
            self.scales_host.copy_(t.scales, non_blocking=True)

        self.pipe.step(i, lambda: self.xs[i].copy_(self.x_host, non_blocking=True),
                       lambda: quant.quantize(self.xs[i], "tensor", 2688.0), d2h)

    e2e_h2d = property(lambda self: self.elems * 2)
    e2e_d2h = property(lambda self: self.elems // 2 + self.elems // 16)

    def value(self, seconds_per_step, world):
        return world * self.algo_bytes / seconds_per_step / 1e9

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        achieved = self.algo_bytes / kernel_s / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "kernel": "quant_tensor_fused_kernel (memset + one cooperative launch)",
                "achieved": round(achieved, 1), "peak": peak,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} copy bandwidth",
                "algorithmic_bytes_per_launch": self.algo_bytes,
                "traffic": profile_traffic("quant_tensor_fused_kernel_4096x4096_tensor"),
                "traffic_source": "profiles/quant_tensor_fused_kernel_4096x4096_tensor.md: ncu dram__bytes_read+write per launch"}

    # CPU: the reference's torch path restated (oracle/torch_port.py), full tensor.
    def cpu_sample(self, reps=None):
        from oracle import torch_port as tp
        x = quantize_input()
        one = torch.tensor(1.0)
        t0 = time.perf_counter()
        n = 0
        while True:
            amax = x.abs().max().float()
            g = amax * (one / torch.tensor(2688.0))
            tp.fused_qdq(x.float() * (one / g), aligned=True, global_sf_max=None) * g
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 30)):
                break
        return self.algo_bytes * n / el / 1e9, f"full [4096,4096] tensor x{n} (torch ops, fp32)"


def attention_inputs(rank=0):
    g = torch.Generator().manual_seed(1 + rank)
    q = torch.randn(1, 32, 4096, 128, generator=g).bfloat16()
    k = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    v = torch.randn(1, 8, 4096, 128, generator=g).bfloat16()
    return q, k, v


class AttentionWorkload:
    name = "attention"
    metric = "NVFP4 attention forward TFLOP/s per B200, % of dense FP4 tensor peak"
    unit = "TFLOP/s"
    dtype = ("nvfp4 QK^T (tcgen05 mxf4nvf4) + fp16 Phat (exact) x Vhat rounded once to fp16 (tcgen05 f16; exact "
             "hi+lo Vhat for the first 128 queries), fp32 accumulate")
    FLAGS = 4 | 8  # FP4ATTN_OUT_BF16 | FP4ATTN_PV_FP16
    B, Hq, Hkv, T, D = 1, 32, 8, 4096, 128

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        from fp4_attn_b200 import shard
        self.flops = 4 * self.B * self.Hq * self.T * self.T * self.D / 2  # causal, algorithmic, per rank
        # weak scaling: the job is a batch of `world` such problems; rank r owns batch row r,
        # i.e. its 8 (batch, kv-head) units (fp4_attn_b200.shard), with inputs from seed 1 + r
        units = shard.attention_shard(world, self.Hq, self.Hkv, world, rank)
        assert all(u.b == rank for u in units) and len(units) == self.Hkv
        self.config = {"workload": "NVFP4 attention fwd, Llama-3-8B shape: B=1, Hq=32, Hkv=8, D=128, T=4096, "
                                   "causal, single-slice Q/P quantization, bf16 output",
                       "flops_per_step": self.flops, "global_batch": world,
                       "shard": "batch row r (its 8 (batch, kv-head) units) on rank r, seed 1 + r"}
        if cpu_only:
            return
        from fp4_attn_b200 import attention as A
        self.A = A
        self.dev = dev
        q, k, v = attention_inputs(rank)
        self.host = [t.pin_memory() for t in (q, k, v)]
        per_set = sum(t.numel() * 2 for t in (q, k, v))
        self.nsets = max(2, int(2 * L2_BYTES // per_set) + 1)
        self.sets = [tuple(t.to(dev) for t in (q, k, v)) for _ in range(self.nsets)]
        self.ws = [A.AttentionWorkspace(self.B, self.Hq, self.Hkv, self.T, self.D, dev) for _ in range(self.nsets)]
        self.out = [torch.empty(self.B, self.T, self.Hq, self.D, device=dev, dtype=torch.bfloat16)
                    for _ in range(self.nsets)]
        self.out_bf16 = self.out
        self.out_host = torch.empty(self.B, self.T, self.Hq, self.D, dtype=torch.bfloat16).pin_memory()
        self.config["l2"] = f"rotating {self.nsets} input sets (> L2)"

    use_graph = True  # each step (one C ABI call, several launches on forked streams) is a CUDA graph replay

    def step(self, i, ev=None):
        """One fp4attn_forward call: Q/K quantize and V-hat prep (K and V on forked streams), then the kernel."""
        from fp4_attn_b200 import _lib
        i %= self.nsets
        q, k, v = self.sets[i]
        ws = self.ws[i]
        _lib.call("fp4attn_forward_ex", q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.DTYPE_CODE[q.dtype], self.B,
                  self.Hq, self.Hkv, self.T, self.D, q.stride(0), q.stride(1), q.stride(2), k.stride(0),
                  k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2), 1, self.D ** -0.5,
                  self.FLAGS, self.out[i].data_ptr(), ws.ptr(), ws.nbytes, _lib.stream_of(q))

    def kernel(self, i):
        """The contraction kernels alone (row maxima, then attention) on the operands step(i) prepared."""
        from fp4_attn_b200 import _lib
        i %= self.nsets
        ws = self.ws[i]
        _lib.call("fp4attn_fwd_packed_heads", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), None, None,
                  None, ws.kc.data_ptr(), ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(),
                  ws.row_max.data_ptr(), self.out[i].data_ptr(), self.B, self.Hq, self.Hkv, self.T, ws.Tp, self.D,
                  0, self.Hkv, 1, self.D ** -0.5, self.FLAGS, _lib.stream_of(self.sets[i][0]))

    def e2e_step(self, i):
        """Public API, host buffers: H2D q/k/v, fp4_attention_fwd (bf16 out, the reference's output
        dtype), D2H the output; steps pipelined over copy and compute streams."""
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets
        q, k, v = self.sets[i]

        def h2d():
            for d, h in zip((q, k, v), self.host):
                d.copy_(h, non_blocking=True)

        self.pipe.step(i, h2d, lambda: self.A.fp4_attention_fwd(q, k, v, causal=True, workspace=self.ws[i],
                                                                 out=self.out_bf16[i], out_dtype=torch.bfloat16,
                                                                 pv_fp16=True),
                       lambda o: self.out_host.copy_(o, non_blocking=True))

    e2e_h2d = property(lambda self: sum(t.numel() * 2 for t in self.host))
    e2e_d2h = property(lambda self: self.out_host.numel() * 2)

    def value(self, seconds_per_step, world):
        return world * self.flops / seconds_per_step / 1e12

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        achieved = self.flops / kernel_s / 1e12
        peak, src = fp4_peak(peaks, peak_src)
        return {"bound": "tensor", "kernel": "fp4_rowmax_t_kernel + fp4_attn_pingpong_kernel",
                "achieved": round(achieved, 1),
                "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_source": src,
                "frac_of_nominal_fp4": round(achieved / 9000.0, 4),
                "algorithmic_flops_per_launch": self.flops,
                "traffic": profile_traffic("fp4_attn_pingpong_kernel_llama3-8b_T4096"),
                "traffic_source": "profiles/fp4_attn_pingpong_kernel_llama3-8b_T4096.md: ncu dram__bytes_read+write "
                                  "per launch of both kernels"}

    def cpu_sample(self, reps=None):
        """The reference's CPU path (torch ops) on one KV-head group (4 of 32 query heads)."""
        from oracle import torch_port as tp
        q, k, v = attention_inputs()
        q, k, v = q[:, :4], k[:, :1], v[:, :1]
        flops = 4 * 4 * self.T * self.T * self.D / 2
        t0 = time.perf_counter()
        n = 0
        while True:
            tp.attention(q, k, v, causal=True)
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 5)):
                break
        return flops * n / el / 1e12, f"1 of 8 KV-head groups (4 query heads, all 4096 rows) x{n}, torch ops fp32"


# ----------------------------------------------------------------- timing
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world, dev):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def measure(wl, K, W, world, rank, dev, peaks, peak_src, cpu_baseline=True):
    """Time one workload: W untimed warm-up steps, K timed steps (device resident, barrier and
    synchronize on both sides, max over ranks), the dominant kernel alone, K end-to-end steps
    through the public API with host buffers, and (rank 0 at N=1) the CPU baseline sample."""
    from fp4_attn_b200 import _lib
    for i in range(W):
        wl.step(i)
    torch.cuda.synchronize(dev)

    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graphs, kgraphs = [], []
    if getattr(wl, "use_graph", False):
        # each step replays a CUDA graph of its launches, so host-side launch cost does not
        # starve the GPU; the dominant kernel is timed from its own graph replays right after
        stream = torch.cuda.Stream(dev)
        wl.stream = stream.cuda_stream
        with torch.cuda.stream(stream):
            for i in range(wl.nsets):
                wl.step(i)
            torch.cuda.synchronize(dev)
            c0 = _lib.launch_count()
            for i in range(wl.nsets):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    wl.step(i)
                graphs.append(g)
            per_step = (_lib.launch_count() - c0) // wl.nsets
            for i in range(wl.nsets):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    wl.kernel(i)
                kgraphs.append(g)
            for i in range(wl.nsets):
                graphs[i].replay()
            torch.cuda.synchronize(dev)
            barrier(world)
            torch.cuda.synchronize(dev)
            with Clocks(dev) as clk:
                start.record()
                for i in range(K):
                    graphs[(W + i) % wl.nsets].replay()
                end.record()
                torch.cuda.synchronize(dev)
            launches = per_step * K
            for i in range(K):
                kev[i][0].record()
                kgraphs[(W + i) % wl.nsets].replay()
                kev[i][1].record()
            torch.cuda.synchronize(dev)
        barrier(world)
    else:
        barrier(world)
        torch.cuda.synchronize(dev)
        n0 = _lib.launch_count()
        with Clocks(dev) as clk:
            start.record()
            for i in range(K):
                wl.step(W + i, kev[i])
            end.record()
            torch.cuda.synchronize(dev)
        launches = _lib.launch_count() - n0
        barrier(world)
    ms = start.elapsed_time(end)
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / K
    ms_max = max_over_ranks(ms, world, dev)
    kernel_ms_max = max_over_ranks(kernel_ms, world, dev)
    sec_per_step = ms_max / 1e3 / K
    del graphs, kgraphs

    # end to end through the public API with host buffers
    for i in range(2):
        wl.e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if hasattr(wl, "pipe"):
        wl.pipe.begin()
    for i in range(K):
        wl.e2e_step(i)
    if hasattr(wl, "pipe"):
        wl.pipe.join()
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    barrier(world)

    cpu = None
    if cpu_baseline and rank == 0 and world == 1:
        v, sample = wl.cpu_sample()
        cpu = {"value": round(v, 4), "unit": wl.unit, "cores": torch.get_num_threads(), "kind": "port",
               "sample": sample}
    return {
        "metric": wl.metric, "value": round(wl.value(sec_per_step, world), 3), "unit": wl.unit,
        "ms_per_step": round(ms_max / K, 5), "scaling": getattr(wl, "scaling", "weak"), "dtype": wl.dtype,
        "config": dict(wl.config, timing="CUDA graph replay per step" if getattr(wl, "use_graph", False)
                       else "stream launches"),
        "roofline": wl.kernel_roofline(kernel_ms_max / 1e3, peaks, peak_src),
        "cpu_baseline": cpu,
        "e2e": {"value": round(wl.value(e2e_ms / 1e3 / K, world), 3), "unit": wl.unit,
                "h2d_bytes_per_step": wl.e2e_h2d, "d2h_bytes_per_step": wl.e2e_d2h},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }


# the default run: the long-context prefill as the headline, the other graded configurations beside it
SUITE_PRIMARY = "prefill"
SUITE_SECONDARY = (("llama3_8b_attention", "attention"), ("quantize_4096x4096", "quantize"),
                   ("weights_llama3_70b", "weights"))


def run_ours(args, world, rank, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, peak_src = measured_peaks()
    peaks = dict(peaks)
    fp4, fp4_mhz = measure_fp4_peak(dev)
    peaks["fp4_tflops"] = max_over_ranks(-fp4, world, dev) * -1  # the slowest rank's (min over ranks)
    peaks["fp4_mhz"] = fp4_mhz
    K, W = args.steps, args.warmup
    suite = args.workload is None
    name = SUITE_PRIMARY if suite else args.workload
    wl = make_workload(name, dev, rank=rank, world=world, layers=args.layers)
    res = measure(wl, K, W, world, rank, dev, peaks, peak_src, cpu_baseline=not args.no_cpu_baseline)
    del wl
    torch.cuda.empty_cache()
    par = ("strong: the fixed job split over ranks" if res["scaling"] == "strong" else "weak: one shard per rank")
    line = {
        "metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": res["scaling"],
        "vs_baseline": None, "dtype": res["dtype"],
        "data": "synthetic (seeded; shapes/distributions of the named configuration)",
        "config": dict(res["config"], parallelism=f"{world} shard(s), {par}, no data-path collective"),
        "roofline": res["roofline"], "cpu_baseline": res["cpu_baseline"], "e2e": res["e2e"],
        "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
        "fp4_peak": {"tflops": round(peaks["fp4_tflops"], 1), "sm_mhz": fp4_mhz,
                     "how": "fp4_mma_peak_run: one CTA per SM, back-to-back tcgen05 mxf4nvf4 M128 N128 K64, "
                            "best of 5 event-timed launches, min over ranks"},
    }
    if suite:
        for key, wname in SUITE_SECONDARY:
            w2 = make_workload(wname, dev, rank=rank, world=world, layers=args.layers)
            r2 = measure(w2, K, W, world, rank, dev, peaks, peak_src, cpu_baseline=not args.no_cpu_baseline)
            line["gpu_launches"] += r2["gpu_launches"]
            line[key] = r2
            del w2
            torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference(args, world, rank):
    """The reference's CPU path (torch ops) on the host cores, rank 0 only."""
    if rank != 0:
        return
    suite = args.workload is None
    wl_name = SUITE_PRIMARY if suite else args.workload
    wl = make_workload(wl_name, None, cpu_only=True, world=world, layers=args.layers)
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        wl.cpu_sample(reps=1)
    vals = []
    for _ in range(args.steps):
        v, sample = wl.cpu_sample(reps=1)
        vals.append(v)
    v = statistics.median(vals)
    par = "strong: the fixed job split over ranks" if getattr(wl, "scaling", "weak") == "strong" else \
        "weak: one shard per rank"
    line = {
        "metric": wl.metric, "value": round(v, 5), "unit": wl.unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None,
        "dtype": wl.dtype, "data": "synthetic (seeded; shapes/distributions of the named configuration)",
        "config": dict(wl.config, parallelism=f"reference CPU path on rank 0's host cores ({par} on the GPU arm)"),
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 5), "unit": wl.unit, "kind": "port", "cores": torch.get_num_threads(),
                         "sample": sample},
        "e2e": {"value": round(v, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if suite:
        for key, wname in SUITE_SECONDARY:
            w2 = make_workload(wname, None, cpu_only=True, world=world, layers=args.layers)
            v2, s2 = w2.cpu_sample()
            line[key] = {"metric": w2.metric, "value": round(v2, 5), "unit": w2.unit, "config": w2.config,
                         "cpu_baseline": {"value": round(v2, 5), "unit": w2.unit, "kind": "port",
                                          "cores": torch.get_num_threads(), "sample": s2}}
    print(json.dumps(line), flush=True)


class DecodeWorkload:
    name = "decode"
    metric = "NVFP4 KV-cache decode attention GB/s per B200 (cache bytes read per step)"
    unit = "GB/s"
    dtype = "nvfp4 K/V cache, tcgen05 mxf4nvf4 QK^T, tcgen05 fp16 V-hat x (P-hat g_v as hi + lo)"
    B, Hq, Hkv, T, D = 8, 32, 8, 32768, 128
    use_graph = True

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        # per (token, KV head): K codes 64 B + K scales 8 B + V codes 64 B + V scales 8 B (one per
        # 16-token group: the appends are whole groups); per token: g_k, g_v
        self.cache_bytes = self.B * self.Hkv * self.T * (64 + 8 + 64 + 8) + 2 * self.B * self.T * 4
        self.config = {"workload": f"NVFP4 KV-cache decode: B={self.B}, Hq=32, Hkv=8, D=128, 32768 cached tokens "
                                   "(appended in calls of 4096, so V scales are read per 16-token group), "
                                   "one new query token per sequence",
                       "cache_bytes": self.cache_bytes, "global_batch": world * self.B,
                       "shard": f"batch rows {self.B}r..{self.B}r+{self.B - 1} on rank r (own cache, seed 2 + r)",
                       "l2": f"cache bytes read {self.cache_bytes / 1e6:.0f} MB > L2"}
        if cpu_only:
            return
        from fp4_attn_b200 import _lib
        from fp4_attn_b200.kv_cache import NVFP4KVCache
        self.lib = _lib
        self.dev = dev
        g = torch.Generator().manual_seed(2 + rank)
        self.cache = NVFP4KVCache(self.B, self.Hkv, self.T, self.D, dev)
        for _ in range(self.T // 4096):
            k = torch.randn(self.B, self.Hkv, 4096, self.D, generator=g).bfloat16().to(dev)
            v = torch.randn(self.B, self.Hkv, 4096, self.D, generator=g).bfloat16().to(dev)
            self.cache.append(k, v)
        self.nsets = 4
        self.q_host = torch.randn(self.B, self.Hq, 1, self.D, generator=g).bfloat16().pin_memory()
        self.qs = [torch.randn(self.B, self.Hq, 1, self.D, generator=g).bfloat16().to(dev) for _ in range(self.nsets)]
        self.ws = torch.empty(_lib.load().fp4attn_decode_workspace_size(self.B, self.Hq, self.T), dtype=torch.uint8,
                              device=dev)
        self.out_host = torch.empty(self.B, 1, self.Hq, self.D).pin_memory()

    def step(self, i, ev=None):
        from fp4_attn_b200.kv_cache import decode_attention
        decode_attention(self.qs[i % self.nsets], self.cache, workspace=self.ws)

    def kernel(self, i):
        self.step(i)

    def e2e_step(self, i):
        """Public API, host buffers: H2D the new query tokens, decode, D2H the output."""
        from fp4_attn_b200.kv_cache import decode_attention
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets
        self.pipe.step(i, lambda: self.qs[i].copy_(self.q_host, non_blocking=True),
                       lambda: decode_attention(self.qs[i], self.cache, workspace=self.ws),
                       lambda o: self.out_host.copy_(o, non_blocking=True))

    e2e_h2d = property(lambda self: self.q_host.numel() * 2)
    e2e_d2h = property(lambda self: self.out_host.numel() * 4)

    def value(self, seconds_per_step, world):
        return world * self.cache_bytes / seconds_per_step / 1e9

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        achieved = self.cache_bytes / kernel_s / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "kernel": "decode step (query quantize, scores, pv, combine)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_src} copy bandwidth", "algorithmic_bytes_per_launch": self.cache_bytes,
                "traffic": profile_traffic("decode_pv_kernel_B8_T32768"),
                "traffic_source": "profiles/decode_pv_kernel_B8_T32768.md: ncu dram bytes of decode_pv_kernel"}

    def cpu_sample(self, reps=None):
        """The reference's CPU path (torch ops): one sequence, one KV-head group, 4096 cached keys."""
        from oracle import torch_port as tp
        g = torch.Generator().manual_seed(2)
        L = 4096
        q = torch.randn(1, 4, 1, self.D, generator=g).bfloat16()
        k = torch.randn(1, 1, L, self.D, generator=g).bfloat16()
        v = torch.randn(1, 1, L, self.D, generator=g).bfloat16()
        # the cache's values: K row mode, V along tokens (column mode on the transposed view)
        Kf = tp.fused_qdq(k.reshape(L, self.D).float()).view(1, 1, L, self.D)
        Vf = tp.fused_qdq(v.reshape(L, self.D).float().T, aligned=False).T.reshape(1, 1, L, self.D)
        sample_bytes = L * (64 + 8 + 64 + 128 + 8)
        t0 = time.perf_counter()
        n = 0
        while True:
            Qf = tp.fused_qdq(q.reshape(1, -1).float()).view(1, 4, 1, self.D)
            tp.eager_attention(Qf, Kf, Vf, False, self.D ** -0.5)
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 200)):
                break
        return sample_bytes * n / el / 1e9, f"1 sequence x 1 KV-head group (4 query heads) x 4096 keys, x{n}"


class QkvWorkload:
    name = "qkv"
    metric = "Q/K projection + RoPE + NVFP4 quantize TFLOP/s per B200"
    unit = "TFLOP/s"
    dtype = "bf16 projection (tcgen05 kind::f16, fp32 accumulate) -> bf16 RoPE -> nvfp4"
    T, K, Hq, Hkv, D = 4096, 4096, 32, 8, 128
    use_graph = True

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        self.flops = 2 * self.T * self.K * (self.Hq + self.Hkv) * self.D
        self.config = {"workload": "Llama-3-8B layer Q/K projections fused with RoPE and NVFP4 quantize: "
                                   "T=4096 tokens, hidden 4096, 32 + 8 heads of 128",
                       "flops_per_step": self.flops, "global_batch": world,
                       "shard": "one sequence of 4096 tokens per rank (seed 3 + r)"}
        if cpu_only:
            return
        self.dev = dev
        g = torch.Generator().manual_seed(3 + rank)
        per_set = self.T * self.K * 2
        self.nsets = max(2, int(2 * L2_BYTES // per_set) + 1)
        self.x_host = torch.randn(self.T, self.K, generator=g).bfloat16().pin_memory()
        self.xs = [self.x_host.to(dev) for _ in range(self.nsets)]
        self.wq = (torch.randn(self.Hq * self.D, self.K, generator=g) * 0.02).bfloat16().to(dev)
        self.wk = (torch.randn(self.Hkv * self.D, self.K, generator=g) * 0.02).bfloat16().to(dev)
        inv = 1.0 / (10000.0 ** (torch.arange(0, self.D, 2, dtype=torch.float32) / self.D))
        ang = torch.arange(self.T, dtype=torch.float32)[:, None] * inv[None, :]
        emb = torch.cat((ang, ang), -1)
        self.cos, self.sin = emb.cos().bfloat16().to(dev), emb.sin().bfloat16().to(dev)
        self.qbuf = [self._bufs(self.Hq) for _ in range(self.nsets)]
        self.kbuf = [self._bufs(self.Hkv) for _ in range(self.nsets)]
        self.codes_host = torch.empty(self.T, self.Hq * self.D // 2, dtype=torch.uint8).pin_memory()
        self.config["l2"] = f"rotating {self.nsets} hidden-state sets (> L2)"

    def _bufs(self, H):
        d = self.dev
        return (torch.empty(self.T, H * self.D // 2, dtype=torch.uint8, device=d),
                torch.empty(self.T // 128 * H * 2 * 512, dtype=torch.uint8, device=d),
                torch.empty(self.T, dtype=torch.float32, device=d))

    def step(self, i, ev=None):
        from fp4_attn_b200.qkv import rope_quant_projection
        i %= self.nsets
        rope_quant_projection(self.xs[i], self.wq, self.cos, self.sin, self.T, *self.qbuf[i])
        rope_quant_projection(self.xs[i], self.wk, self.cos, self.sin, self.T, *self.kbuf[i])

    def kernel(self, i):
        from fp4_attn_b200.qkv import rope_quant_projection
        i %= self.nsets
        rope_quant_projection(self.xs[i], self.wq, self.cos, self.sin, self.T, *self.qbuf[i])

    def e2e_step(self, i):
        """Public API, host buffers: H2D the hidden states, both projections, D2H the packed Q codes."""
        from fp4_attn_b200.qkv import rope_quant_projection
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets

        def compute():
            rope_quant_projection(self.xs[i], self.wk, self.cos, self.sin, self.T, *self.kbuf[i])
            return rope_quant_projection(self.xs[i], self.wq, self.cos, self.sin, self.T, *self.qbuf[i])

        self.pipe.step(i, lambda: self.xs[i].copy_(self.x_host, non_blocking=True), compute,
                       lambda r: self.codes_host.copy_(r[0], non_blocking=True))

    e2e_h2d = property(lambda self: self.x_host.numel() * 2)
    e2e_d2h = property(lambda self: self.codes_host.numel())

    def value(self, seconds_per_step, world):
        return world * self.flops / seconds_per_step / 1e12

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        fl = 2 * self.T * self.K * self.Hq * self.D
        achieved = fl / kernel_s / 1e12
        peak = peaks["bf16_tflops"]
        return {"bound": "tensor", "kernel": "qkv_rope_quant_kernel (Q projection, 32 heads)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_src} dense bf16", "algorithmic_flops_per_launch": fl,
                "traffic": profile_traffic("qkv_rope_quant_kernel_T4096_hidden4096_Hq32"),
                "traffic_source": "profiles/qkv_rope_quant_kernel_T4096_hidden4096_Hq32.md: ncu dram bytes"}

    def cpu_sample(self, reps=None):
        """The reference's CPU path (torch ops): projection, bf16 RoPE and the quantizer on 256 tokens."""
        from oracle import torch_port as tp
        g = torch.Generator().manual_seed(3)
        n_tok = 256
        x = torch.randn(n_tok, self.K, generator=g).bfloat16()
        w = (torch.randn((self.Hq + self.Hkv) * self.D, self.K, generator=g) * 0.02).bfloat16()
        inv = 1.0 / (10000.0 ** (torch.arange(0, self.D, 2, dtype=torch.float32) / self.D))
        ang = torch.arange(n_tok, dtype=torch.float32)[:, None] * inv[None, :]
        emb = torch.cat((ang, ang), -1)
        cos, sin = emb.cos().bfloat16()[:, None], emb.sin().bfloat16()[:, None]
        fl = 2 * n_tok * self.K * (self.Hq + self.Hkv) * self.D
        t0 = time.perf_counter()
        n = 0
        while True:
            y = torch.nn.functional.linear(x, w).view(n_tok, -1, self.D)
            rot = torch.cat((-y[..., 64:], y[..., :64]), -1)
            z = (y * cos) + (rot * sin)
            tp.fused_qdq(z[:, :self.Hq].reshape(n_tok, -1).float())
            tp.fused_qdq(z[:, self.Hq:].reshape(n_tok, -1).float())
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 20)):
                break
        return fl * n / el / 1e12, f"256 tokens (of 4096), both projections x{n}, torch bf16 ops + fp32 quantizer"


class PrefillWorkload(AttentionWorkload):
    """Long-context prefill, strong scaling: the fixed job of 4 x 8 (batch, KV-head) units is split
    over the ranks in contiguous (batch rows) x (KV heads) blocks (fp4_attn_b200.shard).  A rank
    quantizes Q/K/V on every head of its batch rows -- the per-token global scales span the whole
    [B*T, H*D] row -- and attends its own KV heads, so the job's result does not depend on N."""
    name = "prefill"
    metric = "NVFP4 attention forward TFLOP/s (long-context prefill), % of dense FP4 tensor peak"
    scaling = "strong"
    B_JOB, Hq_JOB, Hkv_JOB, T, D = 4, 64, 8, 32768, 128

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        from fp4_attn_b200 import shard
        units = shard.attention_shard(self.B_JOB, self.Hq_JOB, self.Hkv_JOB, world, rank)
        rows, (self.h0, self.h1) = shard.shard_rows(units)
        G = self.Hq_JOB // self.Hkv_JOB
        self.b0, self.b1 = rows.start, rows.stop
        self.B, self.Hkv, self.Hq = self.b1 - self.b0, self.Hkv_JOB, self.Hq_JOB  # operands: whole rows
        self.flops = 4 * self.B * (self.h1 - self.h0) * G * self.T * self.T * self.D / 2  # this rank's units
        self.config = {"workload": "NVFP4 attention fwd, long-context prefill: B=4, Hq=64, Hkv=8, D=128, T=32768, "
                                   "causal, q/k/v N(0,1)*0.5 with a per-(kv-head, channel) N(0,2) bias on k, "
                                   "single-slice Q/P quantization, bf16 output",
                       "flops_job": 4 * self.B_JOB * self.Hq_JOB * self.T * self.T * self.D / 2,
                       "flops_per_step": self.flops,
                       "global_batch": self.B_JOB,
                       "shard": f"units (b {self.b0}..{self.b1 - 1}) x (kv-head {self.h0}..{self.h1 - 1}) on rank "
                                f"{rank}; Q/K/V quantized on every head of those batch rows (per-token scales "
                                f"over the whole row, as unsharded)"}
        if cpu_only:
            return
        from fp4_attn_b200 import attention as A
        self.A = A
        self.dev = dev
        g = torch.Generator(dev).manual_seed(2)  # the whole job's inputs on every rank, then this rank's rows
        q = torch.randn(self.B_JOB, self.Hq_JOB, self.T, self.D, device=dev, generator=g) * 0.5
        q = q[self.b0:self.b1].bfloat16()
        k = torch.randn(self.B_JOB, self.Hkv_JOB, self.T, self.D, device=dev, generator=g) * 0.5
        bias = torch.randn(self.Hkv_JOB, self.D, device=dev, generator=g) * 2.0
        k = (k + bias[None, :, None, :])[self.b0:self.b1].bfloat16()
        v = (torch.randn(self.B_JOB, self.Hkv_JOB, self.T, self.D, device=dev, generator=g) * 0.5)
        v = v[self.b0:self.b1].bfloat16()
        self.host = [t.cpu().pin_memory() for t in (q, k, v)]
        self.nsets = 2  # inputs (2.7 GB at one rank) are far larger than L2; two sets let e2e copies overlap
        self.sets = [(q, k, v)] + [tuple(t.clone() for t in (q, k, v)) for _ in range(self.nsets - 1)]
        del q, k, v
        self.ws = [A.AttentionWorkspace(self.B, self.Hq, self.Hkv, self.T, self.D, dev) for _ in range(self.nsets)]
        Ho = (self.h1 - self.h0) * G
        self.out = [torch.empty(self.B, self.T, Ho, self.D, device=dev, dtype=torch.bfloat16)
                    for _ in range(self.nsets)]
        self.out_bf16 = self.out
        self.out_host = torch.empty(self.B, self.T, Ho, self.D, dtype=torch.bfloat16).pin_memory()
        self.config["l2"] = "inputs > L2 (2.7 GB per set at one rank)"

    def step(self, i, ev=None):
        """One fp4attn_forward_heads call: quantize the rank's batch rows, attend its KV heads."""
        from fp4_attn_b200 import _lib
        i %= self.nsets
        q, k, v = self.sets[i]
        ws = self.ws[i]
        _lib.call("fp4attn_forward_heads", q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.DTYPE_CODE[q.dtype],
                  self.B, self.Hq, self.Hkv, self.T, self.D, q.stride(0), q.stride(1), q.stride(2), k.stride(0),
                  k.stride(1), k.stride(2), v.stride(0), v.stride(1), v.stride(2), 1, self.D ** -0.5,
                  self.FLAGS, self.h0, self.h1, self.out[i].data_ptr(), ws.ptr(), ws.nbytes,
                  _lib.stream_of(q))

    def kernel(self, i):
        """The attention kernel alone on the operands step(i) prepared, this rank's KV heads."""
        from fp4_attn_b200 import _lib
        i %= self.nsets
        ws = self.ws[i]
        _lib.call("fp4attn_fwd_packed_heads", ws.qc.data_ptr(), ws.qs.data_ptr(), ws.gq.data_ptr(), None, None,
                  None, ws.kc.data_ptr(), ws.ks.data_ptr(), ws.gk.data_ptr(), ws.vhi.data_ptr(), ws.vlo.data_ptr(),
                  ws.row_max.data_ptr(), self.out[i].data_ptr(), self.B, self.Hq, self.Hkv, self.T, ws.Tp, self.D,
                  self.h0, self.h1, 1, self.D ** -0.5, self.FLAGS, _lib.stream_of(self.sets[i][0]))

    def e2e_step(self, i):
        """Public API, host buffers: H2D q/k/v of the rank's rows, fp4_attention_fwd on its KV heads
        (bf16 out), D2H the output; steps pipelined over copy and compute streams."""
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets
        q, k, v = self.sets[i]

        def h2d():
            for d, h in zip((q, k, v), self.host):
                d.copy_(h, non_blocking=True)

        self.pipe.step(i, h2d, lambda: self.A.fp4_attention_fwd(q, k, v, causal=True, workspace=self.ws[i],
                                                                 out=self.out_bf16[i], out_dtype=torch.bfloat16,
                                                                 kv_heads=(self.h0, self.h1), pv_fp16=True),
                       lambda o: self.out_host.copy_(o, non_blocking=True))

    def value(self, seconds_per_step, world):
        return world * self.flops / seconds_per_step / 1e12

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        r = super().kernel_roofline(kernel_s, peaks, peak_src)
        r["traffic"], r["traffic_source"] = None, ("not captured at this shape (launch list only: "
                                                   "profiles/attention_prefill_B4_Hq64_T32768_launches.md)")
        return r

    def cpu_sample(self, reps=None):
        """The reference's CPU path (torch ops) on the last 256 query rows of one KV-head group (8 query
        heads) of batch row 0 against all 32768 keys; that head's K/V fake-quant runs in every repetition."""
        from oracle import torch_port as tp
        L, rows, G, D = self.T, 256, self.Hq_JOB // self.Hkv_JOB, self.D
        g = torch.Generator().manual_seed(2)
        q = (torch.randn(rows, G * D, generator=g) * 0.5).bfloat16()
        k = (torch.randn(L, D, generator=g) * 0.5 + torch.randn(D, generator=g) * 2.0).bfloat16()
        v = (torch.randn(L, D, generator=g) * 0.5).bfloat16()
        flops = 4 * D * G * sum(t + 1 for t in range(L - rows, L))
        Qf = torch.zeros(1, G, L, D)
        t0 = time.perf_counter()
        n = 0
        while True:
            Qf[0, :, L - rows:] = tp.fused_qdq(q.float()).view(rows, G, D).transpose(0, 1)
            Kf = tp.fused_qdq(k.float()).view(1, 1, L, D)
            Vf = tp.fused_qdq(v.float().T, aligned=False).T.reshape(1, 1, L, D)
            tp.eager_attention(Qf, Kf, Vf, True, D ** -0.5, q_rows=slice(L - rows, L))
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 5)):
                break
        return flops * n / el / 1e12, f"1 KV-head group (8 query heads), last {rows} of 32768 query rows x{n}"


LAYER_70B = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192),
             ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]


class WeightsWorkload:
    """Per-tensor NVFP4 quantization of the linear weights of a Llama-3-70B-shaped stack.  Weak
    scaling by whole layers: rank r quantizes layers 10r..10r+9, so 8 ranks cover the 80 layers
    with no exchange (each tensor's max is reduced on the rank that holds it)."""
    name = "weights"
    metric = "NVFP4 weight quantize GB/s per B200 (Llama-3-70B-shaped stack), % of HBM roofline"
    unit = "GB/s"
    dtype = "bf16->nvfp4 (fp32 arithmetic)"
    LAYERS_PER_RANK = 10
    use_graph = True

    def __init__(self, dev, cpu_only=False, rank=0, world=1, layers=10):
        self.LAYERS_PER_RANK = layers
        per_layer = sum(m * n for _, m, n in LAYER_70B)
        self.elems = self.LAYERS_PER_RANK * per_layer
        self.algo_bytes = self.elems * (2 + 0.5 + 1 / 16)
        l0 = rank * self.LAYERS_PER_RANK
        self.config = {"workload": "NVFP4 quantize of the linear weights of Llama-3-70B layers (q/o 8192x8192, "
                                   "k/v 1024x8192, gate/up 28672x8192, down 8192x28672), bf16 N(0,0.02), "
                                   "per-tensor scale amax/2688, block 16",
                       "elements": self.elems, "layers": f"{l0}..{l0 + self.LAYERS_PER_RANK - 1}",
                       "global_batch": world * self.LAYERS_PER_RANK,
                       "shard": f"{layers} whole layers per rank (10 per rank at 8 ranks = the 80-layer stack), "
                                f"tensor t from seed 4 + t",
                       "l2": f"{layers * 1.71:.1f} GB of weights per rank > L2"}
        if cpu_only:
            return
        from fp4_attn_b200 import _lib
        self.lib = _lib
        self.dev = dev
        self.nsets = 1
        self.t = []  # (weight, codes, scales, g) per tensor
        for l in range(l0, l0 + self.LAYERS_PER_RANK):
            for idx, (_, m, n) in enumerate(LAYER_70B):
                gen = torch.Generator(dev).manual_seed(4 + 7 * l + idx)
                w = (torch.randn(m, n, device=dev, generator=gen) * 0.02).bfloat16()
                self.t.append((w, torch.empty(m, n // 2, dtype=torch.uint8, device=dev),
                               torch.empty(m, n // 16, dtype=torch.uint8, device=dev),
                               torch.empty(1, dtype=torch.float32, device=dev)))
        self.stream = torch.cuda.current_stream(dev).cuda_stream
        # e2e: one layer's tensors in pinned host memory, copied into every layer's device buffers
        self.host = [w.cpu().pin_memory() for w, *_ in self.t[:len(LAYER_70B)]]
        self.codes_host = [c.cpu().pin_memory() for _, c, *_ in self.t[:len(LAYER_70B)]]
        self.scales_host = [s.cpu().pin_memory() for _, _, s, _ in self.t[:len(LAYER_70B)]]

    def _quantize(self, w, codes, scales, g, gmode=3):
        m, n = w.shape
        self.lib.call("fp4q_quantize", w.data_ptr(), 1, 1, m, 1, n, 0, n, 0, m, gmode, 0, 2688.0, codes.data_ptr(),
                      n // 2, scales.data_ptr(), 0, n // 16, g.data_ptr(), None, 0, 0, self.stream)

    def step(self, i, ev=None):
        for w, c, s, g in self.t:
            self._quantize(w, c, s, g)

    def kernel(self, i):
        """The row kernel alone on one gate weight [28672, 8192] (its per-tensor g already reduced)."""
        self._quantize(*self.t[4], gmode=3 | 0x10)

    def e2e_step(self, i):
        """Public API, host buffers: H2D every weight, quant.quantize per tensor, D2H codes + scales."""
        from fp4_attn_b200 import quant
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(1)
        nl = len(LAYER_70B)

        def h2d():
            for j, (w, *_) in enumerate(self.t):
                w.copy_(self.host[j % nl], non_blocking=True)

        def compute():
            return [quant.quantize(w, "tensor", 2688.0) for w, *_ in self.t]

        def d2h(res):
            for j, pk in enumerate(res):
                self.codes_host[j % nl].copy_(pk.codes, non_blocking=True)
                self.scales_host[j % nl].copy_(pk.scales, non_blocking=True)

        self.pipe.step(0, h2d, compute, d2h)

    e2e_h2d = property(lambda self: self.elems * 2)
    e2e_d2h = property(lambda self: self.elems // 2 + self.elems // 16)

    def value(self, seconds_per_step, world):
        return world * self.algo_bytes / seconds_per_step / 1e9

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        m, n = LAYER_70B[4][1:]
        algo = m * n * (2 + 0.5 + 1 / 16)
        achieved = algo / kernel_s / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "kernel": "quant_rows_vec_kernel on a [28672, 8192] weight (g given)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_src} copy bandwidth", "algorithmic_bytes_per_launch": algo,
                "traffic": profile_traffic("quant_rows_vec_kernel_llama3-70b_weights"),
                "traffic_source": "profiles/quant_rows_vec_kernel_llama3-70b_weights.md: ncu dram bytes of an "
                                  "[8192, 8192] launch x 3.5"}

    def cpu_sample(self, reps=None):
        """The reference's CPU path (torch ops) on the k weight [1024, 8192] of layer 0, per-tensor scale."""
        from oracle import torch_port as tp
        g = torch.Generator().manual_seed(4 + 1)
        w = (torch.randn(1024, 8192, generator=g) * 0.02).bfloat16()
        one = torch.tensor(1.0)
        t0 = time.perf_counter()
        n = 0
        while True:
            gs = w.abs().max().float() * (one / torch.tensor(2688.0))
            tp.fused_qdq(w.float() * (one / gs), aligned=True, global_sf_max=None) * gs
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 30)):
                break
        return w.numel() * (2 + 0.5 + 1 / 16) * n / el / 1e9, f"k weight [1024, 8192] of layer 0 x{n} (torch ops)"


class GemmWorkload:
    """An FP4 linear layer: the activations quantized to NVFP4 (row mode) and multiplied by a
    per-tensor NVFP4 weight on tcgen05, Y = X W^T in fp32.  The weight is layer 0's gate
    projection of the Llama-3-70B-shaped stack (quantized once, as weights are)."""
    name = "gemm"
    metric = "NVFP4 GEMM TFLOP/s per B200 (Llama-3-70B gate projection), % of dense FP4 tensor peak"
    unit = "TFLOP/s"
    dtype = "nvfp4 x nvfp4 (tcgen05 kind::mxf4nvf4), fp32 accumulate and output"
    M, N, K = 8192, 28672, 8192
    use_graph = True

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        self.flops = 2 * self.M * self.N * self.K
        self.config = {"workload": "NVFP4 GEMM Y[8192, 28672] = X[8192, 8192] W^T: X bf16 N(0,1) quantized per "
                                   "token (row mode), W the gate weight of layer 0 (bf16 N(0,0.02), seed 4 + 4, "
                                   "per-tensor scale amax/2688), fp32 output",
                       "flops_per_step": self.flops, "global_batch": world,
                       "shard": "8192 tokens per rank (seed 40 + r), the weight on every rank"}
        if cpu_only:
            return
        from fp4_attn_b200 import _lib, quant
        self.lib, self.quant, self.dev = _lib, quant, dev
        gen = torch.Generator(dev).manual_seed(4 + 4)
        w = (torch.randn(self.N, self.K, device=dev, generator=gen) * 0.02).bfloat16()
        self.wq = quant.quantize(w, "tensor", 2688.0, scale_layout="tcgen05")
        self.gw = self.wq.g.expand(self.N).contiguous()
        del w
        gx = torch.Generator(dev).manual_seed(40 + rank)
        self.nsets = 2
        self.xs = [torch.randn(self.M, self.K, device=dev, generator=gx).bfloat16() for _ in range(self.nsets)]
        self.xq = [quant.quantize(x, "row", 1536.0, scale_layout="tcgen05") for x in self.xs]
        self.c = [torch.empty(self.M, self.N, device=dev) for _ in range(self.nsets)]
        self.x_host = self.xs[0].cpu().pin_memory()
        self.c_host = torch.empty(self.M, self.N).pin_memory()
        self.stream = torch.cuda.current_stream(dev).cuda_stream
        self.config["l2"] = f"weight codes 117 MB + {self.nsets} activation sets of 134 MB (> L2)"

    def _gemm(self, i):
        xq, wq = self.xq[i], self.wq
        self.lib.call("fp4_gemm_nvf4", xq.codes.data_ptr(), xq.scales.data_ptr(), xq.g.data_ptr(),
                      wq.codes.data_ptr(), wq.scales.data_ptr(), self.gw.data_ptr(), self.c[i].data_ptr(),
                      self.M, self.N, self.K, xq.codes.stride(0), wq.codes.stride(0), self.c[i].stride(0),
                      self.stream)

    def step(self, i, ev=None):
        """Quantize the activations (row mode, tcgen05 scale atoms) into their buffers, then the GEMM."""
        i %= self.nsets
        x, xq = self.xs[i], self.xq[i]
        self.lib.call("fp4q_quantize", x.data_ptr(), 1, 1, self.M, 1, self.K, 0, self.K, 0, self.M, 1, 0, 1536.0,
                      xq.codes.data_ptr(), self.K // 2, xq.scales.data_ptr(), 1, (self.K // 16 + 3) // 4,
                      xq.g.data_ptr(), None, 0, 0, self.stream)
        self._gemm(i)

    def kernel(self, i):
        self._gemm(i % self.nsets)

    def e2e_step(self, i):
        """Public API, host buffers: H2D the bf16 activations, quant.quantize + gemm_nvf4, D2H Y."""
        from fp4_attn_b200.gemm import gemm_nvf4
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(self.nsets)
        i %= self.nsets
        self.pipe.step(i, lambda: self.xs[i].copy_(self.x_host, non_blocking=True),
                       lambda: gemm_nvf4(self.quant.quantize(self.xs[i], "row", 1536.0, scale_layout="tcgen05"),
                                         self.wq),
                       lambda y: self.c_host.copy_(y, non_blocking=True))

    e2e_h2d = property(lambda self: self.M * self.K * 2)
    e2e_d2h = property(lambda self: self.M * self.N * 4)

    def value(self, seconds_per_step, world):
        return world * self.flops / seconds_per_step / 1e12

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        achieved = self.flops / kernel_s / 1e12
        peak, src = fp4_peak(peaks, peak_src)
        return {"bound": "tensor", "kernel": "gemm_nvf4_persistent", "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_source": src,
                "frac_of_nominal_fp4": round(achieved / 9000.0, 4), "algorithmic_flops_per_launch": self.flops,
                "traffic": profile_traffic("gemm_nvf4_kernel_8192x28672x8192"),
                "traffic_source": "profiles/gemm_nvf4_kernel_8192x28672x8192.md: ncu dram__bytes_read+write per launch"}

    def cpu_sample(self, reps=None):
        """The reference's way on the host cores: fake-quantized activations (torch ops) times the
        dequantized weight in an fp32 matmul, for 256 of the 8192 tokens."""
        from oracle import torch_port as tp
        if getattr(self, "_wd", None) is None:  # the weight's fake-quant is offline: once, not timed
            g = torch.Generator().manual_seed(4 + 4)
            w = (torch.randn(self.N, self.K, generator=g) * 0.02).bfloat16().float()
            one = torch.tensor(1.0)
            gw = w.abs().max() * (one / torch.tensor(2688.0))
            self._wd = tp.fused_qdq(w * (one / gw), aligned=True, global_sf_max=None) * gw
        wd = self._wd
        x = torch.randn(256, self.K, generator=torch.Generator().manual_seed(40)).bfloat16()
        t0 = time.perf_counter()
        n = 0
        while True:
            torch.matmul(tp.fused_qdq(x.float()), wd.T)
            n += 1
            el = time.perf_counter() - t0
            if (reps and n >= reps) or (not reps and (el > 10.0 or n >= 20)):
                break
        return 2 * 256 * self.N * self.K * n / el / 1e12, f"256 of 8192 tokens x{n} (torch fp32 matmul)"


def llama2_7b_config():
    from transformers import LlamaConfig
    return LlamaConfig(hidden_size=4096, intermediate_size=11008, num_hidden_layers=32, num_attention_heads=32,
                       num_key_value_heads=32, head_dim=128, vocab_size=32000, max_position_embeddings=4096,
                       rope_theta=10000.0, rms_norm_eps=1e-5, attn_implementation="eager")


class LlamaWorkload:
    """One forward pass of a Llama-2-7B-shaped model with the FP4 attention patch installed
    (fp4_attn_b200.llama_patch.install, as eval.py installs the reference's).  Strong scaling:
    the batch of 8 sequences is split over the ranks."""
    name = "llama"
    metric = "Llama-2-7B forward tokens/s per B200 with the NVFP4 attention patch"
    unit = "tokens/s"
    dtype = "bf16 model (torch GEMMs), NVFP4 attention (tcgen05), single-slice Q/P"
    scaling = "strong"
    B_JOB, T = 8, 2048
    use_graph = False  # the patched forward checks the mask and NaNs on the host every layer

    def __init__(self, dev, cpu_only=False, rank=0, world=1):
        if self.B_JOB % world:
            raise ValueError(f"{world} ranks do not split a batch of {self.B_JOB}")
        self.B = self.B_JOB // world
        self.b0 = rank * self.B
        self.attn_flops = 4 * self.B * 32 * self.T * self.T * 128 / 2  # one layer, causal
        self.config = {"workload": "Llama-2-7B (32 layers, hidden 4096, 32 heads MHA, SwiGLU 11008, vocab 32000), "
                                   "random bf16 weights N(0,0.02) from seed 3, FP4 attention patch, one forward "
                                   "of batch 8 x 2048 token ids (seed 3), use_cache=False",
                       "global_batch": self.B_JOB, "seq_len": self.T,
                       "shard": f"sequences {self.b0}..{self.b0 + self.B - 1} on rank {rank}",
                       "quant": "FP4_USE_DUAL_QUANT_Q=false, FP4_USE_DUAL_QUANT_ATTN=false"}
        os.environ["FP4_USE_DUAL_QUANT_Q"] = "false"
        os.environ["FP4_USE_DUAL_QUANT_ATTN"] = "false"
        if cpu_only:
            return
        from transformers import LlamaForCausalLM
        from fp4_attn_b200 import llama_patch as lp
        self.dev = dev
        self.lp = lp
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(dev):
                self.model = LlamaForCausalLM(llama2_7b_config())
        finally:
            torch.set_default_dtype(torch.float32)
        gen = torch.Generator(dev).manual_seed(3)
        with torch.no_grad():
            for prm in self.model.parameters():
                prm.normal_(0.0, 0.02, generator=gen)
        self.model.eval()
        ids = torch.randint(0, 32000, (self.B_JOB, self.T), generator=torch.Generator().manual_seed(3))
        self.ids_host = ids[self.b0:self.b0 + self.B].contiguous().pin_memory()
        self.ids = self.ids_host.to(dev)
        self.out_host = torch.empty(self.B, 32000, dtype=torch.bfloat16).pin_memory()
        self._ev = None

        def timed(module, *a, **kw):  # layer 0's attention call between the step's events
            if self._ev is not None and module.layer_idx == 0:
                self._ev[0].record()
                r = lp.fp4_eager_attention(module, *a, **kw)
                self._ev[1].record()
                return r
            return lp.fp4_eager_attention(module, *a, **kw)

        lp.attention_interface = timed
        lp.install()
        self.nsets = 1
        self.config["l2"] = "13.5 GB of weights per forward > L2"

    def _forward(self, ids):
        with torch.no_grad():
            return self.model(input_ids=ids, use_cache=False).logits

    def step(self, i, ev=None):
        self._ev = ev
        self._forward(self.ids)
        self._ev = None

    def kernel(self, i):
        self.step(i)

    def e2e_step(self, i):
        """Public API, host buffers: H2D the token ids, the patched forward, D2H the last position's logits."""
        if not hasattr(self, "pipe"):
            self.pipe = E2EPipe(1)
        self.pipe.step(0, lambda: self.ids.copy_(self.ids_host, non_blocking=True),
                       lambda: self._forward(self.ids)[:, -1], lambda o: self.out_host.copy_(o, non_blocking=True))

    e2e_h2d = property(lambda self: self.ids_host.numel() * 8)
    e2e_d2h = property(lambda self: self.out_host.numel() * 2)

    def value(self, seconds_per_step, world):
        return world * self.B * self.T / seconds_per_step

    def kernel_roofline(self, kernel_s, peaks, peak_src):
        achieved = self.attn_flops / kernel_s / 1e12
        peak, src = fp4_peak(peaks, peak_src)
        return {"bound": "tensor", "kernel": "layer 0's FP4 attention call (Q/K quantize, V-hat prep, fp4_attn_kernel)",
                "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "peak_source": src,
                "algorithmic_flops_per_launch": self.attn_flops, "traffic": None,
                "traffic_source": "not captured at this shape"}

    def cpu_sample(self, reps=None):
        """The reference's CPU path: one decoder layer (torch ops, FP4 attention simulated with the
        reference's fake-quant) on one 2048-token sequence, plus the LM head; x32 layers."""
        from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
        from fp4_attn_b200 import llama_patch as lp
        from oracle import torch_port as tp
        cfg = llama2_7b_config()
        torch.manual_seed(3)
        torch.set_default_dtype(torch.bfloat16)
        try:
            layer = LlamaDecoderLayer(cfg, layer_idx=0).eval()
            head = torch.nn.Linear(4096, 32000, bias=False)
        finally:
            torch.set_default_dtype(torch.float32)
        rot = LlamaRotaryEmbedding(cfg)
        h = (torch.randn(1, self.T, 4096) * 0.02).bfloat16()
        pe = rot(h, torch.arange(self.T)[None])

        def cpu_attn(module, q, k, v, mask, scaling, dropout=0.0, **kw):
            return tp.attention(q, k, v, True, float(scaling)).to(q.dtype), None

        saved = lp.attention_interface
        lp.attention_interface = cpu_attn
        lp.install()
        try:
            t0 = time.perf_counter()
            n = 0
            with torch.no_grad():
                while True:
                    t1 = time.perf_counter()
                    layer(h, position_embeddings=pe)
                    t2 = time.perf_counter()
                    head(h)
                    t3 = time.perf_counter()
                    n += 1
                    if reps and n >= reps or not reps and (t3 - t0 > 10.0 or n >= 3):
                        break
        finally:
            lp.uninstall()
            lp.attention_interface = saved
        return self.T / (32 * (t2 - t1) + (t3 - t2)), \
            f"1 decoder layer + LM head on 1 x 2048 tokens (last of x{n}), layer time x32"


def make_workload(name, dev, cpu_only=False, rank=0, world=1, layers=10):
    if name == "quantize":
        if cpu_only:
            w = QuantizeWorkload.__new__(QuantizeWorkload)
            w.elems = 4096 * 4096
            w.algo_bytes = w.elems * (2 + 0.5 + 1 / 16)
            w.config = {"workload": "quantize bf16 [4096,4096], per-tensor scale amax/2688, block 16"}
            return w
        return QuantizeWorkload(dev, rank, world)
    if name == "decode":
        return DecodeWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)
    if name == "qkv":
        return QkvWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)
    if name == "prefill":
        return PrefillWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)
    if name == "weights":
        return WeightsWorkload(dev, cpu_only=cpu_only, rank=rank, world=world, layers=layers)
    if name == "llama":
        return LlamaWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)
    if name == "gemm":
        return GemmWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)
    return AttentionWorkload(dev, cpu_only=cpu_only, rank=rank, world=world)


def main():
    args = parse()
    DecodeWorkload.B = args.decode_batch
    if args.impl == "reference":
        # CPU only: rank 0 runs and prints, other ranks exit without work.
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = init_dist()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
