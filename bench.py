"""Benchmark of the hot path on B200 (driver contract: one JSON line).

Headline (C1): W4A16 decode GEMV, x fp16 [M, 4096] @
int4 group-128 weights [4096, 11008] with fp16 scales.  One "step" is one
pass of the decode path over a stack of L = 32 distinct weight copies (like
32 layers; 745 MB in all, far larger than the 126 MB L2, so every GEMV
streams its weights from HBM), replayed as one CUDA graph.

The same JSON line carries one sub-record per other BASELINE config
("workloads": C1 at M=16, C2, C2', C0, C3, C4), each with its own value,
roofline, CPU baseline, end-to-end figure, parity flag and clock record.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--m M] [--sub none]
  python bench.py --workload fa_gqa ...   # one workload as the headline
  python bench.py --impl reference ...    # the reference's CPU algorithm

Multi-GPU (torchrun, one process per GPU): the headline is weak scaling
(each rank owns its own 11008-column shard of an N * 11008-column weight
stack, no collective in the data path; value = bytes all ranks streamed over
the max-over-ranks device time).  The "strong" sub-records split ONE fixed
problem with b200kern.sharding: C1 and C2 over output columns (C2 also with
the NCCL all-gather of the column shards, timed alone and combined), C3 over
kv-head groups, C4 over heads.
"""
import argparse
import faulthandler
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "triton-metal_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

PEAKS_FILE = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PROFILES = os.path.join(REPO, "profiles")


def peaks():
    if os.path.exists(PEAKS_FILE):
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        p["source"] = "measured"
        return p
    p = dict(FALLBACK_PEAKS)
    p["source"] = "fallback"
    return p


def ncu_traffic():
    """DRAM bytes per launch of each workload's dominant kernel(s), read off
    the committed ncu summaries: a line `traffic[<workload>] = <bytes>` in a
    profiles/*.md file (dram__bytes_read.sum + dram__bytes_write.sum of one
    capture, per launch as the bench counts launches)."""
    out = {}
    if not os.path.isdir(PROFILES):
        return out
    pat = re.compile(r"traffic\[([\w.=]+)\]\s*=\s*([0-9][0-9,]*)")
    for fn in sorted(os.listdir(PROFILES)):
        if fn.endswith(".md"):
            with open(os.path.join(PROFILES, fn)) as f:
                for m in pat.finditer(f.read()):
                    out[m.group(1)] = int(m.group(2).replace(",", ""))
    return out


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def dist_init():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------
# clocks sampled during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    """SM clock and throttle reasons of this process's GPU, polled every
    `interval` seconds from a host thread (NVML; nvidia-smi -lms 20 as a
    fallback) from before the warm-up until after the timed region.  Reads
    only: no GPU setting is changed."""
    NAMES = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
             0x4: "sw_power_cap"}

    def __init__(self, cuda_index, interval=0.005):
        self.cuda_index, self.interval = cuda_index, interval
        self.samples = []  # (t, sm_mhz, sm_max_mhz, reasons bitmask)
        self._stop = threading.Event()
        self._thread = None
        self._proc = None
        self.source = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            # "domain:bus:device.0" from torch's integer PCI ids (NVML takes a string)
            p = torch.cuda.get_device_properties(self.cuda_index)
            ids = (int(p.pci_domain_id), int(p.pci_bus_id), int(p.pci_device_id))
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId("%08x:%02x:%02x.0" % ids)
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.cuda_index]) if vis else self.cuda_index
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(idx)

    def _loop(self, nv, h):
        smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((time.perf_counter(), float(sm), float(smax), int(rs)))
            except Exception:
                pass
            self._stop.wait(self.interval)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self._thread = threading.Thread(target=self._loop, args=(nv, h), daemon=True)
            self._thread.start()
            self.source = "nvml"
        except Exception:
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.cuda_index),
                     "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                     "--format=csv,noheader,nounits", "-lms", "20"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.source = "nvidia-smi"
            except OSError:
                self._proc = None
        # let the poller produce its first samples before the caller's region
        t0 = time.perf_counter()
        while self._thread is not None and not self.samples and time.perf_counter() - t0 < 1.0:
            time.sleep(0.002)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            now = time.perf_counter()
            for r in (out or "").strip().splitlines():
                f = [x.strip() for x in r.split(",")]
                try:
                    self.samples.append((now, float(f[0]), float(f[1]), int(f[2], 16)))
                except (ValueError, IndexError):
                    pass

    def summary(self, t0=None, t1=None):
        """Samples inside [t0, t1] (the timed region); if the region is shorter
        than the poll interval, the samples bracketing it (within 50 ms)."""
        s = self.samples
        if t0 is not None and self.source == "nvml":
            inside = [x for x in s if t0 <= x[0] <= t1]
            if len(inside) < 2:
                inside = [x for x in s if t0 - 0.05 <= x[0] <= t1 + 0.05]
            s = inside
        if not s:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({n for x in s for bit, n in self.NAMES.items() if x[3] & bit})
        return {"sm_mhz": statistics.median(x[1] for x in s), "sm_max_mhz": s[0][2], "reasons": reasons,
                "samples": len(s), "source": self.source,
                "window_ms": None if t0 is None else round((t1 - t0) * 1e3, 3)}


# --------------------------------------------------------------------------
# reference-algorithm sampling (CPU), shared by cpu_baseline and --impl reference
# --------------------------------------------------------------------------
def run_samples(fn, units_per_call, warmup, steps=None, budget_s=None):
    """Call fn(i) `warmup` times untimed, then `steps` times (or until
    budget_s elapses); fn returns the units it covered as a float, or
    anything else for units_per_call.  Returns (units per second, calls, seconds)."""
    for i in range(warmup):
        fn(i)
    n, done, t0 = 0, 0.0, time.perf_counter()
    while True:
        r = fn(warmup + n)
        done += r if isinstance(r, float) else units_per_call
        n += 1
        el = time.perf_counter() - t0
        if steps is not None and n >= steps:
            break
        if budget_s is not None and el > budget_s:
            break
    return done / el, n, el


def host_threads():
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return threads


# --------------------------------------------------------------------------
# workload: W4A16 decode GEMV (C1)
# --------------------------------------------------------------------------
W4_N, W4_K, W4_G, W4_LAYERS = 11008, 4096, 128, 32
KDA_HEADS = 0  # --heads: a smaller C4 (fewer heads) for profiler captures


def w4_gemv_bytes(M, N=W4_N, K=W4_K, G=W4_G):
    """Algorithmic HBM bytes of one GEMV: packed weights + scales + x + out."""
    return (K // 8) * N * 4 + (K // G) * N * 2 + M * K * 2 + M * N * 2


class W4Gemv:
    name = "w4a16_gemv"
    metric = "W4A16 decode GEMV HBM throughput"
    unit = "GB/s"
    dtype = "fp16"
    bound = "hbm"
    value_scale = 1e9
    peak_key, peak_unit = "hbm_gbs", "GB/s"

    def __init__(self, M, rank, device=True, N=W4_N, col0=0):
        self.launches_per_step = W4_LAYERS
        import b200kern as bk
        from b200kern import _lib
        from b200kern.synthetic import w4_inputs
        self.bk, self.lib, self.M, self.N = bk, _lib, M, N
        d = w4_inputs(M, N, W4_K, W4_G, dtype=torch.float16, seed=rank)
        self.q0, self.s0_host = d["q"], d["scales"]
        g = torch.Generator().manual_seed(1000 + rank)
        self.x_host = torch.randn(W4_LAYERS, M, W4_K, generator=g).half()
        self.step_work = W4_LAYERS * w4_gemv_bytes(M, N)
        self.workload = f"w4a16_gemv M={M} K={W4_K} N={N} G={W4_G}"
        self.details = {"layers_per_step": W4_LAYERS, "weight_bytes_resident": W4_LAYERS * (W4_K // 8) * N * 4,
                        "l2": "inputs larger than L2 (32 distinct weight copies, 745 MB, streamed per step)"}
        if not device:
            return
        dev = torch.device("cuda")
        base_w = d["qweight"].to(dev)
        base_s = d["scales"].to(dev)
        self.qw = [base_w ^ ((i * 0x2545F491) & 0x7FFFFFFF) if i else base_w for i in range(W4_LAYERS)]
        self.sc = [base_s.clone() for _ in range(W4_LAYERS)]
        self.x_host = self.x_host.pin_memory()
        self.x = self.x_host.to(dev)
        self.out = torch.empty(W4_LAYERS, M, N, dtype=torch.float16, device=dev)
        self.out_host = torch.empty_like(self.out, device="cpu").pin_memory()

    def launch(self, i, stream):
        self.lib.call("b2_int4_matmul", self.x[i].data_ptr(), self.qw[i].data_ptr(), self.out[i].data_ptr(),
                      self.sc[i].data_ptr(), None, self.M, self.N, W4_K, W4_G, 0, stream)

    def step(self, stream):
        for i in range(W4_LAYERS):
            self.launch(i, stream)

    def single_launch(self):
        """One GEMV alone (synchronised on both sides, no programmatic overlap
        with a neighbour): median over the 32 layers' distinct weights."""
        stream = torch.cuda.current_stream()
        ptr = self.lib.current_stream()
        times = []
        for i in range(W4_LAYERS):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            # keep the GPU busy while the host enqueues, so that the events
            # bracket the kernel and not the host's launch latency
            torch.cuda._sleep(200000)
            e0.record(stream)
            self.launch(i, ptr)
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
        us = sorted(times)[len(times) // 2]
        return {"us": round(us, 3), "GB/s": round(w4_gemv_bytes(self.M, self.N) / us / 1e3, 1),
                "note": "one launch timed alone; the headline value is back to back (the next launch "
                        "streams its weights while this one computes)"}

    def e2e_step(self):
        """Public API, host buffers: H2D of the step's x, 32 ops, D2H of outputs."""
        xd = self.x_host.to("cuda", non_blocking=True)
        for i in range(W4_LAYERS):
            self.bk.int4_matmul(xd[i], self.qw[i], self.sc[i], group_size=W4_G, out=self.out[i])
        self.out_host.copy_(self.out, non_blocking=True)
        return self.x_host.numel() * 2, self.out.numel() * 2

    def kernel_work(self):
        return w4_gemv_bytes(self.M, self.N)

    def check(self):
        """Layer 0 (all M rows, all columns) vs the float64 oracle."""
        import numpy as np
        from oracle import quant as oq
        torch.cuda.synchronize()
        ref = oq.int4_matmul(self.x_host[0].double().numpy(), self.q0.numpy(), self.s0_host.double().numpy(),
                             None, W4_G)
        got = self.out[0].double().cpu().numpy()
        return bool(np.allclose(got, ref, rtol=1e-2, atol=1e-2))

    def ref_sampler(self):
        """The reference's dequant-then-matmul (tests/test_emitter.py:3068-3079,
        fp32 torch restatement in oracle/quant.py) on the host cores: one
        whole GEMV of layer 0 per call."""
        from oracle import quant as oq
        q, s, x = self.q0, self.s0_host, self.x_host[0]
        fn = lambda i: oq.int4_matmul_fp32_torch(x, q, s, None, W4_G)
        return fn, w4_gemv_bytes(self.M, self.N) / self.value_scale, \
            f"one GEMV M={self.M} K={W4_K} N={self.N} per call (fp32 dequant-then-matmul, torch)"


class W4GemvRef(W4Gemv):
    """C1 in the reference's own layout, read natively: uint8 [N, K/2] (low
    nibble = even k) and fp16 scales [N, K/G] (same bytes as C1)."""
    name = "w4a16_gemv_ref"
    metric = "W4A16 decode GEMV HBM throughput (reference [N, K/2] layout)"

    def __init__(self, M, rank, device=True):
        super().__init__(M, rank, device)
        self.workload = f"w4a16_gemv_ref M={M} K={W4_K} N={W4_N} G={W4_G} (uint8 [N, K/2])"
        if not device:
            return
        self._gptq0 = self.qw[0]
        ref = self.bk.pack_int4_ref(self.bk.unpack_int4_gptq(self.qw[0].cpu()).t().contiguous())
        base = ref.cuda()
        self.qw = [base ^ (i & 0xFF) if i else base for i in range(W4_LAYERS)]
        self.sc = [s.t().contiguous() for s in self.sc]

    def launch(self, i, stream):
        self.lib.call("b2_int4_matmul_ref", self.x[i].data_ptr(), self.qw[i].data_ptr(), self.out[i].data_ptr(),
                      self.sc[i].data_ptr(), None, self.M, W4_N, W4_K, W4_G, 0, stream)

    def e2e_step(self):
        xd = self.x_host.to("cuda", non_blocking=True)
        for i in range(W4_LAYERS):
            self.bk.int4_matmul(xd[i], self.qw[i], self.sc[i], group_size=W4_G, layout="ref", out=self.out[i])
        self.out_host.copy_(self.out, non_blocking=True)
        return self.x_host.numel() * 2, self.out.numel() * 2

    def check(self):
        import numpy as np
        from oracle import quant as oq
        torch.cuda.synchronize()
        q = oq.unpack_int4_ref(self.qw[0].cpu().numpy()).T
        ref = oq.int4_matmul(self.x_host[0].double().numpy(), q, self.sc[0].t().double().cpu().numpy(), None, W4_G)
        got = self.out[0].double().cpu().numpy()
        rms = np.sqrt((ref ** 2).mean())
        return bool((np.abs(got - ref) <= 1e-2 * (np.abs(ref) + rms)).all())


# --------------------------------------------------------------------------
# workloads: prefill GEMMs (C2 / C2'): x bf16 [4096, 4096] @ W [4096, 14336]
# --------------------------------------------------------------------------
G_M, G_K, G_N, G_G = 4096, 4096, 14336, 128


class Gemm:
    """One step = one GEMM on the C2 shape; x, packed W, scales and the 117 MB
    output together exceed the 126 MB L2 (no flush needed)."""
    unit = "TFLOP/s"
    dtype = "bf16"
    bound = "tensor"
    value_scale = 1e12
    peak_unit = "TFLOP/s"
    # runs of tens of milliseconds: the burst (not the power-capped sustained) peak
    peak_key = "bf16_tflops"
    launches_per_step = 1

    def __init__(self, kind, rank, device=True, M=G_M, N=G_N, K=G_K, col=None):
        import b200kern as bk
        from b200kern import _lib
        from b200kern.synthetic import w4_inputs, w8_inputs
        self.bk, self.lib, self.kind = bk, _lib, kind
        self.name = kind
        self.metric = {"w4a16_gemm": "W4A16 prefill GEMM tensor throughput",
                       "w8a16_gemm": "W8A16 prefill GEMM tensor throughput",
                       "gemm_bf16": "bf16 GEMM tensor throughput"}[kind]
        if kind == "w4a16_gemm":
            d = w4_inputs(M, N, K, G_G, dtype=torch.bfloat16, seed=rank)
            self.q, w, s = d["q"], d["qweight"], d["scales"]
        elif kind == "w8a16_gemm":
            d = w8_inputs(M, N, K, dtype=torch.bfloat16, seed=rank)
            w, s = d["w"], d["scales"]
        else:
            g = torch.Generator().manual_seed(rank)
            d = {"x": torch.randn(M, K, generator=g).bfloat16()}
            w = (torch.randn(N, K, generator=g) / K ** 0.5).bfloat16()
            s = None
        if col is not None:  # one column shard of the fixed problem (b200kern.sharding)
            from b200kern import sharding
            world, r = col
            if kind == "w4a16_gemm":
                w, s, _, (a, b) = sharding.shard_int4(w, s, world=world, rank=r, align=128)
                self.q = self.q[:, a:b]
            else:
                w, s, _, (a, b) = sharding.shard_int8(w, s, world=world, rank=r, align=128)
            N = b - a
        self.M, self.N, self.K = M, N, K
        self.w_host, self.s_host = w, s
        self.x_host = d["x"]
        self.step_work = 2.0 * M * N * K
        self.workload = f"{kind} M={M} K={K} N={N}" + (f" G={G_G}" if kind == "w4a16_gemm" else "")
        self.details = {"l2": "inputs+output 178+ MB > 126 MB L2 (no flush needed)"}
        if not device:
            return
        dev = torch.device("cuda")
        self.w = w.to(dev)
        self.s = None if s is None else s.to(dev)
        self.x_host = self.x_host.pin_memory()
        self.x = self.x_host.to(dev)
        self.out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        self.out_host = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()

    def launch(self, i, stream):
        if self.kind == "w4a16_gemm":
            self.lib.call("b2_int4_matmul", self.x.data_ptr(), self.w.data_ptr(), self.out.data_ptr(),
                          self.s.data_ptr(), None, self.M, self.N, self.K, G_G, 1, stream)
        elif self.kind == "w8a16_gemm":
            self.lib.call("b2_int8_matmul", self.x.data_ptr(), self.w.data_ptr(), self.out.data_ptr(),
                          self.s.data_ptr(), None, self.M, self.N, self.K, 1, stream)
        else:
            self.lib.call("b2_gemm_bf16", self.x.data_ptr(), self.w.data_ptr(), self.out.data_ptr(),
                          self.M, self.N, self.K, stream)

    def step(self, stream):
        self.launch(0, stream)

    def e2e_step(self):
        xd = self.x_host.to("cuda", non_blocking=True)
        if self.kind == "w4a16_gemm":
            self.bk.int4_matmul(xd, self.w, self.s, group_size=G_G, out=self.out)
        elif self.kind == "w8a16_gemm":
            self.bk.int8_matmul(xd, self.w, self.s, out=self.out)
        else:
            self.bk.gemm_bf16(xd, self.w, out=self.out)
        self.out_host.copy_(self.out, non_blocking=True)
        return self.x_host.numel() * 2, self.out.numel() * 2

    def kernel_work(self):
        return self.step_work

    def check(self):
        """Two whole 256-row tiles (the first and the last) vs the float64 oracle."""
        import numpy as np
        from oracle import quant as oq
        torch.cuda.synchronize()
        rows = torch.cat([torch.arange(0, 256), torch.arange(self.M - 256, self.M)])
        xr = self.x_host[rows].double().numpy()
        if self.kind == "w4a16_gemm":
            ref = oq.int4_matmul(xr, self.q.numpy(), self.s_host.double().numpy(), None, G_G)
        elif self.kind == "w8a16_gemm":
            ref = oq.int8_matmul(xr, self.w_host.numpy(), self.s_host.double().numpy())
        else:
            ref = xr @ self.w_host.double().numpy().T
        got = self.out[rows.cuda()].double().cpu().numpy()
        rms = np.sqrt((ref ** 2).mean())
        return bool((np.abs(got - ref) <= 1e-2 * (np.abs(ref) + rms)).all())

    def ref_sampler(self):
        """The reference's dequant-then-matmul (tests/test_emitter.py:3068-3079
        for int4, :2638-2649 for int8) in fp32 torch on all host threads: a
        256-row slice of x against the whole weight per call."""
        from oracle import quant as oq
        rows = 256
        x = self.x_host[:rows]
        if self.kind == "w4a16_gemm":
            q, s = self.q.to(torch.int32), self.s_host
            fn = lambda i: oq.int4_matmul_fp32_torch(x, q, s, None, G_G)
        elif self.kind == "w8a16_gemm":
            w, s = self.w_host, self.s_host
            fn = lambda i: x.float() @ (w.float() * s.float()[:, None]).t()
        else:
            w = self.w_host
            fn = lambda i: x.float() @ w.float().t()
        return fn, 2.0 * rows * self.N * self.K / self.value_scale, \
            f"[{rows} rows of M] x K={self.K} x N={self.N} per call (fp32 dequant-then-matmul, torch)"


# --------------------------------------------------------------------------
# workloads: FlashAttention forward (C3 GQA prefill bf16; C0 fp32)
# --------------------------------------------------------------------------
def fa_visible_pairs(S, window):
    """(query, key) pairs a causal sliding window of W keys leaves visible
    over S positions: sum_i min(i + 1, W)."""
    w = min(window, S)
    return w * (w + 1) // 2 + (S - w) * w


class FlashAttn:
    """C3: B=4, Hq=32, Hkv=8, S=8192, D=128, causal, bf16; q/k/v = 0.5 N(0,1).
    One step = one forward over the whole batch (q/k/v/o 671 MB > L2).
    --window W > 0: causal sliding window (query i sees keys i-W+1 .. i);
    FLOPs then count the visible (query, key) pairs only."""
    name = "fa_gqa"
    metric = "FlashAttention GQA prefill throughput"
    unit = "tokens/s"
    dtype = "bf16"
    bound = "tensor"
    value_scale = 1.0
    roof_scale = 1e12
    peak_key, peak_unit = "bf16_tflops", "TFLOP/s"
    launches_per_step = 1

    def __init__(self, rank, device=True, B=4, Hq=32, Hkv=8, S=8192, D=128, causal=True, window=0, heads=None):
        import b200kern as bk
        self.bk = bk
        g = torch.Generator().manual_seed(rank)
        q = (torch.randn(B, Hq, S, D, generator=g) * 0.5).bfloat16()
        k = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
        v = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
        if heads is not None:  # one kv-head-group shard of the fixed problem
            from b200kern import sharding
            world, r = heads
            q, k, v, _ = sharding.shard_heads(q, k, v, world, r)
            Hq, Hkv = q.shape[1], k.shape[1]
        self.q_host, self.k_host, self.v_host = q, k, v
        self.B, self.Hq, self.Hkv, self.S, self.D, self.causal = B, Hq, Hkv, S, D, causal
        self.window = window
        if window:
            self.flops = 4.0 * B * Hq * fa_visible_pairs(S, window) * D
        else:
            self.flops = 4.0 * B * Hq * S * S * D / (2 if causal else 1)
        self.step_work = B * S          # tokens per step
        self.workload = (f"fa_gqa B={B} Hq={Hq} Hkv={Hkv} S={S} D={D} causal={causal}"
                         + (f" window={window}" if window else ""))
        self.details = {"flop_convention": "4*B*Hq*S^2*D/2 (causal half)" if not window
                        else "4*B*Hq*D*(visible query-key pairs)",
                        "l2": "q/k/v/o 671 MB > 126 MB L2 (no flush needed)"}
        if not device:
            return
        self.q_host, self.k_host, self.v_host = (t.pin_memory() for t in (q, k, v))
        self.q, self.k, self.v = (t.cuda() for t in (self.q_host, self.k_host, self.v_host))
        self.o = torch.empty_like(self.q)
        self.o_host = torch.empty_like(self.q_host).pin_memory()

    def step(self, stream):
        self.bk.flash_attention(self.q, self.k, self.v, causal=self.causal, out=self.o, window=self.window)

    def e2e_step(self):
        q, k, v = (h.to("cuda", non_blocking=True) for h in (self.q_host, self.k_host, self.v_host))
        self.bk.flash_attention(q, k, v, causal=self.causal, out=self.o, window=self.window)
        self.o_host.copy_(self.o, non_blocking=True)
        return sum(t.numel() * t.element_size() for t in (self.q_host, self.k_host, self.v_host)), \
            self.o.numel() * self.o.element_size()

    def kernel_work(self):
        return self.flops

    def _ref_rows(self, b, h, rows):
        """float64 reference for some query rows of one (b, h) (causal offsets kept)."""
        rep = self.Hq // self.Hkv
        q = self.q_host[b, h, rows].double()
        k = self.k_host[b, h // rep].double()
        v = self.v_host[b, h // rep].double()
        s = (q / self.D ** 0.5) @ k.t()
        if self.causal:
            kpos = torch.arange(self.S)[None, :]
            s = s.masked_fill(kpos > rows[:, None], float("-inf"))
            if self.window:
                s = s.masked_fill(kpos <= rows[:, None] - self.window, float("-inf"))
        return torch.softmax(s, -1) @ v

    def check(self):
        torch.cuda.synchronize()
        rows = torch.cat([torch.arange(0, 64), torch.arange(self.S - 64, self.S)])
        ok = True
        for (b, h) in ((0, 0), (self.B - 1, self.Hq - 1)):
            ref = self._ref_rows(b, h, rows)
            got = self.o[b, h, rows.cuda()].double().cpu()
            ok &= bool(((got - ref).abs() <= 1e-2 + 1e-2 * ref.abs()).all())
        return ok

    def ref_sampler(self):
        """The reference's _ref_attention (tests/test_flash_attention.py:107-118)
        restated in fp32 torch on all host threads: per call, a block of 1024
        query rows of one (b, h) slice against every key it may see (GQA
        expansion kv_head = h // (Hq / Hkv)); the value scales the block's
        share of the step's (query, key) pairs to tokens per second."""
        rep = self.Hq // self.Hkv
        blk = min(1024, self.S)
        nblk = self.S // blk
        total = fa_visible_pairs(self.S, self.window or self.S) if self.causal else self.S * self.S
        total *= self.B * self.Hq
        shares = []

        def fn(i):
            b, rest = divmod(i % (self.B * self.Hq * nblk), self.Hq * nblk)
            h, j = divmod(rest, nblk)
            r0 = j * blk
            hi = r0 + blk if self.causal else self.S
            q = self.q_host[b, h, r0:r0 + blk].float()
            k = self.k_host[b, h // rep, :hi].float()
            v = self.v_host[b, h // rep, :hi].float()
            s = (q * (1.0 / self.D ** 0.5)) @ k.t()
            if self.causal:
                qpos = torch.arange(r0, r0 + blk)[:, None]
                kpos = torch.arange(hi)[None, :]
                mask = kpos > qpos
                if self.window:
                    mask |= kpos <= qpos - self.window
                s = s.masked_fill(mask, float("-inf"))
            torch.softmax(s, -1).nan_to_num(0.0) @ v
            return shares[j]
        # share of the step's tokens that the block of rows j stands for, by
        # the (query, key) pairs it computes
        for j in range(nblk):
            r0 = j * blk
            if self.causal:
                w = self.window or self.S
                pairs = sum(min(i + 1, w) for i in range(r0, r0 + blk))
            else:
                pairs = blk * self.S
            shares.append(self.step_work * pairs / total)
        return fn, None, (f"{blk} query rows of one (b, h) slice per call, cycling over blocks and slices "
                          f"(fp32 torch _ref_attention restatement); each call credited with its share of "
                          f"the step's (query, key) pairs")


class FlashAttnC0(FlashAttn):
    """C0: fp32 q/k/v [2, 8, 1024, 64] ~ N(0,1) (torch
    seed 0, q then k then v), causal, scale 1/8.  The problem (16.8 MB) fits
    in L2, so one step runs the forward over 16 distinct input copies (268 MB
    in all) and each copy streams from HBM."""
    name = "fa_c0"
    metric = "FlashAttention fp32 forward throughput (reference CPU config)"
    dtype = "fp32"
    COPIES = 16

    def __init__(self, rank, device=True):
        import b200kern as bk
        self.bk = bk
        B, H, S, D = 2, 8, 1024, 64
        torch.manual_seed(rank)
        self.q_host = torch.randn(B, H, S, D)
        self.k_host = torch.randn(B, H, S, D)
        self.v_host = torch.randn(B, H, S, D)
        self.B, self.Hq, self.Hkv, self.S, self.D, self.causal, self.window = B, H, H, S, D, True, 0
        self.flops = 4.0 * B * H * S * S * D / 2
        self.launches_per_step = self.COPIES
        self.step_work = self.COPIES * B * S
        self.workload = f"fa_c0 B={B} H={H} S={S} D={D} causal=True fp32 scale=1/8"
        self.details = {"flop_convention": "4*B*H*S^2*D/2 (causal half)",
                        "l2": f"{self.COPIES} input copies per step (268 MB > 126 MB L2)"}
        if not device:
            return
        self.q_host, self.k_host, self.v_host = (t.pin_memory() for t in (self.q_host, self.k_host, self.v_host))
        self.qs = [self.q_host.cuda() for _ in range(self.COPIES)]
        self.ks = [self.k_host.cuda() for _ in range(self.COPIES)]
        self.vs = [self.v_host.cuda() for _ in range(self.COPIES)]
        self.os = [torch.empty_like(self.qs[0]) for _ in range(self.COPIES)]
        self.q, self.o = self.qs[0], self.os[0]
        self.o_host = torch.empty_like(self.q_host).pin_memory()

    def step(self, stream):
        for i in range(self.COPIES):
            self.bk.flash_attention(self.qs[i], self.ks[i], self.vs[i], causal=True, scale=0.125, out=self.os[i])

    def e2e_step(self):
        for i in range(self.COPIES):
            q, k, v = (h.to("cuda", non_blocking=True) for h in (self.q_host, self.k_host, self.v_host))
            self.bk.flash_attention(q, k, v, causal=True, scale=0.125, out=self.os[i])
            self.o_host.copy_(self.os[i], non_blocking=True)
        return self.COPIES * 3 * self.q_host.numel() * 4, self.COPIES * self.q_host.numel() * 4

    def check(self):
        import numpy as np
        from oracle import attention as oatt
        torch.cuda.synchronize()
        ref = oatt.attention(self.q_host[:, :2].double().numpy(), self.k_host[:, :2].double().numpy(),
                             self.v_host[:, :2].double().numpy(), causal=True, scale=0.125)
        got = self.o[:, :2].double().cpu().numpy()
        return bool((np.abs(got - ref) <= 1e-2 + 1e-2 * np.abs(ref)).all())

    def ref_sampler(self):
        """The reference's _ref_attention (tests/test_flash_attention.py:107-118)
        in fp32 torch on all host threads: the whole C0 problem per call."""
        q, k, v = self.q_host, self.k_host, self.v_host
        S = self.S
        mask = torch.ones(S, S, dtype=torch.bool).triu(1)

        def fn(i):
            s = (q * 0.125) @ k.transpose(-1, -2)
            torch.softmax(s.masked_fill(mask, float("-inf")), -1).nan_to_num(0.0) @ v
        return fn, self.B * S, "the whole C0 forward per call (fp32 torch _ref_attention restatement)"


# --------------------------------------------------------------------------
# workload: KDA chunked forward (C4)
# --------------------------------------------------------------------------
class KDA:
    """B=1, H=32, T=16384, Dk=Dv=128, chunk 64; q,k L2-normalised bf16, v bf16,
    g = -softplus(N(0,1)) fp32, beta = sigmoid(N(0,1)) bf16, zero fp32 state.
    One step = one forward over all heads (inputs 810 MB > L2)."""
    name = "kda"
    metric = "KDA chunked forward throughput"
    unit = "tokens/s"
    dtype = "bf16 (fp32 state)"
    bound = "hbm"
    value_scale = 1.0
    roof_scale = 1e9
    peak_key, peak_unit = "hbm_gbs", "GB/s"
    launches_per_step = 1

    def __init__(self, rank, device=True, B=1, T=16384, H=32, D=128, heads=None):
        import b200kern as bk
        self.bk = bk
        H = KDA_HEADS or H
        gen = torch.Generator().manual_seed(rank)
        F = torch.nn.functional
        q = F.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1).bfloat16()
        k = F.normalize(torch.randn(B, T, H, D, generator=gen), dim=-1).bfloat16()
        v = torch.randn(B, T, H, D, generator=gen).bfloat16()
        g = -F.softplus(torch.randn(B, T, H, D, generator=gen))
        beta = torch.sigmoid(torch.randn(B, T, H, generator=gen)).bfloat16()
        if heads is not None:  # one head shard of the fixed problem
            from b200kern import sharding
            world, r = heads
            a, b = sharding.shard_range(H, world, r)
            q, k, v, g = (t[:, :, a:b].contiguous() for t in (q, k, v, g))
            beta = beta[:, :, a:b].contiguous()
            H = b - a
        self.q_host, self.k_host, self.v_host, self.g_host, self.b_host = q, k, v, g, beta
        self.B, self.T, self.H, self.D = B, T, H, D
        # algorithmic bytes: q,k,v bf16 + g fp32 + beta + o bf16 + S0 and S_T fp32
        self.bytes = (3 * B * T * H * D * 2 + B * T * H * D * 4 + B * T * H * 2 + B * T * H * D * 2
                      + 2 * B * H * D * D * 4)
        self.step_work = B * T
        self.kernels_per_launch = int(bk.kda.kernels_per_call())
        self.workload = f"kda B={B} T={T} H={H} Dk=Dv={D} chunk=64"
        self.details = {"algorithmic_bytes": self.bytes, "l2": "inputs 810 MB > 126 MB L2",
                        "kernels_per_step": self.kernels_per_launch}
        if not device:
            return
        from b200kern.kda import workspace_size
        hosts = [t.pin_memory() for t in (q, k, v, g, beta)]
        self.q_host, self.k_host, self.v_host, self.g_host, self.b_host = hosts
        self.q, self.k, self.v, self.g, self.beta = (t.cuda() for t in hosts)
        self.o = torch.empty_like(self.v)
        self.S = torch.empty(B, H, D, D, dtype=torch.float32, device="cuda")
        self.o_host = torch.empty_like(self.v_host).pin_memory()
        self.ws = torch.empty(max(1, workspace_size(B, T, H)), dtype=torch.uint8, device="cuda")

    def step(self, stream):
        self.bk.kda_chunk_fwd(self.q, self.k, self.v, self.g, self.beta, out=self.o, workspace=self.ws,
                              final_state_out=self.S)

    def e2e_step(self):
        q, k, v, g, b = (h.to("cuda", non_blocking=True) for h in (self.q_host, self.k_host, self.v_host,
                                                                   self.g_host, self.b_host))
        self.bk.kda_chunk_fwd(q, k, v, g, b, out=self.o, workspace=self.ws, final_state_out=self.S)
        self.o_host.copy_(self.o, non_blocking=True)
        h2d = sum(t.numel() * t.element_size() for t in (self.q_host, self.k_host, self.v_host, self.g_host,
                                                         self.b_host))
        return h2d, self.o.numel() * 2

    def kernel_work(self):
        return self.bytes

    def check(self):
        """Heads 0 and H-1 over the first 512 steps vs the float64 oracle."""
        import numpy as np
        from oracle import kda as okda
        torch.cuda.synchronize()
        n, heads = 512, [0, self.H - 1]
        d = lambda t: t[:, :n, heads].double().numpy()
        oref, _ = okda.recurrent(d(self.q_host), d(self.k_host), d(self.v_host), d(self.g_host),
                                 self.b_host[:, :n, heads].double().numpy())
        got = self.o[:, :n, heads].double().cpu().numpy()
        return bool((np.abs(got - oref) <= 2e-2 + 2e-2 * np.abs(oref)).all())

    def ref_sampler(self):
        """No reference CPU path exists for KDA (triton-metal has no KDA): the
        float64 recurrence oracle (oracle/kda.py, not the reference's code) on
        2 heads x 256 steps per call, scaled to the step's T x H."""
        from oracle import kda as okda
        heads, n = min(2, self.H), 256
        d = lambda t: t[:, :n, :heads].double().numpy()
        args = (d(self.q_host), d(self.k_host), d(self.v_host), d(self.g_host),
                self.b_host[:, :n, :heads].double().numpy())
        fn = lambda i: okda.recurrent(*args)
        return fn, self.B * self.T * (n / self.T) * (heads / self.H), \
            f"{n} steps x {heads} heads per call (numpy float64 recurrence, not reference code), scaled linearly"


# --------------------------------------------------------------------------
# workload: split-KV decode attention over a long KV cache
# --------------------------------------------------------------------------
class Decode:
    """B=32 sequences, Hq=32, Hkv=8, S=8192 cached tokens, D=128, bf16 q and KV
    cache (1.07 GB > L2); q/k/v = 0.5 N(0,1). One step = one decode token for
    every sequence (split-KV kernel + combine kernel)."""
    name = "decode"
    metric = "GQA decode attention KV-cache read bandwidth"
    unit = "tokens/s"
    dtype = "bf16"
    bound = "hbm"
    value_scale = 1.0
    roof_scale = 1e9
    peak_key, peak_unit = "hbm_gbs", "GB/s"
    launches_per_step = 1

    def __init__(self, rank, device=True, B=32, Hq=32, Hkv=8, S=8192, D=128):
        import b200kern as bk
        self.bk, self.B, self.Hq, self.Hkv, self.S, self.D = bk, B, Hq, Hkv, S, D
        g = torch.Generator().manual_seed(rank)
        self.q_host = (torch.randn(B, Hq, D, generator=g) * 0.5).bfloat16()
        k = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
        v = (torch.randn(B, Hkv, S, D, generator=g) * 0.5).bfloat16()
        self.kc, self.vc = k[:2], v[:2]
        self.bytes = 2 * B * Hkv * S * D * 2 + 2 * B * Hq * D * 2
        self.step_work = B              # decoded tokens per step
        self.kernels_per_launch = 1
        self.workload = f"decode B={B} Hq={Hq} Hkv={Hkv} S={S} D={D} kv=bf16"
        self.details = {"algorithmic_bytes": self.bytes, "l2": "KV cache 1.07 GB > 126 MB L2 (no flush needed)",
                        "e2e_note": "the KV cache is device-resident state; e2e copies q in and o out per step"}
        if not device:
            return
        self.k, self.v = k.cuda(), v.cuda()
        self.lens = torch.full((B,), S, dtype=torch.int32, device="cuda")
        self.q_host = self.q_host.pin_memory()
        self.q = self.q_host.cuda()
        self.o = torch.empty_like(self.q)
        self.o_host = torch.empty_like(self.q_host).pin_memory()
        # split kernel, plus the combine kernel when B * Hkv < SMs (KV split)
        self.kernels_per_launch = 1 if B * Hkv >= torch.cuda.get_device_properties(0).multi_processor_count else 2
        self.details["kernels_per_step"] = self.kernels_per_launch

    def step(self, stream):
        self.bk.decode_attention(self.q, self.k, self.v, self.lens, out=self.o)

    def e2e_step(self):
        q = self.q_host.to("cuda", non_blocking=True)
        self.bk.decode_attention(q, self.k, self.v, self.lens, out=self.o)
        self.o_host.copy_(self.o, non_blocking=True)
        return self.q_host.numel() * 2, self.o.numel() * 2

    def kernel_work(self):
        return self.bytes

    def check(self):
        torch.cuda.synchronize()
        ok = True
        rep = self.Hq // self.Hkv
        for b in (0, self.B - 1):
            k = self.k[b].double().cpu()
            v = self.v[b].double().cpu()
            q = self.q_host[b].double().reshape(self.Hkv, rep, self.D)
            s = torch.einsum("hrd,hsd->hrs", q, k) / self.D ** 0.5
            ref = torch.einsum("hrs,hsd->hrd", torch.softmax(s, -1), v).reshape(self.Hq, self.D)
            got = self.o[b].double().cpu()
            ok &= bool(((got - ref).abs() <= 1e-2 + 1e-2 * ref.abs()).all())
        return ok

    def ref_sampler(self):
        """The reference's KV-cache decode check (tests/test_emitter.py:2124,
        softmax(q k^T * scale) v per head) in fp32 torch on all host threads:
        one sequence per call."""
        rep = self.Hq // self.Hkv
        kc, vc = self.kc.float(), self.vc.float()

        def fn(i):
            b = i % 2
            q = self.q_host[b].float().reshape(self.Hkv, rep, self.D)
            s = torch.einsum("hrd,hsd->hrs", q, kc[b]) * (1.0 / self.D ** 0.5)
            torch.einsum("hrs,hsd->hrd", torch.softmax(s, -1), vc[b])
        return fn, 1.0, f"one sequence of {self.B} (S={self.S}) per call; value = sequences decoded per second"


WORKLOADS = {"decode": Decode, "w4a16_gemv_ref": W4GemvRef, "kda": KDA, "fa_gqa": FlashAttn, "fa_c0": FlashAttnC0,
             "w4a16_gemv": W4Gemv, "w4a16_gemm": Gemm, "w8a16_gemm": Gemm, "gemm_bf16": Gemm}

# sub-records of the default run: (label, workload, M for the GEMV)
SUB_RECORDS = [("C1_m16", "w4a16_gemv", 16), ("C2", "w4a16_gemm", None), ("C2p", "w8a16_gemm", None),
               ("C0", "fa_c0", None), ("C3", "fa_gqa", None), ("C4", "kda", None)]


def make_workload(name, rank, m=1, window=0, device=True, **shard):
    if name == "w4a16_gemv":
        return W4Gemv(m, rank, device, **shard)
    if name == "w4a16_gemv_ref":
        return W4GemvRef(m, rank, device)
    if name in ("w4a16_gemm", "w8a16_gemm", "gemm_bf16"):
        return Gemm(name, rank, device, **shard)
    if name == "fa_gqa":
        return FlashAttn(rank, device, window=window, **shard)
    if name == "fa_c0":
        return FlashAttnC0(rank, device)
    if name == "kda":
        return KDA(rank, device, **shard)
    if name == "decode":
        return Decode(rank, device)
    raise SystemExit(f"unknown workload {name}")


def config_of(wl):
    """The `config` both arms print for a workload (identical by construction)."""
    return {"workload": wl.workload}


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def time_graph(wl, steps, warmup, world, local):
    """Eager run + parity check, then `steps` replays of a one-step CUDA graph
    after `warmup` replays, with clocks sampled around the timed region.
    Returns (parity_ok, ms over the K steps on this rank, clock summary)."""
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        wl.step(stream.cuda_stream)
    stream.synchronize()
    parity_ok = wl.check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        wl.step(stream.cuda_stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        barrier(world)
    del graph
    return parity_ok, ev0.elapsed_time(ev1), clk.summary(t0, t1)


def roofline(wl, ms, steps, traffic):
    """Algorithmic work of one launch of the dominant kernel over its average
    device duration.  The timed graph holds only this workload's launches
    (launches_per_step back to back), so the mean launch duration is the step
    time / launches, inter-kernel gaps included (conservative)."""
    k_ms = ms / steps / wl.launches_per_step
    pk = peaks()
    roof_scale = getattr(wl, "roof_scale", wl.value_scale)
    achieved = wl.kernel_work() / (k_ms / 1e3) / roof_scale
    peak = pk[wl.peak_key]
    return {"bound": wl.bound, "achieved": round(achieved, 1), "peak": peak, "unit": wl.peak_unit,
            "frac": round(achieved / peak, 4), "traffic": traffic.get(wl.workload, traffic.get(wl.name)),
            "peak_source": f"{pk['source']} {wl.peak_key}", "kernel_us": round(k_ms * 1e3, 3)}


def time_e2e(wl, steps, world):
    e2e_steps = max(3, min(steps, 200))
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        h2d, d2h = wl.e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    return {"value": round(wl.step_work * e2e_steps * world / (e_ms / 1e3) / wl.value_scale, 1), "unit": wl.unit,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps}


def cpu_baseline(wl, budget_s):
    threads = host_threads()
    fn, units, desc = wl.ref_sampler()
    value, n, el = run_samples(fn, units, warmup=1, budget_s=budget_s)
    return {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{n} calls in {el:.1f} s; {desc}"}


def measure(wl, args, world, local, traffic, with_cpu):
    parity_ok, ms, clocks = time_graph(wl, args.steps, args.warmup, world, local)
    ms_max = max_over_ranks(ms, world)
    value = wl.step_work * args.steps * world / (ms_max / 1e3) / wl.value_scale
    rec = {"metric": wl.metric, "value": round(value, 1), "unit": wl.unit, "ms_per_step": round(ms_max / args.steps, 5),
           "dtype": wl.dtype, "config": config_of(wl), "details": wl.details, "parity_ok": parity_ok,
           "roofline": roofline(wl, ms, args.steps, traffic), "e2e": time_e2e(wl, args.steps, world),
           "gpu_launches": getattr(wl, "kernels_per_launch", 1) * wl.launches_per_step * args.steps,
           "clocks": clocks}
    if hasattr(wl, "single_launch"):
        rec["details"] = dict(wl.details, single_launch=wl.single_launch())
    rec["cpu_baseline"] = cpu_baseline(wl, args.cpu_budget) if with_cpu else None
    return rec


def strong_record(name, args, rank, world, local, traffic):
    """One fixed problem split over the ranks with b200kern.sharding; value =
    the whole problem's units over the max-over-ranks device time."""
    if name == "C1":
        from b200kern.sharding import shard_range
        a, b = shard_range(W4_N, world, rank, 8)
        wl = W4Gemv(1, 0, True, N=b - a)
        full_units = W4_LAYERS * w4_gemv_bytes(1)
    elif name in ("C2", "C2p"):
        wl = Gemm("w4a16_gemm" if name == "C2" else "w8a16_gemm", 0, True, col=(world, rank))
        full_units = 2.0 * G_M * G_N * G_K
    elif name == "C3":
        wl = FlashAttn(0, True, heads=(world, rank))
        full_units = wl.B * wl.S
    else:
        wl = KDA(0, True, heads=(world, rank))
        full_units = wl.B * wl.T
    parity_ok, ms, clocks = time_graph(wl, args.steps, args.warmup, world, local)
    ms_max = max_over_ranks(ms, world)
    rec = {"workload": f"{name} sharded over {world} ranks: {wl.workload} per rank",
           "value": round(full_units * args.steps / (ms_max / 1e3) / wl.value_scale, 1), "unit": wl.unit,
           "ms_per_step": round(ms_max / args.steps, 5), "parity_ok": parity_ok, "clocks": clocks,
           # the committed ncu traffic figures cover the unsharded problem
           "roofline_per_rank": roofline(wl, ms, args.steps, traffic if world == 1 else {})}
    if name in ("C2", "C2p") and world > 1:
        from b200kern.sharding import all_gather_columns_stacked
        gathered = torch.empty(world, *wl.out.shape, dtype=wl.out.dtype, device="cuda")
        stream = torch.cuda.current_stream()
        for _ in range(max(3, args.warmup)):
            all_gather_columns_stacked(wl.out, out=gathered)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        for _ in range(args.steps):
            all_gather_columns_stacked(wl.out, out=gathered)
        e1.record(stream)
        for _ in range(args.steps):
            wl.step(stream.cuda_stream)
            all_gather_columns_stacked(wl.out, out=gathered)
        e2.record(stream)
        torch.cuda.synchronize()
        g_ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
        c_ms = max_over_ranks(e1.elapsed_time(e2), world) / args.steps
        rec["all_gather"] = {"ms": round(g_ms, 5), "bytes_per_rank": wl.out.numel() * wl.out.element_size(),
                             "layout": "[P, M, N/P] (column shards stacked; a permute gives [M, N])"}
        rec["combined"] = {"ms_per_step": round(c_ms, 5),
                           "value": round(full_units / (c_ms / 1e3) / wl.value_scale, 1), "unit": wl.unit}
    del wl
    torch.cuda.empty_cache()
    return rec


def run_ours(args):
    rank, world, local = dist_init()
    traffic = ncu_traffic()
    if world > 1 and args.workload == "w4a16_gemv":
        # weak scaling: this rank's own 11008-column shard of an N * 11008-column stack
        wl = W4Gemv(args.m, rank, True, N=W4_N)
    else:
        wl = make_workload(args.workload, rank, args.m, args.window)
    head = measure(wl, args, world, local, traffic, with_cpu=(world == 1 and rank == 0))
    del wl
    torch.cuda.empty_cache()
    subs, strong = {}, {}
    if args.sub == "auto" and args.workload == "w4a16_gemv" and args.m == 1:
        if world == 1:
            for label, name, m in SUB_RECORDS:
                sw = make_workload(name, rank, m or 1)
                subs[label] = measure(sw, args, world, local, traffic, with_cpu=(rank == 0))
                del sw
                torch.cuda.empty_cache()
        else:
            for label in ("C1", "C2", "C3", "C4"):
                strong[label] = strong_record(label, args, rank, world, local, traffic)
    line = None
    if rank == 0:
        line = {"metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": head["dtype"],
                "data": "synthetic (seeded, BASELINE distributions)", "config": head["config"],
                "details": head["details"], "parity_ok": head["parity_ok"], "roofline": head["roofline"],
                "cpu_baseline": head["cpu_baseline"], "e2e": head["e2e"], "gpu_launches": head["gpu_launches"],
                "clocks": head["clocks"]}
        if subs:
            line["workloads"] = subs
            line["gpu_launches"] += sum(r["gpu_launches"] for r in subs.values())
        if strong:
            line["strong"] = strong
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return line


# --------------------------------------------------------------------------
# reference arm: the reference's algorithm on the host cores
# --------------------------------------------------------------------------
def reference_record(wl, steps, warmup):
    threads = host_threads()
    fn, units, desc = wl.ref_sampler()
    value, n, el = run_samples(fn, units, warmup=warmup, steps=steps)
    unit_step = wl.step_work / wl.value_scale  # one step of our arm, in metric units
    return {"metric": wl.metric, "value": round(value, 4), "unit": wl.unit,
            "ms_per_step": round(unit_step / value * 1e3, 3), "dtype": "fp32" if wl.name != "kda" else "fp64",
            "config": config_of(wl),
            "cpu_baseline": {"value": round(value, 4), "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": f"{n} timed calls in {el:.2f} s after {warmup} warm-up calls; {desc}"},
            "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    wl = make_workload(args.workload, 0, args.m, args.window, device=False)
    head = reference_record(wl, args.steps, args.warmup)
    line = {"metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": head["dtype"],
            "data": "synthetic (seeded, BASELINE distributions)", "config": head["config"], "impl": "reference",
            "cpu_baseline": head["cpu_baseline"], "e2e": head["e2e"]}
    if args.sub == "auto" and args.workload == "w4a16_gemv" and args.m == 1:
        line["workloads"] = {}
        for label, name, m in SUB_RECORDS:
            sw = make_workload(name, 0, m or 1, device=False)
            line["workloads"][label] = reference_record(sw, args.steps, args.warmup)
            del sw
    return line


def main():
    global W4_LAYERS, KDA_HEADS
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="w4a16_gemv", choices=sorted(WORKLOADS))
    ap.add_argument("--m", type=int, default=1, help="GEMV rows (decode batch), 1..16")
    ap.add_argument("--window", type=int, default=0, help="fa_gqa: causal sliding window (0 = none)")
    ap.add_argument("--sub", choices=["auto", "none"], default="auto",
                    help="auto: the default C1 run also measures the other configs as sub-records")
    ap.add_argument("--cpu-budget", type=float, default=5.0, help="seconds of CPU baseline sampling per record")
    ap.add_argument("--layers", type=int, default=W4_LAYERS,
                    help="GEMV weight copies per step (a smaller stack for profiler captures)")
    ap.add_argument("--heads", type=int, default=0, help="kda: heads (a smaller C4 for profiler captures)")
    args = ap.parse_args()
    W4_LAYERS, KDA_HEADS = args.layers, args.heads
    line = run_reference(args) if args.impl == "reference" else run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
