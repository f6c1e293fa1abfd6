#!/usr/bin/env python3
"""Benchmark driver (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload vgg16|lif]

Workloads
  vgg16 (default) -- VGG16-SNN T=4 inference, batch 64 per GPU, 32x32x3 input,
                     BN folded, LIF tau=2 / v_th=1 / hard reset, 2x2 max-pool,
                     classifier 512-4096-4096-10 with the logits averaged over T.
                     Metric: images/s over all ranks (weak scaling: batch 64 per
                     GPU; one NCCL all-gather of the [64, 10] logits per step,
                     through snn_compiler.sharding.ShardedInference).  The line
                     also carries `lif_kernel`: the standalone LIF kernel's HBM
                     GB/s at T=32, N=2^27 per GPU (the metric's second half).
  lif             -- multi-step LIF sweep point T=32, N=2^27 float32 with
                     fp32 spikes + packed spikes + final v.  Metric: HBM GB/s
                     (algorithmic bytes 4TN + 4TN + TN/8 + 4N per step).

Timing: W warm-up steps, then K steps bracketed by barrier + synchronize and
CUDA events on the launching stream; the slowest rank's time is reported.
Inputs are larger than L2 for 'lif'; for 'vgg16' a 256 MB buffer is written
between steps to flush L2.  --impl reference times the reference's CPU
algorithm (this repository's oracle restatement of it) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "triton-pass-analysis_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ----------------------------------------------------------------------------------------
# clocks sampled during the timed region
class ClockSampler:
    """SM clock and clock-event reasons sampled every ~1 ms through NVML (read only) while
    the timed region runs; falls back to nvidia-smi polling when NVML is unavailable."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.samples = []          # (time, sm_mhz, max_mhz, set of reason names)
        self.gpu = gpu_index
        self.window = None
        self.proc = None
        self.stop_flag = False
        self.nvml = None
        self.error = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            # the NVML device of this process's CUDA device, by PCI address (NVML indexes all
            # GPUs of the node, whatever CUDA_VISIBLE_DEVICES selects)
            prop = torch.cuda.get_device_properties(torch.cuda.current_device())
            try:
                bus = "%08x:%02x:%02x.0" % (prop.pci_domain_id, prop.pci_bus_id, prop.pci_device_id)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.nvml, self.h = pynvml, h
            self.bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _sample_nvml(self):
        p = self.nvml
        try:
            sm = p.nvmlDeviceGetClockInfo(self.h, p.NVML_CLOCK_SM)
            mx = p.nvmlDeviceGetMaxClockInfo(self.h, p.NVML_CLOCK_SM)
            try:
                rb = p.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                rb = p.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            rs = {n for n, b in self.bits.items() if rb & b}
            self.samples.append((time.time(), float(sm), float(mx), rs))
        except Exception as e:          # keep the first error for the report
            self.error = self.error or f"{type(e).__name__}: {e}"

    def _poll_nvml(self):
        while not self.stop_flag:
            self._sample_nvml()
            time.sleep(0.001)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [q.strip() for q in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rs = {n for n, v in zip(self.NAMES, parts[5:9]) if v.lower().startswith("active")}
                self.samples.append((time.time(), float(parts[1]), float(parts[2]), rs))
            except ValueError:
                continue

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        self.stop_flag = True
        if self.nvml is not None:
            self.thread.join(timeout=1.0)
            if not self.samples:           # timed region shorter than one poll: sample now
                self._sample_nvml()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.nvml is None and self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no NVML / nvidia-smi"],
                    "samples": 0}
        rows = list(self.samples)
        if self.window and rows:
            inside = [r for r in rows if self.window[0] <= r[0] <= self.window[1]]
            if not inside:      # window shorter than the polling period: nearest samples
                rows = sorted(rows, key=lambda r: min(abs(r[0] - self.window[0]),
                                                      abs(r[0] - self.window[1])))[:2]
            else:
                rows = inside
        sm = [r[1] for r in rows]
        reasons = sorted(set().union(*[r[3] for r in rows])) if rows else []
        out = {"sm_mhz": statistics.median(sm) if sm else None,
               "sm_max_mhz": max(r[2] for r in rows) if rows else None, "reasons": reasons,
               "samples": len(rows), "source": "nvml" if self.nvml else "nvidia-smi"}
        if not rows and self.error:
            out["error"] = self.error
        return out


# ----------------------------------------------------------------------------------------
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        if args.impl == "reference":
            return rank, world, local, None
        torch.cuda.set_device(local)
        # the one collective is a 2.5 KB all-gather running beside the forward: a few CTAs
        # are plenty and leave the forward's SMs alone (a caller's own setting wins)
        os.environ.setdefault("NCCL_MAX_CTAS", "4")
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "4")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return rank, world, local, dist
    if args.impl != "reference":
        torch.cuda.set_device(0)
    return 0, 1, 0, None


def barrier(dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(dist, value):
    if dist is None:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, value):
    if dist is None:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------------------
class LifWorkload:
    name = "lif"

    def __init__(self, T=32, N=1 << 27):
        self.T, self.N = T, N
        self.bytes_per_step = 4 * T * N + 4 * T * N + T * N // 8 + 4 * N
        self.metric = f"LIF kernel HBM GB/s (T={T}, N={N}, fp32 spikes + packed + final v)"
        self.unit = "GB/s"
        self.dtype = "f32"

    def config(self):
        return {"workload": f"lif_sweep_T{self.T}_N{self.N}", "T": self.T, "N": self.N,
                "outputs": "fp32 spikes + packed spikes + final v",
                "l2": f"inputs larger than L2 ({4 * self.T * self.N / 2**30:.2f} GiB per step)"}

    def setup(self, rank, world, dist=None):
        self.world = world
        from snn_compiler.kernels import neurons as K
        self.K = K
        T, N = self.T, self.N
        g = torch.Generator(device="cuda").manual_seed(rank)
        self.x = (torch.randn(T, N, device="cuda", generator=g) + 0.5)
        self.sp = torch.empty(T, N, device="cuda")
        self.pk = torch.empty(T, (N + 31) // 32, device="cuda", dtype=torch.int32)
        self.vo = torch.empty(N, device="cuda")
        from snn_compiler import _lib
        self._lib = _lib
        self.L = _lib.lib()
        self.launches_per_step = 1

    def _launch(self, x, sp, pk, vo, stream):
        st = self.L.snnb_neuron_multistep(
            self._lib.ptr(x), 0, self.T, self.N, None, None, 1, 1, 0, 0.5, 0.5, None, 1, 0.0,
            0, 1.0, None, None, self._lib.ptr(sp), 0, self._lib.ptr(pk), None,
            self._lib.ptr(vo), stream)
        self._lib.check(st, "snnb_neuron_multistep")

    def step(self):
        s = torch.cuda.current_stream().cuda_stream
        import ctypes
        self._launch(self.x, self.sp, self.pk, self.vo, ctypes.c_void_p(s))

    def kernel_events(self, steps):
        """Per-launch durations of the dominant kernel (here: the only one)."""
        return None

    def units_per_step(self):
        return self.bytes_per_step / 1e9

    # --- end to end through the public API with host buffers
    def e2e_setup(self):
        T, N = self.T, min(self.N, 1 << 24)
        self.eN = N
        self.hx = torch.randn(T, N).add_(0.5).pin_memory()
        self.hpk = torch.empty(T, (N + 31) // 32, dtype=torch.int32).pin_memory()
        self.hv = torch.empty(N).pin_memory()
        self.e2e_bytes = 4 * T * N + 4 * T * N + T * N // 8 + 4 * N
        self.h2d = 4 * T * N
        self.d2h = 4 * T * ((N + 31) // 32) + 4 * N

    def e2e_step(self):
        xd = self.hx.to("cuda", non_blocking=True)
        r = self.K.neuron_multistep(xd, decay_factor=0.5, input_scale=0.5, packed=True,
                                    v_out=True)
        self.hpk.copy_(r["packed"], non_blocking=True)
        self.hv.copy_(r["v"], non_blocking=True)

    def e2e_units(self):
        return self.e2e_bytes / 1e9

    def roofline(self, kernel_ms, peaks):
        achieved = self.bytes_per_step / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": peaks["source"], "kernel": "neuron_vec8_kernel<float,float>",
                "algorithmic_bytes_per_launch": self.bytes_per_step}

    # --- CPU (oracle) path
    def cpu_sample(self):
        T, N = self.T, 1 << 22
        x = (torch.randn(T, N, generator=torch.Generator().manual_seed(0)) + 0.5).numpy()
        return {"T": T, "N": N, "x": x, "bytes": 4 * T * N + 4 * T * N + T * N // 8 + 4 * N}

    def cpu_run(self, s, threads):
        from oracle import neurons as ON, bitops as OB
        o = ON.lif_multistep(s["x"], df=np.float32(0.5), sc=np.float32(0.5), want_v=True,
                             nthreads=threads)
        OB.pack_rows(o["spikes"])
        return s["bytes"] / 1e9



class VggWorkload:
    """VGG16-SNN T=4 inference, batch 64 per GPU (config 0 at the benchmark batch)."""
    name = "vgg16"
    flush_l2 = True
    load_choices = None
    save_choices = None
    eager = False

    def __init__(self, B=64, T=4):
        self.B, self.T = B, T
        self.metric = "VGG16-SNN T=4 inference images/s (batch 64 per GPU, 32x32x3, 10 classes)"
        self.unit = "images/s"
        self.dtype = "bf16"

    def config(self):
        return {"workload": "vgg16_snn_T4_b64_per_gpu", "model": "VGG16-SNN",
                "layers": "13 conv3x3 + BN(folded) + LIF + 5 maxpool; fc 512-4096-4096-10",
                "T": self.T, "batch_per_gpu": self.B, "global_batch": self.B * self.world,
                "input": "32x32x3 U(0,1), direct encoding", "classes": 10,
                "lif": "tau=2, v_th=1, hard reset 0, decay_input",
                "weights": "Kaiming-normal seeded, BN folded, bf16 (layer 1 f32)",
                "parallelism": f"dp{self.world}",
                "collective": "ShardedInference: NCCL all_gather (at most 4 CTAs) of the "
                              "[64,10] f32 logits per step on a side stream, started once the "
                              "next step's first four launches are done and overlapping its "
                              "later layers"
                              if self.world > 1 else "none",
                "l2": "256 MB buffer written before every timed step",
                "launch": "eager launches" if self.eager else
                          "one CUDA graph per forward (timing events around the dominant launch)",
                "e2e": "two slots (image buffer, logits buffer, captured forward): each step's "
                       "image goes host -> device and its logits device -> host on a copy "
                       "stream, overlapping the neighbouring steps' forwards; consecutive "
                       "steps, L2 not flushed between them (a serving loop)"}

    def setup(self, rank, world, dist=None):
        from snn_compiler.zoo.vgg import SpikingVGG, random_vgg_params
        self.world, self.dist = world, dist
        P = random_vgg_params(1)
        self.eng = SpikingVGG(P, T=self.T, device="cuda")
        if self.load_choices:
            table = json.load(open(self.load_choices))
            self.eng.choice = {tuple(json.loads(k)): tuple(v) for k, v in table.items()}
        g = torch.Generator(device="cuda").manual_seed(1000 + rank)
        self.img = torch.rand(1, self.B, 3, 32, 32, device="cuda", generator=g)
        steps, out = self.eng.plan(self.img)
        for _ in range(3):
            for _, _, fn in steps:
                fn()
        torch.cuda.synchronize()
        # per-launch device time (each layer from its own CUDA graph) -> dominant kernel
        prof = self.eng.profile_layers(self.img)
        self.layer_names = [n for n, _, _ in prof]
        self.layer_flops = [f for _, f, _ in prof]
        self.layer_ms = [m for _, _, m in prof]
        dom = max(range(1, len(steps)), key=lambda i: self.layer_ms[i])
        self.dom = dom
        if self.save_choices and rank == 0:
            json.dump({json.dumps(list(k)): list(v) for k, v in self.eng.choice.items()},
                      open(self.save_choices, "w"))
        self.launches_per_step = self.eng.kernel_launches(self.B)
        if self.eager:
            # launches issued one by one (for profilers that replay single kernels); same work
            self.steps_eager, self.out = steps, out
        else:
            # one graph per forward, with a timing-event pair around the dominant launch
            self.out = self.eng.capture(self.img, mark=dom)
        self.dom_graph = 1
        self._dom_events = []
        self.flops_img = self.eng.flops_per_image()
        self.sharded = None
        if world > 1:
            # the product API: ShardedInference over the engine's graph-replayed forward; the
            # engine writes its logits into the send slot and the all-gather runs on a side
            # stream, issued at the start of the next step (after its L2 flush) so that it
            # overlaps that step's forward and never the untimed flush
            import functools
            from snn_compiler.sharding import ShardedInference
            # the forward in two graphs: the gather of the previous step waits for the first
            # four launches (image layer, band layers: every SM busy) and runs beside the
            # T-folded layers, whose 128-CTA grids leave SMs free
            self._mid_ev = torch.cuda.Event()
            self.sharded = ShardedInference(functools.partial(
                self.eng.forward, graph=True, mid_event=self._mid_ev, mid_at=4))
            gg = torch.Generator(device="cuda").manual_seed(1000)
            self.img_global = torch.rand(1, world * self.B, 3, 32, 32, device="cuda",
                                         generator=gg)
            for _ in range(2 * self.sharded.slots):         # captures one graph per slot
                self.sharded.submit(self.img_global, 1, out_shape=(10,)).wait()
            torch.cuda.synchronize()
            self._prev = None

    def _kernel_label(self, i):
        """Name of the kernel that runs plan step i (the autotuned variant)."""
        name = self.layer_names[i]
        if i == 0:
            return f"first_conv_lif ({name})"
        bs = self.eng.chain_batch(self.B)
        keys = [k for k in self.eng.choice if k[0] != "first" and k[2] == bs]
        key = sorted(keys, key=lambda k: (k[0] != "conv", k[1]))[i - 1] if i - 1 < len(keys) else None
        if key is None:
            return f"linear_head_kernel ({name})"
        v = self.eng.choice[key]
        kern = {1: "conv_lif_kernel", 2: "conv_lif_tm_kernel", 3: "conv_lif_band_kernel",
                4: "conv_lif_tm_kernel (two M-tiles)", 5: "conv_lif_tm_kernel (CTA pairs)",
                6: "conv_lif_tm_kernel (cluster split-K)",
                7: "conv_lif_band_kernel (column taps in the epilogue)",
                8: "linear_t_kernel (transposed, split-K)"}.get(
            v[0], "conv_lif (auto)")
        return f"{kern}<block_n={v[1]}, splits={v[2]}> ({name})"

    def _between(self, i):
        if i == self.dom_graph:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._pending = e
        elif i == self.dom_graph + 1:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._dom_events.append((self._pending, e))

    def _forward(self, between=None):
        if not self.eager:
            return self.eng.replay()
        groups = [range(self.dom), [self.dom], range(self.dom + 1, len(self.steps_eager))]
        for i, grp in enumerate(groups):
            if between is not None:
                between(i)
            for k in grp:
                self.steps_eager[k][2]()
        if between is not None:
            between(len(groups))
        return self.out

    def step(self):
        if self.sharded is None:
            self._forward(between=self._between)
            return
        p = self.sharded.submit(self.img_global, 1, out_shape=(10,), defer=True)
        if self._prev is not None:
            self._prev.start(after=self._mid_ev)      # the last step's all-gather
        self._prev = p

    def finish(self):
        """End of a run of steps: issue the outstanding all-gather and make the current
        stream wait for it (inside the last step's timing)."""
        if self.sharded is not None and self._prev is not None:
            torch.cuda.current_stream().wait_event(self._prev.start().done_event)
            self._prev = None

    def kernel_events(self, steps):
        if self.eager:
            ev = self._dom_events[-steps:]
            return [a.elapsed_time(b) for a, b in ev]
        # the dominant launch inside the one-graph forward: replays after the timed region,
        # each on a flushed L2 as in the timed steps, reading the in-graph event pair
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        out = []
        for _ in range(min(steps, 20)):
            flush.fill_(1)
            self.eng.replay()
            torch.cuda.synchronize()
            a, b = self.eng.mark_events
            out.append(a.elapsed_time(b))
        del flush
        return out

    def units_per_step(self):
        return self.B

    def e2e_setup(self):
        self.h_img = torch.rand(1, self.B, 3, 32, 32).pin_memory()
        n_out = (self.world * self.B if self.world > 1 else self.B) * 10
        self.h_out = torch.empty(n_out).pin_memory()
        self.h2d = self.h_img.numel() * 4
        self.d2h = n_out * 4
        # Serving-style pipeline over two slots: slot k has its own device image buffer, its
        # own logits buffer and its own captured forward.  A step's image crosses PCIe on a
        # copy stream while the previous step computes, and its logits come back on that
        # stream while the next step computes.
        eng = self.eng
        self.slot_in = [torch.empty_like(self.img) for _ in range(2)]
        self.slot_out = [torch.empty_like(self.out) for _ in range(2)]
        self.slot_graphs = []
        if not self.eager and self.sharded is None:
            # (--eager: the slots are copied around eager launches; N > 1: ShardedInference)
            saved = (eng.graphs, eng.graph_out, eng.mark_events, eng.graph_pool)
            for k in range(2):
                eng.capture(self.slot_in[k], out=self.slot_out[k])
                self.slot_graphs.append(eng.graphs)
            eng.graphs, eng.graph_out, eng.mark_events, eng.graph_pool = saved
        self.copy_stream = torch.cuda.Stream()
        self.copied = [torch.cuda.Event() for _ in range(2)]
        self.fwd_done = [torch.cuda.Event() for _ in range(2)]
        self.read_back = [torch.cuda.Event() for _ in range(2)]
        self._e2e_i, self._e2e_pending = 0, False

    def e2e_begin(self):
        """Before the timed region: drain the copy stream; the first timed step then issues
        its own image copy inside the region."""
        torch.cuda.synchronize()
        self._e2e_pending = False

    def _h2d(self, k):
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.fwd_done[k])      # slot k's last forward is done
            self.slot_in[k].copy_(self.h_img, non_blocking=True)
            self.copied[k].record(self.copy_stream)

    def e2e_step(self):
        k = self._e2e_i % 2
        if not self._e2e_pending:
            self._h2d(k)
        s = torch.cuda.current_stream()
        s.wait_event(self.copied[k])
        s.wait_event(self.read_back[k])      # slot k's logits of two steps ago are on the host
        pend = None
        if self.sharded is not None:
            # this rank's images through ShardedInference: graph-replayed forward into the
            # send slot, all-gather on the side stream, logits back on the copy stream
            pend = self.sharded.submit_local(self.slot_in[k], self.world * self.B, 1,
                                             out_shape=(10,))
        elif self.eager:
            self.img.copy_(self.slot_in[k], non_blocking=True)
            self._forward()
            self.slot_out[k].copy_(self.out, non_blocking=True)
        else:
            for g in self.slot_graphs[k]:
                g.replay()
        self.fwd_done[k].record(s)
        self._h2d(1 - k)                     # the next step's image
        self._e2e_pending = True
        if pend is not None:
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(pend.done_event)
                self.h_out.copy_(pend.wait().view(-1), non_blocking=True)
                self.read_back[k].record(self.copy_stream)
        else:
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(self.fwd_done[k])
                self.h_out.copy_(self.slot_out[k].view(-1), non_blocking=True)
                self.read_back[k].record(self.copy_stream)
        self._e2e_i += 1

    def e2e_units(self):
        return self.B

    def roofline(self, kernel_ms, peaks):
        flops = self.layer_flops[self.dom]
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        peak = peaks["bf16_tflops"]
        traffic = None
        tp = os.path.join(REPO, "profiles", "dram_traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get(self.layer_names[self.dom])
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": peaks["source"] + " bf16 burst (cuBLAS)",
                "kernel": self._kernel_label(self.dom),
                "algorithmic_flops_per_launch": flops,
                "kernel_ms": round(kernel_ms, 5),
                "per_layer_device_ms": {n: round(t, 4) for n, t in
                                        zip(self.layer_names, self.layer_ms)},
                "per_layer_device_ms_note": "each launch alone, 10 back-to-back in a graph, "
                                            "warm L2",
                "per_layer_in_step_ms": {n: round(t, 4) for n, t in
                                         self.eng.layer_times_in_step(self.img)},
                "per_layer_in_step_ms_note": "inside one forward graph, events around every "
                                             "launch, L2 flushed before each replay, median of 10",
                "choices": {str(k): v for k, v in self.eng.choice.items()},
                "model_tflops_per_s": None}

    def cpu_sample(self):
        from oracle import params as OP
        P = OP.vgg16_params(1)
        B = 16
        x = OP.vgg16_input(0, T=self.T, B=B)
        return {"B": B, "T": self.T, "P": P, "x": x, "what": "oracle VGG16 forward, torch-CPU f32 conv + C LIF"}

    def cpu_run(self, s, threads):
        from oracle import vgg as OV
        torch.set_num_threads(threads)
        OV.vgg16_forward(s["x"], s["P"], weights="fp32")
        return s["B"]


class ConvLayerWorkload:
    """One fused conv3x3 + BN(folded) + LIF + 2x2 max-pool layer (config 2); with k / stride
    other than 3 / 1 a ResNet conv instead (3x3 / stride 2 or 1x1, no pool:
    snnb_conv_lif_strided)."""
    name = "conv"
    flush_l2 = True

    def __init__(self, cin=512, cout=512, H=56, B=64, T=4, p=0.15, fixed=None, packed="none",
                 k=3, stride=1):
        self.cin, self.cout, self.H, self.B, self.T, self.p = cin, cout, H, B, T, p
        self.fixed = fixed
        self.k, self.stride = k, stride
        self.strided = (k, stride) != (3, 1)
        assert not (self.strided and packed != "none"), "packed spikes: 3x3 / stride 1 only"
        self.Ho = (H - 1) // stride + 1 if self.strided else H // 2
        # packed spikes between layers: "in" / "out" / "both" run snnb_conv3x3_lif_packed
        self.pk_in, self.pk_out = packed in ("in", "both"), packed in ("out", "both")
        self.packed = packed
        if self.strided:
            self.flops = 2 * T * B * self.Ho * self.Ho * cout * cin * k * k
            self.metric = (f"fused conv{k}x{k}/stride {stride}+BN+LIF TFLOP/s (ResNet conv; Cin={cin}, "
                           f"Cout={cout}, H=W={H}, B={B}, T={T})")
        else:
            self.flops = 2 * T * B * H * H * cout * cin * 9
            pk = "" if packed == "none" else f", packed spikes {packed}"
            self.metric = f"fused conv3x3+BN+LIF+maxpool TFLOP/s (Cin={cin}, Cout={cout}, H=W={H}, B={B}, T={T}{pk})"
        self.unit = "TFLOP/s"
        self.dtype = "bf16"

    def config(self):
        if self.strided:
            return {"workload": f"resnet_conv{self.k}x{self.k}s{self.stride}_{self.cin}x{self.cout}@{self.H}",
                    "T": self.T, "B": self.B, "Cin": self.cin, "Cout": self.cout, "H": self.H,
                    "W": self.H, "kernel": self.k, "stride": self.stride, "spike_p": self.p,
                    "pool": "none", "l2": "256 MB buffer written before every step"}
        return {"workload": f"conv_layer_{self.cin}x{self.cout}@{self.H}", "T": self.T,
                "B": self.B, "Cin": self.cin, "Cout": self.cout, "H": self.H, "W": self.H,
                "spike_p": self.p, "pool": "max 2x2", "packed_spikes": self.packed,
                "l2": "256 MB buffer written before every step"}

    def setup(self, rank, world, dist=None):
        from snn_compiler.kernels import conv as KC
        self.KC = KC
        self.world = world
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        T, B, H, C = self.T, self.B, self.H, self.cin
        self.x = (torch.rand(T, B, H, H, C, device="cuda", generator=g) < self.p).to(torch.bfloat16)
        k = self.k
        w = torch.randn(self.cout, k, k, C, device="cuda", generator=g) * (2.0 / (k * k * C)) ** 0.5
        self.w = w.to(torch.bfloat16).contiguous()
        self.b = torch.rand(self.cout, device="cuda", generator=g) * 0.9 + 0.3
        self.out = torch.empty(T, B, self.Ho, self.Ho, self.cout, device="cuda",
                               dtype=torch.bfloat16)
        self.ws = None
        if self.strided:
            run = lambda v, bn, sp: KC.conv_lif_strided(self.x, self.w, self.b, stride=self.stride,
                                                        out=self.out, variant=v, block_n=bn,
                                                        splits=sp)
            self.choice = self.fixed if self.fixed else KC.pick_fastest(
                run, self.cout, T, k * k * ((C + 63) // 64), variants=(1, 2))
            nws = KC.split_workspace_bytes(T, B, self.Ho, self.Ho, self.cout, self.choice[2])
            self.ws = torch.empty(nws // 4, device="cuda") if nws else None
            self.launches_per_step = 1
            return
        if self.pk_in or self.pk_out:
            # packed spikes: the T-folded kernel; the fastest channel block
            self.xin = KC.pack_spikes(self.x) if self.pk_in else self.x
            if self.pk_out:
                self.out = torch.empty(T, B, H // 2, H // 2, self.cout // 32, device="cuda",
                                       dtype=torch.int32)
            run = lambda bn: KC.conv3x3_lif_packed(self.xin, self.w, self.b, x_packed=self.pk_in,
                                                   out_packed=self.pk_out, pool=True,
                                                   block_n=bn, out=self.out)
            if self.fixed:
                self.choice = (2, self.fixed[1], 1)
            else:
                bns = [bn for bn in (64, 128, 256) if self.cout % bn == 0]
                times = [KC.time_graph(lambda bn=bn: run(bn), 10) for bn in bns]
                self.choice = (2, bns[times.index(min(times))], 1)
            self.launches_per_step = 1
            return
        # pick the fastest (variant, block_n) the way the VGG engine does
        run = lambda v, bn, sp: KC.conv3x3_lif(self.x, self.w, self.b, pool=True, out=self.out,
                                               variant=v, block_n=bn, splits=sp)
        self.choice = self.fixed if self.fixed else KC.pick_fastest(
            run, self.cout, T, 9 * C // 64, band=KC.band_block_ns(H, C, self.cout),
            band_xs=KC.band_xs_block_ns(H, C, self.cout))
        nws = KC.split_workspace_bytes(T, B, H, H, self.cout, self.choice[2])
        self.ws = torch.empty(nws // 4, device="cuda") if nws else None
        self.launches_per_step = 1

    def step(self):
        v, bn, sp = self.choice
        if self.strided:
            self.KC.conv_lif_strided(self.x, self.w, self.b, stride=self.stride, out=self.out,
                                     variant=v, block_n=bn, splits=sp, workspace=self.ws)
            return
        if self.pk_in or self.pk_out:
            self.KC.conv3x3_lif_packed(self.xin, self.w, self.b, x_packed=self.pk_in,
                                       out_packed=self.pk_out, pool=True, block_n=bn,
                                       out=self.out)
            return
        self.KC.conv3x3_lif(self.x, self.w, self.b, pool=True, out=self.out, variant=v, block_n=bn,
                            splits=sp, workspace=self.ws)

    def kernel_events(self, steps):
        return None

    def units_per_step(self):
        return self.flops / 1e12

    def e2e_setup(self):
        xin = self.xin if (self.pk_in or self.pk_out) else self.x
        self.hx = xin.cpu().pin_memory()
        self.hout = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = self.hx.numel() * self.hx.element_size()
        self.d2h = self.hout.numel() * self.hout.element_size()

    def e2e_step(self):
        (self.xin if (self.pk_in or self.pk_out) else self.x).copy_(self.hx, non_blocking=True)
        self.step()
        self.hout.copy_(self.out, non_blocking=True)

    def e2e_units(self):
        return self.flops / 1e12

    def roofline(self, kernel_ms, peaks):
        achieved = self.flops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": peaks["source"] + " bf16 burst (cuBLAS)",
                "kernel": (f"conv_lif{' strided' if self.strided else ''} "
                           f"(variant, block_n, splits = {self.choice})"),
                "algorithmic_flops_per_launch": self.flops, "traffic": None}

    def cpu_sample(self):
        from oracle import params as OP
        B, H, C, k = 1, self.H, self.cin, self.k
        x = OP.spikes(0, (self.T, B, C, H, H), self.p)
        w = torch.randn(self.cout, C, k, k, generator=OP.gen(1)) * (2.0 / (k * k * C)) ** 0.5
        b = torch.rand(self.cout, generator=OP.gen(2)) * 0.9 + 0.3
        what = "oracle conv+LIF, torch-CPU f32" if self.strided else \
            "oracle conv+LIF+pool, torch-CPU f32"
        return {"B": B, "x": x, "w": w, "b": b, "what": what}

    def cpu_run(self, s, threads):
        torch.set_num_threads(threads)
        if self.strided:
            from oracle import resnet as OR
            OR.conv_bn_neuron(s["x"], s["w"], s["b"], stride=self.stride, padding=self.k // 2)
            return 2 * self.T * s["B"] * self.Ho * self.Ho * self.cout * self.cin * self.k ** 2 / 1e12
        from oracle import vgg as OV
        OV.conv_bn_lif_pool(s["x"], s["w"], s["b"], pool=True)
        return 2 * self.T * s["B"] * self.H * self.H * self.cout * self.cin * 9 / 1e12


class ResNetWorkload:
    """Spiking ResNet-18 (the reference zoo's ResNetSNN: 7x7 / stride 2 stem + BN + LIF,
    3x3 / stride 2 max-pool, four BasicBlock stages with 1x1 / stride 2 downsample branches,
    global average pool, linear head) at T = 4 on 224x224 images, batch 64, bf16, fused
    (BN folded): every conv on this library's kernels, the forward captured as one CUDA
    graph.  The image is the same at every step (direct encoding)."""
    name = "resnet18"
    flush_l2 = True

    def __init__(self, B=64, T=4, H=224, classes=10):
        self.B, self.T, self.H, self.classes = B, T, H, classes
        self.metric = (f"ResNet-18-SNN T={T} inference images/s (batch {B} per GPU, "
                       f"{H}x{H}x3, {classes} classes)")
        self.unit = "images/s"
        self.dtype = "bf16"

    def config(self):
        return {"workload": f"resnet18_snn_T{self.T}_b{self.B}_{self.H}px", "model": "ResNet-18-SNN",
                "T": self.T, "batch_per_gpu": self.B, "input": f"{self.H}x{self.H}x3 U(0,1), direct encoding",
                "classes": self.classes, "lif": "tau=2, v_th=1, hard reset 0, decay_input",
                "weights": "Kaiming-uniform (torch default) seeded, BN stats randomised and folded, bf16",
                "layout": "NHWC (channels-last storage)",
                "launch": "one CUDA graph per forward; per-layer kernel schedules from "
                          "snn_compiler.nn.tune_convs; torch ops for the average pool and head",
                "l2": "256 MB buffer written before every timed step"}

    def _model(self):
        from snn_compiler.zoo import resnet18_snn
        torch.manual_seed(0)
        m = resnet18_snn(num_classes=self.classes, layout="NHWC")
        with torch.no_grad():       # a lively network: every layer spikes
            for mod in m.modules():
                if isinstance(mod, torch.nn.Conv2d):
                    mod.weight.mul_(3.0)
                if isinstance(mod, torch.nn.BatchNorm2d):
                    mod.bias.add_(0.3)
        return m.eval().fuse()

    def setup(self, rank, world, dist=None):
        from snn_compiler.nn import FusedConvBN, FusedConvBNAddNeuron, FusedConvBNNeuron
        self.world = world
        self.m = self._model().to("cuda").to(torch.bfloat16)
        g = torch.Generator(device="cuda").manual_seed(5 + rank)
        img = torch.rand(1, self.B, 3, self.H, self.H, device="cuda", generator=g)
        self.x = self._nhwc(img.expand(self.T, -1, -1, -1, -1).to(torch.bfloat16))
        # FLOPs of every conv (dense, padding zeros counted) from one forward's shapes
        self.flops = 0
        kinds = (FusedConvBN, FusedConvBNNeuron, FusedConvBNAddNeuron)

        def hook(mod, inp, out):
            k = mod.weight.shape[2] * mod.weight.shape[3]
            self.flops += 2 * out.numel() * mod.weight.shape[1] * k
        hs = [mod.register_forward_hook(hook) for mod in self.m.modules() if isinstance(mod, kinds)]
        with torch.no_grad():
            self.m(self.x)
        for h in hs:
            h.remove()
        self.n_convs = sum(1 for mod in self.m.modules() if isinstance(mod, kinds))
        self.flops_img = self.flops / self.B
        # per-layer kernel schedules, timed on each conv's real input (snn_compiler.nn.tune_convs)
        from snn_compiler.nn import tune_convs
        self.choices = tune_convs(self.m, self.x)
        # capture the forward (warm the modules' weight caches first)
        with torch.no_grad():
            for _ in range(2):
                self.m(self.x)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.out = self.m(self.x)
        torch.cuda.synchronize()
        # this library's launches per forward: one per conv, the bias-add launch of each
        # float32 downsample conv, the stem's window gather and its max-pool
        self.launches_per_step = self.n_convs + sum(
            1 for mod in self.m.modules() if isinstance(mod, FusedConvBN)) + 2

    @staticmethod
    def _nhwc(t):
        T, B = t.shape[:2]
        return t.reshape(T * B, *t.shape[2:]).contiguous(memory_format=torch.channels_last) \
            .view(T, B, *t.shape[2:])

    def step(self):
        self.graph.replay()

    def kernel_events(self, steps):
        return None

    def units_per_step(self):
        return self.B

    def roofline(self, kernel_ms, peaks):
        achieved = self.flops / (kernel_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": peaks["source"] + " bf16 burst (cuBLAS)",
                "kernel": "whole forward (one CUDA graph; every conv on the tcgen05 kernels)",
                "algorithmic_flops_per_launch": self.flops, "traffic": None,
                "choices": {k: list(v) for k, v in self.choices.items()}}

    def e2e_setup(self):
        self.hx = self.x.cpu().pin_memory()
        self.hout = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = self.hx.numel() * self.hx.element_size()
        self.d2h = self.hout.numel() * self.hout.element_size()

    def e2e_step(self):
        self.x.copy_(self.hx, non_blocking=True)
        self.graph.replay()
        self.hout.copy_(self.out, non_blocking=True)

    def e2e_units(self):
        return self.B

    def cpu_sample(self):
        """One image through the reference's CPU path, restated by the oracle per fused
        module (torch-CPU float32 conv, C LIF), with the same folded weights."""
        m = self._model()                   # float32 weights on the CPU
        g = torch.Generator().manual_seed(5)
        img = torch.rand(1, 1, 3, self.H, self.H, generator=g).expand(self.T, 1, 3, self.H, self.H)
        return {"B": 1, "m": m, "x": img.contiguous(), "what": "oracle ResNet-18-SNN forward, torch-CPU f32 conv + C LIF"}

    def cpu_run(self, s, threads):
        import torch.nn.functional as F
        from oracle import resnet as OR
        torch.set_num_threads(threads)
        m, x = s["m"], s["x"]
        T, B = x.shape[:2]

        def frames(t, fn):
            y = fn(t.reshape(T * B, *t.shape[2:]))
            return y.reshape(T, B, *y.shape[1:])
        x = OR.fused_module_oracle(m.stem_fused, x)[0]
        x = frames(x, lambda z: F.max_pool2d(z, 3, 2, 1))
        for b in m.blocks():
            out = OR.fused_module_oracle(b.block1, x)[0]
            idn = x if b.downsample is None else OR.conv_bias(
                x, b.downsample.weight, b.downsample.bias, stride=b.downsample.stride,
                padding=b.downsample.padding)
            x = OR.fused_module_oracle(b.block2, out, residual=idn)[0]
        f = x.mean(dim=(3, 4)).reshape(T * B, -1)
        m.fc(f).view(T, B, -1)
        return s["B"]


class FirstLayerWorkload:
    """The image (first) layer of VGG16-SNN on its own: float32 image [1, B, 3, 32, 32]
    (direct encoding) -> conv3x3 3->64 + folded BN + LIF over T steps -> spikes
    [T, B, 32, 32, 64] bf16.  The tensor-core kernel (split operands) or the CUDA-core one,
    whichever is faster (or `--choice 1` / `0`)."""
    name = "first"
    flush_l2 = True

    def __init__(self, B=64, T=4, cin=3, cout=64, H=32, fixed=None):
        self.B, self.T, self.cin, self.cout, self.H = B, T, cin, cout, H
        self.fixed = fixed
        self.flops = 2 * T * B * H * H * cout * cin * 9
        # algorithmic bytes: the image read once, the spikes written once
        self.bytes = 4 * B * cin * H * H + 2 * T * B * H * H * cout
        self.metric = (f"image layer conv3x3 {cin}->{cout} (float32 image, split-operand tensor "
                       f"cores) + LIF TFLOP/s (H=W={H}, B={B}, T={T})")
        self.unit = "TFLOP/s"
        self.dtype = "f32 (as 3 bf16 terms)"

    def config(self):
        return {"workload": f"image_layer_{self.cin}x{self.cout}@{self.H}", "T": self.T,
                "B": self.B, "Cin": self.cin, "Cout": self.cout, "H": self.H, "W": self.H,
                "input": "U(0,1) float32 image, direct encoding",
                "l2": "256 MB buffer written before every step"}

    def setup(self, rank, world, dist=None):
        from snn_compiler.kernels import conv as KC
        self.KC = KC
        g = torch.Generator(device="cuda").manual_seed(11 + rank)
        B, C, H = self.B, self.cin, self.H
        self.img = torch.rand(1, B, C, H, H, device="cuda", generator=g)
        self.w = torch.randn(self.cout, C, 3, 3, device="cuda", generator=g) * (2.0 / (9 * C)) ** 0.5
        self.b = torch.rand(self.cout, device="cuda", generator=g) * 0.5 + 0.2
        self.ws = KC.first_conv_split_weight(self.w)
        self.out = torch.empty(self.T, B, H, H, self.cout, device="cuda", dtype=torch.bfloat16)
        runs = [lambda: KC.first_conv_lif(self.img, self.w, self.b, T=self.T, out=self.out),
                lambda: KC.first_conv_lif_tc(self.img, self.ws, self.b, T=self.T, out=self.out)]
        if self.fixed is not None:
            self.choice = self.fixed
        else:
            times = [KC.time_graph(r, 10) for r in runs]
            self.choice = times.index(min(times))
        self.run = runs[self.choice]
        self.launches_per_step = 1

    def step(self):
        self.run()

    def kernel_events(self, steps):
        return None

    def units_per_step(self):
        return self.flops / 1e12

    def e2e_setup(self):
        self.hx = self.img.cpu().pin_memory()
        self.hout = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.h2d = self.hx.numel() * self.hx.element_size()
        self.d2h = self.hout.numel() * self.hout.element_size()

    def e2e_step(self):
        self.img.copy_(self.hx, non_blocking=True)
        self.step()
        self.hout.copy_(self.out, non_blocking=True)

    def e2e_units(self):
        return self.flops / 1e12

    def roofline(self, kernel_ms, peaks):
        # the layer's tensor work is small (0.9 GFLOP standard count); its one large stream
        # is the spikes it writes, so it is reported against HBM bandwidth
        gbs = self.bytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                "peak_source": peaks["source"] + " HBM copy",
                "kernel": ["first_conv_quad_kernel (CUDA cores)",
                           "first_conv_tc_kernel (tcgen05, split operands)"][self.choice],
                "algorithmic_bytes_per_launch": self.bytes,
                "tflops": round(self.flops / (kernel_ms * 1e-3) / 1e12, 2), "traffic": None}

    def cpu_sample(self):
        from oracle import params as OP
        B, H, C = 32, self.H, self.cin
        img = torch.rand(1, B, C, H, H, generator=OP.gen(3))
        w = torch.randn(self.cout, C, 3, 3, generator=OP.gen(1)) * (2.0 / (9 * C)) ** 0.5
        b = torch.rand(self.cout, generator=OP.gen(2)) * 0.5 + 0.2
        return {"B": B, "x": img.expand(self.T, B, C, H, H).contiguous(), "w": w, "b": b,
                "what": "oracle conv+LIF, torch-CPU f32"}

    def cpu_run(self, s, threads):
        from oracle import vgg as OV
        torch.set_num_threads(threads)
        OV.conv_bn_lif_pool(s["x"], s["w"], s["b"], pool=False)
        return 2 * self.T * s["B"] * self.H * self.H * self.cout * self.cin * 9 / 1e12


class AttnWorkload:
    """Spiking self-attention block (config 3): x [T=4, B=32, N=196, D=384] spikes, 12 heads."""
    name = "attention"
    flush_l2 = True

    def __init__(self, B=32, T=4, N=196, D=384, H=12):
        self.B, self.T, self.N, self.D, self.H = B, T, N, D, H
        M = T * B * N
        d = D // H
        self.flops = 2 * M * D * 3 * D + 2 * M * D * D + T * B * H * 4 * N * d * d
        self.metric = ("spiking self-attention block TFLOP/s (T=4, B=32, N=196, D=384, 12 heads; "
                       "Q/K/V Linear+BN+LIF, (QK^T)V*0.125 + LIF, proj Linear+BN+LIF)")
        self.unit = "TFLOP/s"
        self.dtype = "bf16"

    def config(self):
        return {"workload": "spike_attention_block_T4_B32_N196_D384", "T": self.T,
                "batch_per_gpu": self.B, "tokens": self.N, "dim": self.D, "heads": self.H,
                "input": "Bernoulli(0.15) spikes", "weights": "N(0, 0.02) seeded, BN folded, bf16",
                "l2": "256 MB buffer written before every step"}

    def setup(self, rank, world, dist=None):
        from snn_compiler.kernels import conv as KC
        from snn_compiler.nn.attention import SpikeAttentionBlock, random_attention_params
        self.world = world
        self.blk = SpikeAttentionBlock(random_attention_params(1, D=self.D), heads=self.H,
                                       scale=0.125, qkv_vth=1.0, attn_vth=0.5, out_vth=1.0)
        g = torch.Generator(device="cuda").manual_seed(11 + rank)
        self.x = (torch.rand(self.T, self.B, self.N, self.D, device="cuda", generator=g)
                  < 0.15).to(torch.bfloat16)
        stages = self.blk.stages(self.x)
        self.stage_names = [s[0] for s in stages]
        self.stage_flops = [s[1] for s in stages]
        self.stage_ms = [KC.time_graph(s[2]) for s in stages]
        self.dom = max(range(len(stages)), key=lambda i: self.stage_ms[i])
        self.launches_per_step = 3
        self._fns = [s[2] for s in stages]
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for fn in self._fns:
                fn()

    def step(self):
        self.graph.replay()

    def kernel_events(self, steps):
        return None

    def units_per_step(self):
        return self.flops / 1e12

    def e2e_setup(self):
        self.hx = self.x.cpu().pin_memory()
        T, B, N, D = self.x.shape
        self.hy = torch.empty(T, B * N, D, dtype=torch.bfloat16).pin_memory()
        self.h2d = self.hx.numel() * 2
        self.d2h = self.hy.numel() * 2

    def e2e_step(self):
        self.x.copy_(self.hx, non_blocking=True)
        y = self.blk.forward(self.x)
        self.hy.copy_(y.view(self.hy.shape), non_blocking=True)

    def e2e_units(self):
        return self.flops / 1e12

    def roofline(self, kernel_ms, peaks):
        # dominant launch timed alone from its own graph
        ms = self.stage_ms[self.dom]
        achieved = self.stage_flops[self.dom] / (ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": peaks["source"] + " bf16 burst (cuBLAS)",
                "kernel": self.stage_names[self.dom], "traffic": None,
                "per_stage_device_ms": {n: round(m, 4) for n, m in
                                        zip(self.stage_names, self.stage_ms)},
                "block_ms": round(kernel_ms, 4)}

    def cpu_sample(self):
        from oracle import params as OP
        B = 2
        return {"B": B, "x": OP.spikes(0, (self.T, B, self.N, self.D), 0.15),
                "P": OP.attention_params(1, D=self.D, heads=self.H),
                "what": "oracle SSA block, torch-CPU f32 linears + C LIF"}

    def cpu_run(self, s, threads):
        from oracle import attention as OA
        torch.set_num_threads(threads)
        OA.ssa_forward(s["x"], s["P"], heads=self.H, qkv_vth=1.0, attn_vth=0.5, out_vth=1.0)
        return self.flops * s["B"] / self.B / 1e12


class BgemmWorkload:
    """Bit-packed {0,1} x {-1,+1} GEMM (config 4): A Bernoulli(0.2) [M, K], B +-1 [K, N]."""
    name = "bgemm"
    flush_l2 = True

    def __init__(self, M=16384, K=8192, N=8192):
        self.M, self.K, self.N = M, K, N
        w = (K + 31) // 32
        self.bytes = 4 * w * (M + N) + 4 * M * N          # packed A + packed B + int32 C
        self.word_ops = M * N * w
        self.metric = f"binary GEMM (AND+popcount) GB/s, M={M} K={K} N={N}"
        self.unit = "GB/s"
        self.dtype = "u32"

    def config(self):
        return {"workload": f"bgemm_{self.M}x{self.K}x{self.N}", "M": self.M, "K": self.K,
                "N": self.N, "A": "Bernoulli(0.2) {0,1}", "B": "+-1 p=0.5",
                "bytes_per_step": self.bytes, "word_ops_per_step": self.word_ops,
                "l2": "256 MB buffer written before every step"}

    def setup(self, rank, world, dist=None):
        from snn_compiler.kernels import binary as KB
        self.KB = KB
        self.world = world
        g = torch.Generator(device="cuda").manual_seed(3 + rank)
        A = (torch.rand(self.M, self.K, device="cuda", generator=g) < 0.2).to(torch.uint8)
        Bt = (torch.rand(self.N, self.K, device="cuda", generator=g) < 0.5).to(torch.uint8)
        self.Ap, self.Bp = KB.bitpack(A), KB.bitpack(Bt)
        self.C = torch.empty(self.M, self.N, device="cuda", dtype=torch.int32)
        del A, Bt
        self.launches_per_step = 1

    def step(self):
        self.KB.bgemm(self.Ap, self.Bp, self.K, mode=1, out=self.C)

    def kernel_events(self, steps):
        return None

    def units_per_step(self):
        return self.bytes / 1e9

    def e2e_setup(self):
        self.hA, self.hB = self.Ap.cpu().pin_memory(), self.Bp.cpu().pin_memory()
        self.hC = torch.empty(self.C.shape, dtype=torch.int32).pin_memory()
        self.h2d = (self.hA.numel() + self.hB.numel()) * 4
        self.d2h = self.hC.numel() * 4

    def e2e_step(self):
        self.Ap.copy_(self.hA, non_blocking=True)
        self.Bp.copy_(self.hB, non_blocking=True)
        self.step()
        self.hC.copy_(self.C, non_blocking=True)

    def e2e_units(self):
        return self.bytes / 1e9

    @staticmethod
    def popc_peak():
        """Measured peak of the contraction's inner operation (AND + POPC + add per 32-bit
        word) on this GPU: snnb_popc_peak, 4 CTAs of 256 threads per SM, best of 3 timed
        launches after a warm-up (word-ops per second)."""
        from snn_compiler import _lib
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        blocks, iters = 4 * sms, 4096
        sink = torch.empty(256, dtype=torch.int32, device="cuda")
        L = _lib.lib()
        run = lambda: _lib.check(L.snnb_popc_peak(blocks, iters, _lib.ptr(sink),
                                                  _lib.stream_of(sink)), "snnb_popc_peak")
        run()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            run()
            b.record()
            b.synchronize()
            best = min(best, a.elapsed_time(b))
        return blocks * 256 * iters * 64 / (best * 1e-3)

    def roofline(self, kernel_ms, peaks):
        # the AND + popcount contraction is bound by the integer pipes (DRAM ~0.3% in ncu):
        # its roofline is the measured rate of the same word-op mix, not HBM bandwidth
        achieved = self.word_ops / (kernel_ms * 1e-3)
        peak = self.popc_peak()
        gbs = self.bytes / (kernel_ms * 1e-3) / 1e9
        return {"bound": "integer (AND + popcount)", "achieved": round(achieved / 1e12, 3),
                "peak": round(peak / 1e12, 3), "unit": "T word-ops/s",
                "frac": round(achieved / peak, 4),
                "peak_source": "measured on this GPU: snnb_popc_peak (acc += popc(a & b) on "
                               "registers, 64 independent chains per thread)",
                "kernel": "bgemm_kernel<1>", "traffic": None,
                "hbm": {"achieved_gbs": round(gbs, 1), "peak_gbs": peaks["hbm_gbs"],
                        "frac": round(gbs / peaks["hbm_gbs"], 4)}}

    def cpu_sample(self):
        from oracle import params as OP
        M = 64
        A, Bb = OP.binary_gemm_operands(4, M, self.K, self.N)
        return {"M": M, "A": A.numpy().astype("int8"), "B": (Bb.numpy().astype("int8") * 2 - 1),
                "what": "oracle unpacked integer matmul (numpy, int64 accumulate) on 64 rows"}

    def cpu_run(self, s, threads):
        import numpy as np
        torch.set_num_threads(threads)
        a = torch.from_numpy(s["A"].astype(np.float32))
        b = torch.from_numpy(s["B"].astype(np.float32))
        torch.matmul(a, b)                   # exact: |sums| < 2^24
        w = (self.K + 31) // 32
        return (4 * w * (s["M"] + self.N) + 4 * s["M"] * self.N) / 1e9

# ----------------------------------------------------------------------------------------
def time_cpu(workload, threads, reps=3):
    s = workload.cpu_sample()
    workload.cpu_run(s, threads)          # warm-up
    ts = []
    units = 0
    for _ in range(reps):
        t0 = time.perf_counter()
        units = workload.cpu_run(s, threads)
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return units / med, s, med


def run_reference(args, workload):
    """CPU arm: the reference's algorithm (oracle restatement) on all host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle import neurons as ON
    cores = min(threads, ON.max_threads()) if workload.name == "lif" else threads
    vals = []
    s = workload.cpu_sample()
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        u = workload.cpu_run(s, threads)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            vals.append((u, dt))
    tot_u = sum(u for u, _ in vals)
    tot_t = sum(t for _, t in vals)
    v = tot_u / tot_t
    sample = {k: v_ for k, v_ in s.items() if isinstance(v_, (int, float, str))}
    line = {"metric": workload.metric, "value": round(v, 3), "unit": workload.unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * tot_t / len(vals), 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": workload.dtype,
            "data": "synthetic", "config": workload.config(), "impl": "reference",
            "cpu_baseline": {"value": round(v, 3), "unit": workload.unit, "cores": cores,
                             "kind": "port", "sample": json.dumps(sample)},
            "e2e": {"value": round(v, 3), "unit": workload.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def lif_kernel_object(dist, rank, world, local, peaks, T=32, N=1 << 27, steps=5, warmup=3):
    """The second half of the headline metric: the standalone multi-step LIF kernel's HBM
    bandwidth at T=32, N=2^27 float32 per GPU (config 1's largest point), fp32 spikes +
    packed spikes + final v, timed after the VGG16 region in the same process.  Byte model
    per launch: 4TN (x) + 4TN (spikes) + TN/8 (packed) + 4N (v) -- the reference's model
    (snn_compiler/explore/large_T/bench_baseline.py:45, 8 bytes per neuron-step) plus this
    build's extra outputs.  Every rank runs its own N (weak scaling); the value is the sum
    of the ranks' bytes over the slowest rank's time."""
    wl = LifWorkload(T=T, N=N)
    wl.setup(rank, world, dist)
    for _ in range(warmup):
        wl.step()
    barrier(dist)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    t0 = time.time()
    for i in range(steps):
        ev[i][0].record(stream)
        wl.step()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    ms = [a.elapsed_time(b) for a, b in ev]
    tot = max_over_ranks(dist, sum(ms))
    if sampler:
        sampler.mark(t0, t1)
    clocks = sampler.stop() if sampler else None
    slowest_mean = max_over_ranks(dist, statistics.mean(ms))
    per_gpu = wl.bytes_per_step / (slowest_mean * 1e-3) / 1e9      # the slowest rank's
    total = world * wl.bytes_per_step * steps / (tot * 1e-3) / 1e9
    del wl
    torch.cuda.empty_cache()
    return {"metric": f"LIF kernel HBM GB/s (T={T}, N=2^{N.bit_length() - 1} float32 per GPU, "
                      "fp32 spikes + packed spikes + final v)",
            "value": round(total, 1), "unit": "GB/s", "n_gpus": world,
            "per_gpu_gbs": round(per_gpu, 1), "peak": peaks["hbm_gbs"],
            "frac": round(per_gpu / peaks["hbm_gbs"], 4),
            "peak_source": peaks["source"] + " HBM copy",
            "kernel": "neuron_vec8_kernel<float,float>",
            "ms_per_launch": round(tot / steps, 4), "steps": steps, "warmup": warmup,
            "algorithmic_bytes_per_launch": 4 * T * N + 4 * T * N + T * N // 8 + 4 * N,
            "byte_model": "4TN x + 4TN spikes + TN/8 packed + 4N final v",
            "l2": "inputs larger than L2 (16 GiB per tensor)", "clocks": clocks}


def run_ours(args, workload):
    rank, world, local, dist = dist_setup(args)
    peaks = load_peaks()
    workload.setup(rank, world, dist)
    flush = None
    if getattr(workload, "flush_l2", False):
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(args.warmup):
        workload.step()
        if flush is not None:
            flush.fill_(1)
    if hasattr(workload, "finish"):
        workload.finish()
    barrier(dist)
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_wall0 = time.time()
    for i in range(args.steps):
        if flush is not None:
            flush.fill_(1)
        ev[i][0].record(stream)
        workload.step()
        if i == args.steps - 1 and hasattr(workload, "finish"):
            workload.finish()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    barrier(dist)
    t_wall1 = time.time()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    my_ms = sum(step_ms)
    total_ms = max_over_ranks(dist, my_ms)
    kern = workload.kernel_events(args.steps)
    kernel_ms = statistics.mean(kern) if kern else statistics.mean(step_ms)
    kernel_ms = max_over_ranks(dist, kernel_ms)
    if sampler:
        sampler.mark(t_wall0, t_wall1)
    clocks = sampler.stop() if sampler else None
    units = sum_over_ranks(dist, workload.units_per_step() * args.steps)
    value = units / (total_ms * 1e-3)
    roof = workload.roofline(kernel_ms, peaks)
    if getattr(workload, "flops_img", None):
        roof["model_tflops_per_s"] = round(value * workload.flops_img / 1e12 / world, 2)

    # end to end through the public API, host buffers, copies inside the timed region
    workload.e2e_setup()
    for _ in range(max(1, args.warmup)):
        workload.e2e_step()
    barrier(dist)
    if hasattr(workload, "e2e_begin"):
        workload.e2e_begin()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, min(args.steps, 50))
    e0.record(stream)
    for _ in range(e_steps):
        workload.e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(dist, e0.elapsed_time(e1))
    e_units = sum_over_ranks(dist, workload.e2e_units() * e_steps)
    e2e = {"value": round(e_units / (e_ms * 1e-3), 3), "unit": workload.unit,
           "h2d_bytes_per_step": int(workload.h2d), "d2h_bytes_per_step": int(workload.d2h)}

    lif = None
    if workload.name == "vgg16" and not args.no_lif:
        lif = lif_kernel_object(dist, rank, world, local, peaks)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            threads = os.cpu_count() or 1
            torch.set_num_threads(threads)
            v, s, med = time_cpu(workload, threads)
            sample = {k: v_ for k, v_ in s.items() if isinstance(v_, (int, float, str))}
            cpu = {"value": round(v, 3), "unit": workload.unit, "cores": threads,
                   "kind": "port", "sample": json.dumps(sample) + f" median {med:.3f}s"}
        line = {"metric": workload.metric, "value": round(value, 3), "unit": workload.unit,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": workload.dtype,
                "data": "synthetic", "config": workload.config(),
                "roofline": roof,
                "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": int(workload.launches_per_step * args.steps),
                "clocks": clocks}
        if lif is not None:
            line["lif_kernel"] = lif
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="vgg16",
                    choices=["vgg16", "lif", "conv", "first", "attention", "bgemm", "resnet18"])
    ap.add_argument("--lif-shape", default="32,134217728", help="lif workload: T,N")
    ap.add_argument("--gemm-shape", default="16384,8192,8192", help="bgemm workload: M,K,N")
    ap.add_argument("--layer", default="512,512,56",
                    help="conv workload: Cin,Cout,H (3x3 + pool) or Cin,Cout,H,k,stride (ResNet "
                         "conv, k in {1, 3}, stride in {1, 2}, no pool)")
    ap.add_argument("--batch", type=int, default=64, help="conv / resnet18 workload batch")
    ap.add_argument("--choice", default=None,
                    help="conv workload: fixed 'variant,block_n' instead of timing the candidates")
    ap.add_argument("--save-choices", default=None, help="vgg16: write the tuned kernel table")
    ap.add_argument("--load-choices", default=None,
                    help="vgg16: use a tuned kernel table instead of timing (e.g. under ncu)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-lif", action="store_true",
                    help="vgg16: skip the LIF-kernel bandwidth object (lif_kernel) of the line")
    ap.add_argument("--packed", default="none", choices=["none", "in", "out", "both"],
                    help="conv workload: packed spikes in / out (snnb_conv3x3_lif_packed)")
    ap.add_argument("--eager", action="store_true",
                    help="vgg16: launch the forward kernel by kernel instead of replaying CUDA "
                         "graphs (for kernel-replaying profilers; the same work)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.workload == "conv":
        lay = [int(v) for v in args.layer.split(",")]
        cin, cout, hh = lay[:3]
        k, stride = (lay[3], lay[4]) if len(lay) == 5 else (3, 1)
        fixed = tuple(int(v) for v in args.choice.split(",")) if args.choice else None
        if fixed and len(fixed) == 2:
            fixed = fixed + (1,)
        wl = ConvLayerWorkload(cin, cout, hh, B=args.batch, fixed=fixed, packed=args.packed,
                               k=k, stride=stride)
    elif args.workload == "first":
        wl = FirstLayerWorkload(B=args.batch,
                                fixed=int(args.choice) if args.choice is not None else None)
    else:
        if args.workload == "lif":
            lt, ln = (int(v) for v in args.lif_shape.split(","))
            wl = LifWorkload(T=lt, N=ln)
        elif args.workload == "bgemm":
            gm, gk, gn = (int(v) for v in args.gemm_shape.split(","))
            wl = BgemmWorkload(gm, gk, gn)
        else:
            wl = ResNetWorkload(B=args.batch) if args.workload == "resnet18" else \
                {"vgg16": VggWorkload, "attention": AttnWorkload}[args.workload]()
        if args.workload == "vgg16":
            wl.load_choices, wl.save_choices = args.load_choices, args.save_choices
            wl.eager = args.eager
    wl.world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
