"""VGG-SNN on the fused sm_100a kernels (reference snn_compiler/zoo/vgg.py).

``VGGSNN`` keeps the reference's module structure (Conv2d -> BatchNorm2d -> LIF per
cfg entry, 2x2 pool at 'P', classifier Linear+LIF, Linear+LIF, Linear; vgg.py:43-115)
so reference weights load unchanged; ``fc_in`` lets a 32x32 input feed the
classifier (the reference hard-codes 224-pixel inputs at vgg.py:74).  Its forward
runs ``SpikingVGG``, the inference engine:

  layer 1   snnb_first_conv_lif   float32 conv of the real-valued image + bias + LIF
  layers 2+ snnb_conv3x3_lif      tcgen05 conv + folded-BN bias + LIF (+ max-pool)
  fc1, fc2  snnb_linear_lif       tcgen05 GEMM + bias + LIF
  fc3       snnb_linear_mean / snnb_linear_out   logits (averaged over T, or per step)

Activations stay on the device as bf16 channels-last spikes [T, B, H, W, C]; BN is
folded once at construction (fold_conv_bn, fused.py:585-599); a whole forward can be
captured into CUDA graphs (``capture``) so one replay issues every launch.  Only
max-pooling is fused (pool='max'); spikes are {0,1}, so max-pool is an OR.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..kernels import conv as KC
from ..kernels.fused import fold_conv_bn
from ..nn.modules import LIFNode, IFNode

VGG16_CFG = [64, 64, "P", 128, 128, "P", 256, 256, 256, "P",
             512, 512, 512, "P", 512, 512, 512, "P"]
VGG11_CFG = [64, "P", 128, "P", 256, 256, "P", 512, 512, "P", 512, 512, "P"]
VGG13_CFG = [64, 64, "P", 128, 128, "P", 256, 256, "P", 512, 512, "P", 512, 512, "P"]
VGG19_CFG = [64, 64, "P", 128, 128, "P", 256, 256, 256, 256, "P",
             512, 512, 512, 512, "P", 512, 512, 512, 512, "P"]


def random_vgg_params(seed: int = 1, *, cfg=VGG16_CFG, num_classes: int = 10, in_ch: int = 3,
                      fc_hidden: int = 4096, fc_in: int | None = None):
    """Seeded synthetic weights with the benchmark's draws, generated on the host:
    conv / linear weights Kaiming-normal (fan_in, gain sqrt 2), biases U(+-1/sqrt(fan_in)),
    BN gamma U(0.8, 1.2), beta N(0, 0.1), running mean N(0, 0.1), var U(0.5, 1.5), eps 1e-5."""
    g = torch.Generator().manual_seed(int(seed))
    convs = []
    ch = in_ch
    for v in cfg:
        if v == "P":
            convs[-1]["pool"] = True
            continue
        fan_in = ch * 9
        convs.append({
            "w": torch.randn(v, ch, 3, 3, generator=g) * math.sqrt(2.0 / fan_in),
            "b": (torch.rand(v, generator=g) * 2 - 1) / math.sqrt(fan_in),
            "gamma": torch.rand(v, generator=g) * 0.4 + 0.8,
            "beta": torch.randn(v, generator=g) * 0.1,
            "mean": torch.randn(v, generator=g) * 0.1,
            "var": torch.rand(v, generator=g) + 0.5,
            "eps": 1e-5, "pool": False,
        })
        ch = v
    fc_in = ch if fc_in is None else fc_in
    fcs = []
    for fin, fout in ((fc_in, fc_hidden), (fc_hidden, fc_hidden), (fc_hidden, num_classes)):
        fcs.append({"w": torch.randn(fout, fin, generator=g) * math.sqrt(2.0 / fin),
                    "b": (torch.rand(fout, generator=g) * 2 - 1) / math.sqrt(fin)})
    return {"convs": convs, "fcs": fcs, "num_classes": num_classes}


class SpikingVGG:
    """Inference engine: folded bf16 weights resident on one device, fused launches."""

    def __init__(self, P, *, T: int = 4, tau: float = 2.0, decay_input: bool = True,
                 v_threshold: float = 1.0, v_reset: float = 0.0, soft_reset: bool = False,
                 neuron: str = "lif", device="cuda", autotune: bool = True,
                 dense_small: bool = True, check_status: bool = False, chains: int = 1):
        self.T = T
        # chains > 1: captured forwards run the batch as `chains` sub-batches on concurrent
        # streams, so that one chain's layer tails and launch gaps overlap the other's layers.
        # At VGG16 B = 64 per GPU two chains of 32 measured 0.3125 ms per step against 0.2688
        # for one chain of 64 (each B = 32 kernel is too much less efficient), so the
        # default is one chain.
        self.chains = max(1, int(chains))
        self.autotune = autotune
        # unpooled 3x3 layers on images of at most 2x2 pixels run as dense GEMMs
        self.dense_small = dense_small
        self._dense_w = {}
        self.choice = {}          # (layer, B, H, W) -> (variant, block_n) picked by timing
        self.lif = dict(neuron=neuron, tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                        v_threshold=v_threshold, v_reset=v_reset)
        dev = torch.device(device)
        self.device = dev
        self.layers = []
        for i, c in enumerate(P["convs"]):
            w, b = fold_conv_bn(c["w"].float(), None if c.get("b") is None else c["b"].float(),
                                c["gamma"].float(), c["beta"].float(), c["mean"].float(),
                                c["var"].float(), c["eps"])
            if i == 0:
                wd = w.contiguous().to(dev)                       # f32 [Cout, Cin, 3, 3]
            else:
                wd = KC.weight_khwc(w).to(dev)                    # bf16 [Cout, 3, 3, Cin]
            self.layers.append({"w": wd, "b": b.float().contiguous().to(dev),
                                "pool": bool(c["pool"]), "cout": w.shape[0],
                                "cin": w.shape[1]})
        self.fcs = [{"w": f["w"].to(torch.bfloat16).contiguous().to(dev),
                     "b": f["b"].float().contiguous().to(dev)} for f in P["fcs"]]
        self.num_classes = P["fcs"][-1]["w"].shape[0]
        self._bufs = {}
        self._workspace = {}          # chain -> split-K workspace
        self.graphs = None
        self._graph_cache = {}
        self._fwd_pool = None
        self._side_streams = []
        self.check_status = bool(check_status)

    # ---- per-layer launch plan -----------------------------------------------------------
    def plan(self, img: torch.Tensor, *, per_step_logits: bool = False,
             out: torch.Tensor | None = None, chain: int = 0):
        """List of (name, flops, callable) for one forward over img [Ti, B, 3, H, W] f32.
        Buffers are allocated once per (B, H, W, chain) and reused; ``out`` (optional)
        receives the logits instead of the engine's own buffer.  Plans of different chains
        share no buffer or workspace, so they may run concurrently."""
        Ti, B, Cin, H, W = img.shape
        T = self.T
        key = (B, H, W, per_step_logits) if chain == 0 else (B, H, W, per_step_logits, chain)
        if key not in self._bufs:
            bufs = []
            h, w = H, W
            for L in self.layers:
                ho, wo = (h // 2, w // 2) if L["pool"] else (h, w)
                bufs.append(torch.empty(T, B, ho, wo, L["cout"], device=self.device,
                                        dtype=torch.bfloat16))
                h, w = ho, wo
            feat = h * w * self.layers[-1]["cout"]
            assert feat == self.fcs[0]["w"].shape[1], (feat, tuple(self.fcs[0]["w"].shape))
            fbufs = [torch.empty(T, B, f["w"].shape[0], device=self.device, dtype=torch.bfloat16)
                     for f in self.fcs[:-1]]
            logits = torch.empty((T, B, self.num_classes) if per_step_logits
                                 else (B, self.num_classes), device=self.device,
                                 dtype=torch.float32)
            self._bufs[key] = (bufs, fbufs, logits)
        bufs, fbufs, own_out = self._bufs[key]
        if out is None:
            out = own_out
        else:
            assert out.shape == own_out.shape and out.dtype == own_out.dtype and out.is_contiguous()
        steps = []
        h, w = H, W
        x_prev = None
        for i, L in enumerate(self.layers):
            flops = 2 * T * B * h * w * L["cout"] * L["cin"] * 9
            if i == 0:
                fn = self._first_layer(img, L, bufs[0])
            elif h <= 2 and w <= 2 and self.dense_small and (not L["pool"] or h == w == 2):
                # the whole image is every output pixel's window: a dense GEMM over the
                # image's pixels x channels (no zero-padding taps), K1's linear form
                wd, bd = self._dense(i, h, w)
                K, N = h * w * L["cin"], h * w * L["cout"]
                fn = self._tuned(("dconv", i, B, h, w), N, K // 64,
                                 lambda v, bn, sp, L=L, wd=wd, bd=bd, x=x_prev, o=bufs[i],
                                 NN=N:
                                 KC.conv3x3_lif_dense(x, wd, bd, pool=L["pool"], out=o,
                                                      variant=v, block_n=bn, splits=sp,
                                                      workspace=self._ws(T, B, 1, 1, NN,
                                                                         1 if v == 6 else sp,
                                                                         chain, v),
                                                      **self.lif),
                                 dense_pool=L["pool"], linear_t=True)
            else:
                fn = self._tuned(("conv", i, B, h, w), L["cout"], 9 * L["cin"] // 64,
                                 lambda v, bn, sp, L=L, x=x_prev, o=bufs[i], hh=h, ww=w:
                                 KC.conv3x3_lif(x, L["w"], L["b"], pool=L["pool"], out=o,
                                                variant=v, block_n=bn, splits=sp,
                                                workspace=self._ws(T, B, hh, ww, L["cout"],
                                                                   1 if v == 6 else sp, chain),
                                                **self.lif),
                                 band=KC.band_block_ns(w, L["cin"], L["cout"]),
                                 band_xs=KC.band_xs_block_ns(w, L["cin"], L["cout"]))
            steps.append((f"conv{i + 1}_{L['cin']}x{L['cout']}@{h}", flops, fn))
            x_prev = bufs[i]
            if L["pool"]:
                h, w = h // 2, w // 2
        hcur = x_prev.view(T, B, -1)
        for j, f in enumerate(self.fcs[:-1]):
            K, N = f["w"].shape[1], f["w"].shape[0]
            steps.append((f"fc{j + 1}_{K}x{N}", 2 * T * B * K * N,
                          self._tuned(("fc", j, B, 1, 1), N, K // 64,
                                      lambda v, bn, sp, f=f, x=hcur, o=fbufs[j], NN=N:
                                      KC.linear_lif(x, f["w"], f["b"], out=o, variant=v,
                                                    block_n=bn, splits=sp,
                                                    workspace=self._ws(T, B, 1, 1, NN,
                                                                      1 if v == 6 else sp,
                                                                      chain, v),
                                                    **self.lif),
                                      linear_t=True)))
            hcur = fbufs[j]
        f = self.fcs[-1]
        K, N = f["w"].shape[1], f["w"].shape[0]
        head = KC.linear_out if per_step_logits else KC.linear_mean
        steps.append((f"fc{len(self.fcs)}_{K}x{N}", 2 * T * B * K * N,
                      (lambda f=f, x=hcur: head(x, f["w"], f["b"], out=out))))
        return steps, out

    def _first_layer(self, img, L, o):
        """Launcher of the image layer: the float32 CUDA-core kernel, or (direct encoding,
        Cin <= 4, no pooling) the tensor-core kernel with split operands -- whichever the
        autotuner times faster for this input shape."""
        T = self.T
        cuda_core = (lambda: KC.first_conv_lif(img, L["w"], L["b"], T=T, pool=L["pool"], out=o,
                                               **self.lif))
        if not (img.shape[0] == 1 and L["cin"] <= 4 and L["cout"] in (32, 64, 128)
                and not L["pool"]):
            return cuda_core
        if "wsplit" not in L:
            L["wsplit"] = KC.first_conv_split_weight(L["w"])
        tensor_core = (lambda: KC.first_conv_lif_tc(img, L["wsplit"], L["b"], T=T, out=o,
                                                    **self.lif))
        key = ("first", 0) + tuple(img.shape)

        def run():
            if key not in self.choice:
                if self.autotune:
                    ms = [min(KC.time_graph(f) for _ in range(2)) for f in (cuda_core, tensor_core)]
                    self.choice[key] = (1 if ms[1] < ms[0] else 0, 0, 1)
                else:
                    self.choice[key] = (1, 0, 1)
            return (tensor_core if self.choice[key][0] == 1 else cuda_core)()
        return run

    def _dense(self, i, h, w):
        """Dense-GEMM weights of conv layer i on h x w images (dense_conv_weight), cached."""
        key = (i, h, w)
        if key not in self._dense_w:
            L = self.layers[i]
            self._dense_w[key] = (KC.dense_conv_weight(L["w"], h, w, pool=L["pool"]),
                                  KC.dense_conv_bias(L["b"], h, w, pool=L["pool"]))
        return self._dense_w[key]

    def _ws(self, T, B, H, W, Cout, splits, chain=0, variant=0):
        """Split-K workspace, one buffer per chain shared by the chain's layers (they run one
        after another on one stream), grown to the largest request (variant 8: the
        transposed linear's partial sums)."""
        need = KC.linear_t_workspace_bytes(T, B, Cout, splits) if variant == 8 else \
            KC.split_workspace_bytes(T, B, H, W, Cout, splits)
        if need == 0:
            return None
        ws = self._workspace.get(chain)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.empty(need // 4, device=self.device, dtype=torch.float32)
            self._workspace[chain] = ws
        return ws

    def _tuned(self, key, cout, kslabs, launch, band=(), dense_pool=False, band_xs=(),
               linear_t=False):
        """A zero-argument launcher for one tensor-core layer.  With autotune on, the first
        call times every (variant, block_n, splits) the layer admits and keeps the fastest."""
        def run():
            if key not in self.choice:
                self.choice[key] = KC.pick_fastest(launch, cout, self.T, kslabs, band=band,
                                                   dense_pool=dense_pool, band_xs=band_xs,
                                                   linear_t=linear_t) \
                    if self.autotune else (0, 0, 1)
            return launch(*self.choice[key])
        return run

    def kernel_launches(self, B: int) -> int:
        """Kernel launches of one captured forward at batch B after its layers were tuned: per
        chain one per layer, plus the split-K finish (sum + bias + neuron) of every two-launch
        split-K layer (the cluster split-K form, variant 6, finishes in its own launch)."""
        nc = self._chain_count(B, 1)
        bs = B // nc
        n = len(self.layers) + len(self.fcs)
        return nc * (n + sum(1 for k, c in self.choice.items()
                             if k[0] != "first" and k[2] == bs and c[2] > 1 and c[0] != 6))

    # ---- concurrent chains ------------------------------------------------------------------
    def _chain_count(self, B: int, Ti: int = 1, per_step_logits: bool = False) -> int:
        """Chains a captured forward of batch B uses: self.chains when B splits evenly into
        sub-batches of at least 8 images (direct encoding, T-averaged logits), else 1."""
        n = self.chains
        if n <= 1 or per_step_logits or Ti != 1 or B % n or B // n < 8:
            return 1
        return n

    def chain_batch(self, B: int) -> int:
        """Sub-batch of each chain of a captured forward of batch B (its tuned kernels)."""
        return B // self._chain_count(B, 1)

    def _chain_plans(self, img, out=None, per_step_logits=False):
        """[(steps, img part, out part)] per chain: chain c takes samples [c*b, (c+1)*b) of
        img [1, B, ...] and writes their logits to rows [c*b, (c+1)*b) of out [B, classes]."""
        B = img.shape[1]
        nc = self._chain_count(B, img.shape[0], per_step_logits)
        if nc == 1:
            steps, o = self.plan(img, per_step_logits=per_step_logits, out=out)
            return [(steps, img, o)], o
        if out is None:
            key = ("chain_out", B)
            if key not in self._bufs:
                self._bufs[key] = torch.empty(B, self.num_classes, device=self.device,
                                              dtype=torch.float32)
            out = self._bufs[key]
        bs = B // nc
        parts = []
        for c in range(nc):
            im = img.narrow(1, c * bs, bs)
            oc = out.narrow(0, c * bs, bs)
            steps, _ = self.plan(im, out=oc, chain=c)
            parts.append((steps, im, oc))
        return parts, out

    def layer_outputs(self, B: int, H: int = 32, W: int = 32):
        """Each conv layer's spikes [T, B, Ho, Wo, C] of the last captured forward of batch B
        (the chains' sub-batch buffers joined along the batch), for checks and debugging."""
        nc = self._chain_count(B, 1)
        bs = B // nc
        per = [self._bufs[(bs, H, W, False) if c == 0 else (bs, H, W, False, c)][0]
               for c in range(nc)]
        return [torch.cat([p[i] for p in per], dim=1) for i in range(len(per[0]))]

    def _record_chains(self, parts, mark=None):
        """Issue every chain's launches inside a stream capture: chain 0 on the current stream,
        chain c > 0 on side stream c, forked from and joined back to the current stream;
        timing events around chain 0's launch `mark`."""
        s0 = torch.cuda.current_stream()
        while len(self._side_streams) < len(parts) - 1:
            self._side_streams.append(torch.cuda.Stream(device=self.device))
        side = self._side_streams[:len(parts) - 1]
        for st in side:
            st.wait_stream(s0)
        for c, (steps, _, _) in enumerate(parts):
            stream = s0 if c == 0 else side[c - 1]
            with torch.cuda.stream(stream):
                for k, (_, _, fn) in enumerate(steps):
                    if c == 0 and k == mark:
                        self.mark_events[0].record()
                    fn()
                    if c == 0 and k == mark:
                        self.mark_events[1].record()
        for st in side:
            s0.wait_stream(st)

    def forward(self, img: torch.Tensor, *, per_step_logits: bool = False,
                out: torch.Tensor | None = None, graph: bool = False,
                check: bool | None = None, mid_event: torch.cuda.Event | None = None,
                mid_at: int = 4) -> torch.Tensor:
        """img [B, 3, H, W] (direct encoding: the same image at every step) or
        [Ti, B, 3, H, W] f32 -> logits averaged over T [B, classes] (or [T, B, classes]).

        out   : optional float32 buffer of the logits' shape that receives them.
        graph : replay the forward as a CUDA graph (captured on the first call for this
                input shape and ``out``; each call's input is copied into the graph's own
                input buffer, ``graph_input``) -- one graph launch instead of ~16 launches.
        check : read the device status word after the forward (a stream synchronisation)
                and raise SnnbError if a kernel's bounded wait gave up; defaults to the
                engine's ``check_status``.
        mid_event : (graph=True, one chain) the forward is captured as two graphs split
                before launch ``mid_at`` and this event is recorded between their replays,
                so that other work (a collective) can start once the first ``mid_at``
                launches -- VGG16's full-grid image and band layers -- are done and run beside
                the later layers, whose grids leave SMs free."""
        if img.ndim == 4:
            img = img.unsqueeze(0)
        img = img.to(self.device, torch.float32)
        if not img.is_contiguous():
            img = img.contiguous()
        if graph:
            split = mid_at if mid_event is not None else None
            key = (tuple(img.shape), per_step_logits, None if out is None else out.data_ptr(),
                   split)
            ent = self._graph_cache.get(key)
            if ent is None:
                static_in = torch.empty_like(img)          # the engine's own input buffer
                static_in.copy_(img)
                graphs, o = self._capture_graphs(static_in, per_step_logits, out, split)
                ent = (static_in, graphs, o)
                self._graph_cache[key] = ent
            static_in, graphs, o = ent
            if img.data_ptr() != static_in.data_ptr():
                static_in.copy_(img, non_blocking=True)
            for gi, g in enumerate(graphs):
                if gi == 1 and mid_event is not None:
                    mid_event.record()
                g.replay()
            if len(graphs) == 1 and mid_event is not None:
                mid_event.record()
        else:
            steps, o = self.plan(img, per_step_logits=per_step_logits, out=out)
            for _, _, fn in steps:
                fn()
        if self.check_status if check is None else check:
            KC.raise_on_device_status("SpikingVGG.forward")
        return o

    def graph_input(self, shape, *, per_step_logits: bool = False, out=None,
                    mid_at: int | None = None):
        """The input buffer of the graph forward(graph=True) replays for this input shape
        and ``out`` (and ``mid_at`` when it was called with a mid_event) -- a caller that
        writes its input there saves the copy -- or None."""
        key = (tuple(shape), per_step_logits, None if out is None else out.data_ptr(), mid_at)
        ent = self._graph_cache.get(key)
        return None if ent is None else ent[0]

    def _capture_graphs(self, img, per_step_logits, out, split=None):
        parts, o = self._chain_plans(img, out, per_step_logits)
        for steps, _, _ in parts:         # warm up (tunes the layers, sets kernel attributes)
            for _, _, fn in steps:
                fn()
        torch.cuda.synchronize()
        if split is not None and len(parts) == 1 and 0 < split < len(parts[0][0]):
            steps = parts[0][0]
            graphs = []
            for grp in (steps[:split], steps[split:]):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=self._fwd_pool):
                    for _, _, fn in grp:
                        fn()
                graphs.append(g)
            torch.cuda.synchronize()
            return graphs, o
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._fwd_pool):
            self._record_chains(parts)
        torch.cuda.synchronize()
        return [g], o

    __call__ = forward

    def profile_layers(self, img: torch.Tensor, reps: int = 10):
        """[(name, flops, device ms per launch)] for the launches of chain 0 of a captured
        forward (its sub-batch), each launch timed alone from a CUDA graph of `reps`
        repetitions (no host overhead in the figure)."""
        if img.ndim == 4:
            img = img.unsqueeze(0)
        parts, _ = self._chain_plans(img)
        steps = parts[0][0]                 # chain 0's launches (its sub-batch)
        for _, _, fn in steps:
            fn()
        return [(name, flops, KC.time_graph(fn, reps)) for name, flops, fn in steps]

    def layer_times_in_step(self, img: torch.Tensor, reps: int = 10, flush_bytes: int = 256 << 20):
        """[(name, device ms)] of every launch inside one captured forward (one chain), with
        a pair of timing events around each launch, median over `reps` replays each after
        writing `flush_bytes` to flush L2 -- the layers as the step runs them (an event
        between two launches also stops the next one's programmatic early start, so the sum
        is a little above the step)."""
        if img.ndim == 4:
            img = img.unsqueeze(0)
        steps, _ = self.plan(img)
        for _, _, fn in steps:
            fn()
        ev = [(torch.cuda.Event(enable_timing=True, external=True),
               torch.cuda.Event(enable_timing=True, external=True)) for _ in steps]
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for (a, b), (_, _, fn) in zip(ev, steps):
                a.record()
                fn()
                b.record()
        flush = torch.empty(flush_bytes, dtype=torch.uint8, device=self.device)
        samples = []
        for _ in range(reps):
            flush.fill_(1)
            g.replay()
            torch.cuda.synchronize()
            samples.append([a.elapsed_time(b) for a, b in ev])
        del g, flush
        out = []
        for i, (name, _, _) in enumerate(steps):
            col = sorted(s[i] for s in samples)
            out.append((name, col[len(col) // 2]))
        return out

    def flops_per_image(self, H: int = 32, W: int = 32) -> int:
        """Dense algorithmic FLOPs of one image (every conv at every step)."""
        img = torch.empty(1, 1, 3, H, W)
        total = 0
        h, w = H, W
        for L in self.layers:
            total += 2 * self.T * h * w * L["cout"] * L["cin"] * 9
            if L["pool"]:
                h, w = h // 2, w // 2
        for f in self.fcs:
            total += 2 * self.T * f["w"].shape[0] * f["w"].shape[1]
        del img
        return total

    # ---- CUDA graphs ----------------------------------------------------------------------
    def capture(self, img: torch.Tensor, *, split_at: int | None = None,
                mark: int | None = None, out: torch.Tensor | None = None):
        """Capture the forward over the static input buffer ``img`` into CUDA graphs.
        With split_at=i the launches are split into three graphs [0, i), [i], (i, end) so
        that the i-th launch can be timed alone between replays (one chain).  Otherwise the
        forward is one graph of ``chains`` concurrent sub-batch chains (when the batch
        splits evenly); with mark=i it holds a pair of timing events around launch i of
        chain 0 (``self.mark_events``; read them after a replay has completed).  Returns the
        output."""
        if img.ndim == 4:
            img = img.unsqueeze(0)
        self.graph_pool = torch.cuda.graph_pool_handle()
        self.mark_events = None
        if mark is not None:
            self.mark_events = (torch.cuda.Event(enable_timing=True, external=True),
                                torch.cuda.Event(enable_timing=True, external=True))
        if split_at is None and self._chain_count(img.shape[1], img.shape[0]) > 1:
            # concurrent chains in one graph (mark: a launch of chain 0)
            parts, out = self._chain_plans(img, out)
            for steps, _, _ in parts:
                for _, _, fn in steps:
                    fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.graph_pool):
                self._record_chains(parts, mark=mark)
            self.graphs = [g]
            torch.cuda.synchronize()
            self.graph_out = out
            self._graph_parts = parts          # keeps the sub-batch views alive
            return out
        steps, out = self.plan(img, out=out)
        for _, _, fn in steps:            # warm up (sets kernel attributes, caches maps)
            fn()
        torch.cuda.synchronize()
        groups = [list(range(len(steps)))] if split_at is None else \
            [list(range(split_at)), [split_at], list(range(split_at + 1, len(steps)))]
        self.graphs = []
        for grp in groups:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.graph_pool):
                for k in grp:
                    if k == mark:
                        self.mark_events[0].record()
                    steps[k][2]()
                    if k == mark:
                        self.mark_events[1].record()
            self.graphs.append(g)
        torch.cuda.synchronize()
        self.graph_out = out
        return out

    def replay(self, between=None):
        """Replay the captured graphs; ``between(i)`` runs before graph i (events)."""
        for i, g in enumerate(self.graphs):
            if between is not None:
                between(i)
            g.replay()
        if between is not None:
            between(len(self.graphs))
        return self.graph_out


class VGGSNN(nn.Module):
    """Reference-structured VGG-SNN (snn_compiler/zoo/vgg.py:43-115) whose forward runs
    the fused engine.  forward(x_seq [T, B, 3, H, W]) -> logits [T, B, classes]."""

    def __init__(self, cfg, num_classes=1000, *, in_ch=3, fc_hidden=4096, with_bn=True,
                 neuron="lif", tau=2.0, decay_input=True, soft_reset=False, v_threshold=1.0,
                 v_reset=0.0, layout="NCHW", pool="max", fc_in=None, input_size=224):
        super().__init__()
        if pool != "max":
            raise NotImplementedError("the fused kernels implement pool='max' (OR of spikes)")
        if not with_bn:
            raise NotImplementedError("VGGSNN here expects BN layers (folded at fuse time)")
        feats = []
        ch = in_ch
        for v in cfg:
            if v == "P":
                feats.append(nn.MaxPool2d(2, 2))
            else:
                feats.append(nn.Conv2d(ch, v, 3, padding=1, bias=True))
                feats.append(nn.BatchNorm2d(v))
                feats.append(LIFNode(tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                                     v_threshold=v_threshold, v_reset=v_reset, layout=layout)
                             if neuron == "lif" else
                             IFNode(soft_reset=soft_reset, v_threshold=v_threshold,
                                    v_reset=v_reset, layout=layout))
                ch = v
        self.features = nn.Sequential(*feats)
        n_pool = sum(1 for x in cfg if x == "P")
        self.fc_in_dim = fc_in if fc_in is not None else ch * (input_size // 2 ** n_pool) ** 2
        self.classifier = nn.Sequential(
            nn.Linear(self.fc_in_dim, fc_hidden), nn.Identity(),
            nn.Linear(fc_hidden, fc_hidden), nn.Identity(),
            nn.Linear(fc_hidden, num_classes))
        self.cfg = list(cfg)
        self.neuron_kw = dict(tau=tau, decay_input=decay_input, soft_reset=soft_reset,
                              v_threshold=v_threshold, v_reset=v_reset, neuron=neuron)
        self._engine = None

    def params_dict(self):
        convs, it = [], iter(self.features)
        for m in self.features:
            if isinstance(m, nn.Conv2d):
                convs.append({"w": m.weight.detach(), "b": None if m.bias is None else m.bias.detach(),
                              "pool": False})
            elif isinstance(m, nn.BatchNorm2d):
                convs[-1].update(gamma=m.weight.detach(), beta=m.bias.detach(),
                                 mean=m.running_mean.detach(), var=m.running_var.detach(),
                                 eps=m.eps)
            elif isinstance(m, nn.MaxPool2d):
                convs[-1]["pool"] = True
        del it
        lins = [m for m in self.classifier if isinstance(m, nn.Linear)]
        fcs = [{"w": l.weight.detach(), "b": l.bias.detach()} for l in lins]
        return {"convs": convs, "fcs": fcs}

    def fuse(self, T: int = 4):
        dev = next(self.parameters()).device
        self._engine = SpikingVGG(self.params_dict(), T=T, device=dev, **self.neuron_kw)
        return self._engine

    def forward(self, x_seq):
        T = x_seq.shape[0]
        if self._engine is None or self._engine.T != T:
            self.fuse(T)
        return self._engine.forward(x_seq.float().contiguous(), per_step_logits=True)


def _build(cfg, *, fused=True, init_bn=True, **kw):
    m = VGGSNN(cfg, **kw)
    if init_bn:
        g = torch.Generator().manual_seed(0)
        for mod in m.modules():
            if isinstance(mod, nn.BatchNorm2d):
                with torch.no_grad():
                    mod.running_mean.copy_(torch.randn(mod.running_mean.shape, generator=g) * 0.1)
                    mod.running_var.copy_(torch.rand(mod.running_var.shape, generator=g) + 0.5)
                    mod.weight.copy_(torch.rand(mod.weight.shape, generator=g) + 0.5)
                    mod.bias.copy_(torch.randn(mod.bias.shape, generator=g) * 0.1)
    return m.eval()


def vgg11_snn(**kw): return _build(VGG11_CFG, **kw)
def vgg13_snn(**kw): return _build(VGG13_CFG, **kw)
def vgg16_snn(**kw): return _build(VGG16_CFG, **kw)
def vgg19_snn(**kw): return _build(VGG19_CFG, **kw)
