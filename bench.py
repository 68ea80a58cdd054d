"""Benchmark: train views/s (fwd + bwd + L1/SSIM) of the BlitzGS splatting hot path.

Contract (one JSON line from rank 0):
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: BASELINE config 3 ("city"): 8M Gaussians from a clustered mixture in
a 1000x1000x40 box, 1152x864 aerial cameras (pitch 45-90 deg), seeded
synthetic data standing in for Mill-19 / UrbanScene3D (not available here).
A step is one training iteration over a batch of ``bsz`` views per GPU:
activations -> preprocess -> binning -> blend -> L1+SSIM -> backward to the
raw Gaussian parameters (optimizer and densification excluded, as in the
reference's throughput log).  Inputs (8M x 236 B of parameters) are larger
than L2, and consecutive steps use different cameras.

--impl reference times the reference's own rasterizer (BlitzGS
diff_gaussian_rasterization_f/_r CUDA modules built unmodified from the
reference sources into oracle/_ref by oracle/build_ref.py) through its stock
Python operator API and loss helpers on the same workload; when that build is
absent it times the CPU oracle port on a bounded sample instead.
"""
import argparse
import gc
import json
import math
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train views/sec (fwd+bwd+L1/SSIM) at 8M Gaussians, 1/2/4/8 B200; ms/iter"
UNIT = "views/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


_POLLER = r"""
import sys, time
import pynvml as nv
nv.nvmlInit()
g = sys.argv[1]
h = nv.nvmlDeviceGetHandleByIndex(int(g)) if g.isdigit() else nv.nvmlDeviceGetHandleByUUID(g)
mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
rs = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
while True:
    print(time.monotonic_ns(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx, int(rs(h)), flush=True)
    time.sleep(0.05)
"""


class ClockSampler:
    """SM clock and throttle reasons during the timed regions.

    A separate process polls NVML (read-only queries) every 50 ms and prints
    time-stamped samples; samples between pairs of mark() calls count, and a
    region shorter than the period takes the nearest sample.  Falls back to
    nvidia-smi at 200 ms when the NVML bindings are missing.  A separate
    process at a modest rate keeps the queries from competing with this
    process's kernel launches (for the GIL or the driver)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if gpu_index < len(ids):
                gpu_index = ids[gpu_index]
        self.gpu = gpu_index
        self.proc = None
        self.samples = []  # (t_ns, sm_mhz, max_mhz, reason bits)
        self.windows = []
        self.thread = None
        self.source = None

    def mark(self):
        t = time.monotonic_ns()
        if self.windows and len(self.windows[-1]) == 1:
            self.windows[-1].append(t)
        else:
            self.windows.append([t])

    def start(self):
        try:
            import pynvml  # noqa: F401  (the poller needs it)
            self.proc = subprocess.Popen([sys.executable, "-c", _POLLER, str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.source = "nvml"
            self.thread = threading.Thread(target=self._read_nvml, daemon=True)
        except Exception:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except (FileNotFoundError, OSError):
                self.proc = None
                return
            self.source = "nvidia-smi"
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()
        # wait for the first sample, so the poller is up before any timed region
        t0 = time.time()
        while not self.samples and time.time() - t0 < 20 and self.proc.poll() is None:
            time.sleep(0.05)

    def _read_nvml(self):
        for line in self.proc.stdout:
            parts = line.split()
            if len(parts) == 4:
                self.samples.append((int(parts[0]), float(parts[1]), float(parts[2]), int(parts[3])))

    def _read_smi(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                bits = 0
                for n, v in zip(names, parts[5:9]):
                    if v.lower() in ("active", "0x1", "1"):
                        bits |= self.REASONS[n]
                self.samples.append((time.monotonic_ns(), float(parts[1]), float(parts[2]), bits))
            except ValueError:
                continue

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        inside = []
        for w in self.windows:
            if len(w) != 2 or not self.samples:
                continue
            ins = [s for s in self.samples if w[0] <= s[0] <= w[1]]
            # a region shorter than the sampling period takes its nearest sample
            inside += ins or [min(self.samples, key=lambda s: abs(s[0] - (w[0] + w[1]) // 2))]
        if not inside:
            return None
        sms = sorted(s[1] for s in inside)
        bits = 0
        for s in inside:
            bits |= s[3]
        reasons = sorted(n for n, b in self.REASONS.items() if bits & b)
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": max(s[2] for s in inside), "reasons": reasons,
                "samples": len(sms), "source": self.source}


def dist_setup(n_gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------

def load_scene(args):
    """The synthetic scene of args.config.  With --layout zorder (default) the
    Gaussians are stored in z-order of their means, the order the N-GPU
    sharding gives each rank, so 1-GPU and N-GPU runs (and the reference arm)
    see the same memory layout; --layout given keeps the generator's order."""
    from blitzgs_b200 import scene as S, distributed as D
    kw = {"P": args.gaussians} if getattr(args, "gaussians", None) else {}
    sc = S.CONFIGS[args.config](seed=0, **kw)
    if getattr(args, "layout", "zorder") == "zorder":
        order = D.zorder_shards(sc.xyz, 1)[0]
        for name in ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"):
            setattr(sc, name, getattr(sc, name)[order].contiguous())
    return sc


def build_workload(args, device, rank=0, ws=1):
    from blitzgs_b200 import scene as S
    sc = load_scene(args)
    n_cams = len(sc.cameras)
    H, W = sc.cameras[0].image_height, sc.cameras[0].image_width
    gts = [S.target_image(k, H, W) for k in range(n_cams)]
    return sc, gts


class GTPrefetch:
    """Ground-truth upload from pinned host memory one step ahead, on a copy
    stream into two device buffer sets: step i+1's copy overlaps step i's
    compute.  ``host[i]`` = the pinned uint8 images of step i's views.
    Every copy is issued inside the timed region (the first at its start)."""

    def __init__(self, dev, host, H, W, bsz):
        self.dev, self.host = dev, host
        self.stream = torch.cuda.Stream(dev)
        self.bufs = [[torch.empty((3, H, W), dtype=torch.uint8, device=dev) for _ in range(bsz)] for _ in range(2)]
        self.ready = [None, None]
        self.free = [None, None]

    def issue(self, i):
        slot = i % 2
        with torch.cuda.stream(self.stream):
            if self.free[slot] is not None:
                self.stream.wait_event(self.free[slot])  # step i-2 is done with this set
            for buf, src in zip(self.bufs[slot], self.host[i]):
                buf.copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
            self.ready[slot] = ev

    def take(self, i):
        torch.cuda.current_stream(self.dev).wait_event(self.ready[i % 2])
        return self.bufs[i % 2]

    def release(self, i):
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        self.free[i % 2] = ev


def run_ours(args, ws, rank, local):
    from blitzgs_b200 import ops, step as ST
    from blitzgs_b200 import scene as S
    from blitzgs_b200 import distributed as D
    from blitzgs_b200 import dist_step as DS
    dev = torch.device("cuda", local)
    sc, gts_cpu = build_workload(args, dev, rank, ws)
    cams = [c.to(dev) for c in sc.cameras]
    H, W = cams[0].image_height, cams[0].image_width
    if ws > 1:
        shard = D.zorder_shards(sc.xyz, ws)[rank]
        params = [t[shard] for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)]
        D.init_context(rank, ws, H, W, group=None, bsz=args.bsz * ws)
    else:
        params = [sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest]
    model = [t.contiguous().to(dev).requires_grad_(True) for t in params]
    rasters = [S.raster_settings(c, device=dev) for c in cams]
    gts_dev = [g.to(dev) for g in gts_cpu]
    gts_pin = [g.pin_memory() for g in gts_cpu]
    bsz = args.bsz
    n_cams = len(cams)
    history = D.DivisionStrategyHistoryFinal(cams, ws, rank) if ws > 1 else None
    h2d = [0]
    n_launch = [0]  # native kernels of the whole job issued by one_step (see LAUNCHES_PER_VIEW)

    def batch_ids(it):
        return [((it * bsz * ws) + k) % n_cams for k in range(bsz * ws)]

    gx_, gy_ = (W + 15) // 16, (H + 15) // 16
    all_tiles = torch.ones((gy_, gx_), dtype=torch.bool, device=dev)

    def operator_view_loss(raster, gt):
        """One camera through the reference-compatible operator API, as a
        trainer that keeps the reference's renderer calls runs it: torch
        activations, GaussianRasterizer.preprocess_gaussians /
        render_gaussians, the fused L1+SSIM loss and the min-scale
        regulariser over the visible Gaussians."""
        from blitzgs_b200 import rasterizer as RZ
        from blitzgs_b200.loss import band_loss
        xyz, s_raw, q_raw, o_raw, dc, rest = model
        scales = torch.exp(s_raw)
        rast = RZ.GaussianRasterizer(raster)
        ca = {"stats_collector": {}}
        m2, rgb, co, radii, depths = rast.preprocess_gaussians(xyz, scales, torch.nn.functional.normalize(q_raw),
                                                               torch.cat((dc, rest), 1), torch.sigmoid(o_raw), ca)
        abs_pts = torch.zeros_like(xyz) + 0
        color, *_ = rast.render_gaussians(m2, abs_pts, co, rgb, None, depths, radii, all_tiles, None, ca)
        l1, ss = band_loss(color, gt)
        n3 = H * W * 3
        loss = 0.8 * (l1 / n3) + 0.2 * (1.0 - ss / n3)
        vis = radii > 0
        return loss + 10.0 * torch.sort(scales[vis], dim=-1)[0][..., 0].mean()

    def one_step(it, e2e, trace=None, gts_in=None):
        """``e2e``: False (device-resident ground truth), or a 1-element
        pinned host tensor: upload the ground truth from pinned memory (or
        take ``gts_in``, this step's views already uploaded by GTPrefetch)
        and copy the loss into it."""
        upload = e2e is not False
        if trace is not None:
            trace.append(("start", time.perf_counter()))
        for p in model:
            p.grad = None
        if trace is not None:
            trace.append(("grads freed", time.perf_counter()))
        if ws == 1:
            total = None
            for k, ci in enumerate(batch_ids(it)):
                if gts_in is not None:
                    gt = gts_in[k]
                    h2d[0] = 3 * H * W * bsz
                elif upload:
                    gt = torch.empty((3, H, W), dtype=torch.uint8, device=dev)
                    gt.copy_(gts_pin[ci], non_blocking=True)
                    h2d[0] = 3 * H * W * bsz
                else:
                    gt = gts_dev[ci]
                if args.api == "operator":
                    loss = operator_view_loss(rasters[ci], gt)
                else:
                    loss, *_ = ST.view_loss(model, rasters[ci], gt, sparse_grad=args.sparse_grad)
                total = loss if total is None else total + loss
                n_launch[0] += LAUNCHES_PER_VIEW
                if trace is not None:
                    trace.append(("forward", time.perf_counter()))
        else:
            ids = batch_ids(it)
            bcams = [cams[c] for c in ids]
            strategies, _ = D.start_strategy_final(bcams, history)
            gts = []
            nbytes = 0
            for k, c in enumerate(ids):
                rr = strategies[k].row_range(rank)
                if rr is None:
                    gts.append(None)
                    continue
                y0, y1 = rr[0] * 16, min(H, rr[1] * 16)
                if upload:
                    band = torch.empty((3, y1 - y0, W), dtype=torch.uint8, device=dev)
                    band.copy_(gts_pin[c][:, y0:y1], non_blocking=True)
                    nbytes += band.numel()
                else:
                    band = gts_dev[c][:, y0:y1]
                gts.append(band)
            h2d[0] = max(h2d[0], nbytes)
            total = DS.batch_loss(model, [rasters[c] for c in ids], gts, strategies)
            # every rank preprocesses (cull + full), packs and back-propagates every camera of
            # the batch; every rendered band adds unpack, count, binning, blend, loss and pack
            n_launch[0] += ws * DIST_LAUNCHES_PER_CAMERA * len(ids) + \
                DIST_LAUNCHES_PER_BAND * sum(len(st.gpu_ids) for st in strategies)
        total.backward()
        if trace is not None:
            trace.append(("backward", time.perf_counter()))
        if upload:
            # the step's loss to pinned host memory: the copy is queued behind
            # the step (no host wait per step); the timed region ends after a
            # synchronize, so every read has completed inside it
            e2e.copy_(total.detach().reshape(1), non_blocking=True)
        return None

    clocks = ClockSampler(local)
    clocks.start()  # started before warm-up so its start-up cost never lands in the timed region
    # Warm-up visits every camera of the timed sequence (at least W steps), so
    # buffer growth of the allocator and of the binning scratch never lands in
    # the timed region.
    # Two passes over the timed camera sequence: the caching allocator's
    # block splitting only settles in the second (one pass left one cudaMalloc
    # for the first timed step).
    n_warm = max(args.warmup, 2 * args.steps)
    # The collector runs before the warm-up, not between it and the timed
    # region: a full collection idles the GPU long enough for its clocks to
    # drop, which slowed the first timed step by up to 9 ms.
    gc.collect()
    gc.disable()  # no collector pauses inside the timed regions
    for it in range(n_warm):
        one_step(args.warmup + (it % args.steps), False)
        if it == n_warm // 2:
            torch.cuda.synchronize()  # the timed region also starts after one
    torch.cuda.synchronize()
    args.warmup_done = n_warm

    # timed: device-resident inputs (no idle gap after the warm-up)
    barrier(ws)
    torch.cuda.synchronize()
    clocks.mark()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    marks, host_t, trace = [], [time.perf_counter()], []
    mstat0 = torch.cuda.memory_stats(dev)
    n_launch[0] = 0
    t0.record()
    for it in range(args.steps):
        one_step(args.warmup + it, False, trace if it == 0 else None)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()  # no synchronisation: per-step split of the same timed region
        marks.append(ev)
        host_t.append(time.perf_counter())
    t1.record()
    launches = n_launch[0]
    torch.cuda.synchronize()
    clocks.mark()
    barrier(ws)
    ms = max_over_ranks(t0.elapsed_time(t1), ws)
    if rank == 0:
        prev, split = t0, []
        for ev in marks:
            split.append(round(prev.elapsed_time(ev), 3))
            prev = ev
        log("timed-region per-step ms:", split,
            "host ms:", [round((b - a) * 1e3, 3) for a, b in zip(host_t, host_t[1:])],
            "first step host phases ms:", [(n, round((t - trace[0][1]) * 1e3, 3)) for n, t in trace],
            "allocator calls in region:", {k: torch.cuda.memory_stats(dev).get(k, 0) - mstat0.get(k, 0)
                                           for k in ("num_device_alloc", "num_device_free", "num_alloc_retries")})

    # timed: end to end (GT uploaded from pinned host memory, loss read back)
    barrier(ws)
    torch.cuda.synchronize()
    clocks.mark()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    loss_host = torch.empty((args.steps,), dtype=torch.float32, pin_memory=True)
    pf = GTPrefetch(dev, [[gts_pin[c] for c in batch_ids(args.warmup + it)] for it in range(args.steps)], H, W, bsz) \
        if ws == 1 else None
    e0.record()
    if pf is not None:
        pf.issue(0)
    for it in range(args.steps):
        if pf is not None:
            if it + 1 < args.steps:
                pf.issue(it + 1)  # the next step's upload overlaps this step
            one_step(args.warmup + it, loss_host[it:it + 1], gts_in=pf.take(it))
            pf.release(it)
        else:
            one_step(args.warmup + it, loss_host[it:it + 1])
    e1.record()
    torch.cuda.synchronize()
    clocks.mark()
    barrier(ws)
    clk = clocks.stop()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), ws)
    if not bool(torch.isfinite(loss_host).all()):
        raise RuntimeError(f"non-finite loss read back: {loss_host.tolist()}")

    # per-step device times of the same sequence (diagnostic, stderr)
    per = []
    for it in range(args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b_ = torch.cuda.Event(enable_timing=True)
        a.record()
        one_step(args.warmup + it, False)
        b_.record()
        torch.cuda.synchronize()
        per.append(round(a.elapsed_time(b_), 3))
    if rank == 0:
        log("per-step ms:", per)

    # stage timing pass (events around each native call) for the roofline, on warmed cameras
    ops.TIMER.enabled = True
    ops.TIMER.reset()
    for it in range(min(args.steps, 3)):
        one_step(args.warmup + it, False)
    torch.cuda.synchronize()
    stages = ops.TIMER.summary()
    ops.TIMER.enabled = False
    gc.enable()
    n_stage_steps = min(args.steps, 3)
    return dict(ms=ms, ms_e2e=ms_e2e, clocks=clk, stages=stages, H=H, W=W, P=sc.P, bsz=bsz,
                h2d=h2d[0], d2h=4, n_stage_steps=n_stage_steps, launches=launches)


def stage_bytes(name, metas):
    """Algorithmic (minimum) DRAM bytes of one native stage, summed over its
    launches.  P = Gaussians processed, V = Gaussians that touch a rendered
    tile (n_vis of the same view), L = Gaussians with radius > 0 (the visible
    list, when the launch produced or consumed one).
      preprocess_fwd with the fused tile count and the list: every Gaussian
        reads xyz and its log-scales (24: the cull's bound needs the largest
        scale) and writes its radius and tile count (8); listed ones also
        read rotation 16, opacity 4, SH 192 (and xyz, scale again: 24) and
        write their 40 output bytes and list slot 4.
      preprocess_fwd, dense: every Gaussian reads xyz (12) and writes its 44
        output bytes; visible ones also read scale 12, rotation 16, opacity 4,
        SH 192.
      preprocess_bwd over the list: listed Gaussians read their parameters
        (236) and upstream gradients (36) and write their 236 gradient bytes.
      preprocess_bwd, dense: every Gaussian reads its radius (4) and writes
        its 236 gradient bytes; visible ones also read parameters and upstream
        gradients (272)."""
    tot = 0.0
    for m in metas:
        P, V = m.get("P", 0), m.get("n_vis", 0)
        L = int(m["n_list"]) if "n_list" in m else None
        if name == "preprocess_fwd":
            tot += (32.0 * P + 280.0 * L) if (L is not None and m.get("fused_count")) else (56.0 * P + 224.0 * V)
        elif name == "preprocess_bwd":
            tot += 508.0 * L if L is not None else (240.0 * P + 272.0 * V)
        else:
            return None
    return tot


# Fused L1 + SSIM, algorithmic work per output pixel and channel (the
# separable 11-tap window; halo rows and recomputed products not counted):
#   forward: the five moments' horizontal and vertical passes 2 x 5 x 11 x 2
#   = 220, the three products x^2, y^2, xy, the SSIM value and its three
#   partial derivatives 31, |x - y| and the two running sums 4 -> 258 FLOP;
#   reads the image (4 B) and the target (1 B as uint8, 4 as float32) and
#   writes the three partials (12 B).
#   backward: the three partials' two passes 2 x 3 x 11 x 2 = 132 and the
#   pixel gradient 10 -> 142 FLOP; reads image, target and partials and
#   writes the pixel gradient (4 B).
LOSS_FWD_FLOP_PER_PX = 258
LOSS_BWD_FLOP_PER_PX = 142


def _ints(v):
    return [int(x) for x in (v.tolist() if hasattr(v, "tolist") else v)]


def stage_work(name, metas):
    """(FLOP, DRAM bytes) of all launches of one native stage, from the stage
    timer's per-launch metadata; None where the stage has no model in that
    form.  FLOP: the blend stages' per-pair model (forward 10 per evaluated
    and 13 per contributing pair, backward 70 per replayed pair, pairs from
    the kernels' own counters) and the loss's per-pixel counts above.  Bytes:
    stage_bytes for the preprocess stages (only where the launch reports its
    list length L); the binning's 4 P (tile counts read) + 4 V (visible list
    written) + 20 R (each instance's 8-byte key written and read back, its
    4-byte index written), with V and R the view's own totals (not the
    buffer capacities a launch may have been issued with); the tile
    count pass's 16 P (screen mean 8 and radius 4 read, count 4 written);
    the loss's image, target and partial bytes above.  The blend stages'
    DRAM bytes are left out: their per-Gaussian reads are L2 hits shared by
    a tile's strips (ncu: 20-70 MB per city launch against about 8 TFLOP)."""
    flop = byts = None
    if name in ("blend_fwd", "blend_bwd") and all("pairs" in m for m in metas):
        flop = 0.0
        for m in metas:
            pr = _ints(m["pairs"])
            flop += (10.0 * pr[0] + 13.0 * pr[1]) if name == "blend_fwd" else 70.0 * pr[0]
    elif name in ("loss_fwd", "loss_bwd") and all("pixels" in m for m in metas):
        px = sum(int(m["pixels"]) for m in metas)
        gtb = sum(int(m["pixels"]) * int(m.get("gt_bytes", 4)) for m in metas)
        if name == "loss_fwd":
            flop, byts = LOSS_FWD_FLOP_PER_PX * px, 16.0 * px + gtb
        else:
            flop, byts = LOSS_BWD_FLOP_PER_PX * px, 20.0 * px + gtb
    elif name == "binning":
        # "totals" where the launch was sized by capacities; else R / n_vis are exact
        if all("totals" in m or ("R" in m and "n_vis" in m) for m in metas):
            byts = 0.0
            for m in metas:
                R, V = _ints(m["totals"])[:2] if "totals" in m else (int(m["R"]), int(m["n_vis"]))
                byts += 4.0 * m.get("P", 0) + 4.0 * V + 20.0 * R
    elif name == "bin_count":
        byts = sum(16.0 * m.get("P", 0) for m in metas)
    elif name in ("preprocess_fwd", "preprocess_bwd"):
        if all("n_list" in m and (name == "preprocess_bwd" or m.get("fused_count")) for m in metas):
            byts = stage_bytes(name, metas)
    return flop, byts


def stage_rooflines(stages, peaks, peak_kind, fp32_peak):
    """Every native stage against its roofline: the lower bound on its time is
    max(FLOP / FP32 peak, bytes / copy bandwidth) over its modelled work, and
    ``frac`` = that bound / the event-timed duration (1.0 = at the roofline).
    ``bound`` names the larger term; ``achieved`` is that resource's rate."""
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    out = {}
    for name, (calls, ms, metas) in stages.items():
        flop, byts = stage_work(name, metas)
        if (flop is None and byts is None) or ms <= 0 or calls <= 0:
            out[name] = {"model": None, "ms_per_launch": round(ms / max(calls, 1), 4)}
            continue
        t = ms / 1e3
        t_f = flop / (fp32_peak * 1e12) if flop is not None and fp32_peak else 0.0
        t_b = byts / (hbm * 1e9) if byts is not None else 0.0
        if flop is not None and not fp32_peak and t_b == 0.0:
            out[name] = {"model": "fp32", "frac": None, "ms_per_launch": round(ms / calls, 4),
                         "flop_per_launch": round(flop / calls)}
            continue
        e = {"bound": "fp32" if t_f >= t_b else "hbm", "ms_per_launch": round(ms / calls, 4),
             "frac": round(max(t_f, t_b) / t, 4)}
        if e["bound"] == "fp32":
            e.update(achieved=round(flop / t / 1e12, 3), peak=round(fp32_peak, 2), unit="TFLOP/s")
        else:
            e.update(achieved=round(byts / t / 1e9, 1), peak=hbm, unit="GB/s")
        if flop is not None:
            e["flop_per_launch"] = round(flop / calls)
        if byts is not None:
            e["bytes_per_launch"] = round(byts / calls)
        out[name] = e
    out["peaks"] = {"fp32_tflops": round(fp32_peak, 2) if fp32_peak else None,
                    "fp32_source": "measured in this run (FP32 FMA probe, blitz_fp32_probe)",
                    "hbm_gbs": hbm, "hbm_source": peak_kind}
    return out


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each
# stage's kernels, summed over the stage's kernels, measured by ncu on this
# bench's city workload (one-pass capture of the full workload).
# Fill in again whenever the kernels change.
NCU_TRAFFIC = {"preprocess_fwd": 341_700_000, "blend_fwd": 19_800_000, "blend_bwd": 69_700_000,
               "preprocess_bwd": 165_200_000}
NCU_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of bench.py (city, 1 GPU), mean over two "
                      "launches of the full workload")


def roofline_from_stages(stages, peaks, peak_kind, n_vis_per_call, fp32_peak=None):
    """Dominant native stage by time.  HBM-bound stages: algorithmic bytes per
    launch / mean event-timed duration vs the measured copy bandwidth.  The
    blend stages are FP32-issue bound: algorithmic FLOPs from the per-pair
    model (forward 10 FLOP per evaluated pair + 13 per contributing pair,
    backward 70 FLOP per replayed pair; pairs counted by the kernels' own
    per-tile counters) vs the FP32 FMA throughput measured in this run."""
    if not stages:
        return None, {}
    per = {k: (v[0], v[1]) for k, v in stages.items()}
    dom = max(per, key=lambda k: per[k][1])
    calls, tot = per[dom]
    table = {k: {"calls": v[0], "ms_total": round(v[1], 4)} for k, v in per.items()}
    metas = [dict(m, n_vis=n_vis_per_call[i % len(n_vis_per_call)]) for i, m in enumerate(stages[dom][2])]
    hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    if dom in ("blend_fwd", "blend_bwd"):
        flops = 0.0
        for m in metas:
            pr = [int(x) for x in m["pairs"]]
            flops += (10.0 * pr[0] + 13.0 * pr[1]) if dom == "blend_fwd" else 70.0 * pr[0]
        tf = flops / (tot / 1e3) / 1e12
        return {"kernel": dom, "bound": "fp32", "achieved": round(tf, 3), "peak": round(fp32_peak, 2) if fp32_peak else None,
                "unit": "TFLOP/s", "frac": round(tf / fp32_peak, 4) if fp32_peak else None, "traffic": None,
                "peak_source": "measured in this run (FP32 FMA probe, blitz_fp32_probe)",
                "flops_per_launch": round(flops / calls), "ms_per_launch": round(tot / calls, 4)}, table
    byts = stage_bytes(dom, metas)
    if byts is None:
        return {"kernel": dom, "bound": None, "achieved": None, "peak": None, "unit": None, "frac": None,
                "traffic": None}, table
    gbs = byts / (tot / 1e3) / 1e9
    return {"kernel": dom, "bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(gbs / hbm, 4), "traffic": None, "peak_source": peak_kind,
            "bytes_per_launch": round(byts / calls), "ms_per_launch": round(tot / calls, 4)}, table


def hbm_roofline(stages, peaks, peak_kind, n_vis_per_call):
    """The same arithmetic for the slowest HBM-bound stage (preprocess)."""
    cands = [k for k in ("preprocess_fwd", "preprocess_bwd") if k in stages]
    if not cands:
        return None
    sub = {k: stages[k] for k in cands}
    r, _ = roofline_from_stages(sub, peaks, peak_kind, n_vis_per_call)
    return r


def cpu_baseline_sample(budget_s=20.0):
    """CPU oracle on a bounded sample of the city workload: one camera, all 8M
    Gaussians preprocessed, the render + loss + backward restricted to a band
    of tile rows; extrapolated to the full view by the row ratio."""
    from blitzgs_b200 import scene as S
    from oracle import rasterizer_oracle as O
    import numpy as np
    torch.set_num_threads(os.cpu_count() or 1)
    sc = S.city(seed=0)
    cam = sc.cameras[0]
    H, W = cam.image_height, cam.image_width
    gx, gy = (W + 15) // 16, (H + 15) // 16
    rows = 2
    band = np.zeros((gy, gx), bool)
    r0 = gy // 2
    band[r0:r0 + rows] = True
    gt = S.target_image(0, H, W)
    t = time.time()
    s_act = torch.exp(sc.scaling)
    q_act = torch.nn.functional.normalize(sc.rotation)
    o_act = torch.sigmoid(sc.opacity)
    shs = torch.cat((sc.features_dc, sc.features_rest), 1)
    pre = O.preprocess_forward(sc.xyz, s_act, q_act, shs, o_act, cam.world_view_transform, cam.full_proj_transform,
                               cam.camera_center, cam.tanfovx, cam.tanfovy, H, W, 3)
    t_pre = time.time() - t
    t = time.time()
    pl, ranges, _ = O.binning(pre["means2D"].numpy(), pre["depths"].numpy(), pre["radii"].numpy(), H, W, band)
    fwd = O.render_forward(pre["means2D"], pre["conic_opacity"], pre["rgb"], torch.zeros(3), pl, ranges, H, W, band)
    y0, y1 = r0 * 16, min(H, (r0 + rows) * 16)
    loss, l1, ss, dband = O.loss_and_grad(fwd["color"][:, y0:y1], gt[:, y0:y1], H * W)
    dimg = torch.zeros(3, H, W)
    dimg[:, y0:y1] = dband
    rec = O.render_backward(pre["means2D"], pre["conic_opacity"], pre["rgb"], torch.zeros(3), pl, ranges, H, W, dimg,
                            band)
    t_band = time.time() - t
    t = time.time()
    O.preprocess_backward(sc.xyz, s_act, q_act, shs, o_act, cam.world_view_transform, cam.full_proj_transform,
                          cam.camera_center, cam.tanfovx, cam.tanfovy, H, W, 3, pre["radii"], rec[:, 0:2],
                          rec[:, 8:12], rec[:, 12:15])
    t_bwd = time.time() - t
    per_view = t_pre + t_band * (gy / rows) + t_bwd
    return {"value": round(1.0 / per_view, 6), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"city cam 0: preprocess fwd+bwd of all 8M Gaussians ({t_pre + t_bwd:.1f}s) + "
                       f"binning/blend/loss fwd+bwd of {rows} of {gy} tile rows ({t_band:.1f}s), "
                       f"extrapolated by rows")}


# ---------------------------------------------------------------------------
# reference implementation (oracle/_ref)
# ---------------------------------------------------------------------------

def reference_available():
    base = os.path.join(ROOT, "oracle", "_ref")
    return all(os.path.exists(os.path.join(base, p, "_C.so"))
               for p in ("diff_gaussian_rasterization_f", "diff_gaussian_rasterization_r")) and \
        os.path.exists(os.path.join(base, "ref_loss_utils.py"))


def run_reference(args):
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
    import diff_gaussian_rasterization_f as ref
    import ref_loss_utils as LU
    from blitzgs_b200 import scene as S
    dev = torch.device("cuda", 0)
    sc = load_scene(args)
    cams = [c.to(dev) for c in sc.cameras]
    gts_cpu = [S.target_image(k, c.image_height, c.image_width) for k, c in enumerate(sc.cameras)]
    gts_dev = [g.to(dev) for g in gts_cpu]
    gts_pin = [g.pin_memory() for g in gts_cpu]
    model = [t.to(dev).requires_grad_(True) for t in (sc.xyz, sc.scaling, sc.rotation, sc.opacity,
                                                      sc.features_dc, sc.features_rest)]
    H, W = cams[0].image_height, cams[0].image_width
    gx, gy = (W + 15) // 16, (H + 15) // 16
    bg = torch.zeros(3, device=dev)
    n3 = H * W * 3
    strategy = torch.tensor([0, gx * gy], dtype=torch.int32, device=dev)  # division_pos * TILE_X, one rank

    def cuda_args():
        return {"mode": "train", "world_size": "1", "global_rank": "0", "local_rank": "0", "mp_world_size": "1",
                "mp_rank": "0", "log_folder": "/tmp", "log_interval": "1000000", "iteration": "1",
                "avoid_pixel_all2all": False, "stats_collector": {}}

    def view_loss(cam, gt_u8):
        xyz, s_raw, q_raw, o_raw, dc, rest = model
        # GaussianModel getters (scene/gaussian_model.py:248-276)
        scales = torch.exp(s_raw)
        rots = torch.nn.functional.normalize(q_raw)
        shs = torch.cat((dc, rest), dim=1)
        opac = torch.sigmoid(o_raw)
        rs = ref.GaussianRasterizationSettings(
            image_height=H, image_width=W, tanfovx=cam.tanfovx, tanfovy=cam.tanfovy, bg=bg, scale_modifier=1.0,
            viewmatrix=cam.world_view_transform, projmatrix=cam.full_proj_transform, sh_degree=3,
            campos=cam.camera_center, prefiltered=False, debug=False)
        rast = ref.GaussianRasterizer(rs)
        ca = cuda_args()
        means2D, rgb, conic, radii, depths = rast.preprocess_gaussians(xyz, scales, rots, shs, opac, ca)
        cl = torch.ones((gy, gx), dtype=torch.bool, device=dev)
        abs_pts = torch.zeros_like(xyz) + 0
        all_map = torch.zeros((xyz.shape[0], 5), device=dev)
        color, *_ = rast.render_gaussians(means2D, abs_pts, conic, rgb, all_map, depths, radii, cl, None, ca)
        gt = torch.clamp(gt_u8 / 255.0, 0.0, 1.0)
        ones = torch.ones((H, W), dtype=torch.bool, device=dev)
        Ll1 = LU.pixelwise_l1_with_mask(color, gt, ones).sum() / n3
        ss = LU.pixelwise_ssim_with_mask(color, gt, ones).sum() / n3
        loss = 0.8 * Ll1 + 0.2 * (1.0 - ss)
        # render_final's visibility_filter: radius > 0 among the Gaussians
        # get_local2j_ids_bool routes to this rank (all tiles at world size 1)
        routed = ref._C.get_local2j_ids_bool(H, W, 0, 1, means2D.detach(), radii, strategy, ca)[:, 0]
        vis = (radii > 0) & routed
        if vis.sum() > 0:
            loss = loss + 10.0 * torch.sort(scales[vis], dim=-1)[0][..., 0].mean()
        return loss

    bsz = args.bsz

    def batch_ids(it):
        """Cameras of step ``it``: the repo arm's sequence on one GPU."""
        return [(it * bsz + k) % len(cams) for k in range(bsz)]

    def one_step(it, e2e, gts_in=None):
        """``e2e``: False (device-resident ground truth), or a 1-element
        pinned host tensor: upload the ground truth from pinned memory (or
        take ``gts_in``, this step's views already uploaded by GTPrefetch)
        and copy the loss into it."""
        upload = e2e is not False
        for p in model:
            p.grad = None
        total = None
        for k, ci in enumerate(batch_ids(it)):
            if gts_in is not None:
                gt = gts_in[k]
            elif upload:
                gt = torch.empty((3, H, W), dtype=torch.uint8, device=dev)
                gt.copy_(gts_pin[ci], non_blocking=True)
            else:
                gt = gts_dev[ci]
            loss = view_loss(cams[ci], gt)
            total = loss if total is None else total + loss
        total.backward()
        if upload:
            e2e.copy_(total.detach().reshape(1), non_blocking=True)

    clocks = ClockSampler(0)
    clocks.start()
    n_warm = max(args.warmup, args.steps)
    gc.collect()  # before the warm-up: no idle gap right before the timed region
    gc.disable()
    for it in range(n_warm):
        one_step(args.warmup + (it % args.steps), False)
    torch.cuda.synchronize()
    args.warmup_done = n_warm
    clocks.mark()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for it in range(args.steps):
        one_step(args.warmup + it, False)
    t1.record()
    torch.cuda.synchronize()
    clocks.mark()
    ms = t0.elapsed_time(t1)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    loss_host = torch.empty((args.steps,), dtype=torch.float32, pin_memory=True)
    # the same one-step-ahead ground-truth upload as the repo arm on one GPU
    pf = GTPrefetch(dev, [[gts_pin[c] for c in batch_ids(args.warmup + it)] for it in range(args.steps)], H, W, bsz)
    e0.record()
    pf.issue(0)
    for it in range(args.steps):
        if it + 1 < args.steps:
            pf.issue(it + 1)  # the next step's upload overlaps this step
        one_step(args.warmup + it, loss_host[it:it + 1], gts_in=pf.take(it))
        pf.release(it)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    # per-step device times (diagnostic, stderr)
    per = []
    for it in range(args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        one_step(args.warmup + it, False)
        b.record()
        torch.cuda.synchronize()
        per.append(round(a.elapsed_time(b), 2))
    log("reference per-step ms:", per)
    gc.enable()
    ms_e2e = e0.elapsed_time(e1)
    return dict(ms=ms, ms_e2e=ms_e2e, clocks=clk, H=H, W=W, P=sc.P)


def run_ops_case(args):
    """Profiling case for the kernels the fused step does not run (no timing,
    no bench line): on one GPU, a mid-scene camera through the operator API
    (forward and backward), the full rasterizer (forward with
    flag_max_count and its backward, render_simp, render_depth,
    markVisible), SparseGaussianAdam (dense mask and compact rows) and a
    one-rank exchange batch.  Runs it three times, the third between
    cudaProfilerStart / cudaProfilerStop (for ncu --profile-from-start off)."""
    import datetime

    import torch.distributed as dist

    from blitzgs_b200 import scene as S, rasterizer as RZ, dist_step as DS, distributed as D, step as ST
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29561")
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60), device_id=dev)
    sc = S.mid(seed=1, P=args.gaussians or 300_000, n_cams=2)
    raw = [t.to(dev).contiguous().requires_grad_(True) for t in
           (sc.xyz, sc.scaling, sc.rotation, sc.opacity, sc.features_dc, sc.features_rest)]
    xyz, s_raw, q_raw, o_raw, dc, rest = raw
    cams = [c.to(dev) for c in sc.cameras]
    rs = S.raster_settings(cams[0], device=dev)
    H, W = cams[0].image_height, cams[0].image_width
    D.init_context(0, 1, H, W, group=None, bsz=1)
    history = D.DivisionStrategyHistoryFinal(cams, 1, 0)
    gt = S.target_image(0, H, W).to(dev)
    opt = RZ.SparseGaussianAdam([{"params": [p], "lr": 1e-3} for p in raw], lr=1e-3, eps=1e-15)
    ca = {"mode": "train", "world_size": "1", "global_rank": "0", "local_rank": "0", "mp_world_size": "1",
          "mp_rank": "0", "log_folder": "/tmp", "log_interval": "1000000", "iteration": "1",
          "avoid_pixel_all2all": False, "stats_collector": {}}

    def activated():
        return torch.exp(s_raw), torch.nn.functional.normalize(q_raw), torch.sigmoid(o_raw)

    def once():
        rast = RZ.GaussianRasterizer(rs)
        scales, rots, opac = activated()
        m2, rgb, co, radii, depths = rast.preprocess_gaussians(xyz, scales, rots, torch.cat((dc, rest), 1), opac, ca)
        cl = torch.ones(((H + 15) // 16, (W + 15) // 16), dtype=torch.bool, device=dev)
        color, *_ = rast.render_gaussians(m2, torch.zeros((xyz.shape[0], 3), device=dev), co, rgb, None, depths,
                                          radii, cl, None, ca)
        color.sum().backward()
        scales, rots, opac = activated()
        screen = torch.zeros_like(xyz, requires_grad=True)
        cull = torch.zeros(xyz.shape[0], dtype=torch.bool, device=dev)
        c2, _, _ = rast(xyz, screen, opac, cull, dc=dc, shs=rest, scales=scales, rotations=rots,
                        flag_max_count=True)
        c2.sum().backward()
        with torch.no_grad():
            rast.render_simp(xyz, screen, opac, cull, dc=dc, shs=rest, scales=scales, rotations=rots)
            rast.render_depth(xyz, screen, opac, cull, dc=dc, shs=rest, scales=scales, rotations=rots)
            rast.markVisible(xyz)
        opt.step(radii > 0, xyz.shape[0])
        for p in raw:
            p.grad = None
        ST.view_loss(raw, rs, gt, sparse_grad=True)[0].backward()
        opt.step()
        for p in raw:
            p.grad = None
        strategies, _ = D.start_strategy_final(cams, history)
        gts = []
        for k in range(len(cams)):
            y0, y1 = strategies[k].row_range(0)
            gts.append(S.target_image(k, H, W).to(dev)[:, y0 * 16:min(H, y1 * 16)])
        DS.batch_loss(raw, [S.raster_settings(c, device=dev) for c in cams], gts, strategies).backward()
        for p in raw:
            p.grad = None
        torch.cuda.synchronize()

    once()
    once()
    torch.cuda.cudart().cudaProfilerStart()
    once()
    torch.cuda.cudart().cudaProfilerStop()
    dist.destroy_process_group()
    print(json.dumps({"ops_case": "ok", "gaussians": xyz.shape[0]}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="city")
    ap.add_argument("--bsz", type=int, default=1, help="views per GPU per step")
    ap.add_argument("--layout", choices=["zorder", "given"], default="zorder",
                    help="Gaussian memory order of the synthetic scene (both arms)")
    ap.add_argument("--sparse-grad", action="store_true",
                    help="parameter gradients as sparse rows of the visible Gaussians (1 GPU; default dense)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--api", choices=["fused", "operator"], default="fused",
                    help="fused: blitzgs_b200.step.view_loss; operator: the reference-compatible operator API "
                         "(GaussianRasterizer per camera with torch activations), 1 GPU")
    ap.add_argument("--gaussians", type=int, default=None,
                    help="Gaussian count of the scene (default: the config's); a smaller scene of the same "
                         "distribution is the profiling case")
    ap.add_argument("--ops-case", action="store_true",
                    help="profiling case of the kernels outside the fused step (no bench line; see run_ops_case)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ops_case:
        return run_ops_case(args)

    if args.impl == "reference":
        # The reference arm runs in rank 0 alone, on one GPU: no process group
        # is formed, so the other ranks leave at once with nothing to wait on.
        ws, rank, local = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
        if rank != 0:
            return 0
        torch.cuda.set_device(local)
    else:
        ws, rank, local = dist_setup(args.gpus)
    cfg = {"workload": f"{args.config} (BASELINE config 3: 8M clustered Gaussians, 1152x864 aerial views)"
           if args.config == "city" else args.config,
           "gaussians": None, "image": None, "views_per_gpu_per_step": args.bsz,
           "parallelism": f"dp{ws}" if ws > 1 else "single", "l2": "inputs larger than L2 (8M x 236 B params)",
           "grad": "sparse rows (visible Gaussians)" if args.sparse_grad else "dense",
           "layout": "Gaussians in z-order of their means" if args.layout == "zorder" else "generator order",
           "api": "fused training step (blitzgs_b200.step.view_loss)" if args.api == "fused" else
           "operator API (GaussianRasterizer.preprocess_gaussians / render_gaussians per camera, torch activations)"}

    if args.impl == "reference":
        if not reference_available():
            cb = cpu_baseline_sample()
            line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": 0,
                    "steps": 1, "warmup": 0, "ms_per_step": round(1000.0 / cb["value"], 3),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                    "data": "synthetic", "config": cfg, "cpu_baseline": cb,
                    "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    "note": "reference CUDA build absent; CPU oracle port timed instead"}
            print(json.dumps(line), flush=True)
            return 0
        r = run_reference(args)
        views = args.steps * args.bsz
        value = views / (r["ms"] / 1e3)
        e2e = views / (r["ms_e2e"] / 1e3)
        cfg.update(gaussians=r["P"], image=f"{r['W']}x{r['H']}")
        line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 1,
                "steps": args.steps, "warmup": getattr(args, "warmup_done", args.warmup),
                "ms_per_step": round(r["ms"] / args.steps, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": cfg, "clocks": r["clocks"],
                "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": torch.get_num_threads(),
                                 "kind": "reference",
                                 "sample": "reference CUDA rasterizer (oracle/_ref) on 1 B200, full workload"},
                "e2e": {"value": round(e2e, 4), "unit": UNIT, "h2d_bytes_per_step": 3 * r["H"] * r["W"] * args.bsz,
                        "d2h_bytes_per_step": 4}}
        print(json.dumps(line), flush=True)
        return 0

    r = run_ours(args, ws, rank, local)
    views = args.steps * args.bsz * ws
    value = views / (r["ms"] / 1e3)
    e2e = views / (r["ms_e2e"] / 1e3)
    peaks, pk = load_peaks()
    nv = [m.get("n_vis", 0) for m in r["stages"].get("blend_fwd", (0, 0, []))[2]] or [0]
    from blitzgs_b200 import ops as _ops
    fp32 = _ops.fp32_peak_tflops()
    roof, stage_table = roofline_from_stages(r["stages"], peaks, pk, nv, fp32)
    roof_hbm = hbm_roofline(r["stages"], peaks, pk, nv)
    for rf in (roof, roof_hbm):
        # DRAM traffic of the same kernel per launch, from the ncu capture of
        # this workload (city, 1 GPU, dense gradients) recorded in NCU_TRAFFIC
        t = NCU_TRAFFIC.get(rf.get("kernel")) if rf and ws == 1 and args.config == "city" and \
            not args.gaussians and not args.sparse_grad else None
        if t is not None:
            rf["traffic"] = t
            rf["traffic_source"] = NCU_TRAFFIC_SOURCE
    try:
        stage_roof = stage_rooflines(r["stages"], peaks, pk, fp32)
    except Exception as ex:  # the per-stage table must not sink the bench line
        stage_roof = {"error": repr(ex)}
    cb = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            cb = cpu_baseline_sample()
        except Exception as ex:  # the baseline must not sink the bench line
            cb = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {ex}"}
    cfg.update(gaussians=r["P"], image=f"{r['W']}x{r['H']}")
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": getattr(args, "warmup_done", args.warmup), "ms_per_step": round(r["ms"] / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "clocks": r["clocks"], "roofline": roof, "roofline_hbm": roof_hbm, "stages_ms": stage_table,
            "stages_roofline": stage_roof,
            "cpu_baseline": cb,
            "e2e": {"value": round(e2e, 4), "unit": UNIT, "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"],
                    "transfers": ("ground truth from pinned host memory, one step ahead on a copy stream; "
                                  "loss copied to pinned host memory every step" if ws == 1 else
                                  "ground-truth bands from pinned host memory; loss copied to pinned host "
                                  "memory every step")},
            "gpu_launches": r["launches"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


# kernels launched by the binning + blend calls of one view, as counted in the ncu
# launch list of the bench: tile histogram, tile offsets, scatter, per-tile sort,
# cooperative long-list merge (launched every view; it returns at once when no list
# is longer than 4,096), blend
KERNELS_RENDER_FWD = 6
# native kernels of one single-GPU view: preprocess cull + full (2), binning + blend forward,
# loss forward / combination / combination backward / backward (4), blend backward (1),
# preprocess backward (1) -- 14, as the ncu launch list shows
LAUNCHES_PER_VIEW = 2 + KERNELS_RENDER_FWD + 4 + 1 + 1
# multi-GPU: per rank and camera of the batch (preprocess cull + full, exchange pack, preprocess
# backward), and per rendered band (unpack, tile count, binning + blend, loss forward /
# combination / combination backward / backward, blend backward, gradient-record pack)
DIST_LAUNCHES_PER_CAMERA = 4
DIST_LAUNCHES_PER_BAND = 1 + 1 + KERNELS_RENDER_FWD + 4 + 1 + 1

if __name__ == "__main__":
    sys.exit(main())
