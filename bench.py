"""Benchmark of the quantized-linear forward path on B200.

Workload: one INT4 W4A8 linear
  x fp16 [4096, 3072] ~N(0,1) with 1% outlier channels x20, SmoothRot factors
  U[0.5, 4], rot_size 256, PermuQuant perm = randperm(3072), weights INT4
  U[-8, 7] packed [12288, 1536], group-128 scales U[1e-3, 2e-2].
A step = the whole forward of that layer: prep + per-token INT8 quant (one
kernel) and the group-scale W4A8 GEMM with bias (one kernel).
Metric: linear TOPS = 2*M*N*K / step time (higher is better).

* ``value``: device time of the steps (CUDA events per step, L2 flushed by a
  256 MB write between steps, outside the timed events), whole job over all
  ranks (weak scaling: every rank runs its own 4096 tokens; no collective).
* ``e2e``: the same step through the runtime API with the input copied from
  pinned host memory and the output copied back to pinned host memory inside
  the timed region; copies in, compute and copies out run on three streams so
  that consecutive steps overlap (the output copy over PCIe bounds it).
* ``roofline``: the GEMM kernel's algorithmic ops / its event time against the
  dense INT8 peak (2 x the measured bf16 cuBLAS figure); prep against HBM.
* ``cpu_baseline``: the reference's PyTorch CPU path (torch restatement,
  oracle/torch_reference_path.py) on a 256-token sample of the same layer.

``--impl reference`` times that CPU path alone (all host threads), printing
the same metric.  Under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
import types

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = "comfyui-int-crush_b200"
M, K, N, GS, ROT = 4096, 3072, 12288, 128, 256
OPS = 2.0 * M * N * K
# DRAM read + write bytes of one config-2 GEMM launch, from an ncu capture of
# the GEMM kernel (bench.py --kernel-probe gemm)
GEMM_TRAFFIC = 128.2e6


def _pkg():
    if PKG not in sys.modules:
        m = types.ModuleType(PKG)
        m.__path__ = [os.path.join(ROOT, PKG)]
        m.__package__ = PKG
        sys.modules[PKG] = m
    import importlib
    return importlib.import_module(PKG + "._b200_runtime")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def make_inputs(seed: int = 0, device="cpu"):
    import torch
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    ch = torch.randperm(K, generator=g)[: round(0.01 * K)]
    x[:, ch] *= 20
    x = x.half()
    smoothrot = (torch.rand(K, generator=g) * 3.5 + 0.5).half().float()
    perm = torch.randperm(K, generator=g)
    q = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int8)
    qu = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (qu[:, 0::2] | (qu[:, 1::2] << 4)).contiguous()
    scale = (torch.rand(N, K // GS, generator=g) * (2e-2 - 1e-3) + 1e-3).half()
    bias = (torch.randn(N, generator=g) * 0.02).half()
    d = dict(x=x, smoothrot=smoothrot, perm=perm, packed=packed, scale=scale, bias=bias)
    return {k: v.to(device) for k, v in d.items()}


# ───────────────────────────── CPU baseline ─────────────────────────────────

CONFIG = {"workload": "config2_w4a8_linear M4096 K3072 N12288 g128 rot256 perm smoothrot bias",
          "tokens_per_gpu": M, "l2": "flushed (256 MB write) between timed GPU steps"}


def gpu_arm_config(world: int) -> dict:
    """The ``config`` of the default line (both arms print the same)."""
    return dict(CONFIG, parallelism=f"token-sharded dp{world} (no collective)",
                weights="INT4 group-128, packed [12288, 1536] (GPU arm: repacked once at load)")


def _cpu_layer(d, rows: int):
    """One forward of the config-2 layer through the reference's PyTorch CPU
    path (torch restatement, oracle/torch_reference_path.py): group-128
    dequantisation of the weights (every call, as the reference does),
    SmoothRot + rot 256 + perm prep, F.linear, plus the bias the GPU arm adds
    (the reference's INT4 PyTorch path itself drops it)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch_reference_path as TR
    y = TR.forward_int4_pytorch(d["x"][:rows], d["packed"], d["scale"], K, GS, smoothrot=d["smoothrot"],
                                rot_size=ROT, w_in=K, perm=d["perm"])
    return y.add_(d["bias"])


def _time_cpu(d, rows: int, reps: int) -> float:
    ts = []
    for i in range(reps + 1):
        t0 = time.perf_counter()
        _cpu_layer(d, rows)
        if i:
            ts.append(time.perf_counter() - t0)
    ts.sort()
    return ts[len(ts) // 2]


def cpu_baseline(reps: int = 2) -> dict:
    """The reference's CPU path on the whole 4096-token layer with every host
    thread, plus a 256-token sample on one thread."""
    import torch
    d = make_inputs()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t = _time_cpu(d, M, reps)
    torch.set_num_threads(1)
    t1 = _time_cpu(d, 256, 1)
    torch.set_num_threads(threads)
    return {"value": OPS / t / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"all {M} tokens of the config-2 layer with bias, torch CPU fp16 (group-128 dequant + prep + "
                      f"F.linear), median of {reps}: {t * 1e3:.0f} ms",
            "one_thread": {"value": 2.0 * 256 * N * K / t1 / 1e12, "unit": "TOPS", "cores": 1,
                           "sample": f"256 of {M} tokens, {t1 * 1e3:.0f} ms"}}


def run_reference(args, rank: int) -> None:
    """``--impl reference``: the reference's CPU path on the box's host cores,
    each step the whole 4096-token config-2 layer (bias included), all host
    threads.  Under torchrun only rank 0 runs and prints."""
    if rank != 0:
        return
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    d = make_inputs()
    for _ in range(max(args.warmup, 1)):
        _cpu_layer(d, M)
    steps = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _cpu_layer(d, M)
        steps.append(time.perf_counter() - t0)
    ms = sum(steps) / len(steps) * 1e3
    v = OPS / (ms * 1e-3) / 1e12
    torch.set_num_threads(1)
    t1 = _time_cpu(d, 256, 1)
    line = {"metric": "w4a8_linear_tops", "value": v, "unit": "TOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "impl": "reference", "config": gpu_arm_config(args.gpus),
            "reference_run": "the reference's PyTorch CPU path on the host cores (rank 0 only)",
            "cpu_baseline": {"value": v, "unit": "TOPS", "cores": threads, "kind": "port",
                             "sample": f"all {M} tokens per step, torch CPU path of the reference, bias included"},
            "cpu_one_thread": {"value": 2.0 * 256 * N * K / t1 / 1e12, "unit": "TOPS", "cores": 1,
                               "sample": f"256 of {M} tokens, {t1 * 1e3:.0f} ms"},
            "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ───────────────────────────── GPU arm ──────────────────────────────────────

def _gpu_head_start(ms: float = 10.0) -> None:
    """Keep the GPU busy for ~ms before a timed loop (outside its events) so
    that the host queues the loop's launches ahead of the GPU: the per-step
    events then time GPU work, not host launch latency."""
    import torch
    torch.cuda._sleep(int(ms * 1e-3 * 2.0e9))


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during a timed region.
    One sampler per node (local rank 0) covers all of the node's GPUs: a
    sampler per rank stalled single steps by several ms."""

    def __init__(self, local_rank: int, n_gpus: int = 1):
        self.active = local_rank == 0
        self.n_gpus = n_gpus
        self.proc = None
        self.path = os.path.join("/tmp", f"ic_clocks_{os.getpid()}.csv")

    def __enter__(self):
        if os.environ.get("INTCRUSH_NO_CLOCKS") or not self.active:
            return self
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", os.environ.get("INTCRUSH_CLOCK_MS", "100")],
                stdout=self.f, stderr=subprocess.DEVNULL)
            # the sampler needs a moment to start: wait for its first row so that
            # short timed regions are covered too
            # (two rows: nvidia-smi's start-up work on the GPU is over by its
            # second sample)
            t0 = time.time()
            while time.time() - t0 < 5 and self._rows() < 2:
                time.sleep(0.01)
            self.n0 = self._rows()
        except Exception:
            self.proc = None
        return self

    def _rows(self) -> int:
        try:
            with open(self.path) as f:
                return sum(1 for r in f if r.strip())
        except Exception:
            return 0

    def __exit__(self, *a):
        if self.proc is not None:
            # at least one sample taken after the timed region began
            t0 = time.time()
            while time.time() - t0 < 1 and self._rows() <= self.n0:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if os.environ.get("INTCRUSH_NO_CLOCKS"):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "sampling disabled"}
        if not self.active:
            return None
        try:
            rows = [[c.strip() for c in r.split(",")] for r in open(self.path).read().strip().splitlines() if r.strip()]
            rows = [r for r in rows if r[0].isdigit() and int(r[0]) < self.n_gpus]
            sm = sorted(float(r[1]) for r in rows)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i] == "Active"})
            return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                    "samples": len(rows), "gpus_sampled": self.n_gpus}
        except Exception as e:  # pragma: no cover
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": str(e)}


def _plugin_layer(rt, d, dev):
    """The config-2 layer as the reference's plugin builds it: an
    ``IntCrushOps.Linear`` (``make_intcrush_ops("int4_crush", 256)``) loaded
    from the INT-Crush state-dict layout (packed INT4 weight, fp16 group
    scales, perm, SmoothRot factors, bias).  ComfyUI itself is not installed
    on the box; ``tests/comfy_stub.py`` provides the ``comfy.ops`` /
    ``comfy.quant_ops`` classes the layer subclasses."""
    import importlib
    import torch
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import comfy_stub
    comfy_stub.install()
    importlib.import_module(PKG + ".quant_layout").register_intcrush_layouts()
    ops = importlib.import_module(PKG + "._ops")
    Ops = ops.make_intcrush_ops("int4_crush", ROT)
    name = "double_blocks.0.img_mlp.0"
    parent, lin = comfy_stub.make_parent(Ops.Linear, K, N, name=name)
    parent.to(dev)
    sd = {"weight": d["packed"].cpu(), "weight_scale": d["scale"].cpu(), "weight_perm": d["perm"].cpu(),
          "weight_smoothrot_factors": d["smoothrot"].half().cpu(), "bias": d["bias"].cpu()}
    parent.load_state_dict({f"{name}.{k}": v for k, v in sd.items()}, strict=False)
    return lin


def _step_stats(ms):
    ms = sorted(ms)
    return {"median": ms[len(ms) // 2], "max": ms[-1], "min": ms[0]}


def run_gpu(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist
    rt = _pkg()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    d = make_inputs(seed=rank, device=dev)
    s_w = d["scale"].float()
    perm32 = d["perm"].to(torch.int32)
    # load-time weight preparation (once per layer): nibble-repacked INT4
    w_rep = rt.repack_int4(d["packed"], K, 0)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream()

    def step(x):
        xq, s_a, _, _ = rt.prep_quantize(x, smoothrot=d["smoothrot"], rot_size=ROT, w_in=K, perm=perm32)
        return rt.gemm_a8(xq, w_rep, s_w, s_a, bias=d["bias"], out_dtype=torch.float16, group_size=GS,
                          repacked=True)

    for _ in range(args.warmup):
        step(d["x"])
    torch.cuda.synchronize()

    def timed_region():
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with Clocks(local_rank, world) as clk:
            _gpu_head_start()   # after the sampler is up
            for i in range(2):   # untimed: the first steps after an idle GPU run slow
                flush.fill_(float(i))
                step(d["x"])
            t_wall = time.perf_counter()
            for i in range(args.steps):
                flush.fill_(float(i))
                ev[i][0].record(st)
                xq, s_a, _, _ = rt.prep_quantize(d["x"], smoothrot=d["smoothrot"], rot_size=ROT, w_in=K,
                                                 perm=perm32)
                ev[i][1].record(st)
                rt.gemm_a8(xq, w_rep, s_w, s_a, bias=d["bias"], out_dtype=torch.float16, group_size=GS,
                           repacked=True)
                ev[i][2].record(st)
            torch.cuda.synchronize()
            t_wall = time.perf_counter() - t_wall
        if world > 1:
            dist.barrier()
        prep_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
        gemm_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]
        return prep_ms, gemm_ms, t_wall, clk

    # A step that takes more than 3x the median was stalled by something
    # outside this process (seen on shared hosts: single steps of 3-47 ms
    # among 0.45 ms ones).  Such a region is reported in "discarded" and
    # timed again, at most twice; every rank takes the same decision.
    discarded = []
    for attempt in range(3):
        prep_ms, gemm_ms, t_wall, clk = timed_region()
        step_ms = sorted(p + g for p, g in zip(prep_ms, gemm_ms))
        stall = torch.tensor([float(step_ms[-1] > 3.0 * step_ms[len(step_ms) // 2])], device=dev)
        if world > 1:
            dist.all_reduce(stall, op=dist.ReduceOp.MAX)
        if attempt == 2 or stall.item() == 0.0:
            break
        discarded.append({"max_step_ms": round(step_ms[-1], 3), "median_step_ms": round(step_ms[len(step_ms) // 2], 3)})
    # every rank's per-step times (stderr): an isolated slow step shows here
    print(f"rank {rank} gemm_ms {[round(v, 3) for v in gemm_ms]} prep_ms {[round(v, 3) for v in prep_ms]}",
          file=sys.stderr, flush=True)
    tot_ms = sum(prep_ms) + sum(gemm_ms)

    # e2e through the plugin call: IntCrushOps.Linear.forward, host-pinned
    # input in, host-pinned output out.  Three streams pipeline the steps:
    # the input copy of step i+1 and the output copy of step i-1 overlap the
    # forward of step i (two device buffers each way, ordered by events).
    lin = _plugin_layer(rt, d, dev)
    x_host = d["x"].cpu().pin_memory()
    out_host = [torch.empty((M, N), dtype=torch.float16).pin_memory() for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xd = [torch.empty((M, K), dtype=torch.float16, device=dev) for _ in range(2)]
    yd = [None, None]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_steps(n):
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_cmp[b])          # step i-2 has consumed xd[b]
                xd[b].copy_(x_host, non_blocking=True)
                ev_in[b].record(s_in)
            st.wait_event(ev_in[b])
            if i >= 2:
                st.wait_event(ev_out[b])                # step i-2's output has left yd[b]
            yd[b] = lin(xd[b])
            ev_cmp[b].record(st)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[b])
                out_host[b].copy_(yd[b], non_blocking=True)
                ev_out[b].record(s_out)

    with torch.no_grad():
        e2e_steps(2)
        torch.cuda.synchronize()
        # the plugin layer computes what the kernel step computes
        plugin_equal = bool(torch.equal(lin(d["x"]), step(d["x"])))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(s_in)
        s_in.wait_event(e0)
        e2e_steps(args.steps)
        s_out.wait_stream(st)
        s_out.wait_stream(s_in)
        e1.record(s_out)
        torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    vals = torch.tensor([tot_ms, e2e_ms, sum(gemm_ms), sum(prep_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    tot_ms, e2e_ms, gemm_sum, prep_sum = vals.tolist()
    # DiT-block numbers at the same N (every rank takes part)
    block = None if args.no_secondary else flux_block_secondary(args, rank, world, local_rank, dev, rt)
    feat = None if (args.no_secondary or world == 1) else feature_sharded_secondary(world, rank, dev)

    if rank != 0:
        return
    hbm, bf16, src = _peaks()
    int8_peak = 2.0 * bf16
    ms_step = tot_ms / args.steps
    gemm_avg = gemm_sum / args.steps
    prep_avg = prep_sum / args.steps
    gemm_tops = OPS / (gemm_avg * 1e-3) / 1e12
    prep_bytes = M * K * 2 + M * K * 1 + M * 4 + K * 4 * 2    # x in, int8 out, s_a, perm+smoothrot
    prep_gbs = prep_bytes / (prep_avg * 1e-3) / 1e9
    line = {
        "metric": "w4a8_linear_tops", "value": world * OPS / (ms_step * 1e-3) / 1e12, "unit": "TOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": gpu_arm_config(world),
        "e2e": {"value": world * OPS * args.steps / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                "path": "IntCrushOps.Linear.forward (the plugin layer), pinned host buffers",
                "same_bits_as_kernel_step": plugin_equal},
        "roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": int8_peak, "unit": "TOPS",
                     "frac": gemm_tops / int8_peak, "traffic": GEMM_TRAFFIC,
                     "traffic_note": "bytes/launch, dram read+write from one ncu capture of this GEMM",
                     "kernel": "gemm_tc_kernel<W_I4, grouped>",
                     "peak_source": f"2 x {src} bf16 cuBLAS ({bf16} TF/s), burst",
                     "kernel_ms": gemm_avg},
        "prep_roofline": {"bound": "hbm", "achieved": prep_gbs, "peak": hbm, "unit": "GB/s",
                          "frac": prep_gbs / hbm, "kernel_ms": prep_avg, "peak_source": src},
        "gpu_launches": 2 * args.steps,
        "wall_ms": t_wall * 1e3,
        "clocks": clk.summary(),
    }
    if discarded:
        line["discarded_regions"] = discarded
    if block is not None:
        line.setdefault("secondary", {})["flux_block"] = block
    if feat is not None:
        line.setdefault("secondary", {})["feature_sharded"] = feat
    if world == 1 and not args.no_secondary:
        line.setdefault("secondary", {}).update(secondary_lines(dev, flush, hbm, int8_peak, bf16))
        line["secondary"]["gpu_comparators"] = gpu_comparators(dev, flush, d, w_rep, perm32)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    print(json.dumps(line), flush=True)


def run_features(args, rank: int, world: int, local_rank: int) -> None:
    """Output-feature-sharded layer: every rank holds N / world weight rows,
    preps the same 4096 tokens, runs its GEMM slice, and an NCCL all-gather
    assembles the [M, N] output (strong scaling: total work fixed)."""
    import torch
    import torch.distributed as dist
    rt = _pkg()
    import importlib
    sh = importlib.import_module(PKG + "._sharded")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    d = make_inputs(seed=0, device=dev)          # the same layer and tokens on every rank
    lin = sh.FeatureShardedLinear(d["packed"], d["scale"], d["bias"], group_size=GS, smoothrot=d["smoothrot"],
                                  rot_size=ROT, w_in=K, perm=d["perm"], device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream()
    for _ in range(args.warmup):
        lin(d["x"])
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank, world) as clk:
        _gpu_head_start()   # after the sampler is up
        for i in range(2):   # untimed: the first steps after an idle GPU run slow
            flush.fill_(float(i))
            lin(d["x"])
        for i in range(args.steps):
            flush.fill_(float(i))
            ev[i][0].record(st)
            local = lin.local_forward(d["x"], torch.float16)
            ev[i][1].record(st)
            if world > 1:
                parts = [torch.empty_like(local) for _ in range(world)]
                dist.all_gather(parts, local)
                torch.cat(parts, dim=1)
            ev[i][2].record(st)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    tot = sum(ev[i][0].elapsed_time(ev[i][2]) for i in range(args.steps))
    comp = sum(ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps))
    vals = torch.tensor([tot, comp], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    tot, comp = vals.tolist()
    if rank != 0:
        return
    ms_step = tot / args.steps
    line = {
        "metric": "w4a8_linear_tops", "value": OPS / (ms_step * 1e-3) / 1e12, "unit": "TOPS",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": {"workload": "config2_w4a8_linear M4096 K3072 N12288 g128 rot256 perm smoothrot bias",
                   "parallelism": f"output-feature-sharded x{world} + NCCL all-gather",
                   "l2": "flushed (256 MB write) between timed steps"},
        "compute_ms_per_step": comp / args.steps,
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def _w8a8_call(rt, x, w, s8, b8):
    import torch
    xq, s_a, _, _ = rt.prep_quantize(x, rot_size=256)
    return rt.gemm_a8(xq, w, s8, s_a, bias=b8, out_dtype=torch.float16)


def secondary_lines(dev, flush, hbm_gbs: float, int8_peak: float, bf16_peak: float, reps: int = 20) -> dict:
    """BASELINE configs[0] (W8A8, M=256) and configs[2] (W4A16 small M + LoRA)
    on the GPU.  ``ms``: median CUDA-event time of a lone call, L2 flushed
    before each call (outside the events), so weights come from HBM; this
    includes the host launch latency of a Python call.  ``graph_ms``: device
    time per call of 16-32 calls replayed as one CUDA graph, each call on its
    own weight copy (copies > L2, so weights come from HBM), without host
    launch cost; the ``graph_*`` fractions use it."""
    import torch
    rt = _pkg()
    st = torch.cuda.current_stream()
    g = torch.Generator().manual_seed(0)

    def timed(fn):
        fn()
        ts = []
        for i in range(reps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    def graph_ms(calls):
        """Device time per call of the calls captured into one graph."""
        for c in calls:
            c()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for c in calls:
                c()
        gr.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            gr.replay()
            e1.record(st)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / len(calls))
        del gr
        return sorted(ts)[len(ts) // 2]

    out = {}
    # W8A8 linear, M=256, K=N=3072, rot 256, bias, per-channel scales
    M1, K1 = 256, 3072
    x = torch.randn(M1, K1, generator=g)
    x[:, torch.randperm(K1, generator=g)[: round(0.01 * K1)]] *= 20
    x = x.half().to(dev)
    w8 = torch.randint(-127, 128, (K1, K1), generator=g, dtype=torch.int8).to(dev)
    s8 = (torch.rand(K1, 1, generator=g) * 9e-3 + 1e-3).half().float().to(dev)
    b8 = (torch.randn(K1, generator=g) * 0.02).half().to(dev)

    def w8a8():
        xq, s_a, _, _ = rt.prep_quantize(x, rot_size=256)
        return rt.gemm_a8(xq, w8, s8, s_a, bias=b8, out_dtype=torch.float16)
    ms = timed(w8a8)
    w8c = [w8.clone() for _ in range(16)]   # 16 x 9.4 MB > L2
    gms = graph_ms([(lambda w=w: _w8a8_call(rt, x, w, s8, b8)) for w in w8c])
    del w8c
    byt = M1 * K1 * 2 + K1 * K1 + M1 * K1 * 2
    out["config1_w8a8_m256"] = {"ms": ms, "tops": 2 * M1 * K1 * K1 / (ms * 1e-3) / 1e12,
                                "gbs": byt / (ms * 1e-3) / 1e9, "hbm_frac": byt / (ms * 1e-3) / 1e9 / hbm_gbs,
                                "graph_ms": gms, "graph_hbm_frac": byt / (gms * 1e-3) / 1e9 / hbm_gbs,
                                "kernels": 2, "note": "prep + GEMM, HBM-bound shape (12.6 MB)"}
    # W4A16, rot 0, group-128 scales, rank-32 LoRA (strength 1)
    N3 = K3 = 3072
    q = torch.randint(-8, 8, (N3, K3), generator=g, dtype=torch.int8)
    qu = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (qu[:, 0::2] | (qu[:, 1::2] << 4)).contiguous().to(dev)
    w1 = rt.repack_int4(packed, K3, 1)
    sc = (torch.rand(N3, K3 // 128, generator=g) * (2e-2 - 1e-3) + 1e-3).half().to(dev)
    down = (torch.randn(32, K3, generator=g) * 0.01).half().to(dev)
    up = (torch.randn(N3, 32, generator=g) * 0.01).half().to(dev)
    for M3 in (1, 16, 256):
        x3 = torch.randn(M3, K3, generator=g).half().to(dev)

        def w4a16():
            mid = rt.lowrank_down(x3, down)
            return rt.gemm_w4a16(x3, w1, sc, group_size=128, lr_mid=mid, lr_up=up, lr_scale=1.0, w_layout=1)
        ms = timed(w4a16)
        w1c = [w1.clone() for _ in range(32)]   # 32 x 4.7 MB > L2

        def call(w, x3=x3):
            mid = rt.lowrank_down(x3, down)
            return rt.gemm_w4a16(x3, w, sc, group_size=128, lr_mid=mid, lr_up=up, lr_scale=1.0, w_layout=1)
        gms = graph_ms([(lambda w=w: call(w)) for w in w1c])
        del w1c
        byt = N3 * K3 // 2 + sc.numel() * 2 + (down.numel() + up.numel()) * 2 + 2 * M3 * K3 * 2
        fl = 2 * M3 * N3 * K3 + 4 * M3 * 32 * K3
        out[f"config3_w4a16_lora_m{M3}"] = {
            "ms": ms, "gbs": byt / (ms * 1e-3) / 1e9, "hbm_frac": byt / (ms * 1e-3) / 1e9 / hbm_gbs,
            "tflops": fl / (ms * 1e-3) / 1e12, "bf16_frac": fl / (ms * 1e-3) / 1e12 / bf16_peak,
            "graph_ms": gms, "graph_hbm_frac": byt / (gms * 1e-3) / 1e9 / hbm_gbs,
            "graph_bf16_frac": fl / (gms * 1e-3) / 1e12 / bf16_peak,
            "kernels": 2 if M3 <= 128 else 4,
            "note": "low-rank down + W4A16 (LoRA fused for M <= 128; split-K + reduce + low-rank add above)"}
    # host cost of one call (tiny GEMM, host-bound): the ctypes runtime call
    # and the same call through the torch.library op registered over it
    import importlib
    tops = importlib.import_module(PKG + "._torch_ops")
    tops.register()
    xs = torch.randint(-128, 128, (1, 256), generator=g, dtype=torch.int8).to(dev)
    ws = torch.randint(-127, 128, (256, 256), generator=g, dtype=torch.int8).to(dev)
    sws = torch.full((256,), 1e-2, device=dev)
    sas = torch.full((1,), 1e-2, device=dev)
    f16 = tops.dtype_code(torch.float16)

    def host_us(fn, n=500):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / n * 1e6
    out["host_cost_us_per_call"] = {
        "ctypes_runtime": host_us(lambda: rt.gemm_a8(xs, ws, sws, sas, out_dtype=torch.float16, splits=1)),
        "torch_custom_op": host_us(lambda: torch.ops.intcrush_b200.gemm_a8(xs, ws, sws, sas, None, f16, 0, False)),
        "note": "wall clock per call of a 1x256x256 INT8 GEMM issued back to back (GPU work ~3 us)"}
    return out


def gpu_comparators(dev, flush, d, w_rep, perm32, reps: int = 10) -> dict:
    """The library GPU paths the reference falls back to, timed on the same
    box next to this library's kernels (CUDA events, L2 flushed before each
    call, median of ``reps``).

    * ``torch._int_mm`` (cuBLAS int8) + dequantisation in torch: the
      reference's W8A8 / W4A8 math without its Triton kernels; for W4A8 also
      with the per-call INT4 -> INT8 unpack the reference's W4A8 path does
      (``_ops.py:448-457``), here in torch ops.
    * torch dequantisation (INT4 -> fp16 with group scales) + ``F.linear``:
      the reference's PyTorch INT4 path on the GPU (``_ops.py:483-491``).
    The reference's Triton kernels themselves are not on the box: the
    reference's Python sources do not travel with this repository."""
    import torch
    import torch.nn.functional as F
    rt = _pkg()
    st = torch.cuda.current_stream()

    def timed(fn):
        fn()
        ts = []
        for i in range(reps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    def unpack_i8(p):
        lo = ((p & 0xF).to(torch.int16) ^ 8) - 8
        hi = ((p >> 4).to(torch.int16) ^ 8) - 8
        return torch.stack([lo, hi], dim=-1).reshape(p.shape[0], -1).to(torch.int8)

    out = {}
    g = torch.Generator().manual_seed(5)
    # W4A8 per channel at the config-2 shape
    xq, s_a, _, _ = rt.prep_quantize(d["x"], smoothrot=d["smoothrot"], rot_size=ROT, w_in=K, perm=perm32)
    xq = xq.contiguous()
    s_n = d["scale"][:, 0].float().contiguous()
    w8 = unpack_i8(d["packed"])
    bias = d["bias"]

    def torch_w4a8(unpack):
        w = unpack_i8(d["packed"]) if unpack else w8
        acc = torch._int_mm(xq, w.t())
        return (acc.float() * s_a[:, None] * s_n[None, :] + bias.float()).half()
    t_ours = timed(lambda: rt.gemm_a8(xq, w_rep, s_n, s_a, bias=bias, out_dtype=torch.float16, repacked=True))
    t_mm = timed(lambda: torch_w4a8(False))
    t_mm_u = timed(lambda: torch_w4a8(True))
    out["w4a8_per_channel_4096x12288x3072"] = {
        "ours_ms": t_ours, "int_mm_dequant_ms": t_mm, "unpack_int_mm_dequant_ms": t_mm_u,
        "ratio_vs_int_mm": t_mm / t_ours, "ratio_vs_unpack_int_mm": t_mm_u / t_ours}
    # W8A8 per channel: config-1 shape and the config-2 GEMM shape
    for (mm, nn, kk) in ((256, 3072, 3072), (4096, 12288, 3072)):
        xa = torch.randint(-128, 128, (mm, kk), generator=g, dtype=torch.int8).to(dev)
        wb = torch.randint(-127, 128, (nn, kk), generator=g, dtype=torch.int8).to(dev)
        sa = (torch.rand(mm, generator=g) * 5e-2 + 1e-3).to(dev)
        sb = (torch.rand(nn, generator=g) * 1e-2 + 1e-3).to(dev)
        bb = (torch.randn(nn, generator=g) * 0.02).half().to(dev)
        t_ours = timed(lambda: rt.gemm_a8(xa, wb, sb, sa, bias=bb, out_dtype=torch.float16))
        t_mm = timed(lambda: (torch._int_mm(xa, wb.t()).float() * sa[:, None] * sb[None, :] + bb.float()).half())
        out[f"w8a8_{mm}x{nn}x{kk}"] = {"ours_ms": t_ours, "int_mm_dequant_ms": t_mm, "ratio": t_mm / t_ours}
    # W4A16: torch dequantisation + F.linear
    N3 = K3 = 3072
    q = torch.randint(-8, 8, (N3, K3), generator=g, dtype=torch.int8)
    qu = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (qu[:, 0::2] | (qu[:, 1::2] << 4)).contiguous().to(dev)
    w1 = rt.repack_int4(packed, K3, 1)
    sc = (torch.rand(N3, K3 // 128, generator=g) * (2e-2 - 1e-3) + 1e-3).half().to(dev)

    def dequant_f16():
        wq = unpack_i8(packed).float().reshape(N3, -1, 128) * sc.float().unsqueeze(2)
        return wq.reshape(N3, K3).half()
    for M3 in (1, 16, 256):
        x3 = torch.randn(M3, K3, generator=g).half().to(dev)
        t_ours = timed(lambda: rt.gemm_w4a16(x3, w1, sc, group_size=128, w_layout=1))
        t_t = timed(lambda: F.linear(x3, dequant_f16()))
        out[f"w4a16_m{M3}"] = {"ours_ms": t_ours, "torch_dequant_linear_ms": t_t, "ratio": t_t / t_ours}
    return out


def feature_sharded_secondary(world: int, rank: int, dev, steps: int = 5) -> dict:
    """The config-2 layer split by output features over the ranks (each rank
    holds N / world weight rows, preps the same 4096 tokens, runs its GEMM
    slice; an NCCL all-gather assembles [M, N]; strong scaling).  Timed two
    ways: one all-gather after the whole GEMM, and the GEMM in 4 token chunks
    with each chunk's all-gather issued asynchronously behind the next
    chunk's GEMM.  Max over ranks of the per-call time."""
    import importlib
    import torch
    import torch.distributed as dist
    sh = importlib.import_module(PKG + "._sharded")
    d = make_inputs(seed=0, device=dev)
    lin = sh.FeatureShardedLinear(d["packed"], d["scale"], d["bias"], group_size=GS, smoothrot=d["smoothrot"],
                                  rot_size=ROT, w_in=K, perm=d["perm"], device=dev)
    st = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()
    with torch.no_grad():
        plain = lin(d["x"])
        ov = lin.forward_overlapped(d["x"], chunks=4)
        same = bool(torch.equal(plain, ov))
        # the single-GPU layer on the same inputs (every rank checks all columns)
        rt = _pkg()
        xq, s_a, _, _ = rt.prep_quantize(d["x"], smoothrot=d["smoothrot"], rot_size=ROT, w_in=K,
                                         perm=d["perm"].to(torch.int32))
        one = rt.gemm_a8(xq, rt.repack_int4(d["packed"], K, 0), d["scale"].float(), s_a, bias=d["bias"],
                         out_dtype=torch.float16, group_size=GS, repacked=True)
        eq = torch.tensor([float(torch.equal(plain, one))], device=dev)
        dist.all_reduce(eq, op=dist.ReduceOp.MIN)
        del one, xq
        t_plain = timed(lambda: lin(d["x"]))
        t_ov = timed(lambda: lin.forward_overlapped(d["x"], chunks=4))
        t_local = timed(lambda: lin.local_forward(d["x"], torch.float16))
    return {"tops": OPS / (min(t_plain, t_ov) * 1e-3) / 1e12, "ms_all_gather_after_gemm": t_plain,
            "ms_chunked_overlap": t_ov, "ms_local_gemm_only": t_local, "n_gpus": world,
            "all_gather_bytes_per_rank": M * (-(-N // world)) * 2 * (world - 1),
            "overlapped_equals_plain": same, "equals_single_gpu_layer": bool(eq.item() == 1.0),
            "layout": f"output-feature-sharded x{world}: N/{world} weight rows per GPU, NCCL all-gather of [M, N]"}


def flux_block_secondary(args, rank: int, world: int, local_rank: int, dev, rt, steps: int = 5) -> dict:
    """The Flux-class double block at this run's N: every rank
    runs one sample (token sharding, no collective); at N > 1 also one sample
    split over the ranks (sequence parallel, K/V all-gather over NCCL) and the
    time of the block's K/V all-gathers alone.  tokens/s over all ranks,
    block time = max over ranks."""
    import torch
    import torch.distributed as dist
    blk = FluxDoubleBlock(rt, dev)
    g = torch.Generator().manual_seed(100 + rank)
    img = torch.randn(1, 4096, 3072, generator=g).half().to(dev)
    txt = torch.randn(1, 512, 3072, generator=g).half().to(dev)
    vec = torch.randn(1, 3072, generator=g).half().to(dev)
    st = torch.cuda.current_stream()

    def timed_block(im):
        with torch.no_grad():
            for _ in range(2):
                blk(im, txt, vec)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(steps):
                blk(im, txt, vec)
            e1.record(st)
            torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    n_tok = 4096 + 512
    ms = timed_block(img)
    res = {"tokens_per_s": world * n_tok / (ms * 1e-3), "block_ms": ms, "n_gpus": world,
           "layout": f"token-sharded x{world} (one sample per GPU, no collective)",
           "linear_tops": world * blk.linear_ops(4096, 512) / (ms * 1e-3) / 1e12}
    if world > 1:
        # one sample, the same on every rank (seed 100), split by image tokens
        gc = torch.Generator().manual_seed(100)
        img_c = torch.randn(1, 4096, 3072, generator=gc).half().to(dev)
        txt_c = torch.randn(1, 512, 3072, generator=gc).half().to(dev)
        vec_c = torch.randn(1, 3072, generator=gc).half().to(dev)
        blk.sp_group = dist.group.WORLD
        per, pt = 4096 // world, 512 // world
        mine = img_c[:, rank * per:(rank + 1) * per].contiguous()
        mine_t = txt_c[:, rank * pt:(rank + 1) * pt].contiguous()
        # check: the ranks' rows together equal the single-GPU block's
        with torch.no_grad():
            o_img, o_txt = blk(mine, mine_t, vec_c)
            gi = [torch.empty_like(o_img) for _ in range(world)]
            gt = [torch.empty_like(o_txt) for _ in range(world)]
            dist.all_gather(gi, o_img.contiguous())
            dist.all_gather(gt, o_txt.contiguous())
            blk.sp_group = None
            r_img, r_txt = blk(img_c, txt_c, vec_c)
            blk.sp_group = dist.group.WORLD
        sp_err = max(float((torch.cat(a, 1).float() - b.float()).abs().max() / b.float().abs().max())
                     for a, b in ((gi, r_img), (gt, r_txt)))
        txt, vec = mine_t, vec_c
        ms_sp = timed_block(mine)
        # the block's four K/V all-gathers (image and text, K and V) alone
        kv = torch.randn(2, 1, 24, per, 128, generator=g).half().to(dev)
        kvt = torch.randn(2, 1, 24, pt, 128, generator=g).half().to(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(2):
            _gather_tokens(kv[0], dist.group.WORLD)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(steps):
            for t4 in (kvt[0], kvt[1], kv[0], kv[1]):
                _gather_tokens(t4, dist.group.WORLD)
        e1.record(st)
        torch.cuda.synchronize()
        ag = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        res["sequence_parallel"] = {
            "tokens_per_s": n_tok / (ms_sp * 1e-3), "block_ms": ms_sp,
            "kv_all_gather_ms": ag.item(),
            "max_rel_vs_single_gpu_block": sp_err,
            "layout": f"one sample over {world} GPUs: image and text tokens split, K/V all-gather (NCCL)"}
        blk.sp_group = None
    return res


class _QLinear:
    """INT4 W4A8 linear with group-128 scales, SmoothRot, rot 256 and a random
    PermuQuant perm -- the layer of BASELINE configs[3], run through the
    runtime's fused prep and GEMM (random-init weights)."""

    def __init__(self, rt, n_out: int, n_in: int, g, dev):
        import torch
        q = torch.randint(-8, 8, (n_out, n_in), generator=g, dtype=torch.int8)
        qu = (q.to(torch.int16) & 0xF).to(torch.uint8)
        self.rt = rt
        self.w = rt.repack_int4((qu[:, 0::2] | (qu[:, 1::2] << 4)).contiguous().to(dev), n_in, 0)
        self.s = (torch.rand(n_out, n_in // GS, generator=g) * 2e-3 + 1e-4).float().to(dev)
        self.sr = (torch.rand(n_in, generator=g) * 3.5 + 0.5).half().float().to(dev)
        self.perm = torch.randperm(n_in, generator=g).to(torch.int32).to(dev)
        self.b = (torch.randn(n_out, generator=g) * 0.02).half().to(dev)
        self.n_in = n_in

    def __call__(self, x, norm=None, activation=0):
        x2 = x.reshape(-1, x.shape[-1])
        xq, s_a, _, _ = self.rt.prep_quantize(x2, smoothrot=self.sr, rot_size=ROT, w_in=self.n_in, perm=self.perm,
                                              norm=norm)
        y = self.rt.gemm_a8(xq, self.w, self.s, s_a, bias=self.b, out_dtype=x.dtype, group_size=GS, repacked=True,
                            activation=activation)
        return y.reshape(*x.shape[:-1], y.shape[-1])


def _gather_tokens(t, group, async_op=False):
    """All-gather [B, heads, L_local, d] along the token axis over the group.
    With async_op, returns a function that waits for the gather and returns
    the gathered tensor (the gather overlaps whatever is issued meanwhile)."""
    import torch
    import torch.distributed as dist
    t = t.contiguous()
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    work = dist.all_gather(parts, t, group=group, async_op=async_op)
    if not async_op:
        return torch.cat(parts, dim=2)

    def done():
        work.wait()
        return torch.cat(parts, dim=2)
    return done


class FluxDoubleBlock:
    """Flux-class MMDiT double-stream block: hidden 3072,
    24 heads x 128, MLP 12288 GELU(tanh), adaLN modulation from a 3072-d
    vector, separate image / text weights, joint attention over text + image
    tokens.  Every linear is the quantised layer above; norms, modulation,
    GELU and attention (torch SDPA) run in fp16.  Random-init weights.

    With ``fused_norm`` (default) the pre-attention and pre-MLP LayerNorm
    (eps 1e-6, no affine) and the adaLN modulation ``(1 + scale) * x + shift``
    run inside the quantised layer's prep kernel as a LayerNorm with
    per-sample gamma = 1 + scale, beta = shift (batch 1).

    With ``sp_group`` (sequence parallel, one sample over the ranks of the
    group) ``img`` and ``txt`` are this rank's contiguous slices of the image
    and text tokens: each rank projects its own tokens, both streams' K and V
    are all-gathered over the group (NCCL), and each rank's queries attend
    over all keys (text keys first, as in the single-GPU block).  Everything
    else is token-local, so the per-rank outputs are the matching rows of the
    single-GPU block, and no rank repeats another's linear work.
    ``linear`` replaces the quantised layer (tests use a CPU stand-in)."""

    def __init__(self, rt, dev, seed=0, hidden=3072, heads=24, mlp=12288, fused_norm=True, sp_group=None,
                 linear=None, dtype=None):
        import torch
        g = torch.Generator().manual_seed(seed)
        self.fused_norm = fused_norm
        self.sp_group = sp_group
        self.h, self.nh = hidden, heads
        dtype = dtype or torch.float16
        mk = (lambda o, i: _QLinear(rt, o, i, g, dev)) if linear is None else (lambda o, i: linear(o, i, g))
        self.mod = {s: mk(6 * hidden, hidden) for s in ("img", "txt")}
        self.qkv = {s: mk(3 * hidden, hidden) for s in ("img", "txt")}
        self.proj = {s: mk(hidden, hidden) for s in ("img", "txt")}
        self.fc1 = {s: mk(mlp, hidden) for s in ("img", "txt")}
        self.fc2 = {s: mk(hidden, mlp) for s in ("img", "txt")}
        self.qn = {s: (1 + 0.1 * torch.randn(128, generator=g)).to(dtype).to(dev) for s in ("img", "txt")}
        self.kn = {s: (1 + 0.1 * torch.randn(128, generator=g)).to(dtype).to(dev) for s in ("img", "txt")}
        self.mlp = mlp
        # the quantised layer applies GELU(tanh) in the fc1 GEMM epilogue
        self.fused_gelu = linear is None

    def linear_ops(self, n_img: int, n_txt: int) -> float:
        h, m = self.h, self.mlp
        per_tok = 2 * h * (3 * h + h + m) + 2 * m * h
        return (n_img + n_txt) * per_tok + 2 * 2 * (6 * h) * h

    def __call__(self, img, txt, vec):
        import torch
        import torch.nn.functional as F
        h, nh = self.h, self.nh
        B = img.shape[0]
        vs = F.silu(vec)
        mods = {s: self.mod[s](vs).chunk(6, dim=-1) for s in ("img", "txt")}
        qs, ks, vv = [], [], []
        for s, x in (("txt", txt), ("img", img)):
            sh, sc, _, _, _, _ = mods[s]
            if self.fused_norm:
                qkv = self.qkv[s](x, norm=("layer", (1 + sc[0]).float(), sh[0].float(), 1e-6))
            else:
                qkv = self.qkv[s](F.layer_norm(x, (h,), eps=1e-6) * (1 + sc[:, None]) + sh[:, None])
            q, k, v = qkv.view(B, -1, 3, nh, h // nh).permute(2, 0, 3, 1, 4)
            q = F.rms_norm(q, (h // nh,), self.qn[s])
            k = F.rms_norm(k, (h // nh,), self.kn[s])
            if self.sp_group is not None:
                # the text stream's gathers run behind the image stream's
                # projection; the image stream's are waited for at once
                k = _gather_tokens(k, self.sp_group, async_op=True)
                v = _gather_tokens(v, self.sp_group, async_op=True)
            qs.append(q); ks.append(k); vv.append(v)
        if self.sp_group is not None:
            ks = [f() for f in ks]
            vv = [f() for f in vv]
        a = F.scaled_dot_product_attention(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vv, 2))
        a = a.transpose(1, 2).reshape(B, -1, h)
        nt = txt.shape[1]
        outs = []
        for s, x, att in (("txt", txt, a[:, :nt]), ("img", img, a[:, nt:])):
            _, _, g1, sh2, sc2, g2 = mods[s]
            x = x + g1[:, None] * self.proj[s](att)
            kw = {"activation": 3} if self.fused_gelu else {}
            if self.fused_norm:
                f1 = self.fc1[s](x, norm=("layer", (1 + sc2[0]).float(), sh2[0].float(), 1e-6), **kw)
            else:
                f1 = self.fc1[s](F.layer_norm(x, (h,), eps=1e-6) * (1 + sc2[:, None]) + sh2[:, None], **kw)
            if not self.fused_gelu:
                f1 = F.gelu(f1, approximate="tanh")
            x = x + g2[:, None] * self.fc2[s](f1)
            outs.append(x)
        return outs[1], outs[0]


class _QLinear8:
    """INT8 W8A8 linear with per-channel scales and rot 1024 (BASELINE
    configs[4]), through the runtime's fused prep and GEMM (random-init)."""

    def __init__(self, rt, n_out: int, n_in: int, g, dev, rot: int = 1024):
        import torch
        self.rt, self.rot, self.n_in = rt, rot, n_in
        # rotated layers store weights for the padded width (13824 -> 14336), zero past K
        n_in_p = -(-n_in // rot) * rot
        w = torch.zeros(n_out, n_in_p, dtype=torch.int8)
        w[:, :n_in] = torch.randint(-127, 128, (n_out, n_in), generator=g, dtype=torch.int8)
        self.w = w.to(dev)
        self.s = (torch.rand(n_out, generator=g) * 1e-4 + 2e-5).float().to(dev)
        self.b = (torch.randn(n_out, generator=g) * 0.02).half().to(dev)

    def __call__(self, x, activation=0):
        x2 = x.reshape(-1, x.shape[-1])
        xq, s_a, _, _ = self.rt.prep_quantize(x2, rot_size=self.rot)
        y = self.rt.gemm_a8(xq, self.w, self.s, s_a, bias=self.b, out_dtype=x.dtype, activation=activation)
        return y.reshape(*x.shape[:-1], y.shape[-1])


class WanBlock:
    """Wan-class DiT block: hidden 5120, 40 heads x 128,
    self-attention with q/k RMSNorm, cross-attention to 512 text tokens, FFN
    13824 GELU(tanh), adaLN-style modulation (shift/scale/gate for attention
    and FFN, one 6 x 5120 vector per sample, random), all linears W8A8
    per-channel with rot 1024.  Norms, modulation, GELU and attention (torch
    SDPA) run in fp16.  ``sp_group``: the sample's tokens are split over the
    group and self-attention K/V are all-gathered (as in FluxDoubleBlock)."""

    def __init__(self, rt, dev, seed=0, hidden=5120, heads=40, ffn=13824, sp_group=None):
        import torch
        g = torch.Generator().manual_seed(seed)
        self.h, self.nh, self.sp_group = hidden, heads, sp_group
        mk = lambda o, i: _QLinear8(rt, o, i, g, dev)
        self.q, self.k, self.v, self.o = (mk(hidden, hidden) for _ in range(4))
        self.cq, self.ck, self.cv, self.co = (mk(hidden, hidden) for _ in range(4))
        self.fc1, self.fc2 = mk(ffn, hidden), mk(hidden, ffn)
        self.qn = (1 + 0.1 * torch.randn(hidden, generator=g)).half().to(dev)
        self.kn = (1 + 0.1 * torch.randn(hidden, generator=g)).half().to(dev)
        self.n3 = (1 + 0.1 * torch.randn(hidden, generator=g)).half().to(dev)
        self.ffn = ffn

    def linear_ops(self, n_tok: int, n_ctx: int) -> float:
        h = self.h
        return 2 * n_tok * (6 * h * h + 2 * h * self.ffn) + 2 * n_ctx * 2 * h * h

    def __call__(self, x, ctx, mod):
        import torch
        import torch.nn.functional as F
        B, L, h = x.shape
        nh, hd = self.nh, h // self.nh
        sh1, sc1, g1, sh2, sc2, g2 = mod.chunk(6, dim=1)          # [B, 1, h] each
        y = F.layer_norm(x, (h,), eps=1e-6) * (1 + sc1) + sh1
        q = F.rms_norm(self.q(y), (h,), self.qn, eps=1e-6).view(B, L, nh, hd).transpose(1, 2)
        k = F.rms_norm(self.k(y), (h,), self.kn, eps=1e-6).view(B, L, nh, hd).transpose(1, 2)
        v = self.v(y).view(B, L, nh, hd).transpose(1, 2)
        if self.sp_group is not None:
            k, v = _gather_tokens(k, self.sp_group), _gather_tokens(v, self.sp_group)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, L, h)
        x = x + g1 * self.o(a)
        y = F.layer_norm(x, (h,), self.n3, eps=1e-6)
        Lc = ctx.shape[1]
        cq = self.cq(y).view(B, L, nh, hd).transpose(1, 2)
        ck = self.ck(ctx).view(B, Lc, nh, hd).transpose(1, 2)
        cv = self.cv(ctx).view(B, Lc, nh, hd).transpose(1, 2)
        a = F.scaled_dot_product_attention(cq, ck, cv).transpose(1, 2).reshape(B, L, h)
        x = x + self.co(a)
        y = F.layer_norm(x, (h,), eps=1e-6) * (1 + sc2) + sh2
        return x + g2 * self.fc2(self.fc1(y, activation=3))   # GELU(tanh) in the fc1 epilogue


def run_wan(args, rank: int, world: int, local_rank: int) -> None:
    """a stack of 8 Wan-class blocks, batch 2 x 32760
    video tokens, 512 text-context tokens (not specified by BASELINE; stated).
    Weak layout (default): every rank runs the whole batch-2 stack (or its
    share of the batch when world divides 2); sequence layout: the tokens of
    each sample are split over the ranks with a K/V all-gather per block.
    tokens/s = processed tokens / max-over-ranks stack time."""
    import torch
    import torch.distributed as dist
    rt = _pkg()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    seq = args.shard == "sequence" and world > 1
    L, B, n_ctx = args.wan_tokens, 2, 512
    blocks = [WanBlock(rt, dev, seed=10 + i, sp_group=dist.group.WORLD if seq else None) for i in range(args.wan_blocks)]
    g = torch.Generator().manual_seed(200 + (0 if seq else rank))
    x = torch.randn(B, L, 5120, generator=g).half()
    if seq:
        per = L // world
        x = x[:, rank * per:(rank + 1) * per]
    x = x.contiguous().to(dev)
    ctx = (torch.randn(B, n_ctx, 5120, generator=g) * 0.5).half().to(dev)
    mod = (torch.randn(B, 6, 5120, generator=g) * 0.1).half().to(dev)
    st = torch.cuda.current_stream()

    def stack(t):
        for blk in blocks:
            t = blk(t, ctx, mod)
        return t

    with torch.no_grad():
        for _ in range(args.warmup):
            stack(x)
        torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with Clocks(local_rank, world) as clk:
            _gpu_head_start()
            for i in range(args.steps):
                ev[i][0].record(st)
                stack(x)
                ev[i][1].record(st)
            torch.cuda.synchronize()
    tot = sum(e[0].elapsed_time(e[1]) for e in ev)
    vals = torch.tensor([tot], dtype=torch.float64, device=dev)
    if world > 1:
        dist.barrier()
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    if rank != 0:
        return
    ms = vals.item() / args.steps
    toks = B * L * (1 if seq else world)
    lin_rank = blocks[0].linear_ops(B * x.shape[1], B * n_ctx) * len(blocks)   # this rank's linear work
    line = {
        "metric": "wan_stack_tokens_per_s", "value": toks / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if seq else "weak", "vs_baseline": None,
        "dtype": "int8+fp16", "data": "synthetic (random-init weights)",
        "config": {"workload": f"config5 Wan stack: {len(blocks)} blocks, batch 2 x {L} tokens, hidden 5120, "
                               "40x128 heads, FFN 13824, W8A8 per-channel rot 1024; 512 text-context tokens "
                               "(not specified by BASELINE); attention fp16 SDPA",
                   "parallelism": (f"sequence-parallel x{world} (K/V all-gather)" if seq else
                                   f"token-sharded x{world} (whole batch per GPU, no collective)"),
                   "l2": "inputs far larger than L2"},
        "linear_tops": world * lin_rank / (ms * 1e-3) / 1e12,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_block(args, rank: int, world: int, local_rank: int) -> None:
    """one Flux-class double block, 4096 image + 512
    text tokens, batch 1 per GPU (token sharding across GPUs: each rank runs
    its own sample; weights replicated; no collective).  tokens/s = 4608 x
    ranks / max-over-ranks block time."""
    import torch
    import torch.distributed as dist
    rt = _pkg()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    seq = args.shard == "sequence" and world > 1
    blk = FluxDoubleBlock(rt, dev, fused_norm=not args.unfused_norm, sp_group=dist.group.WORLD if seq else None)
    g = torch.Generator().manual_seed(100 + (0 if seq else rank))
    img = torch.randn(1, 4096, 3072, generator=g).half().to(dev)
    if seq:   # one sample over all ranks: this rank's image tokens
        per = 4096 // world
        img = img[:, rank * per:(rank + 1) * per].contiguous()
    txt = torch.randn(1, 512, 3072, generator=g).half().to(dev)
    if seq:   # ... and text tokens
        pt = 512 // world
        txt = txt[:, rank * pt:(rank + 1) * pt].contiguous()
    vec = torch.randn(1, 3072, generator=g).half().to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream()
    with torch.no_grad():
        for _ in range(args.warmup):
            blk(img, txt, vec)
        torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with Clocks(local_rank, world) as clk:
            _gpu_head_start()   # after the sampler is up
            for i in range(2):   # untimed: the first steps after an idle GPU run slow
                flush.fill_(float(i))
                blk(img, txt, vec)
            for i in range(args.steps):
                flush.fill_(float(i))
                ev[i][0].record(st)
                blk(img, txt, vec)
                ev[i][1].record(st)
            torch.cuda.synchronize()
    tot = sum(e[0].elapsed_time(e[1]) for e in ev)
    vals = torch.tensor([tot], dtype=torch.float64, device=dev)
    if world > 1:
        dist.barrier()
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    if rank != 0:
        return
    ms = vals.item() / args.steps
    n_tok = 4096 + 512
    lin = blk.linear_ops(4096, 512)
    attn = 4 * n_tok * n_tok * 3072
    line = {
        "metric": "flux_double_block_tokens_per_s", "value": (1 if seq else world) * n_tok / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if seq else "weak", "vs_baseline": None, "dtype": "int8+fp16",
        "data": "synthetic (random-init weights)",
        "config": {"workload": "config4 Flux double block: 4096 img + 512 txt tokens, hidden 3072, 24x128 heads, "
                               "MLP 12288, all linears INT4 W4A8 g128 rot256 perm; attention fp16 SDPA",
                   "norm": "torch ops" if args.unfused_norm else "LayerNorm + adaLN modulation fused into prep",
                   "parallelism": (f"sequence-parallel x{world}: one sample, image and text tokens split, "
                                   "K/V all-gather (NCCL)") if seq else
                                  f"token-sharded x{world} (one sample per GPU, no collective)",
                   "l2": "flushed (256 MB write) between timed steps"},
        "linear_tops": (1 if seq else world) * lin / (ms * 1e-3) / 1e12, "attn_tflop_per_step": attn / 1e12,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def kernel_probe(which: str) -> None:
    """Three launches of one kernel of the config-2 step (for ncu captures)."""
    import torch
    rt = _pkg()
    dev = torch.device("cuda")
    d = make_inputs(device=dev)
    perm32 = d["perm"].to(torch.int32)
    w_rep = rt.repack_int4(d["packed"], K, 0)
    s_w = d["scale"].float()
    xq, s_a, _, _ = rt.prep_quantize(d["x"], smoothrot=d["smoothrot"], rot_size=ROT, w_in=K, perm=perm32)
    torch.cuda.synchronize()
    for _ in range(3):
        if which == "prep":
            rt.prep_quantize(d["x"], smoothrot=d["smoothrot"], rot_size=ROT, w_in=K, perm=perm32)
        else:
            rt.gemm_a8(xq, w_rep, s_w, s_a, bias=d["bias"], out_dtype=torch.float16, group_size=GS, repacked=True)
    torch.cuda.synchronize()
    assert rt.device_error() == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--unfused-norm", action="store_true",
                    help="flux_block: LayerNorm + modulation as separate torch ops instead of in the prep kernel")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the configs[0] / configs[2] measurements added to the N=1 line")
    ap.add_argument("--workload", choices=["linear", "flux_block", "wan_stack"], default="linear",
                    help="linear: BASELINE configs[1] (default); flux_block: configs[3]; wan_stack: configs[4]")
    ap.add_argument("--wan-tokens", type=int, default=32760, help="wan_stack: tokens per sample")
    ap.add_argument("--wan-blocks", type=int, default=8, help="wan_stack: blocks in the stack")
    ap.add_argument("--shard", choices=["tokens", "features", "sequence"], default="tokens",
                    help="tokens: every rank runs its own tokens / sample (default); "
                         "features: one layer split by output features + all-gather; "
                         "sequence (flux_block): one sample split by image tokens + K/V all-gather")
    ap.add_argument("--kernel-probe", choices=["prep", "gemm"], default=None,
                    help="run only this kernel of the step (3 launches) for profiling; prints nothing")
    args = ap.parse_args()
    if args.kernel_probe:
        kernel_probe(args.kernel_probe)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    try:
        if args.workload == "flux_block":
            run_block(args, rank, world, local_rank)
        elif args.workload == "wan_stack":
            run_wan(args, rank, world, local_rank)
        else:
            (run_features if args.shard == "features" else run_gpu)(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
