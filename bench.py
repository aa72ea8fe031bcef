"""Benchmark of the B200 VC-attention path (driver contract: one JSON line).

Workload (default): non-causal BNSD [1,28,37741,128] bf16,
Q,K ~ N(0,1) with a K channel mean ~ N(0,3), V ~ N(0,1), ExpCast on,
smoothing off; synthetic, seeded per (b,h) head so shards are slices of the
single-GPU tensors.  A step is one full ``sageattn_vc`` call: INT8 Q/K + FP8 V
preparation and the fused attention kernel, inputs resident in HBM (the
811 MB of inputs exceed the 126 MB L2, so no flush is needed).

  value  = 4*B*H*S^2*D / t_step  (TOPS, all ranks, max-over-ranks device time)
  e2e    = same metric through the public API with pinned host buffers:
           H2D of the inputs + the call + D2H of the output every step
  roofline: the fused attention kernel, CUDA-event timed inside the region
  cpu_baseline: the reference's own CPU path (its Config API reference
           backend, installed unmodified under baseline/_ref; else the CPU
           oracle of this path) on a bounded sample, extrapolated linearly

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]
Multi-GPU: torchrun --nproc-per-node N bench.py --gpus N (units split across
ranks; no collective in the timed region).
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
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "cake-opt-vc_attention_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

CONFIGS = {
    # name: B, H, S, D, dtype, k_mean_std, v_smooth, description
    "c2": (1, 28, 37741, 128, torch.bfloat16, 3 ** 0.5, False,
           "BNSD [1,28,37741,128] bf16, ExpCast on, smoothing off"),
    "c3": (1, 28, 37741, 128, torch.bfloat16, 3 ** 0.5, True,
           "BNSD [1,28,37741,128] bf16, ExpCast + V grouping + 128-token block smoothing"),
    "c4": (2, 24, 16384, 64, torch.bfloat16, 3 ** 0.5, False,
           "BNSD [2,24,16384,64] bf16 D64, ExpCast on, 1% of Q/K entries x20"),
    "c5": (2, 40, 75600, 128, torch.bfloat16, 3 ** 0.5, True,
           "BNSD [2,40,75600,128] bf16, V ~ N(0,1), ExpCast + V grouping + block smoothing"),
}
METRIC = "TOPS (4*B*H*S^2*D per call) at BNSD [1,28,37741,128] D128, sageattn_vc ExpCast (prep + fused kernel)"
# DRAM bytes (read + write) of one full config-2 launch of the paired-tile kernel, from ncu
# (profiles/vc_attention_pair_kernel_c2_dram.txt)
TRAFFIC_C2_BYTES = 647.7e6


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# per-config input distributions beyond the CONFIGS tuple (BASELINE's config definitions):
# c3 draws V from a 16-centroid mixture; c4 scales 1% of the Q/K entries by 20
GEN = {"c2": {}, "c3": {"v_mixture": True}, "c4": {"outliers": 0.01}, "c5": {}}


def gen_head(bh: int, S: int, D: int, dtype, k_std: float, smooth: bool, device, seed: int = 0,
             outliers: float = 0.0):
    """Seeded synthetic Q,K,V for one flattened (b,h) head: Q ~ N(0,1), K ~ N(0,1)
    plus a per-channel offset ~ N(0, k_std^2); V ~ N(0,1), or with ``smooth`` a
    16-centroid mixture (centroids ~ N(0,2), within-cluster std 0.3).
    ``outliers``: that fraction of the Q and K entries (Bernoulli mask from the
    same generator) is multiplied by 20."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000003 + bh)
    q = torch.randn(S, D, generator=g, device=device)
    k = torch.randn(S, D, generator=g, device=device) + torch.randn(D, generator=g, device=device) * k_std
    if smooth:
        cent = torch.randn(16, D, generator=g, device=device) * 2 ** 0.5
        lab = torch.randint(0, 16, (S,), generator=g, device=device)
        v = cent[lab] + 0.3 * torch.randn(S, D, generator=g, device=device)
    else:
        v = torch.randn(S, D, generator=g, device=device)
    if outliers > 0:
        for x in (q, k):
            mask = torch.rand(S, D, generator=g, device=device) < outliers
            x[mask] *= 20.0
    return q.to(dtype), k.to(dtype), v.to(dtype)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms with host
    timestamps.  ``start()`` waits for the first sample so that sampling is
    live before the timed region; ``mark(t0, t1)`` records the timed region's
    host-time window.  The summary uses the samples inside that window, and
    when it is shorter than three sample periods, the window from the start
    of the warm-up (same kernels, same load) as well, saying which."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.samples = []          # (host time, csv line)
        self.window = None
        self.t_warm = None

    def start(self, wait_s: float = 10.0):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t_end = time.time() + wait_s
        while not self.samples and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.01)
        self.t_warm = time.time()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self):
        if self.proc is not None:
            time.sleep(0.15)       # let the sample that covers the window's end arrive
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    @staticmethod
    def _parse(lines):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return sm, mx, reasons

    def summary(self):
        if not self.window:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        t0, t1 = self.window
        period = 0.1
        inside = [ln for t, ln in self.samples if t0 <= t <= t1 + period]
        scope = "timed region"
        if len(inside) < 3 and self.t_warm is not None:
            inside = [ln for t, ln in self.samples if self.t_warm <= t <= t1 + period]
            scope = "warm-up + timed region (timed region alone is under 3 sample periods)"
        sm, mx, reasons = self._parse(inside)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "scope": scope}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "scope": scope}


REF_ROOT = REPO / "baseline" / "_ref"


def _reference_core():
    """The reference package installed unmodified under baseline/_ref (pure
    Python, VC_ATTENTION_BUILD_CUDA=0), or None when it is absent."""
    if not (REF_ROOT / "vc_attention" / "core.py").exists():
        return None
    if str(REF_ROOT) not in sys.path:
        sys.path.insert(0, str(REF_ROOT))
    from vc_attention import core
    if not str(Path(core.__file__).resolve()).startswith(str(REF_ROOT.resolve())):
        return None          # another vc_attention shadows the reference install
    return core


def cpu_baseline_sample(B, H, S, D, dtype, k_std, smooth, threads=None, gen=None):
    """Time the reference's CPU path on a bounded sample and extrapolate
    linearly to the full workload.

    With the reference installed under baseline/_ref ("reference"): its own
    public API, ``vc_attention.core.attention(q, k, v, Config(backend=
    "reference", expcast=True, v_smooth=...))`` (E4M3 encode/decode with FP32
    matmul emulation, the numerical contract the north star names), on head 0
    with 128 and 1024 sampled query rows against all keys (after one untimed
    warm-up call); the two sizes give the per-call fixed cost (K/V
    preparation) and the per-row cost.
    Otherwise ("port"): the CPU oracle of this path (one head's INT8/FP8
    preparation plus 128 query rows through the decoded-payload reference)."""
    if threads:
        torch.set_num_threads(threads)
    gen = gen or {}
    q, k, v = gen_head(0, S, D, dtype, k_std, gen.get("v_mixture", False), "cpu", outliers=gen.get("outliers", 0.0))
    q, k, v = (x.reshape(1, 1, S, D) for x in (q, k, v))
    ops_full = 4.0 * B * H * S * S * D
    core = _reference_core()
    if core is not None:
        cfg = core.Config(backend="reference", expcast=True, v_smooth=smooth)
        qf, kf, vf = q.float(), k.float(), v.float()
        times = {}
        core.attention(qf[:, :, :16], kf, vf, cfg)      # warm-up: thread pool, allocator
        for n in (128, 1024):
            rows = torch.linspace(0, S - 1, n).round().long()
            t0 = time.perf_counter()
            core.attention(qf[:, :, rows], kf, vf, cfg)
            times[n] = time.perf_counter() - t0
        per_row = max((times[1024] - times[128]) / 896.0, 1e-12)
        fixed = max(times[128] - 128 * per_row, 0.0)
        t_full = B * H * (fixed + per_row * S)
        return {"value": ops_full / t_full / 1e12, "unit": "TOPS", "cores": torch.get_num_threads(),
                "kind": "reference", "extrapolated": True,
                "sample": f"reference vc_attention.core.attention (baseline/_ref, unmodified) with "
                          f"Config(backend='reference', expcast=True, v_smooth={smooth}) on head 0: 128 rows x {S} keys "
                          f"{times[128]:.2f}s, 1024 rows {times[1024]:.2f}s -> fixed {fixed:.2f}s + {per_row*1e3:.2f} ms/row, "
                          f"extrapolated linearly to {B*H} heads x {S} rows",
                "seconds_extrapolated": t_full}
    from oracle import vc_oracle as O
    t0 = time.perf_counter()
    st = O.prepare(q, k, v, expcast=True, v_smooth=smooth, km=O.k_mean(k))
    t_prep = time.perf_counter() - t0
    rows = torch.arange(0, S, max(1, S // 128))[:128]
    t0 = time.perf_counter()
    O.reference(st, query_indices=rows, chunk=128)
    t_ref = time.perf_counter() - t0
    t_full = B * H * (t_prep + t_ref * (S / rows.numel()))
    return {"value": ops_full / t_full / 1e12, "unit": "TOPS", "cores": torch.get_num_threads(), "kind": "port",
            "extrapolated": True,
            "sample": f"CPU oracle: head-0 prep ({t_prep:.2f}s) + {rows.numel()} query rows x {S} keys "
                      f"({t_ref:.2f}s), extrapolated linearly to {B*H} heads x {S} rows",
            "seconds_extrapolated": t_full}


def config_dict(desc, B, H, S, D, smooth, world):
    """The ``config`` object both arms print (same keys and values)."""
    return {"workload": desc, "B": B, "H": H, "S": S, "D": D, "expcast": True, "v_smooth": smooth,
            "parallelism": f"units split over {world} rank(s), outputs sharded",
            "l2": "inputs (811 MB) exceed the 126 MB L2; no flush needed"}


def run_reference(args, cfg):
    """--impl reference: the reference's own CPU path on the host cores
    (rank 0 only; other ranks exit without work)."""
    B, H, S, D, dtype, k_std, smooth, desc = cfg
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline_sample(B, H, S, D, dtype, k_std, smooth, threads, GEN[args.config])
        if i >= args.warmup:
            vals.append(r)
    value = statistics.median(v["value"] for v in vals)
    ms = 4.0 * B * H * S * S * D / (value * 1e12) * 1e3
    line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32 (E4M3 encode/decode emulation on the CPU)", "data": "synthetic",
            "config": config_dict(desc, B, H, S, D, smooth, args.gpus), "impl": "reference",
            "extrapolated": True,
            "note": "each step times a bounded sample of the workload on the host cores; ms_per_step and value "
                    "are that sample extrapolated linearly to the full call (see cpu_baseline.sample)",
            "cpu_baseline": {**vals[-1], "value": value},
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", choices=tuple(CONFIGS), default="c2")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", action="store_true", help="also time the optional NCCL all-gather of outputs")
    ap.add_argument("--shape", default=None, help="B,H,S,D override of the config shape (profiling cases)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.shape:
        b_, h_, s_, d_ = (int(x) for x in args.shape.split(","))
        cfg = (b_, h_, s_, d_, *cfg[4:7], f"BNSD [{b_},{h_},{s_},{d_}] ({args.config} settings)")
    if args.impl == "reference":
        run_reference(args, cfg)
        return
    B, H, S, D, dtype, k_std, smooth, desc = cfg
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from vc_b200 import ops, parallel
    from vc_b200 import _native
    _native.load()
    sh = parallel.shard(B, H, S, world, rank)
    nbh = sh.bh_end - sh.bh_begin
    # this rank's heads, generated on the device
    qh, kh, vh = [], [], []
    for bh in range(sh.bh_begin, sh.bh_end):
        a, b_, c = gen_head(bh, S, D, dtype, k_std, GEN[args.config].get("v_mixture", False), dev,
                            outliers=GEN[args.config].get("outliers", 0.0))
        qh.append(a), kh.append(b_), vh.append(c)
    q = torch.stack(qh).reshape(1, nbh, S, D)
    k = torch.stack(kh).reshape(1, nbh, S, D)
    v = torch.stack(vh).reshape(1, nbh, S, D)
    del qh, kh, vh
    # a Shard relative to the local head block
    local_shard = parallel.Shard(0, 1, sh.unit_begin - sh.bh_begin * sh.qtiles,
                                 sh.unit_end - sh.bh_begin * sh.qtiles, 0, nbh, sh.qtiles)
    from sageattention_local.vc import prepare
    out = torch.empty((1, nbh, S, D), dtype=dtype, device=dev)
    mean_numel = (B * H * D, B * H * S * D)
    att_events = []

    def step(record=False):
        st = prepare(q, k, v, expcast=True, v_smooth=smooth, mean_numel=mean_numel)
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], st["means"], out=out,
                          sm_scale=st["scale"], expcast=True, block_values=smooth,
                          unit_range=local_shard.local_units)
        if record:
            e1.record()
            att_events.append((e0, e1))

    clocks = ClockSampler(local).start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    h0 = time.time()
    t0.record()
    for _ in range(args.steps):
        step(record=True)
    t1.record()
    torch.cuda.synchronize()
    clocks.mark(h0, time.time())
    clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    att_ms = statistics.mean(a.elapsed_time(b) for a, b in att_events)
    if dist:
        tt = torch.tensor([ms, att_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, att_ms = tt.tolist()
    ops_total = 4.0 * B * H * S * S * D
    value = ops_total / (ms * 1e-3) / 1e12
    err = ops.error_word(local, clear=True)
    if err:
        raise RuntimeError(f"device error word {err:#x} after the timed region")

    # roofline of the fused attention kernel (this rank's launch)
    rows_local = sum(min(128, S - (u % sh.qtiles) * 128) for u in range(sh.unit_begin, sh.unit_end))
    ops_launch = 4.0 * rows_local * S * D
    hbm, bf16, bf16_sus, basis = peaks()
    # dense INT8 rate of this GPU, measured now by this library's own probe (tcgen05 kind::i8,
    # A in tensor memory, N=256: the fastest form); the peak is the lower of it and 2 x bf16
    i8 = ops.tensor_peak("i8", 256, iters=20000, a_tmem=True)
    peak_tops = min(i8["tops"], 2.0 * bf16)
    achieved = ops_launch / (att_ms * 1e-3) / 1e12
    # DRAM bytes per launch: dram__bytes_read.sum + dram__bytes_write.sum of the paired-tile kernel
    # from one ncu capture of the full config-2 launch (profiles/vc_attention_pair_kernel_c2_dram.txt),
    # scaled by the heads in this launch; D128, ExpCast, channel-scaled V.
    traffic = None
    if D == 128 and not smooth and S == 37741:
        traffic = TRAFFIC_C2_BYTES / 28 * nbh
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    plan = ops.attention_plan(sh.qtiles, local_shard.local_units, sms)
    kernel = "vc_attention_pair_kernel"
    if plan["tail_units"]:
        kernel = (f"vc_attention_pair_kernel ({plan['pairs']} pairs) + vc_attention_alt_kernel "
                  f"({plan['tail_units']} tail tiles), one event pair around both")
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tops, "unit": "TFLOP/s",
                "frac": achieved / peak_tops, "traffic": traffic, "kernel": kernel,
                "peak_basis": (f"min(measured dense INT8 {i8['tops']:.1f} TOPS [vc_tensor_peak: tcgen05 kind::i8, "
                               f"A in tensor memory, N=256, this run], 2 x bf16_tflops {2.0 * bf16:.1f} "
                               f"[{basis}, MEASURED_PEAKS.json])"),
                "peak_i8_measured": i8["tops"], "frac_of_i8_measured": achieved / i8["tops"],
                "kernel_ms": att_ms, "algorithmic_ops_per_launch": ops_launch}

    # end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hout = torch.empty((1, nbh, S, D), dtype=dtype).pin_memory()

        def e2e_step():
            if world == 1:
                # public host-tensor API: per-head-chunk copies overlapped with the computation
                from vc_b200.pipeline import sageattn_vc_host
                sageattn_vc_host(hq, hk, hv, hout, device=dev, v_smooth=smooth)
            else:
                # this rank's unit range on its host-resident heads, copies overlapped the same way
                from vc_b200.pipeline import sharded_attention_host
                sharded_attention_host(hq, hk, hv, hout, local_shard.local_units, device=dev,
                                       mean_numel=mean_numel, v_smooth=smooth)

        # the host link alone: one pinned-host -> device copy of the inputs and one
        # device -> pinned-host copy of the output, the floor for the end-to-end time
        link = {}
        dq_l = torch.empty_like(q)
        for name, fn, nbytes in (("h2d_gbs", lambda: [d.copy_(h, non_blocking=True) for d, h in
                                                      ((dq_l, hq), (dq_l, hk), (dq_l, hv))],
                                  3 * q.numel() * q.element_size()),
                                 ("d2h_gbs", lambda: hout.copy_(dq_l.view(hout.shape), non_blocking=True),
                                  q.numel() * q.element_size())):
            fn()
            torch.cuda.synchronize()
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record()
            fn()
            l1.record()
            torch.cuda.synchronize()
            link[name] = nbytes / (l0.elapsed_time(l1) * 1e-3) / 1e9
        del dq_l
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        n_e2e = max(3, min(args.steps, 5))
        for _ in range(n_e2e):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / n_e2e
        if dist:
            tt = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_ms = tt.item()
        e2e = {"value": ops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 3 * nbh * S * D * q.element_size(),
               "d2h_bytes_per_step": nbh * S * D * q.element_size(),
               "path": ("vc_b200.pipeline.sageattn_vc_host on pinned-host inputs (head chunks, copies overlapped)"
                        if world == 1 else
                        "vc_b200.pipeline.sharded_attention_host per rank on pinned-host inputs (head chunks, copies overlapped)"),
               "link_gbs_measured": link}

    gather_ms = None
    if args.gather and dist:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        parallel.gather_rows(out, sh, B, H, S)
        e1.record()
        torch.cuda.synchronize()
        gather_ms = e0.elapsed_time(e1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(B, H, S, D, dtype, k_std, smooth, gen=GEN[args.config])

    if rank == 0:
        # this library's kernels per step: K sums + mean finalize, Q/K tiles, then V channel amax +
        # quantise (no smoothing) or grouping (init, 2 assignments, update, histogram, scan, scatter)
        # + block stats, channel scales, quantise; then the fused attention kernel (the paired-tile
        # kernel, plus the alternating-tile kernel for a short last wave)
        launches_per_step = (2 + 1 + 2) if not smooth else (2 + 1 + 7 + 3)
        launches_per_step += plan["launches"]
        line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8 QK / e4m3 PV (fp32 accumulate), bf16 I/O",
                "data": "synthetic (seeded per head on device)",
                "config": config_dict(desc, B, H, S, D, smooth, world),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
                "gpu_launches": launches_per_step * args.steps, "attention_ms": att_ms}
        if gather_ms is not None:
            line["allgather_ms"] = gather_ms
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
