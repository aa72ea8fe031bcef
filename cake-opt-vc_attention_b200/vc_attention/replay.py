"""Same-input numerical replay of the four VC arms on the sm100a backend.

What it does (the reference's replay contract, src/vc_attention/replay.py:
17-160): the arms ``fp8_control`` (plain FP8), ``expcast``, ``v_smooth`` and
``combined`` run on identical Q/K/V -- a capture written by the LightX2V
layer, or seeded synthetic tensors -- keeping every K/V token even when only
a window of queries is replayed, and each is compared with an exact FP32
result on the same values.  The report records error metrics and timings.

How it is built here: a ``ReplayCase`` holds the inputs and their
provenance; ``exact_attention`` is FP32 dense attention on the GPU, chunked
over queries; each arm is one ``Config(backend="sm100a")`` call through the
public ``attention`` API, timed with CUDA events around the whole call
(preparation included) in an order that alternates between repeats; the
MindIE baselines of the reference exist only on Ascend NPUs and are not
offered.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import platform
import statistics
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch

from .core import Config, attention

# arm name -> (V smoothing, ExpCast): the experiment's four arms
ARMS = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False), "combined": (True, True)}


@dataclass
class ReplayCase:
    q: torch.Tensor          # [B, H, Sq, D]
    k: torch.Tensor          # [B, H, Sk, D]
    v: torch.Tensor
    scale: float
    source: dict = field(default_factory=dict)

    def query_window(self, start: int, limit: int) -> "ReplayCase":
        """Only queries [start, start + limit) (limit 0 = to the end); every
        K/V token is kept, so each replayed row sees its full context."""
        n = self.q.shape[-2]
        if start < 0 or start % 128 or start >= n:
            raise ValueError(f"query window start {start} must be a multiple of 128 inside [0, {n})")
        end = n if limit == 0 else min(n, start + limit)
        return ReplayCase(self.q[..., start:end, :], self.k, self.v, self.scale,
                          {**self.source, "query_range": [start, end]})


def load_capture(path) -> ReplayCase:
    """A capture file of the LightX2V layer: BNSD ``q``/``k``/``v`` and
    ``metadata`` (its ``scale`` is the softmax scale of the captured call)."""
    path = Path(path)
    rec = torch.load(path, map_location="cpu", weights_only=True)
    meta = rec["metadata"]
    digest = hashlib.sha256(path.read_bytes()).hexdigest()
    return ReplayCase(rec["q"], rec["k"], rec["v"], float(meta["scale"]),
                      {"kind": "captured_qkv", "file": str(path.resolve()), "sha256": digest, "metadata": meta})


def synthetic(tokens: int, heads: int, dim: int, seed: int, clustered: bool) -> ReplayCase:
    """Seeded CPU inputs: Q, K ~ N(0, 1); V ~ N(0, 1), or with ``clustered``
    a mixture around 8 well-separated centres per head (the token-level
    structure V grouping exploits)."""
    g = torch.Generator().manual_seed(seed)
    shape = (1, heads, tokens, dim)
    q = torch.randn(shape, generator=g)
    k = torch.randn(shape, generator=g)
    if clustered:
        centres = 6.0 * torch.randn((1, heads, 8, dim), generator=g)
        member = torch.randint(0, 8, (1, heads, tokens), generator=g)
        v = torch.take_along_dim(centres, member[..., None], dim=2) + 0.2 * torch.randn(shape, generator=g)
    else:
        v = torch.randn(shape, generator=g)
    kind = "synthetic_clustered" if clustered else "synthetic_gaussian"
    return ReplayCase(q, k, v, dim ** -0.5, {"kind": kind, "seed": seed})


@torch.no_grad()
def exact_attention(q, k, v, scale: float, chunk: int = 1024) -> torch.Tensor:
    """FP32 softmax(Q K^T scale) V, computed over query chunks of ``chunk`` rows."""
    q, k, v = (x.float() for x in (q, k, v))
    kt = k.transpose(-1, -2)
    parts = [torch.softmax((q[..., s:s + chunk, :] @ kt) * scale, dim=-1) @ v for s in range(0, q.shape[-2], chunk)]
    return torch.cat(parts, dim=-2)


def metrics(actual: torch.Tensor, exact: torch.Tensor) -> dict:
    """Error of ``actual`` against ``exact`` in float64: RMSE, RMSE relative
    to the exact result's RMS, largest absolute error, cosine similarity."""
    a, e = actual.double().flatten(), exact.double().flatten()
    if not torch.isfinite(a).all():
        raise ValueError("Nonfinite values in the attention output")
    err = a - e
    rms_err, rms_ref = err.square().mean().sqrt().item(), e.square().mean().sqrt().item()
    cos = (a @ e / (a.norm() * e.norm()).clamp_min(1e-300)).item()
    return {"rmse": rms_err, "relative_rmse": rms_err / max(rms_ref, 1e-300), "max_abs": err.abs().max().item(),
            "cosine": cos}


def arm_configs(*, clusters: int = 8, iterations: int = 2, hadamard: bool = False) -> dict:
    """The sm100a Config of each arm: INT8 Q/K, or with ``hadamard`` the
    Config contract's Hadamard E4M3 block Q/K."""
    return {name: Config(v_smooth=smooth, expcast=cast, backend="sm100a", clusters=clusters, iterations=iterations,
                         qk_hadamard=bool(hadamard))
            for name, (smooth, cast) in ARMS.items()}


def _timed(fn, device) -> tuple[torch.Tensor, float]:
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    start.record(stream)
    out = fn()
    stop.record(stream)
    stop.synchronize()
    return out, start.elapsed_time(stop)


def run(args) -> dict:
    device = torch.device(args.device)
    if device.type != "cuda":
        raise ValueError("the sm100a replay needs a CUDA device (there is no CPU path)")
    case = load_capture(args.capture) if args.capture else \
        synthetic(args.tokens, args.heads, args.dim, args.seed, args.clustered)
    case = case.query_window(args.q_start, args.q_limit)
    q, k, v = (x.float().to(device) for x in (case.q, case.k, case.v))
    exact = exact_attention(q, k, v, case.scale)
    configs = arm_configs(clusters=args.clusters, iterations=args.iterations, hadamard=args.hadamard)

    def call(cfg):
        return attention(q, k, v, cfg, scale=case.scale)[0]

    for _ in range(args.warmup):
        for cfg in configs.values():
            call(cfg)
    names = list(configs)
    times = {n: [] for n in names}
    errors = {}
    for r in range(args.repeats):
        for n in (names if r % 2 == 0 else names[::-1]):
            out, ms = _timed(lambda: call(configs[n]), device)
            times[n].append(ms)
            errors[n] = metrics(out, exact)
    report = {
        "status": "exploratory", "source": case.source, "device": str(device),
        "device_name": torch.cuda.get_device_name(device), "torch": torch.__version__, "host": platform.platform(),
        "shape_q": list(q.shape), "shape_k": list(k.shape), "scale": case.scale,
        "query_range": case.source.get("query_range"), "full_kv_context": True,
        "reference": "FP32 dense attention on the same input values (GPU)",
        "timing": "CUDA events around each public attention call (preparation included), alternating arm order",
        "warmup": args.warmup, "repeats": args.repeats,
        "arms": {n: {"metrics": errors[n], "wall_ms": times[n], "median_ms": statistics.median(times[n]),
                     "config": asdict(configs[n])} for n in names},
    }
    out_path = Path(args.output)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(json.dumps(report, indent=2, allow_nan=False) + "\n", encoding="utf-8")
    return report


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="Replay the four VC arms on one Q/K/V input (sm100a backend)")
    ap.add_argument("--capture", help="a capture .pt written by the LightX2V layer (else synthetic input)")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--hadamard", action="store_true", help="the arms on the Hadamard E4M3 block Q/K path")
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=2)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--clustered", action="store_true")
    ap.add_argument("--clusters", type=int, default=8)
    ap.add_argument("--iterations", type=int, default=2)
    ap.add_argument("--q-start", type=int, default=0)
    ap.add_argument("--q-limit", type=int, default=0, help="queries to replay (0 = all); K/V always complete")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--output", required=True)
    return ap


def main(argv=None):
    report = run(parser().parse_args(argv))
    print(json.dumps({n: row["metrics"] for n, row in report["arms"].items()}, indent=2))


if __name__ == "__main__":
    main()
