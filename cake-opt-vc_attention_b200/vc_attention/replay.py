"""Same-input numerical replay of the four Config arms on the sm100a backend.

Mirrors the reference's replay (src/vc_attention/replay.py:17-160): the arms
``fp8_control``, ``expcast``, ``v_smooth`` and ``combined`` run on the same
Q/K/V -- a capture written by the model adapter, or seeded synthetic
tensors -- and are compared with an exact FP32 result on the same values,
with wall times.  Differences from the reference, for this backend:
  * the exact result is FP32 dense softmax attention on the GPU (the
    reference's FP32 streaming path has no GPU form here; the two differ only
    in FP32 rounding);
  * the arms run ``Config(backend="sm100a")``.  Arms without ExpCast use the
    INT8 Q/K path; with ``hadamard=True`` the ExpCast arms use the Config
    contract's own Hadamard + E4M3 block Q/K instead;
  * the MindIE baselines exist only on Ascend NPUs and are not offered.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import platform
import statistics
import time
from dataclasses import asdict
from pathlib import Path

import torch

from .core import Config, attention

ARMS = {"fp8_control": (False, False), "expcast": (False, True), "v_smooth": (True, False), "combined": (True, True)}


def metrics(actual: torch.Tensor, reference: torch.Tensor) -> dict:
    """RMSE, relative RMSE, max |error| and cosine of ``actual`` against
    ``reference`` in FP64 (replay.py:20-32 keys); non-finite output raises."""
    x, ref = actual.double(), reference.double()
    if not bool(torch.isfinite(x).all()):
        raise ValueError("Nonfinite attention output")
    delta = x - ref
    mse = delta.square().mean().item()
    energy = ref.square().mean().item()
    return {
        "rmse": math.sqrt(mse),
        "relative_rmse": math.sqrt(mse / max(energy, 1e-30)),
        "max_abs": delta.abs().max().item(),
        "cosine": torch.nn.functional.cosine_similarity(x.flatten(), ref.flatten(), dim=0).item(),
    }


def synthetic(tokens: int, heads: int, dim: int, seed: int, clustered: bool):
    """Seeded BNSD [1, heads, tokens, dim] Q/K/V (replay.py:42-49): N(0,1),
    with ``clustered`` V drawn around 8 centres (scale 8) plus 0.1 noise."""
    generator = torch.Generator().manual_seed(seed)
    q, k, v = [torch.randn((1, heads, tokens, dim), generator=generator) for _ in range(3)]
    if clustered:
        centers = torch.randn((1, heads, 8, dim), generator=generator) * 8
        ids = torch.randint(0, 8, (1, heads, tokens, 1), generator=generator).expand_as(v)
        v = centers.gather(-2, ids) + 0.1 * v
    return q, k, v


@torch.no_grad()
def exact_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, chunk: int = 1024):
    """FP32 dense softmax(Q K^T * scale) V, chunked over queries."""
    q, k, v = (x.float() for x in (q, k, v))
    out = torch.empty((*q.shape[:-1], v.shape[-1]), dtype=torch.float32, device=q.device)
    for s in range(0, q.shape[-2], chunk):
        logits = (q[..., s:s + chunk, :] @ k.transpose(-1, -2)) * scale
        out[..., s:s + chunk, :] = torch.softmax(logits, dim=-1) @ v
    return out


def arm_configs(*, clusters: int = 8, iterations: int = 2, hadamard: bool = False) -> dict:
    return {name: Config(v_smooth=smooth, expcast=cast, backend="sm100a", clusters=clusters, iterations=iterations,
                         qk_hadamard=bool(hadamard and cast))
            for name, (smooth, cast) in ARMS.items()}


def load_capture(path: str | Path):
    """Q/K/V, scale and provenance of a capture file written by the adapter."""
    path = Path(path)
    record = torch.load(path, map_location="cpu", weights_only=True)
    q, k, v = [record[name] for name in ("q", "k", "v")]
    source = {"kind": "captured_qkv", "file": str(path.resolve()),
              "sha256": hashlib.sha256(path.read_bytes()).hexdigest(), "metadata": record["metadata"]}
    return q, k, v, record["metadata"]["scale"], source


def run(args) -> dict:
    device = torch.device(args.device)
    if device.type != "cuda":
        raise ValueError("the sm100a replay runs on a CUDA device; no CPU path")
    if args.capture:
        q, k, v, scale, source = load_capture(args.capture)
    else:
        q, k, v = synthetic(args.tokens, args.heads, args.dim, args.seed, args.clustered)
        source = {"kind": "synthetic_clustered" if args.clustered else "synthetic_gaussian", "seed": args.seed}
        scale = args.dim ** -0.5
    if args.q_start % 128 or args.q_start >= q.shape[-2]:
        raise ValueError("q-start must be a valid 128-token block boundary")
    end = q.shape[-2] if args.q_limit == 0 else min(q.shape[-2], args.q_start + args.q_limit)
    # every K/V token stays: a cropped context would not be the same attention
    q = q[..., args.q_start:end, :]
    q, k, v = [x.float().to(device) for x in (q, k, v)]
    exact = exact_attention(q, k, v, scale)
    configs = arm_configs(clusters=args.clusters, iterations=args.iterations, hadamard=args.hadamard)
    calls = {name: (lambda cfg=cfg: attention(q, k, v, cfg, scale=scale)[0]) for name, cfg in configs.items()}
    for _ in range(args.warmup):
        for call in calls.values():
            call()
    times = {name: [] for name in calls}
    errors = {}
    for repeat in range(args.repeats):
        order = list(calls) if repeat % 2 == 0 else list(reversed(calls))
        for name in order:
            torch.cuda.synchronize(device)
            start = time.perf_counter()
            result = calls[name]()
            torch.cuda.synchronize(device)
            times[name].append((time.perf_counter() - start) * 1000)
            errors[name] = metrics(result.float(), exact)
    report = {
        "status": "exploratory",
        "source": source,
        "device": str(device),
        "device_name": torch.cuda.get_device_name(device),
        "torch": torch.__version__,
        "host": platform.platform(),
        "shape_q": list(q.shape),
        "shape_k": list(k.shape),
        "scale": scale,
        "query_range": [args.q_start, end],
        "reference": "FP32 dense attention on the same input values (GPU)",
        "full_kv_context": True,
        "warmup": args.warmup,
        "repeats": args.repeats,
        "scope": "isolated attention; smoothing active; regrouping included on every measured call",
        "warning": "Wall times are host-timed calls of the public API (preparation included), not kernel times.",
        "arms": {name: {"metrics": errors[name], "wall_ms": times[name], "median_ms": statistics.median(times[name]),
                        "config": asdict(configs[name])} for name in calls},
    }
    output = Path(args.output)
    output.parent.mkdir(parents=True, exist_ok=True)
    output.write_text(json.dumps(report, indent=2, allow_nan=False) + "\n", encoding="utf-8")
    return report


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--capture")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--hadamard", action="store_true", help="ExpCast arms on the Hadamard E4M3 block Q/K path")
    ap.add_argument("--tokens", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=2)
    ap.add_argument("--dim", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--clustered", action="store_true")
    ap.add_argument("--clusters", type=int, default=8)
    ap.add_argument("--iterations", type=int, default=2)
    ap.add_argument("--q-start", type=int, default=0)
    ap.add_argument("--q-limit", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--output", required=True)
    return ap


def main(argv=None):
    report = run(parser().parse_args(argv))
    print(json.dumps({name: row["metrics"] for name, row in report["arms"].items()}, indent=2))


if __name__ == "__main__":
    main()
