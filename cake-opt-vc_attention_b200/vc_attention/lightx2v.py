"""LightX2V (MiniMax-H3 DiT) integration of the sm100a VC attention: an
attention layer that LightX2V's registry can instantiate, a capture mode
that records real Q/K/V for the replay, and a launcher.

The behaviour follows the reference's adapter contract
(src/vc_attention/lightx2v.py:18-239): one dense, non-causal, unmasked
self-attention sequence per call (SND or 1SND, equal head counts, no
packing); the denoising step comes from the H3 scheduler and the layer from
``block_idx``; a new request starts (and the layout cache is cleared) when
the scheduler's layout marker object changes or a layer sees step 0 again;
a repeated or reversed step for a layer is an error.  Capture mode stores the
first heads of chosen steps and layers of one rank, under a byte budget, as
BNSD ``.pt`` files with metadata, and returns ordinary attention to the
model.

Built differently here: the call is parsed into an ``H3Call`` record, request
bookkeeping lives in ``RequestTracker``, captures in ``CaptureSink``, and the
registered layer (``H3VCAttention``) only composes them.  The arms run
``Config(backend="sm100a")``; ``hadamard=True`` puts the arms on the Config
contract's own Hadamard E4M3 block Q/K path.  Capture mode returns
torch's BF16 scaled-dot-product attention (the reference used MindIE on
Ascend, which has no counterpart here).
"""
from __future__ import annotations

import argparse
import atexit
import json
import os
import runpy
import sys
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch

from .core import Config, LayoutCache, attention
from .replay import ARMS

ATTN_TYPE = "sm100a_vc_experiment"
MODES = ("capture", *ARMS)

# keyword options LightX2V passes to an attention layer that this layer understands
_KNOWN_OPTIONS = frozenset({"scheduler", "block_idx", "causal", "softmax_scale", "dropout", "attn_mask", "mask", "pse"})


@dataclass
class H3Call:
    """One attention call of the H3 DiT, normalised to BNSD (batch 1)."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    tokens: int
    scale: float
    scheduler: object = None
    layer: int | None = None


def _single_sequence(cu_seqlens, max_seqlen, tokens: int) -> None:
    if cu_seqlens is not None and [int(x) for x in cu_seqlens.flatten().cpu()] != [0, tokens]:
        raise ValueError("only one unpacked sequence per call is supported (cu_seqlens must be [0, S])")
    if max_seqlen is not None and int(max_seqlen) != tokens:
        raise ValueError(f"max_seqlen {int(max_seqlen)} does not match the sequence length {tokens}")


def parse_call(q, k, v, cu_seqlens_q=None, cu_seqlens_kv=None, max_seqlen_q=None, max_seqlen_kv=None,
               options: dict | None = None) -> H3Call:
    """Check an incoming call against what the VC contract covers and
    return it as an ``H3Call``; everything else raises ValueError rather
    than being dropped silently."""
    options = dict(options or {})
    unknown = sorted(set(options) - _KNOWN_OPTIONS)
    if unknown:
        raise ValueError(f"unsupported attention options {unknown}")
    if options.get("causal") or options.get("dropout"):
        raise ValueError("VC attention is non-causal and dropout-free")
    for name in ("mask", "attn_mask", "pse"):
        if options.get(name) is not None:
            raise ValueError(f"'{name}' (mask or positional bias) cannot be applied by VC attention")
    if q.dim() == 4 and q.shape[0] == 1:
        q, k, v = q[0], k[0], v[0]
    if not (q.dim() == k.dim() == v.dim() == 3) or not (q.shape == k.shape == v.shape):
        raise ValueError("expected one dense self-attention sequence as SND or 1SND with equal Q/K/V shapes")
    tokens = q.shape[0]
    _single_sequence(cu_seqlens_q, max_seqlen_q, tokens)
    _single_sequence(cu_seqlens_kv, max_seqlen_kv, tokens)
    scale = options.get("softmax_scale")
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    bnsd = [x.permute(1, 0, 2).unsqueeze(0) for x in (q, k, v)]
    return H3Call(*bnsd, tokens=tokens, scale=scale, scheduler=options.get("scheduler"),
                  layer=options.get("block_idx"))


def to_snd(out: torch.Tensor, tokens: int, dtype) -> torch.Tensor:
    """BNSD (batch 1) -> the [S, H*D] layout LightX2V expects back."""
    return out[0].permute(1, 0, 2).reshape(tokens, -1).to(dtype)


class RequestTracker:
    """Maps calls to denoising requests.  The H3 scheduler's ``layout_cpu``
    object is the request marker (held by reference, not by id); a layer
    seeing step 0 again also starts a new request.  Steps of one layer must
    increase within a request."""

    def __init__(self):
        self.marker = None
        self.request = 0
        self.last_step: dict[int, int] = {}

    def observe(self, scheduler, layer) -> tuple[int, int, int, bool]:
        """Returns (request, step, total_steps, started_new_request)."""
        if scheduler is None or layer is None:
            raise ValueError("the H3 scheduler and block_idx are required (refiner_attn_type must stay "
                             "npu_flash_attn so the refiner does not reach this layer)")
        marker = getattr(scheduler, "layout_cpu", None)
        if marker is None:
            raise ValueError("scheduler has no layout_cpu marker: not an H3 scheduler this layer supports")
        step, total = int(scheduler.step_index), int(scheduler.infer_steps)
        layer = int(layer)
        new = marker is not self.marker or (step == 0 and layer in self.last_step)
        if new:
            self.marker = marker
            self.request += 1
            self.last_step = {}
        prev = self.last_step.get(layer)
        if prev is not None and step <= prev:
            raise ValueError(f"layer {layer} saw step {step} after step {prev}: repeated or reversed steps "
                             "(head-parallel, CFG or re-entrant calls) are not supported")
        self.last_step[layer] = step
        return self.request, step, total, new


@dataclass
class Audit:
    """Counters written next to the run's outputs."""
    mode: str
    rank: int = 0
    status: str = "running"
    calls: int = 0
    smoothing_calls: int = 0
    regroup_calls: int = 0
    expcast_calls: int = 0
    captures: dict = field(default_factory=dict)
    capture_bytes: int = 0
    extra: dict = field(default_factory=dict)

    def as_dict(self) -> dict:
        d = asdict(self)
        d.update(d.pop("extra"))
        return d


class CaptureSink:
    """Writes the first ``heads`` heads of the selected (rank, step, layer)
    calls as ``captures/rank{r}_step{s}_layer{l}.pt`` -- a dict of BNSD CPU
    tensors ``q``, ``k``, ``v`` plus ``metadata`` -- at most ``max_files``
    files and ``max_bytes`` bytes in all (exceeding the byte budget raises)."""

    def __init__(self, out_dir, *, rank: int, steps, layers, heads: int, max_files: int, max_bytes: int):
        if min(heads, max_files, max_bytes) < 1:
            raise ValueError("capture heads, file count and byte budget must be positive")
        self.root = Path(out_dir) / "captures"
        self.rank, self.steps, self.layers = rank, set(steps), set(layers)
        self.heads, self.max_files, self.max_bytes = heads, max_files, max_bytes

    def wants(self, rank: int, step: int, layer: int) -> bool:
        return rank == self.rank and step in self.steps and layer in self.layers

    def save(self, call: H3Call, step: int, total_steps: int, audit: Audit, rank: int) -> Path | None:
        name = f"rank{rank}_step{step}_layer{call.layer}"
        if not self.wants(rank, step, int(call.layer)) or name in audit.captures or \
                len(audit.captures) >= self.max_files:
            return None
        parts = {n: t[:, : self.heads].detach() for n, t in zip("qkv", (call.q, call.k, call.v))}
        nbytes = sum(t.numel() * t.element_size() for t in parts.values())
        if audit.capture_bytes + nbytes > self.max_bytes:
            raise ValueError(f"capture of {name} ({nbytes} bytes) would exceed the {self.max_bytes}-byte budget; "
                             "capture fewer heads or files, or raise --max-capture-mib")
        meta = {"model": "MiniMax-H3", "layout": "BNSD", "step": step, "total_steps": total_steps,
                "layer": int(call.layer), "rank": rank, "scale": call.scale, "full_shape": list(call.q.shape),
                "post_rope": True, "attention_boundary": "post_rope_and_optional_ulysses", "full_kv_context": True,
                "dtype": str(call.q.dtype)}
        self.root.mkdir(parents=True, exist_ok=True)
        path = self.root / f"{name}.pt"
        torch.save({**{n: t.cpu().contiguous() for n, t in parts.items()}, "metadata": meta}, path)
        audit.captures[name] = str(path.resolve())
        audit.capture_bytes += nbytes
        return path


def arm_config(mode: str, *, hadamard: bool = False) -> Config:
    """The sm100a Config of an experiment arm: INT8 Q/K, or with
    ``hadamard`` the Config contract's Hadamard E4M3 block Q/K."""
    if mode not in ARMS:
        raise ValueError(f"unknown arm {mode!r}; arms are {sorted(ARMS)}")
    smooth, cast = ARMS[mode]
    return Config(v_smooth=smooth, expcast=cast, backend="sm100a", qk_hadamard=bool(hadamard))


def sdpa_bf16(call: H3Call) -> torch.Tensor:
    """Ordinary attention for capture mode: torch's BF16 scaled-dot-product
    attention on the same tensors."""
    q, k, v = (x.to(torch.bfloat16) for x in (call.q, call.k, call.v))
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=call.scale)


class H3VCAttention:
    """The attention layer LightX2V calls (``apply``).  ``mode`` is one of
    ``MODES``; ``attention_fn`` is injectable for host-side tests."""

    def __init__(self, mode: str, *, hadamard: bool = False, capture: CaptureSink | None = None,
                 audit: Audit | None = None, rank: int | None = None, attention_fn=attention):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
        if mode == "capture" and capture is None:
            raise ValueError("capture mode needs a CaptureSink")
        self.mode = mode
        self.rank = int(os.environ.get("RANK", "0")) if rank is None else rank
        self.audit = audit or Audit(mode=mode, rank=self.rank)
        self.capture = capture
        self.tracker = RequestTracker()
        self.attention_fn = attention_fn
        self.vc_config = arm_config(mode, hadamard=hadamard) if mode != "capture" else None
        self.cache = LayoutCache(self.vc_config) if self.vc_config is not None else None

    @torch.no_grad()
    def apply(self, q, k, v, cu_seqlens_q=None, cu_seqlens_kv=None, max_seqlen_q=None, max_seqlen_kv=None,
              **options):
        call = parse_call(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q, max_seqlen_kv, options)
        request, step, total, new = self.tracker.observe(call.scheduler, call.layer)
        if new and self.cache is not None:
            self.cache.reset()
        self.audit.calls += 1
        if self.mode == "capture":
            self.capture.save(call, step, total, self.audit, self.rank)
            out = sdpa_bf16(call)
        else:
            out, stats = self.attention_fn(call.q, call.k, call.v, self.vc_config, cache=self.cache, step=step,
                                           total_steps=total, request_id=request, layer_id=int(call.layer),
                                           scale=call.scale)
            self.audit.smoothing_calls += int(bool(stats["smoothing_active"]))
            self.audit.regroup_calls += int(bool(stats["layout_refreshed"]))
            self.audit.expcast_calls += int(bool(stats["expcast"]))
        return to_snd(out, call.tokens, q.dtype)


# LightX2V configuration rules: (predicate on the config, message if it holds)
_CONFIG_RULES = (
    (lambda c: c.get("use_compile", False), "use_compile must be off: the adapter is eager (in every arm)"),
    (lambda c: c.get("warmup", False), "warmup must be off: warm-up tensors would be captured as the request"),
    (lambda c: c.get("parallel", {}).get("seq_p_head_parallel", False),
     "seq_p_head_parallel must be off: the layer is not told which heads it holds"),
    (lambda c: c.get("parallel", {}).get("seq_p_attn_type", "ulysses") != "ulysses",
     "only Ulysses sequence parallelism is supported (ring / local-softmax composition is not)"),
    (lambda c: c.get("enable_cfg", False), "CFG is not supported by the H3 experiment"),
)


def configure(base: dict) -> dict:
    """The LightX2V config for a VC run: ``base`` checked against the
    rules above, then pointed at this layer (the refiner keeps
    npu_flash_attn) with warm-up off."""
    for broken, message in _CONFIG_RULES:
        if broken(base):
            raise ValueError(message)
    return {**base, "warmup": False, "attn_type": ATTN_TYPE, "refiner_attn_type": "npu_flash_attn"}


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Run LightX2V with the sm100a VC attention layer (or capture Q/K/V)")
    p.add_argument("--mode", choices=MODES, required=True)
    p.add_argument("--hadamard", action="store_true", help="the arms on the Hadamard E4M3 block Q/K path")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--capture-steps", type=int, nargs="+", default=[0, 4])
    p.add_argument("--capture-layers", type=int, nargs="+", default=[0, 12])
    p.add_argument("--capture-rank", type=int, default=0)
    p.add_argument("--capture-heads", type=int, default=1)
    p.add_argument("--max-captures", type=int, default=4)
    p.add_argument("--max-capture-mib", type=int, default=512)
    p.add_argument("--prepare-only", action="store_true", help="write the patched config and stop")
    p.add_argument("lightx_args", nargs=argparse.REMAINDER, help="LightX2V arguments after --, with --config_json")
    return p


def main(argv=None):
    ap = parser()
    opts = ap.parse_args(argv)
    args = list(opts.lightx_args)
    if args[:1] == ["--"]:
        args = args[1:]
    if "--config_json" not in args or args.index("--config_json") + 1 >= len(args):
        ap.error("pass the LightX2V arguments after --, including --config_json PATH")
    if min(opts.capture_heads, opts.max_captures, opts.max_capture_mib) < 1:
        ap.error("capture limits must be positive")
    at = args.index("--config_json") + 1
    source = Path(args[at])
    rank = int(os.environ.get("RANK", "0"))
    out = Path(opts.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    patched = out / f"config.rank{rank}.json"
    patched.write_text(json.dumps(configure(json.loads(source.read_text(encoding="utf-8"))), indent=2) + "\n",
                       encoding="utf-8")
    args[at] = str(patched.resolve())
    if opts.prepare_only:
        print(patched.resolve())
        return patched
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    from lightx2v.utils.registry_factory import ATTN_WEIGHT_REGISTER
    from lightx2v_platform.ops.attn.template import AttnWeightTemplate

    sink = None
    if opts.mode == "capture":
        sink = CaptureSink(out, rank=opts.capture_rank, steps=opts.capture_steps, layers=opts.capture_layers,
                           heads=opts.capture_heads, max_files=opts.max_captures,
                           max_bytes=opts.max_capture_mib * 1024 ** 2)
    audit = Audit(mode=opts.mode, rank=rank, extra={
        "backend": "sm100a", "argv": args, "source_config": str(source.resolve()),
        "vc_config": asdict(arm_config(opts.mode, hadamard=opts.hadamard)) if opts.mode in ARMS else None})

    class Registered(H3VCAttention, AttnWeightTemplate):
        def __init__(self):
            H3VCAttention.__init__(self, opts.mode, hadamard=opts.hadamard, capture=sink, audit=audit, rank=rank)

    ATTN_WEIGHT_REGISTER.register(Registered, key=ATTN_TYPE)
    audit_path = out / f"audit.rank{rank}.json"
    atexit.register(lambda: audit_path.write_text(json.dumps(audit.as_dict(), indent=2) + "\n", encoding="utf-8"))
    print(f"[vc sm100a] LightX2V run, mode={opts.mode}")
    sys.argv = ["lightx2v.infer", *args]
    try:
        runpy.run_module("lightx2v.infer", run_name="__main__")
        audit.status = "completed" if audit.calls else "failed_no_attention_calls"
        if not audit.calls:
            raise RuntimeError("LightX2V ran but no attention call reached the VC layer")
    except BaseException:
        if audit.status == "running":
            audit.status = "failed"
        raise
    finally:
        audit_path.write_text(json.dumps(audit.as_dict(), indent=2) + "\n", encoding="utf-8")
    return audit


if __name__ == "__main__":
    main()
