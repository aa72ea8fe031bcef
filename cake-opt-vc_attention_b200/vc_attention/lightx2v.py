"""Opt-in LightX2V (MiniMax-H3 DiT) attention adapter and capture path for the
sm100a backend.

Mirrors the reference's adapter (src/vc_attention/lightx2v.py:18-144):
  * ``validate_layout`` accepts one dense self-attention sequence in SND or
    1SND with equal heads and rejects masks, causal attention, dropout and
    packed sequences;
  * ``ExperimentAdapter.apply`` runs ``attention`` with a per-request
    ``LayoutCache``, taking the step from the H3 scheduler and the layer from
    ``block_idx``, resetting the cache when the scheduler's layout marker
    changes or step 0 repeats for a seen layer, and rejecting repeated or
    reversed layer steps;
  * ``capture`` mode saves the first heads of chosen steps/layers as BNSD
    ``.pt`` files with metadata, under a byte budget (the replay reads them);
  * ``configure`` patches a LightX2V config for the experiment.
Differences for this backend: the arms run ``Config(backend="sm100a")``
(``hadamard=True`` puts the ExpCast arms on the Hadamard E4M3 block Q/K
path); capture mode returns torch's BF16 scaled-dot-product attention as
the model's output (the reference used MindIE on Ascend); the MindIE arms
are not offered.
"""
from __future__ import annotations

import argparse
import atexit
import json
import os
import runpy
import sys
from dataclasses import asdict
from pathlib import Path

import torch

from .core import Config, LayoutCache, attention
from .replay import ARMS

ATTN_TYPE = "sm100a_vc_experiment"


def validate_layout(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q, max_seqlen_kv, kwargs):
    """SND / 1SND single-sequence self-attention -> BNSD [1, N, S, D] views
    (lightx2v.py:18-35 contract); every unsupported option raises."""
    allowed = {"scheduler", "block_idx", "causal", "softmax_scale", "dropout", "attn_mask", "mask", "pse"}
    if set(kwargs) - allowed:
        raise ValueError(f"Unknown attention options: {sorted(set(kwargs) - allowed)}")
    if kwargs.get("causal", False) or kwargs.get("dropout", 0):
        raise ValueError("Experiment requires noncausal attention and dropout=0")
    if any(kwargs.get(name) is not None for name in ("mask", "attn_mask", "pse")):
        raise ValueError("Mask/bias is unsupported; do not silently discard it")
    if q.ndim == 4 and q.shape[0] == 1:
        q, k, v = q.squeeze(0), k.squeeze(0), v.squeeze(0)
    if any(x.ndim != 3 for x in (q, k, v)) or q.shape != k.shape or k.shape != v.shape:
        raise ValueError("H3 adapter requires one dense self-attention sequence in SND/1SND with equal heads")
    for cu, maximum, length in ((cu_seqlens_q, max_seqlen_q, q.shape[0]), (cu_seqlens_kv, max_seqlen_kv, k.shape[0])):
        if cu is not None and cu.cpu().tolist() != [0, length]:
            raise ValueError("Packed/multi-sequence attention is unsupported")
        if maximum is not None and int(maximum) != length:
            raise ValueError("max_seqlen does not match the single sequence")
    return [x.transpose(0, 1).unsqueeze(0) for x in (q, k, v)]


def baseline_attention(q, k, v, scale):
    """The model's own attention for capture mode: BF16 SDPA on BNSD."""
    q, k, v = (x.to(torch.bfloat16) for x in (q, k, v))
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale)


def experiment_config(mode: str, *, hadamard: bool = False) -> Config:
    smooth, cast = ARMS.get(mode, (False, False))
    return Config(v_smooth=smooth, expcast=cast, backend="sm100a", qk_hadamard=bool(hadamard and cast))


class ExperimentAdapter:
    """Per-process attention hook; ``options`` carries ``mode`` (an arm or
    "capture"), ``hadamard`` and the capture limits (``output_dir``,
    ``capture_rank``, ``capture_steps``, ``capture_layers``,
    ``capture_heads``, ``max_captures``, ``max_capture_mib``)."""

    def __init__(self, options, audit, attention_fn=attention):
        if options.mode != "capture" and options.mode not in ARMS:
            raise ValueError(f"mode must be capture or one of {sorted(ARMS)} (MindIE arms need Ascend NPUs)")
        self.options, self.audit = options, audit
        self.vc_config = experiment_config(options.mode, hadamard=getattr(options, "hadamard", False))
        self.cache = LayoutCache(self.vc_config)
        self._attention = attention_fn
        self._marker = None
        self._generation = 0
        self._last_steps = {}

    @torch.no_grad()
    def apply(self, q, k, v, cu_seqlens_q=None, cu_seqlens_kv=None, max_seqlen_q=None, max_seqlen_kv=None, **kwargs):
        q, k, v = validate_layout(q, k, v, cu_seqlens_q, cu_seqlens_kv, max_seqlen_q, max_seqlen_kv, kwargs)
        scheduler, layer = kwargs.get("scheduler"), kwargs.get("block_idx")
        if scheduler is None or layer is None:
            raise ValueError("H3 DiT scheduler/block_idx missing")
        marker = getattr(scheduler, "layout_cpu", None)
        if marker is None:
            raise ValueError("This adapter targets H3 scheduler.layout_cpu; unsupported framework version")
        step, steps = int(scheduler.step_index), int(scheduler.infer_steps)
        if marker is not self._marker or (step == 0 and layer in self._last_steps):
            # a new request: hold the marker itself, never a recyclable id()
            self.cache.reset()
            self._marker = marker
            self._generation += 1
            self._last_steps.clear()
        if layer in self._last_steps and step <= self._last_steps[layer]:
            raise ValueError("Repeated/reversed layer-step; head_parallel/CFG/reentrant calls are unsupported")
        self._last_steps[layer] = step
        scale = kwargs.get("softmax_scale")
        scale = q.shape[-1] ** -0.5 if scale is None else scale
        self.audit["calls"] += 1
        if self.options.mode == "capture":
            self._capture(q, k, v, step, steps, layer, scale)
            out = baseline_attention(q, k, v, scale)
        else:
            out, stats = self._attention(q, k, v, self.vc_config, cache=self.cache, step=step, total_steps=steps,
                                         request_id=self._generation, layer_id=layer, scale=scale)
            self.audit["smoothing_calls"] += int(stats["smoothing_active"])
            self.audit["regroup_calls"] += int(stats["layout_refreshed"])
            self.audit["expcast_calls"] += int(stats["expcast"])
        return out.squeeze(0).transpose(0, 1).reshape(q.shape[-2], -1).to(q.dtype)

    def _capture(self, q, k, v, step, steps, layer, scale):
        o = self.options
        rank = int(os.environ.get("RANK", "0"))
        if rank != o.capture_rank or step not in o.capture_steps or layer not in o.capture_layers:
            return
        key = f"rank{rank}_step{step}_layer{layer}"
        if key in self.audit["captures"] or len(self.audit["captures"]) >= o.max_captures:
            return
        tensors = [x[:, :o.capture_heads].detach() for x in (q, k, v)]
        byte_count = sum(x.numel() * x.element_size() for x in tensors)
        if self.audit["capture_bytes"] + byte_count > o.max_capture_mib * 1024 ** 2:
            raise ValueError("Capture budget exceeded; reduce heads/captures or explicitly increase max-capture-mib")
        target = Path(o.output_dir) / "captures" / f"{key}.pt"
        target.parent.mkdir(parents=True, exist_ok=True)
        metadata = {"model": "MiniMax-H3", "layout": "BNSD", "step": step, "total_steps": steps, "layer": layer,
                    "rank": rank, "scale": scale, "full_shape": list(q.shape), "post_rope": True,
                    "attention_boundary": "post_rope_and_optional_ulysses", "full_kv_context": True,
                    "dtype": str(q.dtype)}
        torch.save(dict(zip(("q", "k", "v"), [x.cpu().contiguous() for x in tensors]), metadata=metadata), target)
        self.audit["captures"][key] = str(target.resolve())
        self.audit["capture_bytes"] += byte_count


def configure(base: dict) -> dict:
    """A LightX2V config patched for the experiment (lightx2v.py:126-144 checks)."""
    config = dict(base)
    parallel = config.get("parallel", {})
    if config.get("use_compile", False):
        raise ValueError("Disable use_compile for this eager experimental adapter, in every comparison arm")
    if config.get("warmup", False):
        raise ValueError("Disable warmup for this experiment; warmup tensors must not be captured as the real request")
    config["warmup"] = False
    if parallel.get("seq_p_head_parallel", False):
        raise ValueError("Disable seq_p_head_parallel; head identity is not supplied to the adapter")
    if parallel.get("seq_p_attn_type", "ulysses") != "ulysses":
        raise ValueError("Only Ulysses is supported, not ring/local-softmax composition")
    if config.get("enable_cfg", False):
        raise ValueError("CFG is unsupported by this H3 experiment")
    config["attn_type"] = ATTN_TYPE
    return config


def parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--mode", choices=("capture", *ARMS), required=True)
    ap.add_argument("--hadamard", action="store_true")
    ap.add_argument("--output-dir", required=True)
    ap.add_argument("--capture-steps", type=int, nargs="+", default=[0, 4])
    ap.add_argument("--capture-layers", type=int, nargs="+", default=[0, 12])
    ap.add_argument("--capture-rank", type=int, default=0)
    ap.add_argument("--capture-heads", type=int, default=1)
    ap.add_argument("--max-captures", type=int, default=4)
    ap.add_argument("--max-capture-mib", type=int, default=512)
    ap.add_argument("--prepare-only", action="store_true", help="write the patched config without loading LightX2V")
    ap.add_argument("lightx_args", nargs=argparse.REMAINDER)
    return ap


def main(argv=None):
    ap = parser()
    options = ap.parse_args(argv)
    args = options.lightx_args
    if args[:1] == ["--"]:
        args = args[1:]
    if "--config_json" not in args:
        ap.error("Pass existing LightX2V arguments after --, including --config_json PATH")
    if min(options.capture_heads, options.max_captures, options.max_capture_mib) < 1:
        ap.error("Capture limits must be positive")
    index = args.index("--config_json") + 1
    if index >= len(args):
        ap.error("--config_json requires a path")
    source_path = Path(args[index])
    config = configure(json.loads(source_path.read_text(encoding="utf-8")))
    out = Path(options.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    rank = int(os.environ.get("RANK", "0"))
    patched = out / f"config.rank{rank}.json"
    patched.write_text(json.dumps(config, indent=2) + "\n", encoding="utf-8")
    args[index] = str(patched.resolve())
    if options.prepare_only:
        print(patched.resolve())
        return
    try:
        from lightx2v.utils.registry_factory import ATTN_WEIGHT_REGISTER
        from lightx2v_platform.ops.attn.template import AttnWeightTemplate
    except ImportError as e:
        raise RuntimeError("LightX2V is not installed; --prepare-only writes the patched config without it") from e
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    audit = {"mode": options.mode, "backend": "sm100a", "status": "running", "rank": rank, "calls": 0,
             "smoothing_calls": 0, "regroup_calls": 0, "expcast_calls": 0, "captures": {}, "capture_bytes": 0,
             "argv": args, "source_config": str(source_path.resolve()),
             "vc_config": asdict(experiment_config(options.mode, hadamard=options.hadamard))}

    class RegisteredAdapter(ExperimentAdapter, AttnWeightTemplate):
        def __init__(self):
            super().__init__(options, audit)

    ATTN_WEIGHT_REGISTER.register(RegisteredAdapter, key=ATTN_TYPE)

    def save_audit():
        (out / f"audit.rank{rank}.json").write_text(json.dumps(audit, indent=2) + "\n", encoding="utf-8")

    atexit.register(save_audit)
    sys.argv = ["lightx2v.infer", *args]
    try:
        runpy.run_module("lightx2v.infer", run_name="__main__")
    except BaseException:
        audit["status"] = "failed"
        raise
    else:
        if audit["calls"] == 0:
            audit["status"] = "failed_no_attention_calls"
            raise RuntimeError("Experiment was configured but no attention call reached the adapter")
        audit["status"] = "completed"
    finally:
        save_audit()


if __name__ == "__main__":
    main()
