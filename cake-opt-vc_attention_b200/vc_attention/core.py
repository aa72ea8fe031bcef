"""The ``vc_attention`` Config API with a B200 (sm_100a) backend.

Mirrors the reference package's public surface -- ``Config``,
``LayoutCache`` and ``attention(q, k, v, config, *, cache, step,
total_steps, request_id, layer_id, scale, causal, mask) -> (output,
counters)`` -- (src/vc_attention/core.py:15-371, __init__.py) and adds
``backend="sm100a"``.

The sm100a backend runs on the GPU with ExpCast E4M3 probabilities
(``expcast``), per-channel E4M3 V and -- while smoothing is active -- V
grouping with 128-token block means.  Its Q/K format follows
``qk_hadamard``:
  * ``qk_hadamard=True`` (the Config contract's own path, core.py:79-107,
    128-150): K centred by its FP32 channel mean (``k_smooth``), Q and K
    rotated by the normalised Sylvester transform, E4M3 block payloads with
    one scale per ``q_block`` = 128 Q rows and per ``k_quant_block`` K rows,
    QK^T on the FP8 tensor cores.  ExpCast only.
  * ``qk_hadamard=False``: this repository's INT8 ``sageattn_vc`` pipeline
    (Sage per-thread INT8 Q/K after K channel-mean centring).
Both are compared with the reference backend within a tolerance, not byte
for byte (V is quantised per channel here, per tile there).  The reference's
own backends ("reference", "npu_fp8", "cuda_fp8") are accepted by ``Config``
for compatibility but not executed here: there is no CPU path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

BACKENDS = ("reference", "npu_fp8", "cuda_fp8", "sm100a")


@dataclass(frozen=True)
class Config:
    expcast: bool = False
    v_smooth: bool = False
    quantize: bool = True
    q_block: int = 128
    k_quant_block: int = 256
    kv_block: int = 128
    clusters: int = 8
    iterations: int = 2
    active_fraction: float = 0.25
    refresh_interval: int = 4
    mean_dtype: str = "float16"
    backend: str = "reference"
    k_smooth: bool = True
    qk_hadamard: bool = True
    cuda_schedule: str = "batched"
    cuda_fused_pipeline: bool = True
    cuda_fused_specialize: bool = True
    cuda_fused_interleave: bool = True

    def __post_init__(self):
        # the reference's checks (core.py:36-65), same messages
        if self.cuda_schedule not in ("serial", "batched", "fused"):
            raise ValueError("cuda_schedule must be serial, batched, or fused")
        for name in ("k_smooth", "qk_hadamard", "cuda_fused_pipeline", "cuda_fused_specialize", "cuda_fused_interleave"):
            if not isinstance(getattr(self, name), bool):
                raise ValueError(f"{name} must be a bool")
        for name in ("q_block", "k_quant_block", "kv_block", "clusters", "iterations", "refresh_interval"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, int) or value < 1:
                raise ValueError(f"{name} must be a positive integer")
        if not math.isfinite(self.active_fraction) or not 0 <= self.active_fraction <= 1:
            raise ValueError("active_fraction must be in [0, 1]")
        if self.mean_dtype not in ("float16", "bfloat16", "float32"):
            raise ValueError("Unsupported mean_dtype")
        if self.backend not in BACKENDS:
            raise ValueError("backend must be reference, npu_fp8, cuda_fp8, or sm100a")
        if self.backend in ("npu_fp8", "cuda_fp8", "sm100a") and not self.quantize:
            raise ValueError(f"{self.backend} requires quantize=True")
        if self.backend in ("npu_fp8", "cuda_fp8") and self.k_quant_block % self.kv_block:
            raise ValueError(f"{self.backend} requires kv_block to divide k_quant_block")
        if self.backend == "cuda_fp8":
            if self.cuda_schedule == "fused" and self.kv_block != 128:
                raise ValueError("fused CUDA requires kv_block=128")
            if any(x < 32 or x > 256 or x % 32 for x in (self.q_block, self.kv_block)):
                raise ValueError("cuda_fp8 q_block/kv_block must be multiples of 32 in [32, 256]")
            if self.k_quant_block > 4096:
                raise ValueError("cuda_fp8 k_quant_block must be <= 4096")
        # sm100a: the fused kernel's fixed geometry
        if self.backend == "sm100a":
            if self.qk_hadamard and (self.k_quant_block % 128 or self.k_quant_block > 4096):
                raise ValueError("sm100a requires k_quant_block to be a multiple of 128, at most 4096")
            if self.q_block != 128 or self.kv_block != 128:
                raise ValueError("sm100a requires q_block=128 and kv_block=128")
            if self.v_smooth and self.clusters > 256:
                raise ValueError("sm100a groups V into at most 256 clusters (the grouping kernels' range)")
            if self.mean_dtype != "float16":
                raise ValueError("sm100a stores block means as float16")


def expcast_codes(shifted_scores):
    """ExpCast bytes of FP32 shifted scores on the GPU (core.py:68-76 contract).

    CPU tensors are rejected: this package has no CPU path."""
    from vc_b200 import ops
    return ops.expcast_codes(shifted_scores.float())


class LayoutCache:
    """Request-scoped V layout state (core.py:181-226 semantics).

    While smoothing is active (the first ``active_fraction`` of the
    denoising steps), the grouping permutation is recomputed every
    ``refresh_interval`` steps, warm-started from the cached centres; later
    steps reuse the last permutation without means.  A new request id or a
    changed V signature drops the state."""

    def __init__(self, config):
        self.config = config
        self._request_id = None
        self._states = {}

    @property
    def entries(self):
        return len(self._states)

    def reset(self):
        self._request_id = None
        self._states.clear()

    def _group(self, v, centers):
        from . import sm100a
        return sm100a.group_values(v, clusters=self.config.clusters, iterations=self.config.iterations,
                                   centers=centers)

    def layout(self, v, *, step, total_steps, request_id, layer_id):
        if request_id is None:
            raise ValueError("A persistent layout cache requires request_id")
        if total_steps < 1 or not 0 <= step < total_steps:
            raise ValueError("Invalid denoising step/total_steps")
        if request_id != self._request_id:
            self.reset()
            self._request_id = request_id
        signature = (tuple(v.shape), str(v.device), v.dtype, total_steps)
        state = self._states.get(layer_id)
        if state is not None and (state["signature"] != signature or step < state["step"]):
            state = None
            self._states.pop(layer_id, None)
        active = self.config.v_smooth and step < math.ceil(total_steps * self.config.active_fraction)
        refresh = active and (state is None or step - state["refresh_step"] >= self.config.refresh_interval)
        if refresh:
            pi, centers = self._group(v, None if state is None else state["centers"])
            state = {"signature": signature, "pi": pi, "centers": centers, "refresh_step": step, "step": step}
            self._states[layer_id] = state
        if state is not None:
            state["step"] = step
        return (None if state is None else state["pi"]), active, refresh


def _validate(q, k, v, causal, mask):
    # core.py:229-250, same messages
    if causal:
        raise ValueError("This experiment does not support causal attention")
    if mask is not None:
        raise ValueError("This experiment does not support a mask/bias")
    if any(x.ndim != 4 for x in (q, k, v)):
        raise ValueError("Expected BNSD tensors")
    if q.shape[:2] != k.shape[:2] or k.shape[:2] != v.shape[:2]:
        raise ValueError("Batch and heads must match; GQA is not implemented")
    if k.shape[-2] != v.shape[-2] or q.shape[-1] != k.shape[-1]:
        raise ValueError("Incompatible Q/K/V shape")
    if any(0 in x.shape for x in (q, k, v)):
        raise ValueError("Empty Q/K/V are not supported")
    if any(x.device != q.device or x.dtype != q.dtype for x in (k, v)):
        raise ValueError("Q/K/V must have the same device and dtype")
    if q.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("Inputs must be FP16/BF16/FP32 before quantization")
    if not all(bool(torch.isfinite(x).all()) for x in (q, k, v)):
        raise ValueError("Q/K/V must be finite")


@torch.no_grad()
def attention(q, k, v, config=None, *, cache=None, step=0, total_steps=1, request_id=None, layer_id=0, scale=None,
              causal=False, mask=None):
    """Return ``(output, counters)`` (core.py:264-371 signature and errors)."""
    cfg = config or Config()
    _validate(q, k, v, causal, mask)
    if cfg.backend != "sm100a":
        raise ValueError(f"backend {cfg.backend!r} is not built here; this package runs backend='sm100a' "
                         "(no CPU/reference fallback)")
    from . import sm100a
    return sm100a.attention(q, k, v, cfg, cache=cache, step=step, total_steps=total_steps, request_id=request_id,
                            layer_id=layer_id, scale=q.shape[-1] ** -0.5 if scale is None else scale)
