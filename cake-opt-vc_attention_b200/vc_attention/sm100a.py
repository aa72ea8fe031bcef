"""sm100a backend of the Config API: the Hadamard E4M3 block Q/K path
(``qk_hadamard=True``) or the INT8 ``sageattn_vc`` Q/K path, with the
Config contract's own V format and probabilities.

Plays the role of the reference's cuda_backend.py:37-88 (``_attention``):
validate the device, apply the request's V layout, prepare payloads and run
a fused tcgen05 kernel, returning the reference's counter keys.  As in the
contract (core.py:110-123, and the reference's native backend,
csrc/kernels.cu:160-180), V is encoded per 128-token tile: the tile mean when
smoothing is active (else zero), one scale per tile and channel; without
ExpCast the probabilities are the FP8-P control P8 = e4m3(256 exp(s - max))
with exact exp row sums (core.py:357-360).  Per-tile, per-channel V scales
cannot be applied inside a tensor-memory accumulation, so this backend runs
the register-accumulating kernel.
"""
from __future__ import annotations

import math

import torch

from vc_b200 import ops


def _require_device(q):
    if q.device.type != "cuda":
        raise ValueError("sm100a requires CUDA tensors; no CPU/NPU fallback")
    if torch.cuda.get_device_capability(q.device)[0] != 10:
        raise ValueError("sm100a requires a B200-class GPU (compute capability 10.x)")


def group_values(v, *, clusters, iterations, centers=None):
    """Device Lloyd grouping with the reference's return contract
    (core.py:152-178): the stable permutation and the centres after the
    final update (mean of each cluster's tokens; empty clusters keep the
    centre of the final assignment)."""
    pi, labels, used = ops.group_values(v, clusters, iterations, centers=centers, debug=True)
    x = v.float()
    count = used.shape[-2]
    idx = labels.long().unsqueeze(-1).expand_as(x)
    sums = torch.zeros_like(used).scatter_add_(-2, idx, x)
    counts = torch.zeros_like(used[..., :1]).scatter_add_(-2, labels.long().unsqueeze(-1),
                                                           torch.ones_like(x[..., :1]))
    centers_out = torch.where(counts > 0, sums / counts.clamp_min(1), used)
    assert centers_out.shape[-2] == count
    return pi, centers_out


@torch.no_grad()
def attention(q, k, v, cfg, *, cache, step, total_steps, request_id, layer_id, scale):
    _require_device(q)
    if q.shape[-1] not in (64, 128) or v.shape[-1] != q.shape[-1]:
        raise ValueError("sm100a supports Q/K/V head dimensions 64 or 128 (equal)")
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("scale must be positive and finite")
    from .core import LayoutCache

    if cache is None:
        cache = LayoutCache(cfg)
        request_id = "one-shot" if request_id is None else request_id
    elif cache.config != cfg:
        raise ValueError("cache.config must match config")
    with torch.cuda.device(q.device):
        pi, active, refreshed = cache.layout(v, step=step, total_steps=total_steps, request_id=request_id,
                                             layer_id=layer_id)
        B, H, _, D = k.shape
        if cfg.qk_hadamard:
            q8, qs, k8, ks, _ = ops.prep_qk_hadamard(q, k, perm=pi, k_smooth=cfg.k_smooth,
                                                     k_quant_block=cfg.k_quant_block)
        else:
            km = None if cfg.k_smooth else torch.zeros((B, H, 1, D), dtype=k.dtype, device=k.device)
            q8, qs, k8, ks, _ = ops.prep_qk_int8(q, k, perm=pi, km=km)
        # per-tile V: residual over the tile mean (zero means when smoothing is off), per-tile scales
        v8, vs, means = ops.prep_v_blocks(v, perm=pi, channel_scale=False, demean=active)
        out = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, out_dtype=q.dtype, sm_scale=float(scale),
                                expcast=cfg.expcast, block_values=True, k_quant_block=cfg.k_quant_block,
                                control="config")
    tiles = math.ceil(q.shape[-2] / 128) * math.ceil(k.shape[-2] / 128)
    return out, {
        "backend": "sm100a",
        "smoothing_active": active,
        "layout_refreshed": refreshed,
        "expcast": cfg.expcast,
        "k_smooth": cfg.k_smooth,
        "qk_hadamard": cfg.qk_hadamard,
        "numerical_contract_version": 2,
        "tiles": tiles,
        "native_fused_attention": True,
        "preprocessing_fused": False,
        "native_fp8_matmul": True,
        "native_int8_matmul": not cfg.qk_hadamard,
        "cuda_schedule": "fused",
        "cuda_fused_pipeline": True,
        "cuda_fused_variant": "sm100a_tcgen05",
    }
