"""Drop-in ``sageattn_vc``: Sage INT8 QK + ExpCast P + FP8 PV with optional
V grouping / 128-token block smoothing, on B200 (sm_100a).

Mirrors the reference boundary
third_party/sageattention_local/sageattention_local/vc.py:1-235 -- same
signature and defaults, same ``kernel_mode`` / ``v_scale_mode`` /
``grouping_mode`` vocabularies and the same ``ValueError`` contract raised
before any native call.  Differences, all supersets:
  * runs on sm_100 (B200) instead of Hopper; every documented kernel_mode maps
    onto the single tcgen05 kernel (Hopper schedule variants do not exist);
  * any current CUDA stream is accepted (the reference required the default
    stream, vc.py:226-228);
  * NHD inputs are consumed through strides and the NHD output is written in
    place -- no transpose copies (vc.py:229-231, 235).
No CPU or reference fallback: the CUDA library must be present.
"""
import math

import torch

from vc_b200 import ops

# kernel_mode vocabulary of the reference (vc.py:12-46).  The numbers were
# Hopper schedule ids; they are kept only so validation rules match.
DEFAULT_EXPCAST_KERNEL = "vc15"
UNIFIED_MODES = {"vc31_unified": 38, "vc32_full_pv": 39, "vc32_packed_mean": 40}
DESCRIPTOR_CANDIDATES = {"vc30_desc": 37}
STREAM_CONVERT_CANDIDATES = {"vc28_stream_i2f": 35, "vc29_interleave_rows": 36}
REGISTER_CANDIDATES = {"vc18_r128": 128, "vc18_r144": 144, "vc18_r192": 192,
                       "vc18_pv64_r128": 128, "vc18_pv64_r144": 144, "vc18_pv64_r168": 168}
PIPELINE_CANDIDATES = {
    "vc19_k": {"k_buffers": 2, "v_buffers": 1, "early_tma_prefetch": 1},
    "vc19_v": {"k_buffers": 1, "v_buffers": 2, "early_tma_prefetch": 1},
    "vc19_kv": {"k_buffers": 2, "v_buffers": 2, "early_tma_prefetch": 1},
    "vc19_kv_late": {"k_buffers": 2, "v_buffers": 2, "early_tma_prefetch": 0},
}
MASS_CANDIDATES = {"vc25_mass_serial": 7, "vc25_mass_overlap": 8}
DUAL_QUERY_CANDIDATES = {"vc26_shared": 1, "vc26_stagger": 2}
ENCODING_CANDIDATES = {"vc24_bitpack": 6}
STATE_CANDIDATES = {"vc23_maxstate": 4, "vc23_cached_bias": 5}
WORK_CANDIDATES = {"vc22_intmax": 1, "vc22_skip": 2, "vc22_both": 3}
HISTORY_CANDIDATES = {"vc21_history_r128": 128, "vc21_history_r168": 168}
COMPUTE_CANDIDATES = {"vc20_pv_qk": 1, "vc20_serial": 2, "vc20_qk_pv": 3}
SAGE_LAYOUT_MODES = {"vc16": 1, "vc16_early_v": 2, "vc16_pack_first": 3,
                     "vc16_pack_early": 4, "vc16_serial": 5,
                     "vc17_g1": 6, "vc17_g4": 7, "vc17_c4": 8, "vc17_direct": 9,
                     "vc18_r128": 10, "vc18_r144": 11, "vc18_r192": 12,
                     "vc18_pv64_r128": 13, "vc18_pv64_r144": 14, "vc18_pv64_r168": 15,
                     **{mode: i + 16 for i, mode in enumerate(PIPELINE_CANDIDATES)},
                     **{mode: schedule + 19 for mode, schedule in COMPUTE_CANDIDATES.items()},
                     **{mode: i + 23 for i, mode in enumerate(HISTORY_CANDIDATES)},
                     **{mode: i + 24 for mode, i in WORK_CANDIDATES.items()},
                     **{mode: i + 24 for mode, i in STATE_CANDIDATES.items()},
                     **{mode: i + 24 for mode, i in ENCODING_CANDIDATES.items()},
                     **{mode: i + 24 for mode, i in MASS_CANDIDATES.items()},
                     **{mode: i + 32 for mode, i in DUAL_QUERY_CANDIDATES.items()},
                     **STREAM_CONVERT_CANDIDATES, **DESCRIPTOR_CANDIDATES, **UNIFIED_MODES}
BASE_MODES = ("optimized", "vc15", "vc14", "vc13_overlap", "vc13_serial", "vc12", "vc11", "vc10", "vc9", "vc7",
              "vc6", "vc4")
KERNEL_MODES = (*BASE_MODES, *SAGE_LAYOUT_MODES)


def _extension():
    """The native library (raises if it is missing: there is no fallback)."""
    from vc_b200 import _native
    return _native.load()


def sage_vc_build_info():
    lib = _extension()
    return {"vc_extension": str(__import__("vc_b200._native", fromlist=["LIB_PATH"]).LIB_PATH),
            "backend": "sm100a", "build": lib.vc_build_info().decode(),
            "kernel_math_modified": True,
            "algorithm": "Sage per-thread INT8 QK + VC block V residual/mean + ExpCast",
            "qk_hadamard": False, "v_block": 128, "mean_dtype": "float16",
            "clustering": "8 clusters, 2 Lloyd iterations, stable order; fresh every call",
            "grouping_modes": ["fused", "legacy"], "default_grouping_mode": "fused",
            "grouping_implementation": "tiled assignment, fixed-order FP32 centre statistics, stable counting sort",
            "paper_equivalent": False, "sage_vc_api_version": 1,
            "default_kernel_mode": "optimized", "default_expcast_kernel": DEFAULT_EXPCAST_KERNEL,
            "kernel_modes": list(KERNEL_MODES),
            "kernel_mode_mapping": "every documented kernel_mode runs the single sm_100a tcgen05 kernel",
            "v_scale_mode": "channel", "v_scale_modes": ["channel", "block"],
            "probability_scratch_bytes_per_block": 0}


def kernel_resources(output_type=1):
    """Compiled resources of the fused kernel, keyed like the reference's
    report (vc.py:113-118); all modes share one kernel."""
    r = ops.kernel_resources(128)
    out = {"expcast_optimized": r, "expcast_vc15": r, "expcast_vc14": r, "expcast_vc13_overlap": r,
           "expcast_vc12": r}
    return out


def validate_inputs(q, k, v, tensor_layout, is_causal, return_lse, expcast, v_smooth, clusters, iterations):
    """Same checks and messages as the reference (vc.py:121-138)."""
    if is_causal or return_lse:
        raise ValueError("Sage VC supports noncausal forward without LSE only")
    if tensor_layout not in ("HND", "NHD"):
        raise ValueError("tensor_layout must be HND or NHD")
    if not isinstance(expcast, bool) or not isinstance(v_smooth, bool):
        raise ValueError("expcast and v_smooth must be bool")
    if any(isinstance(x, bool) or not isinstance(x, int) for x in (clusters, iterations)) or not (
            1 <= clusters <= 256 and 1 <= iterations <= 100):
        raise ValueError("Invalid clustering parameters")
    if any(x.ndim != 4 or x.numel() == 0 for x in (q, k, v)):
        raise ValueError("Expected nonempty four-dimensional Q/K/V")
    if q.dtype not in (torch.float16, torch.bfloat16) or any(x.dtype != q.dtype or x.device != q.device for x in (k, v)):
        raise ValueError("Q/K/V require matching FP16/BF16 dtype and device")
    head_axis = 1 if tensor_layout == "HND" else 2
    if (k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[head_axis] != k.shape[head_axis]
            or q.shape[-1] != k.shape[-1]):
        raise ValueError("Q/K/V batch/heads/dim must match; GQA is unsupported")
    if q.shape[-1] not in (64, 128):
        raise ValueError("Sage VC requires D=64/128")


def _require_sm100(device):
    if device.type != "cuda" or torch.cuda.get_device_capability(device)[0] != 10:
        raise ValueError("Sage VC requires an sm_100 (B200) CUDA device; no CPU/reference fallback")


@torch.no_grad()
def prepare(q, k, v, *, expcast=True, v_smooth=True, clusters=8, iterations=2, sm_scale=None,
            v_scale_mode="channel", grouping_mode="fused", mean_numel=None):
    """HND preparation on the current stream (reference vc.py:142-170).

    Returns the reference's state-dict keys.  ``state['v']`` is the payload
    in token order [B,H,D,Npad] (the reference stored a Hopper-specific
    16-token permutation of it); ``state['km']`` is the K channel mean.
    """
    if v_scale_mode not in ("channel", "block"):
        raise ValueError("v_scale_mode must be 'channel' or 'block'")
    if grouping_mode not in ("fused", "legacy"):
        raise ValueError("grouping_mode must be 'fused' or 'legacy'")
    permutation = None
    if v_smooth:
        permutation = ops.group_values(v, clusters, iterations)
    # torch's CUDA mean projects the FP32 sum by float(#out)/float(#in)
    if mean_numel is None:
        mean_numel = (q.shape[0] * k.shape[1] * k.shape[3], k.numel())
    q8, qs, k8, ks, km = ops.prep_qk_int8(q, k, perm=permutation, mean_numel=mean_numel)
    if v_smooth:
        v8, vs, means = ops.prep_v_blocks(v, perm=permutation, channel_scale=v_scale_mode == "channel")
    else:
        v8, vs = ops.prep_v_channel(v)
        means = torch.empty(0, device=v.device, dtype=torch.float16)
    return {"q": q8, "k": k8, "v": v8, "qs": qs, "ks": ks, "vs": vs, "means": means,
            "expcast": expcast, "block_values": v_smooth, "output_type": 0 if q.dtype == torch.float16 else 1,
            "scale": q.shape[-1] ** -0.5 if sm_scale is None else sm_scale, "permutation": permutation, "km": km}


def _check_kernel_mode(kernel_mode, *, block_values, expcast, vs_dim, head_dim):
    """Reference rejection rules (vc.py:173-185, 203-216)."""
    sage_schedule = SAGE_LAYOUT_MODES.get(kernel_mode, 0)
    if kernel_mode in UNIFIED_MODES and vs_dim != 3:
        raise ValueError("vc31/vc32 require per-channel V scale")
    if kernel_mode in HISTORY_CANDIDATES and head_dim != 128:
        raise ValueError("Shared-history candidates require D128")
    if sage_schedule:
        if block_values and kernel_mode not in UNIFIED_MODES:
            raise ValueError("Sage layout candidates require v_smooth=False")
        if 6 <= sage_schedule <= 9 and not expcast:
            raise ValueError("Probability candidates require expcast=True")
        if expcast and sage_schedule in (3, 4):
            raise ValueError("Pack-first candidates require expcast=False")
    elif kernel_mode not in BASE_MODES:
        raise ValueError("Unknown kernel_mode; use a documented vc4..vc21 mode or 'optimized'")


def forward_prepared(state, *, kernel_mode="optimized", out=None):
    """Fused attention on a prepared state (reference vc.py:173-197)."""
    _check_kernel_mode(kernel_mode, block_values=state["block_values"], expcast=state["expcast"],
                       vs_dim=state["vs"].ndim, head_dim=state["q"].shape[-1])
    out_dtype = torch.float16 if state["output_type"] == 0 else torch.bfloat16
    return ops.attention_fwd(state["q"], state["qs"], state["k"], state["ks"], state["v"], state["vs"],
                             state["means"], out_dtype=out_dtype, sm_scale=state["scale"],
                             expcast=state["expcast"], block_values=state["block_values"], out=out)


@torch.no_grad()
def sageattn_vc(q, k, v, tensor_layout="HND", is_causal=False, sm_scale=None, return_lse=False,
                *, expcast=True, v_smooth=True, clusters=8, iterations=2, kernel_mode="optimized",
                v_scale_mode="channel", grouping_mode="fused"):
    if kernel_mode not in KERNEL_MODES:
        raise ValueError("Unknown kernel_mode; use a documented vc4..vc21 mode or 'optimized'")
    if kernel_mode in UNIFIED_MODES and v_scale_mode != "channel":
        raise ValueError("vc31/vc32 require per-channel V scale")
    if kernel_mode in HISTORY_CANDIDATES and q.shape[-1] != 128:
        raise ValueError("Shared-history candidates require D128")
    if kernel_mode in SAGE_LAYOUT_MODES:
        if v_smooth and kernel_mode not in UNIFIED_MODES:
            raise ValueError("Sage layout candidates require v_smooth=False")
        if 6 <= SAGE_LAYOUT_MODES[kernel_mode] <= 9 and not expcast:
            raise ValueError("Probability candidates require expcast=True")
        if expcast and SAGE_LAYOUT_MODES[kernel_mode] in (3, 4):
            raise ValueError("Pack-first candidates require expcast=False")
    if v_scale_mode not in ("channel", "block"):
        raise ValueError("v_scale_mode must be 'channel' or 'block'")
    if grouping_mode not in ("fused", "legacy"):
        raise ValueError("grouping_mode must be 'fused' or 'legacy'")
    validate_inputs(q, k, v, tensor_layout, is_causal, return_lse, expcast, v_smooth, clusters, iterations)
    _require_sm100(q.device)
    if sm_scale is not None and (not math.isfinite(sm_scale) or not 0 < sm_scale <= 3.4028234663852886e38):
        raise ValueError("sm_scale must be positive and finite FP32")
    with torch.cuda.device(q.device):
        out = None
        if tensor_layout == "NHD":
            out = torch.empty_like(q, memory_format=torch.contiguous_format)
            mean_numel = (k.shape[0] * k.shape[2] * k.shape[3], k.numel())
            q, k, v = (x.transpose(1, 2) for x in (q, k, v))
            out_view = out.transpose(1, 2)
        else:
            mean_numel = None
            out_view = None
        state = prepare(q, k, v, expcast=expcast, v_smooth=v_smooth, clusters=clusters, iterations=iterations,
                        sm_scale=sm_scale, v_scale_mode=v_scale_mode, grouping_mode=grouping_mode,
                        mean_numel=mean_numel)
        result = forward_prepared(state, kernel_mode=kernel_mode, out=out_view)
        return out if tensor_layout == "NHD" else result
