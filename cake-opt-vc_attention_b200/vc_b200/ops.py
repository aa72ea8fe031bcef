"""Torch-tensor wrappers over the C ABI (device memory and streams from torch).

Each op validates its tensors, allocates outputs and workspace from torch's
caching allocator and calls the library on the current CUDA stream.  There
is no CPU path: non-CUDA tensors raise ValueError.
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import _native as N

_DT = {torch.float16: N.VC_DTYPE_F16, torch.bfloat16: N.VC_DTYPE_BF16, torch.float32: N.VC_DTYPE_F32}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _require_cuda(name, *ts):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"{name}: tensors must be on a CUDA device (no CPU fallback)")


def _rowmajor(x: torch.Tensor) -> torch.Tensor:
    """Keep (b, h, s) strides when the channel axis is contiguous and all
    strides are 16-byte multiples; otherwise make a contiguous copy."""
    es = x.element_size()
    if x.stride(3) == 1 and all((s * es) % 16 == 0 for s in x.stride()[:3]) and x.data_ptr() % 16 == 0:
        return x
    return x.contiguous()


def _perm(name, perm, B, H, S):
    """Per-(batch, head) token permutation: [B, H, S] integers, made int64
    contiguous.  Entries must lie in [0, S); the kernels record an error bit
    and read zeros for any that do not."""
    if perm is None:
        return None
    if tuple(perm.shape) != (B, H, S) or perm.dtype.is_floating_point or perm.dtype == torch.bool:
        raise ValueError(f"{name}: perm must be an integer tensor of shape {(B, H, S)}, got "
                         f"{tuple(perm.shape)} {perm.dtype}")
    return perm.to(torch.int64).contiguous()


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def expcast_codes(x: torch.Tensor) -> torch.Tensor:
    """ExpCast bytes of FP32 scores (shape preserved, uint8)."""
    _require_cuda("expcast_codes", x)
    if x.dtype != torch.float32:
        raise ValueError("expcast_codes requires FP32 input")
    x = x.contiguous()
    y = torch.empty_like(x, dtype=torch.uint8)
    with torch.cuda.device(x.device):
        N.check(N.load().vc_expcast_codes(_p(x), _p(y), x.numel(), _stream(x)), "vc_expcast_codes")
    return y


def prep_qk_int8(q: torch.Tensor, k: torch.Tensor, *, perm: torch.Tensor | None = None,
                 km: torch.Tensor | None = None, mean_numel: tuple[int, int] | None = None):
    """Sage per-thread INT8 Q/K after K channel-mean smoothing (HND inputs).

    Returns (q8, qs, k8, ks, km).  ``km`` ([B,H,1,D], input dtype) is computed
    on the device unless given.  ``mean_numel`` = (outputs, inputs) element
    counts of the logical mean, reproducing torch's CUDA mean factor.
    """
    _require_cuda("prep_qk_int8", q, k, perm, km)
    q, k = _rowmajor(q), _rowmajor(k)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    dt = _DT[q.dtype]
    dev = q.device
    q8 = torch.empty((B, H, Sq, D), dtype=torch.int8, device=dev)
    k8 = torch.empty((B, H, Sk, D), dtype=torch.int8, device=dev)
    qs = torch.empty((B, H, (Sq + 63) // 64 * 32), dtype=torch.float32, device=dev)
    ks = torch.empty((B, H, (Sk + 127) // 128 * 4), dtype=torch.float32, device=dev)
    km_out = torch.empty((B, H, 1, D), dtype=q.dtype, device=dev)
    km_in = None
    if km is not None:
        km_in = km.reshape(B, H, 1, D).to(q.dtype).contiguous()
    perm = _perm("prep_qk_int8", perm, B, H, Sk)
    lib = N.load()
    wsb = lib.vc_prep_qk_workspace_bytes(B, H, Sk, D)
    ws = _workspace(wsb, dev)
    n_out, n_in = mean_numel if mean_numel is not None else (0, 0)
    with torch.cuda.device(dev):
        N.check(lib.vc_prep_qk_int8(_p(q), _p(k), dt, B, H, Sq, Sk, D, q.stride(0), q.stride(1), q.stride(2),
                                    k.stride(0), k.stride(1), k.stride(2), _p(perm), _p(km_in), _p(km_out),
                                    n_out, n_in, _p(q8), _p(qs), _p(k8), _p(ks), _p(ws), ws.numel(), _stream(q)),
                "vc_prep_qk_int8")
    return q8, qs, k8, ks, km_out


def prep_qk_hadamard(q: torch.Tensor, k: torch.Tensor, *, perm: torch.Tensor | None = None, k_smooth: bool = True,
                     k_quant_block: int = 256, km: torch.Tensor | None = None):
    """The Config contract's own Q/K format (qk_hadamard=True): K centred by
    its FP32 channel mean (``k_smooth``), Q and K rotated by the normalised
    Sylvester transform, E4M3 block payloads with one scale per 128 Q rows
    and per ``k_quant_block`` K rows (HND inputs).

    Returns (q8, qs, k8, ks, km): q8/k8 float8_e4m3fn [B,H,S,D] (k8 rows in
    permutation order), qs [B,H,ceil(Sq/128)], ks [B,H,ceil(Sk/k_quant_block)]
    FP32, km [B,H,D] FP32 (None without ``k_smooth``).  ``km`` is computed on
    the device unless given.
    """
    _require_cuda("prep_qk_hadamard", q, k, perm, km)
    q, k = _rowmajor(q), _rowmajor(k)
    B, H, Sq, D = q.shape
    Sk = k.shape[2]
    if k.shape[:2] != (B, H) or k.shape[3] != D:
        raise ValueError("Q/K batch, heads and head dim must match")
    dev = q.device
    q8 = torch.empty((B, H, Sq, D), dtype=torch.float8_e4m3fn, device=dev)
    k8 = torch.empty((B, H, Sk, D), dtype=torch.float8_e4m3fn, device=dev)
    kqb = int(k_quant_block)
    qs = torch.empty((B, H, (Sq + 127) // 128), dtype=torch.float32, device=dev)
    ks = torch.empty((B, H, max(1, (Sk + kqb - 1) // max(kqb, 1))), dtype=torch.float32, device=dev)
    km_in = None if km is None else km.reshape(B, H, D).to(torch.float32).contiguous()
    km_out = torch.empty((B, H, D), dtype=torch.float32, device=dev) if k_smooth else None
    perm = _perm("prep_qk_hadamard", perm, B, H, Sk)
    lib = N.load()
    wsb = lib.vc_prep_qk_hadamard_workspace_bytes(B, H, Sq, Sk, D, kqb)
    if wsb < 0:
        raise ValueError("k_quant_block must be a multiple of 128 in [128, 4096]")
    ws = _workspace(wsb, dev)
    with torch.cuda.device(dev):
        N.check(lib.vc_prep_qk_hadamard_e4m3(_p(q), _p(k), _DT[q.dtype], B, H, Sq, Sk, D, q.stride(0), q.stride(1),
                                             q.stride(2), k.stride(0), k.stride(1), k.stride(2), _p(perm),
                                             int(bool(k_smooth)), _p(km_in), _p(km_out), kqb, _p(q8), _p(qs),
                                             _p(k8), _p(ks), _p(ws), ws.numel(), _stream(q)),
                "vc_prep_qk_hadamard_e4m3")
    return q8, qs, k8, ks, km_out


def prep_v_channel(v: torch.Tensor, *, perm: torch.Tensor | None = None):
    """Unsmoothed per-channel E4M3 V: (v8 [B,H,D,Npad] float8_e4m3fn, vs [B,H,D])."""
    _require_cuda("prep_v_channel", v, perm)
    v = _rowmajor(v)
    B, H, S, D = v.shape
    npad = (S + 127) // 128 * 128
    v8 = torch.empty((B, H, D, npad), dtype=torch.uint8, device=v.device)
    vs = torch.empty((B, H, D), dtype=torch.float32, device=v.device)
    perm = _perm("prep_v_channel", perm, B, H, S)
    lib = N.load()
    ws = _workspace(lib.vc_prep_v_channel_workspace_bytes(B, H, S, D), v.device)
    with torch.cuda.device(v.device):
        N.check(lib.vc_prep_v_channel(_p(v), _DT[v.dtype], B, H, S, D, v.stride(0), v.stride(1), v.stride(2),
                                      _p(perm), _p(v8), _p(vs), _p(ws), ws.numel(), _stream(v)),
                "vc_prep_v_channel")
    return v8.view(torch.float8_e4m3fn), vs


def prep_v_blocks(v: torch.Tensor, *, perm: torch.Tensor | None = None, channel_scale: bool = True,
                  demean: bool = True):
    """Smoothed V: (v8 [B,H,D,Npad] e4m3, vs [B,H,D] or [B,H,T,D], means fp16 [B,H,T,D]).

    ``demean=False`` keeps block means at zero (per-block amax scaling only)."""
    _require_cuda("prep_v_blocks", v, perm)
    v = _rowmajor(v)
    B, H, S, D = v.shape
    tiles = (S + 127) // 128
    v8 = torch.empty((B, H, D, tiles * 128), dtype=torch.uint8, device=v.device)
    vs = torch.empty((B, H, D) if channel_scale else (B, H, tiles, D), dtype=torch.float32, device=v.device)
    means = torch.empty((B, H, tiles, D), dtype=torch.float16, device=v.device)
    perm = _perm("prep_v_blocks", perm, B, H, S)
    lib = N.load()
    ws = _workspace(lib.vc_prep_v_blocks_workspace_bytes(B, H, S, D), v.device)
    with torch.cuda.device(v.device):
        N.check(lib.vc_prep_v_blocks(_p(v), _DT[v.dtype], B, H, S, D, v.stride(0), v.stride(1), v.stride(2),
                                     _p(perm), int(channel_scale), int(demean), _p(v8), _p(vs), _p(means), _p(ws),
                                     ws.numel(),
                                     _stream(v)), "vc_prep_v_blocks")
    return v8.view(torch.float8_e4m3fn), vs, means


def group_values(v: torch.Tensor, clusters: int = 8, iterations: int = 2, *, centers: torch.Tensor | None = None,
                 debug: bool = False):
    """Lloyd grouping of V tokens; returns the stable int64 permutation
    [B,H,S] (and, with ``debug``, int32 labels and the FP32 centres used by
    the final assignment).  ``centers`` warm-starts the iteration."""
    _require_cuda("group_values", v, centers)
    v = _rowmajor(v)
    B, H, S, D = v.shape
    count = min(clusters, S)
    perm = torch.empty((B, H, S), dtype=torch.int64, device=v.device)
    labels = torch.empty((B, H, S), dtype=torch.int32, device=v.device) if debug else None
    centers_in = None
    if centers is not None:
        if tuple(centers.shape) != (B, H, count, D):
            raise ValueError(f"centers must have shape {(B, H, count, D)}")
        centers_in = centers.to(torch.float32).contiguous()
    centers = torch.empty((B, H, count, D), dtype=torch.float32, device=v.device) if debug else None
    lib = N.load()
    ws = _workspace(lib.vc_group_values_workspace_bytes(B, H, S, D, clusters), v.device)
    with torch.cuda.device(v.device):
        N.check(lib.vc_group_values(_p(v), _DT[v.dtype], B, H, S, D, v.stride(0), v.stride(1), v.stride(2),
                                    int(clusters), int(iterations), _p(centers_in), _p(perm), _p(labels),
                                    _p(centers), _p(ws),
                                    ws.numel(), _stream(v)), "vc_group_values")
    return (perm, labels, centers) if debug else perm


def attention_fwd(q8, qs, k8, ks, v8, vs, means, *, out_dtype=torch.bfloat16, sm_scale: float | None = None,
                  expcast: bool = True, block_values: bool = False, out: torch.Tensor | None = None,
                  unit_range: tuple[int, int] | None = None, k_quant_block: int = 256,
                  control: str = "sage") -> torch.Tensor:
    """Fused attention on prepared payloads.  Returns ``out`` [B,H,Sq,D].

    ``expcast``: True = ExpCast with the reference's folded affine encoder
    (its default H200 kernel), ``"exact"`` = the unfused decoded-payload
    contract, False = the FP8-P control with ``control`` "sage" (Sage's
    scaling, vc_reference.py:56-64) or "config" (the Config contract's
    P8 = e4m3(256 exp(s - max)), core.py:357-360).

    ``unit_range`` = [begin, end) over units (b*H+h)*ceil(Sq/128)+q_tile
    computes only that shard (rows outside it are left untouched).

    Q/K payloads from ``prep_qk_hadamard`` (float8_e4m3fn) select the E4M3
    block-QK kernels; ``k_quant_block`` is then their K scale block.
    Per-block V scales (``vs`` [B,H,T,D]) need ``block_values``.
    """
    _require_cuda("attention_fwd", q8, k8, v8)
    B, H, Sq, D = q8.shape
    Sk = k8.shape[2]
    if out is None:
        out = torch.empty((B, H, Sq, D), dtype=out_dtype, device=q8.device)
    if out.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("attention output must be FP16, BF16 or FP32")
    scale = D ** -0.5 if sm_scale is None else float(sm_scale)
    if not (math.isfinite(scale) and scale > 0):
        raise ValueError("sm_scale must be positive and finite")
    if vs.dim() == 4 and not block_values:
        raise ValueError("per-block V scales need block_values=True")
    if control not in ("sage", "config"):
        raise ValueError("control must be 'sage' or 'config'")
    vs_per_block = bool(block_values and vs.dim() == 4)
    mode = 2 if expcast == "exact" else 1 if expcast else (3 if control == "config" else 0)
    ub, ue = unit_range if unit_range is not None else (0, -1)
    lib = N.load()
    if q8.dtype == torch.float8_e4m3fn:
        if k8.dtype != torch.float8_e4m3fn:
            raise ValueError("E4M3 Q needs E4M3 K payloads")
        with torch.cuda.device(q8.device):
            N.check(lib.vc_attention_fwd_e4m3qk(_p(q8), _p(qs), _p(k8), _p(ks), _p(v8.view(torch.uint8)), _p(vs),
                                                _p(means) if block_values else None, _p(out), _DT[out.dtype], B, H,
                                                Sq, Sk, D, out.stride(0), out.stride(1), out.stride(2), mode,
                                                int(block_values), int(vs_per_block), int(k_quant_block), scale,
                                                int(ub), int(ue), _stream(q8)), "vc_attention_fwd_e4m3qk")
        return out
    with torch.cuda.device(q8.device):
        N.check(lib.vc_attention_fwd(_p(q8), _p(qs), _p(k8), _p(ks), _p(v8.view(torch.uint8)), _p(vs),
                                     _p(means) if block_values else None, _p(out), _DT[out.dtype], B, H, Sq, Sk, D,
                                     out.stride(0), out.stride(1), out.stride(2), mode, int(block_values),
                                     int(vs_per_block), scale, int(ub), int(ue), _stream(q8)), "vc_attention_fwd")
    return out


def attention_plan(qtiles: int, unit_range: tuple[int, int], sms: int) -> dict:
    """How ``attention_fwd`` spreads a unit range over its ExpCast kernels
    (channel-scaled V, the default kernel choice), from the library's own rule
    (``vc_attention_plan``; host arithmetic, no device needed).

    One paired-tile CTA per SM takes two consecutive Q tiles of a head; if the
    last wave of pairs is at most half full on ``sms`` SMs, those pairs' units
    run on the alternating-tile kernel after the full waves.
    Returns ``{"pairs", "tail_units", "tail_begin", "launches"}``.
    """
    ub, ue = unit_range
    out = (C.c_int64 * 4)()
    N.check(N.load().vc_attention_plan(int(qtiles), int(ub), int(ue), int(sms), out), "vc_attention_plan")
    return {"pairs": out[0], "tail_units": out[1], "tail_begin": out[2], "launches": out[3]}


def kernel_resources(head_dim: int = 128) -> dict:
    arr = (C.c_int64 * 4)()
    N.check(N.load().vc_kernel_resources(head_dim, arr), "vc_kernel_resources")
    return {"registers_per_thread": arr[0], "static_shared_bytes": arr[1], "dynamic_shared_bytes": arr[2],
            "threads": arr[3]}


def tensor_peak(kind: str = "i8", n: int = 256, iters: int = 20000, device=None, repeats: int = 5,
                a_tmem: bool = False, issuers: int = 1) -> dict:
    """Measured dense tensor-core rate of this GPU for ``kind`` "i8"
    (tcgen05 kind::i8) or "e4m3" (kind::f8f6f4): one CTA per SM issuing
    M=128 x n x K=32 MMAs from shared memory, CUDA-event timed, best of
    ``repeats`` launches (``a_tmem``: A from tensor memory; ``issuers``
    warps issuing at once, each into its own accumulator).  Returns TOPS
    and the issue/completion cycles per MMA instruction of CTA 0."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    stamps = torch.zeros(3 * sms, dtype=torch.int64, device=dev)
    k = {"i8": 0, "e4m3": 1}[kind]
    lib = N.load()
    best = None
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        for _ in range(repeats + 1):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            N.check(lib.vc_tensor_peak(k, int(n), int(iters), sms, int(bool(a_tmem)), int(issuers), _p(stamps),
                                      st.cuda_stream),
                    "vc_tensor_peak")
            e1.record(st)
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
    s = stamps.view(sms, 3).cpu()
    if not bool((s[:, 2] == 1).all()):
        raise RuntimeError("vc_tensor_peak: a CTA's completion wait timed out")
    ops_total = 2.0 * 128 * n * 32 * 4 * iters * issuers * sms
    n_mma = 4 * iters
    return {"kind": kind, "n": n, "tops": ops_total / (best * 1e-3) / 1e12, "ms": best, "ctas": sms,
            "issue_cycles_per_mma": float(s[0, 0]) / n_mma, "cycles_per_mma": float(s[0, 1]) / n_mma}


ERR_WAIT_SELFTEST = 0x100


def wait_timeout_selftest(budget_ns: int = 5_000_000, device=None) -> dict:
    """Make a device wait run out on purpose: one warp waits, through the
    bounded mbarrier wait all kernels use, for a phase nothing completes.
    Returns whether the wait reported success (it must not), the kernel's
    duration and the device error word read afterwards (bit 0x100 set, then
    cleared)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flag = torch.full((1,), -1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        N.check(N.load().vc_selftest_wait_timeout(int(budget_ns), _p(flag), st.cuda_stream),
                "vc_selftest_wait_timeout")
        e1.record(st)
        e1.synchronize()
    return {"wait_ok": int(flag.item()), "ms": e0.elapsed_time(e1), "error_word": error_word(dev.index, clear=True)}


def error_word(device: int = 0, clear: bool = True) -> int:
    return N.error_word(device, clear)
