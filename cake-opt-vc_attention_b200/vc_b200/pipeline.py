"""Host-resident inputs: ``sageattn_vc`` on pinned host tensors with the PCIe
copies overlapped with the computation.

Heads are independent (every per-head statistic -- K mean, V scales,
grouping -- is computed within the head), so the call is split into chunks
of heads.  Chunk i is copied to the device on one stream, computed on a
second and copied back on a third while chunk i+1 is in flight; the result
equals one ``sageattn_vc`` call on the whole tensors bit for bit.
"""
from __future__ import annotations

import torch


_STREAMS: dict[int, tuple] = {}


def _chunks(n: int, size: int):
    return [(i, min(n, i + size)) for i in range(0, n, size)]


def _streams(device: torch.device):
    """The copy-in, compute and copy-out streams of ``device``, created once:
    PyTorch's caching allocator keeps a block pool per stream, so fresh
    streams on every call would send every chunk's allocations to cudaMalloc."""
    if device.index not in _STREAMS:
        _STREAMS[device.index] = tuple(torch.cuda.Stream(device) for _ in range(3))
    return _STREAMS[device.index]


def sageattn_vc_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None, *,
                     device=None, chunk_heads: int = 2, **kwargs) -> torch.Tensor:
    """``sageattn_vc`` on HND host tensors ``[B,H,S,D]`` (pinned for overlap).

    Writes the result into ``out`` (a host tensor, allocated pinned when
    omitted) and returns it once the device work has completed.  ``kwargs``
    are ``sageattn_vc``'s keyword arguments (``tensor_layout`` must stay HND).
    """
    from sageattention_local import sageattn_vc
    if kwargs.get("tensor_layout", "HND") != "HND":
        raise ValueError("sageattn_vc_host takes HND tensors")
    if any(x.device.type != "cpu" for x in (q, k, v)):
        raise ValueError("sageattn_vc_host takes host tensors; call sageattn_vc for device tensors")
    if q.ndim != 4 or k.shape != v.shape or q.shape[:2] != k.shape[:2]:
        raise ValueError("Q/K/V batch/heads/dim must match; GQA is unsupported")
    if chunk_heads < 1:
        raise ValueError("chunk_heads must be positive")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    B, H = q.shape[:2]
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    # flatten (B, H) so chunks are contiguous slices of heads
    qf, kf, vf, of = (x.reshape(B * H, *x.shape[2:]) for x in (q, k, v, out))
    h2d, comp, d2h = _streams(device)
    pending = []
    with torch.cuda.device(device):
        for a, b in _chunks(B * H, chunk_heads):
            with torch.cuda.stream(h2d):
                dq, dk, dv = (x[a:b].unsqueeze(0).to(device, non_blocking=True) for x in (qf, kf, vf))
                copied = torch.cuda.Event()
                copied.record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(copied)
                for t in (dq, dk, dv):
                    t.record_stream(comp)
                res = sageattn_vc(dq, dk, dv, **kwargs)
                done = torch.cuda.Event()
                done.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                res.record_stream(d2h)
                of[a:b].copy_(res[0], non_blocking=True)
            pending.append((dq, dk, dv, res))
        d2h.synchronize()
    return out


def sharded_attention_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                           unit_range: tuple[int, int], *, device=None, chunk_heads: int = 2, mean_numel=None,
                           expcast: bool = True, v_smooth: bool = False, clusters: int = 8, iterations: int = 2,
                           v_scale_mode: str = "channel", sm_scale: float | None = None) -> torch.Tensor:
    """One rank's share of the work on host-resident HND tensors ``[B,H,S,D]``.

    Computes the units ``[u0, u1)`` of the flattened ``(b*H+h)*ceil(S/128) +
    q_tile`` space and writes their rows into the host tensor ``out``; rows
    outside the range are not written.  Heads are processed in chunks with
    the copies overlapped as in ``sageattn_vc_host``; a chunk's K/V are
    always whole heads (the preparation is per head).  ``mean_numel`` is the
    torch mean factor of the full tensor (see ``prepare``), so a shard
    reproduces the single-call K mean.
    """
    from sageattention_local.vc import prepare
    from . import ops
    if any(x.device.type != "cpu" for x in (q, k, v, out)):
        raise ValueError("sharded_attention_host takes host tensors")
    if q.ndim != 4 or k.shape != v.shape or q.shape != k.shape or out.shape != q.shape:
        raise ValueError("Q/K/V/out must have the same [B,H,S,D] shape")
    if chunk_heads < 1:
        raise ValueError("chunk_heads must be positive")
    B, H, S, D = q.shape
    qtiles = (S + 127) // 128
    u0, u1 = (int(x) for x in unit_range)
    if not 0 <= u0 <= u1 <= B * H * qtiles:
        raise ValueError("unit_range outside [0, B*H*ceil(S/128)]")
    if u0 == u1:
        return out
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    qf, kf, vf = (x.reshape(B * H, S, D) for x in (q, k, v))
    of = out.view(B * H * S, D)
    h0, h1 = u0 // qtiles, (u1 - 1) // qtiles + 1

    def row(u):   # first row of unit u in the flattened [B*H*S] row space (u may equal the end)
        bh, qt = divmod(u, qtiles)
        return bh * S + min(qt * 128, S)

    h2d, comp, d2h = _streams(device)
    pending = []
    with torch.cuda.device(device):
        for a, b in _chunks(h1 - h0, chunk_heads):
            a, b = a + h0, b + h0
            lu0, lu1 = max(u0, a * qtiles) - a * qtiles, min(u1, b * qtiles) - a * qtiles
            with torch.cuda.stream(h2d):
                dq, dk, dv = (x[a:b].unsqueeze(0).to(device, non_blocking=True) for x in (qf, kf, vf))
                copied = torch.cuda.Event()
                copied.record(h2d)
            with torch.cuda.stream(comp):
                comp.wait_event(copied)
                for t in (dq, dk, dv):
                    t.record_stream(comp)
                st = prepare(dq, dk, dv, expcast=expcast, v_smooth=v_smooth, clusters=clusters,
                             iterations=iterations, sm_scale=sm_scale, v_scale_mode=v_scale_mode,
                             mean_numel=mean_numel)
                res = ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], st["means"],
                                        out_dtype=q.dtype, sm_scale=st["scale"], expcast=expcast,
                                        block_values=v_smooth, unit_range=(lu0, lu1))
                done = torch.cuda.Event()
                done.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                res.record_stream(d2h)
                r0, r1 = row(lu0), row(lu1)
                of[a * S + r0:a * S + r1].copy_(res.view(-1, D)[r0:r1], non_blocking=True)
            pending.append((dq, dk, dv, res))
        d2h.synchronize()
    return out
