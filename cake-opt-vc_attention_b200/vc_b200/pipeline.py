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
