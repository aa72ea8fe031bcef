"""Multi-GPU partitioning of the VC-attention path.

Work units are (b*H + h, q_tile) pairs flattened as ``(b*H+h)*ceil(Sq/128) +
q_tile``.  Every unit is independent given its head's full K/V payloads, so a
rank owns a contiguous unit range, prepares only the heads that range
touches (at most one extra head of redundant K/V preparation per boundary)
and computes its output rows locally.  Outputs stay sharded; an optional
NCCL all-gather assembles the full tensor.  No data-path collective.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    unit_begin: int      # global unit range [unit_begin, unit_end)
    unit_end: int
    bh_begin: int        # flattened (b*H+h) heads touched [bh_begin, bh_end)
    bh_end: int
    qtiles: int

    @property
    def local_units(self) -> tuple[int, int]:
        """Unit range relative to the first touched head."""
        off = self.bh_begin * self.qtiles
        return self.unit_begin - off, self.unit_end - off

    @property
    def num_units(self) -> int:
        return self.unit_end - self.unit_begin


def pair_unit(pair: int, qtiles: int) -> int:
    """First unit of ``pair`` (pairs are two consecutive Q tiles of one head,
    ``ceil(qtiles/2)`` per head; a head with an odd tile count ends in a
    one-tile pair)."""
    qpairs = (qtiles + 1) // 2
    bh, i = divmod(pair, qpairs)
    return bh * qtiles + 2 * i


def shard(B: int, H: int, Sq: int, world: int, rank: int) -> Shard:
    """Balanced contiguous split of the pair space (pair counts differ by
    <= 1), as a unit range.  The attention kernel runs one pair of Q tiles
    per CTA; cutting shards between pairs, never inside one, keeps every
    rank's pair count at its share (config 2 on 8 GPUs: 518 pairs each, where
    an even split of units gives some ranks 519)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    qtiles = (Sq + 127) // 128
    total = B * H * ((qtiles + 1) // 2)
    base, extra = divmod(total, world)
    pb = rank * base + min(rank, extra)
    pe = pb + base + (1 if rank < extra else 0)
    ub, ue = pair_unit(pb, qtiles), pair_unit(pe, qtiles)
    if ue > ub:
        bh0, bh1 = ub // qtiles, (ue - 1) // qtiles + 1
    else:
        bh0 = bh1 = min(ub // qtiles, B * H)
    return Shard(rank, world, ub, ue, bh0, bh1, qtiles)


def head_slice(x: torch.Tensor, s: Shard) -> torch.Tensor:
    """[B,H,S,D] -> [1, bh_end-bh_begin, S, D] view of the touched heads."""
    B, H = x.shape[:2]
    return x.reshape(1, B * H, *x.shape[2:])[:, s.bh_begin:s.bh_end]


def sharded_attention(q, k, v, s: Shard, *, expcast=True, v_smooth=False, clusters=8, iterations=2,
                      v_scale_mode="channel", sm_scale=None, out=None):
    """Prepare the shard's heads and compute its units (HND inputs).

    Returns the local output [1, nbh, Sq, D]; rows outside the shard's unit
    range are not written.
    """
    from sageattention_local.vc import prepare
    from . import ops
    qh, kh, vh = head_slice(q, s), head_slice(k, s), head_slice(v, s)
    # torch's CUDA mean factor over the full tensor, so shards match 1-GPU km
    mean_numel = (k.shape[0] * k.shape[1] * k.shape[3], k.numel())
    st = prepare(qh, kh, vh, expcast=expcast, v_smooth=v_smooth, clusters=clusters, iterations=iterations,
                 sm_scale=sm_scale, v_scale_mode=v_scale_mode, mean_numel=mean_numel)
    out_dtype = torch.float16 if q.dtype == torch.float16 else torch.bfloat16
    return ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], st["means"],
                             out_dtype=out_dtype, sm_scale=st["scale"], expcast=expcast, block_values=v_smooth,
                             out=out, unit_range=s.local_units)


def unit_rows(u: int, qtiles: int, Sq: int) -> int:
    """First row of unit ``u`` in the flattened [B*H*Sq] row space."""
    bh, qt = divmod(u, qtiles)
    return bh * Sq + qt * 128


def shard_rows(s: Shard, Sq: int) -> tuple[int, int]:
    """The shard's rows [row_begin, row_end) in the flattened [B*H*Sq] row
    space.  Consecutive units cover consecutive rows (a head's last tile is
    ragged, the next head starts right after it), so this range is
    contiguous."""
    if s.unit_end <= s.unit_begin:
        r = unit_rows(s.unit_begin, s.qtiles, Sq) if s.qtiles else 0
        return r, r
    last = s.unit_end - 1
    r1 = unit_rows(last, s.qtiles, Sq) + min(128, Sq - (last % s.qtiles) * 128)
    return unit_rows(s.unit_begin, s.qtiles, Sq), r1


def gather_rows(local: torch.Tensor, s: Shard, B: int, H: int, Sq: int, group=None) -> torch.Tensor:
    """Assemble the full [B,H,Sq,D] output from every rank's shard with one
    all-gather of equal-size row blocks (NCCL over NVLink on GPUs; gloo on
    CPU in tests).  ``local`` is the shard's [1, bh_end-bh_begin, Sq, D]
    output; only its own rows are read."""
    import torch.distributed as dist
    world = s.world
    D = local.shape[-1]
    spans = [shard_rows(shard(B, H, Sq, world, r), Sq) for r in range(world)]
    cap = max(e - b for b, e in spans)
    rb, re = spans[s.rank]
    off = s.bh_begin * Sq
    flat = local.reshape(-1, D)
    buf = torch.zeros(cap, D, dtype=local.dtype, device=local.device)
    buf[:re - rb] = flat[rb - off:re - off]
    allbuf = torch.empty(world * cap, D, dtype=local.dtype, device=local.device)
    if local.device.type == "cuda":
        dist.all_gather_into_tensor(allbuf, buf, group=group)
    else:
        dist.all_gather(list(allbuf.chunk(world)), buf, group=group)
    out = torch.empty(B * H * Sq, D, dtype=local.dtype, device=local.device)
    for r, (b, e) in enumerate(spans):
        out[b:e] = allbuf[r * cap:r * cap + (e - b)]
    return out.reshape(B, H, Sq, D)
