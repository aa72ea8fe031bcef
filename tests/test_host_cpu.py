"""Host-side checks that need no GPU.

* The C-ABI library loads and exports every function ``include/vc_b200.h``
  declares, and rejects bad arguments on the host (before any CUDA call).
* ``sageattn_vc`` / ``forward_prepared`` keep the reference's ValueError
  contract and raise before the native library is touched (mirrors the
  reference's tests/test_sage_vc.py rejection tests).
* Multi-GPU partitioning: unit shards cover the work exactly once, and the
  optional all-gather reassembles the output (gloo, world size 2, CPU).
"""
import ctypes as C
import os
import re
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "vc_b200.h"


@pytest.fixture(scope="module")
def lib():
    from vc_b200 import _native as N
    from vc_b200 import build as B
    if not N.LIB_PATH.exists():
        B.build()
    return N.load()


def _declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(vc_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_function(lib):
    names = _declared_functions()
    assert len(names) >= 16, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared in vc_b200.h but not exported: {missing}"


def test_binding_signatures_cover_the_header():
    from vc_b200 import _native as N
    assert sorted(N.SIGNATURES) == _declared_functions()


def test_identity(lib):
    assert lib.vc_api_version() == 1
    assert b"sm_100a" in lib.vc_build_info()


def _last(lib):
    return lib.vc_last_error().decode()


def test_c_abi_rejects_bad_arguments_on_host(lib):
    from vc_b200 import _native as N
    p = C.c_void_p(1 << 20)                          # never dereferenced: rejected first
    # head dim 96
    rc = lib.vc_prep_v_channel(p, N.VC_DTYPE_BF16, 1, 2, 300, 96, 2 * 300 * 96, 300 * 96, 96, None, p, p, p,
                               1 << 20, None)
    assert rc == N.VC_ERR_ARG and "head dim" in _last(lib)
    # unknown dtype
    rc = lib.vc_prep_v_channel(p, 7, 1, 2, 300, 128, 0, 0, 128, None, p, p, p, 1 << 20, None)
    assert rc == N.VC_ERR_ARG and "dtype" in _last(lib)
    # misaligned input
    rc = lib.vc_prep_v_channel(C.c_void_p((1 << 20) + 2), N.VC_DTYPE_BF16, 1, 2, 300, 128, 2 * 300 * 128,
                               300 * 128, 128, None, p, p, p, 1 << 20, None)
    assert rc == N.VC_ERR_ARG and "16-byte" in _last(lib)
    # workspace too small
    rc = lib.vc_prep_v_channel(p, N.VC_DTYPE_BF16, 1, 2, 300, 128, 2 * 300 * 128, 300 * 128, 128, None, p, p, p,
                               16, None)
    assert rc == N.VC_ERR_WORKSPACE and "workspace" in _last(lib)
    # static-scratch variant beyond its 1 MiB array
    rc = lib.vc_prep_v_channel_static(p, N.VC_DTYPE_BF16, 1, 2049, 128, 128, 2049 * 128 * 128, 128 * 128, 128,
                                      None, p, p, None)
    assert rc == N.VC_ERR_WORKSPACE and "static array" in _last(lib)
    # attention: non-positive scale, per-block scales without block values
    args = [p] * 7 + [p, N.VC_DTYPE_BF16, 1, 2, 300, 300, 128, 2 * 300 * 128, 300 * 128, 128]
    assert lib.vc_attention_fwd(*args, 1, 0, 0, 0.0, 0, -1, None) == N.VC_ERR_ARG
    assert "sm_scale" in _last(lib)
    assert lib.vc_attention_fwd(*args, 1, 0, 1, 0.125, 0, -1, None) == N.VC_ERR_ARG
    assert "block_values" in _last(lib)
    assert lib.vc_kernel_resources(96, None) == N.VC_ERR_ARG
    out4 = (C.c_int64 * 4)()
    assert lib.vc_attention_plan(0, 0, 1, 148, out4) == N.VC_ERR_ARG and "qtiles" in _last(lib)
    assert lib.vc_attention_plan(295, 5, 4, 148, out4) == N.VC_ERR_ARG
    assert lib.vc_attention_plan(295, 0, 10, 148, None) == N.VC_ERR_ARG
    # failure-detection self-test budget and tensor-peak probe shapes
    assert lib.vc_selftest_wait_timeout(10, None, None) == N.VC_ERR_ARG and "budget_ns" in _last(lib)
    assert lib.vc_tensor_peak(0, 136, 1, 1, 0, 1, None, None) == N.VC_ERR_ARG
    assert lib.vc_tensor_peak(0, 256, 1, 1, 1, 2, None, None) == N.VC_ERR_ARG   # accumulators overlap A


def test_e4m3_qk_entries_reject_bad_arguments_on_host(lib):
    """The Hadamard E4M3 Q/K prep and its attention entry validate on the
    host before any device use."""
    from vc_b200 import _native as N
    p = C.c_void_p(1 << 20)                          # never dereferenced: rejected first
    st = (2 * 300 * 128, 300 * 128, 128)
    prep = lambda kqb, ws=1 << 24: lib.vc_prep_qk_hadamard_e4m3(
        p, p, N.VC_DTYPE_BF16, 1, 2, 300, 300, 128, *st, *st, None, 1, None, None, kqb, p, p, p, p, p, ws, None)
    assert prep(200) == N.VC_ERR_ARG and "k_quant_block" in _last(lib)
    assert prep(8192) == N.VC_ERR_ARG and "k_quant_block" in _last(lib)
    assert prep(256, ws=16) == N.VC_ERR_WORKSPACE and "workspace" in _last(lib)
    assert lib.vc_prep_qk_hadamard_workspace_bytes(1, 2, 300, 300, 128, 100) < 0
    assert lib.vc_prep_qk_hadamard_workspace_bytes(1, 2, 300, 300, 128, 256) > 0
    args = [p] * 7 + [p, N.VC_DTYPE_BF16, 1, 2, 300, 300, 128, 2 * 300 * 128, 300 * 128, 128]
    assert lib.vc_attention_fwd_e4m3qk(*args, 4, 0, 0, 256, 0.125, 0, -1, None) == N.VC_ERR_ARG
    assert "expcast" in _last(lib)
    assert lib.vc_attention_fwd_e4m3qk(*args, 1, 0, 1, 256, 0.125, 0, -1, None) == N.VC_ERR_ARG
    assert "block_values" in _last(lib)
    assert lib.vc_attention_fwd_e4m3qk(*args, 1, 0, 0, 100, 0.125, 0, -1, None) == N.VC_ERR_ARG
    assert lib.vc_attention_fwd_e4m3qk(*args, 1, 0, 0, 256, -1.0, 0, -1, None) == N.VC_ERR_ARG
    assert "sm_scale" in _last(lib)


def test_status_codes_map_to_exceptions():
    from vc_b200 import _native as N
    N.check(N.VC_OK, "x")
    with pytest.raises(ValueError):
        N.check(N.VC_ERR_ARG, "x")
    with pytest.raises(ValueError):
        N.check(N.VC_ERR_WORKSPACE, "x")
    with pytest.raises(RuntimeError):
        N.check(N.VC_ERR_LAUNCH, "x")


# --------------------------------------------------------------- API contract

@pytest.fixture
def api(monkeypatch):
    from sageattention_local import vc

    def forbidden(*a, **k):
        raise AssertionError("the native library must not be reached")

    monkeypatch.setattr(vc, "_extension", forbidden)
    return vc


@pytest.mark.parametrize("kwargs,match", [
    ({"is_causal": True}, "noncausal"), ({"return_lse": True}, "LSE"),
    ({"tensor_layout": "XYZ"}, "tensor_layout"), ({"expcast": 1}, "bool"),
    ({"v_smooth": 0}, "bool"),
    ({"clusters": 0}, "clustering"), ({"clusters": 257}, "clustering"), ({"iterations": True}, "clustering"),
    ({"iterations": 101}, "clustering"),
    ({"kernel_mode": "unknown"}, "kernel_mode"),
    ({"v_scale_mode": "unknown"}, "v_scale_mode"),
    ({"grouping_mode": "unknown"}, "grouping_mode"),
])
def test_unsupported_modes_rejected_before_native_dispatch(api, kwargs, match):
    q = torch.zeros(1, 2, 5, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match=match):
        api.sageattn_vc(q, q, q, **kwargs)


def test_gqa_cpu_and_mixed_dtypes_are_not_silent_fallbacks(api):
    q = torch.zeros(1, 2, 5, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="GQA"):
        api.sageattn_vc(q, q[:, :1], q[:, :1])
    with pytest.raises(ValueError, match="matching"):
        api.sageattn_vc(q, q.float(), q)
    with pytest.raises(ValueError, match="D=64/128"):
        api.sageattn_vc(q[..., :32], q[..., :32], q[..., :32])
    with pytest.raises(ValueError, match="four-dimensional"):
        api.sageattn_vc(q[0], q[0], q[0])
    with pytest.raises(ValueError, match="no CPU/reference fallback"):
        api.sageattn_vc(q, q, q)


def test_shared_history_rejects_d64_before_native_dispatch(api):
    q = torch.zeros(1, 1, 65, 64, dtype=torch.bfloat16)
    assert api.HISTORY_CANDIDATES
    for mode in api.HISTORY_CANDIDATES:
        with pytest.raises(ValueError, match="D128"):
            api.sageattn_vc(q, q, q, v_smooth=False, kernel_mode=mode)


def test_every_documented_kernel_mode_is_accepted_or_rejected_like_the_reference(api):
    q = torch.zeros(1, 2, 5, 128, dtype=torch.float16)
    modes = ["optimized", "vc15", "vc14", "vc13_overlap", "vc13_serial", "vc12", "vc11", "vc10", "vc9", "vc7",
             "vc6", "vc4", *api.SAGE_LAYOUT_MODES]
    for mode in modes:
        sched = api.SAGE_LAYOUT_MODES.get(mode, 0)
        kw = {"kernel_mode": mode, "v_smooth": False}
        if 6 <= sched <= 9:
            kw["expcast"] = True
        elif sched in (3, 4):
            kw["expcast"] = False
        # valid combinations fail only at the device check (CPU tensors)
        with pytest.raises(ValueError, match="no CPU/reference fallback"):
            api.sageattn_vc(q, q, q, **kw)
    for mode, sched in api.SAGE_LAYOUT_MODES.items():
        if mode in api.UNIFIED_MODES:
            continue
        with pytest.raises(ValueError, match="v_smooth=False"):
            api.sageattn_vc(q, q, q, kernel_mode=mode)
        if 6 <= sched <= 9:
            with pytest.raises(ValueError, match="expcast=True"):
                api.sageattn_vc(q, q, q, kernel_mode=mode, expcast=False, v_smooth=False)
        if sched in (3, 4):
            with pytest.raises(ValueError, match="expcast=False"):
                api.sageattn_vc(q, q, q, kernel_mode=mode, v_smooth=False)


# ---------------------------------------------------------------- multi-GPU

@pytest.mark.parametrize("B,H,S", [(1, 28, 37741), (2, 40, 75600), (1, 2, 300), (1, 1, 100), (2, 3, 129)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_units_and_rows_exactly_once(B, H, S, world):
    from vc_b200 import parallel as P
    qtiles = (S + 127) // 128
    total = B * H * qtiles
    prev_u, prev_r = 0, 0
    sizes = []
    for r in range(world):
        s = P.shard(B, H, S, world, r)
        assert s.unit_begin == prev_u
        rb, re_ = P.shard_rows(s, S)
        assert rb == prev_r and re_ >= rb
        if s.num_units:
            assert s.bh_begin == s.unit_begin // qtiles and s.bh_end == (s.unit_end - 1) // qtiles + 1
            lb, le = s.local_units
            assert 0 <= lb < le <= (s.bh_end - s.bh_begin) * qtiles
            # cut between pairs: every range starts on a pair's first tile
            assert s.unit_begin % qtiles % 2 == 0
        prev_u, prev_r = s.unit_end, re_
        # pairs met by the range
        sizes.append(len({(u // qtiles, u % qtiles // 2) for u in range(s.unit_begin, s.unit_end)}))
    assert prev_u == total and prev_r == B * H * S
    assert max(sizes) - min(sizes) <= 1


def _pair_units(pair, qtiles):
    qpairs = (qtiles + 1) // 2
    bh, i = divmod(pair, qpairs)
    return [bh * qtiles + t for t in (2 * i, 2 * i + 1) if t < qtiles]


@pytest.mark.parametrize("B,H,S", [(1, 28, 37741), (2, 40, 75600), (2, 24, 16384), (1, 2, 19200), (1, 1, 100),
                                   (2, 3, 129)])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_attention_plan_splits_each_shard_into_full_waves_and_a_short_tail(B, H, S, world):
    """The paired-tile kernel takes whole waves of pairs (one CTA per SM) and
    the alternating-tile kernel the units of a last wave that is at most half
    full; together they cover the shard's units exactly once."""
    from vc_b200 import ops, parallel as P
    sms = 148
    qtiles = (S + 127) // 128
    for r in range(world):
        s = P.shard(B, H, S, world, r)
        ub, ue = s.unit_begin, s.unit_end
        plan = ops.attention_plan(qtiles, (ub, ue), sms)
        if ub == ue:
            assert plan["launches"] == 0
            continue
        pb = (ub // qtiles) * ((qtiles + 1) // 2) + (ub % qtiles) // 2
        paired = {u for i in range(plan["pairs"]) for u in _pair_units(pb + i, qtiles) if ub <= u < ue}
        tail = set(range(plan["tail_begin"], ue))
        assert not paired & tail and paired | tail == set(range(ub, ue))
        assert plan["tail_units"] == len(tail) <= sms
        if plan["tail_units"]:
            assert plan["pairs"] % sms == 0
        else:
            assert plan["pairs"] % sms == 0 or plan["pairs"] % sms > sms // 2
    # config 2 on 8 GPUs: 518 pairs per rank = 3 full waves + a tail of 74 pairs (at most 148 tiles)
    p8 = [ops.attention_plan(295, (P.shard(1, 28, 37741, 8, r).unit_begin, P.shard(1, 28, 37741, 8, r).unit_end),
                             sms) for r in range(8)]
    assert all(p["pairs"] == 444 and p["launches"] == 2 and 147 <= p["tail_units"] <= 148 for p in p8)
    # on 2 and 4 GPUs the pairs fill 14 and 7 waves exactly
    for world, waves in ((2, 14), (4, 7)):
        for r in range(world):
            s = P.shard(1, 28, 37741, world, r)
            assert ops.attention_plan(295, (s.unit_begin, s.unit_end), sms)["pairs"] == waves * sms
    # config 2 on one GPU: 4144 pairs = 28 full waves, no tail
    assert ops.attention_plan(295, (0, 28 * 295), sms) == {"pairs": 4144, "tail_units": 0, "tail_begin": 8260,
                                                         "launches": 1}


def _gather_worker(rank, world, port, B, H, S, D, q):
    import torch.distributed as dist
    from vc_b200 import parallel as P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        full = torch.arange(B * H * S * D, dtype=torch.float32).reshape(B, H, S, D)
        s = P.shard(B, H, S, world, rank)
        local = P.head_slice(full, s).clone()
        # poison the rows this rank does not own: gather must not read them
        rb, re_ = P.shard_rows(s, S)
        flat = local.reshape(-1, D)
        off = s.bh_begin * S
        flat[:rb - off] = float("nan")
        flat[re_ - off:] = float("nan")
        out = P.gather_rows(local, s, B, H, S)
        q.put((rank, bool(torch.equal(out, full))))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("B,H,S", [(1, 3, 300), (2, 2, 129)])
def test_gather_rows_gloo_world2(B, H, S):
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, B, H, S, 8, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}, results


def test_sharded_host_pipeline_rejects_bad_arguments():
    """Argument checks of sharded_attention_host happen before any device use."""
    from vc_b200.pipeline import sharded_attention_host
    x = torch.zeros(1, 2, 200, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        sharded_attention_host(x, x, x, x, (0, 5))          # 2 heads x 2 tiles = 4 units
    with pytest.raises(ValueError):
        sharded_attention_host(x, x, x, x, (3, 2))
    with pytest.raises(ValueError):
        sharded_attention_host(x, x, x[:, :1], x, (0, 1))
    with pytest.raises(ValueError):
        sharded_attention_host(x, x, x, x, (0, 1), chunk_heads=0)
    assert sharded_attention_host(x, x, x, x, (2, 2)) is x   # empty range: nothing to do
