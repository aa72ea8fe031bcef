"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bit-exact for INT8/E4M3/FP16 payloads and scales; attention outputs within
cos >= 0.9999 and rel-L2 <= 1e-3 of the decoded-payload oracle (the
tolerance stated by the reference's north star), also reported against FP32
dense softmax attention.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from inputs import qk_inputs, mixture_values

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
COS_MIN, REL_MAX = 0.9999, 1e-3


@pytest.fixture(scope="module")
def ops(cuda_device):
    from vc_b200 import ops as _ops
    from vc_b200 import _native
    _native.load()
    _ops.error_word(0, clear=True)
    yield _ops
    torch.cuda.synchronize()
    assert _ops.error_word(0, clear=True) == 0, "device error word set (a bounded wait timed out)"


def _np(t):
    return t.detach().cpu().numpy()


def test_expcast_codes_bit_exact(ops):
    f = np.load(GOLDEN / "expcast.npz")
    x = torch.from_numpy(f["shifted"]).cuda()
    assert np.array_equal(_np(ops.expcast_codes(x)), f["codes"])


@pytest.mark.parametrize("name", ["c1_fp32", "tail_bf16_d64", "tail_fp16_d128", "single_bf16", "outlier_bf16"])
def test_qk_int8_bit_exact_vs_reference_triton(ops, name):
    f = np.load(GOLDEN / f"qk_{name}.npz")
    dtype = getattr(torch, str(f["dtype"]))
    q, k, _ = qk_inputs(int(f["seed"]), tuple(f["shape"]), dtype, float(f["koff"]), float(f["outliers"]))
    km = torch.from_numpy(f["km"]).to(dtype).cuda()
    q8, qs, k8, ks, _ = ops.prep_qk_int8(q.cuda(), k.cuda(), km=km)
    torch.cuda.synchronize()
    assert np.array_equal(_np(q8), f["q8"])
    assert np.array_equal(_np(qs), f["qs"])
    assert np.array_equal(_np(k8), f["k8"])
    assert np.array_equal(_np(ks), f["ks"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 2, 1000, 128), (2, 3, 257, 64), (1, 1, 5000, 128)])
def test_k_mean_matches_torch_cuda_mean(ops, dtype, shape):
    q, k, _ = qk_inputs(11, shape, dtype, 3 ** 0.5)
    kc = k.cuda()
    ref = kc.mean(dim=2, keepdim=True)
    _, _, _, _, km = ops.prep_qk_int8(q.cuda(), kc, mean_numel=(shape[0] * shape[1] * shape[3], kc.numel()))
    # FP32 summation order differs from torch's.  For half/bfloat16 the
    # rounding to the input dtype hides it except for a tiny fraction of
    # channels (one ulp); FP32 means differ only in their last bits.
    if dtype != torch.float32:
        diff = (km.float() != ref.float()).float().mean().item()
        assert diff <= 0.02, diff
    torch.testing.assert_close(km.float(), ref.float(), rtol=1e-2 if dtype != torch.float32 else 1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_qk_int8_with_device_mean_and_permutation(ops, dtype):
    shape = (1, 2, 700, 128)
    q, k, _ = qk_inputs(12, shape, dtype, 3 ** 0.5)
    g = torch.Generator().manual_seed(3)
    perm = torch.stack([torch.randperm(700, generator=g) for _ in range(2)]).reshape(1, 2, 700)
    q8, qs, k8, ks, km = ops.prep_qk_int8(q.cuda(), k.cuda(), perm=perm.cuda())
    kp = k.gather(2, perm.unsqueeze(-1).expand_as(k))
    e_q8, e_qs, e_k8, e_ks = O.per_thread_int8(q, kp, km.cpu())
    assert np.array_equal(_np(q8), e_q8) and np.array_equal(_np(qs), e_qs)
    assert np.array_equal(_np(k8), e_k8) and np.array_equal(_np(ks), e_ks)


def _tie_heavy(seed, shape):
    """FP32 Q/K whose quotients x/scale land on (or next to) the .5 ties of the
    Sage rounding: every 2-row Q scale group and every 32-row K scale group
    holds one element 127*c (so scale = RN(RN(127c/127) + 1e-7)) and the rest
    are RN((k + 1/2) * scale) for random integers k."""
    g = np.random.default_rng(seed)
    B, H, S, D = shape
    f32 = np.float32

    def fill(x, rows):
        c = f32(g.uniform(0.01, 3.0))
        amax = f32(f32(127.0) * c)
        scale = f32(f32(amax / f32(127.0)) + f32(1e-7))
        k = g.integers(-126, 126, size=(len(rows), D)).astype(f32)
        x[rows] = ((k + f32(0.5)) * scale).astype(f32)
        x[rows[0], g.integers(0, D)] = amax * (1 if g.random() < 0.5 else -1)

    q = np.zeros(shape, f32)
    k = np.zeros(shape, f32)
    for b in range(B):
        for h in range(H):
            for blk in range(0, S, 16):
                for gg in range(8):
                    rows = [r for r in (blk + gg, blk + gg + 8) if r < S]
                    if rows:
                        fill(q[b, h], rows)
            for blk in range(0, S, 128):
                for tld in range(4):
                    rows = [r for i in range(16) for r in (blk + 8 * i + 2 * tld, blk + 8 * i + 2 * tld + 1) if r < S]
                    if rows:
                        fill(k[b, h], rows)
    return torch.from_numpy(q), torch.from_numpy(k)


@pytest.mark.parametrize("shape", [(1, 2, 1000, 128), (1, 1, 300, 64)])
def test_qk_int8_bit_exact_on_rounding_ties(ops, shape):
    q, k = _tie_heavy(7, shape)
    km = torch.zeros(shape[0], shape[1], 1, shape[3])
    q8, qs, k8, ks, _ = ops.prep_qk_int8(q.cuda(), k.cuda(), km=km.cuda())
    e_q8, e_qs, e_k8, e_ks = O.per_thread_int8(q, k, km)
    assert np.array_equal(_np(qs), e_qs) and np.array_equal(_np(ks), e_ks)
    assert np.array_equal(_np(q8), e_q8)
    assert np.array_equal(_np(k8), e_k8)


def test_out_of_range_permutation_is_reported(ops):
    """Permutation entries outside [0, S) are never dereferenced: those rows read
    as zeros and the error word carries the bad-index bit (0x80).  A permutation
    of the wrong shape is rejected on the host."""
    v = torch.randn(1, 2, 300, 128).to(torch.bfloat16).cuda()
    perm = torch.arange(300).repeat(1, 2, 1)
    perm[0, 1, 5] = 300                       # one past the end
    perm[0, 0, 7] = -1
    perm = perm.cuda()
    assert ops.error_word(0, clear=True) == 0
    ops.prep_v_channel(v, perm=perm)
    ops.prep_v_blocks(v, perm=perm)
    ops.prep_qk_int8(v, v, perm=perm)
    torch.cuda.synchronize()
    assert ops.error_word(0, clear=True) == 0x80
    for bad in (perm[0, 0], perm.float(), perm[:, :, :299]):
        with pytest.raises(ValueError, match="perm must be"):
            ops.prep_v_channel(v, perm=bad)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("n", [1, 127, 128, 129, 1000])
def test_v_channel_bit_exact(ops, dtype, dim, n):
    g = torch.Generator().manual_seed(n + dim)
    v = (torch.randn(2, 2, n, dim, generator=g) * 3).to(dtype)
    v[:, 1, :, 3] = 0                                       # all-zero channel -> zero-safe
    v8, vs = ops.prep_v_channel(v.cuda())
    e_v8, e_vs = O.v_channel_fp8(v.float().numpy())
    assert np.array_equal(_np(vs), e_vs)
    assert np.array_equal(_np(v8.view(torch.uint8)), e_v8)


def _value_cases(dtype, dim, n):
    g = torch.Generator().manual_seed(339)
    v = torch.randn(2, 2, n, dim, generator=g)
    for t, begin in enumerate(range(0, n, 128)):
        v[:, :, begin:begin + 128] = v[:, :, begin:begin + 128] * (t + 1) + t * 3
    v[..., 0] = 1.5
    v[..., 1] = -2.0
    return v.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("n", [1, 127, 128, 129, 257])
@pytest.mark.parametrize("channel", [False, True])
def test_v_blocks_bit_exact(ops, dtype, dim, n, channel):
    # the reference's 60-case preprocessing suite (scripts/validate_sage_vc.py:19-83)
    v = _value_cases(dtype, dim, n)
    v8, vs, means = ops.prep_v_blocks(v.cuda(), channel_scale=channel)
    e_v8, e_vs, e_means = O.v_blocks_fp8(v.float().numpy(), channel_scale=channel)
    assert np.array_equal(_np(vs), e_vs)
    assert np.array_equal(_np(means).view(np.uint16), e_means.view(np.uint16))
    assert np.array_equal(_np(v8.view(torch.uint8)), e_v8)


def test_v_blocks_large_mean_overflow_guard(ops):
    # reference tests/test_sage_vc_preprocess_cuda.py:48-65: near-constant
    # blocks with huge means must keep mean/scale finite in FP16
    v = torch.full((1, 1, 300, 64), 60000.0)
    v[..., ::7, :] += 0.5
    v8, vs, means = ops.prep_v_blocks(v.cuda(), channel_scale=True)
    e_v8, e_vs, e_means = O.v_blocks_fp8(v.numpy(), channel_scale=True)
    assert torch.isfinite(means.float()).all()
    assert np.array_equal(_np(vs), e_vs) and np.array_equal(_np(v8.view(torch.uint8)), e_v8)


def test_v_blocks_many_tiles_channel_reduction(ops):
    # > 32 tiles exercise the channel reduction (reference test :68-80)
    v = _value_cases(torch.bfloat16, 128, 128 * 40 + 3)
    v8, vs, means = ops.prep_v_blocks(v.cuda(), channel_scale=True)
    e_v8, e_vs, e_means = O.v_blocks_fp8(v.float().numpy(), channel_scale=True)
    assert np.array_equal(_np(vs), e_vs)
    assert np.array_equal(_np(v8.view(torch.uint8)), e_v8)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("n,count,iterations", [(1, 8, 2), (127, 3, 3), (129, 8, 2), (2049, 8, 2),
                                                # the wide path (9-256 effective centres)
                                                (1000, 16, 2), (300, 64, 3), (2049, 256, 2), (100, 200, 2),
                                                (20, 256, 1)])
def test_group_values_matches_fp64_lloyd(ops, dtype, dim, n, count, iterations):
    # well-separated clusters, as scripts/validate_sage_vc.py:86-117
    g = torch.Generator().manual_seed(883)
    c = min(n, count)
    ids = torch.from_numpy(O.linspace_ids(n, c))
    labels = torch.arange(n) % c
    labels[ids] = torch.arange(c)
    v = (labels.view(1, 1, n, 1) * 4 + torch.randn(2, 2, n, dim, generator=g) * .01).to(dtype)
    perm, lab, centers = ops.group_values(v.cuda(), count, iterations, debug=True)
    e_lab, e_centers = O.lloyd_fp64(v.float().numpy(), count, iterations)
    assert np.array_equal(_np(lab), e_lab)
    assert np.array_equal(_np(perm), O.stable_argsort(e_lab))
    np.testing.assert_allclose(_np(centers), e_centers, rtol=2e-5, atol=2e-6)


def test_group_values_stable_known_answer_and_constant(ops):
    labels = torch.tensor([2, 0, 1, 2, 1, 0])
    values = labels.float().reshape(1, 1, 6, 1).expand(2, 2, 6, 64).contiguous()
    perm = ops.group_values(values.cuda(), 3, 2)
    for p in _np(perm).reshape(-1, 6):
        assert p.tolist() == [0, 3, 2, 4, 1, 5]
    v = torch.full((2, 2, 257, 128), 2.)
    for count in (8, 100):   # fused and wide paths: all tokens tie, the lowest centre wins
        perm, lab, centers = ops.group_values(v.cuda(), count, 3, debug=True)
        assert int(lab.count_nonzero()) == 0
        assert torch.equal(perm.cpu(), torch.arange(257).expand(2, 2, 257))
        assert bool((centers == 2).all())



def _device_state(ops, q, k, v, *, expcast=True, v_smooth=False, v_scale_mode="channel", perm=None):
    """Prepare payloads on the GPU (bit-exact with the oracle) as a state dict."""
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    pc = perm.cuda() if perm is not None else None
    q8, qs, k8, ks, km = ops.prep_qk_int8(qc, kc, perm=pc)
    if v_smooth:
        v8, vs, means = ops.prep_v_blocks(vc, perm=pc, channel_scale=v_scale_mode == "channel")
    else:
        v8, vs = ops.prep_v_channel(vc)
        means = torch.empty(0, dtype=torch.float16, device="cuda")
    return {"q": q8, "k": k8, "v": v8, "qs": qs, "ks": ks, "vs": vs, "means": means, "expcast": expcast,
            "block_values": v_smooth, "scale": q.shape[-1] ** -0.5, "km": km}


def _cpu_state(st):
    return {**{k: (v.cpu() if torch.is_tensor(v) else v) for k, v in st.items()},
            "v": _np(st["v"].view(torch.uint8)), "means": _np(st["means"]) if st["block_values"] else None}


ATT_CASES = [
    # name, shape, dtype, koff, expcast, v_smooth, v_scale_mode
    ("c1_d128_fp32", (1, 2, 1024, 128), torch.float32, 2 ** 0.5, True, False, "channel"),
    ("tail_d64_bf16", (1, 2, 300, 64), torch.bfloat16, 3 ** 0.5, True, False, "channel"),
    ("tail_d128_fp16", (2, 1, 333, 128), torch.float16, 1.0, True, False, "channel"),
    ("single_key", (1, 1, 1, 128), torch.bfloat16, 0.0, True, False, "channel"),
    ("smooth_channel", (1, 2, 300, 128), torch.bfloat16, 3 ** 0.5, True, True, "channel"),
    ("smooth_block_d64", (2, 1, 257, 64), torch.float16, 1.0, True, True, "block"),
    ("control_no_expcast", (1, 1, 129, 128), torch.bfloat16, 1.0, False, False, "channel"),
    ("control_smooth", (1, 1, 260, 64), torch.bfloat16, 1.0, False, True, "channel"),
    # block means on the tensor-memory kernel: odd / even / single tile counts, D 64 and 128
    ("smooth_channel_1tile", (1, 1, 100, 128), torch.bfloat16, 1.0, True, True, "channel"),
    ("smooth_channel_2tiles", (1, 2, 256, 128), torch.bfloat16, 1.0, True, True, "channel"),
    ("smooth_channel_d64_odd", (2, 1, 645, 64), torch.float16, 1.0, True, True, "channel"),
    ("smooth_channel_long", (1, 1, 3000, 128), torch.bfloat16, 3 ** 0.5, True, True, "channel"),
]


@pytest.mark.parametrize("name,shape,dtype,koff,expcast,v_smooth,vmode", ATT_CASES)
def test_attention_matches_oracle(ops, name, shape, dtype, koff, expcast, v_smooth, vmode):
    q, k, v = qk_inputs(21, shape, dtype, koff)
    perm = None
    if v_smooth:
        v = mixture_values(21, shape, dtype)
        perm = ops.group_values(v.cuda(), 8, 2).cpu()
    st = _device_state(ops, q, k, v, expcast=expcast, v_smooth=v_smooth, v_scale_mode=vmode, perm=perm)
    out = ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], st["means"],
                            out_dtype=torch.float32, sm_scale=st["scale"], expcast=expcast, block_values=v_smooth)
    torch.cuda.synchronize()
    ref = O.reference(_cpu_state(st))
    m = O.metrics(out.cpu(), ref)
    assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m


@pytest.mark.parametrize("name", ["c1_expcast", "tail_expcast_d64", "smooth_channel", "smooth_block_d64",
                                  "control_no_expcast"])
def test_attention_matches_reference_oracle_fixture(ops, name):
    """End to end against outputs of the reference's own vc_reference.reference."""
    f = np.load(GOLDEN / f"att_{name}.npz")
    dtype = getattr(torch, str(f["dtype"]))
    shape = tuple(f["shape"])
    q, k, v = qk_inputs(int(f["seed"]), shape, dtype, float(f["koff"]))
    smooth = bool(f["v_smooth"])
    if smooth:
        v = mixture_values(int(f["seed"]), shape, dtype)
    perm = torch.from_numpy(f["permutation"]) if smooth else None
    # km of the fixture came from torch's CPU mean; use the same for bit-exact payloads
    kk = k.gather(2, perm.unsqueeze(-1).expand_as(k)) if smooth else k
    km = O.k_mean(kk).cuda()
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    pc = perm.cuda() if smooth else None
    q8, qs, k8, ks, _ = ops.prep_qk_int8(qc, kc, perm=pc, km=km)
    if smooth:
        v8, vs, means = ops.prep_v_blocks(vc, perm=pc, channel_scale=str(f["v_scale_mode"]) == "channel")
    else:
        v8, vs = ops.prep_v_channel(vc)
        means = None
    out = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, out_dtype=torch.float32, expcast=bool(f["expcast"]),
                            block_values=smooth)
    m = O.metrics(out.cpu(), torch.from_numpy(f["out"]))
    assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m


@pytest.mark.parametrize("shape", [(1, 2, 1000, 128), (2, 1, 385, 64), (1, 1, 130, 128)])
def test_fast_and_general_kernels_agree_with_oracle(ops, monkeypatch, shape):
    """The TMEM-accumulating fast kernel and the register-accumulating general
    kernel both meet the tolerance on the same payloads."""
    q, k, v = qk_inputs(31, shape, torch.bfloat16, 3 ** 0.5)
    st = _device_state(ops, q, k, v)
    args = (st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], None)
    fast = ops.attention_fwd(*args, out_dtype=torch.float32)
    exact = ops.attention_fwd(*args, out_dtype=torch.float32, expcast="exact")
    monkeypatch.setenv("VC_B200_KERNEL", "general")
    general = ops.attention_fwd(*args, out_dtype=torch.float32)
    monkeypatch.delenv("VC_B200_KERNEL")
    ref = O.reference(_cpu_state(st))
    for out in (fast, exact, general):
        m = O.metrics(out.cpu(), ref)
        assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m
    # the exact encoder reproduces the oracle's bytes: only accumulation order differs
    assert O.metrics(exact.cpu(), ref)["rel_l2"] <= 2e-5


@pytest.mark.parametrize("sm_scale", [None, 1.0])
def test_attention_is_bitwise_repeatable(ops, sm_scale):
    """The pipelined kernel has no timing-dependent arithmetic: repeated calls
    on the same payloads give identical bits (many K tiles, frequent maximum
    changes with the larger scale)."""
    shape = (1, 8, 8192, 128)
    q, k, v = qk_inputs(33, shape, torch.bfloat16, 3 ** 0.5)
    st = _device_state(ops, q, k, v)
    args = (st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], None)
    kw = {} if sm_scale is None else {"sm_scale": sm_scale}
    first = ops.attention_fwd(*args, **kw)
    for _ in range(6):
        assert torch.equal(ops.attention_fwd(*args, **kw), first)


# K-tile counts around the 8-tile batches of the means MMA: 2, 4, 8, 9 (two
# batches open at the end: 8 + 1), 10 (one flushed in the loop, one open), 17
@pytest.mark.parametrize("shape", [(1, 2, 1000, 128), (2, 1, 385, 64), (1, 1, 129, 128), (1, 1, 1100, 128),
                                   (1, 2, 1200, 128), (1, 1, 2100, 64)])
@pytest.mark.parametrize("sm_scale", [None, 1.0, 2.0])
def test_block_means_fast_and_general_agree(ops, monkeypatch, shape, sm_scale):
    """Block means (V smoothing, channel scales): the tensor-memory kernel
    (masses from the denominator column, one FP16 hi/lo means MMA per 8
    tiles) and the register-accumulating general kernel both meet the
    tolerance against the oracle, and the fast kernel is bitwise repeatable.
    Larger scales make row maxima grow often, so pending masses are rescaled."""
    q, k, _ = qk_inputs(35, shape, torch.bfloat16, 3 ** 0.5)
    v = mixture_values(35, shape, torch.bfloat16)
    perm = ops.group_values(v.cuda(), 8, 2).cpu()
    st = _device_state(ops, q, k, v, v_smooth=True, perm=perm)
    scale = st["scale"] if sm_scale is None else sm_scale
    args = (st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], st["means"])
    kw = dict(out_dtype=torch.float32, sm_scale=scale, block_values=True)
    fast = ops.attention_fwd(*args, **kw)
    for _ in range(3):
        assert torch.equal(ops.attention_fwd(*args, **kw), fast)
    exact = ops.attention_fwd(*args, expcast="exact", **kw)
    monkeypatch.setenv("VC_B200_KERNEL", "general")
    general = ops.attention_fwd(*args, **kw)
    monkeypatch.delenv("VC_B200_KERNEL")
    ref = O.reference({**_cpu_state(st), "scale": scale})
    for out in (fast, exact, general):
        m = O.metrics(out.cpu(), ref)
        assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m


def test_attention_large_logits_and_rescales(ops):
    """Strongly peaked rows (large scale) force frequent max changes and
    saturated ExpCast bytes; outputs stay within tolerance."""
    shape = (1, 2, 700, 128)
    q, k, v = qk_inputs(32, shape, torch.bfloat16, 3 ** 0.5)
    st = _device_state(ops, q, k, v)
    for scale in (2.0, 0.01):
        out = ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], None,
                                out_dtype=torch.float32, sm_scale=scale)
        ref = O.reference({**_cpu_state(st), "scale": scale})
        m = O.metrics(out.cpu(), ref)
        assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, (scale, m)


def test_attention_sharded_units_cover_output(ops):
    shape = (2, 3, 300, 128)
    q, k, v = qk_inputs(5, shape, torch.bfloat16, 1.0)
    st = _device_state(ops, q, k, v)
    full = ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], None)
    units = 2 * 3 * 3
    out = torch.zeros_like(full)
    for b, e in ((0, 5), (5, 11), (11, units)):
        ops.attention_fwd(st["q"], st["qs"], st["k"], st["ks"], st["v"], st["vs"], None, out=out, unit_range=(b, e))
    assert torch.equal(out, full)


def test_sageattn_vc_end_to_end_and_nhd(ops):
    from sageattention_local import sageattn_vc
    shape = (1, 2, 520, 128)
    q, k, v = qk_inputs(7, shape, torch.bfloat16, 3 ** 0.5)
    out = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=False)
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    st = O.prepare(q, k, v, v_smooth=False, km=O.k_mean(k))
    ref = O.reference(st)
    m = O.metrics(out.float().cpu(), ref)
    assert m["cos"] >= 0.9999 and m["rel_l2"] <= 4e-3, m    # bf16 output rounding included
    nhd = sageattn_vc(*(x.cuda().transpose(1, 2).contiguous() for x in (q, k, v)), tensor_layout="NHD",
                      v_smooth=False)
    assert torch.equal(nhd.transpose(1, 2), out)
    dense = O.dense_attention(q, k, v)
    print("vs dense fp32:", O.metrics(out.float().cpu(), dense))


@pytest.mark.parametrize("clusters", [16, 64, 256])
def test_sageattn_vc_wide_grouping_end_to_end(ops, clusters):
    """sageattn_vc with 9-256 clusters (the reference's public range beyond
    its fused 8-cluster path): on clustered V whose linspace-initial tokens
    lie in distinct clusters (so Lloyd has no ties), the device labels equal
    the FP64 Lloyd oracle's and the permutation is their stable argsort; the
    output equals the oracle's on the same permutation within the parity
    tolerance."""
    from sageattention_local import sageattn_vc
    n = 1100
    shape = (1, 2, n, 128)
    g = torch.Generator().manual_seed(90 + clusters)
    q, k, _ = qk_inputs(90 + clusters, shape, torch.bfloat16, 3 ** 0.5)
    lab = torch.randint(0, clusters, (n,), generator=g)
    lab[torch.from_numpy(O.linspace_ids(n, clusters))] = torch.arange(clusters)
    centres = torch.randn(1, 2, clusters, 128, generator=g) * 3
    v = (centres[:, :, lab] + 0.05 * torch.randn(shape, generator=g)).to(torch.bfloat16)
    perm, labels, _ = ops.group_values(v.cuda(), clusters, 2, debug=True)
    e_lab, _ = O.lloyd_fp64(v.float().numpy(), clusters, 2)
    assert np.array_equal(_np(labels), e_lab)
    assert np.array_equal(_np(perm), O.stable_argsort(e_lab))
    out = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=True, clusters=clusters)
    torch.cuda.synchronize()
    kk = k.gather(2, perm.cpu().unsqueeze(-1).expand_as(k))
    ref = O.reference(O.prepare(q, k, v, v_smooth=True, permutation=perm.cpu(), km=O.k_mean(kk)))
    m = O.metrics(out.float().cpu(), ref)
    assert m["cos"] >= 0.9999 and m["rel_l2"] <= 4e-3, m


def test_sageattn_vc_smooth_end_to_end(ops):
    from sageattention_local import sageattn_vc
    shape = (1, 2, 400, 64)
    q, k, _ = qk_inputs(8, shape, torch.float16, 1.0)
    v = mixture_values(8, shape, torch.float16)
    out = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=True)
    dense = O.dense_attention(q, k, v)
    m = O.metrics(out.float().cpu(), dense)
    assert m["rel_l2"] < 0.08, m


@pytest.mark.parametrize("name", ["c1_cfg_expcast", "cfg_smooth", "cfg_control_int8"])
def test_config_api_sm100a_against_reference_backend(ops, name):
    """Boundary A: vc_attention.attention(Config(backend="sm100a")) against the
    reference package's own reference backend on the same inputs.  The QK
    quantisers differ (Sage INT8 here, E4M3 blocks there), so this is a
    tolerance check: close to the reference output and as close to FP32
    dense attention as the reference backend is."""
    from vc_attention import Config, attention
    f = np.load(GOLDEN / f"{name}.npz")
    kw = json.loads(str(f["config"]))
    shape = tuple(int(x) for x in f["shape"])
    q, k, v = qk_inputs(int(f["seed"]), shape, torch.float32, float(f["koff"]))
    out, counters = attention(q.cuda(), k.cuda(), v.cuda(), Config(backend="sm100a", **kw))
    ref = torch.from_numpy(f["out"])
    assert out.dtype == torch.float32 and out.shape == ref.shape
    m = O.metrics(out.cpu(), ref)
    assert m["cos"] >= 0.998, m
    dense = O.dense_attention(q, k, v)
    ours, theirs = O.metrics(out.cpu(), dense), O.metrics(ref, dense)
    assert ours["rel_l2"] <= 1.25 * theirs["rel_l2"] + 2e-3, (ours, theirs)
    expected = json.loads((GOLDEN / "manifest.json").read_text())[name]["counters"]
    for key in ("smoothing_active", "layout_refreshed", "expcast", "k_smooth", "qk_hadamard",
                "numerical_contract_version", "tiles"):
        assert counters[key] == expected[key], key
    assert counters["backend"] == "sm100a" and counters["native_fused_attention"]


def test_config_api_layout_cache_across_denoising_steps(ops):
    """A request of 8 steps: smoothing (grouping + block means) for the first
    two, layout refreshed at step 0 only, the cached permutation kept after;
    every step stays close to dense attention."""
    from vc_attention import Config, LayoutCache, attention
    shape = (1, 2, 700, 128)
    q, k, _ = qk_inputs(41, shape, torch.bfloat16, 3 ** 0.5)
    v = mixture_values(41, shape, torch.bfloat16)
    cfg = Config(backend="sm100a", qk_hadamard=False, expcast=True, v_smooth=True, refresh_interval=4)
    cache = LayoutCache(cfg)
    dense = O.dense_attention(q.float(), k.float(), v.float())
    flags = []
    for step in range(8):
        out, c = attention(q.cuda(), k.cuda(), v.cuda(), cfg, cache=cache, step=step, total_steps=8,
                           request_id="req", layer_id=3)
        flags.append((c["smoothing_active"], c["layout_refreshed"]))
        m = O.metrics(out.float().cpu(), dense)
        assert m["cos"] >= 0.998, (step, m)
    assert flags == [(True, True), (True, False)] + [(False, False)] * 6
    assert cache.entries == 1


@pytest.mark.parametrize("smooth", [False, True])
def test_host_pipeline_equals_one_call(ops, smooth):
    """sageattn_vc_host (head chunks, PCIe copies overlapped) gives the bits of
    one sageattn_vc call on the device tensors."""
    from sageattention_local import sageattn_vc
    from vc_b200.pipeline import sageattn_vc_host
    shape = (2, 5, 700, 128)
    q, k, _ = qk_inputs(43, shape, torch.bfloat16, 3 ** 0.5)
    v = mixture_values(43, shape, torch.bfloat16)
    hq, hk, hv = (x.pin_memory() for x in (q, k, v))
    got = sageattn_vc_host(hq, hk, hv, chunk_heads=3, v_smooth=smooth)
    want = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=smooth)
    assert got.device.type == "cpu" and torch.equal(got, want.cpu())


@pytest.mark.parametrize("smooth", [False, True])
def test_sharded_host_pipeline_equals_device_shards(ops, smooth):
    """sharded_attention_host computes exactly a rank's unit range: for every
    rank of a 3-way split (ranges that cut through heads), its rows equal
    the single sageattn_vc call bit for bit, and it writes no other row."""
    from sageattention_local import sageattn_vc
    from vc_b200 import parallel as P
    from vc_b200.pipeline import sharded_attention_host
    shape = (1, 5, 700, 128)
    B, H, S, D = shape
    q, k, _ = qk_inputs(44, shape, torch.bfloat16, 3 ** 0.5)
    v = mixture_values(44, shape, torch.bfloat16)
    hq, hk, hv = (x.pin_memory() for x in (q, k, v))
    want = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=smooth).cpu()
    mean_numel = (B * H * D, B * H * S * D)
    covered = torch.zeros(B * H * S, dtype=torch.bool)
    for rank in range(3):
        s = P.shard(B, H, S, 3, rank)
        out = torch.full(shape, float("nan"), dtype=torch.bfloat16).pin_memory()
        sharded_attention_host(hq, hk, hv, out, (s.unit_begin, s.unit_end), chunk_heads=2,
                               mean_numel=mean_numel, v_smooth=smooth)
        r0, r1 = P.shard_rows(s, S)
        got, ref = out.view(-1, D), want.view(-1, D)
        assert torch.equal(got[r0:r1], ref[r0:r1])
        assert torch.isnan(got[:r0].float()).all() and torch.isnan(got[r1:].float()).all()
        covered[r0:r1] = True
    assert covered.all()


# --- the Config contract's own Q/K path: Hadamard rotation + E4M3 blocks ---------------------------

@pytest.mark.parametrize("name", ["hadamard_qk", "hadamard_qk_d64"])
def test_hadamard_prep_matches_reference_payloads(ops, name):
    """Device Hadamard + E4M3 block preparation against payloads and scales
    written by the reference's preprocess_qk + _encode: bit for bit given its
    FP32 K mean.  The K mean computed on the device (fixed-order FP32 sums)
    agrees with torch's to within rounding."""
    f = np.load(GOLDEN / f"{name}.npz")
    shape = tuple(int(x) for x in f["shape"])
    q, k, _ = qk_inputs(int(f["seed"]), shape, getattr(torch, str(f["dtype"])), float(f["koff"]))
    kqb = int(f["k_quant_block"])
    q8, qs, k8, ks, km = ops.prep_qk_hadamard(q.cuda(), k.cuda(), k_smooth=True, k_quant_block=kqb,
                                              km=torch.from_numpy(f["km"]).cuda())
    assert q8.dtype == torch.float8_e4m3fn and k8.dtype == torch.float8_e4m3fn
    assert np.array_equal(_np(q8.view(torch.uint8)), f["q8"]) and np.array_equal(_np(qs), f["qs"])
    assert np.array_equal(_np(k8.view(torch.uint8)), f["k8"]) and np.array_equal(_np(ks), f["ks"])
    *_, km_dev = ops.prep_qk_hadamard(q.cuda(), k.cuda(), k_smooth=True, k_quant_block=kqb)
    assert torch.allclose(km_dev.cpu(), torch.from_numpy(f["km"]), rtol=1e-5, atol=1e-6)
    assert ops.error_word(0, clear=True) == 0


HAD_CASES = [
    # shape, dtype, koff, k_quant_block, k_smooth, grouped (permutation + block means)
    ((1, 2, 1000, 128), torch.bfloat16, 2 ** 0.5, 256, True, False),
    ((2, 1, 333, 64), torch.float16, 1.0, 128, True, False),
    ((1, 1, 129, 128), torch.float32, 3 ** 0.5, 512, False, False),
    ((1, 2, 700, 128), torch.bfloat16, 1.0, 256, True, True),
    ((1, 1, 1100, 64), torch.bfloat16, 2 ** 0.5, 384, True, True),
]


@pytest.mark.parametrize("shape,dtype,koff,kqb,k_smooth,grouped", HAD_CASES)
def test_hadamard_attention_matches_oracle(ops, shape, dtype, koff, kqb, k_smooth, grouped):
    """E4M3 block Q/K: the device payloads equal the oracle's (given the
    device K mean, with the K permutation when grouped) and the FP8-QK
    attention kernel meets the parity tolerance against the oracle on the
    same payloads, with and without block means; bitwise repeatable."""
    q, k, _ = qk_inputs(41, shape, dtype, koff)
    v = mixture_values(41, shape, dtype) if grouped else torch.randn(shape, generator=torch.Generator().manual_seed(7)).to(dtype)
    perm = ops.group_values(v.cuda(), 8, 2).cpu() if grouped else None
    pc = perm.cuda() if grouped else None
    q8, qs, k8, ks, km = ops.prep_qk_hadamard(q.cuda(), k.cuda(), perm=pc, k_smooth=k_smooth, k_quant_block=kqb)
    ost = O.prepare_hadamard(q, k, k_smooth=k_smooth, k_quant_block=kqb,
                             km=km.cpu() if km is not None else None, perm=perm)
    assert np.array_equal(_np(q8.view(torch.uint8)), ost["q"]) and np.array_equal(_np(qs), ost["qs"])
    assert np.array_equal(_np(k8.view(torch.uint8)), ost["k"]) and np.array_equal(_np(ks), ost["ks"])
    if grouped:
        v8, vs, means = ops.prep_v_blocks(v.cuda(), perm=pc, channel_scale=True)
    else:
        v8, vs = ops.prep_v_channel(v.cuda())
        means = None
    scale = shape[-1] ** -0.5
    kw = dict(out_dtype=torch.float32, sm_scale=scale, block_values=grouped, k_quant_block=kqb)
    out = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, **kw)
    assert torch.equal(ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, **kw), out)
    state = {**ost, "v": _np(v8.view(torch.uint8)), "vs": vs.cpu(), "means": _np(means) if grouped else None,
             "expcast": True, "block_values": grouped, "scale": scale}
    m = O.metrics(out.cpu(), O.reference(state))
    assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m
    assert ops.error_word(0, clear=True) == 0


@pytest.mark.parametrize("name", ["cfg_hadamard", "cfg_hadamard_smooth", "cfg_default", "cfg_default_smooth"])
def test_config_api_sm100a_hadamard_against_reference_backend(ops, name):
    """Boundary A with qk_hadamard=True -- the Config contract's own formats:
    Hadamard + E4M3 block Q/K (FP8 QK^T), V encoded per 128-token tile, and
    with the reference's defaults (``cfg_default*``: expcast=False) the FP8-P
    control with exact exp row sums -- against the reference package's
    reference backend.  Q/K and V payloads follow the same formulas; what
    differs is FP32 accumulation order and exp, so the outputs agree to
    cos >= 0.9999 (written in the test)."""
    from vc_attention import Config, attention
    f = np.load(GOLDEN / f"{name}.npz")
    kw = json.loads(str(f["config"]))
    shape = tuple(int(x) for x in f["shape"])
    q, k, v = qk_inputs(int(f["seed"]), shape, torch.float32, float(f["koff"]))
    out, counters = attention(q.cuda(), k.cuda(), v.cuda(), Config(backend="sm100a", **kw))
    ref = torch.from_numpy(f["out"])
    m = O.metrics(out.cpu(), ref)
    assert m["cos"] >= 0.9999, m
    dense = O.dense_attention(q, k, v)
    ours, theirs = O.metrics(out.cpu(), dense), O.metrics(ref, dense)
    assert ours["rel_l2"] <= 1.05 * theirs["rel_l2"] + 1e-3, (ours, theirs)
    expected = json.loads((GOLDEN / "manifest.json").read_text())[name]["counters"]
    for key in ("smoothing_active", "layout_refreshed", "expcast", "k_smooth", "qk_hadamard",
                "numerical_contract_version", "tiles"):
        assert counters[key] == expected[key], key
    assert counters["qk_hadamard"] and not counters["native_int8_matmul"]


def test_hadamard_attention_cross_lengths_and_shards(ops):
    """E4M3 block Q/K with Sq != Sk against the oracle, and computed as three
    unit ranges into one output: the same bits as one full call."""
    g = torch.Generator().manual_seed(17)
    q = torch.randn(1, 2, 300, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(1, 2, 700, 128, generator=g) + torch.randn(1, 2, 1, 128, generator=g)).to(torch.bfloat16)
    v = torch.randn(1, 2, 700, 128, generator=g).to(torch.bfloat16)
    q8, qs, k8, ks, km = ops.prep_qk_hadamard(q.cuda(), k.cuda(), k_smooth=True, k_quant_block=256)
    v8, vs = ops.prep_v_channel(v.cuda())
    scale = 128 ** -0.5
    full = ops.attention_fwd(q8, qs, k8, ks, v8, vs, None, out_dtype=torch.float32, sm_scale=scale)
    ost = O.prepare_hadamard(q, k, k_smooth=True, k_quant_block=256, km=km.cpu())
    state = {**ost, "v": _np(v8.view(torch.uint8)), "vs": vs.cpu(), "means": None, "expcast": True,
             "block_values": False, "scale": scale}
    m = O.metrics(full.cpu(), O.reference(state))
    assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, m
    out = torch.full_like(full, float("nan"))
    units = 2 * 3   # (b*H + h) * ceil(300/128) + q_tile
    for r in ((0, 2), (2, 5), (5, units)):
        ops.attention_fwd(q8, qs, k8, ks, v8, vs, None, out=out, sm_scale=scale, unit_range=r)
    assert torch.equal(out, full)


# Q-tile counts 1 (tile B of the only pair is empty), 2, 3 (last pair half
# empty), 8; Sq != Sk; D 64 and 128; with and without block means
PAIR_CASES = [
    ((1, 2, 1000, 128), 1000, False),
    ((2, 1, 385, 64), 385, False),
    ((1, 1, 100, 128), 100, False),
    ((1, 2, 256, 128), 700, False),
    ((1, 1, 300, 64), 1300, True),
    ((1, 2, 1000, 128), 1000, True),
    ((2, 1, 129, 128), 2100, True),
    # 150 pairs: one full wave of pairs on 148 SMs, then 4 tail tiles on the
    # alternating-tile kernel (and other splits for the unit-range cuts)
    ((1, 2, 19200, 128), 300, False),
    ((1, 2, 19100, 64), 260, True),
]


@pytest.mark.parametrize("shape,sk,smooth", PAIR_CASES)
def test_paired_tile_kernel_equals_alternating_kernel(ops, monkeypatch, shape, sk, smooth):
    """The paired-tile kernel (two Q tiles per CTA, one softmax chain each)
    performs every row's arithmetic in the same order as the alternating-tile
    kernel (one Q tile per CTA, the groups alternating K tiles), so the two
    give identical bits: INT8 and E4M3 Q/K, with and without block means, and
    as unit ranges that cut pairs in two.  The default schedule (full waves of
    pairs, a short last wave on the alternating-tile kernel) equals both."""
    B, H, Sq, D = shape
    g = torch.Generator().manual_seed(51)
    q = torch.randn(B, H, Sq, D, generator=g).to(torch.bfloat16)
    k = (torch.randn(B, H, sk, D, generator=g) + 1.5 * torch.randn(B, H, 1, D, generator=g)).to(torch.bfloat16)
    if smooth:
        v = mixture_values(51, (B, H, sk, D), torch.bfloat16)
    else:
        v = torch.randn(B, H, sk, D, generator=g).to(torch.bfloat16)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    perm = ops.group_values(vc, 8, 2) if smooth else None
    if smooth:
        v8, vs, means = ops.prep_v_blocks(vc, perm=perm, channel_scale=True)
    else:
        v8, vs = ops.prep_v_channel(vc)
        means = None
    payloads = [ops.prep_qk_int8(qc, kc, perm=perm)[:4],
                ops.prep_qk_hadamard(qc, kc, perm=perm, k_smooth=True, k_quant_block=256)[:4]]
    qtiles = (Sq + 127) // 128
    for (q8, qs, k8, ks), scale in ((payloads[0], None), (payloads[0], 1.0), (payloads[1], None)):
        kw = dict(out_dtype=torch.float32, block_values=smooth)
        if scale is not None:
            kw["sm_scale"] = scale
        default = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, **kw)
        cuts = sorted({0, min(1, B * H * qtiles), B * H * qtiles // 2 + 1, B * H * qtiles})
        outs = {}
        for kernel in ("pair", "default"):
            if kernel == "pair":
                monkeypatch.setenv("VC_B200_KERNEL", "pair")
            split = torch.full_like(default, float("nan"))
            for b, e in zip(cuts[:-1], cuts[1:]):
                ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, out=split, unit_range=(b, e), **kw)
            outs[kernel] = (ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, **kw), split)
            monkeypatch.delenv("VC_B200_KERNEL", raising=False)
        monkeypatch.setenv("VC_B200_KERNEL", "alt")
        alt = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, **kw)
        monkeypatch.delenv("VC_B200_KERNEL")
        assert torch.equal(outs["pair"][0], alt)
        assert torch.equal(default, alt)
        for whole, split in outs.values():
            assert torch.equal(split, whole)
    assert ops.error_word(0, clear=True) == 0


# the register-accumulating kernel's modes beyond the Sage INT8 contract: the
# Config contract's FP8-P control (offset 8), ExpCast and Sage's control with
# per-tile V scales, on INT8 and on E4M3 block Q/K
REG_MODES = [
    # name, expcast, control, demean
    ("config_control", False, "config", False),
    ("config_control_means", False, "config", True),
    ("expcast_tile_scales", True, "sage", True),
    ("sage_control_tile_scales", False, "sage", False),
]


@pytest.mark.parametrize("qk", ["int8", "e4m3"])
@pytest.mark.parametrize("name,expcast,control,demean", REG_MODES)
@pytest.mark.parametrize("shape", [(1, 2, 700, 128), (2, 1, 333, 64)])
def test_register_kernel_modes_match_oracle(ops, qk, name, expcast, control, demean, shape):
    """V encoded per 128-token tile (prep_v_blocks without channel scales,
    tile means or zeros) through the register-accumulating kernel, against
    the oracle on the same payloads: cos >= 0.9999, rel-L2 <= 1e-3."""
    g = torch.Generator().manual_seed(71)
    q = torch.randn(shape, generator=g).to(torch.bfloat16)
    k = (torch.randn(shape, generator=g) + 1.5 * torch.randn(*shape[:2], 1, shape[-1], generator=g)).to(torch.bfloat16)
    v = mixture_values(71, shape, torch.bfloat16) if demean else torch.randn(shape, generator=g).to(torch.bfloat16)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    v8, vs, means = ops.prep_v_blocks(vc, channel_scale=False, demean=demean)
    scale = shape[-1] ** -0.5
    if qk == "int8":
        q8, qs, k8, ks, km = ops.prep_qk_int8(qc, kc)
        qstate = {"q": q8.cpu(), "qs": qs.cpu(), "k": k8.cpu(), "ks": ks.cpu()}
    else:
        q8, qs, k8, ks, km = ops.prep_qk_hadamard(qc, kc, k_smooth=True, k_quant_block=256)
        qstate = O.prepare_hadamard(q, k, k_smooth=True, k_quant_block=256, km=km.cpu())
    out = ops.attention_fwd(q8, qs, k8, ks, v8, vs, means, out_dtype=torch.float32, sm_scale=scale,
                            expcast=expcast, block_values=True, control=control)
    torch.cuda.synchronize()
    state = {**qstate, "v": _np(v8.view(torch.uint8)), "vs": vs.cpu(), "means": _np(means), "expcast": expcast,
             "block_values": True, "scale": scale, "control_offset": 8.0 if control == "config" else 8.807}
    m = O.metrics(out.cpu(), O.reference(state))
    assert m["cos"] >= COS_MIN and m["rel_l2"] <= REL_MAX, (name, qk, m)
    assert ops.error_word(0, clear=True) == 0
