"""Pin the CPU oracle against the reference's own outputs and known answers.

Fixtures under tests/golden/ were produced by tests/golden/gen_golden.py from
the reference's Python code (vc_reference.reference, core.attention and the
Triton INT8 quantiser interpreted on CPU).  Known answers are the reference
tests' literal expected values.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from inputs import qk_inputs, mixture_values

GOLDEN = Path(__file__).resolve().parent / "golden"


def fixture(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def test_expcast_matches_reference_sweep():
    f = fixture("expcast.npz")
    assert np.array_equal(O.expcast_codes(f["shifted"]), f["codes"])
    assert np.array_equal(f["codes"], f["codes_core"])


def test_expcast_known_answers():
    # tests/test_core.py:17-22 and tests/test_sage_vc.py:22-25 of the reference
    u = np.array([0.0, -1.0, -1.6, -8.0, -14.0, -100.0, -np.inf], np.float32)
    codes = O.expcast_codes((u / np.float32(math.log2(math.e))).astype(np.float32))
    assert codes.tolist() == [120, 112, 107, 56, 8, 0, 0]
    assert O.e4m3_decode(codes).tolist() == [256, 128, 88, 1, 2 ** -6, 0, 0]
    assert O.expcast_codes(np.array([-np.inf, -20, 0, 1], np.float32)).tolist() == [0, 0, 120, 120]


def test_value_permutation_known_answer():
    perm = O.value_permutation(256)
    assert perm[:16].tolist() == [0, 1, 4, 5, 8, 9, 12, 13, 2, 3, 6, 7, 10, 11, 14, 15]
    assert sorted(perm.tolist()) == list(range(256))
    x = np.arange(2 * 256, dtype=np.uint8).reshape(2, 256)
    sage = O.to_sage_layout(x)
    assert np.array_equal(sage[:, perm], x)          # vc_reference.py:26 reads it back


def test_e4m3_codec_matches_torch_everywhere():
    bits = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(bits.copy()).view(torch.float8_e4m3fn).float().numpy()
    dec = O.e4m3_decode(bits)
    fin = ~np.isnan(ref)
    assert np.array_equal(dec[fin], ref[fin]) and np.isnan(dec[~fin]).all()
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.randn(200000, generator=g) * s for s in (1e-3, 0.1, 1, 30, 300)])
    x = x.clamp(-448, 448)
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(x.numpy()), ref)
    # satfinite clamps instead of producing NaN
    assert O.e4m3_encode(np.array([460.0, -1e9, 1e30], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]


@pytest.mark.parametrize("name", ["c1_fp32", "tail_bf16_d64", "tail_fp16_d128", "single_bf16", "outlier_bf16"])
def test_int8_quantiser_bit_exact_vs_reference_triton(name):
    f = fixture(f"qk_{name}.npz")
    dtype = getattr(torch, str(f["dtype"]))
    q, k, _ = qk_inputs(int(f["seed"]), tuple(f["shape"]), dtype, float(f["koff"]), float(f["outliers"]))
    km = torch.from_numpy(f["km"]).to(dtype)
    assert torch.equal(O.k_mean(k).float(), km.float())          # same torch CPU reduction
    q8, qs, k8, ks = O.per_thread_int8(q, k, km)
    assert np.array_equal(q8, f["q8"]) and np.array_equal(qs, f["qs"])
    assert np.array_equal(k8, f["k8"]) and np.array_equal(ks, f["ks"])


@pytest.mark.parametrize("name", ["c1_expcast", "tail_expcast_d64", "smooth_channel", "smooth_block_d64",
                                  "control_no_expcast"])
def test_attention_oracle_matches_reference_oracle(name):
    f = fixture(f"att_{name}.npz")
    dtype = getattr(torch, str(f["dtype"]))
    shape = tuple(f["shape"])
    q, k, v = qk_inputs(int(f["seed"]), shape, dtype, float(f["koff"]))
    if bool(f["v_smooth"]):
        v = mixture_values(int(f["seed"]), shape, dtype)
    perm = torch.from_numpy(f["permutation"]) if f["permutation"].size else None
    st = O.prepare(q, k, v, expcast=bool(f["expcast"]), v_smooth=bool(f["v_smooth"]),
                   v_scale_mode=str(f["v_scale_mode"]), permutation=perm)
    out = O.reference(st)
    torch.testing.assert_close(out, torch.from_numpy(f["out"]), rtol=1e-5, atol=1e-6)


def _payload(nq, nk, block_values, expcast, dim=64):
    tiles = (nk + 127) // 128
    return {"q": torch.zeros(1, 1, nq, dim, dtype=torch.int8), "k": torch.zeros(1, 1, nk, dim, dtype=torch.int8),
            "v": np.zeros((1, 1, dim, tiles * 128), np.uint8), "qs": torch.ones(1, 1, ((nq + 63) // 64) * 32),
            "ks": torch.ones(1, 1, tiles * 4),
            "vs": torch.ones(1, 1, tiles, dim) if block_values else torch.ones(1, 1, dim),
            "means": np.zeros((1, 1, tiles, dim), np.float16) if block_values else np.zeros(0, np.float16),
            "expcast": expcast, "block_values": block_values, "output_type": 1, "scale": dim ** -0.5}


@pytest.mark.parametrize("expcast", [False, True])
def test_block_mean_restoration_known_answer(expcast):
    # reference tests/test_sage_vc.py:42-49
    st = _payload(65, 257, True, expcast)
    st["means"][0, 0] = np.array([1., -2., 6.], np.float16)[:, None]
    st["vs"][0, 0] = torch.tensor([2., 3., 4.])[:, None]
    out = O.reference(st, chunk=7)
    expected = (128 * 2 + 128 * (-6) + 24) / 257
    torch.testing.assert_close(out, torch.full_like(out, expected), rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("expcast", [False, True])
def test_shared_scale_nonzero_mean_known_answer(expcast):
    # reference tests/test_sage_vc.py:98-105
    st = _payload(65, 257, True, expcast)
    st["vs"] = torch.full((1, 1, 64), .25)
    st["means"][0, 0] = np.array([8., -24., 96.], np.float16)[:, None]
    out = O.reference(st)
    expected = (128 * 2 - 128 * 6 + 24) / 257
    torch.testing.assert_close(out, torch.full_like(out, expected), rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("block_values", [False, True])
@pytest.mark.parametrize("expcast", [False, True])
def test_single_key_known_answer(block_values, expcast):
    # reference tests/test_sage_vc.py:52-65
    st = _payload(17, 1, block_values, expcast)
    data = np.zeros((1, 1, 64, 128), np.float32)
    data[..., 0] = np.arange(64) % 9 - 4
    st["v"] = O.e4m3_encode(data)
    st["vs"].fill_(0.125)
    if block_values:
        st["means"][...] = 2
    out = O.reference(st)
    weight = 1. if expcast else 448. / (2 ** float(torch.tensor(8.807)))
    expected = torch.from_numpy((data[..., 0] * weight + (2 if block_values else 0)) * 0.125)
    torch.testing.assert_close(out, expected.unsqueeze(2).expand_as(out), rtol=1e-6, atol=1e-6)


def test_query_sampling_keeps_scale_indices():
    # reference tests/test_sage_vc.py:68-79
    st = _payload(129, 129, False, True)
    g = torch.Generator().manual_seed(778)
    st["q"] = torch.randint(-3, 4, st["q"].shape, generator=g, dtype=torch.int8)
    st["k"] = torch.randint(-3, 4, st["k"].shape, generator=g, dtype=torch.int8)
    st["qs"] = torch.rand(st["qs"].shape, generator=g) * 0.2 + 0.1
    st["ks"] = torch.rand(st["ks"].shape, generator=g) * 0.3 + 0.2
    st["v"] = O.e4m3_encode(torch.randn(1, 1, 64, 256, generator=g).numpy())
    ids = [0, 7, 8, 15, 16, 63, 64, 128]
    full = O.reference(st, chunk=32)
    torch.testing.assert_close(O.reference(st, query_indices=ids, chunk=3), full[:, :, ids], rtol=1e-6, atol=1e-6)


def test_v_channel_known_answer_and_zero_safety():
    # reference tests/test_core.py:51-67 requant arithmetic: scale 3/448 -> bytes for [1,3]
    v = np.array([1., 3.], np.float32).reshape(1, 1, 2, 1)
    v8, vs = O.v_channel_fp8(v)
    assert vs[0, 0, 0] == np.float32(3) / np.float32(448)
    assert O.e4m3_decode(v8[0, 0, 0, :2]).tolist() == [144.0, 448.0]
    z = np.zeros((1, 1, 5, 4), np.float32)
    v8, vs = O.v_channel_fp8(z)
    assert (v8 == 0).all() and (vs == 0).all()


def test_v_blocks_statistics_match_reference_validation_formulas():
    # reference scripts/validate_sage_vc.py:19-83 expectations on its own data recipe
    for dim in (64, 128):
        for n in (1, 127, 128, 129, 257):
            g = torch.Generator().manual_seed(339)
            v = torch.randn(2, 2, n, dim, generator=g)
            for t, begin in enumerate(range(0, n, 128)):
                v[:, :, begin:begin + 128] = v[:, :, begin:begin + 128] * (t + 1) + t * 3
            v[..., 0] = 1.5
            v[..., 1] = -2.0
            blocks = []
            for begin in range(0, n, 128):
                rows = v[:, :, begin:begin + 128].double()
                mean = rows.mean(2)
                residual = rows - mean.unsqueeze(2)
                blocks.append((mean, residual, residual.abs().amax(2)))
            for channel in (False, True):
                v8, scales, means = O.v_blocks_fp8(v.numpy(), channel_scale=channel)
                scales = torch.from_numpy(scales).double()
                dec = torch.from_numpy(O.e4m3_decode(v8)).double().transpose(-1, -2)
                if channel:
                    peak = torch.stack([b[2] for b in blocks]).amax(0)
                    mp = torch.stack([b[0].abs() for b in blocks]).amax(0)
                    exp_scale = torch.maximum(torch.where(peak > 0, peak / 448., 1.), mp / 65504.)
                    torch.testing.assert_close(scales, exp_scale, rtol=2e-5, atol=1e-7)
                for t, (mean, residual, peak) in enumerate(blocks):
                    sc = scales if channel else scales[:, :, t]
                    torch.testing.assert_close(torch.from_numpy(means[:, :, t].astype(np.float64)) * sc, mean,
                                               rtol=8e-4, atol=2e-6)
                    d = dec[:, :, t * 128:t * 128 + residual.shape[2]]
                    err = (d * sc.unsqueeze(2) - residual).abs()
                    assert torch.all(err <= residual.abs() * .063 + sc.unsqueeze(2) / 512 + 3e-6)
                if n % 128:
                    assert np.count_nonzero(v8[..., n:]) == 0


def test_block_sum_tree_matches_warp_butterfly_order():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((128, 3)).astype(np.float32) * 1000
    lanes = [np.float32(0)] * 32
    lanes = [[np.float32(0)] * 3 for _ in range(32)]
    for l in range(32):
        for j in range(4):
            lanes[l] = [np.float32(a + b) for a, b in zip(lanes[l], x[l + 32 * j])]
    for shift in (16, 8, 4, 2, 1):   # every lane: x += shfl_xor(x, shift)
        lanes = [[np.float32(a + b) for a, b in zip(lanes[l], lanes[l ^ shift])] for l in range(32)]
    assert np.array_equal(O._block_sum_tree(x), np.array(lanes[0], np.float32))


def test_linspace_ids_match_torch():
    for n in (1, 2, 7, 8, 9, 100, 129, 1000, 37741, 75600):
        for count in range(1, 9):
            c = min(count, n)
            ref = torch.linspace(0, n - 1, c, dtype=torch.float32).long().numpy()
            assert np.array_equal(O.linspace_ids(n, c), ref), (n, c)


def test_stable_grouping_known_answer():
    # reference scripts/validate_sage_vc.py:66-82
    labels = np.array([2, 0, 1, 2, 1, 0])
    values = np.broadcast_to(labels.astype(np.float32).reshape(1, 1, 6, 1), (2, 2, 6, 64)).copy()
    lab, _ = O.lloyd_fp64(values, 3, 2)
    perm = O.stable_argsort(lab)
    for p in perm.reshape(-1, 6):
        assert labels[p].tolist() == [2, 2, 1, 1, 0, 0]
        assert p.tolist() == [0, 3, 2, 4, 1, 5]


def test_config_reference_fixture_within_band_of_oracle():
    # Boundary A: the reference backend uses E4M3 block QK; the INT8 oracle is
    # only expected to agree within the quantisation band of both.
    f = fixture("c1_cfg_expcast.npz")
    q, k, v = qk_inputs(int(f["seed"]), tuple(f["shape"]), torch.float32, float(f["koff"]))
    st = O.prepare(q, k, v, expcast=True)
    out = O.reference(st)
    m = O.metrics(out, torch.from_numpy(f["out"]))
    assert m["rel_l2"] < 0.08 and m["cos"] > 0.995, m


@pytest.mark.parametrize("name", ["hadamard_qk", "hadamard_qk_d64"])
def test_hadamard_e4m3_blocks_match_reference(name):
    """The oracle's Hadamard rotation and E4M3 block encoder (the Config
    contract's own Q/K path) against payloads and scales written by the
    reference's preprocess_qk + _encode, bit for bit, given its K mean."""
    f = fixture(f"{name}.npz")
    q, k, _ = qk_inputs(int(f["seed"]), tuple(int(x) for x in f["shape"]), getattr(torch, str(f["dtype"])),
                        float(f["koff"]))
    st = O.prepare_hadamard(q, k, k_smooth=True, k_quant_block=int(f["k_quant_block"]),
                            km=torch.from_numpy(f["km"]))
    assert np.array_equal(st["q"], f["q8"]) and np.array_equal(st["qs"], f["qs"])
    assert np.array_equal(st["k"], f["k8"]) and np.array_equal(st["ks"], f["ks"])


def test_hadamard_is_orthonormal_and_self_inverse():
    """Known properties of the normalised Sylvester transform: norms kept and
    H(H(x)) = x up to FP32 rounding; a one-hot row maps to +-1/sqrt(D)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(50, 128, generator=g).numpy()
    y = O.hadamard_fp32(x)
    assert np.allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)
    assert np.allclose(O.hadamard_fp32(y), x, atol=1e-5)
    e = np.zeros((1, 64), np.float32)
    e[0, 5] = 1
    assert np.allclose(np.abs(O.hadamard_fp32(e)), 0.125)
