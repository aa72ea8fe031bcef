"""The LightX2V model adapter, capture path and four-arm replay
(vc_attention.lightx2v / vc_attention.replay).  Host logic runs on CPU with
a fake scheduler and an injected attention function; the GPU tests run the
real replay and compare the adapter with a direct attention call."""
import json
import types

import pytest
import torch

from vc_attention import lightx2v as X
from vc_attention import replay as R


def _options(tmp_path, mode="combined", **kw):
    base = dict(mode=mode, hadamard=False, output_dir=str(tmp_path), capture_rank=0, capture_steps=[0, 2],
                capture_layers=[0], capture_heads=1, max_captures=4, max_capture_mib=64)
    base.update(kw)
    return types.SimpleNamespace(**base)


def _audit():
    return {"calls": 0, "smoothing_calls": 0, "regroup_calls": 0, "expcast_calls": 0, "captures": {}, "capture_bytes": 0}


class FakeScheduler:
    def __init__(self, steps=4):
        self.layout_cpu = object()
        self.step_index = 0
        self.infer_steps = steps


def _fake_attention(calls):
    def fn(q, k, v, cfg, *, cache, step, total_steps, request_id, layer_id, scale):
        calls.append((step, total_steps, request_id, layer_id, scale, cfg))
        return q.float() * 2, {"smoothing_active": cfg.v_smooth, "layout_refreshed": step == 0, "expcast": cfg.expcast}
    return fn


def test_validate_layout_accepts_snd_and_1snd():
    x = torch.randn(10, 3, 8)
    q, k, v = X.validate_layout(x, x, x, None, None, None, None, {})
    assert q.shape == (1, 3, 10, 8) and torch.equal(q[0, 1], x[:, 1])
    q2, *_ = X.validate_layout(x[None], x[None], x[None], torch.tensor([0, 10]), None, 10, 10, {"block_idx": 0})
    assert torch.equal(q2, q)


@pytest.mark.parametrize("kwargs,extra,match", [
    ({"foo": 1}, {}, "Unknown attention options"),
    ({"causal": True}, {}, "noncausal"),
    ({"dropout": 0.1}, {}, "noncausal"),
    ({"attn_mask": torch.ones(1)}, {}, "Mask/bias"),
    ({}, {"cu_q": torch.tensor([0, 4, 10])}, "Packed"),
    ({}, {"max_q": 9}, "max_seqlen"),
    ({}, {"k_shape": (10, 2, 8)}, "SND/1SND"),
])
def test_validate_layout_rejects(kwargs, extra, match):
    x = torch.randn(10, 3, 8)
    k = torch.randn(*extra.get("k_shape", (10, 3, 8)))
    with pytest.raises(ValueError, match=match):
        X.validate_layout(x, k, x, extra.get("cu_q"), None, extra.get("max_q"), None, kwargs)


def test_configure_patches_and_rejects():
    cfg = X.configure({"warmup": False, "parallel": {"seq_p_attn_type": "ulysses"}, "model": "h3"})
    assert cfg["attn_type"] == X.ATTN_TYPE and cfg["warmup"] is False and cfg["model"] == "h3"
    for bad, match in (({"use_compile": True}, "use_compile"), ({"warmup": True}, "warmup"),
                       ({"parallel": {"seq_p_head_parallel": True}}, "head_parallel"),
                       ({"parallel": {"seq_p_attn_type": "ring"}}, "Ulysses"), ({"enable_cfg": True}, "CFG")):
        with pytest.raises(ValueError, match=match):
            X.configure(bad)


def test_adapter_steps_layers_and_requests(tmp_path):
    """Steps come from the scheduler, layers from block_idx; a new layout
    marker or step 0 again for a seen layer starts a new request (cache
    reset); a repeated or reversed layer step raises; SND output."""
    calls = []
    a = X.ExperimentAdapter(_options(tmp_path), _audit(), attention_fn=_fake_attention(calls))
    s = FakeScheduler()
    x = torch.randn(12, 2, 8)
    out = a.apply(x, x, x, scheduler=s, block_idx=0, softmax_scale=0.5)
    assert out.shape == (12, 16) and torch.equal(out, (x * 2).reshape(12, 16))
    a.apply(x, x, x, scheduler=s, block_idx=1)
    s.step_index = 1
    a.apply(x, x, x, scheduler=s, block_idx=0)
    with pytest.raises(ValueError, match="Repeated/reversed"):
        a.apply(x, x, x, scheduler=s, block_idx=0)
    assert [c[0] for c in calls] == [0, 0, 1] and {c[2] for c in calls} == {1}
    assert calls[0][4] == 0.5 and calls[1][4] == 8 ** -0.5
    s.step_index = 0   # step 0 again for a seen layer: a new request
    a.apply(x, x, x, scheduler=s, block_idx=0)
    s2 = FakeScheduler()   # a new layout marker: a new request
    a.apply(x, x, x, scheduler=s2, block_idx=0)
    assert [c[2] for c in calls] == [1, 1, 1, 2, 3]
    assert a.audit["calls"] == 5 and a.audit["smoothing_calls"] == 5 and a.audit["regroup_calls"] == 4
    cfg = calls[0][5]
    assert cfg.backend == "sm100a" and cfg.v_smooth and cfg.expcast and not cfg.qk_hadamard
    with pytest.raises(ValueError, match="scheduler/block_idx"):
        a.apply(x, x, x, scheduler=s)
    with pytest.raises(ValueError, match="mode must be"):
        X.ExperimentAdapter(_options(tmp_path, mode="mindie_fp8"), _audit())


def test_adapter_arm_configs():
    assert not X.experiment_config("fp8_control").expcast and not X.experiment_config("fp8_control").v_smooth
    assert X.experiment_config("expcast", hadamard=True).qk_hadamard
    assert not X.experiment_config("v_smooth", hadamard=True).qk_hadamard   # no ExpCast: INT8 Q/K
    cfgs = R.arm_configs(hadamard=True)
    assert set(cfgs) == set(R.ARMS) and cfgs["combined"].qk_hadamard and not cfgs["fp8_control"].qk_hadamard


def test_capture_writes_files_within_budget(tmp_path):
    """Capture mode saves the chosen steps/layers (first heads, BNSD, with
    metadata) once each, returns the BF16 SDPA output, and stops at the byte
    budget with an error; the replay reads the files back."""
    a = X.ExperimentAdapter(_options(tmp_path, mode="capture", capture_heads=2), _audit())
    s = FakeScheduler()
    x = torch.randn(16, 3, 8)
    out = a.apply(x, x, x, scheduler=s, block_idx=0)
    ref = torch.nn.functional.scaled_dot_product_attention(*(t.to(torch.bfloat16) for t in
                                                              X.validate_layout(x, x, x, None, None, None, None, {})))
    assert torch.equal(out, ref.squeeze(0).transpose(0, 1).reshape(16, 24).to(x.dtype))
    a.apply(x, x, x, scheduler=s, block_idx=1)   # layer 1 is not captured
    s.step_index = 2
    a.apply(x, x, x, scheduler=s, block_idx=0)
    assert sorted(a.audit["captures"]) == ["rank0_step0_layer0", "rank0_step2_layer0"]
    q, k, v, scale, source = R.load_capture(a.audit["captures"]["rank0_step0_layer0"])
    assert q.shape == (1, 2, 16, 8) and scale == 8 ** -0.5 and source["metadata"]["layer"] == 0
    assert torch.equal(q[0, 1], x[:, 1]) and len(source["sha256"]) == 64
    small = X.ExperimentAdapter(_options(tmp_path / "b", mode="capture", max_capture_mib=1), _audit())
    big = torch.randn(40000, 1, 8)
    with pytest.raises(ValueError, match="budget"):
        small.apply(big, big, big, scheduler=FakeScheduler(), block_idx=0)


def test_replay_helpers():
    q, k, v = R.synthetic(256, 2, 64, 3, clustered=True)
    q2, k2, v2 = R.synthetic(256, 2, 64, 3, clustered=True)
    assert torch.equal(v, v2) and q.shape == (1, 2, 256, 64)
    m = R.metrics(q + 0.01, q)
    assert abs(m["rmse"] - 0.01) < 1e-6 and m["cosine"] > 0.999 and m["max_abs"] == pytest.approx(0.01, rel=1e-4)
    with pytest.raises(ValueError, match="Nonfinite"):
        R.metrics(torch.tensor([float("nan")]), torch.tensor([1.0]))
    ex = R.exact_attention(q, k, v, 64 ** -0.5, chunk=100)
    dense = torch.softmax((q @ k.transpose(-1, -2)) * 64 ** -0.5, dim=-1) @ v
    assert torch.allclose(ex, dense, atol=1e-5)
    with pytest.raises(ValueError, match="CUDA"):
        R.run(R.parser().parse_args(["--device", "cpu", "--output", "/dev/null"]))


@pytest.mark.gpu
def test_replay_four_arms_on_gpu(tmp_path, cuda_device):
    """The four arms on clustered synthetic input: every arm stays close to
    the exact FP32 result, and the report records metrics and timings."""
    out = tmp_path / "report.json"
    report = R.run(R.parser().parse_args(["--tokens", "640", "--heads", "2", "--dim", "128", "--clustered",
                                          "--repeats", "2", "--output", str(out)]))
    assert json.loads(out.read_text())["arms"].keys() == set(R.ARMS)
    for name, row in report["arms"].items():
        assert row["metrics"]["cosine"] > 0.99 and row["metrics"]["relative_rmse"] < 0.15, (name, row["metrics"])
        assert len(row["wall_ms"]) == 2
    had = R.run(R.parser().parse_args(["--tokens", "384", "--heads", "1", "--hadamard", "--repeats", "1",
                                       "--output", str(tmp_path / "h.json")]))
    assert had["arms"]["expcast"]["config"]["qk_hadamard"] and had["arms"]["expcast"]["metrics"]["cosine"] > 0.99


@pytest.mark.gpu
def test_adapter_matches_direct_attention_on_gpu(tmp_path, cuda_device):
    """The adapter's output equals a direct vc_attention.attention call with
    the same config, cache history and step."""
    from vc_attention import Config, LayoutCache, attention
    a = X.ExperimentAdapter(_options(tmp_path, mode="combined"), _audit())
    s = FakeScheduler(steps=8)
    g = torch.Generator().manual_seed(5)
    x = [torch.randn(300, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3)]
    got = a.apply(*x, scheduler=s, block_idx=3)
    cache = LayoutCache(Config(v_smooth=True, expcast=True, backend="sm100a", qk_hadamard=False))
    q, k, v = (t.transpose(0, 1).unsqueeze(0) for t in x)
    want, _ = attention(q, k, v, cache.config, cache=cache, step=0, total_steps=8, request_id=1, layer_id=3)
    assert torch.equal(got, want.squeeze(0).transpose(0, 1).reshape(300, -1))
