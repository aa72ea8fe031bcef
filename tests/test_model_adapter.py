"""The LightX2V attention layer, capture path and four-arm replay
(vc_attention.lightx2v / vc_attention.replay).  Host logic runs on CPU with
a fake H3 scheduler and an injected attention function; the GPU tests run
the real replay and compare the layer with a direct attention call."""
import json

import pytest
import torch

from vc_attention import lightx2v as X
from vc_attention import replay as R


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


def _sink(tmp_path, **kw):
    base = dict(rank=0, steps=[0, 2], layers=[0], heads=1, max_files=4, max_bytes=64 * 1024 ** 2)
    base.update(kw)
    return X.CaptureSink(tmp_path, **base)


def test_parse_call_accepts_snd_and_1snd():
    x = torch.randn(10, 3, 8)
    call = X.parse_call(x, x, x)
    assert call.q.shape == (1, 3, 10, 8) and torch.equal(call.q[0, 1], x[:, 1])
    assert call.tokens == 10 and call.scale == 8 ** -0.5 and call.layer is None
    c2 = X.parse_call(x[None], x[None], x[None], torch.tensor([0, 10]), None, 10, 10,
                      {"block_idx": 2, "softmax_scale": 0.25})
    assert torch.equal(c2.q, call.q) and c2.layer == 2 and c2.scale == 0.25
    assert torch.equal(X.to_snd(call.q, 10, x.dtype), x.reshape(10, 24))


@pytest.mark.parametrize("options,extra,match", [
    ({"foo": 1}, {}, "unsupported attention options"),
    ({"causal": True}, {}, "non-causal"),
    ({"dropout": 0.1}, {}, "non-causal"),
    ({"attn_mask": torch.ones(1)}, {}, "mask"),
    ({"pse": torch.ones(1)}, {}, "positional bias"),
    ({}, {"cu_q": torch.tensor([0, 4, 10])}, "unpacked"),
    ({}, {"max_q": 9}, "max_seqlen"),
    ({}, {"k_shape": (10, 2, 8)}, "SND or 1SND"),
])
def test_parse_call_rejects(options, extra, match):
    x = torch.randn(10, 3, 8)
    k = torch.randn(*extra.get("k_shape", (10, 3, 8)))
    with pytest.raises(ValueError, match=match):
        X.parse_call(x, k, x, extra.get("cu_q"), None, extra.get("max_q"), None, options)


def test_configure_patches_and_rejects():
    cfg = X.configure({"warmup": False, "parallel": {"seq_p_attn_type": "ulysses"}, "model": "h3"})
    assert cfg["attn_type"] == X.ATTN_TYPE and cfg["warmup"] is False and cfg["model"] == "h3"
    assert cfg["refiner_attn_type"] == "npu_flash_attn"
    for bad, match in (({"use_compile": True}, "use_compile"), ({"warmup": True}, "warmup"),
                       ({"parallel": {"seq_p_head_parallel": True}}, "head_parallel"),
                       ({"parallel": {"seq_p_attn_type": "ring"}}, "Ulysses"), ({"enable_cfg": True}, "CFG")):
        with pytest.raises(ValueError, match=match):
            X.configure(bad)


def test_request_tracker():
    t = X.RequestTracker()
    s = FakeScheduler()
    assert t.observe(s, 0) == (1, 0, 4, True)
    assert t.observe(s, 1) == (1, 0, 4, False)
    s.step_index = 1
    assert t.observe(s, 0)[:3] == (1, 1, 4)
    with pytest.raises(ValueError, match="repeated or reversed"):
        t.observe(s, 0)
    s.step_index = 0                      # step 0 again for a seen layer: a new request
    assert t.observe(s, 0) == (2, 0, 4, True)
    assert t.observe(FakeScheduler(), 0)[0] == 3   # a new layout marker: a new request
    with pytest.raises(ValueError, match="block_idx"):
        t.observe(s, None)
    with pytest.raises(ValueError, match="layout_cpu"):
        t.observe(object(), 0)


def test_layer_steps_layers_and_requests():
    """Steps come from the scheduler, layers from block_idx, the request id
    from the tracker; SND output; audit counters."""
    calls = []
    a = X.H3VCAttention("combined", rank=0, attention_fn=_fake_attention(calls))
    s = FakeScheduler()
    x = torch.randn(12, 2, 8)
    out = a.apply(x, x, x, scheduler=s, block_idx=0, softmax_scale=0.5)
    assert out.shape == (12, 16) and torch.equal(out, (x * 2).reshape(12, 16))
    a.apply(x, x, x, scheduler=s, block_idx=1)
    s.step_index = 1
    a.apply(x, x, x, scheduler=s, block_idx=0)
    with pytest.raises(ValueError, match="repeated or reversed"):
        a.apply(x, x, x, scheduler=s, block_idx=0)
    assert [c[0] for c in calls] == [0, 0, 1] and {c[2] for c in calls} == {1}
    assert calls[0][4] == 0.5 and calls[1][4] == 8 ** -0.5
    s.step_index = 0
    a.apply(x, x, x, scheduler=s, block_idx=0)
    a.apply(x, x, x, scheduler=FakeScheduler(), block_idx=0)
    assert [c[2] for c in calls] == [1, 1, 1, 2, 3]
    d = a.audit.as_dict()
    assert d["calls"] == 5 and d["smoothing_calls"] == 5 and d["regroup_calls"] == 4 and d["expcast_calls"] == 5
    cfg = calls[0][5]
    assert cfg.backend == "sm100a" and cfg.v_smooth and cfg.expcast and not cfg.qk_hadamard
    with pytest.raises(ValueError, match="mode must be"):
        X.H3VCAttention("mindie_fp8")
    with pytest.raises(ValueError, match="CaptureSink"):
        X.H3VCAttention("capture")


def test_arm_configs():
    assert not X.arm_config("fp8_control").expcast and not X.arm_config("fp8_control").v_smooth
    assert X.arm_config("expcast", hadamard=True).qk_hadamard
    assert X.arm_config("fp8_control", hadamard=True).qk_hadamard    # the Config contract's own control arm
    assert not X.arm_config("v_smooth").qk_hadamard
    cfgs = R.arm_configs(hadamard=True)
    assert set(cfgs) == set(R.ARMS) and all(c.qk_hadamard for c in cfgs.values())
    with pytest.raises(ValueError, match="unknown arm"):
        X.arm_config("capture")


def test_capture_writes_files_within_budget(tmp_path):
    """Capture mode saves the chosen steps/layers of one rank (first heads,
    BNSD, with metadata) once each, returns the BF16 SDPA output, and stops
    at the byte budget with an error; the replay reads the files back."""
    a = X.H3VCAttention("capture", capture=_sink(tmp_path, heads=2), rank=0)
    s = FakeScheduler()
    x = torch.randn(16, 3, 8)
    out = a.apply(x, x, x, scheduler=s, block_idx=0)
    c = X.parse_call(x, x, x)
    ref = torch.nn.functional.scaled_dot_product_attention(*(t.to(torch.bfloat16) for t in (c.q, c.k, c.v)))
    assert torch.equal(out, ref[0].permute(1, 0, 2).reshape(16, 24).to(x.dtype))
    a.apply(x, x, x, scheduler=s, block_idx=1)   # layer 1 is not captured
    s.step_index = 2
    a.apply(x, x, x, scheduler=s, block_idx=0)
    assert sorted(a.audit.captures) == ["rank0_step0_layer0", "rank0_step2_layer0"]
    case = R.load_capture(a.audit.captures["rank0_step0_layer0"])
    assert case.q.shape == (1, 2, 16, 8) and case.scale == 8 ** -0.5 and case.source["metadata"]["layer"] == 0
    assert torch.equal(case.q[0, 1], x[:, 1]) and len(case.source["sha256"]) == 64
    other_rank = X.H3VCAttention("capture", capture=_sink(tmp_path / "r"), rank=1)
    other_rank.apply(x, x, x, scheduler=FakeScheduler(), block_idx=0)
    assert other_rank.audit.captures == {}
    small = X.H3VCAttention("capture", capture=_sink(tmp_path / "b", max_bytes=1024 ** 2), rank=0)
    big = torch.randn(40000, 1, 8)
    with pytest.raises(ValueError, match="budget"):
        small.apply(big, big, big, scheduler=FakeScheduler(), block_idx=0)


def test_prepare_only_writes_patched_config(tmp_path):
    src = tmp_path / "h3.json"
    src.write_text(json.dumps({"model": "h3", "parallel": {}}))
    path = X.main(["--mode", "expcast", "--output-dir", str(tmp_path / "out"), "--prepare-only", "--",
                   "--config_json", str(src), "--seed", "1"])
    cfg = json.loads(path.read_text())
    assert cfg["attn_type"] == X.ATTN_TYPE and cfg["model"] == "h3" and cfg["warmup"] is False


def test_replay_helpers():
    a, b = R.synthetic(256, 2, 64, 3, clustered=True), R.synthetic(256, 2, 64, 3, clustered=True)
    assert torch.equal(a.v, b.v) and a.q.shape == (1, 2, 256, 64) and a.scale == 64 ** -0.5
    w = a.query_window(128, 64)
    assert w.q.shape == (1, 2, 64, 64) and w.k.shape == a.k.shape and w.source["query_range"] == [128, 192]
    with pytest.raises(ValueError, match="multiple of 128"):
        a.query_window(64, 0)
    m = R.metrics(a.q + 0.01, a.q)
    assert abs(m["rmse"] - 0.01) < 1e-6 and m["cosine"] > 0.999 and m["max_abs"] == pytest.approx(0.01, rel=1e-4)
    with pytest.raises(ValueError, match="Nonfinite"):
        R.metrics(torch.tensor([float("nan")]), torch.tensor([1.0]))
    ex = R.exact_attention(a.q, a.k, a.v, 64 ** -0.5, chunk=100)
    dense = torch.softmax((a.q @ a.k.transpose(-1, -2)) * 64 ** -0.5, dim=-1) @ a.v
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
        assert len(row["wall_ms"]) == 2 and all(t > 0 for t in row["wall_ms"])
    had = R.run(R.parser().parse_args(["--tokens", "384", "--heads", "1", "--hadamard", "--repeats", "1",
                                       "--output", str(tmp_path / "h.json")]))
    assert had["arms"]["expcast"]["config"]["qk_hadamard"] and had["arms"]["expcast"]["metrics"]["cosine"] > 0.99


@pytest.mark.gpu
def test_layer_matches_direct_attention_on_gpu(tmp_path, cuda_device):
    """The layer's output equals a direct vc_attention.attention call with
    the same config, cache history and step."""
    from vc_attention import Config, LayoutCache, attention
    a = X.H3VCAttention("combined", rank=0)
    s = FakeScheduler(steps=8)
    g = torch.Generator().manual_seed(5)
    x = [torch.randn(300, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3)]
    got = a.apply(*x, scheduler=s, block_idx=3)
    cache = LayoutCache(Config(v_smooth=True, expcast=True, backend="sm100a", qk_hadamard=False))
    q, k, v = (t.transpose(0, 1).unsqueeze(0) for t in x)
    want, _ = attention(q, k, v, cache.config, cache=cache, step=0, total_steps=8, request_id=1, layer_id=3)
    assert torch.equal(got, want.squeeze(0).transpose(0, 1).reshape(300, -1))
