"""The Config API (boundary A): Config validation, the error contract of
``attention`` and the LayoutCache schedule, on the host (no GPU).

Mirrors the reference package's tests of src/vc_attention/core.py: the same
ValueError messages and LayoutCache semantics, plus the sm100a rules.
"""
import dataclasses

import pytest
import torch

from vc_attention import Config, LayoutCache, attention
from vc_attention import core


def test_config_defaults_match_the_reference():
    c = Config()
    assert (c.expcast, c.v_smooth, c.quantize, c.q_block, c.k_quant_block, c.kv_block) == \
        (False, False, True, 128, 256, 128)
    assert (c.clusters, c.iterations, c.active_fraction, c.refresh_interval, c.mean_dtype, c.backend) == \
        (8, 2, 0.25, 4, "float16", "reference")
    assert (c.k_smooth, c.qk_hadamard, c.cuda_schedule) == (True, True, "batched")
    assert dataclasses.is_dataclass(c)
    with pytest.raises(dataclasses.FrozenInstanceError):
        c.expcast = True


@pytest.mark.parametrize("kwargs,match", [
    ({"cuda_schedule": "x"}, "cuda_schedule"),
    ({"k_smooth": 1}, "bool"),
    ({"q_block": 0}, "positive integer"),
    ({"clusters": True}, "positive integer"),
    ({"active_fraction": 1.5}, "active_fraction"),
    ({"mean_dtype": "int8"}, "mean_dtype"),
    ({"backend": "tpu"}, "backend"),
    ({"backend": "cuda_fp8", "quantize": False}, "quantize"),
    ({"backend": "cuda_fp8", "k_quant_block": 200}, "divide"),
    ({"backend": "sm100a", "expcast": True, "k_quant_block": 200}, "multiple of 128"),
    ({"backend": "sm100a", "expcast": True, "k_quant_block": 8192}, "multiple of 128"),
    ({"backend": "sm100a", "qk_hadamard": False, "quantize": False}, "quantize"),
    ({"backend": "sm100a", "qk_hadamard": False, "q_block": 64}, "q_block=128"),
    ({"backend": "sm100a", "qk_hadamard": False, "kv_block": 256, "k_quant_block": 256}, "kv_block=128"),
    ({"backend": "sm100a", "qk_hadamard": False, "v_smooth": True, "clusters": 257}, "256 clusters"),
    ({"backend": "sm100a", "qk_hadamard": False, "mean_dtype": "bfloat16"}, "float16"),
])
def test_config_rejects(kwargs, match):
    with pytest.raises(ValueError, match=match):
        Config(**kwargs)


def test_sm100a_config_accepts_its_contract():
    c = Config(backend="sm100a", qk_hadamard=False, expcast=True, v_smooth=True)
    assert c.backend == "sm100a"
    assert Config(backend="sm100a", qk_hadamard=False, v_smooth=True, clusters=256).clusters == 256
    # the reference's defaults (no ExpCast, Hadamard E4M3 block Q/K) are accepted
    d = Config(backend="sm100a")
    assert not d.expcast and d.qk_hadamard and d.k_quant_block == 256


def _qkv(shape=(1, 2, 5, 64), dtype=torch.float16):
    x = torch.zeros(shape, dtype=dtype)
    return x, x.clone(), x.clone()


@pytest.mark.parametrize("kwargs,match", [
    ({"causal": True}, "causal"),
    ({"mask": torch.zeros(1)}, "mask"),
])
def test_attention_rejects_unsupported_modes(kwargs, match):
    q, k, v = _qkv()
    with pytest.raises(ValueError, match=match):
        attention(q, k, v, Config(backend="sm100a", qk_hadamard=False), **kwargs)


def test_attention_shape_and_dtype_contract():
    cfg = Config(backend="sm100a", qk_hadamard=False)
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="BNSD"):
        attention(q[0], k[0], v[0], cfg)
    with pytest.raises(ValueError, match="GQA"):
        attention(q, k[:, :1], v[:, :1], cfg)
    with pytest.raises(ValueError, match="Incompatible"):
        attention(q, k[..., :32], v, cfg)
    with pytest.raises(ValueError, match="Empty"):
        attention(q[:, :, :0], k, v, cfg)
    with pytest.raises(ValueError, match="same device and dtype"):
        attention(q, k.float(), v, cfg)
    with pytest.raises(ValueError, match="FP16/BF16/FP32"):
        attention(q.double(), k.double(), v.double(), cfg)
    bad = q.clone()
    bad[0, 0, 0, 0] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        attention(bad, k, v, cfg)


def test_attention_has_no_cpu_or_reference_fallback():
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="no CPU/NPU fallback"):
        attention(q, k, v, Config(backend="sm100a", qk_hadamard=False))
    with pytest.raises(ValueError, match="not built here"):
        attention(q, k, v, Config(backend="reference"))


class _FakeGrouping:
    """Stands in for the device grouping: records calls and warm starts."""

    def __init__(self):
        self.calls = []

    def __call__(self, v, centers):
        self.calls.append(centers)
        perm = torch.arange(v.shape[-2]).expand(*v.shape[:-1]).clone()
        return perm, torch.full((*v.shape[:2], 2, v.shape[-1]), float(len(self.calls)))


def test_layout_cache_schedule(monkeypatch):
    cfg = Config(backend="sm100a", qk_hadamard=False, v_smooth=True, active_fraction=0.25, refresh_interval=4)
    cache = LayoutCache(cfg)
    fake = _FakeGrouping()
    monkeypatch.setattr(cache, "_group", fake)
    v = torch.zeros(1, 2, 10, 64)
    seen = []
    for step in range(20):
        pi, active, refreshed = cache.layout(v, step=step, total_steps=20, request_id="r1", layer_id=0)
        seen.append((pi is not None, active, refreshed))
    # active for the first ceil(20 * 0.25) = 5 steps, refreshed every 4 of them, layout kept afterwards
    assert [s[1] for s in seen] == [True] * 5 + [False] * 15
    assert [s[2] for s in seen] == [True, False, False, False, True] + [False] * 15
    assert all(s[0] for s in seen)
    assert len(fake.calls) == 2 and fake.calls[0] is None and fake.calls[1] is not None   # warm start
    assert cache.entries == 1
    # another layer has its own state; a new request drops everything
    cache.layout(v, step=0, total_steps=20, request_id="r1", layer_id=7)
    assert cache.entries == 2
    cache.layout(v, step=0, total_steps=20, request_id="r2", layer_id=0)
    assert cache.entries == 1
    # a changed V signature or a step going backwards drops the layer's state
    cache.layout(v, step=1, total_steps=20, request_id="r2", layer_id=0)
    _, _, refreshed = cache.layout(torch.zeros(1, 2, 12, 64), step=2, total_steps=20, request_id="r2", layer_id=0)
    assert refreshed
    _, _, refreshed = cache.layout(torch.zeros(1, 2, 12, 64), step=0, total_steps=20, request_id="r2", layer_id=0)
    assert refreshed


def test_layout_cache_contract_errors():
    cache = LayoutCache(Config(backend="sm100a", qk_hadamard=False))
    v = torch.zeros(1, 1, 4, 64)
    with pytest.raises(ValueError, match="request_id"):
        cache.layout(v, step=0, total_steps=1, request_id=None, layer_id=0)
    with pytest.raises(ValueError, match="step"):
        cache.layout(v, step=3, total_steps=2, request_id="r", layer_id=0)
    # smoothing off: no grouping, no permutation
    assert cache.layout(v, step=0, total_steps=1, request_id="r", layer_id=0) == (None, False, False)


def test_expcast_codes_has_no_cpu_path():
    with pytest.raises(ValueError, match="CUDA"):
        core.expcast_codes(torch.zeros(4))


def test_sm100a_config_accepts_the_hadamard_path():
    """qk_hadamard=True (the Config contract's E4M3 block Q/K) is accepted
    with ExpCast and K scale blocks that are multiples of 128 rows."""
    from vc_attention import Config
    for kqb in (128, 256, 4096):
        c = Config(backend="sm100a", expcast=True, qk_hadamard=True, k_quant_block=kqb)
        assert c.qk_hadamard and c.k_quant_block == kqb
