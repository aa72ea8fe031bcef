"""vc_prep_v_channel_static: the allocation-free variant of vc_prep_v_channel.

Its scratch is a library-owned static device array shared by every call, so
the test makes two calls in a row whose inputs differ in shape and scale (a
stale amax left by the first call would corrupt the second) and checks each
against the workspace entry point vc_prep_v_channel, bit for bit (the
tolerance every E4M3 V-payload test here uses).  Each call is checked to
allocate nothing: neither torch's caching allocator nor the device's free
memory (cudaMemGetInfo) moves across it.  The array is also filled exactly to
its limit once.  Named to be collected last.
"""
import ctypes as C

import pytest
import torch

from vc_b200 import _native as N
from vc_b200 import ops

pytestmark = pytest.mark.gpu

_DT = {torch.float16: N.VC_DTYPE_F16, torch.bfloat16: N.VC_DTYPE_BF16, torch.float32: N.VC_DTYPE_F32}


def _static_call(v, perm=None):
    lib = N.load()
    B, H, S, D = v.shape
    npad = (S + 127) // 128 * 128
    v8 = torch.empty((B, H, D, npad), dtype=torch.uint8, device=v.device)
    vs = torch.empty((B, H, D), dtype=torch.float32, device=v.device)
    # the entry point works on the current device: make it the tensors' device
    with torch.cuda.device(v.device):
        stream = torch.cuda.current_stream(v.device).cuda_stream
        torch.cuda.synchronize(v.device)
        before = torch.cuda.memory_allocated(v.device)
        free_before = torch.cuda.mem_get_info(v.device)[0]
        rc = lib.vc_prep_v_channel_static(C.c_void_p(v.data_ptr()), _DT[v.dtype], B, H, S, D, v.stride(0),
                                          v.stride(1), v.stride(2),
                                          C.c_void_p(perm.data_ptr() if perm is not None else 0),
                                          C.c_void_p(v8.data_ptr()), C.c_void_p(vs.data_ptr()), C.c_void_p(stream))
        N.check(rc, "vc_prep_v_channel_static")
        torch.cuda.synchronize(v.device)
        assert torch.cuda.memory_allocated(v.device) == before
        assert torch.cuda.mem_get_info(v.device)[0] == free_before, "device memory was allocated"
    return v8, vs


def _input(seed, shape, dtype, scale, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(shape, generator=g) * scale
    x[..., 3] = 0.0                      # an all-zero channel (scale 0, payload 0)
    return x.to(dtype).to(device)


def test_static_scratch_matches_workspace_entry_two_calls(cuda_device):
    cases = [
        # large values first, so a stale amax would inflate the second call's scales
        (11, (2, 3, 1000, 128), torch.bfloat16, 40.0, False),
        (12, (1, 2, 300, 64), torch.float16, 0.25, True),
    ]
    for seed, shape, dtype, scale, with_perm in cases:
        v = _input(seed, shape, dtype, scale, cuda_device)
        perm = None
        if with_perm:
            # one permutation of the S tokens per (batch, head): [B, H, S] int64
            g = torch.Generator(device="cpu").manual_seed(seed + 1)
            B, H, S, _ = shape
            perm = torch.stack([torch.randperm(S, generator=g) for _ in range(B * H)]).reshape(B, H, S)
            perm = perm.to(cuda_device)
        v8_s, vs_s = _static_call(v, perm)
        v8_w, vs_w = ops.prep_v_channel(v, perm=perm)
        torch.cuda.synchronize()
        assert torch.equal(vs_s, vs_w), f"scales differ for {shape}"
        assert torch.equal(v8_s, v8_w.view(torch.uint8)), f"payload differs for {shape}"
        assert (vs_s[..., 3] == 0).all()
    assert N.error_word(0) == 0


def test_static_scratch_exactly_full(cuda_device):
    """B*H*D = 262144 words: the whole array, its last word included."""
    _static_call(_input(13, (1, 2, 200, 128), torch.bfloat16, 1.0, cuda_device))   # first call: address resolved
    v = _input(14, (1, 2048, 16, 128), torch.bfloat16, 3.0, cuda_device)
    v8_s, vs_s = _static_call(v)
    v8_w, vs_w = ops.prep_v_channel(v)
    torch.cuda.synchronize()
    assert torch.equal(vs_s, vs_w) and torch.equal(v8_s, v8_w.view(torch.uint8))
    assert N.error_word(0) == 0


def test_static_scratch_rejects_oversize(cuda_device):
    B, H, S, D = 1, 2049, 128, 128        # B*H*D = 262272 > 262144 words
    v = torch.zeros((B, H, S, D), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="static array"):
        _static_call(v)
