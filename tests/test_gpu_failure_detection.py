"""Failure detection on the GPU without a GPU fault.

Every wait inside this library's kernels is an mbarrier wait bounded in
wall time; when the budget runs out the kernel sets a bit in the device error
word and returns instead of hanging (the reference spins without bound,
third_party/sageattention_local/csrc/vc/vc_sm90.cu:114-128).  Here a wait is
made to run out on purpose -- one warp waits, through that same bounded wait,
for an mbarrier phase that nothing completes, with a 5 ms budget -- and the
test checks the reported status and that the context is still usable.
"""
import pytest
import torch

from oracle import vc_oracle as O
from inputs import qk_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    from vc_b200 import ops as _ops
    from vc_b200 import _native
    _native.load()
    _ops.error_word(0, clear=True)
    return _ops


def test_bounded_wait_runs_out_and_reports(ops):
    r = ops.wait_timeout_selftest(5_000_000)
    assert r["wait_ok"] == 0, r                                  # the wait did not pretend to succeed
    assert r["error_word"] & ops.ERR_WAIT_SELFTEST, r            # and said so in the error word
    assert r["error_word"] & ~ops.ERR_WAIT_SELFTEST == 0, r      # nothing else was flagged
    assert 4.0 <= r["ms"] < 2000.0, r                            # it waited about its budget, then returned
    assert ops.error_word(0, clear=True) == 0                    # the read cleared the word
    # two more in a row: each reports again, none leaves state behind
    for budget in (1_000_000, 20_000_000):
        r = ops.wait_timeout_selftest(budget)
        assert r["wait_ok"] == 0 and r["error_word"] == ops.ERR_WAIT_SELFTEST
        assert budget / 1e6 * 0.8 <= r["ms"] < budget / 1e6 + 2000.0


def test_context_usable_after_a_wait_ran_out(ops):
    """After the self-test gave up, the full pipeline still runs on the same
    context and meets the parity tolerance against the oracle."""
    r = ops.wait_timeout_selftest(2_000_000)
    assert r["wait_ok"] == 0 and r["error_word"] == ops.ERR_WAIT_SELFTEST, r
    from sageattention_local import sageattn_vc
    q, k, v = qk_inputs(61, (1, 2, 300, 128), torch.bfloat16, 3 ** 0.5)
    out = sageattn_vc(q.cuda(), k.cuda(), v.cuda(), v_smooth=False)
    torch.cuda.synchronize()
    ref = O.reference(O.prepare(q, k, v, v_smooth=False, km=O.k_mean(k)))
    m = O.metrics(out.float().cpu(), ref)
    assert m["cos"] >= 0.9999 and m["rel_l2"] <= 4e-3, m
    assert ops.error_word(0, clear=True) == 0
