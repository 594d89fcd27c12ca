"""Bounded device waits: a wait that runs out reports and returns.

Every mbarrier wait in this library's kernels polls a bounded number of times
and then records KDA_DEVICE_ERR_WAIT_TIMEOUT in the caller's status word (the
reference's own waits, IBWait in kda_varlen_recurrent_prefill_h4.cpp:410-414,
have no bound). The library's self-test entry point runs that same wait on an
mbarrier that nothing arrives on, with a short poll limit, so every wait
expires: the status word must read the timeout code, every expiry must be
counted, the kernel must end normally, and the context must stay usable (a
decode launched afterwards matches the oracle). With the CTA-wide give-up word
(as the chunk kernels use it) only the first expiry costs the full poll
budget; the test checks that eight successive waits then take about as long
as one, and far less than eight without the word.
"""

import pytest
import torch

from kda_checks import assert_out_close, assert_state_close, clone_pool

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIMEOUT = 0x101   # KDA_DEVICE_ERR_WAIT_TIMEOUT
POLLS = 2048


def _run(waits: int, give_up: bool):
    from sgl_glm53_ascend_ops import abi
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    expired = torch.zeros(1, dtype=torch.int32, device=DEV)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    rc = abi.selftest_wait_timeout(status, expired, POLLS, waits, give_up)
    b.record()
    torch.cuda.synchronize()
    assert rc == abi.KDA_OK
    return int(status.item()), int(expired.item()), a.elapsed_time(b)


def test_expired_wait_reports_and_returns():
    for give_up in (False, True):
        status, expired, _ = _run(1, give_up)
        assert status == TIMEOUT
        assert expired == 64                      # every thread's wait expired
    torch.cuda.synchronize()


def test_give_up_word_bounds_a_ctas_waits():
    _run(1, True)                                 # warm-up launch
    _, n_one, t_one = _run(1, True)
    status, n_eight, t_eight = _run(8, True)
    _, n_plain, t_plain = _run(8, False)
    assert status == TIMEOUT and n_one == 64 and n_eight == 8 * 64 and n_plain == 8 * 64
    # with the word, waits 2..8 give up at their first poll
    assert t_eight < 2.0 * t_one + 0.5, (t_one, t_eight)
    assert t_eight < 0.5 * t_plain, (t_eight, t_plain)


def test_context_usable_after_expired_waits():
    import kda_workloads as workloads
    from oracle import kda_ref
    from sgl_glm53_ascend_ops import ops
    _run(4, True)
    w = workloads.config2(requests=8, heads=4, slots=16)
    d = w.to(DEV)
    out = ops.kda_varlen_recurrent_g(**d.kwargs(), prefill=False)
    torch.cuda.synchronize()
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out.cpu(), ref)
    idx = w.indices.long()
    assert_state_close(d.pool.cpu()[idx], ref_pool[idx])


def test_selftest_rejects_bad_arguments():
    from sgl_glm53_ascend_ops import abi
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert abi.selftest_wait_timeout(status, status, 0, 1, True) == abi.KDA_ERR_INVALID_ARGUMENT
    assert abi.selftest_wait_timeout(status, status, 16, 65, True) == abi.KDA_ERR_INVALID_ARGUMENT
