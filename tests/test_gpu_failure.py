"""Failure detection on the GPU without a GPU fault: a bounded wait on an
mbarrier that nothing arrives on gives up, records the wait-timeout code
that the host reads, frees its TMEM and exits, and the context keeps
working (a prefill right after it matches the oracle)."""
from __future__ import annotations

import pytest

import inference_c_b200 as P
from tests.gpu_cases import check_close
from tests.test_gpu_prefill import PrefillCase

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 4  # kFaultWaitTimeout


def test_bounded_wait_gives_up_and_context_survives(lib, oracle_mod, cuda):
    assert P.selftest_wait_timeout() == WAIT_TIMEOUT
    assert P.device_fault(0) == 0  # the kernels' own fault words are untouched
    case = PrefillCase([0, 300], [200, 129], 8, 2, "bf16", seed=31, device=cuda)
    check_close(case.run(True), case.oracle(oracle_mod, True), "prefill after the self-test")
    assert P.selftest_wait_timeout() == WAIT_TIMEOUT  # repeatable: TMEM was freed
    assert P.device_fault(0) == 0
