"""Failure detection on the GPU without a fault: a bounded wait that runs out.

cq_device_watchdog_check runs one kernel whose wait -- the library's bounded
mbarrier wait, the one every TMA pipeline here uses -- targets a barrier that
nothing arrives on.  The wait must give up after its limit, record the timeout
in the device status word and let the kernel end; calls that check the word
must then fail with CQ_RUNTIME_ERROR, cq_device_status must report and clear
it, and the next call must succeed with correct results (the context stays
usable).  Nothing here faults, traps or hangs the GPU.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from conftest import assert_parity

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_the_context_stays_usable(cq, oracle_mod):
    rng = np.random.default_rng(12)
    w = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    x = rng.standard_normal((14, 512)).astype(np.float32)
    layer = cq.QuantizedLinear.from_f32(w, 256, 512, np.zeros(256, np.float32), 64, "bf16")
    layer.forward_f32(x, 14)
    assert cq.device_status(0) == 0

    t0 = time.perf_counter()
    assert cq.lib().cq_device_watchdog_check(0) == cq.CQ_OK, cq.last_error()
    waited = time.perf_counter() - t0
    assert 1.5 < waited < 30.0, waited  # the wait's limit is 2 s

    with pytest.raises(cq.CQError) as ei:
        layer.forward_f32(x, 14)
    assert ei.value.status == cq.CQ_RUNTIME_ERROR
    assert "gave up waiting" in str(ei.value)
    assert cq.device_status(0) == 1  # the timeout bit, read and cleared

    y = layer.forward_f32(x, 14).reshape(14, 256)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    want = oracle_mod.qmatmul(oracle_mod.to_t(x, "bf16"), q, s, b, 64, "bf16")
    assert_parity(oracle_mod.to_t(y, "bf16"), want, "bf16", min_exact=0.9)
    assert cq.device_status(0) == 0
