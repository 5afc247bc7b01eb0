"""Failure path of the bounded device waits (needs a B200; no GPU fault is raised).

mib_test_inject_wait_expiry arms a one-shot flag on the host: the next MVM launch holds its MMA warp,
so no accumulator is ever committed, and its abortable waits get a ~1 ms limit.  The epilogue's
first wait therefore runs out by design; the kernel raises its abort flag, drains its in-flight TMA
copies and MMA work, frees its tensor memory and returns.  The test checks that the host sees
MIB_ERR_TIMEOUT from mib_device_status, that the context stays usable, and that the next MVM is
exact again.
"""
import numpy as np
import pytest
import torch

import golden_cases as G
from helpers import gpu_pair, oracle_pair, rel_norm
from oracle import cim_oracle as O

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_next_call_is_exact(cuda):
    from memintelli_flash_b200 import _native as N
    c = G.case("cfg0_int")
    eng, xs, ws = gpu_pair(c, cuda)
    N.device_status()                                   # clean before
    N.call("mib_test_inject_wait_expiry", 2_000_000)    # ~1 ms at 1.9 GHz
    eng(xs, ws)                                         # this launch's output is undefined
    with pytest.raises(RuntimeError, match="bounded device wait expired"):
        N.device_status()
    N.device_status()                                   # the flag was read and cleared
    assert float(torch.ones(4, device=cuda).sum()) == 4.0   # the context still works
    y = eng(xs, ws).double().cpu().numpy()
    oxs, ows, oeng, wl = oracle_pair(c)
    assert rel_norm(y, O.mvm_exact(oxs, ows, oeng, wl)) <= 1e-5
    N.device_status()


def test_injection_arguments_checked():
    from memintelli_flash_b200 import _native as N
    with pytest.raises(ValueError):
        N.call("mib_test_inject_wait_expiry", 0)
