"""The bounded in-kernel waits end with an error status, not a hang (GPU).

`b200_wait_selftest` launches one warp that waits on an mbarrier nothing ever
arrives on.  The wait must give up after its limit, record
B200_DEVERR_WAIT_TIMEOUT in the library's device error word and return; the
context must stay usable, so an attention call right after it still matches
the oracle.  No fault, trap or unbounded loop is involved.
"""

from __future__ import annotations

import time

import pytest
import torch

from helpers import assert_close, oracle, run_gpu, small_batch
from minicpm_b200 import _lib

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_stays_usable():
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    _lib.device_error()  # start from a clear error word
    t0 = time.monotonic()
    _lib.check(lib.b200_wait_selftest(_lib.current_stream(dev)), "b200_wait_selftest")
    assert _lib.device_error() == _lib.DEVERR_WAIT_TIMEOUT
    elapsed = time.monotonic() - t0
    assert 1.0 < elapsed < 60.0, elapsed  # the limit is 2 s of %globaltimer
    assert _lib.device_error() == _lib.DEVERR_NONE  # read-and-clear

    batch = small_batch([17, 1, 64], [111, 255, 2048], seed=20261202)
    got = run_gpu(batch, 4)
    assert_close(got, oracle(batch).to(torch.bfloat16), "attention after a timed-out wait")
    assert _lib.device_error() == _lib.DEVERR_NONE
