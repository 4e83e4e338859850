"""Failure detection on the GPU without a fault: a bounded wait runs out.

Every pipelined kernel waits on mbarriers with a wall-time limit and, when a
wait gives up, sets SCOPE_DEVERR_TIMEOUT in the per-device error word,
winds down (freeing TMEM) and exits.  scope_selftest_wait_timeout runs that
path on a barrier nothing ever arrives on; the host reads the status, and
the context keeps running kernels correctly afterwards."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_stays_usable():
    from scope_b200 import _lib, device_errors, trig_tables
    dev = torch.device("cuda", 0)
    device_errors(dev)                                   # clear
    st = _lib.lib().scope_selftest_wait_timeout(_lib.err_word_ptr(dev), 20000,
                                                 torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, "scope_selftest_wait_timeout")
    torch.cuda.synchronize(dev)
    bits = device_errors(dev)
    assert bits & 0x2, f"expected SCOPE_DEVERR_TIMEOUT, error word {bits:#x}"
    # the context is intact: a kernel launched afterwards runs and is right
    w = torch.tensor([math.pi * 2.0 ** (-k) for k in range(4)], device=dev)
    c, s = trig_tables(w, 256)
    d = torch.arange(256, device=dev, dtype=torch.float32)
    ref = torch.cos(w[:, None] * d[None, :]).to(torch.bfloat16)
    assert torch.equal(c, ref) or (c.float() - ref.float()).abs().max().item() <= 2 ** -8
    assert device_errors(dev) == 0


def test_selftest_rejects_bad_arguments():
    from scope_b200 import _lib
    assert _lib.lib().scope_selftest_wait_timeout(None, 1000, None) == -1
