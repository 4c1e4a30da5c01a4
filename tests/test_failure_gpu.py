"""Failure paths on the GPU, without a GPU fault.

Every device wait in the library is bounded: when what it waits for never
happens it gives up, raises KSH_FLAG_TIMEOUT in the caller's status word and
the kernel returns, so the context stays usable and the host turns the flag
into an exception.  The waits here are made to run out on an mbarrier phase
and a flag word that nothing completes (ksh_check_bounded_wait), with short
limits; nothing is faulted, trapped or left hanging.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT = 64


def _run(polls, arrive):
    from kshipra_b200 import _lib
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    where = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")    # nothing ever sets it
    t0 = time.perf_counter()
    _lib.call("ksh_check_bounded_wait", polls, arrive, word.data_ptr(), flags.data_ptr(),
              where.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    return int(flags.item()), int(where.item()), time.perf_counter() - t0, flags


def test_completed_waits_raise_nothing():
    f, w, _, _ = _run(1000, 1)
    assert (f, w) == (0, 0)


@pytest.mark.parametrize("polls", [1, 64, 4096])
def test_waits_that_never_complete_give_up_and_report(polls):
    from kshipra_b200.model import KshipraDeviceTimeout, _check_flags
    f, w, dt, flags = _run(polls, 0)
    assert f == TIMEOUT and w == 3          # both the mbarrier and the flag wait gave up
    assert dt < 10.0
    with pytest.raises(KshipraDeviceTimeout):
        _check_flags(flags)
    assert int(flags.item()) == 0            # the host clears the word after reporting
    # the context is still usable: an ordinary kernel runs and is right
    from kshipra_b200 import _lib
    x = torch.randn(3, 256, device="cuda")
    wn = torch.ones(256, device="cuda")
    y = torch.empty_like(x)
    _lib.call("ksh_rmsnorm", x.data_ptr(), wn.data_ptr(), y.data_ptr(), 3, 256, 1e-6,
              _lib.stream_ptr())
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(y, ref, rtol=1e-6, atol=1e-6)
