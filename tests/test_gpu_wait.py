"""Bounded waits.  Every kernel of the library waits on its mbarriers for a bounded number of
polls and, when a wait gives up, records an error in its status word and winds down instead of
hanging the GPU.  Here one warp waits on a barrier that nothing arrives on: the wait must give
up, the kernel must finish and the context must stay usable.  A barrier that one thread arrives
on first completes at once.  The measured cycles per poll give the real length of the kernels'
default bounds (mbar_wait_fast: 2^19 polls; mbar_wait: 400000 polls with a 100 us suspend hint),
which should be of the order of a second: long against any kernel step, short against a hang."""

import pytest
import torch

pytestmark = pytest.mark.gpu

FAST, ARRIVED = 1, 2


def _wait(mode, limit):
    from kvstreams import _native as N

    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    rc = N.lib().kvs_selftest_wait(mode, limit, out.data_ptr(), N.stream_ptr(out.device))
    assert rc == 0
    torch.cuda.synchronize()
    o = out.cpu().tolist()
    return o[0], (o[1] & 0xFFFFFFFF) | (o[2] << 32)


@pytest.mark.parametrize("mode,limit", [(FAST, 4096), (0, 20)])
def test_wait_on_a_barrier_nothing_arrives_on_gives_up(mode, limit):
    gave_up, cycles = _wait(mode, limit)
    assert gave_up == 1
    assert cycles > 0
    # the context is usable after the timeout
    x = torch.arange(1000, device="cuda", dtype=torch.int64)
    assert int(x.sum()) == 999 * 1000 // 2


@pytest.mark.parametrize("mode", [ARRIVED, ARRIVED | FAST])
def test_wait_on_an_arrived_barrier_completes(mode):
    gave_up, _ = _wait(mode, 20)
    assert gave_up == 0


def test_default_bounds_are_seconds_not_forever():
    """Cycles per poll of both waits, scaled to their default limits: finite, and long enough
    (well above a step of any kernel) not to give up on a slow but live pipeline."""
    _, c_fast = _wait(FAST, 1 << 14)
    _, c_susp = _wait(0, 50)
    clock_hz = torch.cuda.get_device_properties(0).clock_rate * 1e3 if hasattr(
        torch.cuda.get_device_properties(0), "clock_rate") else 1.9e9
    fast_s = c_fast / (1 << 14) * (1 << 19) / clock_hz
    susp_s = c_susp / 50 * 400000 / clock_hz
    print(f"mbar_wait_fast default bound ~{fast_s:.2f} s, mbar_wait default bound ~{susp_s:.2f} s")
    assert 0.1 < fast_s < 10
    assert 0.1 < susp_s < 10
