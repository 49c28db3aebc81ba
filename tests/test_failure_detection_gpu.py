"""Failure detection on one GPU without faulting it: a host-side deadline on a
step's stream (tk_stream_wait_deadline) reports work that does not finish in
time, and aborts a communicator the caller owns.  The busy stream is a
self-terminating sleep kernel; nothing waits on a flag that is never set."""
import ctypes

import pytest
import torch

from tikun_b200 import _native

pytestmark = pytest.mark.gpu

SLEEP_CYCLES = 400_000_000  # about 0.2 s at the B200's SM clock; ends by itself


def _own_comm():
    L = _native.lib()
    idb = ctypes.create_string_buffer(128)  # TK_NCCL_ID_BYTES
    _native.check(L.tk_nccl_unique_id(idb))
    c = ctypes.c_void_p()
    _native.check(L.tk_nccl_comm_init(idb, 1, 0, ctypes.byref(c)))
    return c


def _last_error():
    return _native.lib().tk_last_error().decode()


def test_deadline_reports_late_work_and_aborts_an_own_communicator():
    from tikun_b200.arena import Arena, LayoutPlan
    from tikun_b200.distributed import ShardedStep, ZeroHParams

    L = _native.lib()
    comm = _own_comm()
    code = ctypes.c_int32(-1)
    _native.check(L.tk_nccl_comm_async_error(comm, ctypes.byref(code)))
    assert code.value == 0

    # a sharded step on the caller's communicator, waited for with a deadline
    plan = LayoutPlan([1000, 37, 4099])
    P, G = Arena(plan, device="cuda"), Arena(plan, device="cuda")
    P.flat.normal_(0, 0.02)
    G.flat.normal_(0, 0.01)
    zp = ShardedStep(plan, P.flat, G.flat, ZeroHParams(max_norm=1.0), exchange="allgather",
                     comm=comm.value)
    zp.deadline_s = 10.0
    scale = zp.step(return_scale=True)
    assert 0.0 < scale <= 1.0
    zp.close()

    s = torch.cuda.Stream()
    sp = ctypes.c_void_p(s.cuda_stream)
    with torch.cuda.stream(s):
        x = torch.full((1024,), 2.0, device="cuda")
    assert L.tk_stream_wait_deadline(sp, 5000, comm) == 0  # finished work

    # busy past the deadline, no communicator: an error, the work goes on
    with torch.cuda.stream(s):
        torch.cuda._sleep(SLEEP_CYCLES)
    assert L.tk_stream_wait_deadline(sp, 20, None) == _native.TK_ERR_DEVICE
    assert "did not finish within 20 ms" in _last_error()
    s.synchronize()

    # again with the communicator: it is aborted (and must not be destroyed)
    with torch.cuda.stream(s):
        torch.cuda._sleep(SLEEP_CYCLES)
    assert L.tk_stream_wait_deadline(sp, 20, comm) == _native.TK_ERR_DEVICE
    assert "communicator was aborted" in _last_error()
    s.synchronize()

    # the device is still usable
    assert bool((x == 2.0).all())
    assert _native.device_status() == 0
