"""The device failure path, made to run on purpose without a fault: a bounded wait that runs out.

Every kernel of the library waits on mbarriers with a limit; when a limit runs out the kernel records
KDB_ERR_TIMEOUT and a site id in the device status word, raises its CTA's abort flag, frees its tensor
memory and returns.  kdb_selftest_wait_timeout runs exactly that path with a 1 ms limit on a barrier
nothing arrives on.  The test checks that the launch returns promptly, that the status word holds the
timeout with the self-test's site, and that the same context then runs a projection correctly."""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

from kdb200 import _lib, proj
from kdb200 import workloads as W
from oracle import proj as op

pytestmark = pytest.mark.gpu

SITE_SELFTEST = 0x1F0


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_wait_timeout_is_reported_and_the_context_stays_usable():
    lib = _lib.lib()
    assert tuple(_lib.status_read(clear=True)) == (0, 0, 0, 0)
    t0 = time.perf_counter()
    _lib.check("kdb_selftest_wait_timeout", lib.kdb_selftest_wait_timeout(1_000_000, _stream()))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, f"a 1 ms bounded wait took {elapsed:.3f} s to give up"
    st = _lib.status_read(clear=True)
    assert st[0] == _lib.KDB_ERR_TIMEOUT and st[1] == SITE_SELFTEST and st[3] == 1, st
    # the context is intact: a normal launch afterwards is correct and reports nothing
    x = W.proj_input(200, 512, 1)
    w = W.proj_weight(512, 300, 1)
    y = proj(x.cuda(), w.cuda())
    torch.cuda.synchronize()
    ok, msg = op.check(y.cpu(), op.proj_ref(x, w))
    assert ok, msg
    assert tuple(_lib.status_read(clear=True)) == (0, 0, 0, 0)


def test_wait_limit_outside_range_is_rejected():
    lib = _lib.lib()
    assert lib.kdb_selftest_wait_timeout(0, _stream()) == _lib.KDB_ERR_INVALID_ARG
    assert lib.kdb_selftest_wait_timeout(3_000_000_000, _stream()) == _lib.KDB_ERR_INVALID_ARG
