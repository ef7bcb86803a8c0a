"""Failure detection on one GPU without a GPU fault.

Every wait on another CTA or rank is bounded (qwen_set_wait_timeout_ns); a
wait that runs out records an error code in the device error word and gives
up, the launch returns, and the context stays usable.  Each test makes one
such wait run out on purpose, with a signal that nothing sends:

* tensor-parallel exchange: a world-2 exchange table whose second rank's
  region is a local allocation nobody publishes into -> ERR_P2P_TIMEOUT (6);
* persistent step kernel: CTA 0 is told not to report one stage done
  (qwen_step_set_drop), so the next stage's grid-wide wait runs out ->
  the step is abandoned with ERR_STEP_TIMEOUT (8); after qwen_step_reset and
  a state reset the same tokens decode bit-identically to a clean run.

No kernel is made to fault, trap or spin without a bound.
"""

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
LIMIT_NS = 50_000_000  # 50 ms


@pytest.fixture(scope="module")
def lib():
    from qwen35_b200 import _lib
    return _lib.fused()


@pytest.fixture()
def short_waits(lib):
    from qwen35_b200 import _lib
    _lib.device_error()  # start clean
    _lib.check(lib.qwen_set_wait_timeout_ns(LIMIT_NS), "qwen_set_wait_timeout_ns")
    yield
    _lib.check(lib.qwen_set_wait_timeout_ns(0), "qwen_set_wait_timeout_ns")


def test_wait_limit_is_validated(lib):
    from qwen35_b200 import _lib
    assert lib.qwen_set_wait_timeout_ns(10) != 0           # below 1 ms
    assert lib.qwen_set_wait_timeout_ns(10 ** 12) != 0     # above the 2 s maximum
    assert lib.qwen_last_error() != 0                       # recorded; reading it clears it
    _lib.check(lib.qwen_set_wait_timeout_ns(0), "default")
    assert lib.qwen_last_error() == 0


def _region(lib, world, n):
    from qwen35_b200 import _lib
    base = P()
    handle = ctypes.create_string_buffer(64)
    _lib.check(lib.qwen_p2p_create(world, n, ctypes.byref(base), handle), "qwen_p2p_create")
    return base


def _table(lib, bases, rank, n):
    from qwen35_b200 import _lib
    arr = (P * len(bases))(*bases)
    t = P()
    _lib.check(lib.qwen_p2p_table(arr, len(bases), rank, n, ctypes.byref(t)), "qwen_p2p_table")
    return t


def test_p2p_peer_that_never_publishes_times_out(lib, short_waits):
    from qwen35_b200 import _lib
    n = 512
    own, silent = _region(lib, 2, n), _region(lib, 2, n)
    table = _table(lib, [own, silent], 0, n)
    res = torch.randn(n, device="cuda").to(torch.bfloat16)
    y = torch.empty_like(res)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(lib.qwen_resid_add_p2p(table, P(res.data_ptr()), P(y.data_ptr()), n, P(0)), "qwen_resid_add_p2p")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert _lib.device_error() == 6  # ERR_P2P_TIMEOUT
    assert LIMIT_NS * 1e-9 * 0.9 < dt < 1.5, dt
    # the context is usable: a one-rank exchange round right after is clean
    solo = _region(lib, 1, n)
    t1 = _table(lib, [solo], 0, n)
    _lib.check(lib.qwen_resid_add_p2p(t1, P(res.data_ptr()), P(y.data_ptr()), n, P(0)), "qwen_resid_add_p2p")
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(y, res)  # zero partials: y = bf16(res + 0)
    for t in (table, t1):
        lib.qwen_p2p_table_free(t)
    for b in (own, silent, solo):
        lib.qwen_p2p_destroy(b)


def test_step_kernel_stage_wait_times_out_and_recovers(lib, short_waits):
    from qwen35_b200 import _lib
    from qwen35_b200.config import qwen35_tiny
    from qwen35_b200.step import Qwen35StepEngine
    from qwen35_b200.weights import random_weights
    cfg = qwen35_tiny()
    w = random_weights(cfg, seed=5, device="cuda")
    eng = Qwen35StepEngine(cfg, w, max_seq=64, keep_logits=True)
    feed = [3, 17, 99, 5, 42, 7, 11, 250]
    clean = [eng.decode(t) for t in feed]
    clean_logits = eng.logits.clone()
    assert _lib.device_error() == 0
    eng.reset()
    eng.token.zero_()
    _lib.check(lib.qwen_step_set_drop(eng.prog, 2), "qwen_step_set_drop")
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        eng.decode(feed[0])
        dt = time.perf_counter() - t0
    finally:
        _lib.check(lib.qwen_step_set_drop(eng.prog, -1), "qwen_step_set_drop")
    assert _lib.device_error() == 8  # ERR_STEP_TIMEOUT: the step was abandoned
    assert LIMIT_NS * 1e-9 * 0.9 < dt < 1.5, dt
    # recovery: clear the program's counters and workspaces and the model state
    _lib.check(lib.qwen_step_reset(eng.prog, P(0)), "qwen_step_reset")
    eng.reset()
    eng.token.zero_()
    again = [eng.decode(t) for t in feed]
    assert _lib.device_error() == 0
    assert again == clean
    assert torch.equal(eng.logits, clean_logits)
    eng.close()
