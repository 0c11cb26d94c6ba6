"""Bounded device waits: an expired wait is reported to the host as QW_ERR_TIMEOUT /
TimeoutError, the context stays usable, and nothing faults or hangs (GPU).

The expiry is made on purpose through the library's test hook
(qw_debug_inject_wait_timeout): the cluster linear kernels announce more bytes on each
weight stage's barrier than they copy, so no stage completes and every wait runs out
after a short limit; the kernels then record the expiry, wait (bounded) for their
copies in flight and return."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LIMIT = 200_000     # cycles, about 0.1 ms per wait


def _linear_case():
    from qwen35_dflash_b200 import w4
    torch.manual_seed(7)
    n, k, g, t = 2048, 2048, 128, 16
    q = torch.randint(-8, 8, (n, k), dtype=torch.int8, device="cuda")
    scale = (torch.rand(n, k // g, device="cuda") * 0.015 + 0.005).to(torch.bfloat16)
    x = torch.randn(t, k, device="cuda").to(torch.bfloat16)
    return w4.pack_w4(q, scale, g), x, n, k, g, t


def _run(stream, x, n, k, g, t):
    from qwen35_dflash_b200 import lib
    y = torch.full((t, n), 7.0, dtype=torch.float32, device="cuda")
    lib.call("qw_w4_linear", x.data_ptr(), stream.data_ptr(), y.data_ptr(), lib.QW_OUT_F32, n, t, n, k, g,
             lib.stream_ptr())
    return y


def test_expired_wait_is_reported_and_cleared(cuda_lib):
    from qwen35_dflash_b200 import lib
    st = lib.stream_ptr()
    stream, x, n, k, g, t = _linear_case()
    lib.call("qw_check_wait_status", 1, st)            # start from a clean word
    ref = _run(stream, x, n, k, g, t)
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    lib.call("qw_wait_status", status.data_ptr(), 0, st)
    assert int(status.item()) == lib.QW_OK
    lib.call("qw_debug_inject_wait_timeout", LIMIT, 16)
    try:
        _run(stream, x, n, k, g, t)
        lib.call("qw_wait_status", status.data_ptr(), 0, st)    # stream-ordered report, kept
        assert int(status.item()) == lib.QW_ERR_TIMEOUT
        with pytest.raises(TimeoutError, match="cluster linear"):
            lib.call("qw_check_wait_status", 1, st)               # synchronous report, cleared
    finally:
        lib.call("qw_debug_inject_wait_timeout", 0, 0)
    lib.call("qw_check_wait_status", 1, st)                       # cleared: QW_OK again
    again = _run(stream, x, n, k, g, t)                           # the context is still usable
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def test_session_raises_timeout_error(cuda_lib):
    """TargetSession.verify raises TimeoutError (no retry, no fallback) when a wait of the
    block's kernels expired, and verifies normally once the cause is gone."""
    from qwen35_dflash_b200 import config, engine, lib, synthetic
    from qwen35_dflash_b200.session import TargetSession
    cfg = config.TINY
    raw = synthetic.init_weights(cfg, seed=3)
    eng = engine.TargetEngine(cfg, engine.weights_from_arrays(cfg, raw), batch=1, block=16, capacity=128)
    sess = TargetSession(eng)
    sess.prefill([int(v) for v in np.random.default_rng(3).integers(0, cfg.vocab_size, 16)])
    props = [sess.next_token, 1, 2, 3]
    want = sess.verify(props).expected_next_tokens
    lib.call("qw_debug_inject_wait_timeout", LIMIT, 16)
    try:
        with pytest.raises(TimeoutError):
            sess.verify(props)
    finally:
        lib.call("qw_debug_inject_wait_timeout", 0, 0)
    assert sess.verify(props).expected_next_tokens == want
