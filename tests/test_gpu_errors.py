"""Bounded device waits end with an error status, not a hang.

Every device-side wait of the library gives up after a limit, records an error bit and lets the
kernel finish; the host reads the bits through rcu_sync / rcu_check_device (RCU_ERR_TIMEOUT).
The waits on other ranks (the fused tensor-parallel all-reduce) use the context's limit
(rcu_set_wait_limit_ms). rcu_diag_expire_peer_wait launches the fused all-reduce norm against
arrival counters no rank will raise: its wait must run out after the limit with the peer
timeout bit (0x10) reported, and the context must still compute afterwards. Nothing faults.
"""
import time

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    import rust_interference_engine_b200 as rie
    return torch, rie, rie.Context(0, torch.cuda.current_stream())


@pytest.mark.parametrize("limit_ms", [50, 300])
def test_peer_wait_expires_with_an_error_status(env, limit_ms):
    torch, rie, ctx = env
    from rust_interference_engine_b200 import _lib
    lib = _lib.load()
    ctx.set_wait_limit_ms(limit_ms)
    t0 = time.perf_counter()
    st = lib.rcu_diag_expire_peer_wait(ctx.ptr)
    el = time.perf_counter() - t0
    assert st == _lib.RCU_ERR_TIMEOUT
    assert "0x10" in lib.rcu_last_error(ctx.ptr).decode()
    assert limit_ms * 1e-3 * 0.9 <= el < limit_ms * 1e-3 + 5.0
    assert ctx.device_error_bits() == 0  # the bits were cleared when reported
    # the context still computes
    rng = O.Rng(3)
    w = rng.weight(O.Q4_K, 64, 1024)
    x = rng.vec(1024, 1.0).reshape(1, 1024)
    wd = rie.Weight.upload(ctx, rie.GgmlType.Q4_K, 64, 1024, w)
    acts = rie.QuantActs(ctx, 1, 1024)
    acts.prepare(torch.from_numpy(x).cuda(), 1, 1024, rie.ActFormat.Q8K)
    out = torch.zeros(64, device="cuda")
    rie.matmul(ctx, acts, wd, out)
    ctx.sync()
    want = O.matmul_multi(x, [(O.Q4_K, w, 1024)], n_threads=4)[0][0]
    got = out.cpu().numpy()
    assert np.max(np.abs(got - want)) <= 1e-3 * np.max(np.abs(want))
    ctx.set_wait_limit_ms(2000)


def test_wait_limit_bounds(env):
    torch, rie, ctx = env
    with pytest.raises(rie.RcuError, match="1..600000"):
        ctx.set_wait_limit_ms(0)
