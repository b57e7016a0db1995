"""The allocation-free matmul entry point (rcu_matmul_f32_static).

It exists for callers that cannot call cudaMalloc when they need a matmul, for example
because their device memory is owned by a pool (PyTorch's caching allocator, or an engine
that reserves HBM for weights and KV cache up front). It quantizes the activations into a
fixed scratch area compiled into the library instead of an allocated one. These tests call
it through the C ABI and compare it with the allocating path (rcu_acts_prepare +
rcu_matmul) on two calls in a row, within the matmul tolerance used everywhere else.
This file is collected last on purpose.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
RTOL = 1e-3


@pytest.fixture(scope="module")
def env():
    import torch
    import rust_interference_engine_b200 as rie
    return torch, rie, rie.Context(0, torch.cuda.current_stream())


def close(a, b):
    scale = max(float(np.max(np.abs(b))), 1e-6)
    assert float(np.max(np.abs(a - b))) <= RTOL * scale


@pytest.mark.parametrize("t,rows,k", [(O.Q4_0, 300, 2048), (O.Q4_K, 257, 4096), (O.Q6_K, 64, 12288),
                                      (O.Q8_0, 100, 16384)])
def test_static_matmul_matches_allocating_path(env, t, rows, k):
    torch, rie, ctx = env
    rng = O.Rng(77 + t)
    w = rie.Weight.upload(ctx, rie.GgmlType(t), rows, k, rng.weight(t, rows, k))
    for call in range(2):  # two calls in a row: the shared scratch is rewritten each time
        n_tok = 1 if call == 0 else 3
        x = torch.from_numpy(rng.vec(n_tok * k, 1.0 + call).reshape(n_tok, k)).cuda()
        got = torch.full((n_tok, rows), float("nan"), device="cuda")
        rie.matmul_f32_static(ctx, w, x, n_tok, got)
        acts = rie.QuantActs(ctx, n_tok, k)
        acts.prepare(x, n_tok, k, rie.formats_for([w]))
        want = torch.zeros((n_tok, rows), device="cuda")
        rie.matmul(ctx, acts, w, want)
        ctx.sync()
        close(got.cpu().numpy(), want.cpu().numpy())


def test_static_matmul_limits(env):
    torch, rie, ctx = env
    rng = O.Rng(5)
    w = rie.Weight.upload(ctx, rie.GgmlType.Q4_0, 8, 32768, rng.weight(O.Q4_0, 8, 32768))
    x = torch.zeros((9, 32768), device="cuda")
    out = torch.zeros((9, 8), device="cuda")
    with pytest.raises(rie.RcuError, match="at most 8 tokens"):
        rie.matmul_f32_static(ctx, w, x, 9, out)
    with pytest.raises(rie.RcuError, match="longer than 16384"):
        rie.matmul_f32_static(ctx, w, x, 1, out)
    assert ctx.device_error_bits() == 0
