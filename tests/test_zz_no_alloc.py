"""The allocation-free matmul entry point (rcu_matmul_f32_static).

It exists for callers that cannot call cudaMalloc when they need a matmul, for example
because their device memory is owned by a pool (PyTorch's caching allocator, or an engine
that reserves HBM for weights and KV cache up front). It quantizes the activations into a
fixed scratch area compiled into the library instead of an allocated one. These tests call
it through the C ABI on two calls in a row and compare it with the allocating path
(rcu_acts_prepare + rcu_matmul: the same kernels, so bit for bit) and with the CPU oracle
within the matmul tolerance used everywhere else. They cover the largest advertised call
(8 tokens of 16384 values, in both activation formats), a K-quant weight of more than
8 MiB (the tensor-core batch-1 GEMV), and check that free device memory does not change
across calls. This file is collected last on purpose.
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


# (type, rows, k, tokens of the first and second call); Q4_K 4096 x 4096 is 9.4 MB (the
# tensor-core GEMV at one token), the 16384-value cases at 8 tokens fill the whole scratch
CASES = [(O.Q4_0, 300, 2048, (1, 3)), (O.Q4_K, 257, 4096, (1, 3)), (O.Q6_K, 64, 12288, (1, 3)),
         (O.Q8_0, 100, 16384, (1, 3)), (O.Q4_K, 4096, 4096, (1, 1)), (O.Q4_0, 96, 16384, (8, 8)),
         (O.Q8_0, 40, 16384, (8, 7)), (O.Q4_K, 80, 16384, (8, 8)), (O.Q6_K, 48, 16384, (8, 8))]


@pytest.mark.parametrize("t,rows,k,toks", CASES)
def test_static_matmul_matches_allocating_path_and_oracle(env, t, rows, k, toks):
    torch, rie, ctx = env
    rng = O.Rng(77 + t + k)
    wq = rng.weight(t, rows, k)
    w = rie.Weight.upload(ctx, rie.GgmlType(t), rows, k, wq)
    for call, n_tok in enumerate(toks):  # two calls in a row: the shared scratch is rewritten each time
        xh = rng.vec(n_tok * k, 1.0 + call).reshape(n_tok, k)
        x = torch.from_numpy(xh).cuda()
        got = torch.full((n_tok, rows), float("nan"), device="cuda")
        rie.matmul_f32_static(ctx, w, x, n_tok, got)
        acts = rie.QuantActs(ctx, n_tok, k)
        acts.prepare(x, n_tok, k, rie.formats_for([w]))
        want = torch.zeros((n_tok, rows), device="cuda")
        rie.matmul(ctx, acts, w, want)
        ctx.sync()
        g, a = got.cpu().numpy(), want.cpu().numpy()
        assert np.array_equal(g.view(np.uint32), a.view(np.uint32)), "static and allocating paths differ"
        ref = O.matmul_multi(xh, [(t, wq, k)], n_threads=8)[0]
        close(g, ref)
    assert ctx.device_error_bits() == 0


def test_static_matmul_allocates_nothing(env):
    torch, rie, ctx = env
    rng = O.Rng(9)
    rows, k = 4096, 4096
    w = rie.Weight.upload(ctx, rie.GgmlType.Q4_K, rows, k, rng.weight(O.Q4_K, rows, k))
    w0 = rie.Weight.upload(ctx, rie.GgmlType.Q4_0, 64, 16384, rng.weight(O.Q4_0, 64, 16384))
    x = torch.from_numpy(rng.vec(8 * 16384, 1.0).reshape(8, 16384)).cuda()
    x1 = x[0, :k].contiguous()
    out = torch.zeros((8, rows), device="cuda")
    rie.matmul_f32_static(ctx, w, x1, 1, out)  # first call: looks the scratch up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):  # second and third calls
        rie.matmul_f32_static(ctx, w, x1, 1, out)
        rie.matmul_f32_static(ctx, w0, x, 8, out, 4096)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
    assert ctx.device_error_bits() == 0


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
