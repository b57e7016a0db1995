"""GPU parity of the quantized matmul path against the CPU oracle (through the C ABI).

Contract (north star): Q8_0/Q8_K activation codes and scales bit-exact, per-block int32
dot sums bit-exact, f32 outputs within 1e-3 relative error (measured like the reference's
assert_close: |a - b| <= rtol * max|b|, tests/common/mod.rs:25-31).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
RTOL = 1e-3


@pytest.fixture(scope="module")
def env(gemv_ctx):
    return gemv_ctx


def close(a, b, rtol=RTOL):
    scale = max(float(np.max(np.abs(b))), 1e-6)
    err = float(np.max(np.abs(a - b)))
    assert err <= rtol * scale, f"max err {err} > {rtol} * {scale}"


def gpu_matmul(env, weights, x, rounding=None):
    """weights: list of (type, uint8 [rows, row_bytes], cols). Returns list of outputs."""
    torch, rie, ctx = env
    if rounding is not None:
        ctx.set_rounding(rounding)
    n_tok, k = x.shape
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    ws = [rie.Weight.upload(ctx, rie.GgmlType(t), w.shape[0], cols, w) for (t, w, cols) in weights]
    acts = rie.QuantActs(ctx, n_tok, k)
    acts.prepare(xd, n_tok, k, rie.formats_for(ws))
    outs = [torch.full((n_tok, w.rows), float("nan"), device="cuda") for w in ws]
    rie.matmul_multi(ctx, acts, [rie.MatmulJob(w, o, w.rows) for w, o in zip(ws, outs)])
    ctx.sync()
    if rounding is not None:
        ctx.set_rounding(rie.Rounding.NEAREST_EVEN)
    return [o.cpu().numpy() for o in outs], acts, ws


@pytest.mark.parametrize("rounding", [0, 1])
def test_q8_0_activation_codes_bit_exact(env, rounding):
    torch, rie, ctx = env
    rng = np.random.default_rng(10 + rounding)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :64] *= 1e-30
    x[2, 32:64] = np.arange(32, dtype=np.float32) - 16.0  # ties after scaling
    ctx.set_rounding(rounding)
    acts = rie.QuantActs(ctx, 5, 4096)
    acts.prepare(torch.from_numpy(x).cuda(), 5, 4096, rie.ActFormat.Q8_0)
    got = acts.export(rie.ActFormat.Q8_0).view(O.BLOCK_Q8_0)
    ctx.set_rounding(0)
    want = O.quantize_row_q8_0(x, O.PATH_AVX2 if rounding == 0 else O.PATH_SCALAR).reshape(-1)
    np.testing.assert_array_equal(got["qs"], want["qs"])
    np.testing.assert_array_equal(got["d"].view(np.uint32), want["d"].view(np.uint32))
    np.testing.assert_array_equal(got["s"].view(np.uint32), want["s"].view(np.uint32))


def test_q8_k_activation_codes_bit_exact(env):
    torch, rie, ctx = env
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4, 4096)).astype(np.float32) * 3
    x[0, :256] = 0.0
    x[1, 10], x[1, 20] = 5.0, -5.0  # equal magnitude: the first one wins
    acts = rie.QuantActs(ctx, 4, 4096)
    acts.prepare(torch.from_numpy(x).cuda(), 4, 4096, rie.ActFormat.Q8K)
    got = acts.export(rie.ActFormat.Q8K).view(O.BLOCK_Q8K)
    want = O.quantize_row_q8_k(x).reshape(-1)
    np.testing.assert_array_equal(got["qs"], want["qs"])
    np.testing.assert_array_equal(got["bsums"], want["bsums"])
    np.testing.assert_array_equal(got["d"].view(np.uint32), want["d"].view(np.uint32))


TYPES = [O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K]


@pytest.mark.parametrize("t", TYPES, ids=[O.TYPE_NAMES[t] for t in TYPES])
def test_block_sums_bit_exact(env, t):
    torch, rie, ctx = env
    rng = O.Rng(100 + t)
    k = 2048
    w = rng.weight(t, 4, k)
    x = rng.vec(3 * k, 2.0).reshape(3, k)
    _, acts, ws = gpu_matmul(env, [(t, w, k)], x)
    a = O.quantize_acts(t, x, O.PATH_AVX2)
    n = 2 * (k // 256) if t in (O.Q4_K, O.Q5_K) else k // O.block_size(t)
    for row in range(4):
        for tok in range(3):
            out = torch.zeros(n, dtype=torch.int32, device="cuda")
            rie.block_sums(ctx, acts, ws[0], row, tok, out)
            want = O.block_sums(t, w[row], a[tok], k)
            np.testing.assert_array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("t", TYPES, ids=[O.TYPE_NAMES[t] for t in TYPES])
@pytest.mark.parametrize("n_tok", [1, 2, 3, 4, 7, 8, 13])
def test_matmul_matches_oracle(env, t, n_tok):
    # tests/kernels.rs:144-185 shapes (200 rows x 512) and decode shapes
    rng = O.Rng(42 + t)
    for rows, k in ((200, 512), (333, 4096)):
        w = rng.weight(t, rows, k)
        x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
        got = gpu_matmul(env, [(t, w, k)], x)[0][0]
        want = O.matmul_multi(x, [(t, w, k)], n_threads=4)[0]
        close(got, want)


def test_matmul_multi_mixed_types(env):
    rng = O.Rng(7)
    k = 4096
    specs = [(O.Q4_K, 96), (O.Q6_K, 64), (O.Q8_0, 40), (O.Q4_0, 100), (O.Q5_K, 17)]
    weights = [(t, rng.weight(t, r, k), k) for t, r in specs]
    for n_tok in (1, 3):
        x = rng.vec(n_tok * k, 1.5).reshape(n_tok, k)
        got, _, _ = gpu_matmul(env, weights, x)
        want = O.matmul_multi(x, weights, n_threads=4)
        for g, w_ in zip(got, want):
            close(g, w_)


@pytest.mark.parametrize("t,k", [(O.Q6_K, 12288), (O.Q4_K, 12288), (O.Q6_K, 6144), (O.Q4_K, 6144), (O.Q8_0, 14336),
                                 (O.Q4_0, 768), (O.Q6_K, 768)])
def test_long_and_ragged_rows(env, t, k):
    # long rows are split over several warps (lane GEMV) or into several k slices per tile
    # (K-quant GEMV at one token: 16-row tiles x 3 slices at 12288, 32-row tiles x 3 slices at
    # 6144); 41 rows leave a ragged last tile; 768-wide Q6_K rows are not 16-byte multiples
    rng = O.Rng(3 + k)
    w = rng.weight(t, 41, k)
    for n_tok in (1, 2):
        x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
        got = gpu_matmul(env, [(t, w, k)], x)[0][0]
        want = O.matmul_multi(x, [(t, w, k)], n_threads=4)[0]
        close(got, want)


def test_config1_gemv_shape(env):
    # benchmark configuration 1: W 6144x2048 ~ N(0, 0.02) -> Q4_0 (quant/mod.rs:279-298), x ~ N(0, 1)
    rng = np.random.default_rng(1)
    wf = rng.normal(0.0, 0.02, (6144, 2048)).astype(np.float32)
    w = O.quantize_weight(O.Q4_0, wf)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    got = gpu_matmul(env, [(O.Q4_0, w, 2048)], x)[0][0]
    want = O.matmul_multi(x, [(O.Q4_0, w, 2048)], n_threads=8)[0]
    close(got, want)
    # and against float math on the dequantized operands
    ref = O.dequantize(O.Q4_0, w, 2048).astype(np.float64) @ O.dequantize_q8(O.quantize_row_q8_0(x))[0].astype(np.float64)
    close(got[0], ref.astype(np.float32))


def test_errors_are_reported(env):
    torch, rie, ctx = env
    rng = O.Rng(1)
    w = rie.Weight.upload(ctx, rie.GgmlType.Q4_0, 8, 512, rng.weight(O.Q4_0, 8, 512))
    acts = rie.QuantActs(ctx, 2, 1024)
    x = torch.zeros(2, 1024, device="cuda")
    acts.prepare(x, 2, 1024, rie.ActFormat.Q8_0)
    out = torch.zeros(2, 8, device="cuda")
    with pytest.raises(rie.RcuError, match="inner dimension"):
        rie.matmul(ctx, acts, w, out)
    with pytest.raises(rie.RcuError, match="empty batch"):
        acts.prepare(x, 0, 1024, rie.ActFormat.Q8_0)
    with pytest.raises(rie.RcuError, match="multiple of 256"):
        acts.prepare(x, 1, 992, rie.ActFormat.Q8K)
    with pytest.raises(rie.RcuError):
        rie.Weight.upload(ctx, rie.GgmlType.Q4_K, 2, 100, np.zeros(0, np.uint8))
    assert ctx.device_error_bits() == 0


@pytest.mark.parametrize("n_tok,rows,k", [(32, 200, 512), (64, 333, 4096), (100, 1000, 2048), (128, 256, 4096),
                                          (200, 130, 1024), (512, 4096, 4096)])
def test_prefill_gemm_q4_0(env, n_tok, rows, k):
    # tcgen05 int8 GEMM path (n_tok >= 32): ragged token and row tiles, several K
    rng = O.Rng(1000 + n_tok + rows)
    w = rng.weight(O.Q4_0, rows, k)
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    got = gpu_matmul(env, [(O.Q4_0, w, k)], x)[0][0]
    want = O.matmul_multi(x, [(O.Q4_0, w, k)], n_threads=8)[0]
    close(got, want)


ALL_TYPES = [O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K]


@pytest.mark.parametrize("t", ALL_TYPES, ids=[O.TYPE_NAMES[t] for t in ALL_TYPES])
@pytest.mark.parametrize("n_tok,rows,k", [(32, 200, 2048), (65, 333, 4096), (130, 1000, 2048), (300, 129, 4096)])
def test_prefill_gemm_f16_all_types(env, t, n_tok, rows, k):
    # f16 tensor-core GEMM (n_tok >= 32): ragged row and token tiles (64/128/192/256 tokens
    # per CTA), every weight type dequantized in shared memory
    rng = O.Rng(2000 + 7 * t + n_tok + rows)
    w = rng.weight(t, rows, k)
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    got = gpu_matmul(env, [(t, w, k)], x)[0][0]
    want = O.matmul_multi(x, [(t, w, k)], n_threads=8)[0]
    close(got, want)


def test_prefill_gemm_split_k_is_deterministic(env):
    # few row tiles: K is split over CTAs and the partial tiles are added in a fixed order by
    # the last CTA of each tile (counters reset for the next launch): repeated calls agree bit
    # for bit and with the oracle
    torch, rie, ctx = env
    rng = O.Rng(99)
    n_tok, rows, k = 96, 256, 8192
    w = rng.weight(O.Q4_K, rows, k)
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    outs = [gpu_matmul(env, [(O.Q4_K, w, k)], x)[0][0] for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    close(outs[0], O.matmul_multi(x, [(O.Q4_K, w, k)], n_threads=8)[0])


def test_prefill_gemm_f16_jobs_share_a_launch(env):
    # q/k/v-like jobs of one type share a launch; a second type and format follow
    rng = O.Rng(77)
    k, n_tok = 4096, 96
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    ws = [(O.Q4_K, rng.weight(O.Q4_K, r, k), k) for r in (512, 128, 128)]
    ws += [(O.Q6_K, rng.weight(O.Q6_K, 256, k), k), (O.Q8_0, rng.weight(O.Q8_0, 200, k), k)]
    got = gpu_matmul(env, ws, x)[0]
    want = O.matmul_multi(x, ws, n_threads=8)
    for g, wv in zip(got, want):
        close(g, wv)


@pytest.mark.parametrize("t", [O.Q4_0, O.Q4_K, O.Q6_K], ids=["Q4_0", "Q4_K", "Q6_K"])
def test_prefill_gemm_f16_large_activations(env, t):
    # rows whose values pass the f16 range (65504) are scaled by a power of two per token
    rng = O.Rng(4242 + t)
    n_tok, rows, k = 64, 300, 2048
    w = rng.weight(t, rows, k)
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    x *= np.array([10.0 ** (i % 8) for i in range(n_tok)], np.float32)[:, None]  # up to 1e7
    got = gpu_matmul(env, [(t, w, k)], x)[0][0]
    want = O.matmul_multi(x, [(t, w, k)], n_threads=8)[0]
    assert np.all(np.isfinite(got))
    for i in range(n_tok):  # every token row against its own scale
        close(got[i], want[i])


def gpu_matmul_i8(env, weights, x):
    """gpu_matmul through the int8 GEMM (exact per-block int32 sums, Q4_0 weights)."""
    torch, rie, ctx = env
    ctx.set_prefill_gemm(rie.PrefillGemm.I8)
    try:
        return gpu_matmul(env, weights, x)[0]
    finally:
        ctx.set_prefill_gemm(rie.PrefillGemm.F16)


@pytest.mark.parametrize("n_tok,rows,k", [(32, 200, 512), (128, 256, 4096), (64, 333, 4096), (100, 1000, 2048),
                                          (200, 130, 1024), (300, 129, 4096), (512, 4096, 4096)])
def test_prefill_gemm_q4_0_int8_kind(env, n_tok, rows, k):
    # the int8 GEMM (tcgen05 kind::i8, exact per-block sums): ragged token and row tiles, several K
    rng = O.Rng(3000 + n_tok + rows)
    w = rng.weight(O.Q4_0, rows, k)
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    got = gpu_matmul_i8(env, [(O.Q4_0, w, k)], x)[0]
    want = O.matmul_multi(x, [(O.Q4_0, w, k)], n_threads=8)[0]
    close(got, want)


def test_prefill_gemm_int8_jobs_share_a_launch(env):
    # up to four weights over the same activations run as one launch (five jobs: 4 + 1), each
    # with ragged rows; repeated calls agree bit for bit (one thread owns each output)
    rng = O.Rng(31)
    k, n_tok = 2048, 160
    x = rng.vec(n_tok * k, 1.0).reshape(n_tok, k)
    ws = [(O.Q4_0, rng.weight(O.Q4_0, r, k), k) for r in (512, 130, 128, 1, 300)]
    got = gpu_matmul_i8(env, ws, x)
    want = O.matmul_multi(x, ws, n_threads=8)
    for g, wv in zip(got, want):
        close(g, wv)
    again = gpu_matmul_i8(env, ws, x)
    assert all(np.array_equal(a, b) for a, b in zip(got, again))


def test_prefill_gemm_int8_config2(env):
    # benchmark configuration 2 through the int8 GEMM: M = 512 tokens x K = 4096 against the
    # N = 14336 and N = 4096 weights (W ~ N(0, 0.02) -> Q4_0) in one launch
    rng = np.random.default_rng(2)
    x = rng.standard_normal((512, 4096)).astype(np.float32)
    ws = [(O.Q4_0, O.quantize_weight(O.Q4_0, rng.normal(0.0, 0.02, (n, 4096)).astype(np.float32)), 4096)
          for n in (14336, 4096)]
    got = gpu_matmul_i8(env, ws, x)
    want = O.matmul_multi(x, ws, n_threads=8)
    for g, wv in zip(got, want):
        close(g, wv)


def test_prefill_gemm_config2(env):
    # benchmark configuration 2: M = 512 tokens x K = 4096, N = 4096 and 14336, W ~ N(0, 0.02) -> Q4_0
    rng = np.random.default_rng(2)
    x = rng.standard_normal((512, 4096)).astype(np.float32)
    for n in (4096, 14336):
        w = O.quantize_weight(O.Q4_0, rng.normal(0.0, 0.02, (n, 4096)).astype(np.float32))
        got = gpu_matmul(env, [(O.Q4_0, w, 4096)], x)[0][0]
        want = O.matmul_multi(x, [(O.Q4_0, w, 4096)], n_threads=8)[0]
        close(got, want)
