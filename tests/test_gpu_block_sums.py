"""The hot-path GEMVs' own per-block integer sums, bit for bit against the oracle.

rcu_matmul_block_sums runs the batch-1 matmul on the kernel it is given -- the lane GEMV
(k_gemv) or the tensor-core GEMV (k_gemv_kq, mma.m16n8k32 fragments) -- and captures every
exact int32 block sum that kernel forms on the way to its f32 outputs: per 32-value block for
Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 (quant/reference.rs:221-290), (sumi, summ) per superblock for
Q4_K / Q5_K and sumi per superblock for Q6_K (quant/reference.rs:295-386). Each must equal the
oracle's block_sums exactly, on the benchmark configurations' weight shapes (config 1: 6144 x
2048 Q4_0 from N(0, 0.02) weights; config 3: the Q4_K gate/up and Q6_K down of Qwen3-8B; config
5: the Q4_0 gate of Llama-3.1-70B) and on every block type; the f32 outputs of the same launch
stay within the matmul tests' 1e-3.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
TYPES = [O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K]
TC_TYPES = [O.Q4_0, O.Q4_K, O.Q5_K, O.Q6_K]


@pytest.fixture(scope="module")
def env():
    import torch
    import rust_interference_engine_b200 as rie
    return torch, rie, rie.Context(0, torch.cuda.current_stream())


def per_row(t, k):
    if t in (O.Q4_K, O.Q5_K):
        return 2 * (k // 256)
    return k // O.block_size(t)


def check(env, t, w, x, kernel, rows_checked=None):
    torch, rie, ctx = env
    rows, k = w.shape[0], x.shape[1]
    wd = rie.Weight.upload(ctx, rie.GgmlType(t), rows, k, w)
    acts = rie.QuantActs(ctx, 1, k)
    acts.prepare(torch.from_numpy(x).cuda(), 1, k, rie.formats_for([wd]))
    n = per_row(t, k)
    out = torch.full((rows,), float("nan"), device="cuda")
    sums = torch.full((rows * n,), -7, dtype=torch.int32, device="cuda")
    rie.matmul_block_sums(ctx, acts, wd, out, sums, kernel)
    ctx.sync()
    got = sums.cpu().numpy().reshape(rows, n)
    a = O.quantize_acts(t, x, O.PATH_AVX2)[0]
    for r in (range(rows) if rows_checked is None else rows_checked):
        want = O.block_sums(t, w[r], a, k)
        if not np.array_equal(got[r], want):
            bad = np.nonzero(got[r] != want)[0]
            raise AssertionError(f"{O.TYPE_NAMES[t]} kernel {kernel} row {r}: {len(bad)} sums differ, first at "
                                 f"{bad[:4].tolist()}: {got[r][bad[:4]].tolist()} vs {want[bad[:4]].tolist()}")
    y = out.cpu().numpy()
    ref = O.matmul_multi(x, [(t, w, k)], n_threads=16)[0][0]
    assert np.max(np.abs(y - ref)) <= 1e-3 * max(float(np.max(np.abs(ref))), 1e-6)


@pytest.mark.parametrize("t", TYPES, ids=[O.TYPE_NAMES[t] for t in TYPES])
def test_lane_gemv_block_sums(env, t):
    rng = O.Rng(300 + t)
    for rows, k in ((200, 512), (97, 4096)):
        check(env, t, rng.weight(t, rows, k), rng.vec(k, 1.5).reshape(1, k), 0)


@pytest.mark.parametrize("t", TC_TYPES, ids=[O.TYPE_NAMES[t] for t in TC_TYPES])
def test_tensor_core_gemv_block_sums(env, t):
    rng = O.Rng(400 + t)
    # ragged 16-row blocks, long rows (Q6_K rows are tileable from 8 superblocks: 2048 values)
    for rows, k in ((200, 2048 if t == O.Q6_K else 512), (97, 4096), (37, 12288)):
        check(env, t, rng.weight(t, rows, k), rng.vec(k, 1.5).reshape(1, k), 1)


@pytest.mark.parametrize("kernel", [0, 1], ids=["lane", "tensor_core"])
def test_config1_q4_0_block_sums(env, kernel):
    """Configuration 1: 6144 x 2048 Q4_0 weights quantized from N(0, 0.02), x ~ N(0, 1)."""
    rng = np.random.default_rng(2024)
    wf = rng.normal(0.0, 0.02, (6144, 2048)).astype(np.float32)
    w = O.quantize_weight(O.Q4_0, wf)
    x = rng.standard_normal((1, 2048)).astype(np.float32)
    check(env, O.Q4_0, w, x, kernel)


@pytest.mark.parametrize("kernel", [0, 1], ids=["lane", "tensor_core"])
@pytest.mark.parametrize("shape", [("Q4_K", 12288, 4096), ("Q6_K", 4096, 12288), ("Q4_0", 28672, 8192)],
                         ids=["config3_gate_q4_k", "config3_down_q6_k", "config5_gate_q4_0"])
def test_config_shapes_block_sums(env, kernel, shape):
    """Configurations 3 and 5: the decode GEMVs' weight shapes, every row's sums checked
    (config 5: a sample of 2048 rows spread over the 28672)."""
    name, rows, k = shape
    t = getattr(O, name)
    rng = O.Rng(500 + t + kernel)
    w = rng.weight(t, rows, k)
    x = rng.vec(k, 1.0).reshape(1, k)
    sample = None if rows <= 12288 else list(range(0, rows, 14))
    check(env, t, w, x, kernel, sample)


def test_block_sum_capture_errors(env):
    torch, rie, ctx = env
    rng = O.Rng(9)
    w = rng.weight(O.Q8_0, 4, 256)
    wd = rie.Weight.upload(ctx, rie.GgmlType.Q8_0, 4, 256, w)
    acts = rie.QuantActs(ctx, 1, 256)
    acts.prepare(torch.from_numpy(rng.vec(256, 1.0).reshape(1, 256)).cuda(), 1, 256, rie.formats_for([wd]))
    out = torch.zeros(4, device="cuda")
    sums = torch.zeros(4 * 8, dtype=torch.int32, device="cuda")
    with pytest.raises(rie.RcuError, match="tensor-core GEMV takes"):
        rie.matmul_block_sums(ctx, acts, wd, out, sums, 1)
    with pytest.raises(rie.RcuError, match="kernel: 0"):
        rie.matmul_block_sums(ctx, acts, wd, out, sums, 2)
