"""The device weight quantizer (rcu_quantize_weight) against the oracle's, byte for byte.

Q8_0 and Q4_0 follow the reference's weight quantizers (quant/mod.rs:262-307); the other block
types use this library's own rules, restated in the oracle. The rows mix N(0, 0.02) values
(the benchmark configurations' weights) with edge cases: an all-zero block, one outlier,
all-positive and all-negative rows, values at the f16 subnormal scale, and exact ties of the
rounding steps. A model whose tensors go in from device memory (rcu_model_set_tensor_device)
must give the same logits, bit for bit, as one loaded from host bytes.
"""
import numpy as np
import pytest

import oracle as O
from rust_interference_engine_b200 import GgmlType

pytestmark = pytest.mark.gpu
TYPES = [O.Q8_0, O.Q4_0, O.Q4_1, O.Q5_0, O.Q5_1, O.Q4_K, O.Q5_K, O.Q6_K]


@pytest.fixture(scope="module")
def env():
    import torch
    import rust_interference_engine_b200 as rie
    return torch, rie, rie.Context(0, torch.cuda.current_stream())


def rows_with_edges(rows, cols, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32)
    x[0, :] = 0.0                                  # zero blocks
    x[1, :] = np.abs(x[1, :])                      # all positive (K-quant mins of zero)
    x[2, :] = -np.abs(x[2, :])                     # all negative
    x[3, 7] = 3.0                                  # one outlier
    x[4, :] = rng.normal(0.0, 1e-6, cols)          # f16 subnormal scales
    x[5, :] = np.round(x[5, :] * 1000) / 1000      # many exact values
    x[6, :32] = np.linspace(-1, 1, 32, dtype=np.float32)  # rounding ties in Q4_0 / Q8_0 steps
    return x


@pytest.mark.parametrize("t", TYPES, ids=[O.TYPE_NAMES[t] for t in TYPES])
def test_quantize_weight_matches_oracle(env, t):
    torch, rie, ctx = env
    rows, cols = 37, 1024
    x = rows_with_edges(rows, cols, 11 + t)
    want = O.quantize_weight(t, x)
    out = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
    rie.quantize_weight(ctx, rie.GgmlType(t), rows, cols, torch.from_numpy(x).cuda(), out)
    ctx.sync()
    got = out.cpu().numpy().reshape(want.shape)
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{O.TYPE_NAMES[t]}: {len(bad)} bytes differ, first at {bad[:4].tolist()}"


@pytest.mark.parametrize("t", [O.Q4_0, O.Q6_K])
def test_quantize_weight_column_slice(env, t):
    """ld > cols: the quantized column slice equals the slice of the quantized matrix (whole
    blocks), as the row-parallel shards of tensor parallelism need."""
    torch, rie, ctx = env
    rows, cols = 9, 2048
    x = rows_with_edges(rows, cols, 5)
    half = cols // 2
    want = O.quantize_weight(t, x[:, half:])
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
    rie.quantize_weight(ctx, rie.GgmlType(t), rows, half, xd[:, half:].contiguous(), out)
    out2 = torch.zeros_like(out)
    rie.quantize_weight(ctx, rie.GgmlType(t), rows, half, int(xd.data_ptr()) + 4 * half, out2, ld=cols)
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), want.reshape(-1))
    assert np.array_equal(out2.cpu().numpy(), want.reshape(-1))


def test_quantize_weight_errors(env):
    torch, rie, ctx = env
    x = torch.zeros(4, 100, device="cuda")
    out = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(rie.RcuError, match="multiple of the block size"):
        rie.quantize_weight(ctx, rie.GgmlType.Q4_0, 4, 100, x, out)
    with pytest.raises(rie.RcuError, match="no quantizer"):
        rie.quantize_weight(ctx, rie.GgmlType.F32, 4, 96, x, out)


def test_model_from_device_bytes_matches_host_bytes(env):
    torch, rie, ctx = env
    from rust_interference_engine_b200 import model as M
    spec = M.SyntheticSpec.tiny("qwen3", GgmlType.Q4_K)
    spec.type_overrides = {"attn_v.weight": GgmlType.Q6_K, "ffn_down.weight": GgmlType.Q6_K}
    rng = O.Rng(21)
    tensors = list(M.synthetic_tensors(spec, lambda t, r, c: rng.weight(int(t), r, c), lambda n, s: rng.vec(n, s),
                                       lambda n: (1.0 + 0.1 * rng.vec(n, 1.0)).astype(np.float32)))
    cfg = spec.config()
    mh, md = M.Model(ctx, cfg), M.Model(ctx, cfg)
    for name, t, rows, cols, data in tensors:
        mh.set_tensor(name, int(t), rows, cols, data)
        dev = torch.from_numpy(np.ascontiguousarray(data).view(np.uint8).reshape(-1).copy()).cuda()
        md.set_tensor_device(name, int(t), rows, cols, dev)
        del dev  # the model keeps its own copy
    torch.cuda.synchronize()
    toks = np.array([5, 17, 200, 3], np.uint32)
    outs = []
    for m in (mh, md):
        be = M.CudaBackend(m, 16, 8, rie.KvType.F16)
        outs.append((be.forward(toks, 0, True), be.forward(np.array([9], np.uint32), 4)))
        be.free()
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
