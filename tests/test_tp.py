"""Tensor-parallel sharding (host side, no GPU): rcu_tp_shard keeps, for each rank, the part
of every GGUF tensor its GPU needs. Column-parallel tensors (q/k/v by head, gate/up rows,
the output head's vocabulary rows, q/k/v biases) must reassemble by concatenating the rank
shards; row-parallel ones (attn_output, ffn_down) by concatenating every row's column
blocks; and the partial matmuls of a column split must add up to the full matmul (the
all-reduce of the backend). The multi-process path runs as two gloo ranks on the CPU.
"""
import os

import numpy as np
import pytest

import oracle as O
from rust_interference_engine_b200 import GgmlType
from rust_interference_engine_b200 import model as M

ROWS = (".attn_q.weight", ".attn_k.weight", ".attn_v.weight", ".ffn_gate.weight", ".attn_q.bias", ".attn_k.bias",
        ".attn_v.bias")
COLS = (".attn_output.weight", ".ffn_down.weight")
EXPERTS = (".ffn_gate_exps.weight", ".ffn_up_exps.weight", ".ffn_down_exps.weight")


def tp_spec(arch, wtype):
    s = M.SyntheticSpec.tiny(arch, wtype)
    s.n_head, s.n_head_kv, s.head_dim, s.rope_dim = 8, 4, 64, 64  # q dim 512: whole 256-blocks per rank at TP 2
    s.n_embd, s.n_ff = 512, 1024
    return s


def tensors(spec, seed=3):
    rng = O.Rng(seed)
    weight = lambda t, r, c: rng.weight(int(t), r, c)
    vec = lambda n, s: rng.vec(n, s)
    norm = lambda n: (1.0 + 0.1 * rng.vec(n, 1.0)).astype(np.float32)
    return list(M.synthetic_tensors(spec, weight, vec, norm))


def raw(data):
    return np.ascontiguousarray(data).view(np.uint8).reshape(-1)


@pytest.mark.parametrize("arch,wtype,world", [("qwen3", GgmlType.Q4_K, 2), ("qwen2", GgmlType.Q8_0, 2),
                                              ("phi3", GgmlType.Q4_0, 2), ("llama", GgmlType.Q4_0, 4),
                                              ("qwen3moe", GgmlType.Q4_K, 2), ("qwen2moe", GgmlType.Q8_0, 4)])
def test_shards_reassemble(arch, wtype, world):
    spec = tp_spec(arch, wtype)
    cfg = spec.config()
    qd, kvd = spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim
    for name, t, rows, cols, data in tensors(spec):
        full = raw(data)
        parts = [M.tp_shard(cfg, name, t, rows, cols, data, r, world) for r in range(world)]
        if name.endswith(EXPERTS):  # expert parallelism: whole experts, rank by rank
            rb = full.size // rows
            assert all(p[1] == rows // world for p in parts), name
            assert np.array_equal(np.concatenate([p[0] for p in parts]), full), name
        elif name.endswith(ROWS) or name == "output.weight" or (name.endswith("ffn_up.weight") and rows == spec.n_ff):
            total = spec.n_vocab if name == "output.weight" else rows
            rb = full.size // rows
            assert all(p[1] == (total // world if rows > 1 else 1) for p in parts), name
            assert np.array_equal(np.concatenate([p[0] for p in parts]), full[: total * rb] if rows > 1 else full), name
        elif name.endswith("attn_qkv.weight"):
            rb = full.size // rows
            q = np.concatenate([p[0][: qd // world * rb] for p in parts])
            k = np.concatenate([p[0][qd // world * rb: (qd + kvd) // world * rb] for p in parts])
            v = np.concatenate([p[0][(qd + kvd) // world * rb:] for p in parts])
            assert np.array_equal(np.concatenate([q, k, v]), full), name
        elif name.endswith("ffn_up.weight"):  # fused gate+up halves
            rb = full.size // rows
            h = spec.n_ff // world * rb
            gate = np.concatenate([p[0][:h] for p in parts])
            up = np.concatenate([p[0][h:] for p in parts])
            assert np.array_equal(np.concatenate([gate, up]), full), name
        elif name.endswith(COLS):
            rb = full.size // rows
            assert all(p[2] == cols // world and p[1] == rows for p in parts), name
            re = np.concatenate([p[0].reshape(rows, -1) for p in parts], axis=1)
            assert np.array_equal(re.reshape(-1), full[: rows * rb]), name
        else:
            assert all(np.array_equal(p[0], full) for p in parts), name


@pytest.mark.parametrize("arch,wtype", [("qwen2", GgmlType.Q8_0), ("phi3", GgmlType.Q8_0), ("qwen3moe", GgmlType.Q8_0)])
def test_kv_heads_replicated_when_fewer_than_ranks(arch, wtype):
    """2 KV heads over 4 ranks: ranks 0-1 keep KV head 0 and ranks 2-3 KV head 1 (k / v rows,
    biases, the k / v part of a fused q/k/v tensor); query heads still split four ways, and they
    are the heads of the rank's KV group (8 query heads, 4 per KV head, 2 per rank)."""
    spec = tp_spec(arch, wtype)
    spec.n_head_kv = 2
    cfg = spec.config()
    world, hd = 4, spec.head_dim
    qd, kvd = spec.n_head * hd, spec.n_head_kv * hd
    rep = world // spec.n_head_kv
    seen = set()
    for name, t, rows, cols, data in tensors(spec):
        full = raw(data)
        rb = full.size // rows
        parts = [M.tp_shard(cfg, name, t, rows, cols, data, r, world) for r in range(world)]
        kv = name.endswith((".attn_k.weight", ".attn_v.weight", ".attn_k.bias", ".attn_v.bias"))
        if kv:
            seen.add(name.split(".", 2)[2])
            es = full.size // (cols if rows == 1 else rows)  # bytes per row (or per bias element)
            for r, p in enumerate(parts):
                h = r // rep
                assert (p[2] if rows == 1 else p[1]) == hd, name
                assert np.array_equal(p[0], full[h * hd * es:(h + 1) * hd * es]), (name, r)
        elif name.endswith("attn_qkv.weight"):
            seen.add("attn_qkv.weight")
            nq = qd // world
            for r, p in enumerate(parts):
                h = r // rep
                assert p[1] == nq + 2 * hd, name
                assert np.array_equal(p[0][: nq * rb], full[r * nq * rb:(r + 1) * nq * rb]), name
                assert np.array_equal(p[0][nq * rb:(nq + hd) * rb], full[(qd + h * hd) * rb:(qd + (h + 1) * hd) * rb]), name
                k0 = qd + kvd + h * hd
                assert np.array_equal(p[0][(nq + hd) * rb:], full[k0 * rb:(k0 + hd) * rb]), name
        elif name.endswith(".attn_q.weight"):
            assert all(p[1] == qd // world for p in parts), name
    assert seen, "no k / v tensors in the spec"


def test_kv_heads_that_do_not_split_are_an_error():
    spec = tp_spec("qwen2", GgmlType.Q8_0)
    spec.n_head, spec.n_head_kv = 12, 3  # 3 KV heads over 4 ranks: neither divides the other
    cfg = spec.config()
    w = O.Rng(2).weight(int(GgmlType.Q8_0), 3 * spec.head_dim, spec.n_embd)
    with pytest.raises(RuntimeError):
        M.tp_shard(cfg, "blk.0.attn_k.weight", GgmlType.Q8_0, 3 * spec.head_dim, spec.n_embd, w, 0, 4)


@pytest.mark.parametrize("wtype", [GgmlType.Q4_0, GgmlType.Q4_K, GgmlType.Q6_K])
def test_row_parallel_partials_add_up(wtype):
    """Splitting K at block boundaries keeps every activation block: the ranks' partial
    matmuls (oracle) sum to the full one up to f32 summation order."""
    spec = tp_spec("llama", wtype)
    cfg = spec.config()
    rng = O.Rng(11)
    rows, cols, world = 64, spec.n_ff, 2
    w = rng.weight(int(wtype), rows, cols)
    x = np.random.default_rng(5).standard_normal((3, cols)).astype(np.float32)
    full = O.matmul_multi(x, [(int(wtype), w.reshape(rows, -1), cols)], n_threads=4)[0]
    acc = np.zeros_like(full)
    for r in range(world):
        part, pr, pc = M.tp_shard(cfg, "blk.0.ffn_down.weight", wtype, rows, cols, w, r, world)
        xs = x[:, r * pc:(r + 1) * pc]
        acc += O.matmul_multi(xs, [(int(wtype), part.reshape(pr, -1), pc)], n_threads=4)[0]
    scale = float(np.max(np.abs(full)))
    assert float(np.max(np.abs(acc - full))) <= 1e-5 * scale


def test_bad_split_is_an_error():
    spec = tp_spec("qwen3", GgmlType.Q4_K)
    cfg = spec.config()
    w = O.Rng(1).weight(int(GgmlType.Q4_K), 8, 512)
    with pytest.raises(RuntimeError):  # 512 / 4 = 128 values: not whole 256-value blocks
        M.tp_shard(cfg, "blk.0.attn_output.weight", GgmlType.Q4_K, 8, 512, w, 0, 4)


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = tp_spec("qwen3", GgmlType.Q4_K)
        cfg = spec.config()
        ok = True
        for name, t, rows, cols, data in tensors(spec):
            mine = M.tp_shard(cfg, name, t, rows, cols, data, rank, world)
            got = [None] * world
            dist.all_gather_object(got, (mine[0].tobytes(), mine[1], mine[2]))
            if rank == 0 and name.endswith(COLS):
                re = np.concatenate([np.frombuffer(g[0], np.uint8).reshape(g[1], -1) for g in got], axis=1)
                ok &= np.array_equal(re.reshape(-1), raw(data))
            elif rank == 0 and name.endswith(("attn_q.weight", "ffn_gate.weight")):
                ok &= np.array_equal(np.concatenate([np.frombuffer(g[0], np.uint8) for g in got]), raw(data))
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_model():
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
