"""Layer-by-layer (teacher-forced) parity of the device forward with the oracle forward, at the
benchmark configuration shapes (Qwen3-8B-shape Q4_K_M, config 3; Qwen3-30B-A3B-shape MoE,
config 4) and on the small synthetic presets of testing.rs.

End-to-end logits of two implementations of a quantized forward drift apart: an output that
differs in its last bits can move an int8 activation code of the next layer across a rounding
boundary, and through attention that reaches every later token. The reference therefore
compares two quantized forwards at 0.03 (tests/model.rs:302-364). Teacher forcing removes the
drift between layers, so every layer is checked on its own:
  * both sides get the oracle's residual rows at the entry of layer l (the GPU through
    rcu_backend_forward_layers), and the GPU's rows after layer l are compared with the oracle's
    rows after layer l, as is the layer's own contribution (rows after minus rows before),
    which the residual would otherwise hide; the head's logits from the oracle's final rows are
    compared with the oracle's logits;
  * the rows after each layer and the logits must agree within 1e-3 of their largest magnitude
    or twice the oracle's own spread when that is larger: the
    reference's two CPU tiers (AVX2: round half to even, 8-lane sums; scalar: round half away,
    sequential sums) run teacher-forced on the same rows, and a code flip inside a layer can
    move them apart (tiny Q8_0 models: 8e-3);
  * a layer's own contribution is smaller than its rows, so a code flip inside the layer (the
    GPU's f32 sums, exp and RMS run in a third order, and flip other codes than the CPU tiers)
    shows more in it: measured at the Qwen3-8B shape, layers agree within 1e-6 at one token and
    1e-4 at six, and a flipped code moves one token's contribution by up to 2.2e-3 of its largest
    value. Each contribution must therefore be within 5e-3 (or twice the tiers' spread), and the
    median over all layers and steps within 1e-4, which no flip can hide.
The prompt runs layer by layer this way, so each layer's KV cache on the GPU holds the keys and
values of the oracle's rows, and the decode steps after the prompt are teacher-forced too. The
plain forward (no teacher forcing) is also compared end to end at the reference's 0.03 with
greedy agreement.
"""
import numpy as np
import pytest

import oracle as O
from rust_interference_engine_b200 import GgmlType

pytestmark = pytest.mark.gpu
RTOL_LAYER = 1e-3
RTOL_CONTRIB = 5e-3     # one code flip inside a layer (measured up to 2.2e-3 at the Qwen3-8B shape)
RTOL_CONTRIB_MED = 1e-4  # median over layers and steps
RTOL_E2E = 0.03  # tests/model.rs:302-364

# Qwen3-8B shape, Q4_K_M mix (config 3) and Qwen3-30B-A3B shape (config 4)
QWEN3_8B = dict(arch="qwen3", n_vocab=151936, n_embd=4096, n_layer=36, n_head=32, n_head_kv=8, head_dim=128,
                n_ff=12288, rope_dim=128, rope_base=1_000_000.0, rms_eps=1e-6)
QWEN3_30B_A3B = dict(arch="qwen3moe", n_vocab=151936, n_embd=2048, n_layer=48, n_head=32, n_head_kv=4, head_dim=128,
                     n_ff=6144, rope_dim=128, rope_base=1_000_000.0, rms_eps=1e-6, n_expert=128, n_expert_used=8,
                     n_ff_exp=768, n_ff_shexp=0)


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.fixture(scope="module")
def env():
    import torch
    import rust_interference_engine_b200 as rie
    from rust_interference_engine_b200 import model as M
    return torch, rie, M, rie.Context(0, torch.cuda.current_stream())


def build_pair(env, spec, kv_type, n_ctx=32, max_batch=8, seed=1):
    torch, rie, M, ctx = env
    rng = O.Rng(seed)
    cfg = spec.config()
    gm = M.Model(ctx, cfg)
    om = O.OracleModel(O.ModelConfig.from_buffer_copy(bytes(cfg)))
    weight = lambda t, r, c: rng.weight(int(t), r, c)
    vec = lambda n, s: rng.vec(n, s)
    norm = lambda n: (1.0 + 0.1 * rng.vec(n, 1.0)).astype(np.float32)
    for name, t, rows, cols, data in M.synthetic_tensors(spec, weight, vec, norm):
        gm.set_tensor(name, int(t), rows, cols, data)
        om.set_tensor(name, int(t), rows, cols, data)
    ob = O.OracleBackend(om, n_ctx, max_batch, kv_type=kv_type, n_threads=16)
    return gm, om, ob


def teacher_forced(env, gm, om, ob, spec, kv_type, prompt, decode, n_ctx=32, max_batch=8):
    """Worst relative errors over all layers and steps: (rows, layer contribution, logits,
    largest rows bound used, median contribution error beyond the tiers' spread)."""
    torch, rie, M, ctx = env
    gb = M.CudaBackend(gm, n_ctx, max_batch, rie.KvType(kv_type))
    # the reference's scalar tier, teacher-forced on the AVX2 tier's rows
    os_ = O.OracleBackend(om, n_ctx, max_batch, kv_type=kv_type, n_threads=16, path=O.PATH_SCALAR)
    L = spec.n_layer
    ob.set_capture(True)
    os_.set_capture(True)
    worst = [0.0, 0.0, 0.0, RTOL_LAYER]
    contrib = []
    pos = 0
    for step, toks in enumerate([prompt] + [[t] for t in decode]):
        toks = np.asarray(toks, dtype=np.uint32)
        want_logits = ob.forward(toks, pos, all_logits=True)
        X = ob.layer_x()
        os_.set_teacher(X)
        s_logits = os_.forward(toks, pos, all_logits=True)
        S = os_.layer_x()
        for il in range(L):
            got, _ = gb.forward_layers(X[il], pos, il, il + 1)
            e_full, e_delta = rel(got, X[il + 1]), rel(got - X[il], X[il + 1] - X[il])
            s_full, s_delta = rel(S[il + 1], X[il + 1]), rel(S[il + 1] - X[il], X[il + 1] - X[il])
            b_full, b_delta = max(RTOL_LAYER, 2 * s_full), max(RTOL_CONTRIB, 2 * s_delta)
            worst = [max(worst[0], e_full), max(worst[1], e_delta), worst[2], max(worst[3], b_full)]
            contrib.append(max(0.0, e_delta - 2 * s_delta))
            assert e_full <= b_full, f"step {step} layer {il}: rows {e_full} (oracle tiers {s_full})"
            assert e_delta <= b_delta, f"step {step} layer {il}: layer contribution {e_delta} (oracle tiers {s_delta})"
        _, lg = gb.forward_layers(X[L], pos, L, L, logits=True)
        e, b = rel(lg, want_logits), max(RTOL_LAYER, 2 * rel(s_logits, want_logits))
        worst[2], worst[3] = max(worst[2], e), max(worst[3], b)
        assert e <= b, f"step {step}: head logits {e}"
        pos += len(toks)
    med = float(np.median(contrib))
    assert med <= RTOL_CONTRIB_MED, f"median layer-contribution error {med}"
    ob.set_capture(False)
    gb.free()
    return worst + [med]


def end_to_end(env, gm, om, spec, kv_type, prompt, decode, n_ctx=32, max_batch=8):
    torch, rie, M, ctx = env
    gb = M.CudaBackend(gm, n_ctx, max_batch, rie.KvType(kv_type))
    ob = O.OracleBackend(om, n_ctx, max_batch, kv_type=kv_type, n_threads=16)
    toks = np.asarray(prompt, dtype=np.uint32)
    g, o = gb.forward(toks, 0, all_logits=True), ob.forward(toks, 0, all_logits=True)
    errs = [rel(g, o)]
    pos = len(prompt)
    for t in decode:
        g, o = gb.forward(np.array([t], np.uint32), pos), ob.forward(np.array([t], np.uint32), pos)
        errs.append(rel(g, o))
        top2 = np.sort(o[0])[-2:]
        assert int(np.argmax(g[0])) == int(np.argmax(o[0])) or top2[1] - top2[0] <= RTOL_E2E * np.max(np.abs(o))
        pos += 1
    gb.free()
    assert max(errs) <= RTOL_E2E, errs
    return max(errs)


def tiny(arch, wtype, mix=False):
    from rust_interference_engine_b200 import model as M
    s = M.SyntheticSpec.tiny(arch, wtype)
    if mix:  # Q4_K_M-style: attn_v and ffn_down in Q6_K, embeddings Q6_K
        s.embd_type = GgmlType.Q6_K
        s.type_overrides = {"attn_v.weight": GgmlType.Q6_K, "ffn_down.weight": GgmlType.Q6_K}
    return s


TINY = [("qwen3", GgmlType.Q4_K, True, O.KV_F16), ("llama", GgmlType.Q4_0, False, O.KV_F16),
        ("qwen3", GgmlType.Q4_K, False, O.KV_TURBO4), ("qwen3", GgmlType.Q8_0, False, O.KV_Q8_0),
        ("qwen3moe", GgmlType.Q4_K, False, O.KV_F16), ("gemma2", GgmlType.Q4_K, False, O.KV_F16),
        ("phi3", GgmlType.Q4_0, False, O.KV_F16)]


@pytest.mark.parametrize("arch,wtype,mix,kv", TINY,
                         ids=["qwen3_q4km", "llama_q4_0", "qwen3_turbo4", "qwen3_q8kv", "qwen3moe", "gemma2", "phi3"])
def test_layerwise_tiny(env, arch, wtype, mix, kv):
    spec = tiny(arch, wtype, mix)
    gm, om, ob = build_pair(env, spec, kv)
    w = teacher_forced(env, gm, om, ob, spec, kv, [5, 17, 200, 3, 99, 42, 7], [11, 12, 13])
    print(arch, O.TYPE_NAMES[int(wtype)], "kv", kv, "worst (rows, contribution, logits, rows bound, median contribution):", w)


def test_layerwise_qwen3_8b_config3(env):
    """The Qwen3-8B-shape Q4_K_M model of benchmark configuration 3 (36 layers, vocabulary
    151936), weights as the reference's random_weight draws them."""
    from rust_interference_engine_b200 import model as M
    spec = M.SyntheticSpec(wtype=GgmlType.Q4_K, embd_type=GgmlType.Q6_K, qk_norm=True,
                           type_overrides={"attn_v.weight": GgmlType.Q6_K, "ffn_down.weight": GgmlType.Q6_K},
                           **QWEN3_8B)
    gm, om, ob = build_pair(env, spec, O.KV_F16, seed=3)
    w = teacher_forced(env, gm, om, ob, spec, O.KV_F16, [101, 2024, 77, 5, 150000, 42], [9, 31337])
    print("config 3 teacher-forced worst rel errors (rows, layer contribution, logits, rows bound, median contribution):", w)
    e = end_to_end(env, gm, om, spec, O.KV_F16, [101, 2024, 77, 5, 150000, 42], [9, 31337])
    print("config 3 end-to-end worst rel error:", e)


def test_layerwise_qwen3_moe_config4(env):
    """The Qwen3-30B-A3B-shape mixture of experts of benchmark configuration 4 (48 layers, 128
    experts, top-8 routing, 4 KV heads)."""
    from rust_interference_engine_b200 import model as M
    spec = M.SyntheticSpec(wtype=GgmlType.Q4_K, embd_type=GgmlType.Q4_K, qk_norm=True, **QWEN3_30B_A3B)
    gm, om, ob = build_pair(env, spec, O.KV_F16, seed=4)
    w = teacher_forced(env, gm, om, ob, spec, O.KV_F16, [3, 1000, 77, 12345, 8], [19, 151000])
    print("config 4 teacher-forced worst rel errors (rows, layer contribution, logits, rows bound, median contribution):", w)


@pytest.mark.parametrize("group", [4, 8])
@pytest.mark.parametrize("kv", [O.KV_F16, O.KV_Q8_0, O.KV_TURBO4], ids=["f16", "q8_0", "turbo4"])
def test_layerwise_decode_attention_hd128(env, kv, group):
    """head_dim 128 with 4 or 8 query heads per KV head over every cache type: the decode steps
    run the decode attention kernels with the q/k post-processing (q/k norm, RoPE, KV append)
    folded into them (turbo4 caches fold it at one or two KV heads, as here); the prompt uses the
    standalone kernels. All held to the layer bounds above."""
    from rust_interference_engine_b200 import model as M
    spec = M.SyntheticSpec(arch="qwen3", wtype=GgmlType.Q4_K, embd_type=GgmlType.Q8_0, qk_norm=True, n_vocab=512,
                           n_embd=1024, n_layer=2, n_head=8, n_head_kv=8 // group, head_dim=128, n_ff=2048,
                           rope_dim=128, rope_base=1_000_000.0, rms_eps=1e-6)
    gm, om, ob = build_pair(env, spec, kv, seed=40 + group)
    w = teacher_forced(env, gm, om, ob, spec, kv, [5, 17, 200, 3, 99, 42, 7], [11, 12, 13, 14])
    print("hd128 G", group, "kv", kv, "worst (rows, contribution, logits, rows bound, median contribution):", w)

