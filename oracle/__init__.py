"""TEST INFRASTRUCTURE ONLY: ctypes/numpy front end of the CPU oracle (liboracle.so).

The oracle restates the Rust Inference Engine's CPU path (quant formats, scalar and AVX2
dot kernels, matmul driver, turbo4 KV cache, attention); see rie_oracle.cpp for the
reference file:line each piece follows. Only tests/, __graft_entry__.smoke() and the CPU
baseline legs of bench.py may import this package: the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

# ggml type ids (crates/rie-core/src/quant/mod.rs:34-51)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 30
TYPE_NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
ALL_TYPES = [F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K]
QUANT_TYPES = [Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q5_K, Q6_K]
PATH_SCALAR, PATH_AVX2 = 0, 1
KV_F16, KV_Q8_0, KV_TURBO4 = 0, 1, 2

# Activation blocks, repr(C, align(16)) (quant/mod.rs:139-168)
BLOCK_Q8_0 = np.dtype({"names": ["qs", "d", "s"], "formats": [("i1", 32), "<f4", "<f4"],
                       "offsets": [0, 32, 36], "itemsize": 48})
BLOCK_Q8K = np.dtype({"names": ["qs", "bsums", "d"], "formats": [("i1", 256), ("<i2", 16), "<f4"],
                      "offsets": [0, 256, 288], "itemsize": 304})


def build(force: bool = False) -> str:
    srcs = [os.path.join(_HERE, f) for f in ("rie_oracle.cpp", "rie_oracle_model.cpp", "rie_oracle.h")]
    if force or not os.path.exists(_LIB_PATH) or any(os.path.getmtime(_LIB_PATH) < os.path.getmtime(s) for s in srcs):
        subprocess.run(["make", "-C", _HERE, "-B" if force else "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        _declare(_lib)
    return _lib


def _declare(L):
    P, S, I, U64, F = C.c_void_p, C.c_size_t, C.c_int, C.c_uint64, C.c_float
    sig = {
        "orc_have_avx2": (I, []),
        "orc_block_size": (S, [I]), "orc_block_bytes": (S, [I]), "orc_row_bytes": (S, [I, S]),
        "orc_sizeof_block_q8_0": (S, []), "orc_sizeof_block_q8_k": (S, []),
        "orc_f32_to_f16": (C.c_uint16, [F]), "orc_f16_to_f32": (F, [C.c_uint16]),
        "orc_f32_to_f16_n": (None, [P, P, S, I]),
        "orc_rng_new": (U64, [U64]), "orc_rng_next": (U64, [P]), "orc_rng_vec": (None, [P, P, S, F]),
        "orc_random_weight": (I, [P, I, S, S, F, P]),
        "orc_quantize_row_q8_0": (None, [P, S, P, I]), "orc_quantize_row_q8_k": (None, [P, S, P]),
        "orc_quantize_weight": (S, [I, P, S, P]), "orc_dequantize_row": (I, [I, P, P, S]),
        "orc_vec_dot": (F, [I, P, P, S, I]), "orc_block_sums": (S, [I, P, P, S, P]),
        "orc_matmul_multi": (None, [I, P, S, S, P, S, I]),
        "orc_matmul_multi_q": (None, [I, P, P, P, S, S, P, S, I]),
        "orc_kv_seed": (U64, []), "orc_turbo_sign": (F, [U64, S]), "orc_turbo_block_size": (S, [S]),
        "orc_turbo_row_bytes_4": (S, [S]), "orc_turbo_rotate": (None, [U64, P, S, I]),
        "orc_turbo_fwht": (None, [P, S]), "orc_turbo_quantize_4": (None, [U64, P, S, P]),
        "orc_turbo_quantize_rotated_4": (None, [P, S, P]),
        "orc_turbo_dot_rotated_4": (F, [P, P, S, I]), "orc_turbo_axpy_rotated_4": (None, [P, F, P, S, I]),
        "orc_turbo_dequantize_4": (None, [U64, P, P, S]), "orc_turbo_codebook": (None, [I, P]),
        "orc_turbo_kv_levels": (None, [P]),
        "orc_attention": (None, [I, S, S, S, S, S, S, F, P, I, P, P, S, P, I]),
        "orc_kv_store": (None, [I, P, S, P, I]),
        "orc_rmsnorm": (None, [P, P, P, S, F, I]), "orc_rope_table": (None, [S, F, F, S, P, P]),
        "orc_rope_apply": (None, [P, S, I, P, P]), "orc_silu": (F, [F]), "orc_dot_f32": (F, [P, P, S, I]),
        "orc_model_create": (P, [P]), "orc_model_free": (None, [P]),
        "orc_model_set_tensor": (I, [P, C.c_char_p, I, U64, U64, P]),
        "orc_backend_create": (P, [P, U64, U64, I, I, I]), "orc_backend_free": (None, [P]),
        "orc_backend_forward": (I, [P, P, U64, U64, I, P]), "orc_backend_error": (C.c_char_p, [P]),
        "orc_backend_hidden": (I, [P, P, U64]),
        "orc_backend_set_capture": (None, [P, I]), "orc_backend_layer_x": (C.c_int64, [P, P, U64]),
        "orc_backend_set_teacher": (None, [P, P, U64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def have_avx2() -> bool:
    return bool(lib().orc_have_avx2())


def default_path() -> int:
    """The tier RIE itself would pick on this host (x86: AVX2 when present)."""
    return PATH_AVX2 if have_avx2() else PATH_SCALAR


def block_size(t): return lib().orc_block_size(t)
def block_bytes(t): return lib().orc_block_bytes(t)
def row_bytes(t, n): return lib().orc_row_bytes(t, n)


def act_format(t: int) -> str:
    if t in (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0):
        return "q8_0"
    if t in (Q4_K, Q5_K, Q6_K, Q2_K, Q3_K):
        return "q8k"
    return "f32"


def f32_to_f16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_n(_p(x), _p(out), x.size, PATH_SCALAR)
    return out


def f32_to_f16_simd(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_n(_p(x), _p(out), x.size, PATH_AVX2)
    return out


class Rng:
    """xorshift64 of crates/rie-core/src/testing.rs:10-30."""

    def __init__(self, seed: int):
        self.state = np.array([lib().orc_rng_new(seed)], dtype=np.uint64)

    def next_u64(self) -> int:
        return int(lib().orc_rng_next(_p(self.state)))

    def vec(self, n: int, scale: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().orc_rng_vec(_p(self.state), _p(out), n, scale)
        return out

    def weight(self, t: int, rows: int, cols: int, gain: float = 1.0) -> np.ndarray:
        """random_weight (testing.rs:46-91): random bytes with valid f16 scales patched in."""
        nbytes = rows * row_bytes(t, cols)
        out = np.zeros(nbytes, dtype=np.uint8)
        assert lib().orc_random_weight(_p(self.state), t, rows, cols, gain, _p(out)) == 0
        return out.reshape(rows, row_bytes(t, cols))


def quantize_row_q8_0(x, path: int | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.shape[-1] % 32 == 0
    out = np.zeros(x.size // 32, dtype=BLOCK_Q8_0)
    lib().orc_quantize_row_q8_0(_p(x), x.size, _p(out), default_path() if path is None else path)
    return out.reshape(x.shape[:-1] + (x.shape[-1] // 32,))


def quantize_row_q8_k(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.shape[-1] % 256 == 0
    out = np.zeros(x.size // 256, dtype=BLOCK_Q8K)
    lib().orc_quantize_row_q8_k(_p(x), x.size, _p(out))
    return out.reshape(x.shape[:-1] + (x.shape[-1] // 256,))


def quantize_acts(t: int, x, path: int | None = None) -> np.ndarray:
    f = act_format(t)
    if f == "q8_0":
        return quantize_row_q8_0(x, path)
    if f == "q8k":
        return quantize_row_q8_k(x)
    return np.ascontiguousarray(x, dtype=np.float32)


def dequantize_q8(blocks: np.ndarray) -> np.ndarray:
    qs = blocks["qs"].astype(np.float32)
    return (qs * blocks["d"][..., None]).reshape(blocks.shape[:-1] + (-1,))


def quantize_weight(t: int, x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.zeros(rows * row_bytes(t, cols), dtype=np.uint8)
    n = lib().orc_quantize_weight(t, _p(x), x.size, _p(out))
    if n == 0:
        raise ValueError(f"no quantizer for {TYPE_NAMES.get(t, t)}")
    return out.reshape(rows, row_bytes(t, cols))


def dequantize(t: int, w: np.ndarray, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rows = w.size // row_bytes(t, cols)
    out = np.empty((rows, cols), dtype=np.float32)
    assert lib().orc_dequantize_row(t, _p(w), _p(out), rows * cols) == 0
    return out


def vec_dot(t: int, w_row: np.ndarray, act: np.ndarray, n: int, path: int | None = None) -> float:
    w_row = np.ascontiguousarray(w_row, dtype=np.uint8)
    act = np.ascontiguousarray(act)
    return float(lib().orc_vec_dot(t, _p(w_row), _p(act), n, default_path() if path is None else path))


def block_sums(t: int, w_row: np.ndarray, act: np.ndarray, n: int) -> np.ndarray:
    per = 2 if t in (Q4_K, Q5_K) else 1
    out = np.zeros(per * n // block_size(t), dtype=np.int32)
    k = lib().orc_block_sums(t, _p(np.ascontiguousarray(w_row, dtype=np.uint8)), _p(np.ascontiguousarray(act)), n, _p(out))
    assert k == out.size
    return out


JOB = np.dtype({"names": ["ty", "pad", "rows", "cols", "w", "out", "ld"],
                "formats": ["<i4", "<i4", "<u8", "<u8", "<u8", "<u8", "<u8"],
                "offsets": [0, 4, 8, 16, 24, 32, 40], "itemsize": 48})


def matmul_multi(x, weights, n_threads: int = 1, path: int | None = None):
    """weights: list of (type, uint8 [rows, row_bytes], cols). Returns list of [n_tok, rows] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None]
    n_tok, k = x.shape
    jobs = np.zeros(len(weights), dtype=JOB)
    outs, keep = [], []
    for i, (t, w, cols) in enumerate(weights):
        assert cols == k
        w = np.ascontiguousarray(w, dtype=np.uint8)
        rows = w.size // row_bytes(t, cols)
        o = np.zeros((n_tok, rows), dtype=np.float32)
        jobs[i] = (t, 0, rows, cols, w.ctypes.data, o.ctypes.data, rows)
        outs.append(o)
        keep.append(w)
    lib().orc_matmul_multi(n_threads, _p(x), n_tok, k, _p(jobs), len(weights), default_path() if path is None else path)
    return outs


def matmul_multi_q(acts_q8_0, acts_q8k, n_tok, k, weights, n_threads=1, path=None):
    """Like matmul_multi on already-quantized activations (numpy block arrays or None)."""
    jobs = np.zeros(len(weights), dtype=JOB)
    outs, keep = [], []
    for i, (t, w, cols) in enumerate(weights):
        w = np.ascontiguousarray(w, dtype=np.uint8)
        rows = w.size // row_bytes(t, cols)
        o = np.zeros((n_tok, rows), dtype=np.float32)
        jobs[i] = (t, 0, rows, cols, w.ctypes.data, o.ctypes.data, rows)
        outs.append(o)
        keep.append(w)
    a0 = _p(np.ascontiguousarray(acts_q8_0)) if acts_q8_0 is not None else None
    ak = _p(np.ascontiguousarray(acts_q8k)) if acts_q8k is not None else None
    lib().orc_matmul_multi_q(n_threads, a0, ak, None, n_tok, k, _p(jobs), len(weights),
                             default_path() if path is None else path)
    return outs


# ---- turbo4 -------------------------------------------------------------------------
def kv_seed() -> int:
    return int(lib().orc_kv_seed())


def turbo_sign(seed: int, i: int) -> float:
    return float(lib().orc_turbo_sign(seed, i))


def turbo_block_size(d: int) -> int:
    return lib().orc_turbo_block_size(d)


def row_bytes_4(d: int) -> int:
    return lib().orc_turbo_row_bytes_4(d)


def rotate(x, seed: int | None = None, inverse: bool = False) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    d = y.shape[-1]
    seed = kv_seed() if seed is None else seed
    for r in y.reshape(-1, d):
        lib().orc_turbo_rotate(seed, _p(r), d, int(inverse))
    return y


def turbo_quantize_4(x, seed: int | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = x.shape[-1]
    rows = x.reshape(-1, d)
    out = np.zeros((rows.shape[0], row_bytes_4(d)), dtype=np.uint8)
    seed = kv_seed() if seed is None else seed
    for i in range(rows.shape[0]):
        lib().orc_turbo_quantize_4(seed, _p(np.ascontiguousarray(rows[i])), d, _p(out[i]))
    return out.reshape(x.shape[:-1] + (row_bytes_4(d),))


def turbo_dot_rotated_4(q_blocks, row, d: int, path: int | None = None) -> float:
    return float(lib().orc_turbo_dot_rotated_4(_p(np.ascontiguousarray(q_blocks)), _p(np.ascontiguousarray(row)), d,
                                              default_path() if path is None else path))


def turbo_axpy_rotated_4(y: np.ndarray, a: float, row, path: int | None = None) -> None:
    lib().orc_turbo_axpy_rotated_4(_p(y), a, _p(np.ascontiguousarray(row)), y.size,
                                   default_path() if path is None else path)


def turbo_dequantize_4(row, d: int, seed: int | None = None) -> np.ndarray:
    out = np.zeros(d, dtype=np.float32)
    lib().orc_turbo_dequantize_4(kv_seed() if seed is None else seed, _p(np.ascontiguousarray(row)), _p(out), d)
    return out


def turbo_codebook(bits: int) -> np.ndarray:
    out = np.zeros(2 ** bits, dtype=np.float32)
    lib().orc_turbo_codebook(bits, _p(out))
    return out


def kv_levels() -> np.ndarray:
    out = np.zeros(16, dtype=np.float32)
    lib().orc_turbo_kv_levels(_p(out))
    return out


def kv_row_bytes(kv_type: int, hd: int) -> int:
    if kv_type == KV_F16:
        return 2 * hd
    if kv_type == KV_Q8_0:
        return hd // 32 * 34
    return row_bytes_4(hd)


def kv_store(kv_type: int, x, path: int | None = None) -> np.ndarray:
    """Encode rows [..., hd] into the cache format (model/cpu.rs:300-328)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    hd = x.shape[-1]
    rows = x.reshape(-1, hd)
    rb = kv_row_bytes(kv_type, hd)
    out = np.zeros((rows.shape[0], rb), dtype=np.uint8)
    for i in range(rows.shape[0]):
        lib().orc_kv_store(kv_type, _p(np.ascontiguousarray(rows[i])), hd, _p(out[i]),
                           default_path() if path is None else path)
    return out.reshape(x.shape[:-1] + (rb,))


def attention(q, kcache, vcache, n_head, n_head_kv, hd, pos0, slots, kv_type, window=0, softcap=0.0,
              n_threads=1, path=None) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_tok = q.size // (n_head * hd)
    out = np.zeros((n_tok, n_head * hd), dtype=np.float32)
    lib().orc_attention(n_threads, n_head, n_head_kv, hd, n_tok, pos0, window, softcap, _p(q), kv_type,
                        _p(np.ascontiguousarray(kcache)), _p(np.ascontiguousarray(vcache)), slots, _p(out),
                        default_path() if path is None else path)
    return out


def rmsnorm(x, w, eps, path=None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, dtype=np.float32)), x.size, eps,
                      default_path() if path is None else path)
    return out


def rope_table(dim, base, pos, freq_scale=1.0):
    c = np.zeros(dim // 2, dtype=np.float32)
    s = np.zeros(dim // 2, dtype=np.float32)
    lib().orc_rope_table(dim, base, freq_scale, pos, _p(c), _p(s))
    return c, s


def rope_apply(x, neox, c, s) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().orc_rope_apply(_p(y), y.size, int(neox), _p(np.ascontiguousarray(c)), _p(np.ascontiguousarray(s)))
    return y


# ---- transformer forward (model/cpu.rs:210-409) -------------------------------------------
class ModelConfig(C.Structure):
    """Same field order as orc_model_config / rcu_model_config."""
    _fields_ = [("n_vocab", C.c_uint32), ("n_embd", C.c_uint32), ("n_layer", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("n_ff", C.c_uint32), ("rope_dim", C.c_uint32),
                ("rope_neox", C.c_int32), ("rope_base", C.c_float), ("rope_freq_scale", C.c_float),
                ("rms_eps", C.c_float), ("attn_scale", C.c_float), ("embd_scale", C.c_float),
                ("residual_scale", C.c_float), ("logit_scale", C.c_float), ("attn_softcap", C.c_float),
                ("final_softcap", C.c_float), ("swa_window", C.c_uint32), ("swa_pattern", C.c_uint32),
                ("rope_base_swa", C.c_float), ("act", C.c_int32), ("n_expert", C.c_uint32),
                ("n_expert_used", C.c_uint32), ("n_ff_exp", C.c_uint32), ("expert_norm_topk", C.c_int32),
                ("expert_unit_weights", C.c_int32)]


class OracleModel:
    def __init__(self, cfg: ModelConfig):
        self.cfg = cfg
        self.ptr = lib().orc_model_create(C.byref(cfg))

    def set_tensor(self, name: str, t: int, rows: int, cols: int, data) -> None:
        a = np.ascontiguousarray(data).view(np.uint8)
        assert a.size == rows * row_bytes(t, cols), name
        lib().orc_model_set_tensor(self.ptr, name.encode(), t, rows, cols, _p(a))

    def __del__(self):
        try:
            lib().orc_model_free(self.ptr)
        except Exception:
            pass


class OracleBackend:
    """CpuBackend of the reference, restated (forward / hidden)."""

    def __init__(self, model: OracleModel, n_ctx: int, max_batch: int, kv_type: int = KV_F16, n_threads: int = 8,
                 path: int | None = None):
        self.model = model
        self.n_vocab = model.cfg.n_vocab
        self.ptr = lib().orc_backend_create(model.ptr, n_ctx, max_batch, kv_type, n_threads,
                                            default_path() if path is None else path)

    def forward(self, tokens, pos: int, all_logits: bool = False) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = tok.size
        out = np.zeros(((n if all_logits else 1), self.n_vocab), dtype=np.float32)
        st = lib().orc_backend_forward(self.ptr, _p(tok), n, pos, int(all_logits), _p(out))
        if st != 0:
            raise RuntimeError(lib().orc_backend_error(self.ptr).decode())
        return out

    def set_capture(self, on: bool) -> None:
        """Record the residual stream at every layer's entry (and after the last layer)."""
        lib().orc_backend_set_capture(self.ptr, int(bool(on)))

    def set_teacher(self, x) -> None:
        """Teacher forcing: replace the residual rows at every layer's entry and before the head by
        x ([n_layer + 1, n, n_embd]) in the following forwards (None: off)."""
        if x is None:
            lib().orc_backend_set_teacher(self.ptr, None, 0)
        else:
            self._teacher = np.ascontiguousarray(x, dtype=np.float32)
            lib().orc_backend_set_teacher(self.ptr, _p(self._teacher), self._teacher.size)

    def layer_x(self) -> np.ndarray:
        """[n_layer + 1, n, n_embd] residual rows of the latest forward (capture on)."""
        cnt = int(lib().orc_backend_layer_x(self.ptr, None, 0))
        out = np.zeros(cnt, dtype=np.float32)
        assert lib().orc_backend_layer_x(self.ptr, _p(out), cnt) == cnt
        L, e = self.model.cfg.n_layer, self.model.cfg.n_embd
        return out.reshape(L + 1, -1, e)

    def __del__(self):
        try:
            lib().orc_backend_free(self.ptr)
        except Exception:
            pass
