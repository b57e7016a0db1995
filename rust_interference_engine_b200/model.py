"""Transformer forward on the device: the reference's `Backend` trait (model/mod.rs:303-320)
implemented by the CUDA library's scheduler (rcu_model_* / rcu_backend_* of rie_cuda.h).

  Model(ctx, config)                  Model::load without the file: tensors by GGUF name
  CudaBackend(model, n_ctx, ...)      CpuBackend::with_kv_type (model/cpu.rs:100-177)
  CudaBackend.forward(tokens, pos)    Backend::forward (model/mod.rs:313)
  CudaBackend.hidden()                Backend::hidden (model/mod.rs:318)
  synthetic_tensors(spec, gen)        the tensor set of SyntheticSpec::build (testing.rs:229-383)
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import GgmlType, KvType, _check, _dptr, _lib


class ModelConfig(C.Structure):
    """rcu_model_config (flattened reference ModelConfig, model/config.rs:54-104)."""
    _fields_ = [("n_vocab", C.c_uint32), ("n_embd", C.c_uint32), ("n_layer", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("n_ff", C.c_uint32), ("rope_dim", C.c_uint32),
                ("rope_neox", C.c_int32), ("rope_base", C.c_float), ("rope_freq_scale", C.c_float),
                ("rms_eps", C.c_float), ("attn_scale", C.c_float), ("embd_scale", C.c_float),
                ("residual_scale", C.c_float), ("logit_scale", C.c_float), ("attn_softcap", C.c_float),
                ("final_softcap", C.c_float), ("swa_window", C.c_uint32), ("swa_pattern", C.c_uint32),
                ("rope_base_swa", C.c_float), ("act", C.c_int32), ("n_expert", C.c_uint32),
                ("n_expert_used", C.c_uint32), ("n_ff_exp", C.c_uint32), ("expert_norm_topk", C.c_int32),
                ("expert_unit_weights", C.c_int32)]




@dataclass
class SyntheticSpec:
    """Shape of a synthetic transformer (testing.rs:93-124)."""
    arch: str = "qwen3"
    n_vocab: int = 384
    n_embd: int = 256
    n_layer: int = 2
    n_head: int = 4
    n_head_kv: int = 2
    head_dim: int = 64
    n_ff: int = 512
    rope_dim: int = 64
    wtype: int = GgmlType.Q4_0
    embd_type: int = GgmlType.Q8_0
    tied_output: bool = False
    qkv_bias: bool = False
    qk_norm: bool = True
    post_norms: bool = False
    fused: bool = False
    swa_window: int = 0
    rope_base: float = 10000.0
    rms_eps: float = 1e-6
    type_overrides: dict = field(default_factory=dict)  # per-tensor-suffix ggml type (Q4_K_M style mixes)
    n_expert: int = 0        # mixture of experts (testing.rs:115-120): 0 = dense
    n_expert_used: int = 2
    n_ff_exp: int = 256
    n_ff_shexp: int = 0      # always-on shared expert (qwen2moe)

    @classmethod
    def tiny(cls, arch: str, wtype: int) -> "SyntheticSpec":  # testing.rs:127-154
        return cls(arch=arch, wtype=wtype, embd_type=GgmlType.Q8_0 if GgmlType(wtype).block_size > 1 else wtype,
                   qkv_bias=arch == "qwen2", qk_norm=arch in ("qwen3", "gemma3"),
                   post_norms=arch in ("gemma2", "gemma3"), fused=arch == "phi3",
                   swa_window=5 if arch in ("gemma2", "gemma3") else 0,
                   n_expert=8 if arch in ("qwen3moe", "qwen2moe") else 0,
                   n_ff_shexp=256 if arch == "qwen2moe" else 0)

    def config(self) -> ModelConfig:
        """ModelConfig::from_gguf rules for the synthetic metadata (model/config.rs:106-247)."""
        gemma = self.arch in ("gemma", "gemma2", "gemma3")
        c = ModelConfig()
        c.n_vocab, c.n_embd, c.n_layer = self.n_vocab, self.n_embd, self.n_layer
        c.n_head, c.n_head_kv, c.head_dim, c.n_ff = self.n_head, self.n_head_kv, self.head_dim, self.n_ff
        c.rope_dim = self.rope_dim
        c.rope_neox = int(self.arch in ("qwen2", "qwen3", "phi3", "gemma", "gemma2", "gemma3", "qwen3moe", "qwen2moe"))
        c.rope_base = 1_000_000.0 if self.arch == "gemma3" else self.rope_base
        c.rope_freq_scale = 1.0
        c.rms_eps = self.rms_eps
        c.attn_scale = 1.0 / np.sqrt(np.float32(self.head_dim))
        c.embd_scale = float(np.sqrt(np.float32(self.n_embd))) if gemma else 1.0
        c.residual_scale = 1.0
        c.logit_scale = 1.0
        c.attn_softcap = 50.0 if self.arch == "gemma2" else 0.0
        c.final_softcap = 30.0 if self.arch == "gemma2" else 0.0
        c.swa_window = self.swa_window
        c.swa_pattern = 2 if self.arch == "gemma2" else (6 if self.arch == "gemma3" else 0)
        c.rope_base_swa = 10000.0 if self.arch == "gemma3" else 0.0
        c.act = 1 if gemma else 0
        # expert_feed_forward_length, else feed_forward_length (config.rs:165)
        c.n_expert, c.n_expert_used = self.n_expert, self.n_expert_used
        c.n_ff_exp = self.n_ff_exp if self.n_expert else self.n_ff
        c.expert_norm_topk = int(self.arch != "qwen2moe")  # expert_weights_norm default (config.rs:167)
        c.expert_unit_weights = 0
        return c

    def type_of(self, name: str) -> int:
        for suffix, t in self.type_overrides.items():
            if name.endswith(suffix):
                return t
        return self.wtype


def synthetic_tensors(spec: SyntheticSpec, weight, vec_f32, norm):
    """Yield (name, ggml_type, rows, cols, bytes) in SyntheticSpec::build order (testing.rs:314-381).

    weight(type, rows, cols) -> uint8 GGUF bytes; vec_f32(n, scale) / norm(n) -> float32."""
    e, ff = spec.n_embd, spec.n_ff
    qd, kvd, hd = spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim, spec.head_dim
    yield "token_embd.weight", spec.embd_type, spec.n_vocab, e, weight(spec.embd_type, spec.n_vocab, e)
    yield "output_norm.weight", GgmlType.F32, 1, e, norm(e)
    if not spec.tied_output:
        yield "output.weight", spec.embd_type, spec.n_vocab, e, weight(spec.embd_type, spec.n_vocab, e)
    for il in range(spec.n_layer):
        p = f"blk.{il}."
        yield p + "attn_norm.weight", GgmlType.F32, 1, e, norm(e)
        if spec.fused:
            t = spec.type_of("attn_qkv.weight")
            yield p + "attn_qkv.weight", t, qd + 2 * kvd, e, weight(t, qd + 2 * kvd, e)
        else:
            for nm, rows in (("attn_q.weight", qd), ("attn_k.weight", kvd), ("attn_v.weight", kvd)):
                t = spec.type_of(nm)
                yield p + nm, t, rows, e, weight(t, rows, e)
        if spec.qkv_bias:
            yield p + "attn_q.bias", GgmlType.F32, 1, qd, vec_f32(qd, 0.1)
            yield p + "attn_k.bias", GgmlType.F32, 1, kvd, vec_f32(kvd, 0.1)
            yield p + "attn_v.bias", GgmlType.F32, 1, kvd, vec_f32(kvd, 0.1)
        if spec.qk_norm:
            yield p + "attn_q_norm.weight", GgmlType.F32, 1, hd, norm(hd)
            yield p + "attn_k_norm.weight", GgmlType.F32, 1, hd, norm(hd)
        t = spec.type_of("attn_output.weight")
        yield p + "attn_output.weight", t, e, qd, weight(t, e, qd)
        if spec.post_norms:
            yield p + "post_attention_norm.weight", GgmlType.F32, 1, e, norm(e)
            yield p + "post_ffw_norm.weight", GgmlType.F32, 1, e, norm(e)
        yield p + "ffn_norm.weight", GgmlType.F32, 1, e, norm(e)
        if spec.n_expert:  # testing.rs:358-372 (router F32, experts stacked [expert][rows][cols])
            ne, fx, t = spec.n_expert, spec.n_ff_exp, spec.wtype
            yield p + "ffn_gate_inp.weight", GgmlType.F32, ne, e, vec_f32(ne * e, 0.5)
            yield p + "ffn_gate_exps.weight", t, fx * ne, e, weight(t, fx * ne, e)
            yield p + "ffn_up_exps.weight", t, fx * ne, e, weight(t, fx * ne, e)
            yield p + "ffn_down_exps.weight", t, e * ne, fx, weight(t, e * ne, fx)
            if spec.n_ff_shexp:
                fs = spec.n_ff_shexp
                yield p + "ffn_gate_shexp.weight", t, fs, e, weight(t, fs, e)
                yield p + "ffn_up_shexp.weight", t, fs, e, weight(t, fs, e)
                yield p + "ffn_down_shexp.weight", t, e, fs, weight(t, e, fs)
                yield p + "ffn_gate_inp_shexp.weight", GgmlType.F32, 1, e, vec_f32(e, 0.3)
        elif spec.fused:
            t = spec.type_of("ffn_up.weight")
            yield p + "ffn_up.weight", t, 2 * ff, e, weight(t, 2 * ff, e)
            t = spec.type_of("ffn_down.weight")
            yield p + "ffn_down.weight", t, e, ff, weight(t, e, ff)
        else:
            for nm, rows, cols in (("ffn_gate.weight", ff, e), ("ffn_up.weight", ff, e), ("ffn_down.weight", e, ff)):
                t = spec.type_of(nm)
                yield p + nm, t, rows, cols, weight(t, rows, cols)


def tp_unique_id() -> bytes:
    """Communicator id for a tensor-parallel backend: made on one rank, given to all."""
    buf = (C.c_uint8 * 128)()
    st = _lib.load().rcu_tp_unique_id(buf, 128)
    if st:
        raise _lib.RcuError(st, "rcu_tp_unique_id failed")
    return bytes(buf)


def tp_shard(cfg: ModelConfig, name: str, ty: int, rows: int, cols: int, data, rank: int, world: int):
    """The part of a GGUF tensor that rank `rank` of a tensor-parallel model keeps (host-only):
    (bytes as uint8, rows, cols)."""
    a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    r, c = C.c_uint64(0), C.c_uint64(0)
    lib = _lib.load()
    st = lib.rcu_tp_shard(C.byref(cfg), name.encode(), int(ty), rows, cols, a.ctypes.data_as(C.c_void_p), rank, world,
                          None, 0, C.byref(r), C.byref(c))
    if st:
        raise _lib.RcuError(st, f"rcu_tp_shard({name})")
    out = np.zeros(a.size, dtype=np.uint8)  # a shard is never larger than the tensor
    st = lib.rcu_tp_shard(C.byref(cfg), name.encode(), int(ty), rows, cols, a.ctypes.data_as(C.c_void_p), rank, world,
                          out.ctypes.data_as(C.c_void_p), out.size, C.byref(r), C.byref(c))
    if st:
        raise _lib.RcuError(st, f"rcu_tp_shard({name})")
    if rows == 1 and int(ty) in (0, 1, 30):  # 1-D f32 / f16 / bf16 vector
        nbytes = c.value * (4 if int(ty) == 0 else 2)
    else:
        nbytes = r.value * rcu_row_bytes_host(ty, c.value)
    return out[:nbytes], r.value, c.value


def rcu_row_bytes_host(ty: int, cols: int) -> int:
    return int(_lib.load().rcu_row_bytes(int(ty), cols))


class Model:
    """Model::load without the file. With world > 1 the model holds rank `rank`'s shard of a
    tensor-parallel split (set_tensor still takes the full tensors)."""

    def __init__(self, ctx, cfg: ModelConfig, rank: int = 0, world: int = 1):
        self.ctx, self.cfg, self.rank, self.world = ctx, cfg, rank, world
        lib = _lib.load()
        self.ptr = C.c_void_p()
        _check(ctx.ptr, lib.rcu_model_create_tp(ctx.ptr, C.byref(cfg), rank, world, C.byref(self.ptr)))

    @classmethod
    def load_gguf(cls, ctx, path_or_file, rank: int = 0, world: int = 1) -> "Model":
        """A model of a GGUF file (or parsed GgufFile): configuration from its metadata
        (model/config.rs:106-247), every tensor's GGUF bytes uploaded unchanged; with world > 1
        each rank keeps its tensor-parallel shard."""
        from rust_interference_engine_b200 import gguf
        g = path_or_file if isinstance(path_or_file, gguf.GgufFile) else gguf.GgufFile.open(path_or_file)
        m = cls(ctx, gguf.config_from_gguf(g), rank, world)
        for t in g.tensors:
            m.set_tensor(t.name, t.type, t.n_rows, t.row_len, g.tensor_data(t))
        return m

    def set_tensor(self, name: str, ty: int, rows: int, cols: int, data) -> None:
        a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        _check(self.ctx.ptr, _lib.load().rcu_model_set_tensor(self.ptr, name.encode(), int(ty), rows, cols,
                                                              a.ctypes.data_as(C.c_void_p)))

    def set_tensor_device(self, name: str, ty: int, rows: int, cols: int, dev) -> None:
        """set_tensor from GGUF bytes already in device memory (a CUDA tensor or pointer)."""
        _check(self.ctx.ptr, _lib.load().rcu_model_set_tensor_device(self.ptr, name.encode(), int(ty), rows, cols,
                                                                     C.c_void_p(_dptr(dev))))

    def free(self):
        if getattr(self, "ptr", None):
            _lib.load().rcu_model_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class CudaBackend:
    """`impl Backend for CudaBackend`: forward / hidden / max_batch / n_ctx."""

    def __init__(self, model: Model, n_ctx: int, max_batch: int, kv_type: KvType = KvType.F16,
                 comm_id: bytes | None = None):
        """comm_id: tp_unique_id() of rank 0, for a tensor-parallel model (every rank passes it)."""
        self.model, self.ctx = model, model.ctx
        self.ptr = C.c_void_p()
        uid = None if comm_id is None else (C.c_uint8 * len(comm_id)).from_buffer_copy(comm_id)
        _check(self.ctx.ptr, _lib.load().rcu_backend_create_tp(model.ptr, n_ctx, max_batch, int(kv_type), uid,
                                                               C.byref(self.ptr)))
        self.n_vocab = model.cfg.n_vocab
        self.n_embd = model.cfg.n_embd

    def name(self) -> str:
        return "CUDA (sm_100a)"

    def max_batch(self) -> int:
        return int(_lib.load().rcu_backend_max_batch(self.ptr))

    def n_ctx(self) -> int:
        return int(_lib.load().rcu_backend_n_ctx(self.ptr))

    def forward(self, tokens, pos: int, all_logits: bool = False) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, dtype=np.uint32).reshape(-1)
        rows = tok.size if all_logits else 1
        out = np.empty((rows, self.n_vocab), dtype=np.float32)  # every value is written by the call
        _check(self.ctx.ptr, _lib.load().rcu_backend_forward(self.ptr, tok.ctypes.data_as(C.c_void_p), tok.size, pos,
                                                             int(all_logits), out.ctypes.data_as(C.c_void_p),
                                                             out.size))
        return out

    def forward_device(self, tokens_dev, n: int, pos: int, logits_dev, all_logits: bool = False) -> None:
        _check(self.ctx.ptr, _lib.load().rcu_backend_forward_device(self.ptr, C.c_void_p(_dptr(tokens_dev)), n, pos,
                                                                    int(all_logits), C.c_void_p(_dptr(logits_dev))))

    def forward_layers(self, x, pos: int, layer0: int, layer1: int, logits: bool = False):
        """Layers [layer0, layer1) from hidden rows x (n x n_embd f32, numpy or CUDA tensor) at
        positions pos..pos+n-1: the residual rows after layer1 - 1 and, with logits (layer1 =
        n_layer), every row's logits, as numpy arrays."""
        import torch
        xd = torch.as_tensor(np.ascontiguousarray(x, dtype=np.float32)).cuda() if isinstance(x, np.ndarray) else x
        n = xd.shape[0]
        xo = torch.empty_like(xd)
        lg = torch.empty((n, self.n_vocab), device=xd.device) if logits else None
        _check(self.ctx.ptr, _lib.load().rcu_backend_forward_layers(
            self.ptr, C.c_void_p(_dptr(xd)), n, pos, layer0, layer1, C.c_void_p(_dptr(xo)),
            C.c_void_p(_dptr(lg)) if logits else None))
        self.ctx.sync()
        return xo.cpu().numpy(), (lg.cpu().numpy() if logits else None)

    def kv_cache(self, layer: int):
        """The rcu_kv handle of one layer's cache (owned by the backend)."""
        kv = C.c_void_p()
        _check(self.ctx.ptr, _lib.load().rcu_backend_kv(self.ptr, layer, C.byref(kv)))
        return kv

    def hidden(self) -> np.ndarray | None:
        rows = C.c_uint64(0)
        cap = 4096 * self.n_embd
        buf = np.zeros(cap, dtype=np.float32)
        _check(self.ctx.ptr, _lib.load().rcu_backend_hidden(self.ptr, buf.ctypes.data_as(C.c_void_p), cap,
                                                            C.byref(rows)))
        return buf[: rows.value * self.n_embd].reshape(rows.value, self.n_embd) if rows.value else None

    def free(self):
        if getattr(self, "ptr", None):
            _lib.load().rcu_backend_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
