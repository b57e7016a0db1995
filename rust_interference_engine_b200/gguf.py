"""GGUF v2/v3 container: reader, writer and the model configuration it carries.

The reference reads GGUF files zero-copy through a memory map (crates/rie-core/src/gguf.rs:
reader :106-330, writer :331-438) and derives its ModelConfig from the metadata
(crates/rie-core/src/model/config.rs:106-247). This module restates both from the public GGUF
layout so that `model.Model.load_gguf` can feed real GGUF files to the CUDA backend:

    u32 magic "GGUF" | u32 version (2 or 3) | u64 n_tensors | u64 n_kv
    n_kv x (string key, u32 value type, value)
    n_tensors x (string name, u32 n_dims, u64 dims[n_dims], u32 ggml type, u64 offset)
    padding to general.alignment (default 32) | tensor data (offsets relative to its start)

Strings are a u64 length and UTF-8 bytes; arrays a u32 element type, a u64 count and the
elements. dims[0] is the row length (innermost dimension).
"""
from __future__ import annotations

import enum
import struct
from dataclasses import dataclass

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little endian
DEFAULT_ALIGNMENT = 32


class ValueType(enum.IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


_SCALAR = {ValueType.UINT8: "<B", ValueType.INT8: "<b", ValueType.UINT16: "<H", ValueType.INT16: "<h",
           ValueType.UINT32: "<I", ValueType.INT32: "<i", ValueType.FLOAT32: "<f", ValueType.BOOL: "<?",
           ValueType.UINT64: "<Q", ValueType.INT64: "<q", ValueType.FLOAT64: "<d"}


class GgufError(ValueError):
    pass


@dataclass
class Value:
    """A metadata value with its GGUF type (arrays: a list of Value)."""
    type: ValueType
    value: object

    def as_u64(self):
        """Unsigned view of integer and bool values (negative integers: None), gguf.rs:34-46."""
        if self.type in (ValueType.FLOAT32, ValueType.FLOAT64, ValueType.STRING, ValueType.ARRAY):
            return None
        v = int(self.value)
        return v if v >= 0 else None

    def as_f64(self):
        return float(self.value) if self.type in (ValueType.FLOAT32, ValueType.FLOAT64) else None


@dataclass
class TensorInfo:
    name: str
    dims: tuple
    type: int
    offset: int

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= int(d)
        return n

    @property
    def row_len(self) -> int:
        return int(self.dims[0]) if self.dims else 1

    @property
    def n_rows(self) -> int:
        return self.n_elements // max(self.row_len, 1)


def _row_bytes(ggml_type: int, cols: int) -> int:
    from rust_interference_engine_b200 import GgmlType
    return GgmlType(ggml_type).row_bytes(cols)


class _Reader:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def take(self, n: int):
        if self.pos + n > len(self.buf):
            raise GgufError("unexpected end of file")
        b = bytes(self.buf[self.pos:self.pos + n])
        self.pos += n
        return b

    def scalar(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        if n > (1 << 24):
            raise GgufError(f"string of {n} bytes")
        try:
            return self.take(n).decode("utf-8")
        except UnicodeDecodeError as e:
            raise GgufError(f"string is not UTF-8: {e}") from None

    def value(self, vt: int, depth: int = 0) -> Value:
        try:
            vt = ValueType(vt)
        except ValueError:
            raise GgufError(f"unknown metadata value type {vt}") from None
        if vt == ValueType.STRING:
            return Value(vt, self.string())
        if vt == ValueType.ARRAY:
            if depth > 8:
                raise GgufError("nested arrays too deep")
            et = self.scalar("<I")
            n = self.scalar("<Q")
            if n > (1 << 28):
                raise GgufError(f"array of {n} elements")
            return Value(vt, [self.value(et, depth + 1) for _ in range(n)])
        return Value(vt, self.scalar(_SCALAR[vt]))


class GgufFile:
    """Parsed GGUF file; tensor data stays in the (memory-mapped) buffer."""

    def __init__(self, buf):
        self.buf = buf
        r = _Reader(buf)
        if r.scalar("<I") != GGUF_MAGIC:
            raise GgufError("not a GGUF file (bad magic)")
        self.version = r.scalar("<I")
        if self.version not in (2, 3):
            raise GgufError(f"GGUF version {self.version} (only v2 and v3 are supported)")
        n_tensors = r.scalar("<Q")
        n_kv = r.scalar("<Q")
        if n_tensors > (1 << 24) or n_kv > (1 << 24):
            raise GgufError("implausible tensor / metadata count")
        self.metadata = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.scalar("<I"))
        self.tensors = []
        for _ in range(n_tensors):
            name = r.string()
            nd = r.scalar("<I")
            if nd == 0 or nd > 4:
                raise GgufError(f"tensor {name}: {nd} dimensions")
            dims = tuple(r.scalar("<Q") for _ in range(nd))
            ty = r.scalar("<I")
            off = r.scalar("<Q")
            self.tensors.append(TensorInfo(name, dims, ty, off))
        align = self.get_u64("general.alignment")
        self.alignment = max(int(DEFAULT_ALIGNMENT if align is None else align), 1)
        self.data_offset = -(-r.pos // self.alignment) * self.alignment
        self._index = {t.name: t for t in self.tensors}
        for t in self.tensors:
            nbytes = t.n_rows * _row_bytes(t.type, t.row_len)
            if t.offset % self.alignment or self.data_offset + t.offset + nbytes > len(buf):
                raise GgufError(f"tensor {t.name}: data out of bounds or misaligned")

    @classmethod
    def open(cls, path) -> "GgufFile":
        return cls(np.memmap(path, dtype=np.uint8, mode="r"))

    @classmethod
    def from_bytes(cls, data: bytes) -> "GgufFile":
        return cls(np.frombuffer(data, dtype=np.uint8))

    def tensor(self, name: str):
        return self._index.get(name)

    def tensor_data(self, t: TensorInfo) -> np.ndarray:
        """uint8 view [n_rows, row_bytes] of the tensor's GGUF bytes (no copy)."""
        rb = _row_bytes(t.type, t.row_len)
        start = self.data_offset + t.offset
        return np.asarray(self.buf[start:start + t.n_rows * rb]).reshape(t.n_rows, rb)

    def get(self, key: str):
        return self.metadata.get(key)

    def get_u64(self, key: str):
        v = self.metadata.get(key)
        return v.as_u64() if v is not None else None

    def get_f32(self, key: str):
        v = self.metadata.get(key)
        return v.as_f64() if v is not None else None

    def get_str(self, key: str):
        v = self.metadata.get(key)
        return v.value if v is not None and v.type == ValueType.STRING else None

    def get_bool(self, key: str):
        v = self.metadata.get(key)
        return bool(v.value) if v is not None and v.type == ValueType.BOOL else None

    def get_arr(self, key: str):
        v = self.metadata.get(key)
        return v.value if v is not None and v.type == ValueType.ARRAY else None


class GgufWriter:
    """Builds a GGUF v3 file in memory (gguf.rs:331-438)."""

    def __init__(self):
        self.kvs = []
        self.tensors = []

    def kv(self, key: str, vtype: ValueType, value) -> "GgufWriter":
        self.kvs.append((key, ValueType(vtype), value))
        return self

    def tensor(self, name: str, rows: int, cols: int, ggml_type: int, data) -> "GgufWriter":
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        if data.size != rows * _row_bytes(ggml_type, cols):
            raise GgufError(f"tensor {name}: {data.size} bytes for {rows} x {cols} of type {ggml_type}")
        dims = (cols,) if rows == 1 else (cols, rows)
        self.tensors.append((name, dims, int(ggml_type), data))
        return self

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    def _val(self, vt: ValueType, v) -> bytes:
        if vt == ValueType.STRING:
            return self._str(v)
        if vt == ValueType.ARRAY:
            et, items = v
            et = ValueType(et)
            return struct.pack("<IQ", et, len(items)) + b"".join(self._val(et, x) for x in items)
        return struct.pack(_SCALAR[vt], v)

    def to_bytes(self, alignment: int = DEFAULT_ALIGNMENT) -> bytes:
        out = [struct.pack("<IIQQ", GGUF_MAGIC, 3, len(self.tensors), len(self.kvs))]
        for key, vt, v in self.kvs:
            out.append(self._str(key) + struct.pack("<I", vt) + self._val(vt, v))
        off = 0
        offsets = []
        for name, dims, ty, data in self.tensors:
            offsets.append(off)
            out.append(self._str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims) +
                       struct.pack("<IQ", ty, off))
            off = -(-(off + data.size) // alignment) * alignment
        head = b"".join(out)
        blob = bytearray(head + bytes(-len(head) % alignment))
        for (name, dims, ty, data), o in zip(self.tensors, offsets):
            blob += bytes(len(head) + (-len(head) % alignment) + o - len(blob))
            blob += data.tobytes()
        return bytes(blob)

    def write(self, path, alignment: int = DEFAULT_ALIGNMENT) -> None:
        with open(path, "wb") as f:
            f.write(self.to_bytes(alignment))


# ---- model configuration (model/config.rs:106-247) ------------------------------------------
ARCHS = ("llama", "mistral", "qwen2", "qwen3", "phi3", "gemma", "gemma2", "gemma3", "granite", "qwen3moe",
         "qwen2moe")


def config_from_gguf(g: GgufFile):
    """ModelConfig::from_gguf restated: rcu_model_config of the file's metadata."""
    from rust_interference_engine_b200.model import ModelConfig
    arch = g.get_str("general.architecture")
    if arch is None:
        raise GgufError("missing general.architecture")
    if arch not in ARCHS:
        raise GgufError(f"architecture '{arch}' (supported: {', '.join(ARCHS)})")

    def key(k):
        return f"{arch}.{k}"

    def req(k):
        v = g.get_u64(key(k))
        if v is None:
            raise GgufError(f"missing metadata {key(k)}")
        return v

    def opt(k, default):  # unwrap_or: the default only when the key is absent
        v = g.get_u64(key(k))
        return default if v is None else v

    n_embd, n_layer, n_head = req("embedding_length"), req("block_count"), req("attention.head_count")
    n_head_kv = opt("attention.head_count_kv", n_head)
    head_dim = opt("attention.key_length", n_embd // n_head)
    vl = g.get_u64(key("attention.value_length"))
    if vl is not None and vl != head_dim:
        raise GgufError(f"value head dim {vl} != key head dim {head_dim}")
    n_ff = g.get_u64(key("feed_forward_length"))
    if n_ff is None:
        n_ff = g.get_u64(key("expert_feed_forward_length"))
    if n_ff is None:
        raise GgufError(f"missing metadata {key('feed_forward_length')}")
    toks = g.get_arr("tokenizer.ggml.tokens")
    n_vocab = len(toks) if toks is not None else g.get_u64(key("vocab_size"))
    if n_vocab is None:
        raise GgufError("missing vocabulary")
    rms_eps = g.get_f32(key("attention.layer_norm_rms_epsilon"))
    rope_dim = opt("rope.dimension_count", head_dim)
    rope_base = g.get_f32(key("rope.freq_base"))
    freq_scale = 1.0
    if g.get_str(key("rope.scaling.type")) == "linear":
        f = g.get_f32(key("rope.scaling.factor"))
        if f is not None and f > 0:
            freq_scale = 1.0 / f
    s = g.get_f32(key("rope.scale_linear"))
    if s is not None and s > 0:
        freq_scale = 1.0 / s
    gemma = arch in ("gemma", "gemma2", "gemma3")
    c = ModelConfig()
    c.n_vocab, c.n_embd, c.n_layer, c.n_head, c.n_head_kv = n_vocab, n_embd, n_layer, n_head, n_head_kv
    c.head_dim, c.n_ff, c.rope_dim = head_dim, n_ff, rope_dim
    c.rope_neox = int(arch in ("qwen2", "qwen3", "phi3", "gemma", "gemma2", "gemma3", "qwen3moe", "qwen2moe"))
    c.rope_base = 10000.0 if rope_base is None else rope_base
    c.rope_freq_scale = freq_scale
    c.rms_eps = 1e-5 if rms_eps is None else rms_eps
    c.attn_scale = float(1.0 / np.sqrt(np.float32(head_dim)))
    c.embd_scale = float(np.sqrt(np.float32(n_embd))) if gemma else 1.0
    c.residual_scale = c.logit_scale = 1.0
    c.attn_softcap = c.final_softcap = 0.0
    c.swa_window = c.swa_pattern = 0
    c.rope_base_swa = 0.0
    c.act = 1 if gemma else 0
    c.n_expert = opt("expert_count", 0)
    c.n_expert_used = opt("expert_used_count", 2)
    c.n_ff_exp = opt("expert_feed_forward_length", n_ff)
    nt = g.get_bool(key("expert_weights_norm"))
    c.expert_norm_topk = int(arch != "qwen2moe" if nt is None else nt)
    c.expert_unit_weights = 0
    if arch == "gemma2":
        a, f = g.get_f32(key("attn_logit_softcapping")), g.get_f32(key("final_logit_softcapping"))
        c.attn_softcap = 50.0 if a is None else a
        c.final_softcap = 30.0 if f is None else f
        c.swa_window = opt("attention.sliding_window", 4096)
        c.swa_pattern = 2
        if n_layer == 46:
            c.attn_scale = float(1.0 / np.sqrt(np.float32(n_embd // n_head)))
    elif arch == "gemma3":
        c.swa_window = opt("attention.sliding_window", 1024)
        c.swa_pattern = 6
        c.rope_base_swa = 10000.0
        if n_layer == 62:
            c.attn_scale = float(1.0 / np.sqrt(np.float32(n_embd // n_head)))
        f, a = g.get_f32(key("final_logit_softcapping")), g.get_f32(key("attn_logit_softcapping"))
        c.final_softcap = 0.0 if f is None else f
        c.attn_softcap = 0.0 if a is None else a
    elif arch == "granite":
        e, r, lg, sc = (g.get_f32(key(k)) for k in ("embedding_scale", "residual_scale", "logit_scale",
                                                    "attention.scale"))
        c.embd_scale = 1.0 if e is None else e
        c.residual_scale = 1.0 if r is None else r
        c.logit_scale = 1.0 if lg is None else lg
        if sc is not None:
            c.attn_scale = sc
    if n_head % n_head_kv:
        raise GgufError(f"n_head {n_head} not divisible by n_head_kv {n_head_kv}")
    if rope_dim > head_dim or rope_dim % 2:
        raise GgufError(f"invalid rope dimension {rope_dim}")
    return c


def spec_writer(spec, tensors) -> GgufWriter:
    """A GGUF of a synthetic model: the metadata config_from_gguf reads back as spec.config(),
    then every (name, type, rows, cols, data) of `tensors`."""
    w = GgufWriter()
    a = spec.arch
    u32, f32 = ValueType.UINT32, ValueType.FLOAT32
    w.kv("general.architecture", ValueType.STRING, a)
    w.kv("general.alignment", u32, DEFAULT_ALIGNMENT)
    w.kv(f"{a}.vocab_size", u32, spec.n_vocab)
    w.kv(f"{a}.embedding_length", u32, spec.n_embd)
    w.kv(f"{a}.block_count", u32, spec.n_layer)
    w.kv(f"{a}.attention.head_count", u32, spec.n_head)
    w.kv(f"{a}.attention.head_count_kv", u32, spec.n_head_kv)
    w.kv(f"{a}.attention.key_length", u32, spec.head_dim)
    w.kv(f"{a}.attention.value_length", u32, spec.head_dim)
    w.kv(f"{a}.feed_forward_length", u32, spec.n_ff)
    w.kv(f"{a}.rope.dimension_count", u32, spec.rope_dim)
    w.kv(f"{a}.rope.freq_base", f32, 1_000_000.0 if a == "gemma3" else spec.rope_base)
    w.kv(f"{a}.attention.layer_norm_rms_epsilon", f32, spec.rms_eps)
    if spec.swa_window or a in ("gemma2", "gemma3"):
        w.kv(f"{a}.attention.sliding_window", u32, spec.swa_window)
    if spec.n_expert:
        w.kv(f"{a}.expert_count", u32, spec.n_expert)
        w.kv(f"{a}.expert_used_count", u32, spec.n_expert_used)
        w.kv(f"{a}.expert_feed_forward_length", u32, spec.n_ff_exp)
    for name, t, rows, cols, data in tensors:
        w.tensor(name, rows, cols, int(t), data)
    return w
