"""B200 (sm_100a) implementation of the Rust Inference Engine's quantized-matmul and
turbo4 KV-cache hot path.

The compute lives in librie_cuda.so behind a C ABI (include/rie_cuda.h). This module is
the host-side mirror of the reference's kernel-level interface, with the same names and
argument meaning:

  reference (crates/rie-core/src/...)           here
  quant::GgmlType / ActFormat                    GgmlType / ActFormat
  tensor::Weight (+ slice_rows)                  Weight
  kernels::matmul::QuantActs::prepare            QuantActs.prepare
  kernels::matmul::{MatmulJob, matmul, matmul_multi, formats_for}
  turbo::{row_bytes_4, quantize_4, Rotation}     turbo.row_bytes_4 / quantize_4 / rotate
  model::cpu::{KvType, LayerCache, attention}    KvType / LayerCache / attention

Device memory is passed as torch CUDA tensors (or raw device pointers); torch is only the
allocator and stream plumbing. There is no CPU fallback: without the CUDA library or a
GPU every call raises.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass
from typing import Iterable, Sequence

from . import _lib
from ._lib import RcuError, RcuJob

__all__ = ["GgmlType", "ActFormat", "KvType", "Rounding", "PrefillGemm", "Context", "Weight", "QuantActs", "MatmulJob",
           "matmul", "matmul_multi", "matmul_f32_static", "formats_for", "block_sums", "quantize_weight", "LayerCache",
           "attention", "turbo", "RcuError"]


class GgmlType(enum.IntEnum):  # quant/mod.rs:15-68 (GGUF ids)
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    BF16 = 30

    @property
    def block_size(self) -> int:
        if self in (GgmlType.F32, GgmlType.F16, GgmlType.BF16):
            return 1
        return 32 if self in (GgmlType.Q4_0, GgmlType.Q4_1, GgmlType.Q5_0, GgmlType.Q5_1, GgmlType.Q8_0) else 256

    def row_bytes(self, n: int) -> int:
        return int(_lib.load().rcu_row_bytes(int(self), n))

    def act_format(self) -> "ActFormat":  # quant/mod.rs:118-124
        if self in (GgmlType.Q4_0, GgmlType.Q4_1, GgmlType.Q5_0, GgmlType.Q5_1, GgmlType.Q8_0):
            return ActFormat.Q8_0
        if self in (GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K, GgmlType.Q2_K, GgmlType.Q3_K):
            return ActFormat.Q8K
        return ActFormat.F32


class ActFormat(enum.IntFlag):  # quant/mod.rs:127-132 (as flags of the C ABI)
    F32 = 1
    Q8_0 = 2
    Q8K = 4


class KvType(enum.IntEnum):  # model/cpu.rs:12-36
    F16 = 0
    Q8_0 = 1
    Turbo4 = 2

    @staticmethod
    def parse(s: str) -> "KvType | None":
        return {"f16": KvType.F16, "q8": KvType.Q8_0, "q8_0": KvType.Q8_0, "turbo4": KvType.Turbo4,
                "tq4": KvType.Turbo4, "turbo": KvType.Turbo4}.get(s.lower())


class Rounding(enum.IntEnum):
    NEAREST_EVEN = 0  # AVX2 / NEON tiers of the reference
    HALF_AWAY = 1     # scalar tier (RIE_DISABLE=simd)


class PrefillGemm(enum.IntEnum):
    F16 = 0  # every weight type: f16-dequantized operands on the tensor cores (default)
    I8 = 1   # Q4_0: int8 MMA with the exact per-block int32 sums


def _check(ctx_ptr, status: int):
    if status != 0:
        msg = _lib.load().rcu_last_error(ctx_ptr) if ctx_ptr else b""
        raise RcuError(status, (msg or b"").decode(errors="replace"))


def _dptr(x) -> int:
    """Device address of a torch CUDA tensor (or a raw integer pointer)."""
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        if not x.is_cuda:
            raise ValueError("expected a CUDA tensor")
        if not x.is_contiguous():
            raise ValueError("expected a contiguous tensor")
        return int(x.data_ptr())
    raise TypeError(f"not a device buffer: {type(x)}")


class Context:
    """A device + stream the library issues work on (replaces the CPU ThreadPool)."""

    def __init__(self, device: int = 0, stream=None, rounding: Rounding = Rounding.NEAREST_EVEN):
        lib = _lib.load()
        self._lib = lib
        ptr = C.c_void_p()
        err = C.create_string_buffer(512)
        handle = _stream_handle(stream)
        st = lib.rcu_ctx_create(device, handle, C.byref(ptr), err, 512)
        if st != 0:
            raise RcuError(st, err.value.decode(errors="replace"))
        self.ptr = ptr
        self.device = device
        self.set_rounding(rounding)

    def set_stream(self, stream) -> None:
        _check(self.ptr, self._lib.rcu_set_stream(self.ptr, _stream_handle(stream)))

    def set_rounding(self, mode: Rounding) -> None:
        _check(self.ptr, self._lib.rcu_set_rounding(self.ptr, int(mode)))

    def set_static_weights(self, on: bool) -> None:
        """Promise that weights are never written by a kernel after upload (lets matmuls
        stream them before the previous kernel finishes)."""
        _check(self.ptr, self._lib.rcu_set_static_weights(self.ptr, int(bool(on))))

    def set_wait_limit_ms(self, ms: int) -> None:
        """Limit of the device-side waits on other ranks (the fused all-reduce)."""
        _check(self.ptr, self._lib.rcu_set_wait_limit_ms(self.ptr, int(ms)))

    def set_prefill_gemm(self, kind: "PrefillGemm") -> None:
        _check(self.ptr, self._lib.rcu_set_prefill_gemm(self.ptr, int(kind)))

    def sync(self) -> None:
        _check(self.ptr, self._lib.rcu_sync(self.ptr))

    def device_error_bits(self) -> int:
        bits = C.c_uint32(0)
        st = self._lib.rcu_check_device(self.ptr, C.byref(bits))
        if st not in (0, _lib.RCU_ERR_TIMEOUT):
            _check(self.ptr, st)
        return int(bits.value)

    def close(self) -> None:
        if getattr(self, "ptr", None):
            self._lib.rcu_ctx_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _stream_handle(stream) -> C.c_void_p:
    if stream is None:
        return C.c_void_p(0)
    if isinstance(stream, int):
        return C.c_void_p(stream)
    return C.c_void_p(int(stream.cuda_stream))


class Weight:
    """A rows x cols weight in GGUF block layout on the device (tensor.rs:6-98)."""

    def __init__(self, ctx: Context, ptr: C.c_void_p, ty: GgmlType, rows: int, cols: int, keep=None):
        self.ctx, self.ptr, self.ty, self.rows, self.cols = ctx, ptr, GgmlType(ty), rows, cols
        self._keep = keep

    @classmethod
    def upload(cls, ctx: Context, ty: GgmlType, rows: int, cols: int, data) -> "Weight":
        """Copy raw GGUF block bytes (bytes / numpy uint8 array) to the device."""
        import numpy as np
        buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray))
                                   else np.asarray(data, dtype=np.uint8))
        if buf.size != rows * GgmlType(ty).row_bytes(cols):
            raise ValueError("weight size mismatch")
        ptr = C.c_void_p()
        _check(ctx.ptr, ctx._lib.rcu_weight_upload(ctx.ptr, int(ty), rows, cols, buf.ctypes.data_as(C.c_void_p),
                                                   C.byref(ptr)))
        return cls(ctx, ptr, ty, rows, cols)

    @classmethod
    def view(cls, ctx: Context, ty: GgmlType, rows: int, cols: int, dev) -> "Weight":
        """Zero-copy view of GGUF bytes already on the device (16-byte aligned)."""
        ptr = C.c_void_p()
        _check(ctx.ptr, ctx._lib.rcu_weight_view(ctx.ptr, int(ty), rows, cols, C.c_void_p(_dptr(dev)), C.byref(ptr)))
        return cls(ctx, ptr, ty, rows, cols, keep=dev)

    def slice_rows(self, start: int, n: int) -> "Weight":
        ptr = C.c_void_p()
        _check(self.ctx.ptr, self.ctx._lib.rcu_weight_slice_rows(self.ptr, start, n, C.byref(ptr)))
        return Weight(self.ctx, ptr, self.ty, n, self.cols, keep=self)

    @property
    def row_bytes(self) -> int:
        return self.ty.row_bytes(self.cols)

    def data_ptr(self) -> int:
        return int(self.ctx._lib.rcu_weight_device_ptr(self.ptr) or 0)

    def free(self) -> None:
        if getattr(self, "ptr", None):
            self.ctx._lib.rcu_weight_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def formats_for(ws: Iterable[Weight]) -> ActFormat:  # matmul.rs:119-128
    f = ActFormat(0)
    for w in ws:
        f |= w.ty.act_format()
    return f


class QuantActs:
    """One batch of quantized activations on the device (matmul.rs:19-97)."""

    def __init__(self, ctx: Context, max_tok: int, max_k: int):
        self.ctx = ctx
        self.ptr = C.c_void_p()
        _check(ctx.ptr, ctx._lib.rcu_acts_create(ctx.ptr, max_tok, max_k, C.byref(self.ptr)))
        self.n_tok = 0
        self.k = 0

    def prepare(self, x, n_tok: int, k: int, formats: ActFormat) -> None:
        """Quantize x (n_tok x k f32, device) once into every format in `formats`."""
        fl = int(formats) & ~int(ActFormat.F32)
        _check(self.ctx.ptr, self.ctx._lib.rcu_acts_prepare(self.ctx.ptr, self.ptr, C.c_void_p(_dptr(x)), n_tok, k, fl))
        self.n_tok, self.k = n_tok, k

    def export(self, fmt: ActFormat):
        """Blocks in the reference's layout (BlockQ8_0: 48 B, BlockQ8K: 304 B) as numpy bytes."""
        import numpy as np
        bs, sz = (32, 48) if fmt == ActFormat.Q8_0 else (256, 304)
        out = np.zeros(self.n_tok * (self.k // bs) * sz, dtype=np.uint8)
        _check(self.ctx.ptr, self.ctx._lib.rcu_acts_export(self.ctx.ptr, self.ptr, int(fmt),
                                                           out.ctypes.data_as(C.c_void_p)))
        return out

    def free(self) -> None:
        if getattr(self, "ptr", None):
            self.ctx._lib.rcu_acts_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class MatmulJob:  # matmul.rs:110-116
    w: Weight
    out: object  # device tensor / pointer: out[t * ld + r]
    ld: int | None = None


def matmul_multi(ctx: Context, acts: QuantActs, jobs: Sequence[MatmulJob]) -> None:
    """Several matmuls sharing one activation batch, in one launch (matmul.rs:136-176)."""
    arr = (RcuJob * len(jobs))()
    for i, j in enumerate(jobs):
        arr[i].w = j.w.ptr.value
        arr[i].out = _dptr(j.out)
        arr[i].ld = j.ld if j.ld is not None else j.w.rows
    _check(ctx.ptr, ctx._lib.rcu_matmul_multi(ctx.ptr, acts.ptr, arr, len(jobs)))


def matmul(ctx: Context, acts: QuantActs, w: Weight, out) -> None:  # matmul.rs:130-133
    matmul_multi(ctx, acts, [MatmulJob(w, out, w.rows)])


def matmul_f32_static(ctx: Context, w: Weight, x, n_tok: int, out, ld: int | None = None) -> None:
    """W . X for f32 activations without allocating device memory.

    For callers that cannot cudaMalloc when they run a matmul (their device memory belongs
    to a pool such as PyTorch's caching allocator, or allocation would stall a decode step):
    the activations are quantized into a fixed scratch area inside the library. At most 8
    tokens and rows of at most 16384 values; calls that overlap on the GPU share that
    scratch and must not run concurrently."""
    _check(ctx.ptr, ctx._lib.rcu_matmul_f32_static(ctx.ptr, w.ptr, C.c_void_p(_dptr(x)), n_tok,
                                                   C.c_void_p(_dptr(out)), w.rows if ld is None else ld))


def quantize_weight(ctx: Context, ty: GgmlType, rows: int, cols: int, x, out, ld: int | None = None) -> None:
    """f32 weights (rows x cols, row stride ld, device) -> GGUF blocks of `ty` in `out` (device,
    rows x row_bytes(cols) bytes). Q8_0 / Q4_0 follow the reference's quantizers
    (quant/mod.rs:262-307); the other block types use this library's own rules."""
    _check(ctx.ptr, ctx._lib.rcu_quantize_weight(ctx.ptr, int(ty), rows, cols, C.c_void_p(_dptr(x)),
                                                 cols if ld is None else ld, C.c_void_p(_dptr(out))))


def block_sums(ctx: Context, acts: QuantActs, w: Weight, row: int, tok: int, out) -> None:
    """Exact per-block int32 sums of W[row] . X[tok] into a device int32 buffer."""
    _check(ctx.ptr, ctx._lib.rcu_block_sums(ctx.ptr, acts.ptr, w.ptr, row, tok, C.c_void_p(_dptr(out))))


def matmul_block_sums(ctx: Context, acts: QuantActs, w: Weight, out, sums, kernel: int) -> None:
    """Row 0 of acts times every row of w on the named GEMV (0: lane kernel, 1: tensor-core
    kernel), f32 results in `out` and the exact per-block int32 sums that kernel formed in
    `sums` (rows x blocks per row, the block_sums layout; device buffers)."""
    _check(ctx.ptr, ctx._lib.rcu_matmul_block_sums(ctx.ptr, acts.ptr, w.ptr, C.c_void_p(_dptr(out)),
                                                   C.c_void_p(_dptr(sums)), int(kernel)))


class LayerCache:
    """One layer's KV cache, layout [kv_head][slot][row] (model/cpu.rs:38-50)."""

    def __init__(self, ctx: Context, ty: KvType, n_head_kv: int, head_dim: int, slots: int):
        self.ctx, self.ty, self.n_head_kv, self.head_dim, self.slots = ctx, KvType(ty), n_head_kv, head_dim, slots
        self.ptr = C.c_void_p()
        _check(ctx.ptr, ctx._lib.rcu_kv_create(ctx.ptr, int(ty), n_head_kv, head_dim, slots, C.byref(self.ptr)))

    @property
    def row_bytes(self) -> int:
        if self.ty == KvType.F16:
            return 2 * self.head_dim
        if self.ty == KvType.Q8_0:
            return self.head_dim // 32 * 34
        return turbo.row_bytes_4(self.head_dim)

    def store(self, k, v, n_tok: int, pos0: int) -> None:
        """Append n_tok tokens' keys/values (n_tok x n_head_kv*head_dim f32, device)."""
        _check(self.ctx.ptr, self.ctx._lib.rcu_kv_store(self.ctx.ptr, self.ptr, C.c_void_p(_dptr(k)),
                                                        C.c_void_p(_dptr(v)), n_tok, pos0))

    def export(self):
        import numpy as np
        n = self.n_head_kv * self.slots * self.row_bytes
        k = np.zeros(n, dtype=np.uint8)
        v = np.zeros(n, dtype=np.uint8)
        _check(self.ctx.ptr, self.ctx._lib.rcu_kv_export(self.ctx.ptr, self.ptr, k.ctypes.data_as(C.c_void_p),
                                                         v.ctypes.data_as(C.c_void_p)))
        return k.reshape(self.n_head_kv * self.slots, -1), v.reshape(self.n_head_kv * self.slots, -1)

    def import_(self, k, v) -> None:
        import numpy as np
        k = np.ascontiguousarray(k, dtype=np.uint8)
        v = np.ascontiguousarray(v, dtype=np.uint8)
        _check(self.ctx.ptr, self.ctx._lib.rcu_kv_import(self.ctx.ptr, self.ptr, k.ctypes.data_as(C.c_void_p),
                                                         v.ctypes.data_as(C.c_void_p)))

    def free(self) -> None:
        if getattr(self, "ptr", None):
            self.ctx._lib.rcu_kv_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def attention(ctx: Context, cache: LayerCache, q, n_tok: int, n_head: int, pos0: int, out, window: int = 0,
              softcap: float | None = None) -> None:
    """Causal GQA attention over the cache (model/cpu.rs:552-634); q already x attn_scale."""
    _check(ctx.ptr, ctx._lib.rcu_attention(ctx.ptr, cache.ptr, C.c_void_p(_dptr(q)), n_tok, n_head, pos0, window,
                                           float(softcap or 0.0), C.c_void_p(_dptr(out))))


class turbo:  # noqa: N801  (namespace mirroring turbo.rs)
    KV_SEED = 0x7542_6F51_7561_6E74

    @staticmethod
    def row_bytes_4(d: int) -> int:
        return int(_lib.load().rcu_turbo4_row_bytes(d))

    @staticmethod
    def quantize_4(ctx: Context, x, n_rows: int, d: int, out) -> None:
        """Rotate + 4-bit encode n_rows rows of d f32 (device) into reference-format rows."""
        _check(ctx.ptr, ctx._lib.rcu_turbo4_quantize(ctx.ptr, C.c_void_p(_dptr(x)), n_rows, d, C.c_void_p(_dptr(out))))

    @staticmethod
    def rotate(ctx: Context, x, n_rows: int, d: int, inverse: bool = False) -> None:
        _check(ctx.ptr, ctx._lib.rcu_turbo4_rotate(ctx.ptr, C.c_void_p(_dptr(x)), n_rows, d, int(inverse)))
