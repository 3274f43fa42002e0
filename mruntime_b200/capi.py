"""ctypes binding of the C ABI in include/mrt_b200.h.

This is the Python caller of the same entry points a C++ or cgo host binds;
the tests and bench.py go through it.  Device buffers are passed as raw
pointers (``tensor.data_ptr()`` of a torch CUDA tensor works), streams as
``cudaStream_t`` values (``torch.cuda.current_stream().cuda_stream``).

Every failing call raises :class:`MrtError` with the library's message.  The
library must have been built (``python -m mruntime_b200.build``); there is no
fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from . import build as _build

LIB_PATH = _build.LIB
HEADER = os.path.join(_build.INCLUDE, "mrt_b200.h")

MRT_OK = 0
MRT_ERR_TIMEOUT = 6
FP16, BF16, FP32 = 0, 1, 2
GEMM_BIAS = 1

_lib: C.CDLL | None = None


class MrtError(RuntimeError):
    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def header_functions() -> list[str]:
    """Names of every entry point declared in include/mrt_b200.h."""
    text = open(HEADER).read()
    return re.findall(r"^\s*(?:int|void|const char\*)\s+(mrt_\w+)\s*\(", text, flags=re.M)


_vp, _i64, _int, _u32, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_uint, C.c_size_t
_SIGS = {
    "mrt_version": (_int, []),
    "mrt_init": (_int, [_int]),
    "mrt_last_error_string": (C.c_char_p, []),
    "mrt_sync": (_int, [_vp]),
    "mrt_reserve_workspace": (_int, [_sz]),
    "mrt_device_sm_count": (_int, [C.POINTER(_int)]),
    "mrt_launch_count": (_int, [C.POINTER(_i64)]),
    "mrt_selftest_wait_timeout": (_int, [_int, _vp]),
    "mrt_weight_upload": (_int, [_vp, _int, _int, _i64, _i64, C.POINTER(_i64), _i64, _i64, _i64, _vp,
                                 C.POINTER(_vp)]),
    "mrt_weight_attach_bias": (_int, [_vp, _vp, _int, _int, _vp]),
    "mrt_weight_free": (_int, [_vp]),
    "mrt_weight_view": (_int, [_vp, _i64, _i64, C.POINTER(_vp)]),
    "mrt_device_alloc": (_int, [_sz, C.POINTER(_vp)]),
    "mrt_device_free": (_int, [_vp]),
    "mrt_memcpy": (_int, [_vp, _vp, _sz, _vp]),
    "mrt_pointer_kind": (_int, [_vp, C.POINTER(_int)]),
    "mrt_weight_shape": (_int, [_vp, C.POINTER(_i64), C.POINTER(_i64)]),
    "mrt_weight_data": (_int, [_vp, C.POINTER(_vp), C.POINTER(_int)]),
    "mrt_weight_read": (_int, [_vp, _vp, _i64, _vp]),
    "mrt_gemm": (_int, [_vp, _vp, _i64, _vp, _i64, _i64, _u32, _vp]),
    "mrt_gemm_f32": (_int, [_vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "mrt_gemm_swiglu": (_int, [_vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "mrt_gemm_residual": (_int, [_vp, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _u32, _vp]),
    "mrt_tp_p2p_init": (_int, [_vp, _i64]),
    "mrt_tp_p2p_buffers": (_int, [_vp, C.POINTER(_vp), C.POINTER(_vp)]),
    "mrt_tp_p2p_allreduce_f32_to_f16": (_int, [_vp, _i64, _vp, _i64, _i64, _vp]),
    "mrt_tp_gemm_rowpar": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _i64, _vp]),
    "mrt_gemm_plan": (_int, [_i64, _i64, _i64, _int] + [C.POINTER(_int)] * 6),
    "mrt_gemm_host": (_int, [_vp, _vp, _vp, _i64, _u32, _vp]),
    "mrt_gemm_host_async": (_int, [_vp, _vp, _vp, _i64, _u32, _vp]),
    "mrt_gemm_general": (_int, [_vp, _int, _i64, _i64, _vp, _int, _i64, _i64, _vp, _int, C.c_float, C.c_float,
                                _int, _int, _vp]),
    "mrt_argmax_f16": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mrt_argmax_f16_noalloc": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mrt_lm_head_argmax": (_int, [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "mrt_convert": (_int, [_vp, _int, _vp, _int, _i64, _vp]),
    "mrt_rmsnorm": (_int, [_vp, _int, _vp, _int, _vp, _int, _i64, _i64, C.c_float, _vp]),
    "mrt_rope": (_int, [_vp, _int, _i64, _i64, _i64, _i64, _i64, C.c_float, _vp]),
    "mrt_silu": (_int, [_vp, _int, _vp, _int, _i64, _vp]),
    "mrt_mul": (_int, [_vp, _int, _vp, _int, _vp, _int, _i64, _vp]),
    "mrt_add": (_int, [_vp, _int, _vp, _int, _vp, _int, _i64, _vp]),
    "mrt_softmax": (_int, [_vp, _int, _vp, _int, _i64, _i64, _i64, _vp]),
    "mrt_embedding": (_int, [_vp, _int, _i64, _i64, _vp, _i64, _vp, _int, _vp]),
    "mrt_attention": (_int, [_vp, _int, C.POINTER(_i64), _vp, _int, C.POINTER(_i64), _vp, _int, C.POINTER(_i64),
                             _vp, _int, C.POINTER(_i64), _i64, _i64, _i64, _i64, _i64, _i64, C.c_float, _int, _vp]),
    "mrt_shard_rows": (_int, [C.POINTER(_i64), _i64, _int, _int, C.POINTER(_i64)]),
    "mrt_shard_cols": (_int, [_i64, _int, _int, C.POINTER(_i64), C.POINTER(_i64)]),
    "mrt_tp_unique_id": (_int, [_vp, _sz]),
    "mrt_tp_init": (_int, [_int, _int, _vp, _sz, C.POINTER(_vp)]),
    "mrt_tp_destroy": (_int, [_vp]),
    "mrt_tp_allreduce_f32_to_f16": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "mrt_tp_allgather_cols_f16": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "mrt_tp_argmax": (_int, [_vp, _vp, _vp, _i64, _vp, _vp]),
    "mrt_decoder_create": (_int, [_vp, C.POINTER(_vp)]),
    "mrt_decoder_create_tp": (_int, [_vp, _vp, C.POINTER(_vp)]),
    "mrt_decoder_load": (_int, [_vp, C.c_char_p, _vp, _int, _int, _i64, _i64]),
    "mrt_decoder_generate": (_int, [_vp, _vp, _i64, _i64, C.c_int32, _vp, C.POINTER(_i64), _vp, _vp]),
    "mrt_decoder_free": (None, [_vp]),
    "mrt_safetensors_open": (_int, [C.c_char_p, C.POINTER(_vp)]),
    "mrt_safetensors_close": (_int, [_vp]),
    "mrt_safetensors_count": (_int, [_vp, C.POINTER(_i64)]),
    "mrt_safetensors_name": (_int, [_vp, _i64, C.POINTER(C.c_char_p)]),
    "mrt_safetensors_info": (_int, [_vp, C.c_char_p, C.POINTER(_int), C.POINTER(_int), C.POINTER(_i64),
                                    C.POINTER(C.c_uint64)]),
    "mrt_safetensors_read": (_int, [_vp, C.c_char_p, _vp, C.c_uint64, _vp]),
    "mrt_safetensors_upload_weight": (_int, [_vp, C.c_char_p, C.POINTER(_i64), _i64, _i64, _i64, _vp,
                                             C.POINTER(_vp)]),
    "mrt_decoder_load_safetensors": (_int, [_vp, _vp, C.POINTER(_i64)]),
}


def lib() -> C.CDLL:
    """Load libmrt_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `python -m mruntime_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int, fn: str) -> None:
    if rc != MRT_OK:
        msg = lib().mrt_last_error_string()
        raise MrtError(rc, fn, msg.decode() if msg else "")


def call(fn: str, *args) -> None:
    """Call an entry point and raise MrtError on a non-zero status."""
    _check(getattr(lib(), fn)(*args), fn)


def init(device: int = 0) -> None:
    call("mrt_init", device)


def sync(stream: int | None = None) -> None:
    call("mrt_sync", stream)


def launch_count() -> int:
    v = C.c_int64(0)
    call("mrt_launch_count", C.byref(v))
    return v.value


def sm_count() -> int:
    v = C.c_int(0)
    call("mrt_device_sm_count", C.byref(v))
    return v.value


class Weight:
    """An uploaded weight (or shard) -- the handle returned by mrt_weight_upload."""

    def __init__(self, src_ptr: int, src_dtype: int, src_on_device: bool, N: int, K: int,
                 row_ranges: list[tuple[int, int]] | None = None, k_range: tuple[int, int] | None = None,
                 stream: int | None = None):
        h = C.c_void_p()
        rr = None
        n_ranges = 0
        if row_ranges:
            flat = [v for pair in row_ranges for v in pair]
            rr = (C.c_int64 * len(flat))(*flat)
            n_ranges = len(row_ranges)
        k0, k1 = k_range if k_range is not None else (0, K)
        call("mrt_weight_upload", src_ptr, src_dtype, int(src_on_device), N, K, rr, n_ranges, k0, k1, stream,
             C.byref(h))
        self.h = h
        n, k = C.c_int64(), C.c_int64()
        call("mrt_weight_shape", h, C.byref(n), C.byref(k))
        self.n, self.k = n.value, k.value

    @classmethod
    def adopt(cls, h: C.c_void_p) -> "Weight":
        """Wrap a handle another entry point returned (e.g. a checkpoint upload)."""
        self = cls.__new__(cls)
        self.h = h
        n, k = C.c_int64(), C.c_int64()
        call("mrt_weight_shape", h, C.byref(n), C.byref(k))
        self.n, self.k = n.value, k.value
        return self

    def attach_bias(self, src_ptr: int, src_dtype: int, src_on_device: bool, stream: int | None = None):
        call("mrt_weight_attach_bias", self.h, src_ptr, src_dtype, int(src_on_device), stream)

    def data_ptr(self) -> int:
        """Device storage in the library's layout (see mrt_weight_data)."""
        p = C.c_void_p()
        call("mrt_weight_data", self.h, C.byref(p), None)
        return p.value

    def tiled(self) -> bool:
        p, t = C.c_void_p(), C.c_int()
        call("mrt_weight_data", self.h, C.byref(p), C.byref(t))
        return bool(t.value)

    def read(self, dst_ptr: int, ld: int | None = None, stream: int | None = None) -> None:
        """Copy the weight as row-major FP16 [n, k] to a device buffer."""
        call("mrt_weight_read", self.h, dst_ptr, self.k if ld is None else ld, stream)

    def free(self):
        if self.h:
            lib().mrt_weight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def gemm(w: Weight, x_ptr: int, ldx: int, y_ptr: int, ldy: int, M: int, bias: bool = False,
         stream: int | None = None) -> None:
    call("mrt_gemm", w.h, x_ptr, ldx, y_ptr, ldy, M, GEMM_BIAS if bias else 0, stream)


def gemm_plan(M: int, N: int, K: int, sms: int = 0) -> dict:
    """The kernel and tiling mrt_gemm picks for an M x N x K product."""
    vals = [C.c_int() for _ in range(6)]
    call("mrt_gemm_plan", M, N, K, sms, *[C.byref(v) for v in vals])
    keys = ("kernel", "bn", "full_tiles", "tail_splits", "kb_per", "grid")
    d = dict(zip(keys, (v.value for v in vals)))
    d["cluster"] = d["kernel"] == 3  # swap mode, K-slices summed inside clusters
    d["pair"] = d["kernel"] == 4  # normal mode on SM pairs (cta_group::2)
    d["kernel"] = {1: "tcgen05", 2: "tcgen05-swap", 3: "tcgen05-swap", 4: "tcgen05", 5: "gemv"}[d["kernel"]]
    return d


def gemm_f32(w: Weight, x_ptr: int, ldx: int, y_ptr: int, ldy: int, M: int, stream: int | None = None) -> None:
    call("mrt_gemm_f32", w.h, x_ptr, ldx, y_ptr, ldy, M, stream)


def gemm_swiglu(w: Weight, x_ptr: int, ldx: int, act_ptr: int, ld_act: int, M: int,
                stream: int | None = None) -> None:
    """act = fp16(silu(gate) * up) for a weight whose rows interleave gate and up."""
    call("mrt_gemm_swiglu", w.h, x_ptr, ldx, act_ptr, ld_act, M, stream)


def gemm_residual(w: Weight, x_ptr: int, ldx: int, res_ptr: int, ldr: int, y_ptr: int, ldy: int, M: int,
                  bias: bool = False, stream: int | None = None) -> None:
    """y = fp16(res + fp16(x W^T (+ bias))); y may be res."""
    call("mrt_gemm_residual", w.h, x_ptr, ldx, res_ptr, ldr, y_ptr, ldy, M, GEMM_BIAS if bias else 0, stream)


def gemm_host(w: Weight, x_host_ptr: int, y_host_ptr: int, M: int, bias: bool = False,
              stream: int | None = None) -> None:
    call("mrt_gemm_host", w.h, x_host_ptr, y_host_ptr, M, GEMM_BIAS if bias else 0, stream)


def gemm_host_async(w: Weight, x_host_ptr: int, y_host_ptr: int, M: int, bias: bool = False,
                    stream: int | None = None) -> None:
    """mrt_gemm_host without the wait (pinned buffers; valid until sync())."""
    call("mrt_gemm_host_async", w.h, x_host_ptr, y_host_ptr, M, GEMM_BIAS if bias else 0, stream)


def gemm_general(a_ptr, a_dtype, a_shape, b_ptr, b_dtype, b_shape, c_ptr, c_dtype, alpha=1.0, beta=0.0,
                 trans_a=False, trans_b=False, stream=None) -> None:
    call("mrt_gemm_general", a_ptr, a_dtype, a_shape[0], a_shape[1], b_ptr, b_dtype, b_shape[0], b_shape[1],
         c_ptr, c_dtype, alpha, beta, int(trans_a), int(trans_b), stream)


def argmax_f16(logits_ptr: int, M: int, V: int, ld: int, index_base: int, idx_ptr: int | None,
               val_ptr: int | None, stream: int | None = None) -> None:
    call("mrt_argmax_f16", logits_ptr, M, V, ld, index_base, idx_ptr, val_ptr, stream)


def lm_head_argmax(w: Weight, x_ptr: int, ldx: int, M: int, logits_ptr: int | None, index_base: int, idx_ptr: int,
                   val_ptr: int | None, stream: int | None = None) -> None:
    """Logits (unless logits_ptr is None) and the greedy pick of every row."""
    call("mrt_lm_head_argmax", w.h, x_ptr, ldx, M, logits_ptr, index_base, idx_ptr, val_ptr, stream)


def convert(src_ptr: int, src_dtype: int, dst_ptr: int, dst_dtype: int, n: int, stream: int | None = None):
    call("mrt_convert", src_ptr, src_dtype, dst_ptr, dst_dtype, n, stream)


def shard_rows(part_rows: list[int], world: int, rank: int) -> list[tuple[int, int]]:
    parts = (C.c_int64 * len(part_rows))(*part_rows)
    out = (C.c_int64 * (2 * len(part_rows)))()
    call("mrt_shard_rows", parts, len(part_rows), world, rank, out)
    return [(out[2 * i], out[2 * i + 1]) for i in range(len(part_rows))]


def shard_cols(K: int, world: int, rank: int) -> tuple[int, int]:
    k0, k1 = C.c_int64(), C.c_int64()
    call("mrt_shard_cols", K, world, rank, C.byref(k0), C.byref(k1))
    return k0.value, k1.value


class TensorParallel:
    """One rank of a tensor-parallel group (NCCL communicator inside the library)."""

    ID_BYTES = 128

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(TensorParallel.ID_BYTES)
        call("mrt_tp_unique_id", buf, TensorParallel.ID_BYTES)
        return buf.raw

    def __init__(self, rank: int, world: int, uid: bytes):
        h = C.c_void_p()
        buf = C.create_string_buffer(uid, len(uid))
        call("mrt_tp_init", rank, world, buf, len(uid), C.byref(h))
        self.h, self.rank, self.world = h, rank, world

    def allreduce_f32_to_f16(self, partial_ptr: int, out_ptr: int, count: int, stream: int | None = None):
        call("mrt_tp_allreduce_f32_to_f16", self.h, partial_ptr, out_ptr, count, stream)

    def allgather_cols_f16(self, local_ptr: int, M: int, n_local: int, out_ptr: int, stream: int | None = None):
        call("mrt_tp_allgather_cols_f16", self.h, local_ptr, M, n_local, out_ptr, stream)

    def argmax(self, val_ptr: int, idx_ptr: int, M: int, out_ptr: int, stream: int | None = None):
        call("mrt_tp_argmax", self.h, val_ptr, idx_ptr, M, out_ptr, stream)

    def p2p_init(self, max_count: int) -> None:
        """Map every rank's exchange region (collective); raises MrtError if peers cannot be mapped."""
        call("mrt_tp_p2p_init", self.h, max_count)

    def p2p_buffers(self) -> tuple[int, int]:
        """(partial, output) device pointers of this rank's exchange region."""
        part, out = C.c_void_p(), C.c_void_p()
        call("mrt_tp_p2p_buffers", self.h, C.byref(part), C.byref(out))
        return part.value, out.value

    def p2p_allreduce_f32_to_f16(self, count: int, out_ptr: int | None = None, ld_out: int = 0, row_len: int = 0,
                                 stream: int | None = None) -> None:
        call("mrt_tp_p2p_allreduce_f32_to_f16", self.h, count, out_ptr, ld_out, row_len, stream)

    def gemm_rowpar(self, w: "Weight", x_ptr: int, ldx: int, M: int, y_ptr: int, ldy: int,
                    stream: int | None = None) -> None:
        """This rank's K-shard GEMM, summed over all ranks over NVLink, rounded once to FP16 into y."""
        call("mrt_tp_gemm_rowpar", self.h, w.h, x_ptr, ldx, M, y_ptr, ldy, stream)

    def destroy(self):
        if self.h:
            lib().mrt_tp_destroy(self.h)
            self.h = None


class SafeTensors:
    """A checkpoint opened by mrt_safetensors_open (mmap + header index; the
    reference's SafeTensorsFile).  Host-only until a read or upload."""

    def __init__(self, path: str):
        h = C.c_void_p()
        call("mrt_safetensors_open", os.fsencode(path), C.byref(h))
        self.h = h

    def names(self) -> list[str]:
        n = C.c_int64()
        call("mrt_safetensors_count", self.h, C.byref(n))
        out = []
        for i in range(n.value):
            p = C.c_char_p()
            call("mrt_safetensors_name", self.h, i, C.byref(p))
            out.append(p.value.decode())
        return out

    def info(self, name: str) -> tuple[int, tuple[int, ...], int]:
        """(dtype, shape, byte size) of a tensor."""
        dt, nd, nb = C.c_int(), C.c_int(), C.c_uint64()
        shape = (C.c_int64 * 8)()
        call("mrt_safetensors_info", self.h, name.encode(), C.byref(dt), C.byref(nd), shape, C.byref(nb))
        return dt.value, tuple(shape[i] for i in range(nd.value)), nb.value

    def read(self, name: str, dst_ptr: int, dst_bytes: int, stream: int | None = None) -> None:
        call("mrt_safetensors_read", self.h, name.encode(), dst_ptr, dst_bytes, stream)

    def upload_weight(self, name: str, row_ranges=None, k_range=None, stream: int | None = None) -> "Weight":
        _, shape, _ = self.info(name)
        rr, n_ranges = None, 0
        if row_ranges:
            flat = [v for pair in row_ranges for v in pair]
            rr = (C.c_int64 * len(flat))(*flat)
            n_ranges = len(row_ranges)
        k0, k1 = k_range if k_range is not None else (0, shape[1])
        h = C.c_void_p()
        call("mrt_safetensors_upload_weight", self.h, name.encode(), rr, n_ranges, k0, k1, stream, C.byref(h))
        return Weight.adopt(h)

    def close(self):
        if self.h:
            lib().mrt_safetensors_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecoderConfig(C.Structure):
    """mrt_decoder_config (the reference's QwenConfig fields plus the KV capacity)."""

    _fields_ = [("vocab_size", C.c_int64), ("hidden_size", C.c_int64), ("num_layers", C.c_int64),
                ("num_attention_heads", C.c_int64), ("num_kv_heads", C.c_int64),
                ("intermediate_size", C.c_int64), ("max_seq_len", C.c_int64), ("rms_norm_eps", C.c_float),
                ("rope_theta", C.c_float)]


class DecoderStats(C.Structure):
    _fields_ = [("prefill_ms", C.c_float), ("first_step_ms", C.c_float), ("decode_ms", C.c_float),
                ("decode_steps", C.c_int64)]


class Decoder:
    """Device-resident greedy decoder (mrt_decoder_*): load tensors by their
    checkpoint names, then generate."""

    def __init__(self, hf_config: dict, max_seq_len: int, tp: "TensorParallel | None" = None):
        cfg = DecoderConfig(hf_config["vocab_size"], hf_config["hidden_size"], hf_config["num_hidden_layers"],
                            hf_config["num_attention_heads"], hf_config["num_key_value_heads"],
                            hf_config["intermediate_size"], max_seq_len, hf_config.get("rms_norm_eps", 1e-6),
                            hf_config.get("rope_theta", 10000.0) or 10000.0)
        h = C.c_void_p()
        if tp is None:
            call("mrt_decoder_create", C.byref(cfg), C.byref(h))
        else:
            call("mrt_decoder_create_tp", C.byref(cfg), tp.h, C.byref(h))
        self.h = h

    def load_safetensors(self, f: SafeTensors) -> int:
        """Every tensor of the checkpoint this decoder takes; returns how many."""
        n = C.c_int64()
        call("mrt_decoder_load_safetensors", self.h, f.h, C.byref(n))
        return n.value

    def load(self, name: str, ptr: int, dtype: int, on_device: bool, shape) -> None:
        rows = int(shape[0])
        cols = int(shape[1]) if len(shape) > 1 else 1
        call("mrt_decoder_load", self.h, name.encode(), ptr, dtype, int(on_device), rows, cols)

    def generate(self, prompt, max_new: int, eos: int = -1, stream: int | None = None):
        """Returns (generated ids, DecoderStats)."""
        import numpy as np

        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = C.c_int64()
        st = DecoderStats()
        call("mrt_decoder_generate", self.h, p.ctypes.data, len(p), max_new, eos, out.ctypes.data, C.byref(n),
             C.byref(st), stream)
        return out[: n.value].tolist(), st

    def free(self):
        if self.h:
            lib().mrt_decoder_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
