"""ctypes bindings for the oracle libraries.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline / reference arm, never by the product package.

Two libraries sit behind this module:

* ``_build/libmrt_oracle.so`` -- this repository's C restatement of the
  reference arithmetic (``mrt_oracle.c``; every function cites the reference
  file:line it follows).
* ``_ref/libmrt_ref.so`` -- the reference's own ``CpuBackend::gemm`` and dtype
  converters compiled from its sources (``Makefile``), used to pin the
  restatement and as the timed CPU baseline.

Arrays are numpy; FP16/BF16 data travel as ``uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmrt_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmrt_ref.so")

FP16, BF16, FP32 = 0, 1, 2
_NP_OF = {FP16: np.uint16, BF16: np.uint16, FP32: np.float32}

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")

_oracle = None
_ref = None


def _ptr(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def oracle_lib() -> C.CDLL:
    """Load the C restatement (built by ``make -C oracle``)."""
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle`")
        lib = C.CDLL(ORACLE_SO)
        lib.orc_f32_to_f16.restype = C.c_uint16
        lib.orc_f32_to_f16.argtypes = [C.c_float]
        lib.orc_f16_to_f32.restype = C.c_float
        lib.orc_f16_to_f32.argtypes = [C.c_uint16]
        for name, a, b in (("orc_f32_to_f16_n", _f32p, _u16p), ("orc_f16_to_f32_n", _u16p, _f32p),
                           ("orc_f32_to_bf16_n", _f32p, _u16p), ("orc_bf16_to_f16_n", _u16p, _u16p)):
            fn = getattr(lib, name)
            fn.restype = None
            fn.argtypes = [a, b, C.c_size_t]
        lib.orc_gemm.restype = C.c_int
        lib.orc_gemm.argtypes = [C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                 C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                 C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                 C.c_float, C.c_float, C.c_int, C.c_int, C.c_size_t, C.c_size_t]
        lib.orc_gemm_f64.restype = None
        lib.orc_gemm_f64.argtypes = [_u16p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_int,
                                     C.c_size_t, _f64p]
        lib.orc_add_bias_f16.restype = None
        lib.orc_add_bias_f16.argtypes = [_u16p, _u16p, C.c_size_t, C.c_size_t]
        lib.orc_add_f16.restype = None
        lib.orc_add_f16.argtypes = [_u16p, _u16p, _u16p, C.c_size_t]
        lib.orc_argmax_f16.restype = C.c_int64
        lib.orc_argmax_f16.argtypes = [_u16p, C.c_size_t]
        lib.orc_rel_frobenius_f16.restype = C.c_double
        lib.orc_rel_frobenius_f16.argtypes = [_u16p, _f64p, C.c_size_t]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> C.CDLL:
    """Load the reference's own CPU code (built by ``make -C oracle`` where the
    reference sources are present; the built file travels with the repo)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle` with the reference present")
        lib = C.CDLL(REF_SO)
        lib.refb_create.restype = C.c_void_p
        lib.refb_create.argtypes = [C.c_size_t]
        lib.refb_destroy.restype = None
        lib.refb_destroy.argtypes = [C.c_void_p]
        lib.refb_gemm.restype = C.c_int
        lib.refb_gemm.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                  C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                  C.c_void_p, C.c_int, C.c_size_t, C.c_size_t,
                                  C.c_float, C.c_float, C.c_int, C.c_int]
        for name, a, b in (("refb_f32_to_f16_n", _f32p, _u16p), ("refb_f16_to_f32_n", _u16p, _f32p),
                           ("refb_f32_to_bf16_n", _f32p, _u16p), ("refb_bf16_to_f32_n", _u16p, _f32p)):
            fn = getattr(lib, name)
            fn.restype = None
            fn.argtypes = [a, b, C.c_size_t]
        lib.refb_add_bias.restype = None
        lib.refb_add_bias.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_size_t, C.c_size_t]
        lib.refb_add.restype = None
        lib.refb_add.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]
        lib.refb_argmax.restype = C.c_int64
        lib.refb_argmax.argtypes = [C.c_void_p, C.c_int, C.c_size_t]
        _ref = lib
    return _ref


# --------------------------------------------------------------------------
# converters
# --------------------------------------------------------------------------

def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    oracle_lib().orc_f32_to_f16_n(x.reshape(-1), out.reshape(-1), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    oracle_lib().orc_f16_to_f32_n(h.reshape(-1), out.reshape(-1), h.size)
    return out


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    oracle_lib().orc_f32_to_bf16_n(x.reshape(-1), out.reshape(-1), x.size)
    return out


def bf16_to_f16(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, np.uint16)
    oracle_lib().orc_bf16_to_f16_n(b.reshape(-1), out.reshape(-1), b.size)
    return out


def ref_f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    ref_lib().refb_f32_to_f16_n(x.reshape(-1), out.reshape(-1), x.size)
    return out


def ref_f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    ref_lib().refb_f16_to_f32_n(h.reshape(-1), out.reshape(-1), h.size)
    return out


def ref_f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    ref_lib().refb_f32_to_bf16_n(x.reshape(-1), out.reshape(-1), x.size)
    return out


# --------------------------------------------------------------------------
# gemm
# --------------------------------------------------------------------------

def gemm(A: np.ndarray, a_dtype: int, B: np.ndarray, b_dtype: int, c_dtype: int = FP16,
         alpha: float = 1.0, beta: float = 0.0, trans_a: bool = False, trans_b: bool = False,
         C0: np.ndarray | None = None, rows: tuple[int, int] | None = None) -> np.ndarray:
    """Oracle restatement of ``CpuBackend::gemm`` (cpu_backend.cpp:72-169).

    ``rows=(m0, m1)`` computes only those output rows; the others are left as
    in ``C0`` (zeros by default)."""
    A = np.ascontiguousarray(A)
    B = np.ascontiguousarray(B)
    a_rows, a_cols = A.shape
    b_rows, b_cols = B.shape
    M = a_cols if trans_a else a_rows
    N = b_rows if trans_b else b_cols
    Cm = np.zeros((M, N), _NP_OF[c_dtype]) if C0 is None else np.array(C0, dtype=_NP_OF[c_dtype], copy=True)
    m0, m1 = rows if rows is not None else (0, M)
    rc = oracle_lib().orc_gemm(_ptr(A), a_dtype, a_rows, a_cols, _ptr(B), b_dtype, b_rows, b_cols,
                               _ptr(Cm), c_dtype, M, N, alpha, beta, int(trans_a), int(trans_b), m0, m1)
    if rc != 0:
        raise ValueError("oracle gemm: shape mismatch")
    return Cm


class RefBackend:
    """The reference's own ``CpuBackend`` (compiled from its sources)."""

    def __init__(self, threads: int = 0):
        self.lib = ref_lib()
        self.h = self.lib.refb_create(threads)

    def close(self):
        if self.h:
            self.lib.refb_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def gemm(self, A: np.ndarray, a_dtype: int, B: np.ndarray, b_dtype: int, c_dtype: int = FP16,
             alpha: float = 1.0, beta: float = 0.0, trans_a: bool = False, trans_b: bool = False,
             C0: np.ndarray | None = None, out: np.ndarray | None = None) -> np.ndarray:
        A = np.ascontiguousarray(A)
        B = np.ascontiguousarray(B)
        a_rows, a_cols = A.shape
        b_rows, b_cols = B.shape
        M = a_cols if trans_a else a_rows
        N = b_rows if trans_b else b_cols
        if out is not None:
            Cm = out
        else:
            Cm = np.zeros((M, N), _NP_OF[c_dtype]) if C0 is None else np.array(C0, dtype=_NP_OF[c_dtype], copy=True)
        rc = self.lib.refb_gemm(self.h, _ptr(A), a_dtype, a_rows, a_cols, _ptr(B), b_dtype, b_rows, b_cols,
                                _ptr(Cm), c_dtype, M, N, alpha, beta, int(trans_a), int(trans_b))
        if rc != 0:
            raise ValueError("reference gemm: shape mismatch")
        return Cm


def ref_add_bias(out_f16: np.ndarray, bias_f16: np.ndarray) -> np.ndarray:
    out = np.array(out_f16, dtype=np.uint16, copy=True)
    rows = out.size // bias_f16.size
    ref_lib().refb_add_bias(_ptr(out), FP16, _ptr(np.ascontiguousarray(bias_f16, np.uint16)), FP16,
                            rows, bias_f16.size)
    return out


def ref_add(a_f16: np.ndarray, b_f16: np.ndarray, threads: int = 1) -> np.ndarray:
    """The reference's CpuBackend::add on two FP16 arrays of one shape."""
    a = np.ascontiguousarray(a_f16, np.uint16)
    b = np.ascontiguousarray(b_f16, np.uint16)
    assert a.shape == b.shape
    out = np.empty_like(a)
    lib = ref_lib()
    be = lib.refb_create(threads)
    try:
        lib.refb_add(be, _ptr(a), _ptr(b), _ptr(out), a.size)
    finally:
        lib.refb_destroy(be)
    return out


def ref_argmax(logits_f16: np.ndarray) -> int:
    row = np.ascontiguousarray(logits_f16, dtype=np.uint16)
    return int(ref_lib().refb_argmax(_ptr(row), FP16, row.size))


def add_bias(out_f16: np.ndarray, bias_f16: np.ndarray) -> np.ndarray:
    out = np.array(out_f16, dtype=np.uint16, copy=True)
    rows = out.size // bias_f16.size
    oracle_lib().orc_add_bias_f16(out.reshape(-1), np.ascontiguousarray(bias_f16, np.uint16), rows,
                                  bias_f16.size)
    return out


def add(a_f16: np.ndarray, b_f16: np.ndarray) -> np.ndarray:
    """Element-wise FP16 add with the reference's rounding (orc_add_f16)."""
    a = np.ascontiguousarray(a_f16, np.uint16)
    b = np.ascontiguousarray(b_f16, np.uint16)
    assert a.shape == b.shape
    out = np.empty_like(a)
    oracle_lib().orc_add_f16(a.reshape(-1), b.reshape(-1), out.reshape(-1), a.size)
    return out


def argmax(logits_f16: np.ndarray) -> int:
    row = np.ascontiguousarray(logits_f16, dtype=np.uint16).reshape(-1)
    return int(oracle_lib().orc_argmax_f16(row, row.size))


def gemm_f64(X_f16: np.ndarray, W: np.ndarray, w_dtype: int) -> np.ndarray:
    """FP64 ground truth of X * W^T (X FP16 [M,K], W [N,K])."""
    X = np.ascontiguousarray(X_f16, np.uint16)
    W = np.ascontiguousarray(W)
    M, K = X.shape
    N = W.shape[0]
    Y = np.empty((M, N), np.float64)
    oracle_lib().orc_gemm_f64(X, M, K, _ptr(W), w_dtype, N, Y)
    return Y


def rel_frobenius(got_f16: np.ndarray, want_f64: np.ndarray) -> float:
    g = np.ascontiguousarray(got_f16, np.uint16).reshape(-1)
    w = np.ascontiguousarray(want_f64, np.float64).reshape(-1)
    return float(oracle_lib().orc_rel_frobenius_f16(g, w, g.size))
