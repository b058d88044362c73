"""ctypes binding of the CPU oracle. TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py``, always as the checker or the timed CPU baseline, never on the product path.

* :func:`attention` runs ``oracle_attention_slices`` from ``attention_oracle.c``, the C
  restatement of the reference's ``ReferenceAttention`` (ROCmKernels.Tests/AttentionTests.cpp:28-125).
* :func:`reference_attention` runs the reference's own function, compiled from the reference
  tree into ``oracle/_ref/libref_attention.so`` (only present where the reference was available
  at build time); :func:`reference_available` says whether it is.
* :func:`uniform`, :func:`normal`, :func:`lengths` reproduce the reference's seeded inputs
  (``std::mt19937`` + libstdc++ distributions; TestSupport.hpp:11-21).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIBRARY = ORACLE_DIR / "_build" / "liboracle_attention.so"
REFERENCE_LIBRARY = ORACLE_DIR / "_ref" / "libref_attention.so"
REFERENCE_TESTS = ORACLE_DIR / "_ref" / "attention_tests"
REFERENCE_BENCH = ORACLE_DIR / "_ref" / "attention_bench"
REFERENCE_GENERIC_TESTS = ORACLE_DIR / "_ref" / "generic_tests"
REFERENCE_POSITIONAL_LIBRARY = ORACLE_DIR / "_ref" / "libref_positional.so"
REFERENCE_POSITIONAL_TESTS = ORACLE_DIR / "_ref" / "positional_tests"
REFERENCE_ROTARY_BENCH = ORACLE_DIR / "_ref" / "rotary_bench"
REFERENCE_GENERIC_BENCH = ORACLE_DIR / "_ref" / "generic_bench"

_F32 = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_U8 = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_I32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_U32 = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")

_oracle = None
_reference = None


def build() -> None:
    """Builds the C restatement (make -C oracle oracle)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "oracle"], check=True)


def _load_oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_LIBRARY.exists():
            build()
        lib = ctypes.CDLL(str(ORACLE_LIBRARY))
        lib.oracle_attention_slices.argtypes = [_F32, _F32, _F32, _U8, ctypes.c_void_p] + [ctypes.c_int] * 6 + \
            [_F32, _F32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5
        lib.oracle_attention_slices.restype = ctypes.c_int
        lib.oracle_uniform_fill.argtypes = [_F32, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float, ctypes.c_float]
        lib.oracle_normal_fill.argtypes = [_F32, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_float, ctypes.c_float]
        lib.oracle_mt19937_raw.argtypes = [_U32, ctypes.c_size_t, ctypes.c_uint32]
        lib.oracle_lengths.argtypes = [_I32, ctypes.c_int, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32]
        lib.oracle_rotary.argtypes = [_F32, _F32, _F32, _F32] + [ctypes.c_int] * 4
        lib.oracle_rotary.restype = None
        _oracle = lib
    return _oracle


def reference_available() -> bool:
    return REFERENCE_LIBRARY.exists()


def _load_reference() -> ctypes.CDLL:
    global _reference
    if _reference is None:
        lib = ctypes.CDLL(str(REFERENCE_LIBRARY))
        lib.ref_attention.argtypes = [_F32, _F32, _F32, _U8, _F32] + [ctypes.c_int] * 6 + [_F32] * 5
        lib.ref_attention.restype = ctypes.c_int
        lib.ref_random_values.argtypes = [_F32, ctypes.c_size_t, ctypes.c_uint, ctypes.c_float, ctypes.c_float]
        _reference = lib
    return _reference


def uniform(count: int, seed: int, low: float = -1.0, high: float = 1.0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    _load_oracle().oracle_uniform_fill(out, count, seed, low, high)
    return out


def normal(count: int, seed: int, mean: float = 0.0, stddev: float = 1.0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    _load_oracle().oracle_normal_fill(out, count, seed, mean, stddev)
    return out


def mt19937(count: int, seed: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint32)
    _load_oracle().oracle_mt19937_raw(out, count, seed)
    return out


def lengths(count: int, seed: int, low: int, high: int) -> np.ndarray:
    out = np.empty(count, dtype=np.int32)
    _load_oracle().oracle_lengths(out, count, seed, low, high)
    return out


def attention(q, k, v, mask, upstream, radius: int = -1, *, threads: int = 1, forward_only: bool = False,
              double_gradients: bool = False, slices: tuple[int, int] | None = None) -> dict:
    """Reference attention on contiguous [B, H, S, D] float32 arrays and a [B, K] uint8 mask.

    Returns dict(output, lse, grad_q, grad_k, grad_v) (gradients absent when forward_only).
    `slices` restricts the work to flattened (batch, head) slices [s0, s1); other slices of the
    outputs stay zero.
    """
    q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    B, H, Q, D = q.shape
    K = k.shape[2]
    out = {"output": np.zeros_like(q), "lse": np.zeros((B, H, Q, 2), np.float32)}
    if not forward_only:
        upstream = np.ascontiguousarray(upstream, dtype=np.float32)
        out.update(grad_q=np.zeros_like(q), grad_k=np.zeros_like(k), grad_v=np.zeros_like(v))
    s0, s1 = slices if slices is not None else (0, B * H)

    def address(name):
        return None if forward_only else out[name].ctypes.data

    status = _load_oracle().oracle_attention_slices(
        q, k, v, mask, None if forward_only else upstream.ctypes.data, D, B, H, Q, K, radius, out["output"], out["lse"],
        address("grad_q"), address("grad_k"), address("grad_v"), s0, s1, threads, int(forward_only), int(double_gradients))
    if status != 0:
        raise ValueError("oracle_attention_slices rejected its arguments")
    return out


def reference_attention(q, k, v, mask, upstream, radius: int = -1) -> dict:
    """The reference's own ReferenceAttention (compiled from its source), same contract as attention()."""
    q, k, v, upstream = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v, upstream))
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    B, H, Q, D = q.shape
    K = k.shape[2]
    out = {"output": np.zeros_like(q), "lse": np.zeros((B, H, Q, 2), np.float32), "grad_q": np.zeros_like(q),
           "grad_k": np.zeros_like(k), "grad_v": np.zeros_like(v)}
    _load_reference().ref_attention(q, k, v, mask, upstream, D, B, H, Q, K, radius, out["output"], out["lse"],
                                    out["grad_q"], out["grad_k"], out["grad_v"])
    return out


def reference_random_values(count: int, seed: int, low: float = -1.0, high: float = 1.0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    _load_reference().ref_random_values(out, count, seed, low, high)
    return out


def rotary(x, cos, sin, backward: bool = False) -> np.ndarray:
    """The reference's ReferenceRotary (PositionalTests.cpp:18-50) restated in attention_oracle.c:
    x token-major [B, L, H, 32], cos/sin [B, L, 32] float32; returns the rotated [B, L, H, 32]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    cos, sin = (np.ascontiguousarray(t, dtype=np.float32) for t in (cos, sin))
    B, L, H, W = x.shape
    if W != 32 or cos.shape != (B, L, 32) or sin.shape != (B, L, 32):
        raise ValueError("rotary expects x [B, L, H, 32] and tables [B, L, 32]")
    out = np.empty_like(x)
    _load_oracle().oracle_rotary(x, cos, sin, out, B, H, L, int(backward))
    return out


_positional = None


def reference_positional_available() -> bool:
    return REFERENCE_POSITIONAL_LIBRARY.exists()


def reference_rotary(x, cos, sin, backward: bool = False) -> np.ndarray:
    """The reference's own ReferenceRotary, compiled from its source (same contract as rotary())."""
    global _positional
    if _positional is None:
        lib = ctypes.CDLL(str(REFERENCE_POSITIONAL_LIBRARY))
        lib.ref_rotary.argtypes = [_F32, _F32, _F32, _F32] + [ctypes.c_int] * 4
        lib.ref_rotary.restype = None
        _positional = lib
    x = np.ascontiguousarray(x, dtype=np.float32)
    cos, sin = (np.ascontiguousarray(t, dtype=np.float32) for t in (cos, sin))
    B, L, H, _ = x.shape
    out = np.empty_like(x)
    _positional.ref_rotary(x, cos, sin, out, B, H, L, int(backward))
    return out


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
