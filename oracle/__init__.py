"""Checkers for the sampling path -- TEST INFRASTRUCTURE ONLY.

Nothing in ``miniserve_b200`` imports this package.  ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (CPU baseline and the
``--impl reference`` arm) use it to check or time the reference algorithm.

* ``sampler_oracle``  -- float64 Python restatement of Sampler.sample
                         (miniserve/sampler.py:23-68) with boundary margins.
* ``ms_oracle.c``     -- the same steps in plain C, built into
                         ``libmsoracle.so`` by ``oracle/Makefile``; bit-identical
                         to the Python restatement on the same machine and fast
                         enough for full-size parity checks.
* ``json_oracle``     -- restatement of JSONLogitsProcessor.is_valid_prefix
                         (miniserve/sampler.py:139-148) and the token mask
                         built from it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build_c_oracle() -> str:
    """Compile ``libmsoracle.so`` in place (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "libmsoracle.so")


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libmsoracle.so")
        if not os.path.exists(path):
            build_c_oracle()
        lib = ctypes.CDLL(path)
        lib.mso_sample.restype = ctypes.c_int
        lib.mso_sample.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_int]
        lib.mso_py_sum.restype = ctypes.c_double
        lib.mso_py_sum.argtypes = [ctypes.c_void_p, ctypes.c_int64]
        _LIB = lib
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data


def c_py_sum(x) -> float:
    x = np.ascontiguousarray(x, dtype=np.float64)
    return _lib().mso_py_sum(_ptr(x), x.size)


def c_sample(logits, temperature, top_k, top_p, uniforms, mask=None, *, bf16_bits=False,
             nthreads: int = 0):
    """Run the C restatement over a [B, V] host array.

    ``logits`` is float32, or uint16 bf16 bit patterns with ``bf16_bits=True``.
    ``mask`` is an optional [B, ceil(V/32)] uint32 bitmask (bit set = allowed).
    Returns (tokens int64, probs float64, status int32, margin_p, margin_u).
    """
    if bf16_bits:
        x = np.ascontiguousarray(logits, dtype=np.uint16)
        dtype = 1
    else:
        x = np.ascontiguousarray(logits, dtype=np.float32)
        dtype = 0
    B, V = x.shape
    T = np.ascontiguousarray(temperature, dtype=np.float64)
    k = np.ascontiguousarray(top_k, dtype=np.int32)
    p = np.ascontiguousarray(top_p, dtype=np.float64)
    u = np.ascontiguousarray(uniforms, dtype=np.float64)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
    tok = np.empty(B, np.int64)
    prob = np.empty(B, np.float64)
    st = np.empty(B, np.int32)
    mp = np.empty(B, np.float64)
    mu = np.empty(B, np.float64)
    if nthreads <= 0:
        nthreads = os.cpu_count() or 1
    rc = _lib().mso_sample(_ptr(x), dtype, B, V, V, _ptr(T), _ptr(k), _ptr(p), _ptr(u), _ptr(m),
                           0 if m is None else m.shape[1], _ptr(tok), _ptr(prob), _ptr(st),
                           _ptr(mp), _ptr(mu), nthreads)
    if rc != 0:
        raise RuntimeError(f"mso_sample failed: {rc}")
    return tok, prob, st, mp, mu
