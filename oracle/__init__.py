"""CPU oracle for the MLA decode path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and the ``--impl reference`` arm) import this package.
It is the checker and the reported CPU baseline; the product path under
``ada-mla_b200/`` never imports it and has no CPU fallback.

Two CPU implementations live behind this module:

* ``_build/libmla_oracle.so`` -- our plain-C restatement (``mla_oracle.c``) of
  the reference's ``run_mla_decode_cpu``
  (lechebs/ada-mla csrc/mla_decode_naive_fp32_cpu.cpp:5-61).
* ``_ref/libref_mla_cpu.so`` -- the reference's own function, compiled unchanged
  from its sources by ``oracle/Makefile`` (only where the reference checkout is
  present; the library then travels with the repository snapshot).

Parity is pinned by ``tests/golden`` (fixtures produced by the reference's own
function) and directly against ``_ref`` when it is available.

Adapter (the reference CPU kernel divides by sqrt(head_dim_c) = 24 and returns
all 576 columns): to get ``softmax(scale * Q C^T) C[:, :dv]`` we pass
``Q * scale * sqrt(576)`` and keep the first ``dv`` columns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(_HERE, "_build", "libmla_oracle.so")
_REF_SO = os.path.join(_HERE, "_ref", "libref_mla_cpu.so")
_lock = threading.Lock()
_libs: dict[str, ctypes.CDLL | None] = {}

_F32P = ctypes.POINTER(ctypes.c_float)


def reference_dir(ref_dir: str | None = None) -> str | None:
    """The reference checkout: the argument, else $MLA_REFERENCE_DIR, else a
    checkout named ``reference`` beside this repository.  None when its CPU
    kernel's source is not there (e.g. on a machine that only runs the tests)."""
    cands = [ref_dir, os.environ.get("MLA_REFERENCE_DIR"),
             os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")]
    for d in cands:
        if d and os.path.isfile(os.path.join(d, "csrc", "mla_decode_naive_fp32_cpu.cpp")):
            return os.path.abspath(d)
    return None


def build(ref_dir: str | None = None) -> None:
    """Compile the oracle (and the reference CPU kernel when its sources exist)."""
    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    ref = reference_dir(ref_dir)
    if ref is not None:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={ref}"], check=True)


def _load(path: str, build_if_missing: bool) -> ctypes.CDLL | None:
    with _lock:
        if path in _libs:
            return _libs[path]
        if not os.path.isfile(path) and build_if_missing:
            subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
        if not os.path.isfile(path):
            _libs[path] = None
            return None
        lib = ctypes.CDLL(path)
        _libs[path] = lib
        return lib


def oracle_lib() -> ctypes.CDLL:
    lib = _load(_ORACLE_SO, build_if_missing=True)
    assert lib is not None, "oracle library could not be built"
    lib.mla_oracle_decode_f32.restype = ctypes.c_int
    lib.mla_oracle_decode_f32.argtypes = [_F32P, _F32P, _F32P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.mla_oracle_decode_f64.restype = ctypes.c_int
    lib.mla_oracle_decode_f64.argtypes = [_F32P, _F32P, _F32P, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_double]
    return lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own CPU kernel, or None when it was not built here."""
    lib = _load(_REF_SO, build_if_missing=False)
    if lib is not None:
        lib.ref_run_mla_decode_cpu.restype = None
        lib.ref_run_mla_decode_cpu.argtypes = [_F32P, _F32P, _F32P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    return lib


def have_ref() -> bool:
    return ref_lib() is not None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_F32P)


def _f32c(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def run_mla_decode_cpu(query, cache, *, impl: str = "oracle", threads: int = 1) -> np.ndarray:
    """Reference semantics: softmax(Q C^T / sqrt(D)) C over all D columns.

    ``impl`` = "oracle" (our restatement) or "reference" (the reference's own
    function from ``_ref``).  Rows (heads) are independent, so ``threads > 1``
    splits the heads over host threads, each thread calling the single-threaded
    kernel on its head block (ctypes releases the GIL during the call).
    """
    q = _f32c(query)
    c = _f32c(cache)
    nh, d = q.shape
    n = c.shape[0]
    assert c.shape[1] == d
    out = np.empty((nh, d), dtype=np.float32)
    if impl == "oracle":
        fn = oracle_lib().mla_oracle_decode_f32
    elif impl == "reference":
        rl = ref_lib()
        if rl is None:
            raise RuntimeError("reference CPU kernel not built (oracle/_ref missing)")
        fn = rl.ref_run_mla_decode_cpu
    else:
        raise ValueError(impl)

    def run_block(h0: int, h1: int) -> None:
        qp = ctypes.cast(ctypes.c_void_p(q.ctypes.data + h0 * d * 4), _F32P)
        op = ctypes.cast(ctypes.c_void_p(out.ctypes.data + h0 * d * 4), _F32P)
        r = fn(qp, _ptr(c), op, h1 - h0, d, n)
        if r not in (None, 0):
            raise RuntimeError(f"oracle returned {r}")

    threads = max(1, min(int(threads), nh))
    if threads == 1:
        run_block(0, nh)
    else:
        bounds = [(nh * i // threads, nh * (i + 1) // threads) for i in range(threads)]
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(lambda b: run_block(*b), bounds))
    return out


def mla_decode_oracle(query, cache, scale: float, dv: int = 512, *, impl: str = "oracle",
                      threads: int = 1) -> np.ndarray:
    """Weight-absorbed decode softmax(scale * Q C^T) C[:, :dv] via the reference CPU kernel.

    Q is pre-multiplied by scale * sqrt(D) so that the kernel's internal
    division by sqrt(D) leaves exactly ``scale``.
    """
    q = _f32c(query)
    d = q.shape[1]
    qs = (q.astype(np.float64) * (scale * np.sqrt(d))).astype(np.float32)
    return run_mla_decode_cpu(qs, cache, impl=impl, threads=threads)[:, :dv]


def mla_decode_f64(query, cache, scale: float, dv: int = 512) -> np.ndarray:
    """Double-precision second opinion: softmax(scale * Q C^T) C[:, :dv]."""
    q = _f32c(query)
    c = _f32c(cache)
    nh, d = q.shape
    out = np.empty((nh, dv), dtype=np.float32)
    r = oracle_lib().mla_oracle_decode_f64(_ptr(q), _ptr(c), _ptr(out), nh, d, dv, c.shape[0], float(scale))
    if r != 0:
        raise RuntimeError(f"oracle f64 returned {r}")
    return out


def mla_decode_batched_oracle(query, cache, cu_seqlens, scale: float, dv: int = 512, *,
                              impl: str = "oracle", threads: int = 1) -> np.ndarray:
    """Per-sequence oracle over a packed cache: query [B, n_h, D], cache [sum N_b, D]."""
    q = _f32c(query)
    c = _f32c(cache)
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    b, nh, _ = q.shape
    out = np.zeros((b, nh, dv), dtype=np.float32)
    for i in range(b):
        lo, hi = int(cu[i]), int(cu[i + 1])
        if hi > lo:
            out[i] = mla_decode_oracle(q[i], c[lo:hi], scale, dv, impl=impl, threads=threads)
    return out


def lse_partial_oracle(query, cache, scale: float, dv: int = 512):
    """(O normalized, lse) of one KV slice, in float64 numpy (for merge-math tests).

    lse is the natural-log log-sum-exp of the scaled logits; an empty slice
    gives O = 0 and lse = -inf.
    """
    q = np.asarray(query, dtype=np.float64)
    c = np.asarray(cache, dtype=np.float64)
    if c.shape[0] == 0:
        return np.zeros((q.shape[0], dv)), np.full((q.shape[0],), -np.inf)
    s = scale * (q @ c.T)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    o = (p @ c[:, :dv]) / l
    return o, (m + np.log(l))[:, 0]
