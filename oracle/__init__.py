"""CPU oracle for the FP8 decode GEMM -- TEST INFRASTRUCTURE ONLY.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.  It
wraps two shared libraries through ctypes:

* ``liboracle.so`` -- the restatement in ``oracle.cpp`` of the reference's host
  generators and scalar GEMM (``kernels/smoke_test.cu:60-207``,
  ``bench/bench_decode.cu:404-470``, ``kernels/weight_prepack.cuh:55-97``);
* ``_ref/libref_oracle.so`` -- the reference's own ``kernels/smoke_test.cu``
  host code compiled in place (``ref_shim.cu``), present where the reference
  checkout was available at build time.  ``load_ref()`` returns None without it.

All arrays are numpy; fp8 tensors are ``uint8`` arrays of e4m3 bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)

# Seeds the reference's smoke test uses (kernels/smoke_test.cu:502-507) and
# its per-M activation seed mix (kernels/smoke_test.cu:523).
SMOKE_SHAPES = {
    "A_contract": (6144, 7168, 0x5EED1234),
    "B_big": (7168, 16384, 0xABCDEF01),
    "C_smalln": (2048, 4096, 0x0F0F5678),
    "D_kimi3": (7168, 12288, 0x1234ABCD),
}
BENCH_SEED = 20260913  # bench/bench_decode.cu:109
REL_L2_GATE = 2.0e-3  # kernels/smoke_test.cu:48


def smoke_act_seed(shape_seed: int, m: int) -> int:
    """seed ^ (0x9e3779b97f4a7c15 * m) mod 2^64 (kernels/smoke_test.cu:523)."""
    return (shape_seed ^ ((0x9E3779B97F4A7C15 * m) & 0xFFFFFFFFFFFFFFFF)) & 0xFFFFFFFFFFFFFFFF


def reference_root():
    """The reference checkout the reference builds compile from: the
    environment variable DG_REF_ROOT, else a ``reference`` directory beside
    this repository; None when neither holds the reference's smoke test."""
    cands = [os.environ.get("DG_REF_ROOT", ""),
             os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")]
    for c in cands:
        if c and os.path.isfile(os.path.join(c, "kernels", "smoke_test.cu")):
            return os.path.abspath(c)
    return None


def build() -> None:
    """Compile liboracle.so, plus the reference builds (``_ref/``) when a
    reference checkout is found (:func:`reference_root`)."""
    cmd = ["make", "-s", "-j", str(max(1, min(8, os.cpu_count() or 1))), "-C", _HERE]
    ref = reference_root()
    if ref is not None:
        cmd.append(f"REF_ROOT={ref}")
    subprocess.run(cmd, check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def load():
    global _LIB
    if _LIB is not None:
        return _LIB
    path = os.path.join(_HERE, "liboracle.so")
    if not os.path.exists(path):
        build()
    lib = ctypes.CDLL(path)
    lib.orc_fp8_lut.argtypes = [_f32p]
    lib.orc_bf16_round.argtypes = [ctypes.c_float]
    lib.orc_bf16_round.restype = ctypes.c_float
    lib.orc_quant_e4m3.argtypes = [ctypes.c_float]
    lib.orc_quant_e4m3.restype = ctypes.c_uint8
    gen = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, _u8p, _f32p]
    for name in ("orc_gen_weight_smoke", "orc_gen_activation_smoke",
                 "orc_gen_weight_bench", "orc_gen_activation_bench"):
        getattr(lib, name).argtypes = gen
    lib.orc_gen_pertensor.argtypes = gen + [ctypes.c_int, ctypes.c_int]
    lib.orc_gen_pertensor.restype = ctypes.c_float
    ref = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p, _f32p, _u8p, _f32p, _f32p]
    lib.orc_compute_reference.argtypes = ref
    lib.orc_compute_reference_mt.argtypes = ref + [ctypes.c_int]
    pk = [_u8p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.orc_prepack.argtypes = pk
    lib.orc_prepack_swizzled.argtypes = pk
    lib.orc_quantize_rows.argtypes = [ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int, _u8p, _f32p]
    _LIB = lib
    return lib


def load_ref():
    """The reference's own host oracle, or None when it was not built here."""
    global _REF
    if _REF is not None:
        return _REF
    path = os.path.join(_HERE, "_ref", "libref_oracle.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    gen = [ctypes.c_int, ctypes.c_int, ctypes.c_uint64, _u8p, _f32p]
    lib.ref_gen_weight.argtypes = gen
    lib.ref_gen_activation.argtypes = gen
    lib.ref_compute_reference.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p, _f32p,
                                          _u8p, _f32p, _f32p]
    _REF = lib
    return lib


# --------------------------------------------------------------------------
# numpy-facing helpers (the same calls on either library)
# --------------------------------------------------------------------------

def fp8_lut() -> np.ndarray:
    out = np.zeros(256, np.float32)
    load().orc_fp8_lut(_ptr(out, _f32p))
    return out


def gen_weight_smoke(n: int, k: int, seed: int, lib=None):
    """kernels/smoke_test.cu generate_weight -> (weight[N,K] u8, scales[ceil(N/128),K/128])."""
    w = np.zeros((n, k), np.uint8)
    s = np.zeros(((n + 127) // 128, k // 128), np.float32)
    if lib is None:
        load().orc_gen_weight_smoke(n, k, seed, _ptr(w, _u8p), _ptr(s, _f32p))
    else:
        lib.ref_gen_weight(n, k, seed, _ptr(w, _u8p), _ptr(s, _f32p))
    return w, s


def gen_activation_smoke(m: int, k: int, seed: int, lib=None):
    """kernels/smoke_test.cu generate_activation (seed already mixed)."""
    a = np.zeros((m, k), np.uint8)
    s = np.zeros((m, k // 128), np.float32)
    if lib is None:
        load().orc_gen_activation_smoke(m, k, seed, _ptr(a, _u8p), _ptr(s, _f32p))
    else:
        lib.ref_gen_activation(m, k, seed, _ptr(a, _u8p), _ptr(s, _f32p))
    return a, s


def gen_weight_bench(n_log: int, k: int, seed: int):
    """bench/bench_decode.cu make_weights -> (weight[n_ker,K], scales[n_ker/128+1, K/128])."""
    n_ker = (n_log + 127) // 128 * 128
    w = np.zeros((n_ker, k), np.uint8)
    s = np.zeros((n_ker // 128 + 1, k // 128), np.float32)
    load().orc_gen_weight_bench(n_log, k, seed, _ptr(w, _u8p), _ptr(s, _f32p))
    return w, s


def gen_activation_bench(rows: int, k: int, seed: int):
    a = np.zeros((rows, k), np.uint8)
    s = np.zeros((rows, k // 128), np.float32)
    load().orc_gen_activation_bench(rows, k, seed, _ptr(a, _u8p), _ptr(s, _f32p))
    return a, s


def quantize_rows(x: np.ndarray):
    """fp32 rows [M, K] -> (e4m3 bytes [M, K], scales [M, K/128]): the block
    quantisation of bench/bench_decode.cu:459-467."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    q = np.zeros((m, k), np.uint8)
    s = np.zeros((m, k // 128), np.float32)
    load().orc_quantize_rows(m, k, _ptr(x, _f32p), k, _ptr(q, _u8p), _ptr(s, _f32p))
    return q, s


def gen_pertensor(rows: int, k: int, seed: int, scale_rows: int | None = None, threads: int = 1):
    """Per-tensor-scaled N(0,1) inputs -> (q[rows,K] u8, scales[scale_rows,K/128], s)."""
    if scale_rows is None:
        scale_rows = rows
    q = np.zeros((rows, k), np.uint8)
    s = np.zeros((scale_rows, k // 128), np.float32)
    scale = load().orc_gen_pertensor(rows, k, seed, _ptr(q, _u8p), _ptr(s, _f32p), scale_rows,
                                     threads)
    return q, s, float(scale)


def compute_reference(act, a_scales, weight, w_scales, n: int | None = None, threads: int = 1,
                      lib=None) -> np.ndarray:
    """kernels/smoke_test.cu compute_reference -> out[M,N] fp32 (bf16-rounded)."""
    act = np.ascontiguousarray(act, np.uint8)
    weight = np.ascontiguousarray(weight, np.uint8)
    a_scales = np.ascontiguousarray(a_scales, np.float32)
    w_scales = np.ascontiguousarray(w_scales, np.float32)
    m, k = act.shape
    if n is None:
        n = weight.shape[0]
    out = np.zeros((m, n), np.float32)
    args = (m, n, k, _ptr(act, _u8p), _ptr(a_scales, _f32p), _ptr(weight, _u8p),
            _ptr(w_scales, _f32p), _ptr(out, _f32p))
    if lib is not None:
        lib.ref_compute_reference(*args)
    elif threads > 1:
        load().orc_compute_reference_mt(*args, threads)
    else:
        load().orc_compute_reference(*args)
    return out


def prepack(weight: np.ndarray, bm: int, swizzled: bool = False) -> np.ndarray:
    """kernels/weight_prepack.cuh packed layout (or the swizzled B200 variant)."""
    weight = np.ascontiguousarray(weight, np.uint8)
    n, k = weight.shape
    padded = (n + bm - 1) // bm * bm
    out = np.zeros(padded * k, np.uint8)
    fn = load().orc_prepack_swizzled if swizzled else load().orc_prepack
    fn(_ptr(weight, _u8p), _ptr(out, _u8p), n, k, bm)
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rel_l2(got: np.ndarray, want: np.ndarray) -> float:
    """The reference's gate metric (kernels/smoke_test.cu:362-377)."""
    d = got.astype(np.float64) - want.astype(np.float64)
    return float(np.sqrt((d * d).sum() / max(float((want.astype(np.float64) ** 2).sum()), 1e-30)))


def elementwise_ok(got: np.ndarray, want: np.ndarray, rel: float = 1e-2, floor_frac: float = 1e-2):
    """|got-want| <= rel * max(|want|, floor_frac * rms(want)), elementwise.

    Per-element relative error is ill-conditioned at outputs near zero, so the
    denominator is floored at 1% of the output's RMS.  Returns (ok, worst ratio).
    """
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    rms = float(np.sqrt((want * want).mean())) if want.size else 0.0
    denom = np.maximum(np.abs(want), floor_frac * rms)
    denom = np.where(denom > 0, denom, 1.0)
    ratio = np.abs(got - want) / denom
    worst = float(ratio.max()) if ratio.size else 0.0
    return bool(np.all(np.isfinite(got)) and worst <= rel), worst
