"""ctypes front end of ``oracle/native_cpu.cpp`` — TEST INFRASTRUCTURE ONLY.

The C++ restatement of the reference's Zig CPU inference kernels (kernels/src/tropical.zig,
kernels/src/lut.zig): an extra oracle for the eval forward and an optional CPU baseline for the
eval workloads of ``bench.py``. Only ``tests/`` and ``bench.py`` (its CPU legs) use it; the
product path never does.

``build()`` compiles ``native_cpu.cpp`` with g++ into ``oracle/_build/liboracle_cpu.so``
(``-O3 -march=x86-64-v3 -ffp-contract=off``: AVX2 vectors and F16C conversions, products and sums
rounded separately, as the Zig kernels do).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "native_cpu.cpp"
LIBRARY = HERE / "_build" / "liboracle_cpu.so"

_lib: ctypes.CDLL | None = None


def build(force: bool = False) -> Path:
    """Compiles the library when it is missing or older than its source."""
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-ffp-contract=off", "-march=x86-64-v3",
           "-Wno-psabi", str(SOURCE), "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    tmp.replace(LIBRARY)
    return LIBRARY


def _cpu_flags() -> set[str]:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("flags"):
                return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        missing = {"avx2", "fma", "f16c"} - _cpu_flags()
        if missing:
            raise RuntimeError(f"the native CPU kernels are built for x86-64-v3; this CPU lacks {sorted(missing)}")
        if not LIBRARY.exists():
            raise FileNotFoundError(f"{LIBRARY} is missing: run oracle.native.build() (g++)")
        lib = ctypes.CDLL(str(LIBRARY))
        i64, p, f32, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_int
        lib.oracle_cpu_default_threads.restype = i32
        lib.oracle_cpu_default_threads.argtypes = []
        lib.oracle_cpu_trop_route_hidden.restype = i32
        lib.oracle_cpu_trop_route_hidden.argtypes = [i64, i64, i64, i64, f32, p, p, p, p, i32, p, i32]
        lib.oracle_cpu_lut_forward.restype = i32
        lib.oracle_cpu_lut_forward.argtypes = [i64, i64, i64, i64, i64, p, i32, p, p, p, p, i32]
        _lib = lib
    return _lib


def _param(a: np.ndarray) -> tuple[np.ndarray, int]:
    """f32 or f16 parameter array, C-contiguous, and its f16 flag (other dtypes are widened)."""
    if a.dtype == np.float16:
        return np.ascontiguousarray(a), 1
    return np.ascontiguousarray(a, dtype=np.float32), 0


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def trop_route_hidden(
    latent: np.ndarray,
    router_weight: np.ndarray,
    router_bias: np.ndarray,
    code: np.ndarray,
    *,
    code_scale: float,
    threads: int = 0,
) -> np.ndarray:
    """trop_route_hidden_batch_f32 / _f16 (kernels/src/tropical.zig:299-350): hidden [N, D]
    from latent [N, D] (inference: winner codes only). f16 parameters stay f16."""
    lat = np.ascontiguousarray(latent, dtype=np.float32)
    n, d = lat.shape
    heads, cells, dim = router_weight.shape
    if dim != d or code.shape != router_weight.shape or router_bias.shape != (heads, cells):
        raise ValueError("trop_route_hidden: shape mismatch")
    w, f16 = _param(router_weight)
    b = np.ascontiguousarray(router_bias, dtype=np.float16 if f16 else np.float32)
    c = np.ascontiguousarray(code, dtype=np.float16 if f16 else np.float32)
    hidden = np.empty((n, d), dtype=np.float32)
    status = load().oracle_cpu_trop_route_hidden(n, heads, cells, d, float(code_scale), _ptr(lat), _ptr(w), _ptr(b),
                                                 _ptr(c), f16, _ptr(hidden), int(threads))
    if status != 0:
        raise ValueError("oracle_cpu_trop_route_hidden: bad arguments")
    return hidden


def lut_forward(x: np.ndarray, anchors: np.ndarray, thresholds: np.ndarray, lut: np.ndarray, *,
                threads: int = 0) -> np.ndarray:
    """lut_forward_batch_with_offsets_no_cache / lut_forward_batch_f16_no_cache
    (kernels/src/lut.zig:255-318): out [N, out] = sum_t lut[t, idx_t] (no output scale)."""
    xs = np.ascontiguousarray(x, dtype=np.float32)
    n, inn = xs.shape
    tables, comparisons, _ = anchors.shape
    weights, f16 = _param(lut)
    out_f = weights.shape[2]
    anc = np.ascontiguousarray(anchors, dtype=np.int64)
    off = np.ascontiguousarray(thresholds, dtype=np.float32)
    out = np.empty((n, out_f), dtype=np.float32)
    status = load().oracle_cpu_lut_forward(n, tables, comparisons, inn, out_f, _ptr(weights), f16, _ptr(anc), _ptr(off),
                                           _ptr(xs), _ptr(out), int(threads))
    if status != 0:
        raise ValueError("oracle_cpu_lut_forward: bad arguments (sizes, or an anchor outside the input)")
    return out


def default_threads() -> int:
    return int(load().oracle_cpu_default_threads())


def trop_linear_eval(x: np.ndarray, params: dict[str, np.ndarray], *, code_scale: float, threads: int = 0,
                     param_dtype: str | None = None) -> np.ndarray:
    """TropLinear eval forward with the route step on the native kernel, as the reference's
    ``backend="zig"`` runs it (layers/tropical.py:89-99, backends/tropical_zig.py:60-105): the
    projection and the output map as float32 matrix products (numpy), z rounded to the parameter
    dtype first, the route + code sum in C++ (f16 parameters stay f16)."""
    from .tropnn_oracle import _f32, _param_dtype, _round_to

    pdt = _param_dtype(params, param_dtype)
    x = np.asarray(x).reshape(-1, np.asarray(x).shape[-1])
    z = _round_to(_round_to(x, pdt) @ _f32(params["proj.weight"]).T, pdt)
    hidden = trop_route_hidden(z, params["router_weight"], params["router_bias"], params["code"],
                               code_scale=code_scale, threads=threads)
    return (hidden @ _f32(params["output_proj.weight"]).T + _f32(params["output_proj.bias"])).astype(np.float32)


def pairwise_eval(x: np.ndarray, params: dict[str, np.ndarray], *, output_scale: float, threads: int = 0) -> np.ndarray:
    """PairwiseLinear eval forward as the reference's ``backend="zig"`` runs it
    (layers/pairwise.py:77-80, backends/pairwise_zig.py): the native LUT sum, then output_scale."""
    x = np.asarray(x).reshape(-1, np.asarray(x).shape[-1])
    out = lut_forward(x, params["anchors"], params["thresholds"], params["lut"], threads=threads)
    if output_scale != 1.0:
        out = (out * np.float32(output_scale)).astype(np.float32)
    return out
