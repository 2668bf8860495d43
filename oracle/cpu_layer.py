"""ctypes front end of the C oracle (``cpu_moe.c``) and of the reference's own
CPU expert kernel compiled by ``make ref`` (``_ref/libcpumoe_ref.so``).

TEST INFRASTRUCTURE ONLY (tests and bench.py's CPU legs).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libcpumoe.so"
REF_LIB = HERE / "_ref" / "libcpumoe_ref.so"
P = ctypes.c_void_p


def reference_root() -> Path | None:
    """The reference project's root: REFERENCE_ROOT, else the ``reference_path``
    that BASELINE.json at the repository root names; None when neither is a
    directory here (the GPU boxes use the prebuilt ``_ref`` library)."""
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        base = HERE.parent / "BASELINE.json"
        if base.exists():
            import json

            root = json.loads(base.read_text()).get("reference_path")
    return Path(root) if root and Path(root).is_dir() else None


def build(ref: bool = False) -> None:
    """Compile the C oracle (and, with ``ref``, the reference's CPU kernel)."""
    env = dict(os.environ)
    if ref:
        root = reference_root()
        if root is None:
            raise FileNotFoundError("the reference tree is not present: set REFERENCE_ROOT")
        env["REFERENCE_ROOT"] = str(root)
    subprocess.run(["make", "-s", "-C", str(HERE)] + (["ref"] if ref else []), check=True, env=env)


def _ptr(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(P)


class CpuMoe:
    """One routed-MoE layer on the host cores, straight from packed weights.

    ``experts[e]`` = dict(fmt=0 (NVFP4) | 1 (MXFP4), w13c, w13s, g13 (2 floats),
    w2c, w2s, g2).  ``forward`` follows the reference's CPU layer loop
    (harness/benchmarks/nvfp4_8r/cpu_moe.py:43-51): one expert call per
    distinct routed expert, rows and weights gathered from the routing.
    ``avx2`` picks the vectorised form (the timed baseline) over the scalar
    checker; both run on ``threads()`` OpenMP threads."""

    def __init__(self, hidden: int, inter: int, max_rows: int = 64, avx2: bool = False):
        if not LIB.exists():
            build()
        self.dll = ctypes.CDLL(str(LIB))
        args = [ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P, P,
                ctypes.c_float, P, P, P, ctypes.c_int, ctypes.c_float, P, P]
        for name in ("oracle_expert", "oracle_expert_avx2"):
            getattr(self.dll, name).argtypes = args
            getattr(self.dll, name).restype = None
        self.dll.oracle_set_threads.argtypes = [ctypes.c_int]
        self.dll.oracle_set_threads(threads())
        self._expert_fn = self.dll.oracle_expert_avx2 if avx2 else self.dll.oracle_expert
        self.dll.oracle_dequant.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P,
                                            ctypes.c_float, P]
        self.hidden, self.inter, self.max_rows = hidden, inter, max_rows
        self.scratch = np.zeros(max_rows * (4 * inter + 3 * hidden), np.float32)

    def expert(self, ex: dict, x: np.ndarray, rows: np.ndarray, w: np.ndarray, out: np.ndarray,
               limit: float = 10.0) -> None:
        rows = np.ascontiguousarray(rows, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        g13 = np.ascontiguousarray(ex["g13"], np.float32)
        for s in range(0, rows.size, self.max_rows):
            r, ww = rows[s:s + self.max_rows], w[s:s + self.max_rows]
            self._expert_fn(int(ex["fmt"]), self.hidden, self.inter, _ptr(ex["w13c"]),
                                   _ptr(ex["w13s"]), _ptr(g13), _ptr(ex["w2c"]), _ptr(ex["w2s"]),
                                   float(ex["g2"]), _ptr(x), _ptr(r), _ptr(ww), int(r.size),
                                   float(limit), _ptr(out), _ptr(self.scratch))

    def forward(self, x: np.ndarray, ids: np.ndarray, w: np.ndarray, experts, only=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0], self.hidden), np.float32)
        wanted = np.unique(ids) if only is None else np.intersect1d(np.unique(ids), only)
        for e in wanted:
            rows, slots = np.nonzero(ids == e)
            self.expert(experts[int(e)], x, rows, w[rows, slots], out)
        return out

    def dequant(self, fmt: int, codes: np.ndarray, scales: np.ndarray, glob: float) -> np.ndarray:
        rows, k = codes.shape[0], codes.shape[1] * 2
        out = np.empty((rows, k), np.float32)
        self.dll.oracle_dequant(fmt, rows, k, _ptr(codes), _ptr(scales), float(glob), _ptr(out))
        return out


class RefCpuExpert:
    """The reference's own CPU kernel (harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c),
    fixed at hidden 5120, TP slice 576, W2 K padded to 640, MXFP4 records."""

    HIDDEN, INTER, W2K = 5120, 576, 640

    def __init__(self):
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle ref)")
        self.dll = ctypes.CDLL(str(REF_LIB))
        self.dll.expert_slice.argtypes = [P, P, P, P, ctypes.c_int, P, P, P, P]
        self.dll.expert_slice.restype = None
        self.xs = np.zeros((16, self.HIDDEN), np.float32)
        self.gu = np.zeros((16, 2 * self.INTER), np.float32)
        self.act = np.zeros((16, self.W2K), np.float32)

    @classmethod
    def record(cls, w13c, w13s, w2c, w2s) -> np.ndarray:
        """One expert record in the reference layout (nvfp4_8r_native.py:59-75):
        w1 codes | w1 E8M0 | w3 codes | w3 E8M0 | w2 codes [H][320] | w2 E8M0 [H][20]."""
        i = cls.INTER
        w2cp = np.zeros((cls.HIDDEN, cls.W2K // 2), np.uint8)
        w2sp = np.full((cls.HIDDEN, cls.W2K // 32), 127, np.uint8)
        w2cp[:, : i // 2] = w2c
        w2sp[:, : i // 32] = w2s
        return np.concatenate([w13c[:i].ravel(), w13s[:i].ravel(), w13c[i:].ravel(), w13s[i:].ravel(),
                               w2cp.ravel(), w2sp.ravel()])

    def expert(self, rec: np.ndarray, x: np.ndarray, rows: np.ndarray, w: np.ndarray, out: np.ndarray):
        rows = np.ascontiguousarray(rows, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        self.dll.expert_slice(_ptr(rec), _ptr(x), _ptr(rows), _ptr(w), int(rows.size), _ptr(out),
                              _ptr(self.xs), _ptr(self.gu), _ptr(self.act))


def threads() -> int:
    """Every host core this process may run on (its CPU affinity), whatever
    OMP_NUM_THREADS says: torchrun sets that variable to 1."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1
