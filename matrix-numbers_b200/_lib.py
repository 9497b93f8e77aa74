"""ctypes binding of libozaki_b200.so (the C ABI declared in include/ozaki_b200.h).

The reference engine binds its GPU path the same way (ctypes over NVRTC / cuBLASLt, dl1683/matrix-numbers
code/ozaki_engine.py:20-431); here the library is built ahead of time for sm_100a (csrc/build.py) and loaded from the
package directory.  There is no fallback: if the library is missing or was built for another architecture, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libozaki_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ozaki_b200.h")

_lib = None

P = ctypes.c_void_p
I32 = ctypes.c_int
F64 = ctypes.c_double
SZ = ctypes.c_size_t

_SIGNATURES = {
    "ozk_version": ([], I32),
    "ozk_error_string": ([I32], ctypes.c_char_p),
    "ozk_device_sm_count": ([P], I32),
    "ozk_modulus": ([I32], I32),
    "ozk_modulus_product": ([I32], F64),
    "ozk_limbs_for": ([I32], I32),
    "ozk_pmax_bits": ([I32, F64, F64, I32], I32),
    "ozk_stats_workspace_bytes": ([I32, I32, I32], SZ),
    "ozk_stats": ([P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, SZ, P], I32),
    "ozk_stats_noalloc": ([P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P], I32),
    "ozk_stats_colmax": ([P, I32, I32, P, P], I32),
    "ozk_stats_finish": ([P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P, SZ, P], I32),
    "ozk_stats_rows": ([P, I32, I32, P, P, P, P, P], I32),
    "ozk_stats_rowmax": ([P, I32, I32, P, P], I32),
    "ozk_stats_gamma": ([P, P, I32, I32, P, P, P], I32),
    "ozk_stats_cols_workspace_bytes": ([I32, I32], SZ),
    "ozk_stats_cols": ([P, I32, I32, P, P, P, P, P, SZ, P], I32),
    "ozk_rule_certified": ([P, P, P, I32, I32, I32, P, P, P, P, P], I32),
    "ozk_certificate_workspace_bytes": ([I32, I32, I32], SZ),
    "ozk_certificate": ([P, P, I32, I32, I32, P, P, P, P, P, F64, F64, P, P, P, P, P, SZ, P], I32),
    "ozk_rule_workspace_bytes": ([I32, I32, I32], SZ),
    "ozk_rule_probe_offset": ([I32, I32, I32], SZ),
    "ozk_rule_prepare": ([P, P, P, P, P, P, P, I32, I32, I32, P, I32, P, I32, I32, I32, P, P, P, P, SZ, P], I32),
    "ozk_rule_probe": ([P, P, I32, I32, I32, I32, I32, P, SZ, P], I32),
    "ozk_rule_probe_block": ([P, P, I32, I32, I32, I32, I32, I32, I32, P, SZ, P], I32),
    "ozk_rule_finish": ([P, P, P, P, I32, I32, I32, F64, F64, P, P, P, P, SZ, P], I32),
    "ozk_rule": ([P, P, I32, I32, I32, P, P, P, P, P, P, P, P, I32, P, I32, F64, F64, I32, I32, P, P, P, P, SZ, P], I32),
    "ozk_residue_symmetric": ([P, I32, SZ, P, P], I32),
    "ozk_split_a": ([P, P, P, P, I32, I32, I32, P, P, P], I32),
    "ozk_split_b": ([P, P, P, P, I32, I32, I32, P, P, P], I32),
    "ozk_gemm_residues": ([P, P, I32, I32, I32, I32, P, P, P], I32),
    "ozk_gemm_i32": ([P, P, I32, I32, I32, P, P, P], I32),
    "ozk_wait_selftest": ([I32, ctypes.c_int64, P, P, P], I32),
    "ozk_reconstruct": ([P, P, P, P, I32, I32, I32, P, P, P], I32),
    "ozk_core": ([P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, P], I32),
}


class OzkError(RuntimeError):
    """An entry point of libozaki_b200.so returned an error code."""


def lib():
    """Load libozaki_b200.so (once).  Raises if it has not been built: run __graft_entry__.build()."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OzkError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                           "(nvcc, sm_100a). The engine has no CPU or library fallback.")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def exported_names():
    return list(_SIGNATURES)


def error_string(code: int) -> str:
    s = lib().ozk_error_string(int(code))
    return s.decode() if s else "unknown"


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise OzkError(f"{what}: {error_string(rc)} (code {rc})")


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def split_kernels(src, out, vectors: int, k: int, is_b: bool) -> int:
    """Kernels one ozk_split_a / ozk_split_b call launches: 2 when the tensor-core split takes the shape (it and the
    general kernel are both launched; each returns at once for the p it does not cover), else 1.  Mirrors the
    shape test of ozk_split_tc_launch (csrc/split_tc.cu)."""
    if os.environ.get("OZK_SPLIT_TC", "1").startswith("0"):
        return 1
    ok = (vectors * k < 2 ** 32 and k % 32 == 0 and src.data_ptr() % 16 == 0 and out.data_ptr() % 8 == 0
          and (not is_b or vectors % 16 == 0))
    return 2 if ok else 1
