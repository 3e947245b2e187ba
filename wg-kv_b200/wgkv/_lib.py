"""ctypes binding of libwgkv.so, typed from include/wgkv.h.

The C ABI is the boundary: every entry point takes raw device pointers,
sizes, element strides and a stream handle.  Argument and return types are
read from the header so the binding cannot drift from the declarations.
There is no fallback: if the library or a CUDA device is missing, the call
fails with an error.
"""
from __future__ import annotations

import ctypes
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("WGKV_LIB", os.path.join(_PKG, "libwgkv.so"))
HEADER = os.path.join(os.path.dirname(os.path.dirname(_PKG)), "include", "wgkv.h")

_CTYPES = {
    "int": ctypes.c_int,
    "float": ctypes.c_float,
    "double": ctypes.c_double,
    "size_t": ctypes.c_size_t,
    "int64_t": ctypes.c_int64,
    "uint64_t": ctypes.c_uint64,
    "int32_t": ctypes.c_int32,
    "uint32_t": ctypes.c_uint32,
    "void": None,
}


def _ctype(decl: str):
    decl = decl.replace("const ", "").strip()
    if "*" in decl:
        return ctypes.c_void_p
    base = decl.split()[0]
    return _CTYPES[base]


def parse_header(path: str = HEADER):
    """{name: (restype, [argtypes])} for every ``WGKV_API`` declaration."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"WGKV_API\s+([\w\s\*]+?)\s*\b(wgkv_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        ret, name, args = m.group(1), m.group(2), m.group(3).strip()
        argtypes = []
        if args and args != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                # strip the parameter name
                t = re.sub(r"\b\w+$", "", a).strip() if not a.endswith("*") else a
                argtypes.append(_ctype(t))
        out[name] = (_ctype(ret), argtypes)
    return out


class _Lib:
    def __init__(self):
        self._lib = None
        self.decls = parse_header()
        self.launches = 0

    def load(self):
        if self._lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"libwgkv.so not built ({LIB_PATH}); run `python wg-kv_b200/build.py`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in self.decls.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            self._lib = lib
        return self._lib

    def __getattr__(self, name):
        if name.startswith("wgkv_"):
            fn = getattr(self.load(), name)
            n = KERNELS_PER_CALL.get(name)
            if n is None:
                return fn

            def counted(*args, _fn=fn, _n=n):
                self.launches += _n
                return _fn(*args)
            return counted
        raise AttributeError(name)


# kernels each compute entry point launches (for the benchmark's launch count)
KERNELS_PER_CALL = {"wgkv_paged_decode": 1, "wgkv_gate_scores": 1, "wgkv_decode_append": 1, "wgkv_decode_gate_append": 1, "wgkv_promote": 2,
                    "wgkv_prefill_admit": 3, "wgkv_sparse_indices": 3, "wgkv_sparse_prefill": 1, "wgkv_sparse_prefill_pooled": 1, "wgkv_gather_columns": 1,
                    "wgkv_paged_decode_noalloc": 1, "wgkv_ring_advance": 1, "wgkv_decode_prologue": 1,
                    "wgkv_rms_norm": 1, "wgkv_silu_mul": 1, "wgkv_skinny_gemm": 1, "wgkv_quest_select": 2, "wgkv_argmax": 1,
                    "wgkv_selftest_wait_limit": 1, "wgkv_oproj_allreduce": 1}
# wgkv_snapkv_evict launches 3 kernels per layer + 1; it is not counted (no benchmark step runs it)


lib = _Lib()

STATUS = {0: "ok", -1: "invalid argument", -2: "CUDA error", -3: "workspace too small"}
ERR_BITS = {0x1: "tokens exceed max_tokens_per_head", 0x2: "pool exhausted (allocation exceeds total_blocks)",
            0x4: "a device wait timed out", 0x8: "page id out of range",
            0x10: "RoPE position outside the tables"}


def check(status: int, what: str):
    if status != 0:
        raise RuntimeError(f"{what}: {STATUS.get(status, status)}")
