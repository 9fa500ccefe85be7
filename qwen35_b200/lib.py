"""Loader for libq35b.so: binds every function include/q35.h declares.

The library is the product; there is no fallback.  If the shared object is
missing this raises, so a GPU run can never silently take another path.
"""
import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
HEADER = os.path.join(ROOT, "include", "q35.h")
LIB_PATH = os.path.join(PKG, "lib", "libq35b.so")

TT = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
      "Q8_K": 15, "IQ4_NL": 20, "IQ4_XS": 23}
GEOM = {8: (32, 34), 20: (32, 18), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 12: (256, 144),
        13: (256, 176), 14: (256, 210), 23: (256, 136)}


class Config(ctypes.Structure):
    """q35b_config (include/q35.h)"""
    _fields_ = [(n, ctypes.c_int) for n in ("n_layers", "full_attention_interval", "hidden", "n_heads",
                                             "n_kv_heads", "head_dim", "n_ff", "vocab")] + \
               [("rms_eps", ctypes.c_float), ("rope_freq_base", ctypes.c_float)] + \
               [(n, ctypes.c_int) for n in ("gdn_n_heads", "gdn_num_k_heads", "gdn_head_dim", "conv_kernel")]


def _ctype(t):
    t = " ".join(t.replace("*", " * ").split())
    if "*" in t:
        return ctypes.c_char_p if t in ("const char *",) else ctypes.c_void_p
    base = t.replace("const ", "")
    return {"int": ctypes.c_int, "float": ctypes.c_float, "long long": ctypes.c_longlong,
            "unsigned long long": ctypes.c_ulonglong, "double": ctypes.c_double, "void": None}[base]


def parse_header(path=HEADER):
    """[(name, restype, [argtypes])] for every function prototype in q35.h"""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)
    src = re.sub(r"//[^\n]*", " ", src)
    src = re.sub(r"#[^\n]*", " ", src)
    out = []
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(q35\w*)\s*\(([^()]*)\)\s*;", src):
        ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
        ret = ret.split("}")[-1].strip()
        args = []
        if params and params != "void":
            for p in params.split(","):
                p = p.strip()
                toks = re.match(r"(.*?)(\b\w+)?$", p)
                ty = p
                # drop the parameter name (last identifier not part of the type)
                mm = re.match(r"^(.*[\s\*])(\w+)$", p)
                if mm and mm.group(2) not in ("int", "float", "void", "char", "long", "double"):
                    ty = mm.group(1)
                args.append(_ctype(ty.strip()))
                del toks
        out.append((name, _ctype(ret), args))
    return out


_LIB = None


def load(path=LIB_PATH):
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m qwen35_b200.build` "
                           "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, res, args in parse_header():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(rc, what=""):
    if rc != 0:
        raise RuntimeError(f"libq35b {what} failed: cuda error {rc}")
    return rc
