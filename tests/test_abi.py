"""The C-ABI library loads and exports every entry point declared in include/rgpt.h (CPU only:
no kernels are launched), and the Python binding declares a signature for each of them."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rgpt.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(rgpt_\w+)\s*\(", text)))


def test_header_declares_the_path():
    syms = declared_symbols()
    for must in ("rgpt_gemm_bf16", "rgpt_attn_fwd", "rgpt_attn_bwd", "rgpt_rownorm_fwd", "rgpt_rownorm_bwd",
                 "rgpt_qkv_prep_fwd", "rgpt_qkv_prep_bwd", "rgpt_cross_entropy", "rgpt_adamw", "rgpt_muon_prep",
                 "rgpt_muon_apply", "rgpt_last_error"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    from rgpt_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built (run make -C rgpt_b200/csrc)")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    from rgpt_b200 import _lib
    missing = [s for s in declared_symbols() if s not in _lib._SIGNATURES]
    assert not missing, missing


def test_version_and_error_buffer_without_gpu():
    from rgpt_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    lib = _lib.load()
    assert lib.rgpt_version() >= 100
    buf = ctypes.create_string_buffer(64)
    assert lib.rgpt_last_error(buf, 64) == 0


def test_binding_argument_counts_match_the_header():
    """Each ctypes binding passes exactly as many arguments as the header declares (a missing or extra
    argument would shift every later one)."""
    from rgpt_b200 import _lib
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = dict(re.findall(r"\bint\s+(rgpt_\w+)\s*\(([^)]*)\)\s*;", text))
    mismatched = []
    for name, params in decls.items():
        params = params.strip()
        n = 0 if params in ("", "void") else len(params.split(","))
        if len(_lib._SIGNATURES[name]) != n:
            mismatched.append((name, n, len(_lib._SIGNATURES[name])))
    assert not mismatched, mismatched


def test_binding_argument_types_match_the_header():
    """Each ctypes argument type is the one the header's parameter needs (a float bound as an int, or a
    64-bit size bound as 32 bits, would be read wrongly by the library)."""
    import ctypes

    from rgpt_b200 import _lib
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    decls = dict(re.findall(r"\bint\s+(rgpt_\w+)\s*\(([^)]*)\)\s*;", text))
    scalar = {"int": ctypes.c_int, "float": ctypes.c_float, "long long": ctypes.c_longlong,
              "unsigned": ctypes.c_uint, "size_t": ctypes.c_ulonglong, "unsigned long long": ctypes.c_ulonglong}

    def ctype_of(param):
        if "*" in param:
            return ctypes.c_char_p if re.match(r"\s*(const\s+)?char\s*\*", param) else ctypes.c_void_p
        words = [w for w in param.split()[:-1] if w != "const"]  # the type, without the name
        return scalar[" ".join(words)]

    bad = []
    for name, params in decls.items():
        ps = [] if params.strip() in ("", "void") else params.split(",")
        want = [ctype_of(p) for p in ps]
        if want != list(_lib._SIGNATURES[name]):
            bad.append(name)
    assert not bad, bad
