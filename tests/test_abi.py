"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every entry point include/*.h declares, the Python binding covers them, and
the product path neither imports the oracle nor carries a CPU fallback."""
import glob
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        syms |= set(re.findall(r"\b(pb_[a-z0-9_]+)\s*\(", txt))
    return syms


def test_library_exports_every_declared_symbol(native):
    lib = os.path.join(ROOT, "purebee_b200", "libpurebee_b200.so")
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (pb_[a-z0-9_]+)$", out, flags=re.M))
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_binding_covers_header(native):
    assert declared_symbols() <= set(native.SIGNATURES)
    L = native.lib()
    for s in declared_symbols():
        assert hasattr(L, s)


def test_header_is_plain_c():
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        assert "torch" not in txt.lower()
        assert 'extern "C"' in txt


def test_product_does_not_import_oracle():
    for f in glob.glob(os.path.join(ROOT, "purebee_b200", "**", "*.py"), recursive=True):
        txt = open(f).read()
        assert "import oracle" not in txt and "from oracle" not in txt, f
        assert "_work/" not in txt and "'_work'" not in txt, f
    for f in glob.glob(os.path.join(ROOT, "purebee_b200", "csrc", "*")):
        txt = open(f).read()
        assert "pb_oracle" not in txt and "orc_" not in txt, f


def test_no_device_fails_loudly(native):
    import torch
    if torch.cuda.is_available():
        return
    import pytest
    with pytest.raises(native.PureBeeError):
        native.Context(0)


def test_abi_version(native):
    assert native.lib().pb_abi_version() == 1


def declared_arity():
    """name -> number of parameters, from the prototypes in include/*.h."""
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        txt = re.sub(r"//[^\n]*", "", txt)
        for name, params in re.findall(r"\b(pb_[a-z0-9_]+)\s*\(([^;{}]*?)\)\s*;", txt, flags=re.S):
            p = params.strip()
            out[name] = 0 if p in ("", "void") else p.count(",") + 1
    return out


def test_binding_arity_matches_header(native):
    """Every ctypes signature passes as many arguments as the C prototype
    takes (a mismatch would silently misread arguments at the C ABI)."""
    ar = declared_arity()
    assert set(ar) == declared_symbols()  # every prototype was parsed
    wrong = {n: (k, len(native.SIGNATURES[n][1])) for n, k in ar.items()
             if n in native.SIGNATURES and len(native.SIGNATURES[n][1]) != k}
    assert not wrong, f"(header, binding) parameter counts differ: {wrong}"


def _c_kind(decl):
    d = decl.strip()
    if "*" in d or "[" in d:
        return "ptr"
    d = re.sub(r"\b(const|unsigned|signed)\b", " ", d).split()
    t = d[0] if d else ""
    if t in ("double",):
        return "f64"
    if t in ("float",):
        return "f32"
    if t in ("size_t", "int64_t", "uint64_t", "long"):
        return "i64"
    if t in ("int", "int32_t", "uint32_t", "bool"):
        return "i32"
    return "other:" + t


def _py_kind(ct):
    import ctypes
    if ct in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(ct, type) and issubclass(ct, ctypes._Pointer)):
        return "ptr"
    if ct is ctypes.c_double:
        return "f64"
    if ct is ctypes.c_float:
        return "f32"
    if ctypes.sizeof(ct) == 8:
        return "i64"
    if ctypes.sizeof(ct) == 4:
        return "i32"
    return "other"


def test_binding_argument_kinds_match_header(native):
    """Each argument's kind (pointer, 4- or 8-byte integer, float, double)
    agrees between the prototype and the ctypes binding: a 4-byte int passed
    where the C side reads a size_t leaves the upper half undefined."""
    wrong = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for name, params in re.findall(r"\b(pb_[a-z0-9_]+)\s*\(([^;{}]*?)\)\s*;", txt, flags=re.S):
            p = params.strip()
            kinds = [] if p in ("", "void") else [_c_kind(x) for x in p.split(",")]
            got = [_py_kind(t) for t in native.SIGNATURES[name][1]]
            if kinds != got:
                wrong[name] = (kinds, got)
    assert not wrong, f"(header, binding) argument kinds differ: {wrong}"


def test_binding_return_kinds_match_header(native):
    """Return kinds agree too (a pointer or 64-bit result read as a 4-byte int
    would be truncated)."""
    wrong, seen = {}, set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for ret, name in re.findall(r"(?:^|;|\})\s*((?:const\s+)?[a-z_0-9]+(?:\s*\*)?)\s*\b(pb_[a-z0-9_]+)\s*\([^;{}]*?\)\s*;",
                                    txt, flags=re.S | re.M):
            seen.add(name)
            want = "void" if ret.strip() == "void" else _c_kind(ret)
            rt = native.SIGNATURES[name][0]
            got = "void" if rt is None else _py_kind(rt)
            if want != got:
                wrong[name] = (ret.strip(), want, got)
    assert seen == declared_symbols()
    assert not wrong, f"(header, binding) return kinds differ: {wrong}"
