"""The C-ABI library loads and exports every entry point declared in include/*.h.

Runs without a GPU: only symbol lookup and argument validation paths that
return before any launch are exercised.
"""

import ctypes
import glob
import os
import re

import pytest

from conftest import REPO


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s+(csaq_[a-z0-9_]+)\s*\(", src, re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared_functions()
    for expected in ("csaq_quant_pack", "csaq_dequant", "csaq_qgemv", "csaq_unpack"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    from csaq import _lib
    L = _lib.lib()
    missing = [n for n in _declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    from csaq import _lib
    _lib.lib()
    declared = set(_declared_functions())
    bound = set(_lib.exported_symbols())
    assert declared <= bound, sorted(declared - bound)


def _prototypes():
    """name -> (return type, [parameter types]) from every prototype in include/*.h."""
    out = {}
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"^\s*((?:const\s+)?[A-Za-z_0-9]+\s*\**)\s*(csaq_[a-z0-9_]+)\s*\(([^)]*)\)\s*;",
                             src, re.M):
            params = []
            for p in m.group(3).split(","):
                p = " ".join(p.split())
                if p and p != "void":
                    params.append(re.sub(r"\s*\b[A-Za-z_0-9]+$", "", p).replace(" *", "*"))
            out[m.group(2)] = (" ".join(m.group(1).split()).replace(" *", "*"), params)
    return out


# C scalar type -> the ctypes class that passes it (same width, same signedness or float)
_C_SCALARS = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "uint64_t": ctypes.c_uint64,
              "uint32_t": ctypes.c_uint32, "float": ctypes.c_float}
# pointee of a typed pointer -> the ctypes element a POINTER() argument may use
_C_POINTEES = {"int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "uint64_t": ctypes.c_uint64,
               "uint32_t": ctypes.c_uint32, "uint16_t": ctypes.c_uint16, "uint8_t": ctypes.c_uint8,
               "float": ctypes.c_float}


def _arg_matches(c_type, ct):
    if c_type.endswith("*"):
        if ct in (ctypes.c_void_p, ctypes.c_char_p):
            return True
        if not (isinstance(ct, type) and issubclass(ct, ctypes._Pointer)):
            return False
        pointee = c_type[:-1].replace("const ", "").strip()
        if pointee in _C_POINTEES:
            return ctypes.sizeof(ct._type_) == ctypes.sizeof(_C_POINTEES[pointee])
        return True  # a struct, checked by the layout tests
    want = _C_SCALARS.get(c_type)
    return want is not None and ct is want


def test_python_signatures_match_the_header():
    """Every ctypes binding passes what the C prototype takes: the same
    number of arguments, pointers where it takes pointers and scalars of the
    same width and kind (a c_int bound to an int64_t parameter would leave
    the upper half of the register undefined)."""
    from csaq import _lib
    _lib.lib()
    protos = _prototypes()
    assert set(protos) == set(_declared_functions())
    bad = []
    for name, (ret, params) in sorted(protos.items()):
        restype, argtypes = _lib._SIGNATURES[name]
        if len(argtypes) != len(params):
            bad.append((name, "arity", len(params), len(argtypes)))
            continue
        for i, (c_type, ct) in enumerate(zip(params, argtypes)):
            if not _arg_matches(c_type, ct):
                bad.append((name, i, c_type, ct))
        want_ret = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "const char*": ctypes.c_char_p,
                    "void": None}[ret]
        if restype is not want_ret:
            bad.append((name, "return", ret, restype))
    assert not bad, bad


def test_version_and_status_strings():
    from csaq import _lib
    L = _lib.lib()
    assert b"sm_100a" in L.csaq_version()
    assert L.csaq_status_string(0) == b"ok"
    assert L.csaq_status_string(-2) == b"unsupported bit-width"
    assert L.csaq_packed_row_bytes(37, 4) == 19
    assert L.csaq_packed_row_bytes(37, 2) == 10
    assert L.csaq_packed_row_bytes(37, 8) == 37
    assert L.csaq_packed_row_bytes(37, 16) == 74
    assert L.csaq_packed_row_bytes(37, 3) == -1


def test_checked_build_switch():
    """The default library has no index guards; libcsaq_b200_checked.so
    (CSAQ_LIB=checked) reports itself as checked and exports the same ABI."""
    import subprocess
    import sys
    from csaq import _lib
    L = _lib.lib()
    assert L.csaq_checked_build() == 0
    v = [ctypes.c_int64(7) for _ in range(4)]
    assert L.csaq_guard_report(*[ctypes.byref(x) for x in v]) == -5
    assert [x.value for x in v] == [0, 0, 0, 0]
    assert L.csaq_guard_clear() == -5
    assert L.csaq_guard_report(None, None, None, None) == -1
    code = ("import sys; sys.path.insert(0, 'csaq-quant_b200'); from csaq import _lib; "
            "L = _lib.lib(); print(L.csaq_checked_build(), _lib.LIB_PATH.endswith('_checked.so'))")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, CSAQ_LIB="checked"), cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.split() == ["1", "True"]


def test_c_consumer_compiles_links_and_runs(tmp_path):
    """include/csaq_b200.h compiles as strict C99 and a C program linked to the
    library gets the same host-side answers as the Python binding."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lib_dir = os.path.join(REPO, "csaq-quant_b200", "csaq", "lib")
    exe = str(tmp_path / "abi_c_consumer")
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(REPO, "include"),
                        os.path.join(REPO, "tests", "abi_c_consumer.c"), "-L", lib_dir, "-lcsaq_b200",
                        f"-Wl,-rpath,{lib_dir}", "-o", exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = dict(l.split(" ", 1) for l in out.stdout.strip().splitlines())
    assert "sm_100a" in lines["version"]
    assert lines["status"] == "unsupported bit-width"
    assert lines["row_bytes"] == "10 19 37 74"
    assert lines["quant_pack_null"] == "-1" and lines["quant_pack_bits"] == "-2"
    assert lines["qgemv_bits"] == "-2" and lines["qgemv_tiers"] == "-1"
    assert lines["greedy_null"] == "-1"
    assert lines["checked"] == "0 guard -5"
    # the ctypes mirrors of the ABI structs have the C layout
    from csaq import _lib
    T, E, G = _lib.CsaqTier, _lib.CsaqGemvExt, _lib.CsaqP2PGroup
    assert lines["layout_tier"] == f"{ctypes.sizeof(T)} {T.blocks.offset} {T.y.offset} {T.ldr.offset}"
    assert lines["layout_gemv_ext"] == f"{ctypes.sizeof(E)} {E.x_mul.offset}"
    assert lines["layout_p2p_group"] == f"{ctypes.sizeof(G)} {G.flags.offset} {G.err.offset}"


def test_argument_validation_without_launch():
    """Bad arguments are rejected on the host before any kernel launch."""
    from csaq import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(16)
    assert L.csaq_quant_pack(None, 0, 4, 4, 4, 4, 128, dummy, dummy, dummy, None) == -1
    assert L.csaq_quant_pack(dummy, 0, 4, 4, 4, 3, 128, dummy, dummy, dummy, None) == -2
    assert L.csaq_quant_pack(dummy, 7, 4, 4, 4, 4, 128, dummy, dummy, dummy, None) == -1
    assert L.csaq_unpack(dummy, 5, 4, 4, dummy, None) == -2
    assert L.csaq_dequant(dummy, None, None, 4, 4, 4, -1, 0, 0, dummy, None) == -1
    t = _lib.CsaqTier(bits=3, n_rows=1, group_size=128, n_groups=1, row_bytes=64)
    arr = _lib.tier_array([t])
    assert L.csaq_qgemv(arr, 1, 128, dummy, 2, 1, 128, None) == -2
    assert L.csaq_qgemv(arr, 0, 128, dummy, 2, 1, 128, None) == -1
    assert L.csaq_qgemv(arr, 17, 128, dummy, 2, 1, 128, None) == -1


def test_kernels_fail_loudly_without_cuda():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from csaq.kernels import quantize_per_channel
    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_per_channel(torch.randn(4, 8), 4)
