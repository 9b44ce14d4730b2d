"""The C-ABI library loads and exports every entry point include/t2sx.h declares (no GPU)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "t2sx.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(t2sx_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(t2sx_mod):
    import ctypes
    lib = ctypes.CDLL(t2sx_mod.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    # the binding covers the whole header
    assert set(syms) == set(t2sx_mod.SIGNATURES), set(syms) ^ set(t2sx_mod.SIGNATURES)


def test_errors_without_device(t2sx_mod):
    """Invalid arguments are rejected on the host, before any device work."""
    import ctypes
    L = t2sx_mod.lib()
    h = ctypes.c_void_p()
    assert L.t2sx_model_load(None, 0, ctypes.byref(h)) == t2sx_mod.ERR_INVALID
    assert b"null" in L.t2sx_last_error()
    assert L.t2sx_session_create(None, 1, 1, None, ctypes.byref(h)) == t2sx_mod.ERR_INVALID
    assert L.t2sx_session_find_free_slot(None) == -1
    assert L.t2sx_session_slot_n_pos(None, 0) == -1
    assert L.t2sx_version() == 1


def test_weight_create_rejects_large_k(t2sx_mod):
    """K above 2048 (the few-row kernel's shared-memory bound) is rejected before any device work."""
    import ctypes
    L = t2sx_mod.lib()
    K = 2048 + 32
    buf = (ctypes.c_uint8 * (K // 32 * 34))()
    h = ctypes.c_void_p()
    assert L.t2sx_weight_create(0, 8, buf, 1, K, ctypes.byref(h)) == t2sx_mod.ERR_INVALID
    assert b"K above 2048" in L.t2sx_last_error()
    assert not h.value


def test_header_compiles_as_c_and_links(t2sx_mod, tmp_path):
    """include/t2sx.h is a C header: a C99 program (the kind a cgo or plain-C caller writes) compiles
    warning-free against it, links to the library and runs its host-side error paths without a GPU."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    assert gcc, "gcc is required to build the C program"
    src = tmp_path / "abi_c.c"
    src.write_text(
        '#include <stdio.h>\n'
        '#include "t2sx.h"\n'
        'int main(void) {\n'
        '    t2sx_model* m = 0;\n'
        '    if (t2sx_version() != 1) return 1;\n'
        '    if (t2sx_model_load(0, 0, &m) != T2SX_ERR_INVALID || m) return 2;\n'
        '    puts(t2sx_last_error());\n'
        '    return 0;\n'
        '}\n')
    exe = str(tmp_path / "abi_c")
    pkg = os.path.dirname(t2sx_mod.LIB_PATH)
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
                        str(src), "-L", pkg, "-lt2sx", f"-Wl,-rpath,{pkg}", "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.strip()
