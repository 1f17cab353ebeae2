"""The C-ABI boundary, checked without a GPU: libdiffrast.so loads, exports every
entry point include/diffrast.h declares (and the binding types each one), and
its host-only pieces agree with the oracle."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "diffrast.h")
LIB = os.path.join(ROOT, "mlx-swift-diffrast_b200", "diffrast", "libdiffrast.so")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^DR_API\s+[\w\s\*]*?\b(dr_\w+)\s*\(", src, re.M)))


def test_header_declares_the_reference_surface():
    names = declared()
    for op in ["rasterize", "interpolate", "texture", "antialias"]:
        assert f"dr_{op}_fwd" in names and f"dr_{op}_bwd" in names
    assert "dr_antialias_construct_topology_hash" in names
    assert "dr_texture_construct_mip" in names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "run mlx-swift-diffrast_b200/build.py (or __graft_entry__.build())"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (dr_\w+)$", out, re.M))
    assert set(declared()) <= exported, set(declared()) - exported
    lib = ctypes.CDLL(LIB)
    for n in declared():
        assert hasattr(lib, n)


def test_binding_types_every_symbol():
    from diffrast import _lib
    assert set(_lib.SIGNATURES) == set(declared())
    assert _lib.lib().dr_abi_version() == 2


def test_antialias_work_bytes():
    # 16 B of betas + 1 B of edge codes per pixel, the code bytes rounded up to 16.
    from diffrast import _lib
    f = _lib.lib().dr_antialias_work_bytes
    assert f(2, 3, 5) == 30 * 16 + 32
    assert f(32, 1024, 1024) == 32 * 1024 * 1024 * 17
    assert f(0, 4, 4) == 0 and f(1, -1, 4) == 0


def test_mip_layout_matches_oracle():
    import oracle
    from diffrast import _lib
    for shape in [(1, 2048, 2048, 4), (3, 12, 8, 2), (1, 1, 1, 1), (2, 64, 32, 3)]:
        for ml in (-1, 0, 2):
            n = ctypes.c_int()
            off = (ctypes.c_int64 * 32)()
            hh = (ctypes.c_int * 32)()
            ww = (ctypes.c_int * 32)()
            tot = ctypes.c_int64()
            st = _lib.lib().dr_texture_mip_layout(*shape, ml, ctypes.byref(n), off, hh, ww, ctypes.byref(tot))
            assert st == 0
            L, o2, h2, w2, t2 = oracle.mip_layout(*shape, ml)
            assert n.value == L and list(hh[:L]) == h2 and list(ww[:L]) == w2
            assert list(off[:L]) == o2 and tot.value == t2


def test_null_context_is_an_error_not_a_crash():
    from diffrast import _lib
    L = _lib.lib()
    assert L.dr_last_error(None) == b"null context"
    assert L.dr_rasterize_fwd(None, None, 0, None, 0, None, 0, 0, 0, None, None, None) == _lib.DR_EINVAL
    assert L.dr_ctx_create(0, None) == _lib.DR_EINVAL
    n = ctypes.c_int64(0)
    assert L.dr_ctx_set_raster_list_capacity(None, 10) == _lib.DR_EINVAL
    assert L.dr_ctx_raster_overflow(None, ctypes.byref(n)) == _lib.DR_EINVAL


def test_ctx_create_without_gpu_reports_status():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from diffrast import _lib
    h = ctypes.c_void_p()
    assert _lib.lib().dr_ctx_create(0, ctypes.byref(h)) == _lib.DR_ECUDA


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    import diffrast
    pos = torch.zeros(1, 3, 4)
    tri = torch.zeros(1, 3, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        diffrast.rasterize(pos, tri, (4, 4))


def test_first_call_path_does_not_deadlock():
    # The first op of a process creates the context before anything else has
    # loaded the library; that path must return (an error without a GPU).
    import sys
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from diffrast import _lib\n"
            "try:\n    _lib.ctx_for(0)\n    print('ctx')\n"
            "except _lib.DiffRastError as e:\n    print('err', e)\n") % os.path.join(ROOT, "mlx-swift-diffrast_b200")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith(("ctx", "err"))


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++11")])
def test_header_compiles_cleanly(lang, std):
    # A C or C++ host includes the header alone: no warnings, no extensions.
    cc = "gcc" if lang == "c" else "g++"
    r = subprocess.run([cc, "-x", lang, std, "-fsyntax-only", "-Wall", "-Wextra", "-pedantic", "-Werror",
                        os.path.join(ROOT, "include", "diffrast.h")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
