"""The C-ABI library loads and exports every function include/*.h declares
(no compute: these run without a GPU)."""
import ctypes
import glob
import os
import re

from conftest import ROOT

import kmamba_b200 as kb

DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?[\s\*]([a-z_][a-z0-9_]*)\s*\(",
                  re.M)


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        txt = re.sub(r"typedef[^;]*;", "", txt)
        # header-only helpers (static inline, as in the reference) are not exports
        txt = re.sub(r"static\s+inline[^;{]*\{.*?\n\}", "", txt, flags=re.S)
        for m in DECL.finditer(txt):
            name = m.group(1)
            if name in ("if", "while", "return", "sizeof"):
                continue
            names.add(name)
    return sorted(names)


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) > 40, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_symbols_have_c_linkage():
    out = os.popen(f"nm -D --defined-only {kb.LIB_PATH}").read()
    for n in ("om_scan1d_forward", "om_scan1d_backward", "scan1d", "scannd", "convnd",
              "om_convnd_forward", "km_wavefront_plan_create", "kmb_scan1d_fwd"):
        assert re.search(rf"\bT {n}$", out, re.M), n


def test_invalid_arguments_rejected_without_gpu(lib):
    a = kb.KmbScan1D()
    assert lib.kmb_scan1d_fwd(ctypes.byref(a)) == kb.KMB_EINVAL
    assert b"sizes" in lib.kmb_last_error()
    a.batch, a.L, a.D, a.N = 1, 4, 4, 200
    assert lib.kmb_scan1d_fwd(ctypes.byref(a)) == kb.KMB_EUNSUPPORTED
    lib.kmb_clear_error()
    assert lib.kmb_last_status() == 0


def test_ckpt_size(lib):
    assert lib.kmb_scan1d_ckpt_elems(8, 4096, 1536, 16) == 8 * (4096 // kb.KMB_SCAN1D_CHUNK) * 1536 * 16
    assert lib.kmb_scan1d_ckpt_elems(1, 17, 2, 3) == 3 * 2 * 3
    assert lib.kmb_scan1d_ckpt_elems(0, 17, 2, 3) == 0


def test_stream_and_sync_controls(lib):
    assert lib.kmb_get_sync() == 1
    lib.kmb_set_sync(0)
    assert lib.kmb_get_sync() == 0
    lib.kmb_set_sync(1)
    lib.kmb_set_stream(None)
    assert lib.kmb_get_stream() is None
