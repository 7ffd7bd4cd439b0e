"""The C-ABI library loads on a machine without a GPU and exports every symbol that
``include/*.h`` declares (no compute calls)."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re

from conftest import PKG_DIR, ROOT


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(pnb_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_entry_points():
    names = _declared_symbols()
    for must in ("pnb_keygen", "pnb_pbs_batch", "pnb_keyswitch", "pnb_lwe_contract",
                 "pnb_encrypt_lwe", "pnb_phase_lwe", "pnb_test_vector"):
        assert must in names


def test_library_exports_every_declared_symbol():
    path = os.path.join(PKG_DIR, "libpenumbra_b200.so")
    assert os.path.exists(path), "build the library first (make -C penumbra-fhe_b200)"
    lib = C.CDLL(path)
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"symbols declared but not exported: {missing}"


def test_error_path_without_gpu(pnb):
    # A NULL output pointer is rejected before any device work, with a readable message.
    L = pnb.lib()
    rc = L.pnb_keygen(0, None, 0, None)
    assert rc == 1
    assert b"NULL" in L.pnb_last_error()
    p = pnb.default_params()
    assert (p.n, p.k, p.N, p.pbs_base_log, p.pbs_level, p.ks_base_log, p.ks_level) == \
        (834, 1, 2048, 23, 1, 3, 5)
