"""The C-ABI library loads without a GPU and exports every symbol include/*.h declares."""
import ctypes
import glob
import os
import re

from conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"GKV_API\s+[^;(]*?\b(gkv_\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_header_declares_the_abi():
    names = _declared()
    assert len(names) >= 40
    for must in ("gkv_pool_create", "gkv_upload_step", "gkv_kv_append", "gkv_paged_decode",
                 "gkv_compute_attention", "gkv_block_copy", "gkv_table_append_token", "gkv_sync"):
        assert must in names


def test_library_exports_every_declared_symbol():
    import glacier_kv

    lib = ctypes.CDLL(glacier_kv.LIB_PATH)
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_every_declared_symbol():
    from glacier_kv import _lib

    assert _declared() == set(_lib.SIGNATURES), (
        sorted(_declared() ^ set(_lib.SIGNATURES)))


def test_only_declared_symbols_are_exported():
    """The shim hides its internals (-fvisibility=hidden): nothing but the C ABI leaks."""
    import subprocess

    import glacier_kv

    out = subprocess.run(["nm", "-D", "--defined-only", glacier_kv.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    gkv = {n for n in exported if n.startswith("gkv_")}
    assert gkv == _declared()


def test_version_and_error_string():
    import glacier_kv

    assert "sm_100a" in glacier_kv.version()
    assert isinstance(glacier_kv.last_error(), str)


def test_integration_guide_binds_every_declared_symbol():
    """INTEGRATION.md's C# P/Invoke layer has a [LibraryImport] line for every entry point."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = set(re.findall(r'EntryPoint = "(gkv_\w+)"', doc))
    assert bound == _declared(), sorted(bound ^ _declared())
