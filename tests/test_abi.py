"""The C-ABI library loads without a GPU and exports every entry point that
include/gofish_b200.h declares (no compute call is made here)."""

import re
import subprocess
from pathlib import Path

from gofish_b200 import _native
from gofish_b200.build import LIBRARY, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "gofish_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gf_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    build()
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIBRARY)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    declared = declared_functions()
    assert declared, "no declarations parsed"
    missing = [name for name in declared if name not in exported]
    assert not missing, missing


def test_ctypes_binding_covers_the_header():
    assert sorted(_native.EXPORTED_SYMBOLS) == declared_functions()


def test_library_loads_and_reports_abi_version():
    lib = _native.load()
    assert lib.gf_abi_version() == 6


def test_create_rejects_bad_configuration():
    import ctypes

    lib = _native.load()
    cfg = _native.GfTracerConfig()
    cfg.k_buffer_size = 7
    assert not lib.gf_tracer_create(ctypes.byref(cfg))
    assert b"k_buffer_size" in lib.gf_last_error()
    cfg.k_buffer_size = 16
    cfg.sort_key = 5
    assert not lib.gf_tracer_create(ctypes.byref(cfg))
    cfg.sort_key = 0
    handle = lib.gf_tracer_create(ctypes.byref(cfg))
    assert handle
    lib.gf_tracer_destroy(handle)
