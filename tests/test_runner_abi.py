"""The C-ABI runner library loads without a GPU and exports every function
include/thompiler_runner.h declares; without a driver it reports an error
status instead of crashing."""

import ctypes
import re

from conftest import ROOT
from thompiler import runner


def declared():
    text = (ROOT / "include" / "thompiler_runner.h").read_text()
    return sorted(set(re.findall(r"^int\s+(thr_\w+)\s*\(", text, re.M)))


def test_header_declares_the_runner_calls():
    names = declared()
    for n in ("thr_init", "thr_module_load", "thr_get_function", "thr_launch", "thr_run", "thr_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = runner.library()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.thr_version() >= 1


def test_last_error_is_readable():
    lib = runner.library()
    buf = ctypes.create_string_buffer(64)
    assert lib.thr_last_error(buf, 64) == 0
