"""The C-ABI library: loads, exports every symbol the header declares, and its struct layout
matches the ctypes binding.  CPU only (no compute calls)."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from common_b200 import native
from tests.conftest import has_gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qwen3_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qw_[a-z_0-9]+)\s*\(", text)))


def test_header_declarations_match_binding():
    assert declared_functions() == sorted(native.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = native.load()
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (qw_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None


def test_abi_version_and_build_info():
    lib = native.load()
    assert lib.qw_abi_version() == 1
    assert b"sm_100a" in lib.qw_build_info()


def test_config_struct_layout_matches_c():
    src = r"""
    #include <stddef.h>
    #include <stdio.h>
    #include "qwen3_b200.h"
    int main(void) {
        printf("%zu %zu %zu %zu %zu\n", sizeof(qw_config), offsetof(qw_config, num_pages),
               offsetof(qw_config, reserved), offsetof(qw_config, rope_theta), offsetof(qw_config, eps));
        return 0;
    }
    """
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(src)
        subprocess.run(["/usr/bin/gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        vals = list(map(int, subprocess.run([exe], capture_output=True, text=True).stdout.split()))
    Q = native.QwConfig
    assert vals == [C.sizeof(Q), Q.num_pages.offset, Q.reserved.offset, Q.rope_theta.offset, Q.eps.offset]


def test_status_codes_match_header():
    text = open(HEADER).read()
    for code, name in native.STATUS_NAMES.items():
        m = re.search(rf"\b{name}\s*=\s*(\d+)", text)
        assert m and int(m.group(1)) == code, name


def test_null_arguments_are_rejected_without_a_device():
    lib = native.load()
    assert lib.qw_create(None, 0, 0, 1, None, None) == 1  # QW_ERR_ARG
    assert lib.qw_get_unique_id(None) == 1
    assert isinstance(lib.qw_last_error(None), bytes)
    lib.qw_destroy(None)


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_create_without_gpu_fails_loudly():
    cfg = native.make_config(64, 128, 1, 4, 2, 64, 100, 16)
    with pytest.raises(native.QwenError) as e:
        native.NativeModel(cfg)
    assert e.value.status in (4, 3)  # QW_ERR_CUDA (no device) / OOM


def test_missing_library_is_an_error(monkeypatch, tmp_path):
    monkeypatch.setattr(native, "_lib", None)
    monkeypatch.setattr(native, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        native.load()
