"""The C ABI library loads and exports exactly what include/kvssd_b200.h declares.

No kernel is launched here; argument checks that run before any CUDA call are exercised.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
from conftest import ROOT

from kvssd_b200 import _native

HEADER = ROOT / "include" / "kvssd_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"KVSSD_B200_API\s+[\w\s\*]+?\b(kvssd_b200_\w+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared_functions() == set(_native.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _native.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == declared_functions(), "library exports only the declared ABI"


def test_version_and_status_strings():
    lib = _native.library()
    assert lib.kvssd_b200_version() == 1
    assert _native.status_string(0) == "ok"
    for s in range(1, 6):
        assert _native.status_string(s) not in ("ok", "unknown status")


def test_decode_rejects_null_pointers_before_touching_cuda():
    lib = _native.library()
    args = [None, 0, None, None, None, None, None, None, 1, 1, 8, 4, 2, 32, 4, 16, 0.1, None, None,
            None, 0, None]
    assert lib.kvssd_b200_decode(*args) == _native.ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.kvssd_b200_last_error()


def test_workspace_query_rejects_bad_geometry_before_touching_cuda():
    lib = _native.library()
    n = ctypes.c_size_t()
    cases = [
        ((1, 8, 4, 2, 32, 3, 16), b"bits"),
        ((0, 8, 4, 2, 32, 4, 16), b"at least one block"),
        ((1, 8, 4, 2, 32, 4, 12), b"divide"),
        ((1, 8, 3, 2, 32, 4, 16), b"divisible by KV heads"),
        ((1, 8, 4, 2, 36, 2, 6), b"pack-aligned"),
        ((1, 8, 4, 2, 2**31 - 1, 4, 1), b"packed dimension"),  # checked before head_dim <= 256
    ]
    for geom, msg in cases:
        assert lib.kvssd_b200_decode_workspace_size(*geom, ctypes.byref(n)) == _native.ERR_INVALID_ARGUMENT
        assert msg in lib.kvssd_b200_last_error()
    assert lib.kvssd_b200_decode_workspace_size(1, 8, 4, 2, 512, 4, 16, ctypes.byref(n)) == \
        _native.ERR_UNSUPPORTED


def test_path_selection_table():
    lib = _native.library()
    p = ctypes.c_int()
    expect = {(128, 4, 32): 1, (128, 2, 32): 1, (64, 4, 16): 1, (256, 4, 64): 1, (128, 4, 128): 1,
              (32, 4, 16): 2, (128, 4, 8): 2, (96, 4, 32): 2, (64, 2, 64): 1}
    for (d, bits, group), path in expect.items():
        assert lib.kvssd_b200_decode_path(d, bits, group, ctypes.byref(p)) == 0
        assert p.value == path, (d, bits, group)
    assert lib.kvssd_b200_set_path_override(2) == 0
    lib.kvssd_b200_decode_path(128, 4, 32, ctypes.byref(p))
    assert p.value == 2
    assert lib.kvssd_b200_set_path_override(1) == 0
    assert lib.kvssd_b200_decode_path(32, 4, 16, ctypes.byref(p)) == _native.ERR_UNSUPPORTED
    # the cp.async-fed streaming kernel is a member of the tensor-core family: same answers
    assert lib.kvssd_b200_set_path_override(_native.PATH_TENSOR_CORE_CPASYNC) == 0
    assert lib.kvssd_b200_decode_path(128, 4, 32, ctypes.byref(p)) == 0
    assert p.value == _native.PATH_TENSOR_CORE
    assert lib.kvssd_b200_decode_path(32, 4, 16, ctypes.byref(p)) == _native.ERR_UNSUPPORTED
    assert lib.kvssd_b200_set_path_override(0) == 0
    assert lib.kvssd_b200_set_path_override(5) == _native.ERR_INVALID_ARGUMENT
    assert lib.kvssd_b200_set_path_override(7) == _native.ERR_INVALID_ARGUMENT


def test_merge_and_dequant_argument_checks():
    lib = _native.library()
    assert lib.kvssd_b200_merge_chunks(None, None, 2, 4, 8, None, None, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.kvssd_b200_merge_pair(None, None, None, None, 4, 8, None, None, None) == \
        _native.ERR_INVALID_ARGUMENT
    dummy = ctypes.c_void_p(16)
    assert lib.kvssd_b200_dequantize(dummy, dummy, 4, 128, 3, 32, 0, dummy, dummy, None) == \
        _native.ERR_INVALID_ARGUMENT
    assert lib.kvssd_b200_dequantize(dummy, dummy, 3, 128, 4, 32, 1, dummy, dummy, None) == \
        _native.ERR_INVALID_ARGUMENT


def test_missing_library_fails_loudly(monkeypatch, tmp_path: Path):
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "absent.so")
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(RuntimeError, match="not built"):
        _native.library()
    assert not _native.available()


def test_documented_ctypes_stub_binds():
    """The ctypes binding that the integration guide gives kvssd maintainers loads this library,
    and its workspace query and error text work as written (host-side calls only)."""
    guide = (ROOT / "INTEGRATION.md").read_text()
    stub = re.search(r"```python\n(import ctypes, torch\n.*?)```", guide, re.S).group(1)
    stub = stub.replace('"/path/to/libkvssd_b200.so"', repr(str(_native.LIB_PATH)))
    scope: dict = {}
    exec(compile(stub, "INTEGRATION.md", "exec"), scope)
    lib = scope["_lib"]
    need = ctypes.c_size_t()  # a geometry refused before the query reaches the device
    assert lib.kvssd_b200_decode_workspace_size(1, 8, 4, 2, 32, 3, 16,
                                                ctypes.byref(need)) == _native.ERR_INVALID_ARGUMENT
    assert b"bits" in lib.kvssd_b200_last_error()  # restype c_char_p: the text, not an int
    assert callable(scope["fused_decode"])


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "kvssd_b200.h"

int main(void) {
  size_t bytes = 0;
  /* bits = 3 is refused before the query reaches the device */
  int st = kvssd_b200_decode_workspace_size(1, 8, 4, 2, 32, 3, 16, &bytes);
  if (st != KVSSD_B200_ERR_INVALID_ARGUMENT) return 1;
  if (!strstr(kvssd_b200_last_error(), "bits")) return 2;
  printf("%d|%s\n", kvssd_b200_version(), kvssd_b200_status_string(st));
  return 0;
}
"""


def test_plain_c_host_builds_and_links(tmp_path):
    """A C99 host (the language a cgo or JNI shim is written in) compiles against the header
    with -pedantic -Werror, links libkvssd_b200.so and calls its host-side entry points."""
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    lib_dir = _native.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", str(ROOT / "include"), str(src), "-o", str(exe), f"-L{lib_dir}",
                    "-lkvssd_b200", f"-Wl,-rpath,{lib_dir}"], check=True)
    done = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert done.returncode == 0, done.stderr
    version, text = done.stdout.strip().split("|", 1)
    assert int(version) == _native.library().kvssd_b200_version() and text


def test_every_declaration_states_its_reference_counterpart():
    """Each entry point's comment (its own, or that of the group it is declared in) cites the
    reference interface it replaces (file:line) or says it has none."""
    text = HEADER.read_text()
    comments = [(m.end(), m.group(0)) for m in re.finditer(r"/\*.*?\*/", text, re.S)]
    missing = []
    for m in re.finditer(r"KVSSD_B200_API\s+[\w\s\*]+?\b(kvssd_b200_\w+)\s*\(", text):
        before = [c for end, c in comments if end <= m.start()]
        comment = before[-1] if before else ""
        if not (re.search(r"\.(py|cu|cpp|h):\d", comment) or "counterpart" in comment):
            missing.append(m.group(1))
    assert not missing, missing


def test_integration_guide_lists_every_entry_point():
    """The integration guide's table names every exported function (groups may abbreviate the
    shared prefix, as in `kvssd_b200_ipc_handle` / `_open` / `_close`)."""
    guide = (ROOT / "INTEGRATION.md").read_text()
    missing = []
    for name in sorted(declared_functions()):
        if name in guide:
            continue
        stem, _, tail = name.rpartition("_")  # abbreviated: `<stem>_first` / `_<tail>`
        if f"`{stem}_" not in guide or f"`_{tail}`" not in guide:
            missing.append(name)
    assert not missing, missing
