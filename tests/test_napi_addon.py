"""The Node-API addon (wgblas_b200/napi/wgblas_napi.c) and its JavaScript shim
(wgblas_b200/napi/js), checked on CPU: Node is not part of this image, so the
addon is compiled and linked here with warnings as errors, its undefined
symbols are checked against the documented Node-API functions, the C ABI and
the CUDA runtime, and the shim's calls are checked against the addon's export
table and its module imports against the files they name."""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NAPI = os.path.join(ROOT, "wgblas_b200", "napi")
JS = os.path.join(NAPI, "js")
sys.path.insert(0, os.path.join(ROOT, "wgblas_b200"))

# Node-API functions the addon may import (js_native_api.h / node_api.h, NAPI_VERSION <= 8).
DOCUMENTED_NAPI = {
    "napi_call_threadsafe_function", "napi_create_arraybuffer", "napi_create_double", "napi_create_error",
    "napi_create_external", "napi_create_function", "napi_create_int32", "napi_create_int64",
    "napi_create_object", "napi_create_promise", "napi_create_string_utf8", "napi_create_threadsafe_function",
    "napi_create_typedarray", "napi_get_arraybuffer_info", "napi_get_cb_info", "napi_get_last_error_info",
    "napi_get_null", "napi_get_typedarray_info", "napi_get_undefined", "napi_get_value_bool",
    "napi_get_value_double", "napi_get_value_external", "napi_get_value_int32", "napi_get_value_int64",
    "napi_is_arraybuffer", "napi_is_exception_pending", "napi_is_typedarray", "napi_ref_threadsafe_function",
    "napi_reject_deferred", "napi_release_threadsafe_function", "napi_resolve_deferred",
    "napi_set_named_property", "napi_throw_error", "napi_throw_type_error", "napi_typeof",
    "napi_unref_threadsafe_function",
}


def _source():
    with open(os.path.join(NAPI, "wgblas_napi.c")) as fh:
        return fh.read()


def _exports():
    table = _source().split("kExports[] = {", 1)[1].split("};", 1)[0]
    return dict(re.findall(r'\{"(\w+)",\s*(\w+)\}', table))


def _js_files():
    for d, _, files in os.walk(JS):
        for f in files:
            if f.endswith(".mjs"):
                yield os.path.join(d, f)


@pytest.fixture(scope="module")
def addon_so(tmp_path_factory):
    import build

    build.build()
    out = str(tmp_path_factory.mktemp("napi") / "wgblas_napi.node")
    r = subprocess.run(build.napi_command(out), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def test_addon_compiles_and_links_with_warnings_as_errors(addon_so):
    assert os.path.getsize(addon_so) > 0


def test_addon_exports_the_module_entry_points(addon_so):
    out = subprocess.run(["nm", "-D", "--defined-only", addon_so], capture_output=True, text=True).stdout
    names = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert "napi_register_module_v1" in names
    assert "node_api_module_get_api_version_v1" in names
    assert not [n for n in names if n.startswith("js_")], "internal functions leaked into the dynamic table"


def test_addon_imports_only_documented_napi_the_c_abi_and_cuda(addon_so):
    out = subprocess.run(["nm", "-D", "--undefined-only", addon_so], capture_output=True, text=True).stdout
    undefined = {line.split()[-1].split("@")[0] for line in out.splitlines() if line.strip()}
    with open(os.path.join(ROOT, "include", "wgblas.h")) as fh:
        abi = set(re.findall(r"\b(wg_\w+)\s*\(", fh.read()))
    libc = {"memcpy", "memset", "snprintf", "calloc", "free", "strlen", "__stack_chk_fail", "__cxa_finalize",
            "_ITM_deregisterTMCloneTable", "_ITM_registerTMCloneTable", "__gmon_start__", "__snprintf_chk",
            "__memcpy_chk"}
    for name in undefined:
        if name.startswith("napi_"):
            assert name in DOCUMENTED_NAPI, name
        elif name.startswith("wg_"):
            assert name in abi, f"{name} is not declared in include/wgblas.h"
        elif name.startswith("cuda"):
            continue
        else:
            assert name in libc, name


def test_every_status_of_a_napi_call_is_checked():
    """No Node-API call's status is dropped: each call is inside NAPI_CALL, an `if`
    / `==` / `!=` test, an assignment, or a return."""
    body = _source().split("/* ---- status plumbing", 1)[1]
    for m in re.finditer(r"\bnapi_(?!value\b|env\b|status\b|ref\b|deferred\b|callback\w*\b|threadsafe_function\b|"
                         r"finalize\b|valuetype\b|typedarray_type\b|extended_error_info\b|tsfn_\w+|ok\b|"
                         r"\w+_array\b|undefined\b|null\b|boolean\b|number\b|string\b|symbol\b|object\b|"
                         r"function\b|external\b|bigint\b|register_module_v1\b)(\w+)\(", body):
        line_start = body.rfind("\n", 0, m.start()) + 1
        line = body[line_start:body.find("\n", m.start())]
        before = body[max(0, m.start() - 40):m.start()]
        ok = ("NAPI_CALL" in line or re.search(r"(if \(|==|!=|&&|\|\||= |return )", before[-20:]) is not None
              or line.strip().startswith(("napi_reject_deferred", "napi_resolve_deferred", "napi_throw_error",
                                          "napi_throw_type_error", "napi_release_threadsafe_function",
                                          "napi_unref_threadsafe_function", "napi_call_threadsafe_function")))
        assert ok, f"unchecked status: {line.strip()}"


def test_shim_calls_exactly_the_exported_functions():
    exports = set(_exports())
    used = set()
    for path in _js_files():
        with open(path) as fh:
            used |= set(re.findall(r"\baddon\.(\w+)\(", fh.read()))
    assert used <= exports, f"the shim calls functions the addon does not export: {used - exports}"
    assert exports - used <= set(), f"exported but never called from the shim: {exports - used}"


def test_shim_imports_resolve_and_package_exports_exist():
    import json

    for path in _js_files():
        with open(path) as fh:
            for spec in re.findall(r'from\s+"(\.{1,2}/[^"]+)"', fh.read()):
                target = os.path.normpath(os.path.join(os.path.dirname(path), spec))
                assert os.path.exists(target), f"{path}: {spec}"
    with open(os.path.join(JS, "package.json")) as fh:
        pkg = json.load(fh)
    for sub, target in pkg["exports"].items():
        assert os.path.exists(os.path.join(JS, target)), sub
    # the reference's public names are all exported by index.mjs
    with open(os.path.join(JS, "index.mjs")) as fh:
        index = fh.read()
    for name in ("init", "cleanup", "gpuName", "sgemm", "dgemm", "GpuMatrix", "GpuVector",
                 "randomFloat32Array", "randomFloat64Array"):
        assert re.search(rf"\b{name}\b", index), name


def test_shim_error_messages_match_the_python_mirror():
    """The shim's validation messages are the reference's, the same strings the
    Python mirror raises (wgblas_b200/gemm.py, classes.py, _runtime.py)."""
    py = ""
    for f in ("gemm.py", "classes.py", "_runtime.py"):
        with open(os.path.join(ROOT, "wgblas_b200", f)) as fh:
            py += fh.read()
    js = ""
    for path in _js_files():
        with open(path) as fh:
            js += fh.read()
    for msg in ("transA must be 'no-transpose' or 'transpose'.", "m, n, and k must be non-negative.",
                "lda, ldb, and ldc must be positive.", "C must be a GpuMatrix when A or B is a GpuMatrix.",
                "A and B must be GpuMatrix when C is a GpuMatrix.", "device must be a GPUDevice.",
                "m, n, k, lda, ldb, and ldc must be integers.", "rows must be a positive integer.",
                "data does not have enough elements for the given rows, cols, and lda.",
                "belongs to a different GPUDevice than the one passed in."):
        assert msg in py and msg in js, msg
