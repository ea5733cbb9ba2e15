"""Replays the reference's spec-driven argument validation for sgemm / dgemm, the
gemmtr family (sgemmtr, ssyrk, ssyr2k and their d twins), ssymm / strmm (and
d twins), strsm and sgemv / dgemv.

Follows tests/helpers/validation.js (runValidation, :455-560): a baseline
argument set is built from the specs in tests/golden/validation_params.json
(the reference's tests/validation/params/*.json); each invalid entry replaces
exactly one argument and must raise an error whose message contains the
entry's text, and each edge entry must not raise. The spec set per routine is
the one tests/sgemm/src/test.sgemm.js:23-56, tests/dgemm/src/test.dgemm.js:36-88,
tests/sgemmtr/src/test.sgemmtr.js, tests/ssyrk/src/test.ssyrk.js and
tests/ssyr2k/src/test.ssyr2k.js assemble (the d twins derive the Float64Array
specs the same way).
"""
from __future__ import annotations

import copy
import math

import numpy as np

from conftest import load_golden

SPECIALS = {
    "NaN": math.nan, "Infinity": math.inf, "-Infinity": -math.inf, "null": None,
    "undefined": None, "string": "100", "array": [], "object": {}, "number": 42,
}
_UNDEF = object()


def _derive64(spec):
    """derive64 (tests/helpers/validation.js:90-140) for the array specs B and C."""
    out = copy.deepcopy(spec)
    out["type"] = "float64array" if spec["type"] != "float" else "float64"
    for e in out.get("invalid", []):
        if isinstance(e.get("error"), str):
            e["error"] = e["error"].replace("Float32Array", "Float64Array")
    if spec["type"] == "float32array":
        out["invalid"].append({"scenario": "wrongDtypeGpuMatrix",
                               "error": "must be a Float64Array-backed GpuMatrix",
                               "label": "GpuMatrix backed by the wrong dtype (Float32Array)"})
    return out


def build_specs(routine: str) -> dict:
    P = load_golden("validation_params.json", decode=False)
    rank = routine[1:] in ("syrk", "syr2k")
    n_spec = copy.deepcopy(P["n"])
    n_spec["baseline"] = 2
    n_spec["edge"] = [e for e in n_spec["edge"] if e.get("value") != -1]
    n_spec["invalid"] = n_spec["invalid"] + [
        {"value": -1, "error": "must be non-negative" if rank else "m, n, and k must be non-negative",
         "label": "negative"}]
    m_spec = copy.deepcopy(P["m"])
    m_spec["baseline"] = 2
    a_base = copy.deepcopy(P["A"])
    lvl3 = a_base.pop("level-3")
    a_spec = {**a_base, **lvl3}
    if routine[1:] == "gemv":
        # tests/sgemv/src/test.sgemv.js:29-51 (tests/dgemv/src/test.dgemv.js the same at f64)
        n_spec = copy.deepcopy(P["n"])
        n_spec["edge"] = [e for e in n_spec["edge"] if e.get("value") != -1]
        n_spec["invalid"] = n_spec["invalid"] + [{"value": -1, "error": "n must be non-negative", "label": "negative"}]
        a_gemv = copy.deepcopy(P["A"])
        a_gemv.pop("level-3", None)
        specs = {"device": P["device"], "trans": P["trans"], "m": P["m"], "n": n_spec, "alpha": P["alpha"],
                 "beta": P["beta"], "lda": P["lda"], "A": a_gemv, "x": P["x"], "incx": P["incx"], "y": P["y"],
                 "incy": P["incy"], "layout": P["layout"]}
        if routine.startswith("d"):
            for name in ("A", "x", "y"):
                specs[name] = _derive64(specs[name])
        return specs
    if routine[1:] in ("symm", "trmm", "trsm"):
        # tests/ssymm/src/test.ssymm.js, tests/strmm/src/test.strmm.js and
        # tests/strsm/src/test.strsm.js:32-63 (strsm's A spec adds a fill of
        # well-conditioned triangles, which changes no validation outcome)
        n_spec["invalid"][-1]["error"] = "must be non-negative"
        specs = {"device": P["device"], "side": P["side"], "uplo": P["uplo"]}
        if routine[1:] in ("trmm", "trsm"):
            specs.update(transA=P["trans"], diag=P["diag"])
        specs.update(layout=P["layout"], m=m_spec, n=n_spec, alpha=P["alpha"])
        if routine[1:] == "symm":
            specs["beta"] = P["beta"]
        specs.update(A={**a_base, "dependsOn": ["m", "n", "lda", "side"]}, lda=P["ld"],
                     B={**copy.deepcopy(P["B"]), "dependsOn": ["m", "n", "ldb"]}, ldb=P["ld"])
        if routine[1:] == "symm":
            specs.update(C=copy.deepcopy(P["C"]), ldc=P["ld"])
    elif rank:
        specs = {"device": P["device"], "uplo": P["uplo"], "trans": P["trans"], "layout": P["layout"],
                 "n": n_spec, "k": P["k"], "alpha": P["alpha"], "beta": P["beta"],
                 "A": {**a_spec, "dependsOn": ["n", "k", "lda", "trans"]}, "lda": P["ld"]}
        if routine[1:] == "syr2k":
            specs["B"] = {**copy.deepcopy(P["B"]), "dependsOn": ["n", "k", "ldb", "trans"]}
            specs["ldb"] = P["ld"]
        specs["C"] = {**copy.deepcopy(P["C"]), "dependsOn": ["n", "ldc"]}
        specs["ldc"] = P["ld"]
    else:
        specs = {
            "device": P["device"], "transA": P["trans"], "transB": P["trans"], "layout": P["layout"],
            "m": m_spec, "n": n_spec, "k": P["k"], "alpha": P["alpha"], "beta": P["beta"],
            "A": a_spec, "lda": P["ld"], "B": P["B"], "ldb": P["ld"], "C": P["C"], "ldc": P["ld"],
        }
        if routine.endswith("gemmtr"):
            specs = {"device": specs.pop("device"), "uplo": P["uplo"], **specs}
    if routine.startswith("d"):
        a64 = copy.deepcopy(specs["A"])
        a64.pop("level-3", None)
        a64["type"] = "float64array"
        for e in a64["invalid"]:
            e["error"] = e["error"].replace("Float32Array", "Float64Array")
        a64["invalid"].append({"scenario": "wrongDtypeGpuMatrix",
                               "error": "must be a Float64Array-backed GpuMatrix",
                               "label": "GpuMatrix backed by the wrong dtype (Float32Array)"})
        specs["A"] = a64
        if "B" in specs:
            specs["B"] = {**_derive64(P["B"]), "dependsOn": specs["B"]["dependsOn"]}
        if "C" in specs:
            specs["C"] = {**_derive64(P["C"]), "dependsOn": specs["C"]["dependsOn"]}
    return specs


def _dtype(spec_type):
    return np.float64 if spec_type == "float64array" else np.float32


def _matrix_len(depends_on, dims):
    """ndArrayLen for a matrix spec (tests/helpers/validation.js:192-253)."""
    if "incx" in depends_on or "incy" in depends_on:  # a level-2 vector (validation.js ndArrayLen case 2)
        no_t = dims.get("trans", "no-transpose") == "no-transpose"
        inc_key = "incx" if "incx" in depends_on else "incy"
        length = (dims["n"] if no_t else dims["m"]) if inc_key == "incx" else (dims["m"] if no_t else dims["n"])
        return max(0, (length - 1) * dims[inc_key] + 1)
    ld_key = next(d for d in depends_on if d.startswith("ld"))
    trans_key = next((d for d in depends_on if d.startswith("trans")), None)
    cm = dims.get("layout") == "column-major"
    if "side" in depends_on:  # the square operand of symm / trmm: order m (left) or n (right)
        order = dims["m"] if dims.get("side", "left") == "left" else dims["n"]
        return max(0, (order - 1) * dims[ld_key] + order)
    if trans_key and "k" in depends_on:
        d1, d2 = [d for d in depends_on if d in ("m", "n", "k")]
        rows, cols = (dims[d2], dims[d1]) if cm else (dims[d1], dims[d2])
        no_t = dims.get(trans_key, "no-transpose") == "no-transpose"
        outer, inner = (rows, cols) if no_t else (cols, rows)
    elif "m" in depends_on:  # plain m x n (C)
        outer, inner = (dims["n"], dims["m"]) if cm else (dims["m"], dims["n"])
    else:  # n x n (the C of syrk / syr2k)
        outer = inner = dims["n"]
    return max(0, (outer - 1) * dims[ld_key] + inner)


def baselines(specs, device):
    b = {}
    for name, spec in specs.items():
        if "baseline" in spec:
            v = spec["baseline"]
            b[name] = np.array(v, _dtype(spec["type"])) if isinstance(v, list) else v
    b["device"] = device
    for name, spec in specs.items():
        if spec.get("type") not in ("float32array", "float64array") or name in b:
            continue
        deps = spec["dependsOn"]
        inc = next((d for d in deps if d.startswith("inc")), None)
        if inc:
            # applyTransBaselines + buildArrayBaselines (validation.js:469-511): level-2
            # vectors long enough for either trans, at the largest stride of the spec.
            length = (max(b["m"], b["n"]) - 1) * specs[inc]["range"]["max"] + 1
        else:
            length = _matrix_len(deps, dict(b, lda=specs["lda"]["range"]["max"]))
        b[name] = np.ones(length, _dtype(spec["type"]))
    return b


def resolve(entry, name, spec, base, make_wrong_dtype_matrix=None):
    if "scenario" in entry:
        sc = entry["scenario"]
        if sc == "wrongDtypeGpuMatrix":
            return make_wrong_dtype_matrix() if make_wrong_dtype_matrix else _UNDEF
        n = _matrix_len(spec["dependsOn"], base)
        if sc == "minimal":
            return np.ones(n, _dtype(spec["type"]))
        if sc == "tooShort":
            return np.ones(max(0, n - 1), _dtype(spec["type"]))
        raise ValueError(sc)
    if "special" in entry:
        return SPECIALS[entry["special"]]
    v = entry["value"]
    if isinstance(v, list) and spec.get("type") in ("float32array", "float64array"):
        return np.array(v, _dtype(spec["type"]))
    return v


def cases(routine, device, kind, make_wrong_dtype_matrix=None):
    """Yields (label, args, expected_error_or_None) for kind 'invalid' or 'edge'."""
    specs = build_specs(routine)
    base = baselines(specs, device)
    for name, spec in specs.items():
        for entry in spec.get(kind, []):
            v = resolve(entry, name, spec, base, make_wrong_dtype_matrix)
            if v is _UNDEF:
                continue
            args = dict(base)
            args[name] = v
            yield f"{name} {kind}: {entry.get('label', entry)}", args, entry.get("error")


def call(fn, a):
    if "incx" in a:  # gemv
        return fn(a["device"], a["trans"], a["m"], a["n"], a["alpha"], a["A"], a["lda"], a["x"], a["incx"], a["beta"],
                  a["y"], a["incy"], a["layout"])
    if "side" in a:  # symm / trmm
        if "diag" in a:
            return fn(a["device"], a["side"], a["uplo"], a["transA"], a["diag"], a["m"], a["n"], a["alpha"], a["A"],
                      a["lda"], a["B"], a["ldb"], a["layout"])
        return fn(a["device"], a["side"], a["uplo"], a["m"], a["n"], a["alpha"], a["A"], a["lda"], a["B"], a["ldb"],
                  a["beta"], a["C"], a["ldc"], a["layout"])
    if "trans" in a:  # syrk / syr2k
        if "B" in a:
            return fn(a["device"], a["uplo"], a["trans"], a["n"], a["k"], a["alpha"], a["A"], a["lda"], a["B"],
                      a["ldb"], a["beta"], a["C"], a["ldc"], a["layout"])
        return fn(a["device"], a["uplo"], a["trans"], a["n"], a["k"], a["alpha"], a["A"], a["lda"], a["beta"],
                  a["C"], a["ldc"], a["layout"])
    head = (a["device"], a["uplo"]) if "uplo" in a else (a["device"],)
    return fn(*head, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], a["A"],
              a["lda"], a["B"], a["ldb"], a["beta"], a["C"], a["ldc"], a["layout"])
