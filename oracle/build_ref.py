"""Build the unmodified reference mtorch (CPU) into ``oracle/_ref/`` — test infrastructure only.

The reference's portable (non-macOS) build does not compile as shipped: two helpers,
``erf_approx_float`` (cpp/mtorch/core/tensor.cpp:3853) and ``sum_float16_as_float_contiguous``
(cpp/mtorch/core/tensor.cpp:1055), are defined only inside ``#if defined(MTORCH_USE_ACCELERATE)``
blocks but are used unconditionally (tensor.cpp:4445, 19725).  This script writes a
forced-include header into ``oracle/_ref/`` (never into the repository's history) that

* forward-declares ``half_bits_to_float`` (defined later in the same anonymous namespace),
* provides ``erf_approx_float`` by extracting the function text from the reference source at
  build time (so no reference source is committed here), and
* provides a scalar ``sum_float16_as_float_contiguous`` (the plain summation loop the
  reference uses when NEON is absent).

It then compiles ``tensor.cpp`` + ``module.cpp`` from where they lie with g++ (no edits, no
reference build system) into ``oracle/_ref/mtorch/_C<ext>`` and copies the pure-Python
``mtorch/__init__.py`` beside it, so ``sys.path.insert(0, 'oracle/_ref'); import mtorch`` gives
the reference's own CPU implementation.  Nothing under ``oracle/`` is part of the product.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
# The reference checkout: MTORCH_REFERENCE, else a "reference" folder beside this repository.
REF = Path(os.environ.get("MTORCH_REFERENCE", str(HERE.parent.parent / "reference")))


def _extract_function(source: str, signature: str) -> str:
    start = source.index(signature)
    depth = 0
    i = source.index("{", start)
    while True:
        c = source[i]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return source[start : i + 1]
        i += 1


def write_shim() -> Path:
    tensor_cpp = (REF / "cpp/mtorch/core/tensor.cpp").read_text()
    erf = _extract_function(tensor_cpp, "float erf_approx_float(float value)")
    shim = "\n".join(
        [
            "#pragma once",
            "#include <cstdint>",
            "#include <cmath>",
            "namespace mtorch { namespace {",
            "float half_bits_to_float(uint16_t value);",
            erf,
            "static float sum_float16_as_float_contiguous(const uint16_t* p, int64_t n) {",
            "  float s = 0.0f;",
            "  for (int64_t i = 0; i < n; ++i) s += half_bits_to_float(p[i]);",
            "  return s;",
            "}",
            "} }",
            "",
        ]
    )
    OUT.mkdir(parents=True, exist_ok=True)
    path = OUT / "shim.h"
    path.write_text(shim)
    return path


def built_module() -> Path:
    return OUT / "mtorch" / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def available() -> bool:
    return built_module().exists() and (OUT / "mtorch" / "__init__.py").exists()


def build(force: bool = False) -> Path:
    target = built_module()
    if available() and not force:
        return target
    if not REF.exists():
        raise FileNotFoundError(f"reference tree not found at {REF}")
    shim = write_shim()
    (OUT / "mtorch").mkdir(parents=True, exist_ok=True)
    objs = []
    for src in ("cpp/mtorch/core/tensor.cpp", "cpp/mtorch/python/module.cpp"):
        obj = OUT / (Path(src).stem + ".o")
        cmd = [
            "g++", "-std=c++20", "-O3", "-fPIC", "-w", "-c", str(REF / src), "-o", str(obj),
            "-I", str(REF / "cpp"), "-I", sysconfig.get_paths()["include"], "-include", str(shim),
        ]
        objs.append((cmd, obj))
    procs = [subprocess.Popen(c) for c, _ in objs]
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("reference compile failed")
    subprocess.check_call(["g++", "-shared", "-o", str(target)] + [str(o) for _, o in objs])
    shutil.copyfile(REF / "mtorch/__init__.py", OUT / "mtorch/__init__.py")
    for _, o in objs:
        o.unlink()
    return target


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
