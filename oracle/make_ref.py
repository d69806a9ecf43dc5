#!/usr/bin/env python
"""Builds the reference (bzzling/spar) CPU implementation from its own sources into
oracle/_ref/libspar_ref.so. TEST INFRASTRUCTURE: the library is the checker the oracle is pinned
against and the CPU baseline bench.py times; the product never loads it.

Spar is written as C++23 modules with `import std;` (CMakeLists.txt:3,39), which g++ 13 cannot
build, and the reference's own CMake build is not used. This recipe compiles the reference's
sources where they lie, after a mechanical module -> header rewrite done in a temporary
directory under oracle/_ref/ (removed after the build; only objects and the .so remain):
  * each module interface `X.cppm`: the global-module-fragment #includes are kept, `import std;`
    becomes the standard headers it stands for, `[export] import spar.Y;` becomes #include "spar.Y.hpp", every
    `export namespace ... { ... }` block goes (without `export`) into `X.hpp`; any remaining
    definitions (the backend modules' bodies) become a translation unit `X.iface.cpp`;
  * each implementation unit `*.cpp`: `module X;` becomes #include "X.hpp" and imports become
    includes.
Nothing else is changed. Three libraries come out of the same sources (VARIANTS below): the CPU
path (SPAR_ENABLE_CUDA=0), the drop-in build on libspar_b200.so, and the unchanged reference GPU
path. oracle/ref_driver.cpp (ours) exposes a C API over Spar's public API in each.

Usage: python oracle/make_ref.py [--src <reference checkout>/src] [--jobs N]
(default: $SPAR_REFERENCE_SRC, else the src/ of a `reference` checkout beside this repository)
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import re
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
CXX = os.environ.get("CXX", "g++")
FLAGS = ["-std=c++23", "-O2", "-fPIC", "-DSPAR_ENABLE_CUDA=0", "-w"]


def _strip_code(text: str) -> str:
    """Replaces comments, string and char literals by spaces (same length) so braces can be
    matched on the result while slicing the original text."""
    out = list(text)
    i, n = 0, len(text)
    while i < n:
        c = text[i]
        if text.startswith("//", i):
            j = text.find("\n", i)
            j = n if j < 0 else j
            for k in range(i, j):
                out[k] = " "
            i = j
        elif text.startswith("/*", i):
            j = text.find("*/", i + 2)
            j = n if j < 0 else j + 2
            for k in range(i, j):
                if text[k] != "\n":
                    out[k] = " "
            i = j
        elif c == '"' or c == "'":
            if c == '"' and i > 0 and text[i - 1] == "R":  # raw strings are not used in Spar
                raise ValueError("raw string literal")
            j = i + 1
            while j < n and text[j] != c:
                j += 2 if text[j] == "\\" else 1
            for k in range(i, min(j + 1, n)):
                out[k] = " "
            i = j + 1
        else:
            i += 1
    return "".join(out)


# Stands in for `import std;`: the standard headers the reference uses (bits/stdc++.h would drag
# in the C <stdatomic.h>, which g++ 13 rejects in C++23 mode).
STD_PRELUDE = "\n".join(f"#include <{h}>" for h in (
    "algorithm", "array", "atomic", "bit", "bitset", "cassert", "cctype", "chrono", "cmath",
    "compare", "concepts", "cstddef", "cstdint", "cstdio", "cstdlib", "cstring", "deque",
    "exception", "expected", "filesystem", "fstream", "functional", "initializer_list",
    "iomanip", "ios", "iostream", "istream", "iterator", "limits", "list", "map", "memory",
    "mutex", "new", "numbers", "numeric", "optional", "ostream", "queue", "random", "ranges",
    "set", "span", "sstream", "stack", "stdexcept", "string", "string_view", "system_error",
    "tuple", "type_traits", "typeinfo", "unordered_map", "unordered_set", "utility", "variant",
    "vector"))


def _include_for(module: str) -> str:
    return f'#include "{module}.hpp"'


IMPORT_RE = re.compile(r"^\s*(export\s+)?import\s+([\w.]+)\s*;\s*$", re.M)


def _imports_to_includes(text: str) -> str:
    def repl(m):
        mod = m.group(2)
        return "" if mod == "std" else _include_for(mod)
    return IMPORT_RE.sub(repl, text)


def convert_interface(path: Path, build: Path) -> tuple[str, Path | None]:
    text = path.read_text()
    m = re.search(r"^export\s+module\s+([\w.]+)\s*;\s*$", text, re.M)
    if not m:
        raise ValueError(f"{path}: no export module line")
    module = m.group(1)
    preamble = text[:m.start()]
    preamble = re.sub(r"^\s*module\s*;\s*$", "", preamble, flags=re.M)
    body = text[m.end():]
    code = _strip_code(body)
    exported, rest = [], []
    pos = 0
    for em in re.finditer(r"\bexport\s+namespace\b", code):
        if em.start() < pos:
            continue
        brace = code.find("{", em.end())
        depth, j = 0, brace
        while True:
            if code[j] == "{":
                depth += 1
            elif code[j] == "}":
                depth -= 1
                if depth == 0:
                    break
            j += 1
        rest.append(body[pos:em.start()])
        exported.append(body[em.start():j + 1].replace("export", "", 1))
        pos = j + 1
    rest.append(body[pos:])
    rest_text = "".join(rest)
    header = ["#pragma once", STD_PRELUDE, preamble.strip(),
              _imports_to_includes(rest_text_imports(rest_text))]
    header += exported
    (build / f"{module}.hpp").write_text("\n".join(header) + "\n")
    leftover = IMPORT_RE.sub("", rest_text)
    if _strip_code(leftover).strip():
        tu = build / f"{module}.iface.cpp"
        tu.write_text("\n".join([_include_for(module), preamble.strip(), leftover]) + "\n")
        return module, tu
    return module, None


def rest_text_imports(text: str) -> str:
    return "\n".join(m.group(0) for m in IMPORT_RE.finditer(text))


def convert_unit(path: Path, build: Path) -> Path:
    text = path.read_text()
    text = re.sub(r"^\s*module\s+([\w.]+)\s*;\s*$", lambda m: _include_for(m.group(1)), text,
                  count=1, flags=re.M)
    text = _imports_to_includes(text)
    rel = path.relative_to(path.parents[1])
    out = build / ("unit_" + str(rel).replace("/", "_"))
    out.write_text(STD_PRELUDE + "\n" + text)
    return out


def compile_one(src: Path, obj: Path, include: Path, flags: list[str]) -> None:
    subprocess.run([CXX, *flags, f"-I{include}", "-c", str(src), "-o", str(obj)], check=True)


CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
REPO = HERE.parent

# Variants (all TEST INFRASTRUCTURE, outputs under oracle/_ref/):
#   cpu   libspar_ref.so        the reference's CPU path (SPAR_ENABLE_CUDA=0): the oracle's pin and
#                               the CPU baseline.
#   b200  libspar_ref_b200.so   the reference built with SPAR_ENABLE_CUDA=1 as a Spar build that
#                               adopts the drop-in would be: src/backend/cuda_kernels.cu left out and
#                               libspar_b200.so linked in its place (its spar_cuda_* entry points),
#                               and the product's spar_b200/spar/cuda_blas.cppm compiled in place of
#                               src/backend/cuda_blas.cppm; the product's spar_b200/spar/fused.cppm
#                               (module spar.b200) added. Every other reference source unchanged.
#   stock libspar_ref_stock.so  the unchanged reference GPU path (its own cuda_kernels.cu, built
#                               with nvcc for sm_100a, and cuBLAS): the GPU bar, timed only.
VARIANTS = {"cpu": "libspar_ref.so", "b200": "libspar_ref_b200.so", "stock": "libspar_ref_stock.so"}


def _inputs(src: Path, variant: str) -> list[Path]:
    files = [*src.rglob("*.cppm"), *src.rglob("*.cpp"), *src.rglob("*.cu"), *src.rglob("*.hpp"),
             HERE / "ref_driver.cpp", Path(__file__)]
    if variant == "b200":
        files += [REPO / "spar_b200" / "spar" / "cuda_blas.cppm",
                  REPO / "spar_b200" / "spar" / "fused.cppm", *(REPO / "include").glob("*.h")]
    return files


def build_variant(src: Path, variant: str, jobs: int) -> Path:
    lib = OUT / VARIANTS[variant]
    inputs = _inputs(src, variant)
    if lib.exists() and lib.stat().st_mtime >= max(f.stat().st_mtime for f in inputs):
        return lib
    objdir = OUT / ("obj" if variant == "cpu" else f"obj_{variant}")
    objdir.mkdir(parents=True, exist_ok=True)
    build = Path(tempfile.mkdtemp(prefix="conv_", dir=OUT))
    flags = list(FLAGS)
    link: list[str] = []
    try:
        units = []
        glue = REPO / "spar_b200" / "spar" / "cuda_blas.cppm"
        interfaces = sorted(src.rglob("*.cppm"))
        if variant == "b200":  # the product's fused differentiable operations (module spar.b200)
            interfaces.append(REPO / "spar_b200" / "spar" / "fused.cppm")
        for cppm in interfaces:
            if variant == "b200" and cppm.is_relative_to(src) and \
                    cppm.relative_to(src).as_posix() == "backend/cuda_blas.cppm":
                cppm = glue  # the product's module in place of the reference's cuBLAS seam
            _, tu = convert_interface(cppm, build)
            if tu:
                units.append(tu)
        for cpp in sorted(src.rglob("*.cpp")):
            units.append(convert_unit(cpp, build))
        objs = [objdir / (u.stem + ".o") for u in units]
        if variant != "cpu":
            flags = [f for f in flags if not f.startswith("-DSPAR_ENABLE_CUDA")]
            flags += ["-DSPAR_ENABLE_CUDA=1", f"-I{CUDA_HOME / 'include'}"]
            link += [f"-L{CUDA_HOME / 'lib64'}", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}", "-lcudart"]
        if variant == "b200":
            # cuda_ops.cppm includes "cuda_kernels.hpp": here it resolves to the product's header.
            (build / "cuda_kernels.hpp").write_text('#include "spar_cuda_kernels.h"\n')
            flags += [f"-I{REPO / 'include'}", "-DSPAR_B200_FUSED=1"]
            link = [f"-L{REPO / 'spar_b200'}", "-l:libspar_b200.so",
                    "-Wl,-rpath,$ORIGIN/../../spar_b200", *link]
        if variant == "stock":
            flags += [f"-I{src / 'backend'}"]
            kernels_obj = objdir / "cuda_kernels.o"
            subprocess.run([str(CUDA_HOME / "bin" / "nvcc"), "-gencode",
                            "arch=compute_100a,code=sm_100a", "-O2", "-std=c++20", "-Xcompiler",
                            "-fPIC", "-c", str(src / "backend" / "cuda_kernels.cu"), "-o",
                            str(kernels_obj)], check=True)
            objs.append(kernels_obj)
            link += ["-lcublas"]
        driver = HERE / "ref_driver.cpp"
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
            futs = [pool.submit(compile_one, u, o, build, flags)
                    for u, o in zip(units, objs) if u.suffix != ".o"]
            futs.append(pool.submit(compile_one, driver, objdir / "ref_driver.o", build, flags))
            for f in futs:
                f.result()
        subprocess.run([CXX, "-shared", "-Wl,-Bsymbolic", "-o", str(lib), *map(str, objs),
                        str(objdir / "ref_driver.o"), *link], check=True)
    finally:
        shutil.rmtree(build, ignore_errors=True)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("SPAR_REFERENCE_SRC") or
                    str(HERE.parents[1] / "reference" / "src"))
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--variant", action="append", choices=sorted(VARIANTS),
                    help="default: all three")
    args = ap.parse_args()
    src = Path(args.src)
    if not src.is_dir():
        print(f"reference sources not found at {src}", file=sys.stderr)
        return 1
    OUT.mkdir(exist_ok=True)
    for variant in args.variant or ["cpu", "b200", "stock"]:
        print(build_variant(src, variant, args.jobs))
    return 0


if __name__ == "__main__":
    sys.exit(main())
