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
Nothing else is changed. The CUDA backend is disabled (SPAR_ENABLE_CUDA=0): the path pinned here
is the reference's CPU path. oracle/ref_driver.cpp (ours) exposes a C API over Spar's public API.

Usage: python oracle/make_ref.py [--src <reference checkout>/src] [--jobs N]
(default: $SPAR_REFERENCE_SRC, else the reference checkout this build environment provides)
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


def compile_one(src: Path, obj: Path, include: Path) -> None:
    subprocess.run([CXX, *FLAGS, f"-I{include}", "-c", str(src), "-o", str(obj)], check=True)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("SPAR_REFERENCE_SRC", "/root/reference/src"))
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    args = ap.parse_args()
    src = Path(args.src)
    if not src.is_dir():
        print(f"reference sources not found at {src}", file=sys.stderr)
        return 1
    OUT.mkdir(exist_ok=True)
    objdir = OUT / "obj"
    objdir.mkdir(exist_ok=True)
    build = Path(tempfile.mkdtemp(prefix="conv_", dir=OUT))
    try:
        units = []
        for cppm in sorted(src.rglob("*.cppm")):
            _, tu = convert_interface(cppm, build)
            if tu:
                units.append(tu)
        for cpp in sorted(src.rglob("*.cpp")):
            units.append(convert_unit(cpp, build))
        driver = HERE / "ref_driver.cpp"
        objs = [objdir / (u.stem + ".o") for u in units]
        with concurrent.futures.ThreadPoolExecutor(max_workers=args.jobs) as pool:
            futs = [pool.submit(compile_one, u, o, build) for u, o in zip(units, objs)]
            futs.append(pool.submit(compile_one, driver, objdir / "ref_driver.o", build))
            for f in futs:
                f.result()
        lib = OUT / "libspar_ref.so"
        subprocess.run([CXX, "-shared", "-o", str(lib), *map(str, objs),
                        str(objdir / "ref_driver.o")], check=True)
        print(lib)
    finally:
        shutil.rmtree(build, ignore_errors=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
