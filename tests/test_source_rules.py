"""Rules every source file of this repository keeps, checked on the CPU.

* None of the batched memcpy entry points of the CUDA runtime / driver:
  programs calling them raised GPU faults on the B200 driver in use.
* Kernels never trap: device-side failures are recorded in an error word and
  the kernel returns, so a failure never takes the GPU context down.
* Code and comments stand on their own: they do not point at the project's
  planning documents or at paths of a particular machine.

The banned strings are assembled at run time so this file does not contain
them itself.
"""

import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SKIP_DIRS = {".git", "build", "_work", "gpurun_out", "baseline", "__pycache__", ".pytest_cache"}
SOURCE_EXT = (".cu", ".cuh", ".h", ".hpp", ".cpp", ".cc", ".py", ".sh")

BATCH_MEMCPY = re.compile(r"[Mm]emcpy(3D)?" + "Batch" + "Async")
TRAP = re.compile(r"__" + r"trap\s*\(|\btrap\s*;")
PLAN_DOCS = re.compile(r"\b(" + "|".join(["SUR" + "VEY", "DE" + "SIGN", "BASE" + "LINE", "VER" + "DICT", "AD" + "VICE"])
                       + r")\." + "md")
MACHINE_PATH = re.compile(re.escape("/ro" + "ot/"))


def _sources():
    for dirpath, dirnames, filenames in os.walk(ROOT):
        dirnames[:] = [d for d in dirnames if d not in SKIP_DIRS and not d.startswith(".")]
        for name in filenames:
            if name.endswith(SOURCE_EXT):
                yield os.path.join(dirpath, name)


def _strip_c_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _hits(pattern, code_only=False, exts=SOURCE_EXT):
    bad = []
    for path in _sources():
        if not path.endswith(exts):
            continue
        with open(path, encoding="utf-8", errors="replace") as f:
            text = f.read()
        if code_only:
            text = _strip_c_comments(text)
        for lineno, line in enumerate(text.splitlines(), 1):
            if pattern.search(line):
                bad.append(f"{os.path.relpath(path, ROOT)}:{lineno}: {line.strip()[:120]}")
    return bad


def test_sources_found():
    files = list(_sources())
    assert any(p.endswith(".cu") for p in files) and any(p.endswith(".py") for p in files)


@pytest.mark.parametrize("name,pattern", [("batched memcpy", BATCH_MEMCPY)])
def test_banned_calls_absent(name, pattern):
    bad = _hits(pattern)
    assert not bad, f"{name} named in:\n" + "\n".join(bad)


def test_kernels_do_not_trap():
    bad = _hits(TRAP, code_only=True, exts=(".cu", ".cuh", ".h", ".hpp"))
    assert not bad, "trap in device code:\n" + "\n".join(bad)


@pytest.mark.parametrize("name,pattern", [("planning document", PLAN_DOCS), ("machine path", MACHINE_PATH)])
def test_sources_stand_alone(name, pattern):
    bad = _hits(pattern)
    assert not bad, f"{name} referenced in:\n" + "\n".join(bad)


def test_patterns_catch_examples():
    assert BATCH_MEMCPY.search("cuda" + "Memcpy" + "Batch" + "Async(")
    assert BATCH_MEMCPY.search("cu" + "Memcpy3D" + "Batch" + "Async(")
    assert TRAP.search("  __" + "trap();") and TRAP.search('asm("' + "trap" + ';");')
    assert not TRAP.search("bool trapped = false;")
    assert PLAN_DOCS.search("see " + "DE" + "SIGN" + ".md")
    assert MACHINE_PATH.search("/ro" + "ot/repo")
