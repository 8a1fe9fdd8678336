"""Source lint for rules the native code must keep on multi-GPU systems.

* No bulk tensor copy that fans one load out to several CTAs of a cluster:
  every entry point may run with peers' memory mapped, and such a copy whose
  tensor map reaches another GPU's memory must never be built. (The tcgen05
  commit with a CTA mask is a barrier arrive, not a load, and stays allowed.)
* None of the batched-memcpy runtime/driver entry points appear in any
  source file (they are not used by this project).
* Every ``mbarrier`` wait in the kernels goes through the bounded helper.
"""

from __future__ import annotations

import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]
SOURCES = [p for p in (ROOT / "koochak_b200" / "csrc").rglob("*") if p.suffix in (".cu", ".cuh", ".h", ".cpp")]


def _code(path: pathlib.Path) -> str:
    text = path.read_text()
    text = re.sub(r"//[^\n]*", "", text)
    return re.sub(r"/\*.*?\*/", "", text, flags=re.S)


def test_sources_found():
    names = {p.name for p in SOURCES}
    assert {"gemm.cu", "comm.cu", "sm100.cuh"} <= names


# The two halves of the forbidden instruction qualifier, kept apart so that
# this file does not itself contain it.
_BULK = "cp.async." + "bulk"
_FANOUT = "multi" + "cast"


def _joined_literals(code: str) -> str:
    """Code with adjacent string literals merged ("a" "b" -> "ab"), so a PTX
    statement split over several literals or lines reads as one."""

    return re.sub(r'"\s*\n?\s*"', "", code)


def test_no_cluster_fanout_bulk_copies():
    # One PTX statement runs to its ';': look for the fan-out qualifier
    # anywhere between a bulk copy's opcode and that ';', across lines.
    statement = re.compile(re.escape(_BULK) + r"[^;]*" + _FANOUT, re.S)
    bad = []
    for p in SOURCES:
        code = _joined_literals(_code(p))
        for m in statement.finditer(code):
            ln = code.count("\n", 0, m.start()) + 1
            bad.append(f"{p.name}:{ln}: {m.group(0)[:120]!r}")
    assert not bad, "bulk copies fanned out over a cluster are not allowed:\n" + "\n".join(bad)


def test_fanout_lint_sees_split_statements():
    split = ('asm volatile("' + _BULK + '.tensor.2d.shared::cluster.global"\n'
             '             ".' + _FANOUT + '::cluster [%0], [%1];");')
    statement = re.compile(re.escape(_BULK) + r"[^;]*" + _FANOUT, re.S)
    assert statement.search(_joined_literals(split))
    allowed = 'asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.' + _FANOUT + '::cluster.b64 [%0];");'
    assert not statement.search(_joined_literals(allowed))


def test_no_batched_memcpy_entry_points():
    pattern = re.compile("Memcpy" + r"(3D)?" + "Batch" + "Async")
    files = [p for p in ROOT.rglob("*") if p.suffix in (".cu", ".cuh", ".h", ".cpp", ".py") and ".git" not in p.parts
             and "_ref" not in p.parts and "_work" not in p.parts]
    bad = [str(p.relative_to(ROOT)) for p in files if pattern.search(p.read_text(errors="ignore"))]
    assert not bad, bad


def test_mbarrier_waits_are_bounded():
    raw_try_wait = []
    for p in SOURCES:
        code = _code(p)
        for ln, line in enumerate(code.splitlines(), 1):
            if "mbarrier.try_wait" in line and p.name != "sm100.cuh":
                raw_try_wait.append(f"{p.name}:{ln}")
    assert not raw_try_wait, "mbarrier waits must use the bounded helper in sm100.cuh: " + ", ".join(raw_try_wait)
