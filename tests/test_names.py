"""Every global name a function in bench.py or the package reads is defined
(CPU only).  A name left undefined by an edit fails only when the code path
that reads it runs -- for bench.py's e2e and multi-GPU legs, only on a GPU
box -- so it is checked here from the symbol tables."""

from __future__ import annotations

import builtins
import symtable
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
FILES = [ROOT / "bench.py", ROOT / "__graft_entry__.py"] + sorted((ROOT / "phew_b200").rglob("*.py"))


def _undefined(path: Path) -> list[str]:
    src = path.read_text()
    top = symtable.symtable(src, str(path), "exec")
    defined = {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported()}
    defined |= set(dir(builtins)) | {"__file__", "__name__", "__doc__", "__spec__", "__path__"}
    bad = []

    def walk(t):
        for child in t.get_children():
            if child.get_type() in ("function", "class"):
                for s in child.get_symbols():
                    if (s.is_referenced() and s.is_global() and not s.is_declared_global()
                            and s.get_name() not in defined):
                        bad.append(f"{path.name}:{child.get_name()}: {s.get_name()}")
            walk(child)

    walk(top)
    return bad


@pytest.mark.parametrize("path", FILES, ids=lambda p: str(p.relative_to(ROOT)))
def test_no_undefined_globals(path):
    assert _undefined(path) == []
