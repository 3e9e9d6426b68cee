"""Static check of the benchmark entry point: every name a function reads is
defined somewhere (its own scope, an enclosing one, the module or builtins),
so a path that only runs on a GPU box (the reference arm, the scaling runs)
cannot fail on a misspelt or missing variable."""

import builtins
import os
import symtable

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _undefined(path):
    src = open(path).read()
    top = symtable.symtable(src, path, "exec")
    module = {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported() or s.is_namespace()}
    bad = []

    def walk(t):
        for sym in t.get_symbols():
            if sym.is_global() and not sym.is_assigned() and sym.is_referenced():
                n = sym.get_name()
                if n not in module and not hasattr(builtins, n) and n not in ("__file__", "__name__", "__doc__"):
                    bad.append((t.get_name(), n))
        for c in t.get_children():
            walk(c)

    walk(top)
    return bad


def test_bench_py_has_no_undefined_names():
    assert _undefined(os.path.join(ROOT, "bench.py")) == []


def test_graft_entry_has_no_undefined_names():
    assert _undefined(os.path.join(ROOT, "__graft_entry__.py")) == []


def test_reference_arm_config_matches_the_preset():
    """The reference arm's model fields are written out in bench.py (so that its
    process imports nothing from this repository); they must be the preset's."""
    import importlib.util

    from llm_research_b200.models.presets import build_hlrt_config

    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    for preset, fields in bench.REFERENCE_FIELDS.items():
        cfg = build_hlrt_config(preset)
        for k, v in fields.items():
            assert getattr(cfg, k) == v, (preset, k)
