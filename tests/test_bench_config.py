"""bench.py's workloads stay inside the reference's defined domain (no GPU needed)."""
import importlib.util
import pathlib

ROOT = pathlib.Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_sweep_points_are_defined_and_cover_config3(O):
    b = _bench()
    for S, L, p, k in b.SWEEP:
        assert O.shape_defined(S, L, p, k), (S, L, p, k)
        assert b._sel_len(S, L, p, k) == O.sel_len(S, L, p, k)
    # k in {1536..6144} at p=4, L=3; L in {3,4,5} at p=2; p in {2,4,8} at L=3
    ks = {k for S, L, p, k in b.SWEEP if (L, p) == (3, 4)}
    assert ks == {1536, 2048, 3072, 4096, 6144}
    assert {L for S, L, p, k in b.SWEEP if (p, k) == (2, 1536)} == {3, 4, 5}
    assert {p for S, L, p, k in b.SWEEP if (L, k) == (3, 1536)} == {2, 4, 8}
    # where the reference is defined at S=131072 the sweep runs there
    for S, L, p, k in b.SWEEP:
        if S != 131072:
            assert not O.shape_defined(131072, L, p, k) or (131072, L, p, k) in b.SWEEP


def test_headline_workload_is_defined(O):
    b = _bench()
    c = b.CFG
    assert O.shape_defined(c["S"], c["L"], c["p"], c["k"])
    assert b._sel_len(c["S"], c["L"], c["p"], c["k"]) == 24576


def test_bench_functions_read_no_undefined_globals():
    """Every global name a bench.py function reads is defined at module level or
    is a builtin (a NameError in a rarely run --workload would otherwise only
    show on the GPU box)."""
    import builtins
    import symtable
    src = (ROOT / "bench.py").read_text()
    top = symtable.symtable(src, "bench.py", "exec")
    defined = set(top.get_identifiers()) | set(dir(builtins))
    missing = []

    def walk(tab):
        for child in tab.get_children():
            if child.get_type() == "function":
                for sym in child.get_symbols():
                    if sym.is_global() and sym.is_referenced() and sym.get_name() not in defined:
                        missing.append((child.get_name(), sym.get_name()))
            walk(child)

    walk(top)
    assert not missing, missing
