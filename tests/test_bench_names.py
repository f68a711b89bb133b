"""bench.py only runs on a GPU box, so a name that its functions use but never define would
surface there first.  This reads the file's syntax tree on CPU and checks that every name a
function loads is a local, a module-level definition or a builtin."""

import ast
import builtins
from pathlib import Path

BENCH = Path(__file__).resolve().parent.parent / "bench.py"


def _module_names(tree):
    names = set()
    for n in tree.body:
        if isinstance(n, (ast.FunctionDef, ast.ClassDef)):
            names.add(n.name)
        elif isinstance(n, (ast.Import, ast.ImportFrom)):
            names.update((a.asname or a.name).split(".")[0] for a in n.names)
        elif isinstance(n, (ast.Assign, ast.AnnAssign)):
            for t in n.targets if isinstance(n, ast.Assign) else [n.target]:
                if isinstance(t, ast.Name):
                    names.add(t.id)
    return names


def _local_names(fn):
    names = set()
    for node in ast.walk(fn):
        if isinstance(node, ast.Name) and isinstance(node.ctx, (ast.Store, ast.Del)):
            names.add(node.id)
        elif isinstance(node, ast.FunctionDef):
            names.add(node.name)
        elif isinstance(node, (ast.Import, ast.ImportFrom)):
            names.update((a.asname or a.name).split(".")[0] for a in node.names)
        elif isinstance(node, ast.arg):
            names.add(node.arg)
        elif isinstance(node, ast.ExceptHandler) and node.name:
            names.add(node.name)
    return names


def test_bench_functions_use_only_defined_names():
    tree = ast.parse(BENCH.read_text())
    known = _module_names(tree) | set(dir(builtins))
    for fn in (n for n in tree.body if isinstance(n, ast.FunctionDef)):
        used = {n.id for n in ast.walk(fn) if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Load)}
        assert not (used - _local_names(fn) - known), (fn.name, sorted(used - _local_names(fn) - known))
