"""Every relative import in the package -- including the lazy ones inside
functions, which only run on a GPU host (worker stages, calibration,
trainers) -- names a module that exists and, for ``from .x import name``,
a name that module defines.  Static (AST), so nothing is executed."""
import ast
import importlib
from pathlib import Path

PACKAGE = Path(__file__).resolve().parents[1] / "tempname_dcu_b200"


def _modules():
    for path in sorted(PACKAGE.rglob("*.py")):
        if "__pycache__" in path.parts:
            continue
        rel = path.relative_to(PACKAGE.parent).with_suffix("")
        parts = list(rel.parts)
        if parts[-1] == "__init__":
            parts = parts[:-1]
        yield path, ".".join(parts)


def test_relative_imports_resolve():
    problems = []
    for path, modname in _modules():
        package = modname if path.name == "__init__.py" else modname.rpartition(".")[0]
        for node in ast.walk(ast.parse(path.read_text())):
            if not isinstance(node, ast.ImportFrom) or node.level == 0:
                continue
            base = package.split(".")
            if node.level > 1:
                base = base[: len(base) - (node.level - 1)]
            target = ".".join(base + ([node.module] if node.module else []))
            try:
                mod = importlib.import_module(target)
            except ImportError as exc:
                problems.append(f"{path.name}:{node.lineno} from {'.' * node.level}{node.module or ''}: {exc}")
                continue
            for alias in node.names:
                if alias.name == "*" or hasattr(mod, alias.name):
                    continue
                try:
                    importlib.import_module(f"{target}.{alias.name}")
                except ImportError:
                    problems.append(f"{path.name}:{node.lineno} {target} has no {alias.name}")
    assert not problems, "\n".join(problems)
