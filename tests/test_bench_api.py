"""bench.py's decode leg drives cppinf_b200.qwen3.Qwen3Model, and only runs on a GPU. This checks on the CPU that every
use of the model in bench.py matches the class: properties read as attributes, methods called."""
import ast
import inspect
from pathlib import Path

from cppinf_b200.qwen3 import Qwen3Model

REPO = Path(__file__).resolve().parent.parent


def _members():
    props, methods = set(), set()
    for name, value in inspect.getmembers(Qwen3Model):
        if isinstance(value, property):
            props.add(name)
        elif callable(value) and not name.startswith("__"):
            methods.add(name)
    return props, methods


def test_bench_uses_qwen3_model_members_as_declared():
    props, methods = _members()
    assert "step_launches" in props and "decode" in methods
    tree = ast.parse((REPO / "bench.py").read_text())
    seen = 0
    for fn in ast.walk(tree):
        if not isinstance(fn, ast.FunctionDef) or not _binds_model(fn):
            continue
        parents = {child: node for node in ast.walk(fn) for child in ast.iter_child_nodes(node)}
        for node in ast.walk(fn):
            if not (isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id == "model"):
                continue
            parent = parents.get(node)
            called = isinstance(parent, ast.Call) and parent.func is node
            if node.attr in props:
                assert not called, f"bench.py:{node.lineno} calls the property Qwen3Model.{node.attr}"
            else:
                assert node.attr in methods, f"bench.py:{node.lineno} uses Qwen3Model.{node.attr}, which it lacks"
            seen += 1
    assert seen > 0


def _binds_model(fn):
    """Whether the function assigns `model = Qwen3Model(...)`."""
    for node in ast.walk(fn):
        if (isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "model" for t in node.targets)
                and isinstance(node.value, ast.Call) and isinstance(node.value.func, ast.Name)
                and node.value.func.id == "Qwen3Model"):
            return True
    return False
