"""The self-contained Python examples of docs/*.md run as written (CPU)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (file, index of the ```python block); the other blocks need a DDP model
# or a GPU
RUNNABLE = [("getting_started.md", 0), ("checkpointing.md", 0), ("determinism.md", 0), ("determinism.md", 1),
            ("entropy_reduction.md", 0)]


def _blocks(name):
    text = open(os.path.join(ROOT, "docs", name)).read()
    return re.findall(r"```python\n(.*?)```", text, flags=re.S)


@pytest.mark.parametrize("name,idx", RUNNABLE)
def test_doc_example_runs(name, idx, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    code = _blocks(name)[idx]
    exec(compile(code, f"docs/{name}[{idx}]", "exec"), {"__name__": "__doc_example__"})


def test_every_doc_is_listed_or_has_no_python():
    for name in sorted(os.listdir(os.path.join(ROOT, "docs"))):
        if name.endswith(".md"):
            assert isinstance(_blocks(name), list)


def test_example_commands_name_existing_modules_and_flags():
    """Every `python -m`/`torchrun -m` command of docs/examples.md names an
    app module that exists, and every --flag it passes is one that module
    (or bench.py) declares."""
    text = open(os.path.join(ROOT, "docs", "examples.md")).read()
    spans = re.findall(r"`([^`]*(?:-m mini_nangila_b200\.apps\.\w+|python bench\.py)[^`]*)`", text)
    assert len(spans) >= 20
    for cmd in spans:
        m = re.search(r"mini_nangila_b200\.apps\.(\w+)", cmd)
        path = os.path.join(ROOT, "mini_nangila_b200", "apps", m.group(1) + ".py") if m else os.path.join(ROOT, "bench.py")
        assert os.path.exists(path), cmd
        src = open(path).read()
        for flag in re.findall(r"(?<![\w-])(--[a-z][\w-]*)", cmd.split("mini_nangila_b200.apps.")[-1]):
            assert f'"{flag}"' in src, (cmd, flag)
