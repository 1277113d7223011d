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
