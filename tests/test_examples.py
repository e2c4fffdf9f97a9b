"""Examples (CPU): datasets and per-rollout MCP configs of the Wordle and Minesweeper examples,
argument defaults, and shell syntax of their serve / launch scripts."""
import importlib.util
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1] / "examples"


def _load(name):
    sys.path.insert(0, str(ROOT))
    spec = importlib.util.spec_from_file_location(f"ex_{name}", ROOT / name / "train.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_wordle_example_dataset():
    mod = _load("wordle")
    ds = mod.dataset(0)
    assert len(ds) > 2000
    item = ds[0]
    srv = item["mcp_config"]["mcpServers"]["wordle"]
    assert srv["args"][:2] == ["-m", "agent_factory_3_b200.envs.wordle"]
    assert srv["args"][-1] == item["target"] and len(item["target"]) == 5
    a = mod.base_args().parse_args([])
    assert a.group_size == 8 and a.server_urls.startswith("http")


def test_minesweeper_example_dataset():
    mod = _load("minesweeper")
    ds = mod.dataset(3, 1)
    assert len(ds) == 3 and len({d["board_seed"] for d in ds}) == 3
    args = ds[0]["mcp_config"]["mcpServers"]["minesweeper"]["args"]
    assert "--text" in args and args[args.index("--seed") + 1] == str(ds[0]["board_seed"])


@pytest.mark.parametrize("script", sorted(str(p) for p in ROOT.glob("*/*.sh")))
def test_example_scripts_parse(script):
    assert subprocess.run(["bash", "-n", script]).returncode == 0
