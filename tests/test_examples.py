"""The runtime demo (BASELINE config 1 flow) runs end to end for each codec."""

import importlib.util
import json
from pathlib import Path

import pytest


@pytest.mark.parametrize("codec", ["raw", "svd"])
def test_runtime_demo(tmp_path, codec, capsys):
    path = Path(__file__).resolve().parents[1] / "examples" / "runtime_demo.py"
    spec = importlib.util.spec_from_file_location("runtime_demo", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    module.main(["--output", str(tmp_path / "out"), "--codec", codec])
    report = json.loads((tmp_path / "out" / "result.json").read_text())
    assert report["status"] == "passed"
    limit = 0.0 if codec == "raw" else 0.05
    assert max(report["restart_relative_KV_errors"].values()) <= limit
