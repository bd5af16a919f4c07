"""bench.py's CPU legs run end to end on a shrunken workload (no GPU needed): the ``--impl reference``
arm prints its JSON line and the ``cpu_baseline`` leg returns its object.  Both time the reference's
recurrence restated in torch (oracle/cpu_reference.py) on the host cores; here on one 128-token
sequence so that the check takes seconds, with every name the legs use resolved."""

import json
import types

import pytest
import torch

import bench
from archbench_b200.workloads import Config


@pytest.fixture()
def tiny_cfg1(monkeypatch):
    threads = torch.get_num_threads()
    monkeypatch.setitem(bench.CONFIGS, "cfg1", Config("cfg1", 1, 128, 1, 64, 64, torch.bfloat16, "shrunken for a test"))
    yield
    torch.set_num_threads(threads)  # the legs take every host core


def test_reference_arm_prints_one_line(tiny_cfg1, capsys, monkeypatch):
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    bench.run_reference(types.SimpleNamespace(steps=2, warmup=1))
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "tok/s"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cpu_baseline_leg(tiny_cfg1):
    out = bench.cpu_baseline(budget_s=0.05)
    assert out["value"] > 0 and out["unit"] == "tok/s" and out["kind"] == "port"
    assert "64-token slices" in out["sample"]
