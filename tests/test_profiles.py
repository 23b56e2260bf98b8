"""The committed ncu summaries under profiles/ that bench.py reads, and the capture commands they record (CPU only).

bench.py takes the roofline's DRAM traffic per GEMM launch from profiles/tc_gemm_cfg3_step_launches.json and the
fused attention kernels' traffic from profiles/fused_attention_cfg4_kernels.json: a malformed or implausible file
would put a wrong figure on every bench line. Every summary also records the command that produced it; those
commands must run committed files only and keep the GPU's clocks unlocked (`--clock-control none`)."""
import json
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PROFILES = ROOT / "profiles"


def test_step_launch_traffic_is_complete_and_plausible():
    d = json.loads((PROFILES / "tc_gemm_cfg3_step_launches.json").read_text())
    for key in ("traffic_bytes_per_launch", "read_bytes_per_launch", "write_bytes_per_launch",
                "algorithmic_bytes_per_launch", "launches", "source", "command"):
        assert key in d, key
    # one config-3 micro-batch: 147 GEMM launches
    assert d["launches"] == 147
    assert abs(d["read_bytes_per_launch"] + d["write_bytes_per_launch"] - d["traffic_bytes_per_launch"]) < 1e3
    # no operand re-read from DRAM: traffic within a few percent of the algorithmic bytes either way
    ratio = d["traffic_bytes_per_launch"] / d["algorithmic_bytes_per_launch"]
    assert 0.8 < ratio < 1.2, ratio
    assert (PROFILES / d["source"]).exists()


def test_attention_kernel_traffic_is_complete_and_plausible():
    d = json.loads((PROFILES / "fused_attention_cfg4_kernels.json").read_text())
    # algorithmic bytes at config 4 (96 matrices x 3072 x 64): forward 190 MB, backward 377 MB
    for kernel, algorithmic in (("fa_forward_kernel", 190e6), ("fb_backward_kernel", 377e6)):
        entry = d[kernel]
        assert abs(entry["dram_read_bytes"] + entry["dram_write_bytes"] - entry["dram_bytes"]) < 2e6
        assert 0.9 < entry["dram_bytes"] / algorithmic < 1.5, (kernel, entry["dram_bytes"])


def _commands(text: str):
    """The fenced command blocks of a summary, and a JSON file's `command` field."""
    blocks = re.findall(r"```\n(.*?)```", text, flags=re.S)
    return [line for b in blocks for line in b.splitlines() if line.strip()]


@pytest.mark.parametrize("path", sorted(PROFILES.glob("*.md")) + sorted(PROFILES.glob("*.json")),
                         ids=lambda p: p.name)
def test_profile_commands_run_committed_files_and_leave_clocks_alone(path):
    text = path.read_text()
    if path.suffix == ".json":
        data = json.loads(text)
        lines = [data["command"]] if isinstance(data, dict) and "command" in data else []
    else:
        lines = _commands(text)
    for line in lines:
        assert "_work/" not in line, line
        for ncu in re.findall(r"\bncu\b[^&|;]*", line):
            if " -i " in ncu:   # reading a report back needs no clock setting
                continue
            assert "--clock-control none" in ncu, line
        for script in re.findall(r"python\S* (\S+\.py)", line):
            assert (ROOT / script).exists(), script
