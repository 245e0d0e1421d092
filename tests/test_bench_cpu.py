"""CPU checks of bench.py's bookkeeping: the roofline `traffic` figure is
read from a committed ncu summary only while that summary's source digest
matches the kernel's sources in this tree, and the latest capture in a
summary wins.  Nothing is timed and no kernel is launched."""

from __future__ import annotations

import sys

from conftest import REPO

sys.path.insert(0, str(REPO))
import bench  # noqa: E402


def write_profile(tmp_path, digest: str, values=(123, 456)) -> str:
    lines = ["# test profile", ""] + [f"dram_bytes_per_launch: {v}" for v in values] + [f"kernel_sources: {digest}"]
    (tmp_path / "x_canonical.md").write_text("\n".join(lines) + "\n")
    return "x_canonical.md"


def test_digest_covers_included_headers():
    # decode_step.cuh includes qkv_fused.cuh: a different set of files gives a different digest
    assert bench.kernel_source_digest("decode_step.cuh") != bench.kernel_source_digest("qkv_fused.cuh")
    assert bench.kernel_source_digest("decode_step.cuh") == bench.kernel_source_digest("decode_step.cuh")


def test_traffic_needs_a_matching_digest(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    (tmp_path / "profiles").mkdir()
    monkeypatch.setattr(bench, "KERNEL_HEADERS", {"x": "decode_step.cuh"})
    good = bench.kernel_source_digest("decode_step.cuh")
    name = write_profile(tmp_path / "profiles", good)
    assert bench.ncu_traffic("x", name) == 456.0  # the last capture
    write_profile(tmp_path / "profiles", "0" * 16)
    assert bench.ncu_traffic("x", name) is None  # stale: captured from other sources
    assert bench.ncu_traffic("x", "missing.md") is None

