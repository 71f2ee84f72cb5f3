"""Host-side logic of bench.py that needs no GPU: the nvidia-smi index
mapping of the clock sampler, the parsing of its samples (median SM clock,
maximum, throttle reasons), and the byte counts of the decoder-attention
cases."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_smi_indices_follow_cuda_visible_devices(monkeypatch):
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    assert bench.smi_indices([0, 1, 2]) == [0, 1, 2]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "4,5,6,7")
    assert bench.smi_indices([0, 3]) == [4, 7]
    assert bench.smi_indices([0, 5]) == [4]  # past the visible list: dropped
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-1234,GPU-5678")  # UUIDs: left as given
    assert bench.smi_indices([1]) == [1]


def test_clock_summary_parses_samples(tmp_path):
    c = bench.Clocks([0, 1])
    c.path = str(tmp_path / "clocks.csv")
    rows = [
        "0, 1400, 1965, 950.1, 0x4, Not Active, Not Active, Not Active, Active",
        "1, 1420, 1965, 948.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1500, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
        "1, 1380, 1965, 990.0, 0x8, Active, Not Active, Not Active, Not Active",
    ]
    open(c.path, "w").write("\n".join(rows) + "\n")
    s = c.summary()
    assert s["samples"] == 4
    assert s["sm_mhz"] == 1410.0  # median of 1400, 1420, 1500, 1380
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_summary_inactive_or_empty(tmp_path):
    assert bench.Clocks([0], active=False).summary() is None
    c = bench.Clocks([0])
    c.path = str(tmp_path / "none.csv")
    assert c.summary() is None  # no file
    open(c.path, "w").write("")
    assert c.summary() is None  # no samples


def test_decoder_case_bytes():
    P, N, D = bench.DEC_P, bench.DEC_NK, bench.DEC_D
    cases = {c[0]: c for c in bench.decoder_cases(8)}
    # per-prompt K/V: queries in and out, K and V of every prompt, fp32
    assert cases["t2i_per_prompt_kv_8tok"][6] == 4 * (P * 8 * D * 2 + 2 * P * N * D)
    # shared K/V: one K and one V
    assert cases["t2i_shared_kv_8tok"][6] == 4 * (P * 8 * D * 2 + 2 * N * D)
    # image -> token: the image queries in and out dominate
    assert cases["i2t_8tok"][6] == 4 * (P * N * D * 2 + 2 * P * 8 * D)
    assert cases["t2i_shared_kv_8tok"][5] is True
