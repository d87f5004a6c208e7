"""Host-side pieces of bench.py that need no GPU: the clock record of the timed region and the
committed DRAM-traffic figures the roofline fields read."""
import json
import re
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def test_clock_summary_reports_median_max_and_active_reasons():
    import bench
    s = bench.ClockSampler(device=0)          # not entered: no nvidia-smi process is started
    rows = [
        "0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1312, 1965, 998.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1950, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active",
        "garbage line",
        "0, N/A, 1965, 0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    s.file.write("\n".join(rows) + "\n")
    got = s.summary()
    assert got["samples"] == 3
    assert got["sm_mhz"] == 1950.0
    assert got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap"]


def test_clock_summary_flags_thermal_and_hw_slowdown():
    import bench
    s = bench.ClockSampler(device=0)
    s.file.write("0, 1200, 1965, 900, 0x48, Active, Not Active, Active, Not Active\n")
    got = s.summary()
    assert got["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_every_traffic_key_bench_reads_is_committed():
    src = (ROOT / "bench.py").read_text()
    keys = set(re.findall(r'traffic_bytes\("([a-z0-9_]+)"\)', src))
    assert keys, "bench.py reads no traffic figure"
    table = json.loads((ROOT / "profiles" / "traffic.json").read_text())
    for k in sorted(keys):
        assert isinstance(table.get(k), int) and table[k] > 0, k


def test_launch_counts_match_the_layer_chain():
    # the default line's per-layer launch count on one GPU follows the kernels that
    # enqueue_layer_prefill launches (gyro-dx_b200/csrc/gx_abi.cu): router, top-k, the three
    # grouping kernels of launch_group, rotation + pack, two grouped GEMMs (the TMEM GEMM writes
    # the down operand itself, so the second pack runs only for the other GEMM), combine
    src = (ROOT / "bench.py").read_text()
    m = re.search(r"launches_per_layer = (\d+) if world == 1 else (\d+) if exchange == abi.GX_EP_PEER else (\d+)", src)
    assert m and tuple(map(int, m.groups())) == (9, 14, 12)
    abi_src = (ROOT / "gyro-dx_b200" / "csrc" / "gx_abi.cu").read_text()
    start = abi_src.index("gx_result enqueue_layer_prefill(")
    body = abi_src[start:abi_src.index("\n}\n", start)]
    calls = re.findall(r"(launch_[a-z_]+)\(", body)
    kernels = {"launch_router_logits": 1, "launch_topk": 1, "launch_group": 3, "launch_rotate_pack": 1,
               "launch_moe_gemm": 1, "launch_combine": 1}
    assert sorted(set(calls)) == sorted(set(kernels) | {"launch_pack_rows"}), calls
    assert sum(kernels[c] for c in calls if c in kernels) == 9
    assert "if (!gx::gemm_ts_routed(L.type)) GX_CUDA(gx::launch_pack_rows" in body
