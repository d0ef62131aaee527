"""bench.py's reporting pieces that need no GPU: every workload names a
known kind, the roofline traffic figures come from the committed ncu
summaries, and the algorithmic byte / flop counts of the projection
workloads follow their definitions."""
import bench


def test_workloads_have_known_kinds():
    kinds = {w.get("kind", "decode") for w in bench.WORKLOADS.values()}
    assert kinds <= {"decode", "mix", "qkv", "oproj", "prefill", "paging", "layer"}


def test_profiled_traffic_reads_the_committed_summaries():
    # plain line of a decode summary, keyed lines of the others
    assert bench.profiled_traffic("olmoe") > 2e9
    assert bench.profiled_traffic("qwen3-qkv") == 6.153e7
    assert bench.profiled_traffic("qwen3-oproj") == 4.623e7
    assert bench.profiled_traffic("olmoe-paging", "copy") == 9.774e8
    assert bench.profiled_traffic("no-such-workload") is None


def test_projection_byte_and_flop_counts():
    w = bench.WORKLOADS["qwen3-qkv"]
    hd = (32 + 2 * 8) * 128
    assert bench.qkv_bytes(w, 128) == 2 * (hd * 4096 + 128 * 4096 + 128 * hd)
    assert bench.qkv_flops(w, 128) == 2 * 128 * 4096 * hd
    o = bench.WORKLOADS["qwen3-oproj"]
    assert bench.qkv_bytes(o, 128) == 2 * 4096 * 4096 + 4 * 128 * 4096 + 4 * 128 * 4096
    assert bench.qkv_flops(o, 128) == 2 * 128 * 4096 * 4096


def test_stdout_is_exactly_one_json_line():
    """The reference arm (host cores, no GPU needed) prints one JSON line on
    stdout and nothing else; library output goes to stderr."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, str(repo / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-seconds", "1"], capture_output=True, text=True, timeout=600,
                         cwd=str(repo))
    assert res.returncode == 0, res.stderr[-2000:]
    lines = res.stdout.splitlines()
    assert len(lines) == 1, res.stdout[:2000]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0
