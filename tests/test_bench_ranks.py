"""bench.py's multi-GPU host logic on two CPU ranks (gloo): the path shards by sequence, so ranks share nothing
but the timing rule -- every rank times its own requests, the slowest rank's time is reported, and the whole-job
rate counts every rank's tokens.  The GPU work of each rank is the single-GPU path covered by the gpu tests."""
import json
import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_report_the_slowest_time_and_serve_their_own_requests(tmp_path):
    port = str(_free_port())
    outs = [str(tmp_path / f"rank{r}.json") for r in range(2)]
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ranks_worker.py"), str(r), "2", port, outs[r]])
             for r in range(2)]
    try:
        for p in procs:
            assert p.wait(timeout=180) == 0
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    res = [json.load(open(o)) for o in outs]
    expected = [110.0, 40.0, 60.5]   # element-wise max of the two ranks' (total, prefill, decode) times
    for r in res:
        assert r["got"] == expected
    assert res[0]["ids"] != res[1]["ids"]   # each rank streams its own prompt
    for r in range(2):
        assert res[r]["ids"] == bench.prompt_ids(1000 + r)[:16].tolist()
    assert res[1]["reference_arm"] == "returned"   # the reference arm runs on rank 0 alone


def test_whole_job_rate_counts_every_rank():
    assert bench.aggregate_rate(1, 640, 0.5) == pytest.approx(1280.0)
    assert bench.aggregate_rate(8, 640, 0.5) == pytest.approx(8 * 1280.0)


def test_rank_max_without_a_process_group_is_the_identity():
    assert bench.rank_max([3.0, 1.5], "cpu") == [3.0, 1.5]


def test_config3_sequences_shard_without_overlap():
    """BASELINE config 3 shards its 64 sequences evenly: every sequence is served by exactly one rank."""
    for world in (1, 2, 4, 8):
        served = [s for r in range(world) for s in bench.shard(64, r, world)]
        assert sorted(served) == list(range(64))
        assert all(len(bench.shard(64, r, world)) == 64 // world for r in range(world))


def test_chat_prompt_pins_its_system_prefix():
    """The config 3 / 4 prompts: a ChatML system prefix closing at exactly n_pin tokens, then break tokens."""
    ids = bench.chat_prompt(5, 512, 4608)
    assert len(ids) == 4608 and ids[0] == 151644 and ids[1] == 8948 and ids[510] == 151645 and ids[511] == 198
    body = ids[512:]
    gaps = [i for i, t in enumerate(body) if t == 198]
    assert len(gaps) > 4096 // 49


def test_clock_summary_reads_nvml_rows():
    """The clock record of a bench line: NVML samples (sm clock, max clock, event-reason bits as Active flags) give
    the median SM clock, the max clock and the names of the active throttle reasons."""
    c = bench.ClockSampler(0)
    bits = bench.ClockSampler.NVML_BITS
    for sm, reasons in ((1965, 0x0), (1950, 0x4), (1965, 0x0)):
        c.rows.append(["0", str(sm), "1965", "", hex(reasons)] +
                      ["Active" if reasons & b else "Not Active" for b in bits])
    s = c.summary()
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    assert bench.ClockSampler(0).summary()["reasons"] == ["unavailable"]
