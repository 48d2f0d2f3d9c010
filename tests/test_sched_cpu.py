"""The CTA-pair GEMM's work schedule (tt-flow_b200/csrc/pair_sched.h), on the CPU.

The header is plain C++ shared by the kernel, its launcher and the planner.
tests/native/sched_check.cpp includes it and checks, for every tile count up to
600 with 13 k-block counts, 6 pair counts and 4 slot budgets, under both split
policies: each (tile, k-block) is computed by exactly one work item; a split
tile's main pair owns k-blocks [0, kc) and waits on exactly the slots its
helpers write; every slot is written once; the busiest pair's load is the one
the planner's cost model reports and never above the plain data-parallel
schedule's.
"""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ is not available")
    exe = tmp_path_factory.mktemp("sched") / "sched_check"
    subprocess.run([gxx, "-std=c++17", "-O2", "-Wall", "-Werror", "-o", str(exe),
                    str(ROOT / "tests" / "native" / "sched_check.cpp")], check=True)
    return exe


def _run(exe, *args):
    r = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_every_k_block_once(checker):
    out = _run(checker, 600)
    assert "OK 748800 schedules" in out


def test_benchmark_shapes(checker):
    """The shapes of one GPU's share of the row-sharded workloads on 74 CTA pairs (B200)."""
    lines = {ln.split(":")[0]: ln for ln in _run(checker, 1).splitlines() if ln.startswith("T=")}
    # QKV at 1024 rows: 96 tiles on 74 pairs; the 22 tiles of the second wave are split with two parts each over
    # 44 of the 52 idle pairs.
    assert "rem=22 parts=2 kc=20 busiest=86 dp=128" in lines["T=96 KB=64"]
    # MLP down-projection at 4096 rows: 256 tiles of 256 k-blocks; the last 34 split in halves.
    assert "rem=34 parts=1 kc=128 busiest=896 dp=1024" in lines["T=256 KB=256"]
    # MLP down-projection at 1024 rows: 64 tiles, 10 idle pairs; one part per helper cannot cover 64 tiles, so the
    # plain schedule stays (helpers with 6-7 parts each measured slower than the idle pairs).
    assert "rem=0 parts=0 kc=0 busiest=256 dp=256" in lines["T=64 KB=256"]
    # 8192 rows: the gains are under 2 %, so no split.
    assert "rem=0" in lines["T=2048 KB=64"] and "rem=0" in lines["T=512 KB=256"]
