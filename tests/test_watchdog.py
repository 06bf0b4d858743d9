"""The engine's no-progress detector (`fmd::ProgressWatch`, csrc/fmd_watch.h),
driven on the host with injected stalls.

`fmd_engine_step` polls the device counters every 16 steps and stops with
FMD_ETIMEDOUT after 4 polls in which neither generated tokens, prefilled rows
nor finished requests moved. The header is plain C++; this test compiles it
into a small harness that replays counter sequences -- a healthy run, a run
that stalls (the device stops advancing, as a stuck scheduler would), a stall
that recovers before the limit, and progress on only one counter -- and checks
when the detector fires. No GPU is involved.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "fast-moss-diarization_b200" / "csrc"

HARNESS = r"""
#include <cstdio>
#include "fmd_watch.h"
// stdin: the limit, then one poll per line "gen prefill done"; prints the
// 0-based index of the first poll that reports a stall, or -1.
int main() {
  int limit;
  if (std::scanf("%d", &limit) != 1) return 2;
  fmd::ProgressWatch w(limit);
  long long g, p, d;
  int i = 0;
  while (std::scanf("%lld %lld %lld", &g, &p, &d) == 3) {
    if (w.stalled(g, p, d)) { std::printf("%d\n", i); return 0; }
    ++i;
  }
  std::printf("-1\n");
  return 0;
}
"""


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    d = tmp_path_factory.mktemp("watch")
    src = d / "watch.cc"
    src.write_text(HARNESS)
    exe = d / "watch"
    subprocess.run([cxx, "-O1", "-std=c++17", "-I", str(CSRC), str(src), "-o", str(exe)], check=True)

    def run(polls, limit=4):
        text = f"{limit}\n" + "".join(f"{g} {p} {q}\n" for g, p, q in polls)
        return int(subprocess.run([str(exe)], input=text, capture_output=True, text=True, check=True).stdout)

    return run


def test_a_healthy_run_never_stalls(harness):
    assert harness([(16 * i, 100, i // 4) for i in range(200)]) == -1


def test_an_injected_stall_fires_after_four_idle_polls(harness):
    healthy = [(16 * i, 2048 * i, 0) for i in range(6)]
    stuck = [healthy[-1]] * 10  # the device stops advancing
    assert harness(healthy + stuck) == len(healthy) - 1 + 4


def test_a_stall_that_recovers_before_the_limit_is_not_reported(harness):
    polls = [(0, 0, 0), (16, 0, 0)] + [(16, 0, 0)] * 3 + [(32, 0, 0)] + [(32, 0, 0)] * 3 + [(48, 0, 1)]
    assert harness(polls) == -1


def test_progress_on_any_one_counter_counts(harness):
    # prefill rows only (a long prompt being chunked), then finished requests only
    polls = [(5, 2048 * i, 0) for i in range(8)] + [(5, 2048 * 8, i) for i in range(1, 8)]
    assert harness(polls) == -1


def test_the_limit_is_the_engines(harness):
    """The runtime passes kEngineIdlePolls = 4 polls of 16 steps each."""
    src = (CSRC / "fmd_runtime.cu").read_text()
    assert "constexpr int kEngineIdlePolls = 4;" in src and "ProgressWatch watch{kEngineIdlePolls};" in src
    # one detector per handle, reset when the engine starts: polls of several
    # short fmd_engine_step calls add up
    assert "h->watch = ProgressWatch(kEngineIdlePolls);" in src and "ProgressWatch& watch = h->watch;" in src
    assert harness([(1, 1, 1)] * 3, limit=2) == 2
