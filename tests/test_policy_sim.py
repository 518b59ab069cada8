"""The page-cache policy simulator (tests/policy_sim/cachesim.c, a design-time
tool kept with the tests)
compiles and replays known traces to known hit ratios: a cache that holds
every line hits on every repeat; admission makes a line's first two misses
read through once the cache is full; a one-slot cache never hits on
alternating lines."""
import os
import shutil
import subprocess

import numpy as np
import pytest

SIM = os.path.join(os.path.dirname(os.path.abspath(__file__)), "policy_sim", "cachesim.c")


@pytest.fixture(scope="module")
def sim(tmp_path_factory):
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    exe = str(tmp_path_factory.mktemp("sim") / "cachesim")
    subprocess.run(["gcc", "-O2", "-o", exe, SIM], check=True)
    return exe


def run(exe, tmp_path, batches, n_lines, slots, spec):
    t = str(tmp_path / "t.npy")
    ln = str(tmp_path / "t_len.npy")
    np.save(t, np.concatenate([np.asarray(b, dtype=np.int32) for b in batches]))
    np.save(ln, np.array([len(b) for b in batches], dtype=np.int64))
    out = subprocess.run([exe, t, ln, str(n_lines), str(slots), spec], check=True, capture_output=True, text=True)
    return [float(x) for x in out.stdout.split(":", 1)[1].split()]


def test_everything_fits(sim, tmp_path):
    b = list(range(100))
    for pol in ("seq", "warp32", "warpN"):
        h = run(sim, tmp_path, [b, b[::-1], b], 100, 128, f"{pol},1,1,0")
        assert h == [0.0, 1.0, 1.0], pol


def test_admission_reads_first_misses_through(sim, tmp_path):
    fill = list(range(64))               # fills the 64-slot cache: the hand goes round
    fresh = list(range(100, 110))
    h = run(sim, tmp_path, [fill, fresh, fresh, fresh], 200, 64, "seq,1,1,2")
    # first sight of `fresh` reads through, second inserts, third hits
    assert h == [0.0, 0.0, 0.0, 1.0]
    h = run(sim, tmp_path, [fill, fresh, fresh], 200, 64, "seq,1,1,0")  # no admission: second sight hits
    assert h == [0.0, 0.0, 1.0]


def test_sharded_lines_follow_their_owner(sim, tmp_path):
    b = list(range(32))
    h = run(sim, tmp_path, [b, b], 32, 16, "warpN,2,1,0")  # 2 shards x 16 slots hold the 32 lines
    assert h == [0.0, 1.0]
