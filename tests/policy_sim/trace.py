"""Line traces for the page-cache policy simulator (cachesim.c): the input
nodes of `n` minibatches of one trainer of a bench.py config, as int32 line ids
(rows of one cache line each), and with --ranks R the minibatches of R trainers
interleaved minibatch by minibatch, as the sharded cache sees them.

Usage: python trace.py c2 40 out_prefix [--ranks 8]
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [REPO, os.path.join(REPO, "gids-study_b200")]

import bench  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("config")
    ap.add_argument("n", type=int)
    ap.add_argument("out")
    ap.add_argument("--ranks", type=int, default=1)
    a = ap.parse_args()
    cfg = dict(bench.CONFIGS[a.config])
    per_rank = [list(bench.batch_stream(cfg, a.n, r, "cpu")) for r in range(a.ranks)]
    parts = [per_rank[r][i].numpy().astype(np.int32) for i in range(a.n) for r in range(a.ranks)]
    np.save(a.out + ".npy", np.concatenate(parts))
    np.save(a.out + "_len.npy", np.array([len(p) for p in parts], dtype=np.int64))
    print(len(parts), "minibatches,", sum(len(p) for p in parts), "line references")


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    main()
