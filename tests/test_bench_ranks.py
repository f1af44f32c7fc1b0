"""The multi-rank arithmetic of bench.py on CPU: two gloo ranks report their
device time and token count; the whole-job value is the tokens of all ranks
(replicas) or of the one shared sequence (tensor parallelism) over the slowest
rank's time, the same on every rank."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

RANK = r"""
import os, sys, datetime, json
sys.path.insert(0, {root!r})
import torch.distributed as dist
import bench
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
ms = [800.0, 1000.0][rank]
tok = [500, 520][rank]
out = {{}}
for tp in (False, True):
    out[str(tp)] = bench.aggregate(ms, tok, tp, dist, "cpu")
dist.destroy_process_group()
print(json.dumps(out))
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_aggregate_like_the_driver_expects():
    import json
    code = RANK.format(root=ROOT)
    port = str(_free_port())
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=port)
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    res = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        assert p.returncode == 0, err[-2000:]
        res.append(json.loads(out.strip().splitlines()[-1]))
    for r, got in enumerate(res):
        v, ms_max, tok = got["False"]          # replicas: all ranks' tokens, slowest rank's time
        assert ms_max == 1000.0 and tok == 1020.0 and v == pytest.approx(1020.0)
        v, ms_max, tok = got["True"]           # tensor parallelism: one sequence
        assert ms_max == 1000.0 and tok == [500.0, 520.0][r] and v == pytest.approx(tok)


def test_single_rank_needs_no_collective():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.aggregate(250.0, 100, False) == (400.0, 250.0, 100.0)
