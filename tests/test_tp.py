"""Tensor parallelism: the row split (CPU) and 2-rank runs against the golden
token streams and a single-GPU run (GPU, needs 2 devices).

Each rank holds the rows qb_tp_rows gives it of every quantised matrix; a
GEMV stores its rows into every rank's copy of the output and ends with a
cross-rank barrier, so all ranks must hold the same activations and tokens.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, qb


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("rows", [1, 31, 32, 48, 1024, 5120, 6144, 17408, 248320])
def test_row_split_covers_rows_in_whole_tile_pairs(rows, world):
    ranges = [qb.tp_rows(rows, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == rows
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0   # contiguous, disjoint
    pairs = [((r1 - r0) + 31) // 32 if r1 > r0 else 0 for r0, r1 in ranges]
    for r0, r1 in ranges:
        assert r0 % 32 == 0 and r1 >= r0
    full = (rows + 31) // 32
    assert sum(pairs) == full
    assert max(pairs) - min(pairs) <= 1   # balanced to one tile pair


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


RANK = r"""
import os, sys, datetime
import numpy as np
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
import torch, torch.distributed as dist
from conftest import qb
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))

def rel(a, b):
    return float(np.linalg.norm(np.float64(a) - b) / max(np.linalg.norm(np.float64(b)), 1e-30))

def group(path, n_ctx):
    m = qb.Model(path, n_ctx, rank, world)
    hs = [None] * world
    dist.all_gather_object(hs, m.tp_handle())
    m.tp_connect(hs)
    dist.barrier()
    return m

def close(m):
    dist.barrier()   # no rank still writes into a peer
    m.close()
    dist.barrier()

for name, seed, profile in (("tiny_spec", 1, 0), ("tiny_mixed_spec", 2, 1)):
    g = np.load(os.path.join({root!r}, "tests", "golden", name + ".npz"))
    path = qb.write_synth_gguf(os.path.join({tmp!r}, f"{{name}}_{{rank}}.gguf"), qb.TINY, seed=seed, profile=profile)
    m = group(path, 256)
    m.prefill(g["prompt"], 1)
    r = rel(m.logits()[:64], g["prefill_logits64"])
    assert r < 1e-4, (name, r)
    toks, js = m.spec_generate(int(g["n_predict"]), 3, forced=g["forced"])
    assert np.array_equal(toks, g["tokens"]), (name, rank, toks[:16], g["tokens"][:16])
    assert np.array_equal(js, g["accept"]), (name, rank, js, g["accept"])
    close(m)

# full layer widths: the same tokens and logits as one GPU
path = qb.write_synth_gguf(os.path.join({tmp!r}, f"wide_{{rank}}.gguf"), qb.WIDE4, seed=4)
p = np.random.default_rng(7).integers(0, qb.WIDE4["vocab"], 12).astype(np.uint32)
forced = np.array([3, 0, 2, 1, 3, 3, 0, 1], np.uint32)
ref = None
if rank == 0:
    s = qb.Model(path, 128)
    s.prefill(p, 1)
    l0 = s.logits().copy()
    st, sj = s.spec_generate(24, 3, forced=forced)
    ref = (l0, st, sj, s.logits().copy())
    s.close()
obj = [ref]
dist.broadcast_object_list(obj, 0)
l0, st, sj, l1 = obj[0]
m = group(path, 128)
m.prefill(p, 1)
assert rel(m.logits(), l0) < 1e-5, rel(m.logits(), l0)
tt, tj = m.spec_generate(24, 3, forced=forced)
assert np.array_equal(tt, st) and np.array_equal(tj, sj), (tt, st, tj, sj)
assert rel(m.logits(), l1) < 1e-5, rel(m.logits(), l1)
close(m)
dist.destroy_process_group()
print("tp ok", rank)
"""


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_rank_tensor_parallel(tmp_path):
    code = RANK.format(root=ROOT, tmp=str(tmp_path))
    port = str(_free_port())
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=port,
                   NCCL_NVLS_ENABLE="0")
        env.pop("QB_TC", None)
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = []
    for pr in procs:
        try:
            outs.append(pr.communicate(timeout=900))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    bad = [(r, out[-2000:], err[-3000:]) for r, (pr, (out, err)) in enumerate(zip(procs, outs))
           if pr.returncode != 0 or f"tp ok {r}" not in out]
    assert not bad, bad
