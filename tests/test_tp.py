"""Tensor parallelism: the vocabulary row split (CPU) and 2-rank runs against
the compiled reference engine and a single-GPU run (GPU, needs 2 devices).

Each rank keeps its share of the DeltaNet k-heads (with their v-heads),
attention q-/kv-heads and FFN columns, so the mixers and the FFN run on
local data; the out-projections and the down projection write partial sums
that every rank adds up in rank order; the output head splits over the
vocabulary: inside the decode loops each rank keeps its rows and the ranks
exchange their row maxima, elsewhere (and for the logits a decode call leaves
behind) every rank holds all rows.  All ranks must hold the same logits and
emit the same tokens as one GPU and as the reference.
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

from conftest import oracle

def single(path, shape, n_ctx, p, forced, n, reference):
    # logits after the prompt, tokens, accept lengths, logits after them, then
    # greedy tokens and the logits after those, on one GPU (or the reference)
    s = oracle.RefModel(path, n_ctx, 8) if reference else qb.Model(path, n_ctx)
    s.prefill(p, 1)
    l0 = s.logits().copy()
    st, sj = s.spec_generate(n, 3, forced=forced)
    l1 = s.logits().copy()
    sg = np.asarray(s.greedy_generate(6))
    out = (l0, np.asarray(st), np.asarray(sj), l1, sg, s.logits().copy())
    s.close()
    return out

for shape, name, seed, n_ctx, n, refs in ((qb.SMALL, "small", 3, 256, 40, (False, True)),
                                          (qb.WIDE4, "wide4", 4, 128, 24, (False,))):
    path = qb.write_synth_gguf(os.path.join({tmp!r}, f"{{name}}_{{rank}}.gguf"), shape, seed=seed)
    p = np.random.default_rng(7).integers(0, shape["vocab"], 12).astype(np.uint32)
    forced = np.array([3, 0, 2, 1, 3, 3, 0, 1], np.uint32)
    obj = [[single(path, shape, n_ctx, p, forced, n, r) for r in refs] if rank == 0 else None]
    dist.broadcast_object_list(obj, 0)
    m = group(path, n_ctx)
    m.prefill(p, 1)
    l0 = m.logits().copy()
    tt, tj = m.spec_generate(n, 3, forced=forced)
    l1 = m.logits().copy()
    tg = np.asarray(m.greedy_generate(6))
    l2 = m.logits().copy()
    close(m)
    for r, (s0, st, sj, s1, sg, s2) in zip(refs, obj[0]):
        who = (name, "reference" if r else "one GPU", rank)
        assert rel(l0, s0) < 1e-4, (who, rel(l0, s0))
        assert np.array_equal(tt, st) and np.array_equal(tj, sj), (who, tt, st, tj, sj)
        assert rel(l1, s1) < 1e-4, (who, rel(l1, s1))
        assert np.array_equal(tg, sg), (who, tg, sg)
        assert rel(l2, s2) < 1e-4, (who, rel(l2, s2))
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


LEAVE = r"""
import os, sys, time, datetime
import numpy as np
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
import torch, torch.distributed as dist
from conftest import qb, oracle
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
path = qb.write_synth_gguf(os.path.join({tmp!r}, f"small_{{rank}}.gguf"), qb.SMALL, seed=3)
m = qb.Model(path, 128, rank, world)
hs = [None] * world
dist.all_gather_object(hs, m.tp_handle())
m.tp_connect(hs)
dist.barrier()
p = np.random.default_rng(7).integers(0, qb.SMALL["vocab"], 12).astype(np.uint32)
m.prefill(p, 0)
first = m.greedy_generate(4)          # both ranks: a normal step
dist.barrier()                        # no kernel of either rank in flight from here
if rank == 1:
    dist.barrier()                    # rank 1 leaves: it takes no further step (and keeps its memory)
else:
    t0 = time.time()
    try:
        m.greedy_generate(4)
        raise SystemExit("rank 0: the step without its peer did not fail")
    except RuntimeError as e:
        msg = str(e)
    waited = time.time() - t0
    assert "tensor-parallel peer" in msg and "code 4" in msg, msg
    assert waited < 60, waited        # bounded: about one 2 s wait, not one per exchange
    # the context is still usable: device work through the C ABI and torch
    K, rows = 1024, 96
    raw = qb.synth_matrix(qb.GGML_IQ4_XS, rows, K, seed=1, d_sigma=0.01)
    x = qb.synth_normal(2 * K, seed=2).reshape(2, K)
    got = qb.gemv_batch(qb.tensor(raw, qb.GGML_IQ4_XS, K, rows), x)
    want = oracle.port_gemv(raw, qb.GGML_IQ4_XS, K, x)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-5
    assert float(torch.arange(10, device="cuda", dtype=torch.float32).sum()) == 45.0
    torch.cuda.synchronize()
    print("waited", round(waited, 2), "first", first.tolist(), flush=True)
    dist.barrier()
m.close()                             # each rank frees its own memory after the other is done with it
dist.destroy_process_group()
print("leave ok", rank)
"""


@pytest.mark.gpu
@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_rank_leaves_between_steps(tmp_path):
    """A rank that stops taking part between steps: the survivor's next
    exchange gives up after its bounded wait, the call returns the error
    (qb_last_error, code 4), and the device stays usable.  No GPU faults:
    the leaving rank stays alive and keeps its memory mapped; only host
    barriers (gloo) coordinate the ranks; no NVLink multicast is involved."""
    code = LEAVE.format(root=ROOT, tmp=str(tmp_path))
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
            outs.append(pr.communicate(timeout=600))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    bad = [(r, out[-2000:], err[-3000:]) for r, (pr, (out, err)) in enumerate(zip(procs, outs))
           if pr.returncode != 0 or f"leave ok {r}" not in out]
    assert not bad, bad
