"""qb_argmax_rows_noalloc: the allocation-free greedy argmax on device rows.

Checked against model_sample_greedy (the reference-named entry point, which
scans host logits through library-allocated scratch) on two calls in a row,
the second with smaller maxima so that keys left over from the first call
would give wrong indices.  Runs last so that it also sees a device the other
tests have used; it passes alone as well.
"""
import numpy as np
import pytest

from conftest import qb

pytestmark = pytest.mark.gpu


def _rows(seed, rows, n, scale):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, n)) * scale).astype(np.float32)
    x[0, 7] = x[0, 4099] = x[0].max() + 1.0          # tie: the first maximum wins
    x[1] = -np.abs(x[1]) - 1.0                        # all negative
    x[2, :] = -np.inf
    x[2, n - 1] = -1e30                               # maximum at the last entry
    return x


def _call(torch, x_dev, out_dev, rows, stream):
    rc = qb.argmax_rows_noalloc(x_dev.data_ptr(), x_dev.stride(0), x_dev.shape[1], rows,
                                out_dev.data_ptr(), stream.cuda_stream)
    assert rc == 0
    stream.synchronize()
    return out_dev[:rows].cpu().numpy().astype(np.uint32)


def test_noalloc_argmax_matches_sample_greedy():
    torch = pytest.importorskip("torch")
    n = 248320                                         # vocabulary of the full model
    first = _rows(11, 8, n, scale=4.0)
    second = _rows(12, 5, n, scale=0.25)               # smaller maxima than the first call
    want1 = np.array([qb.sample_greedy(r) for r in first], np.uint32)
    want2 = np.array([qb.sample_greedy(r) for r in second], np.uint32)
    assert want1[0] == 7

    dev = torch.device("cuda:0")
    stream = torch.cuda.Stream(device=dev)
    # the row stride differs from n to exercise ld
    buf1 = torch.full((8, n + 64), float("nan"), dtype=torch.float32, device=dev)
    buf1[:, :n] = torch.from_numpy(first).to(dev)
    buf2 = torch.full((5, n + 64), float("nan"), dtype=torch.float32, device=dev)
    buf2[:, :n] = torch.from_numpy(second).to(dev)
    out = torch.full((32,), 0xFFFF, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    got1 = _call(torch, buf1[:, :n], out, 8, stream)
    free_before, _ = torch.cuda.mem_get_info(dev)
    got2 = _call(torch, buf2[:, :n], out, 5, stream)
    free_after, _ = torch.cuda.mem_get_info(dev)
    np.testing.assert_array_equal(got1, want1)
    np.testing.assert_array_equal(got2, want2)
    assert free_after == free_before                   # the second call allocated nothing


def test_noalloc_argmax_rejects_oversize():
    torch = pytest.importorskip("torch")
    lib = qb.lib()
    lib.qb_clear_error()
    x = torch.zeros((33, 16), dtype=torch.float32, device="cuda:0")
    out = torch.zeros((33,), dtype=torch.int32, device="cuda:0")
    rc = lib.qb_argmax_rows_noalloc(x.data_ptr(), 16, 16, 33, out.data_ptr(), None)
    assert rc == -1
    msg = lib.qb_last_error_str().decode()
    lib.qb_clear_error()
    assert "exceeds the static scratch maximum of 32" in msg
