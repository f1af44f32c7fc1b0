"""model_init on malformed GGUF files: -1 with a message, no crash, no device
work.  Mirrors the reference's model_init / gguf_open failure paths
(src/model.c:31-53, 55-150, 287-289; src/gguf.c:493-618): a truncated file,
a wrong magic or version, a tensor with wrong dimensions, a missing tensor of
the MTP block, a tensor of a format the engine does not decode.

These run without a GPU: the library parses and checks the file before its
first CUDA call, so the error each case reports is the parse error itself."""
import ctypes as C
import os
import shutil
import struct

import pytest

from conftest import qb


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    d = tmp_path_factory.mktemp("ggufbad")
    return qb.write_synth_gguf(os.path.join(str(d), "tiny.gguf"), qb.TINY, seed=1)


def _init(path):
    lib = qb.lib()
    lib.qb_clear_error()
    m = qb.QwenModel()
    rc = lib.model_init(C.byref(m), os.fsencode(path), 64)
    msg = lib.qb_last_error_str().decode()
    lib.qb_clear_error()
    if rc == 0:
        lib.model_free(C.byref(m))
    return rc, msg


def _variant(good, tmp_path, name, edit):
    p = os.path.join(str(tmp_path), name)
    shutil.copyfile(good, p)
    with open(p, "r+b") as f:
        data = bytearray(f.read())
        data = edit(data)
        f.seek(0)
        f.truncate()
        f.write(data)
    return p


def _tensor_info_at(data, name):
    """Offset of the n_dims field of tensor `name` in the GGUF tensor table
    (the name is stored as a u64 length followed by its bytes)."""
    key = struct.pack("<Q", len(name)) + name
    i = bytes(data).find(key)
    assert i > 0, name
    return i + len(key)


def test_valid_file_passes_the_host_checks(good):
    rc, msg = _init(good)
    if rc == 0:
        return   # a GPU is present: the model loaded
    assert "model_init:" not in msg and "GGUF" not in msg and "file" not in msg, msg


def test_truncated_file(good, tmp_path):
    p = _variant(good, tmp_path, "trunc.gguf", lambda d: d[: len(d) - 4096])
    rc, msg = _init(p)
    assert rc == -1 and "extends past the end of the file" in msg, msg


def test_header_only_file(good, tmp_path):
    p = _variant(good, tmp_path, "hdr.gguf", lambda d: d[:200])
    rc, msg = _init(p)
    assert rc == -1 and "truncated GGUF header" in msg, msg


def test_bad_magic(good, tmp_path):
    p = _variant(good, tmp_path, "magic.gguf", lambda d: b"GGUX" + d[4:])
    rc, msg = _init(p)
    assert rc == -1 and "not a GGUF v2/v3 file" in msg, msg


def test_bad_version(good, tmp_path):
    p = _variant(good, tmp_path, "ver.gguf", lambda d: d[:4] + struct.pack("<I", 7) + d[8:])
    rc, msg = _init(p)
    assert rc == -1 and "not a GGUF v2/v3 file" in msg, msg


def test_wrong_dims(good, tmp_path):
    def edit(d):
        at = _tensor_info_at(d, b"blk.0.ffn_gate.weight")
        ne1 = struct.unpack_from("<Q", d, at + 4 + 8)[0]
        struct.pack_into("<Q", d, at + 4 + 8, ne1 - 256)
        return d
    p = _variant(good, tmp_path, "dims.gguf", edit)
    rc, msg = _init(p)
    assert rc == -1 and "blk.0.ffn_gate.weight dimension mismatch" in msg, msg


def test_missing_mtp_tensor(good, tmp_path):
    n = qb.TINY["n_layer"]
    old = f"blk.{n}.nextn.eh_proj.weight".encode()
    p = _variant(good, tmp_path, "mtp.gguf", lambda d: bytearray(bytes(d).replace(old, old[:-1] + b"X", 1)))
    rc, msg = _init(p)
    assert rc == -1 and f"missing tensor blk.{n}.nextn.eh_proj.weight" in msg, msg


def test_unsupported_tensor_type(good, tmp_path):
    def edit(d):
        at = _tensor_info_at(d, b"blk.1.ffn_down.weight")
        n_dims = struct.unpack_from("<I", d, at)[0]
        struct.pack_into("<I", d, at + 4 + 8 * n_dims, 2)   # GGML_Q4_0
        return d
    p = _variant(good, tmp_path, "type.gguf", edit)
    rc, msg = _init(p)
    assert rc == -1 and "blk.1.ffn_down.weight has unsupported type 2" in msg, msg


def test_missing_file(tmp_path):
    rc, msg = _init(os.path.join(str(tmp_path), "nope.gguf"))
    assert rc == -1 and "cannot open" in msg, msg
