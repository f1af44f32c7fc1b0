"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "qwen3.8-27b-in-c_b200")
sys.path.insert(0, ROOT)


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


qb = _load("qwen_b200", os.path.join(PKG_DIR, "qwen_b200.py"))
oracle = _load("qb_oracle", os.path.join(ROOT, "oracle", "ref.py"))


def reference_dir():
    """The reference checkout ($QB_REFERENCE_DIR, else "reference" beside this
    repository), or None where its sources are absent (e.g. the GPU box)."""
    ref = os.environ.get("QB_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
    return ref if os.path.isfile(os.path.join(ref, "src", "model.c")) else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("qb")


def _gguf(workdir, name, shape, seed, profile=0):
    path = os.path.join(str(workdir), f"{name}_{seed}_{profile}.gguf")
    if not os.path.exists(path):
        qb.write_synth_gguf(path, shape, seed=seed, profile=profile)
    return path


@pytest.fixture(scope="session")
def tiny_gguf(workdir):
    return _gguf(workdir, "tiny", qb.TINY, seed=1)


@pytest.fixture(scope="session")
def tiny_mixed_gguf(workdir):
    return _gguf(workdir, "tinymix", qb.TINY, seed=2, profile=1)


@pytest.fixture(scope="session")
def small_gguf(workdir):
    return _gguf(workdir, "small", qb.SMALL, seed=3)


@pytest.fixture(scope="session")
def wide_gguf(workdir):
    return _gguf(workdir, "wide4", qb.WIDE4, seed=4)


def full_gguf_path():
    """The FULL benchmark model (seed 0), shared with bench.py: one 15.3 GB file
    in /dev/shm, written once per box."""
    d = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    return os.path.join(d, "qb_bench_full_seed0.gguf")


@pytest.fixture(scope="session")
def full_gguf():
    path = full_gguf_path()
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        qb.write_synth_gguf(tmp, qb.FULL, seed=0)
        os.replace(tmp, path)
    return path
