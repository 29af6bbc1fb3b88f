"""CPU checks of the C-ABI boundary: the library builds/loads and exports every declared symbol."""
import ctypes
import os
import re

import pytest

from flashact_b200 import _capi
from flashact_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "flashact.h")).read()
    return sorted(set(re.findall(r"^FA_API\s+[\w\s\*]+?\b(fa_\w+)\s*\(", src, flags=re.M)))


def test_header_lists_match_binding():
    assert declared_functions() == sorted(_capi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(build())
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_create_without_gpu_fails_cleanly():
    """On a box without an sm_100 GPU fa_create returns an error status, never crashes."""
    import torch
    if torch.cuda.is_available():
        return
    lib = _capi.load_library(build())
    cfg = _capi.FaConfig(18, 1024, 8, 1, 256, 4096, 50, 32, 968, 1, 10, 0)
    h = ctypes.c_void_p()
    st = lib.fa_create(_capi.FA_MODEL_PI05, ctypes.byref(cfg), 0, ctypes.byref(h))
    assert st in (_capi.FA_ERR_INVALID, _capi.FA_ERR_CUDA, _capi.FA_ERR_UNSUPPORTED)
    assert not h.value
    assert len(lib.fa_last_error(None)) > 0


def test_struct_layouts():
    assert ctypes.sizeof(_capi.FaConfig) == 12 * 4
    assert ctypes.sizeof(_capi.FaMa2Weights) == 18 * 16
    assert ctypes.sizeof(_capi.FaTensor) == 16
    assert ctypes.sizeof(_capi.FaPi05Weights) == 21 * 16


def test_compat_launch_signatures():
    """flashact_b200.compat mirrors the reference's pybind launch() signatures argument for
    argument (src/pi05/binding.cpp:28-37, src/molmoact2/binding.cpp:28-35)."""
    import inspect

    from flashact_b200 import compat
    pi05 = ["w1", "wo", "w2", "w3", "s1", "so_", "s2", "s3", "mods", "mod_final", "rope_cos", "rope_sin", "w_ain",
            "b_ain", "w_aout", "b_aout", "kvsrc_k", "kvsrc_v", "srows", "kcache", "vtcache", "Lp", "Lmax",
            "num_steps", "Tv", "x_t", "x", "xp", "stage_cycles", "xn", "q", "attn", "hmlp", "scores", "probs",
            "nblocks", "nthreads"]
    ma2 = ["ws", "bs", "mods", "mod_final", "rope_cos", "rope_sin", "w_ain", "b_ain", "w_aout", "b_aout", "kctx",
           "vtctx", "Lk", "Lkmax", "Tv", "adim", "num_steps", "x_t", "x", "xp", "stage_cycles", "bufs", "scores",
           "probs", "nblocks", "nthreads"]
    assert list(inspect.signature(compat.pi05_launch).parameters) == pi05
    assert list(inspect.signature(compat.ma2_launch).parameters) == ma2


def _build_c_probe(tmp_path):
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    lib = os.path.join(ROOT, "flashact_b200", "_lib")
    exe = str(tmp_path / "capi_probe")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "capi_probe.c"), "-L", lib, "-lflashact",
                    f"-Wl,-rpath,{lib}", "-o", exe], check=True)
    return exe


def test_c_caller_without_gpu(tmp_path):
    """A plain C program links libflashact.so through include/flashact.h; without a GPU,
    fa_create returns an error status and message instead of crashing."""
    import subprocess
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: covered by test_c_caller_with_gpu")
    exe = _build_c_probe(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)


@pytest.mark.gpu
def test_c_caller_with_gpu(tmp_path, require_gpu):
    """The same C program on a GPU: create succeeds, sampling before weights is FA_ERR_STATE."""
    import subprocess
    exe = _build_c_probe(tmp_path)
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
