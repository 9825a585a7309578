"""The argmax key of the fused lm_head argmax (csrc/argmax_key.cuh, the code the GPU epilogue runs), built
for the host: the row of the largest key is torch.argmax's answer -- first of equal values, -0.0 equal to
+0.0, NaN above everything (first NaN), infinities in order -- on bf16-valued rows."""

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("needs g++")
    out = tmp_path_factory.mktemp("native") / "libargmax_host.so"
    subprocess.run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-Werror",
                    str(HERE / "native" / "argmax_host.cpp"), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.host_argmax.argtypes = [ctypes.c_void_p, ctypes.c_int]
    lib.host_argmax.restype = ctypes.c_int64
    return lib


def _rows(rng):
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 3.5], dtype=np.float32)
    for _ in range(400):
        n = int(rng.integers(1, 300))
        x = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16).float().numpy()
        kind = rng.integers(0, 5)
        if kind == 1:  # ties at the maximum
            x[rng.integers(0, n, size=3)] = np.float32(x.max() + 1.0)
        elif kind == 2:  # specials sprinkled in
            idx = rng.integers(0, n, size=min(n, 4))
            x[idx] = rng.choice(specials, size=len(idx))
        elif kind == 3:  # all equal (signed zeros mixed)
            x[:] = rng.choice(np.array([0.0, -0.0], dtype=np.float32), size=n)
        elif kind == 4:  # all -inf but one NaN somewhere, or all -inf
            x[:] = -np.inf
            if rng.random() < 0.5:
                x[rng.integers(0, n)] = np.nan
        yield np.ascontiguousarray(x, dtype=np.float32)


def test_argmax_key_matches_torch_argmax(lib):
    rng = np.random.default_rng(0)
    for x in _rows(rng):
        got = lib.host_argmax(x.ctypes.data, x.size)
        want = int(torch.argmax(torch.from_numpy(x)))
        assert got == want, (x, got, want)
