"""The C-ABI library loads and exports exactly what include/retree_b200.h declares (CPU only)."""

import os
import re
from pathlib import Path

import pytest
import torch

from retree_b200 import _lib, kernels

HEADER = Path(__file__).resolve().parents[1] / "include" / "retree_b200.h"


def _declared():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"^\s*(?:const\s+)?[\w\s\*]+?\b(rt_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
        args = [a.strip() for a in m.group(2).split(",")]
        decls[m.group(1)] = [] if args == ["void"] else args
    return decls


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    decls = _declared()
    assert decls, "no declarations parsed"
    for name in decls:
        assert hasattr(lib, name), name
    assert set(decls) == set(_lib.SIGNATURES)
    assert lib.rt_abi_version() == 2


def test_ctypes_signatures_match_header():
    import ctypes
    decls = _declared()
    for name, args in decls.items():
        res, argtypes = _lib.SIGNATURES[name]
        assert len(argtypes) == len(args), name
        for a, t in zip(args, argtypes):
            if "*" in a or "rt_stream_t" in a:
                assert t is ctypes.c_void_p or t is ctypes.c_char_p, (name, a)
            elif a.startswith("int64_t"):
                assert t is ctypes.c_int64, (name, a)
            elif a.startswith("size_t"):
                assert t is ctypes.c_size_t, (name, a)
            elif a.startswith("double"):
                assert t is ctypes.c_double, (name, a)
            elif a.startswith("float"):
                assert t is ctypes.c_float, (name, a)
            elif a.startswith("int"):
                assert t is ctypes.c_int, (name, a)


def test_status_strings():
    assert _lib.status_string(0) == "ok"
    assert "wait" in _lib.status_string(_lib.RT_DEV_WAIT_TIMEOUT)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.RT_ERR_INVALID_ARGUMENT, "x")


def test_host_argument_checks_need_no_gpu():
    lib = _lib.load()
    # negative sizes and keep > window are rejected before any launch
    assert lib.rt_kv_compact(None, None, 1, 0, 1, 0, 0, 256, 0, None, 4, None, 5, None, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_tree_attn(None, 0, 0, None, None, 0, 0, 0, None, 0, 0, None, 1, 1, 0, None, 32, 8, 128, 1.0,
                            0, 0, None, 0, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_draft_topk(None, 0, 10, 1, 10, 2000, None, None, None, None, 0, None) == _lib.RT_ERR_UNSUPPORTED
    assert lib.rt_tree_build(None, None, 15, 16, 2000, 0, None, 0, None, 0, 2, 0.0, 8, 1, 1, None, 6.0, None, 0,
                             None, None, None, None, 1, None, None, None, 0, None, 0, None, None, None) in (
        _lib.RT_ERR_UNSUPPORTED, _lib.RT_ERR_INVALID_ARGUMENT)


def test_wrappers_refuse_cpu_tensors():
    x = torch.zeros(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.draft_topk(x, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.kv_compact(torch.zeros(1, 2, 5, 4), 1, torch.zeros(2, dtype=torch.long))


def test_qkv_epilogue_struct_layout():
    import ctypes
    # int, int, 2 pointers, float (+pad), 2 pointers, int64, 4 pointers, 4 int64, pointer
    assert ctypes.sizeof(_lib.QkvEpilogue) == 128
    assert _lib.QkvEpilogue.eps.offset == 24 and _lib.QkvEpilogue.offset_dev.offset == 120


def test_linear_shape_checks_without_gpu():
    lib = _lib.load()
    # every shape the GPU tests and the Qwen3 projections use has a valid plan (smem within the SM's limit)
    for m in (1, 17, 33, 40, 65, 200, 257, 300, 512):
        for n_out, k in ((128, 64), (2560, 4096), (6144, 2560), (19456, 2560), (2560, 9728), (151936, 2560),
                         (256, 128), (384, 256), (1536, 512)):
            for epi in (0, 1):
                assert lib.rt_linear_check(m, n_out, k, epi) == 0, (m, n_out, k, epi)
    assert lib.rt_linear_check(17, 6144, 2560, 2) == 0  # QKV epilogue
    assert lib.rt_linear_check(17, 6144, 2560, 3) != 0
    assert lib.rt_linear_check(513, 128, 64, 0) != 0
    assert lib.rt_linear_check(17, 200, 64, 0) != 0
    assert lib.rt_linear_check(17, 256, 60, 0) != 0


def test_peer_exchange_argument_checks_without_gpu():
    import ctypes
    lib = _lib.load()
    two = (ctypes.c_void_p * 2)(1 << 20, 2 << 20)
    bad = (ctypes.c_void_p * 2)(1 << 20, (2 << 20) + 8)  # not 16-byte aligned
    epoch = ctypes.c_void_p(3 << 20)
    assert lib.rt_peer_signal(bad, 2, 0, epoch, 0, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_peer_signal(two, 2, 2, epoch, 0, None) == _lib.RT_ERR_INVALID_ARGUMENT  # rank out of range
    assert lib.rt_peer_signal(two, 9, 0, epoch, 0, None) == _lib.RT_ERR_INVALID_ARGUMENT  # more than 8 ranks
    out = ctypes.c_void_p(4 << 20)
    # row bytes not a multiple of 16, destination narrower than world * row, missing flags
    assert lib.rt_peer_gather(two, 2, 4, 24, 32, out, 64, epoch, epoch, 0, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_peer_gather(two, 2, 4, 32, 32, out, 48, epoch, epoch, 0, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_peer_gather(two, 2, 4, 32, 32, out, 64, None, epoch, 0, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_peer_gather(two, 2, 0, 32, 32, out, 64, epoch, epoch, 0, None, None) == _lib.RT_OK  # no rows
    assert lib.rt_ipc_alloc(0, ctypes.byref(ctypes.c_void_p()), (ctypes.c_ubyte * 64)()) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_ipc_open(None, ctypes.byref(ctypes.c_void_p())) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_peer_epoch_step(None, 1, None) == _lib.RT_ERR_INVALID_ARGUMENT


def test_a_plain_c_host_compiles_links_and_calls_the_abi(tmp_path):
    """include/retree_b200.h is C11 (pedantic, warnings as errors), and a C program links the library and
    calls its host-only entry points (no GPU needed for these)."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lib = _lib.LIB_PATH
    assert lib.exists(), "build the library first (python -m retree_b200.build)"
    src = tmp_path / "host.c"
    src.write_text(r"""
#include <stdio.h>
#include "retree_b200.h"
int main(void) {
  printf("%d %s %zu %d\n", rt_abi_version(), rt_status_string(RT_ERR_INVALID_ARGUMENT),
         rt_tree_attn_workspace_size(17, 32, 8, 128, 2048, 17), rt_linear_check(17, 2560, 4096, RT_EPI_STORE));
  return 0;
}
""")
    exe = tmp_path / "host"
    subprocess.run([gcc, "-std=c11", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(HEADER.parent), str(src),
                    "-o", str(exe), "-L", str(lib.parent), "-lretree_b200", f"-Wl,-rpath,{lib.parent}"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    want_ws = _lib.load().rt_tree_attn_workspace_size(17, 32, 8, 128, 2048, 17)
    assert out[0] == "2" and " ".join(out[1:-2]) == "invalid argument"
    assert int(out[-2]) == want_ws > 0 and out[-1] == "0"


def test_integration_ctypes_stub_matches_the_library():
    """The ctypes binding INTEGRATION.md points to (tests/integration_stub.py) sets argtypes that agree with
    the header and loads the built library (it runs here up to its first device call)."""
    from tests import integration_stub as stub

    assert os.path.realpath(stub.LIB) == os.path.realpath(str(_lib.LIB_PATH))
    for name in ("rt_kv_compact", "rt_status_string"):
        res, argtypes = _lib.SIGNATURES[name]
        assert list(getattr(stub.lib, name).argtypes) == list(argtypes), name
        assert getattr(stub.lib, name).restype is res, name
    assert stub.lib.rt_status_string(_lib.RT_ERR_INVALID_ARGUMENT).decode() == "invalid argument"
    assert callable(stub.compact_tail_inplace)
