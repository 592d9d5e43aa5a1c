"""C-ABI checks that need no GPU: the library loads, exports every declared
symbol with the declared arity, and rejects bad arguments with a status and a
message (never an abort)."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "neuratensor_native.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"NT_API\s+[\w\s\*]+?\b(nt_\w+)\s*\(([^)]*)\)\s*;", src, flags=re.S):
        args = [a.strip() for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        out[m.group(1)] = len(args)
    return out


@pytest.fixture(scope="module")
def nat():
    from neuratensor_b200 import build, native
    build.build()
    native.load()
    return native


def test_header_declares_entry_points():
    d = _declared()
    for name in ("nt_lif_scan", "nt_selective_scan", "nt_ssm_forward", "nt_sparse_out_proj", "nt_rmsnorm_in_proj",
                 "nt_block_forward", "nt_lif_ssm_fused", "nt_last_error", "nt_get_error_flag"):
        assert name in d


def test_library_exports_every_declared_symbol(nat):
    lib = ctypes.CDLL(nat.library_path())
    for name in _declared():
        assert hasattr(lib, name), name


def test_binding_arity_matches_header(nat):
    d = _declared()
    assert set(d) == set(nat.EXPORTED)
    for name, n in d.items():
        assert len(nat._SIGS[name][0]) == n, name


def test_abi_version(nat):
    assert nat.load().nt_abi_version() == 1


def test_bad_arguments_return_status_not_abort(nat):
    L = nat.load()
    rc = L.nt_lif_scan(0, 1, 4, 8, None, 32, 8, None, None, None, None, None, 32, 8, None, None)
    assert rc == 1
    assert b"null pointer" in L.nt_last_error()
    rc = L.nt_lif_scan(7, 1, 4, 8, None, 32, 8, None, None, None, None, None, 32, 8, None, None)
    assert rc == 2
    rc = L.nt_selective_scan(0, 0, 1, 4, 8, 300, *([None] * 10), None)
    assert rc == 1 and b"256" in L.nt_last_error()
    rc = L.nt_block_forward(1, 1, 1, 4, 64, 128, 8, *([None] * 17), 1, None, 0, None)
    assert rc == 1
    fake = ctypes.c_void_p(256)
    need = L.nt_block_workspace_bytes(1, 2, 16, 64, 128, 8)
    args = [fake] * 17
    rc = L.nt_block_forward(1, 1, 2, 16, 64, 128, 8, *args, 1, fake, need - 1, None)
    assert rc == 6 and b"workspace" in L.nt_last_error()


def test_device_query_without_gpu(nat):
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    L = nat.load()
    assert L.nt_device_supported(0) != 0
    assert len(L.nt_last_error()) > 0


def test_workspace_sizes(nat):
    L = nat.load()
    M, dm, di, N = 16384, 640, 1280, 32
    ws = L.nt_block_workspace_bytes(1, 8, 2048, dm, di, N)
    # xn + h + gate + spikes + dt + o (+ B|C, counts, flags, indices) in bf16
    assert ws >= M * (dm + 5 * di + 2 * N) * 2
    assert ws < M * (dm + 5 * di + 2 * N) * 2 * 1.2
    assert L.nt_ssm_workspace_bytes(0, 2, 10, 24, 16) >= 20 * (24 + 32) * 4
    assert L.nt_sparse_out_proj_workspace_bytes(1, 32768, 4096, 2048) >= 32768 * 4096 * 2


def test_cpu_tensors_fail_loudly(nat):
    from neuratensor_b200 import LIFLayer, FusedSpikeBlock
    with pytest.raises(RuntimeError, match="CUDA"):
        LIFLayer(8)(torch.randn(1, 4, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        FusedSpikeBlock(16, 4)(torch.randn(1, 4, 16))
