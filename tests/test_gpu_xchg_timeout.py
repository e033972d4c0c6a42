"""The peer-memory exchange's waits are bounded: one GPU, two exchange blocks in one process, this rank 0 of a
2-rank exchange whose rank 1 never announces its lookups (a flag nothing sets). The forward gives up after the
wait bound, raises SMLM_FLAG_TIMEOUT in the status word, and the requester's wait then ends at once; the
context stays usable."""
import ctypes
import time

import pytest
import torch

from smlm_b200 import _lib as L

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_with_status():
    lib = L.lib()
    dev = torch.device("cuda", 0)
    world, n, k, d = 2, 64, 8, 64
    nbytes = lib.smlm_xchg_bytes(world, n, k, d)
    blocks = []
    for _ in range(world):
        b = ctypes.c_void_p()
        h = (ctypes.c_char * 64)()
        L.check(lib.smlm_xchg_alloc(nbytes, ctypes.byref(b), h), "xchg_alloc")
        blocks.append(b.value)
    try:
        peers = torch.tensor(blocks, dtype=torch.int64, device=dev)
        idx = torch.randint(0, 100, (n, k), dtype=torch.int32, device=dev)
        w = torch.rand(n, k, device=dev)
        table = torch.randn(50, d, device=dev)
        all_idx = torch.empty(world * n, k, dtype=torch.int32, device=dev)
        all_w = torch.empty(world * n, k, device=dev)
        out = torch.empty(n, d, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        t0 = time.time()
        # rows per rank 50: rank 0 holds rows 0 .. 49 (the table), rank 1 rows 50 .. 99
        rc = lib.smlm_xchg_forward(L.ptr(peers), ctypes.c_void_p(blocks[0]), 0, world, L.ptr(idx), L.ptr(w), n, k, n,
                                   50, L.ptr(table), L.F32, 0, 50, d, L.ptr(all_idx), L.ptr(all_w), None, L.F32,
                                   L.ptr(out), L.F32, 1, L.ptr(status), L.stream(dev))
        assert rc == L.OK
        torch.cuda.synchronize()
        elapsed = time.time() - t0
        assert int(status.item()) & L.FLAG_TIMEOUT
        assert 5.0 < elapsed < 60.0
        # the context is still usable
        assert float(torch.ones(4, device=dev).sum()) == 4.0
        # a missing status word is refused on the host, before any launch
        rc = lib.smlm_xchg_forward(L.ptr(peers), ctypes.c_void_p(blocks[0]), 0, world, L.ptr(idx), L.ptr(w), n, k, n,
                                   50, L.ptr(table), L.F32, 0, 50, d, L.ptr(all_idx), L.ptr(all_w), None, L.F32,
                                   L.ptr(out), L.F32, 2, None, L.stream(dev))
        assert rc == L.ERR_INVALID
    finally:
        torch.cuda.synchronize()
        for b in blocks:
            lib.smlm_xchg_free(ctypes.c_void_p(b))
