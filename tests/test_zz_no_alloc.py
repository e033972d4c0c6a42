"""The allocation-free scoring + selection entry point (smlm_score_select_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory at call time (a host framework whose memory pool has
reserved the GPU, a serving loop where cudaMalloc would synchronise the device): its scratch is a static array
inside the library instead of a workspace. Here it must give exactly the results of the workspace entry point
(smlm_score_select) on two calls in a row (the second call also shows that the shared scratch carries nothing
over), and refuse calls larger than its scratch. This file sorts last so that a run stopping at the first
failure has run every other test already."""
import pytest
import torch

from smlm_b200 import _lib as L
from smlm_b200 import kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ROWS = 16384      # SMLM_NOALLOC_MAX_ROWS in include/smlm_b200.h


def noalloc(q, keys, knn):
    N, H, _ = q.shape
    NK, half = keys.shape[2], keys.shape[3]
    scores = torch.empty(N, H, knn, dtype=torch.bfloat16, device=DEV)
    idx = torch.empty(N, H, knn, dtype=torch.int64, device=DEV)
    w = torch.empty(N, H, knn, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = L.lib().smlm_score_select_noalloc(L.ptr(q), L.ptr(keys), N, H, NK, half, knn, L.ptr(scores), L.ptr(idx),
                                           L.ptr(w), L.ptr(status), L.stream(q.device))
    return rc, scores, idx, w, status


def test_noalloc_equals_workspace_entry_point_on_two_calls():
    for call, (N, H, NK, knn) in enumerate([(3000, 4, 1024, 32), (777, 2, 512, 8)]):
        check_against_workspace_entry_point(N, H, NK, knn, 100 + call)


def test_noalloc_at_its_row_limit_and_for_one_token():
    """n * heads exactly SMLM_NOALLOC_MAX_ROWS (the last rows of the static array written and read, one key-range
    split), then one token (a decoding call: the key range split over many CTAs inside the same array)."""
    check_against_workspace_entry_point(MAX_ROWS // 4, 4, 4096, 32, 7)
    check_against_workspace_entry_point(1, 4, 4096, 32, 8)


def check_against_workspace_entry_point(N, H, NK, knn, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(N, H, 256, generator=gen).bfloat16().to(DEV)
    keys = (torch.randn(H, 2, NK, 128, generator=gen) * 128 ** -0.5).bfloat16().to(DEV)
    rc, sc, idx, w, status = noalloc(q, keys, knn)
    assert rc == L.OK, L.lib().smlm_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    rsc, ridx, rw = K.score_select(q, keys, knn)
    assert torch.equal(idx, ridx)
    assert torch.equal(sc, rsc)
    torch.testing.assert_close(w, rw, rtol=0, atol=1e-6)


def test_noalloc_rejects_calls_beyond_its_scratch():
    q = torch.zeros(MAX_ROWS // 4 + 1, 4, 256, dtype=torch.bfloat16, device=DEV)
    keys = torch.zeros(4, 2, 128, 128, dtype=torch.bfloat16, device=DEV)
    rc, *_ = noalloc(q, keys, 8)
    assert rc == L.ERR_INVALID
    assert b"SMLM_NOALLOC_MAX_ROWS" in L.lib().smlm_last_error()
