"""rv_index_topk_noalloc, checked against the allocating rv_index_topk_device.

Some callers cannot call cudaMalloc: a host application whose own allocator or memory pool owns
the device budget, or a serving thread that must not let an allocation synchronise the device.
The no-allocation entry point serves them with all of its scratch in one fixed device array
inside the library.  It must return exactly what the allocating entry point returns (the scan's
indices and f64 scores are bit-exact, so the comparison is equality), and keep doing so on
consecutive calls, because the fixed array still holds the previous call's contents when the
next call starts.

This file is collected last so that a run stopping at the first failure has run everything else;
it passes on its own in a fresh process as well as after the other tests.
"""

import pytest

pytestmark = pytest.mark.gpu


def _outputs(torch, nq, k, fill):
    return (torch.full((nq, k), fill, dtype=torch.int64, device="cuda"),
            torch.full((nq, k), float(fill), dtype=torch.float32, device="cuda"),
            torch.full((nq, k), float(fill), dtype=torch.float64, device="cuda"))


def test_noalloc_topk_matches_allocating_entry_point_on_consecutive_calls(cuda_device):
    import torch

    from ripvec_b200 import _lib as L
    from ripvec_b200 import synth
    from ripvec_b200.index import SearchIndex

    lib = L.lib()
    dim = 768
    db = synth.normalized_gaussian(100_000, dim, seed=41)
    idx = SearchIndex(db, device=cuda_device)  # fresh: no scan scratch of its own reserved yet
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row, both made before the allocating entry point ever runs on this index;
    # the second has fewer queries, a different k and a threshold, so any stale candidate state
    # left in the shared array by the first call would show.
    cases = ((7, 50, float("-inf"), 42), (3, 20, 0.05, 43))
    got = []
    for i, (nq, k, thr, seed) in enumerate(cases):
        q = torch.from_numpy(synth.normalized_gaussian(nq, dim, seed=seed)).cuda()
        gi, gs, g64 = _outputs(torch, nq, k, -7)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = lib.rv_index_topk_noalloc(idx._h, q.data_ptr(), nq, k, thr, gi.data_ptr(), gs.data_ptr(),
                                       g64.data_ptr(), stream)
        torch.cuda.synchronize()
        assert rc == L.RV_OK, lib.rv_index_last_error(idx._h).decode()
        if i > 0:
            # after the first call (which may load kernels on first use), a call leaves the
            # device's free memory unchanged: nothing was allocated for it
            assert torch.cuda.mem_get_info()[0] == free0
        got.append((q, gi, gs, g64))
    for (nq, k, thr, _), (q, gi, gs, g64) in zip(cases, got):
        ri, rs, r64 = _outputs(torch, nq, k, -3)
        idx.topk_device(q, k, ri, rs, r64, threshold=thr, stream=stream)
        torch.cuda.synchronize()
        assert torch.equal(gi, ri)
        assert torch.equal(g64, r64)
        assert torch.equal(gs, rs)
        assert (gi[:, 0] >= 0).all()
    assert lib.rv_index_topk_noalloc(idx._h, None, 0, 10, 0.0, None, None, None, stream) == L.RV_OK

    # Requests beyond the fixed scratch are refused with a clear error, not truncated.
    q = torch.zeros(17, dim, device="cuda")
    gi, gs, g64 = _outputs(torch, 17, 10, 0)
    rc = lib.rv_index_topk_noalloc(idx._h, q.data_ptr(), 17, 10, float("-inf"), gi.data_ptr(), gs.data_ptr(),
                                   g64.data_ptr(), stream)
    assert rc == L.RV_E_INVALID
    assert b"at most 16 queries" in lib.rv_index_last_error(idx._h)
    rc = lib.rv_index_topk_noalloc(idx._h, q.data_ptr(), 1, 65, float("-inf"), gi.data_ptr(), gs.data_ptr(),
                                   g64.data_ptr(), stream)
    assert rc == L.RV_E_INVALID
    idx.close()
