"""The allocation-free search entry point (vdbgpu_index_search_noalloc), for callers that must not
allocate device memory while they search: its results equal the regular entry point's on flat and
SQ8-flat indexes, on two calls in a row (the second reuses the fixed scratch array that the first
one left behind), and the device's free memory does not move across those calls. Collected last so
that a run stopping at its first failure has run the rest."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _check_twice(idx, qs, k, rerank):
    import torch
    ids_ref, d_ref = idx.search(qs, k=k, rerank=rerank)
    q_dev = torch.from_numpy(qs).cuda()
    outs = [(torch.full((qs.shape[0], k), -1, dtype=torch.int32, device="cuda"),
             torch.full((qs.shape[0], k), float("nan"), dtype=torch.float32, device="cuda")) for _ in range(3)]
    # A first call loads the library's module data on this device (the fixed array included);
    # from then on no call may change the device's free memory.
    idx.search_noalloc(q_dev, outs[0][0], outs[0][1], k=k, rerank=rerank)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for ids_dev, d_dev in outs[1:]:
        idx.search_noalloc(q_dev, ids_dev, d_dev, k=k, rerank=rerank)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, f"device free memory moved by {free_before - free_after} bytes"
    for ids_dev, d_dev in outs[1:]:
        ids = ids_dev.cpu().numpy().view(np.uint32)
        d = d_dev.cpu().numpy()
        np.testing.assert_array_equal(ids, ids_ref)
        np.testing.assert_array_equal(d, d_ref)


def test_noalloc_matches_regular_search():
    import torch
    import vdb_b200
    from vdb_b200 import synth
    ctx = vdb_b200.Context(0)
    base, qs = synth.flat_int(20_000, 100, dim=128, seed=21)
    flat = vdb_b200.Index.create(ctx, "flat", "l2", base, 128)
    _check_twice(flat, qs, 10, -1)
    base, qs = synth.sq8_cosine(30_000, 128, dim=128, seed=22)
    sq8 = vdb_b200.Index.create(ctx, "sq8_flat", "cosine", base, 128)
    _check_twice(sq8, qs, 10, 100)
    # An empty index gives misses in every slot, as the regular search does.
    empty = vdb_b200.Index.create(ctx, "flat", "l2", np.zeros((0, 128), np.float32), 128)
    ids_ref, d_ref = empty.search(qs[:7], k=5)
    ids = torch.zeros((7, 5), dtype=torch.int32, device="cuda")
    d = torch.zeros((7, 5), dtype=torch.float32, device="cuda")
    empty.search_noalloc(torch.from_numpy(qs[:7]).cuda(), ids, d, k=5)
    np.testing.assert_array_equal(ids.cpu().numpy().view(np.uint32), ids_ref)
    np.testing.assert_array_equal(d.cpu().numpy(), d_ref)
    assert np.all(ids_ref == np.uint32(0xFFFFFFFF)) and np.all(np.isinf(d_ref))
    # Requests beyond the fixed scratch are rejected with a clear error.
    too_many = torch.zeros((129, 128), dtype=torch.float32, device="cuda")
    ids = torch.empty((129, 10), dtype=torch.int32, device="cuda")
    d = torch.empty((129, 10), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError, match="at most 128 queries"):
        sq8.search_noalloc(too_many, ids, d, k=10, rerank=100)
    # Host buffers are refused (staging them would need an allocation).
    with pytest.raises(ValueError, match="device pointers"):
        sq8.search_noalloc(np.zeros((4, 128), np.float32), np.zeros((4, 10), np.uint32),
                           np.zeros((4, 10), np.float32), k=10)
