"""GPU: the allocation-free embedding backward (malus_embedding_bwd_noalloc).

It exists for callers that cannot call cudaMalloc where they need the op; its
scratch is a fixed device array inside the library.  The test compares it,
through the C ABI, with the allocating entry point __embedding_bwd on two
calls in a row (the second with a different shape, so stale contents of the
shared array would show), and checks that an oversize request is refused."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run_noalloc(M, lib, dout, idx, vocab):
    td = M.Tensor.from_numpy(dout)
    ti = M.Tensor.from_numpy(idx)
    out = M.Tensor.from_numpy(np.full((vocab, dout.shape[1]), np.nan, np.float32))
    dt = 5 if idx.dtype == np.int32 else 6
    rc = lib.malus_embedding_bwd_noalloc(lib.malus_tensor_data(td.h), lib.malus_tensor_data(ti.h), dt,
                                         idx.size, vocab, dout.shape[1], lib.malus_tensor_data(out.h),
                                         lib.malus_stream())
    assert rc == 0
    return out.numpy()


def _run_existing(M, lib, dout, idx, vocab):
    w = M.Tensor.from_numpy(np.zeros((vocab, dout.shape[1]), np.float32))
    td = M.Tensor.from_numpy(dout)
    ti = M.Tensor.from_numpy(idx)
    return M.Tensor(lib.__embedding_bwd(w.h, ti.h, td.h)).numpy()


def test_noalloc_matches_allocating_entry_point(M, rt):
    rng = np.random.default_rng(42)
    cases = [(16384, 65, 384, np.int32), (3000, 256, 128, np.int64)]
    for n, vocab, dim, dt in cases:          # two calls in a row on the shared scratch
        idx = rng.integers(0, vocab, n).astype(dt)
        dout = rng.standard_normal((n, dim)).astype(np.float32)
        got = _run_noalloc(M, rt, dout, idx, vocab)
        ref = _run_existing(M, rt, dout, idx, vocab)
        scale = np.zeros((vocab, dim))
        np.add.at(scale, idx, np.abs(dout))
        err = np.max(np.abs(got.astype(np.float64) - ref) / np.maximum(scale, 1e-6))
        assert err < 1e-5, err
        assert not np.isnan(got).any()


def test_noalloc_rejects_oversize(M, rt):
    rc = rt.malus_embedding_bwd_noalloc(None, None, 5, 65537, 65, 8, None, None)
    assert rc < 0
    rc = rt.malus_embedding_bwd_noalloc(None, None, 5, 8192, 100000, 8, None, None)
    assert rc < 0
