"""GPU: the allocation-free embedding backward (malus_embedding_bwd_noalloc).

It exists for callers that cannot call cudaMalloc where they need the op
(inside a stream capture that must not gain memory nodes, or inside another
framework's memory arena); its scratch is a fixed device array inside the
library.  Through the C ABI the tests check that it
  * equals the allocating entry point __embedding_bwd bit for bit, and the
    oracle's token-order scatter-add (the same additions in the same order),
    on calls in a row with different shapes (stale contents of the shared
    array would show), including a vocabulary far larger than the id count
    (rows without ids must be exact zeros) and the largest id count allowed;
  * writes zeros for n = 0;
  * skips an out-of-range id without a report, as documented;
  * refuses sizes beyond its limits with a negative return.
This file is collected last, so a run that stops at the first failure has run
every other test first."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(M, lib, dout, idx, vocab, dim):
    td = M.Tensor.from_numpy(dout)
    ti = M.Tensor.from_numpy(idx)
    out = M.Tensor.from_numpy(np.full((vocab, dim), np.nan, np.float32))
    dt = 5 if idx.dtype == np.int32 else 6
    rc = lib.malus_embedding_bwd_noalloc(lib.malus_tensor_data(td.h), lib.malus_tensor_data(ti.h), dt,
                                         idx.size, vocab, dim, lib.malus_tensor_data(out.h),
                                         lib.malus_stream())
    got = out.numpy()
    return rc, got


def _allocating(M, lib, dout, idx, vocab, dim):
    w = M.Tensor.from_numpy(np.zeros((vocab, dim), np.float32))
    td = M.Tensor.from_numpy(dout)
    ti = M.Tensor.from_numpy(idx)
    return M.Tensor(lib.__embedding_bwd(w.h, ti.h, td.h)).numpy()


CASES = [(16384, 65, 384, np.int32),      # C4's token count and vocabulary
         (3000, 256, 128, np.int64),
         (100, 4096, 64, np.int32),       # far more rows than ids: most rows get no id
         (65536, 65, 32, np.int32)]       # the largest id count per call


def test_noalloc_matches_allocating_entry_point_and_oracle(M, rt, orc):
    rng = np.random.default_rng(42)
    for n, vocab, dim, dt in CASES:          # calls in a row on the shared scratch
        idx = rng.integers(0, vocab, n).astype(dt)
        dout = rng.standard_normal((n, dim)).astype(np.float32)
        rc, got = _noalloc(M, rt, dout, idx, vocab, dim)
        assert rc == 0
        ref = _allocating(M, rt, dout, idx, vocab, dim)
        np.testing.assert_array_equal(got, ref)
        np.testing.assert_array_equal(got, orc.embedding_bwd(dout, idx.astype(np.int32), vocab))
        unused = np.setdiff1d(np.arange(vocab), idx)
        if unused.size:
            assert np.all(got[unused] == 0.0)


def test_noalloc_empty_writes_zeros(M, rt):
    rc, got = _noalloc(M, rt, np.zeros((0, 16), np.float32), np.zeros(0, np.int32), 7, 16)
    assert rc == 0
    assert got.shape == (7, 16) and np.all(got == 0.0)


def test_noalloc_skips_out_of_range_ids(M, rt, orc):
    rng = np.random.default_rng(7)
    n, vocab, dim = 2048, 50, 32
    idx = rng.integers(0, vocab, n).astype(np.int32)
    idx[5], idx[1500] = vocab, -3           # outside [0, vocab): skipped, not reported
    dout = rng.standard_normal((n, dim)).astype(np.float32)
    rc, got = _noalloc(M, rt, dout, idx, vocab, dim)
    assert rc == 0
    keep = (idx >= 0) & (idx < vocab)
    np.testing.assert_array_equal(got, orc.embedding_bwd(dout[keep], idx[keep], vocab))
    assert rt.malus_device_error() == 0      # the runtime's error word is untouched


def test_noalloc_rejects_oversize(M, rt):
    rc = rt.malus_embedding_bwd_noalloc(None, None, 5, 65537, 65, 8, None, None)
    assert rc < 0
    rc = rt.malus_embedding_bwd_noalloc(None, None, 5, 8192, 100000, 8, None, None)
    assert rc < 0
    rc = rt.malus_embedding_bwd_noalloc(None, None, 3, 16, 4, 8, None, None)   # not an index dtype
    assert rc < 0
