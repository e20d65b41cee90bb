"""GPU: saving device tensors to SafeTensors files and loading them back
(malus_save_safetensors / malus_load_safetensors; the interop spec's
`save(tensors, path)` and `load(path)`, docs/spec/08-interop.md).  Files
written from device memory are read by the published `safetensors` library;
loading gives back the same bits.  Views and deferred results are saved as
the values they stand for; a model's parameters survive a round trip."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
st_np = pytest.importorskip("safetensors.numpy")


def test_round_trip_of_plain_view_and_deferred_tensors(M, rt, rng, tmp_path):
    w = rng.standard_normal((384, 1152)).astype(np.float32)
    x = rng.standard_normal((64, 32, 48)).astype(np.float32)
    big = rng.standard_normal((256, 512)).astype(np.float32)
    ids = rng.integers(0, 65, (8, 128)).astype(np.int32)
    pos = np.arange(1000, dtype=np.int64)
    tw, tx, tb, ti, tp = (M.Tensor.from_numpy(a) for a in (w, x, big, ids, pos))
    ts = M.Tensor.from_numpy(np.array([[0.125]], np.float32))
    view = M.Tensor(rt.tensor_permute(tx.h, (C.c_size_t * 3)(2, 0, 1), 3))        # strided view
    scaled = M.Tensor(rt.__broadcast_mul_fwd(tb.h, ts.h))                         # deferred x * s
    tensors = {"w": tw, "x.permuted": view, "big.scaled": scaled, "ids": ti, "pos": tp}
    want = {"w": w, "x.permuted": np.transpose(x, (2, 0, 1)), "big.scaled": big * np.float32(0.125),
            "ids": ids, "pos": pos}
    path = tmp_path / "t.safetensors"
    M.save_safetensors(path, tensors)
    got = st_np.load_file(str(path))
    assert list(got) and set(got) == set(want)
    for k, a in want.items():
        assert got[k].dtype == a.dtype and got[k].shape == a.shape, k
        np.testing.assert_array_equal(got[k], a)
    back = M.load_safetensors(path)
    assert M.safetensors_names(path) == list(tensors)          # header order = the order given
    for k, a in want.items():
        np.testing.assert_array_equal(back[k].numpy(), a)
    assert rt.malus_load_safetensors(str(path).encode(), b"absent") == 0


def test_published_file_loaded_onto_the_gpu(M, rng, tmp_path):
    arrays = {"a": rng.standard_normal((3, 5)).astype(np.float32), "b": np.arange(7, dtype=np.int32),
              "scalar": np.array(3.5, np.float32)}
    path = tmp_path / "p.safetensors"
    st_np.save_file(arrays, str(path))
    back = M.load_safetensors(path)
    for k, a in arrays.items():
        b = back[k].numpy()
        assert b.dtype == a.dtype and b.shape == a.shape
        np.testing.assert_array_equal(b, a)


def test_model_parameters_round_trip(M, rt, tmp_path):
    cfg = dict(vocab=65, n_layer=2, n_head=4, n_embd=64, block_size=32, batch=4)
    g = M.GPT(**cfg, lr=1e-3, mode=1)
    rng = np.random.default_rng(3)
    m = cfg["batch"] * cfg["block_size"]
    g.step(rng.integers(0, 65, m).astype(np.int32), rng.integers(0, 65, m).astype(np.int32))
    n = rt.malus_gpt_num_params(g.h)
    handles = {f"param.{i}": rt.malus_gpt_param(g.h, i) for i in range(n)}
    path = tmp_path / "model.safetensors"
    M.save_safetensors(path, handles)
    before = g.params()
    back = M.load_safetensors(path)
    for i, p in enumerate(before):
        np.testing.assert_array_equal(back[f"param.{i}"].numpy().reshape(p.shape), p)
    g.close()
