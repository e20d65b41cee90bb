"""CPU: SafeTensors files written and read by the runtime's host entry points
(malus_safetensors_write_host / _names / _read_host), checked against the
published `safetensors` library in both directions, plus files the reader
must refuse (interop spec: docs/spec/08-interop.md "SafeTensors [v1]")."""
import ctypes as C
import json
import struct

import numpy as np
import pytest

st_np = pytest.importorskip("safetensors.numpy")

DT = {np.dtype(np.float32): 0, np.dtype(np.int32): 5, np.dtype(np.int64): 6}
CODE = {v: k for k, v in DT.items()}


@pytest.fixture(scope="module")
def lib():
    import malus_b200 as M
    return M.load()


def write_host(lib, path, arrays: dict):
    names = list(arrays)
    arrs = [a if a.flags.c_contiguous else a.copy() for a in arrays.values()]   # keeps 0-d arrays 0-d
    n = len(arrs)
    shape_bufs = [(C.c_size_t * max(1, a.ndim))(*a.shape) for a in arrs]
    shapes = (C.POINTER(C.c_size_t) * n)(*[C.cast(b, C.POINTER(C.c_size_t)) for b in shape_bufs])
    ndims = (C.c_size_t * n)(*[a.ndim for a in arrs])
    dts = (C.c_int32 * n)(*[DT[a.dtype] for a in arrs])
    data = (C.c_void_p * n)(*[a.ctypes.data for a in arrs])
    nm = (C.c_char_p * n)(*[k.encode() for k in names])
    return lib.malus_safetensors_write_host(str(path).encode(), n, nm, dts, shapes, ndims, data)


def read_host(lib, path, name):
    dt, nd = C.c_int32(), C.c_size_t()
    shape = (C.c_size_t * 8)()
    nbytes = lib.malus_safetensors_read_host(str(path).encode(), name.encode(), C.byref(dt), shape, C.byref(nd),
                                             None, 0)
    if nbytes < 0:
        return nbytes
    a = np.empty(tuple(shape[i] for i in range(nd.value)), CODE[dt.value])
    assert a.nbytes == nbytes
    got = lib.malus_safetensors_read_host(str(path).encode(), name.encode(), None, None, None,
                                          a.ctypes.data_as(C.c_void_p), a.nbytes)
    assert got == nbytes
    return a


def names(lib, path):
    need = lib.malus_safetensors_names(str(path).encode(), None, 0)
    if need < 0:
        return need
    buf = C.create_string_buffer(need + 1)
    lib.malus_safetensors_names(str(path).encode(), buf, need + 1)
    return [n for n in buf.value.decode().split("\n") if n]


def sample(rng):
    return {"wte": rng.standard_normal((65, 384)).astype(np.float32),
            "h.0.attn.wq": rng.standard_normal((384, 384)).astype(np.float32),
            "ids": rng.integers(0, 65, (4, 256)).astype(np.int32),
            "step": np.array(7, np.int64),
            "empty": np.zeros((0, 3), np.float32),
            'quote"and\\slash': np.arange(5, dtype=np.float32)}


def test_written_files_read_by_the_published_library(lib, tmp_path):
    rng = np.random.default_rng(1)
    arrays = sample(rng)
    path = tmp_path / "w.safetensors"
    assert write_host(lib, path, arrays) == 0
    got = st_np.load_file(str(path))
    assert set(got) == set(arrays)
    for k, a in arrays.items():
        assert got[k].dtype == a.dtype and got[k].shape == a.shape
        np.testing.assert_array_equal(got[k], a)
    raw = path.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    assert hlen % 8 == 0 and json.loads(raw[8:8 + hlen])["__metadata__"]["writer"] == "malus_b200"


def test_published_files_read_by_the_runtime(lib, tmp_path):
    rng = np.random.default_rng(2)
    arrays = sample(rng)
    path = tmp_path / "p.safetensors"
    st_np.save_file(arrays, str(path), metadata={"origin": "test"})
    assert sorted(names(lib, path)) == sorted(arrays)
    for k, a in arrays.items():
        b = read_host(lib, path, k)
        assert b.dtype == a.dtype and b.shape == a.shape
        np.testing.assert_array_equal(b, a)
    assert read_host(lib, path, "absent") == -6


def test_refusals(lib, tmp_path):
    a = {"x": np.ones((2, 2), np.float32)}
    good = tmp_path / "g.safetensors"
    assert write_host(lib, good, a) == 0
    raw = good.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + hlen])

    def variant(name, blob):
        p = tmp_path / name
        p.write_bytes(blob)
        return names(lib, p)

    assert variant("short", raw[:5]) == -2                                   # no length field
    assert variant("long", struct.pack("<Q", 10 ** 6) + raw[8:]) == -2       # header past the end
    assert variant("json", struct.pack("<Q", 8) + b"{not js}" + raw[8 + hlen:]) == -3
    for field, value, code in (("dtype", "F16", -4), ("shape", [2, -1], -4), ("data_offsets", [0, 12], -5),
                               ("data_offsets", [8, 24], -5)):
        h = json.loads(json.dumps(header))
        h["x"][field] = value
        hb = json.dumps(h).encode()
        hb += b" " * (-len(hb) % 8)
        assert variant(f"bad_{field}_{code}", struct.pack("<Q", len(hb)) + hb + raw[8 + hlen:]) == code
    # overlapping tensors
    h = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
         "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}
    hb = json.dumps(h).encode()
    assert variant("overlap", struct.pack("<Q", len(hb)) + hb + bytes(16)) == -5
    assert names(lib, tmp_path / "missing.safetensors") == -1


def test_write_refuses_bad_names(lib, tmp_path):
    x = np.ones(3, np.float32)
    assert write_host(lib, tmp_path / "a", {"": x}) == -4
    assert write_host(lib, tmp_path / "b", {"__metadata__": x}) == -4
    assert write_host(lib, tmp_path / "c", {"ok": np.ones(3, np.float64).astype(np.float32)}) == 0
