"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the checker used by tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg.  Nothing in malus_b200/ imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

i32, i64, u64, f32, vp = C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_void_p


class OrCfg(C.Structure):
    _fields_ = [("vocab", i32), ("n_layer", i32), ("n_head", i32), ("n_embd", i32),
                ("block_size", i32), ("batch", i32), ("tied", i32),
                ("lr", f32), ("beta1", f32), ("beta2", f32), ("eps", f32), ("wd", f32),
                ("init_std", f32), ("mode", i32), ("use_graph", i32), ("seed", u64)]


_SIG = {
    "or_set_threads": (None, [C.c_int]),
    "or_get_threads": (C.c_int, []),
    "or_matmul": (None, [vp, vp, vp, i64, i64, i64, i64, i64, i64]),
    "or_broadcast_shape": (C.c_int, [vp, C.c_int, vp, C.c_int, vp]),
    "or_broadcast": (None, [C.c_int, vp, vp, C.c_int, vp, vp, C.c_int, vp]),
    "or_reduce": (None, [C.c_int, vp, i64, i64, i64, vp]),
    "or_softmax": (None, [vp, i64, i64, i64, vp]),
    "or_softmax_bwd": (None, [vp, vp, i64, i64, i64, vp]),
    "or_layernorm": (None, [vp, i64, i64, i64, f32, vp, vp]),
    "or_layernorm_bwd": (None, [vp, vp, vp, i64, i64, i64, f32, vp]),
    "or_unary": (None, [C.c_int, vp, vp, i64, f32]),
    "or_unary_bwd": (None, [C.c_int, vp, vp, vp, i64]),
    "or_xent": (None, [vp, vp, i64, i64, vp, vp]),
    "or_xent_bwd": (None, [vp, vp, f32, i64, i64, vp]),
    "or_embedding": (None, [vp, vp, i64, i64, i64, vp]),
    "or_embedding_bwd": (None, [vp, vp, i64, i64, i64, vp]),
    "or_permute": (None, [vp, vp, C.c_int, vp, vp]),
    "or_philox4x32_10": (None, [vp, C.c_uint32, C.c_uint32]),
    "or_randn": (None, [vp, i64, u64]),
    "or_rand_int": (i64, [i64, u64]),
    "or_rand_uniform": (f32, [u64]),
    "or_adamw": (None, [vp, vp, vp, vp, i64, f32, f32, f32, f32, f32, i64, f32]),
    "or_xor_train": (None, [C.c_int, f32, vp, vp]),
    "or_gpt_create": (i64, [C.POINTER(OrCfg)]),
    "or_gpt_destroy": (None, [i64]),
    "or_gpt_num_params": (i32, [i64]),
    "or_gpt_param_size": (i64, [i64, i32]),
    "or_gpt_get_param": (None, [i64, i32, vp]),
    "or_gpt_set_param": (None, [i64, i32, vp]),
    "or_gpt_get_grad": (None, [i64, i32, vp]),
    "or_gpt_step": (f32, [i64, vp, vp]),
}

_lib = None


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "oracle.cpp").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
    return LIB


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = C.CDLL(str(LIB))
        for k, (r, a) in _SIG.items():
            f = getattr(lib, k)
            f.restype = r
            f.argtypes = a
        _lib = lib
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(vp)


def f32a(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def matmul(a, b):
    a, b = f32a(a), f32a(b)
    if a.ndim == 2 and b.ndim == 2:
        out = np.empty((a.shape[0], b.shape[1]), np.float32)
        load().or_matmul(_p(a), _p(b), _p(out), a.shape[0], a.shape[1], b.shape[1], 1, 0, 0)
    elif a.ndim == 3 and b.ndim == 3:
        out = np.empty((a.shape[0], a.shape[1], b.shape[2]), np.float32)
        load().or_matmul(_p(a), _p(b), _p(out), a.shape[1], a.shape[2], b.shape[2], a.shape[0],
                         a.shape[1] * a.shape[2], b.shape[1] * b.shape[2])
    else:  # (3, 2)
        out = np.empty((a.shape[0], a.shape[1], b.shape[1]), np.float32)
        load().or_matmul(_p(a), _p(b), _p(out), a.shape[1], a.shape[2], b.shape[1], a.shape[0],
                         a.shape[1] * a.shape[2], 0)
    return out


def broadcast(op: int, a, b):
    a, b = f32a(a), f32a(b)
    sa = np.array(a.shape or (1,), np.int64)
    sb = np.array(b.shape or (1,), np.int64)
    so = np.zeros(8, np.int64)
    n = load().or_broadcast_shape(_p(sa), len(sa), _p(sb), len(sb), _p(so))
    if n < 0:
        raise ValueError("broadcast mismatch")
    out = np.empty(tuple(so[:n]), np.float32)
    load().or_broadcast(op, _p(a), _p(sa), len(sa), _p(b), _p(sb), len(sb), _p(out))
    return out


def _split(shape, axis):
    axis = axis % len(shape)
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    return outer, shape[axis], inner, axis


def reduce(op: int, x, axis: int, keepdim: bool = False):
    x = f32a(x)
    outer, n, inner, ax = _split(x.shape, axis)
    out = np.empty(outer * inner, np.float32)
    load().or_reduce(op, _p(x), outer, n, inner, _p(out))
    if x.ndim == 1:
        return out.reshape(1)
    shp = list(x.shape)
    if keepdim:
        shp[ax] = 1
    else:
        shp.pop(ax)
    return out.reshape(shp)


def softmax(x, axis):
    x = f32a(x)
    outer, n, inner, _ = _split(x.shape, axis)
    y = np.empty_like(x)
    load().or_softmax(_p(x), outer, n, inner, _p(y))
    return y


def softmax_bwd(s, g, axis):
    s, g = f32a(s), f32a(g)
    outer, n, inner, _ = _split(s.shape, axis)
    dx = np.empty_like(s)
    load().or_softmax_bwd(_p(s), _p(g), outer, n, inner, _p(dx))
    return dx


def layernorm(x, axis, eps=1e-5):
    x = f32a(x)
    outer, n, inner, ax = _split(x.shape, axis)
    y = np.empty_like(x)
    var = np.empty(outer * inner, np.float32)
    load().or_layernorm(_p(x), outer, n, inner, eps, _p(y), _p(var))
    vs = list(x.shape)
    vs[ax] = 1
    return y, var.reshape(vs)


def layernorm_bwd(y, var, g, axis, eps=1e-5):
    y, var, g = f32a(y), f32a(var), f32a(g)
    outer, n, inner, _ = _split(y.shape, axis)
    dx = np.empty_like(y)
    load().or_layernorm_bwd(_p(y), _p(var), _p(g), outer, n, inner, eps, _p(dx))
    return dx


UNARY = {"relu": 0, "sigmoid": 1, "tanh": 2, "exp": 3, "log": 4, "sqrt": 5, "abs": 6, "gelu": 7,
         "rsqrt_eps": 8, "neg": 9}
UNARY_BWD = {"sigmoid": 0, "relu": 1, "tanh": 2, "sqrt": 3, "abs": 4, "gelu": 5, "eq": 6}


def unary(name, x, p=0.0):
    x = f32a(x)
    y = np.empty_like(x)
    load().or_unary(UNARY[name], _p(x), _p(y), x.size, p)
    return y


def unary_bwd(name, x, g):
    x, g = f32a(x), f32a(g)
    y = np.empty_like(x)
    load().or_unary_bwd(UNARY_BWD[name], _p(x), _p(g), _p(y), x.size)
    return y


def xent(logits, t):
    logits = f32a(logits)
    t = np.ascontiguousarray(t, np.int32)
    probs = np.empty_like(logits)
    loss = np.zeros(1, np.float32)
    load().or_xent(_p(logits), _p(t), logits.shape[0], logits.shape[1], _p(probs), _p(loss))
    return loss, probs


def xent_bwd(probs, t, dout0):
    probs = f32a(probs)
    t = np.ascontiguousarray(t, np.int32)
    dx = np.empty_like(probs)
    load().or_xent_bwd(_p(probs), _p(t), dout0, probs.shape[0], probs.shape[1], _p(dx))
    return dx


def embedding(w, idx):
    w = f32a(w)
    idx = np.ascontiguousarray(idx, np.int32)
    out = np.empty((idx.size, w.shape[1]), np.float32)
    load().or_embedding(_p(w), _p(idx), idx.size, w.shape[0], w.shape[1], _p(out))
    return out


def embedding_bwd(dout, idx, vocab):
    dout = f32a(dout)
    idx = np.ascontiguousarray(idx, np.int32)
    dw = np.empty((vocab, dout.shape[1]), np.float32)
    load().or_embedding_bwd(_p(dout), _p(idx), idx.size, vocab, dout.shape[1], _p(dw))
    return dw


def permute(x, perm):
    x = f32a(x)
    shp = np.array(x.shape, np.int64)
    p = np.array(perm, np.int32)
    out = np.empty(tuple(x.shape[i] for i in perm), np.float32)
    load().or_permute(_p(x), _p(shp), x.ndim, _p(p), _p(out))
    return out


def randn(shape, call_idx):
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    load().or_randn(_p(out), n, call_idx)
    return out.reshape(shape)


def philox4x32_10(ctr, key):
    """The Philox4x32-10 block function on a 4-word counter and a 2-word key."""
    c = np.ascontiguousarray(ctr, np.uint32).copy()
    load().or_philox4x32_10(c.ctypes.data_as(C.c_void_p), int(key[0]), int(key[1]))
    return c


def rand_int(n, call_idx):
    return load().or_rand_int(n, call_idx)


def rand_uniform(call_idx):
    return load().or_rand_uniform(call_idx)


def adamw(p, g, m, v, lr, b1, b2, eps, wd, step, gscale=1.0):
    """In place on float32 arrays p, m, v."""
    load().or_adamw(_p(p), _p(g) if g is not None else None, _p(m), _p(v), p.size, lr, b1, b2,
                    eps, wd, step, gscale)


def xor_train(steps=10000, lr=1.5):
    loss = np.zeros(1, np.float32)
    preds = np.zeros(4, np.float32)
    load().or_xor_train(steps, lr, _p(loss), _p(preds))
    return float(loss[0]), preds


class Gpt:
    def __init__(self, vocab, n_layer, n_head, n_embd, block_size, batch, tied=False, lr=1e-3,
                 beta1=0.9, beta2=0.99, eps=1e-8, wd=0.1, init_std=0.02, seed=0):
        self.cfg = OrCfg(vocab, n_layer, n_head, n_embd, block_size, batch, int(tied), lr, beta1,
                         beta2, eps, wd, init_std, 0, 0, seed)
        self.h = load().or_gpt_create(C.byref(self.cfg))

    def step(self, x, y) -> float:
        x = np.ascontiguousarray(x, np.int32)
        y = np.ascontiguousarray(y, np.int32)
        return float(load().or_gpt_step(self.h, _p(x), _p(y)))

    def params(self):
        lib = load()
        out = []
        for i in range(lib.or_gpt_num_params(self.h)):
            a = np.empty(lib.or_gpt_param_size(self.h, i), np.float32)
            lib.or_gpt_get_param(self.h, i, _p(a))
            out.append(a)
        return out

    def grads(self):
        lib = load()
        out = []
        for i in range(lib.or_gpt_num_params(self.h)):
            a = np.empty(lib.or_gpt_param_size(self.h, i), np.float32)
            lib.or_gpt_get_grad(self.h, i, _p(a))
            out.append(a)
        return out

    def close(self):
        if self.h:
            load().or_gpt_destroy(self.h)
            self.h = 0


def set_threads(n: int | None = None) -> int:
    n = n or os.cpu_count() or 1
    load().or_set_threads(n)
    return n
