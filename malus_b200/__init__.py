"""malus_b200 — the sm_100a (B200) runtime behind malus's C ABI.

The product is ``libmalus_runtime_cuda.so`` (CUDA kernels + the C ABI declared
in ``include/malus_runtime.h``).  This module only loads it and gives Python
callers the same entry points with ctypes signatures, plus two thin
conveniences (``Tensor`` for handles, ``GPT`` for the compiled training step).
There is no CPU fallback: loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libmalus_runtime_cuda.so"

i32, i64, u64, f32, sz, vp = C.c_int32, C.c_int64, C.c_uint64, C.c_float, C.c_size_t, C.c_void_p
P_sz, P_i64, P_u64, P_f32, P_u8, P_i32 = (C.POINTER(C.c_size_t), C.POINTER(C.c_int64),
                                          C.POINTER(C.c_uint64), C.POINTER(C.c_float),
                                          C.POINTER(C.c_uint8), C.POINTER(C.c_int32))


class TcOperand(C.Structure):
    _fields_ = [("hi", vp), ("lo", vp), ("rows", i64), ("cols", i64), ("pitch", i64),
                ("nz", i32), ("zstride", i64), ("mn_major", i32), ("zmode", i32), ("seg", i32)]


class TcLayout(C.Structure):
    _fields_ = [("d1", i64), ("s1", i64), ("d2", i64), ("s2", i64), ("s3", i64)]


class TcProblem(C.Structure):
    _fields_ = [("M", i32), ("N", i32), ("K", i32), ("batch", i32), ("a", TcOperand), ("b", TcOperand),
                ("epi", i32), ("oz", TcLayout), ("om", TcLayout), ("on", TcLayout),
                ("out", vp), ("out_hi", vp), ("out_lo", vp), ("aux", vp), ("alpha", f32), ("beta", f32),
                ("causal", i32), ("aux_lo", vp), ("rowv", vp)]


class GptConfig(C.Structure):
    _fields_ = [("vocab", i32), ("n_layer", i32), ("n_head", i32), ("n_embd", i32),
                ("block_size", i32), ("batch", i32), ("tied", i32),
                ("lr", f32), ("beta1", f32), ("beta2", f32), ("eps", f32), ("wd", f32),
                ("init_std", f32), ("mode", i32), ("use_graph", i32), ("seed", u64)]


# name -> (restype, argtypes); mirrors include/malus_runtime.h one to one
SIGNATURES: dict[str, tuple] = {
    # 1. RuntimeSymbols
    "tensor_alloc_gpu": (i64, [i32, P_sz, sz, vp]),
    "tensor_alloc_zeros_gpu": (i64, [P_sz, sz]),
    "tensor_alloc_ones_gpu": (i64, [P_sz, sz]),
    "tensor_free": (None, [i64]),
    "tensor_retain": (None, [i64]),
    "tensor_release": (None, [i64]),
    "tensor_print": (None, [i64]),
    "tensor_len": (i64, [i64]),
    "tensor_ndim": (i64, [i64]),
    "tensor_dim": (i64, [i64, i64]),
    "kernel_dispatch": (i64, [u64, P_i64, sz]),
    "kernel_dispatch_v2": (i64, [u64, P_i64, sz, P_sz, P_sz, P_sz, sz, i32, vp, sz]),
    "gpu_barrier": (None, []),
    "tensor_matmul": (i64, [i64, i64]),
    "tensor_reshape": (i64, [i64, P_sz, sz]),
    "tensor_permute": (i64, [i64, P_sz, sz]),
    "tensor_causal_mask": (i64, [i64]),
    "tensor_randn": (i64, [P_sz, sz]),
    "malus_rand_uniform": (f32, []),
    "malus_rand_int": (i64, [i64]),
    "malus_tensor_get_f32": (f32, [i64, i64]),
    "tape_record_binop": (None, [i32, i64, i64, i64]),
    "tape_record_unary": (None, [i32, i64, i64]),
    "tape_record_reduce": (None, [i32, i64, i64, i64, i64]),
    "tape_record_perm": (None, [i32, i64, i64, P_sz, sz]),
    "tape_record_layernorm": (None, [i32, i64, i64, i64, i64]),
    "tape_record_cross_entropy": (None, [i32, i64, i64, i64, i64]),
    "tape_record_embedding": (None, [i32, i64, i64, i64]),
    "tape_register_leaf": (None, [i64]),
    "tape_pause": (None, []),
    "tape_resume": (None, []),
    "tape_clear": (None, []),
    "tape_get_grad": (i64, [i64]),
    "backward": (None, [i64]),
    "tape_zero_grad": (None, [P_i64, sz]),
    "tape_register_backward_fn": (None, [i32, sz]),
    "malus_buffer_i32": (i64, [i64]),
    "malus_buffer_get_i32": (i64, [i64, i64]),
    "malus_buffer_set_i32": (None, [i64, i64, i64]),
    "malus_buffer_free": (None, [i64]),
    "malus_buffer_freeze_i32": (i64, [i64]),
    "malus_record_diff": (None, [f32]),
    "bench_step_begin": (None, []),
    "bench_step_end": (None, []),
    "malus_str_box": (i64, [P_u8, sz]),
    "malus_read_file": (i64, [i64]),
    "malus_str_len": (i64, [i64]),
    "malus_str_char_at": (i64, [i64, i64]),
    "malus_str_from_char": (i64, [i64]),
    # 2. runtime API
    "malus_runtime_init": (None, [P_u64, C.POINTER(C.c_char_p), sz]),
    "malus_cpu_compute_count": (i64, []),
    "malus_cpu_compute_reset": (None, []),
    "malus_gradcheck_max_diff": (f32, []),
    "malus_gradcheck_reset": (None, []),
    "malus_rc_counts": (None, [P_i64, P_i64, P_i64]),
    "malus_rc_reset": (None, []),
    "malus_pool_stats": (None, [P_i64, P_i64, P_i64, P_i64]),
    "malus_pool_reset": (None, []),
    "malus_set_mem_budget": (None, [i64]),
    "bench_enable": (None, []),
    "bench_report": (C.c_double, [P_i64]),
    "bench_report_range": (None, [C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "bench_reset": (None, []),
    "malus_tape_reset": (None, []),
    "malus_tape_registry_lens": (None, [P_i64, P_i64]),
    "malus_tensor_data": (vp, [i64]),
    "malus_tensor_dtype": (i32, [i64]),
    "malus_tensor_read": (None, [i64, vp, sz]),
    "malus_tensor_write": (None, [i64, vp, sz]),
    "malus_tensor_wrap": (i64, [i32, vp, P_sz, sz]),
    "malus_rng_reset": (None, [u64]),
    "malus_philox4x32_10": (None, [C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "malus_set_device": (None, [i32]),
    "malus_launch_count": (i64, []),
    "malus_launch_count_reset": (None, []),
    "malus_stream": (vp, []),
    # 3. native stdlib host functions
    "__broadcast_add_fwd": (i64, [i64, i64]),
    "__broadcast_sub_fwd": (i64, [i64, i64]),
    "__broadcast_mul_fwd": (i64, [i64, i64]),
    "__broadcast_div_fwd": (i64, [i64, i64]),
    "__softmax_fwd": (i64, [i64, i64]),
    "__layernorm_fwd": (i64, [i64, i64]),
    "__cross_entropy_fwd": (i64, [i64, i64]),
    "__embedding_fwd": (i64, [i64, i64]),
    "__gelu_fwd": (i64, [i64]),
    "__reduce_sum_fwd": (i64, [i64, i64, i64]),
    "__reduce_mean_fwd": (i64, [i64, i64, i64]),
    "__reduce_max_fwd": (i64, [i64, i64, i64]),
    "__reduce_var_fwd": (i64, [i64, i64, i64]),
    "__reduce_all_sum_fwd": (i64, [i64]),
    "__permute_nd_fwd": (i64, [i64] * 9),
    "__transpose_2d_fwd": (i64, [i64]),
    "__scale_fwd": (i64, [i64, f32]),
    "__fill_like_fwd": (i64, [i64, f32]),
    "__eq_fwd": (i64, [i64, i64]),
    "__expand_axis_fwd": (i64, [i64, i64, i64]),
    "__sum_to_shape_bwd": (i64, [i64, i64]),
    "__rsqrt_eps_fwd": (i64, [i64, f32]),
    "__add_bwd_a": (i64, [i64, i64]),
    "__add_bwd_b": (i64, [i64, i64]),
    "__sub_bwd_a": (i64, [i64, i64]),
    "__sub_bwd_b": (i64, [i64, i64]),
    "__mul_bwd_a": (i64, [i64, i64, i64]),
    "__mul_bwd_b": (i64, [i64, i64, i64]),
    "__div_bwd_a": (i64, [i64, i64, i64]),
    "__div_bwd_b": (i64, [i64, i64, i64]),
    "__sigmoid_bwd": (i64, [i64, i64]),
    "__relu_bwd": (i64, [i64, i64]),
    "__tanh_bwd": (i64, [i64, i64]),
    "__sqrt_bwd": (i64, [i64, i64]),
    "__abs_bwd": (i64, [i64, i64]),
    "__sum_bwd": (i64, [i64, i64]),
    "__reduce_sum_axis_bwd": (i64, [i64, i64, i64]),
    "__reduce_mean_axis_bwd": (i64, [i64, i64, i64]),
    "__reduce_max_axis_bwd": (i64, [i64, i64, i64, i64]),
    "__reduce_var_axis_bwd": (i64, [i64, i64, i64]),
    "__softmax_bwd": (i64, [i64, i64, i64]),
    "__layernorm_bwd": (i64, [i64, i64, i64, i64]),
    "__gelu_bwd": (i64, [i64, i64]),
    "__cross_entropy_bwd": (i64, [i64, i64, i64]),
    "__embedding_bwd": (i64, [i64, i64, i64]),
    "__matmul_bwd_a": (i64, [i64, i64, i64]),
    "__matmul_bwd_b": (i64, [i64, i64, i64]),
    # 4. new in this build
    "malus_adamw_multi": (None, [P_i64, P_i64, P_i64, P_i64, sz, f32, f32, f32, f32, f32, i64, f32]),
    "malus_dp_unique_id": (i32, [P_u8]),
    "malus_dp_init": (i32, [i32, i32, P_u8, i32]),
    "malus_dp_allreduce_f32": (i32, [vp, sz]),
    "malus_dp_finish": (i32, []),
    "malus_dp_destroy": (i32, []),
    "malus_jit_translate": (i32, [C.c_char_p, C.c_char_p, sz]),
    "malus_jit_compile_check": (i32, [C.c_char_p, C.c_char_p, sz]),
    "malus_attn_fwd": (i32, [vp, vp, i32, i32, i32, i32, f32, vp, vp, vp, vp, vp]),
    "malus_attn_set_resident": (i32, [i32]),
    "malus_safetensors_write_host": (i32, [C.c_char_p, sz, C.POINTER(C.c_char_p), C.POINTER(i32),
                                             C.POINTER(C.POINTER(sz)), C.POINTER(sz), C.POINTER(vp)]),
    "malus_safetensors_names": (i32, [C.c_char_p, C.c_char_p, i32]),
    "malus_safetensors_read_host": (i64, [C.c_char_p, C.c_char_p, C.POINTER(i32), C.POINTER(sz), C.POINTER(sz),
                                          vp, sz]),
    "malus_save_safetensors": (i32, [C.c_char_p, sz, C.POINTER(C.c_char_p), C.POINTER(i64)]),
    "malus_load_safetensors": (i64, [C.c_char_p, C.c_char_p]),
    "malus_attn_bwd": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, vp, vp]),
    "malus_graph_begin": (i32, []),
    "malus_graph_end": (i64, []),
    "malus_graph_replay": (i32, [i64]),
    "malus_graph_destroy": (i32, [i64]),
    "malus_dp_abort": (i32, []),
    "malus_dp_register_leaves": (i32, [P_i64, sz, sz]),
    "malus_dp_grad_ready": (i32, [i64, i64]),
    "malus_dp_world": (i32, []),
    "malus_gpt_create": (i64, [C.POINTER(GptConfig)]),
    "malus_gpt_destroy": (None, [i64]),
    "malus_gpt_step": (f32, [i64, P_i32, P_i32]),
    "malus_gpt_step_device": (None, [i64, vp, vp]),
    "malus_gpt_last_loss": (f32, [i64]),
    "malus_gpt_num_params": (i32, [i64]),
    "malus_gpt_param": (i64, [i64, i32]),
    "malus_gpt_grad": (i64, [i64, i32]),
    "malus_gpt_moment": (i64, [i64, i32, i32]),
    "malus_gpt_num_elements": (i64, [i64]),
    "malus_gpt_layout": (i32, [C.POINTER(GptConfig), P_i64, P_i64, i32, P_i64]),
    "malus_gpt_dp_buckets": (i32, [C.POINTER(GptConfig), P_i64, P_i64, i32]),
    "malus_device_error": (i32, []),
    "malus_tc_gemm": (None, [C.POINTER(TcProblem)]),
    "malus_gemm_pair_clusters": (i32, []),
    "malus_gemm_pair_mode": (i32, [i32]),
    "malus_tf32_split": (None, [vp, i64, i64, i64, i64, i64, vp, vp, i64]),
    "malus_prof_enable": (None, [i32]),
    "malus_embedding_bwd_noalloc": (i32, [vp, vp, i32, sz, sz, sz, vp, vp]),
    "malus_prof_report": (None, [i32, P_i64, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                 C.POINTER(C.c_double)]),
    "malus_prof_kernels": (i32, [C.c_char_p, i32]),
}

_lib: C.CDLL | None = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load the runtime library (once) and bind every declared entry point."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"malus_b200: {p} is missing — build it with `python malus_b200/build.py`"
                           " (there is no CPU fallback)")
    lib = C.CDLL(str(p), mode=C.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _shape_arr(shape):
    arr = (C.c_size_t * max(1, len(shape)))(*shape)
    return arr, len(shape)


DTYPES = {np.dtype(np.float32): 0, np.dtype(np.int32): 5, np.dtype(np.int64): 6}
NP_OF = {0: np.float32, 5: np.int32, 6: np.int64}


class Tensor:
    """Owning wrapper around a runtime handle (refcount released on close/del)."""

    __slots__ = ("h", "_owned")

    def __init__(self, handle: int, owned: bool = True):
        self.h = int(handle)
        self._owned = owned

    @staticmethod
    def from_numpy(a: np.ndarray) -> "Tensor":
        lib = load()
        a = np.ascontiguousarray(a)
        if a.dtype not in DTYPES:
            a = a.astype(np.float32)
        s, n = _shape_arr(a.shape)
        h = lib.tensor_alloc_gpu(DTYPES[a.dtype], s, n, a.ctypes.data_as(C.c_void_p))
        return Tensor(h)

    @property
    def shape(self) -> tuple:
        lib = load()
        return tuple(lib.tensor_dim(self.h, i) for i in range(lib.tensor_ndim(self.h)))

    @property
    def dtype(self):
        return NP_OF[load().malus_tensor_dtype(self.h)]

    def numpy(self) -> np.ndarray:
        lib = load()
        out = np.empty(self.shape, dtype=self.dtype)
        lib.malus_tensor_read(self.h, out.ctypes.data_as(C.c_void_p), out.nbytes)
        return out

    def close(self):
        if self._owned and self.h:
            load().tensor_release(self.h)
        self.h = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def save_safetensors(path: str | os.PathLike, tensors: dict) -> None:
    """Write named tensors (Tensor objects or raw handles) to a SafeTensors
    file, as malus's interop spec's `save(tensors, path)`."""
    lib = load()
    names = list(tensors)
    hs = [t.h if isinstance(t, Tensor) else int(t) for t in tensors.values()]
    arr_n = (C.c_char_p * len(names))(*[n.encode() for n in names])
    arr_h = (C.c_int64 * len(hs))(*hs)
    rc = lib.malus_save_safetensors(os.fsencode(path), len(names), arr_n, arr_h)
    if rc != 0:
        raise OSError(f"malus_save_safetensors({path}) failed with code {rc}")


def safetensors_names(path: str | os.PathLike) -> list[str]:
    lib = load()
    need = lib.malus_safetensors_names(os.fsencode(path), None, 0)
    if need < 0:
        raise ValueError(f"{path}: not a valid SafeTensors file (code {need})")
    buf = C.create_string_buffer(need + 1)
    lib.malus_safetensors_names(os.fsencode(path), buf, need + 1)
    return [n for n in buf.value.decode().split("\n") if n]


def load_safetensors(path: str | os.PathLike) -> dict:
    """Every tensor of a SafeTensors file on the GPU, by name (the spec's
    `load(path)`)."""
    lib = load()
    out = {}
    for n in safetensors_names(path):
        h = lib.malus_load_safetensors(os.fsencode(path), n.encode())
        if not h:
            raise ValueError(f"{path}: loading {n} failed")
        out[n] = Tensor(h)
    return out


def tuple_fields(box: int) -> tuple[int, int]:
    """Read (field+8, field+16) of a calloc'd tuple box and free it."""
    arr = (C.c_int64 * 3).from_address(box)
    a, b = int(arr[1]), int(arr[2])
    C.CDLL(None).free(C.c_void_p(box))
    return a, b


class GPT:
    """The compiled nanoGPT training step (malus_gpt_*)."""

    def __init__(self, vocab, n_layer, n_head, n_embd, block_size, batch, tied=False, lr=1e-3,
                 beta1=0.9, beta2=0.99, eps=1e-8, wd=0.1, init_std=0.02, mode=1, use_graph=0,
                 seed=0):
        lib = load()
        self.cfg = GptConfig(vocab, n_layer, n_head, n_embd, block_size, batch, int(tied), lr, beta1,
                             beta2, eps, wd, init_std, mode, use_graph, seed)
        self.h = lib.malus_gpt_create(C.byref(self.cfg))
        self.tokens_per_step = batch * block_size

    def step(self, x: np.ndarray, y: np.ndarray) -> float:
        x = np.ascontiguousarray(x, dtype=np.int32)
        y = np.ascontiguousarray(y, dtype=np.int32)
        return load().malus_gpt_step(self.h, x.ctypes.data_as(P_i32), y.ctypes.data_as(P_i32))

    def params(self) -> list[np.ndarray]:
        lib = load()
        return [Tensor(lib.malus_gpt_param(self.h, i), owned=False).numpy()
                for i in range(lib.malus_gpt_num_params(self.h))]

    def grads(self) -> list[np.ndarray]:
        """Gradients of the last step (before the update), in parameter order."""
        lib = load()
        return [Tensor(lib.malus_gpt_grad(self.h, i), owned=False).numpy()
                for i in range(lib.malus_gpt_num_params(self.h))]

    def moments(self) -> tuple[list[np.ndarray], list[np.ndarray]]:
        """AdamW first and second moments, in parameter order."""
        lib = load()
        n = lib.malus_gpt_num_params(self.h)
        return ([Tensor(lib.malus_gpt_moment(self.h, i, 0), owned=False).numpy() for i in range(n)],
                [Tensor(lib.malus_gpt_moment(self.h, i, 1), owned=False).numpy() for i in range(n)])

    def close(self):
        if self.h:
            load().malus_gpt_destroy(self.h)
            self.h = 0
