"""User-kernel path on CPU: codegen-gpu's MSL is translated to CUDA C++ and
compiled by NVRTC for sm_100a (compilation needs no GPU)."""
import ctypes as C

import pytest

import msl_kernels as K


def translate(rt, src):
    buf = C.create_string_buffer(1 << 16)
    n = rt.malus_jit_translate(src.encode(), buf, len(buf))
    return n, buf.value.decode()


@pytest.mark.parametrize("name", sorted(K.ALL))
def test_translate_and_compile_for_sm100a(rt, name):
    src = K.ALL[name]
    n, cuda = translate(rt, src)
    assert n > 0, cuda
    assert 'extern "C" __global__ void malus_kernel_' in cuda
    assert "metal" not in cuda and "[[" not in cuda and "threadgroup_barrier" not in cuda
    log = C.create_string_buffer(1 << 16)
    rc = rt.malus_jit_compile_check(src.encode(), log, len(log))
    assert rc == 0, log.value.decode() + "\n" + cuda


def test_translation_details(rt):
    _, add = translate(rt, K.ADD)
    assert "if ((unsigned long long)tid >= __malus_n) return;" in add       # implicit: exact thread count
    assert "const uint tid = (uint)(blockIdx.x * blockDim.x + threadIdx.x);" in add
    _, sm = translate(rt, K.SOFTMAX)
    assert "__shared__ float scratch[1024];" in sm
    assert sm.count("__syncthreads()") == 3
    assert "fmaxf(" in sm and "expf(" in sm
    assert "const Uniforms_20 u" in sm and "const TensorMeta input_meta" in sm
    assert "const uint _tgid = (uint)blockIdx.x;" in sm
    assert "__malus_n) return" not in sm                                      # explicit: no guard
    _, ln = translate(rt, K.LAYERNORM)
    assert "rsqrtf(" in ln


@pytest.mark.parametrize("bad", [
    "int main() { return 0; }",
    K.HEAD + "kernel void k(\n    texture2d<float> t [[texture(0)]]\n) {\n}\n",
    K.HEAD + "kernel void k(\n    device float* out [[buffer(0)]],\n    uint s [[simdgroup_index_in_threadgroup]]\n) {\n}\n",
])
def test_unsupported_sources_are_rejected(rt, bad):
    n, msg = translate(rt, bad)
    assert n == -1 and msg.startswith("error:")


def test_compile_errors_are_reported(rt):
    src = K.ADD.replace("(a[tid] + b[tid])", "(a[tid] + undefined_name)")
    log = C.create_string_buffer(1 << 16)
    assert rt.malus_jit_compile_check(src.encode(), log, len(log)) == -2
    assert "undefined_name" in log.value.decode()
