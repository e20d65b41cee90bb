"""User-kernel sources in the exact form malus-codegen-gpu emits
(crates/malus-codegen-gpu/src/lib.rs: synthesize_* :373-418, implicit-map
lowering :432-546, explicit lowering :643-1006 with the TensorMeta struct and
Uniforms_<id> struct, `threadgroup` arrays and barriers).  The kernels are
written here for the tests; their bodies follow the emitter's formatting
(parenthesised binary ops, `{:?}f` float literals, `(int)` thread ids)."""

HEAD = "#include <metal_stdlib>\nusing namespace metal;\n\n"

META = """struct TensorMeta {
    uint ndim;
    uint shape[8];
    uint strides[8];
};

"""

# builtin add (synthesize_elementwise_builtin)
ADD = HEAD + """kernel void malus_kernel_7(
    device float* a [[buffer(0)]],
    device float* b [[buffer(1)]],
    device float* out [[buffer(2)]],
    uint tid [[thread_position_in_grid]]
) {
    out[tid] = (a[tid] + b[tid]);
}
"""

# builtin sigmoid (synthesize_unary_builtin) and mul_scalar (synthesize_scalar_builtin)
SIGMOID = HEAD + """kernel void malus_kernel_900(
    device float* a [[buffer(0)]],
    device float* out [[buffer(1)]],
    uint tid [[thread_position_in_grid]]
) {
    out[tid] = 1.0f / (1.0f + exp(-a[tid]));
}
"""

MUL_SCALAR = HEAD + """kernel void malus_kernel_901(
    device float* a [[buffer(0)]],
    device float* scalar_val [[buffer(1)]],
    device float* out [[buffer(2)]],
    uint tid [[thread_position_in_grid]]
) {
    out[tid] = (a[tid] * scalar_val[0]);
}
"""

# examples/xor.ml:1-2 `kernel sigmoid_backward(grad_out, sig_z)` lowered as an implicit map
SIGMOID_BWD = HEAD + """kernel void malus_kernel_902(
    device float* grad_out [[buffer(0)]],
    device float* sig_z [[buffer(1)]],
    device float* out [[buffer(2)]],
    uint tid [[thread_position_in_grid]]
) {
    out[tid] = ((grad_out[tid] * sig_z[tid]) * (1.0f - sig_z[tid]));
}
"""

# multi-statement implicit body (let then return)
RELU_BWD = HEAD + """kernel void malus_kernel_3(
    device float* grad_out [[buffer(0)]],
    device float* x [[buffer(1)]],
    device float* out [[buffer(2)]],
    uint tid [[thread_position_in_grid]]
) {
    float mask = (x[tid] > 0.0f);
    out[tid] = (grad_out[tid] * mask);
}
"""

# explicit, thread_id, TensorMeta bound, tanh
GELU = HEAD + META + """kernel void malus_kernel_12(
    device const float* input [[buffer(0)]],
    device float* out [[buffer(1)]],
    constant TensorMeta& input_meta [[buffer(3)]],
    constant TensorMeta& out_meta [[buffer(4)]],
    uint _tid [[thread_position_in_grid]]
) {
    int i = (int)_tid;
    if ((i < (int)input_meta.shape[0])) {
        float x = input[i];
        out[i] = ((0.5f * x) * (1.0f + tanh((0.7978846f * (x + ((0.044715f * x) * (x * x)))))));
    }
}
"""

# explicit, one row per threadgroup: threadgroup scratch, barriers, a uniform, loops, fmax/exp
SOFTMAX = HEAD + META + """struct Uniforms_20 {
    int cols;
};

kernel void malus_kernel_20(
    device const float* input [[buffer(0)]],
    device float* out [[buffer(1)]],
    constant Uniforms_20& u [[buffer(2)]],
    constant TensorMeta& input_meta [[buffer(3)]],
    constant TensorMeta& out_meta [[buffer(4)]],
    uint _tgid [[threadgroup_position_in_grid]],
    uint _lid [[thread_position_in_threadgroup]]
) {
    int row = (int)_tgid;
    int col = (int)_lid;
    threadgroup float scratch[1024];
    if ((col == 0)) {
        float m = input[(row * u.cols)];
        for(int i = 1; i < u.cols; i++) {
            m = fmax(m, input[((row * u.cols) + i)]);
        }
        scratch[0] = m;
    }
    threadgroup_barrier(mem_flags::mem_threadgroup);
    if ((col < u.cols)) {
        scratch[(col + 1)] = exp((input[((row * u.cols) + col)] - scratch[0]));
    }
    threadgroup_barrier(mem_flags::mem_threadgroup);
    if ((col == 0)) {
        float s = 0.0f;
        for(int j = 0; j < u.cols; j++) {
            s = (s + scratch[(j + 1)]);
        }
        scratch[0] = s;
    }
    threadgroup_barrier(mem_flags::mem_threadgroup);
    if ((col < u.cols)) {
        out[((row * u.cols) + col)] = (scratch[(col + 1)] / scratch[0]);
    }
}
"""

# explicit: three uniforms of two types, strided 2-D indexing, rsqrt
LAYERNORM = HEAD + META + """struct Uniforms_21 {
    int cols;
    float inv_cols;
    float eps;
};

kernel void malus_kernel_21(
    device const float* input [[buffer(0)]],
    device float* out [[buffer(1)]],
    constant Uniforms_21& u [[buffer(2)]],
    constant TensorMeta& input_meta [[buffer(3)]],
    constant TensorMeta& out_meta [[buffer(4)]],
    uint _tgid [[threadgroup_position_in_grid]],
    uint _lid [[thread_position_in_threadgroup]]
) {
    int row = (int)_tgid;
    int col = (int)_lid;
    threadgroup float scratch[1024];
    scratch[col] = input[(row) * (int)input_meta.strides[0] + (col) * (int)input_meta.strides[1]];
    threadgroup_barrier(mem_flags::mem_threadgroup);
    if ((col == 0)) {
        float s = 0.0f;
        for(int i = 0; i < u.cols; i++) {
            s = (s + scratch[i]);
        }
        float mean = (s * u.inv_cols);
        float v = 0.0f;
        for(int i = 0; i < u.cols; i++) {
            v = (v + ((scratch[i] - mean) * (scratch[i] - mean)));
        }
        scratch[1000] = mean;
        scratch[1001] = rsqrt(((v * u.inv_cols) + u.eps));
    }
    threadgroup_barrier(mem_flags::mem_threadgroup);
    out[(row) * (int)out_meta.strides[0] + (col) * (int)out_meta.strides[1]] = ((scratch[col] - scratch[1000]) * scratch[1001]);
}
"""

ALL = {"add": ADD, "sigmoid": SIGMOID, "mul_scalar": MUL_SCALAR, "sigmoid_backward": SIGMOID_BWD,
       "relu_backward": RELU_BWD, "gelu": GELU, "softmax": SOFTMAX, "layernorm": LAYERNORM}
