// kernel_dispatch / kernel_dispatch_v2 (metal.rs:1860-2065).
//
// The reference compiles MSL for every kernel id handed to runtime_init.  This
// runtime has no MSL compiler; malus_runtime_init binds each id to a native
// kernel by name instead:
//  * builtins synthesised by codegen-gpu (lib.rs:373-418, names from
//    malus-syntax ast.rs:59-81): malus_{add,sub,mul,div}, malus_*_scalar,
//    relu/sigmoid/tanh/exp/log/sqrt/abs;
//  * every stdlib kernel of crates/malus-stdlib/stdlib (e.g.
//    "__softmax_kernel"), interpreting grid/uniforms exactly as its .ml host
//    function supplies them (uniforms are 4-byte f32/i32 in declaration
//    order, codegen-cpu lib.rs:2261-2297);
//  * the XOR example's user kernel "sigmoid_backward" (examples/xor.ml:1-2).
// A source text (containing `kernel void`) instead of a name is a user kernel
// body as codegen-gpu emits it: nvrtc.cu translates it to CUDA C++ and compiles
// it with NVRTC for sm_100a.
#include "common.cuh"

#include <mutex>
#include <string>
#include <unordered_map>

namespace malus {
void binary_project_into_a(int op, int64_t ha, int64_t hb, float* out);
struct JitKernel;
bool looks_like_msl(const char* s);
JitKernel* jit_compile(const std::string& msl);
void jit_dispatch_implicit(JitKernel* k, const int64_t* h, size_t count, int64_t out);
void jit_dispatch_explicit(JitKernel* k, const int64_t* h, size_t hc, const size_t* grid, const size_t* tg,
                           int64_t out, const void* u, size_t ub);
}
using namespace malus;

namespace {

enum Kid {
  K_ADD, K_SUB, K_MUL, K_DIV,
  K_ADD_S, K_SUB_S, K_RSUB_S, K_MUL_S, K_DIV_S, K_RDIV_S,
  K_RELU, K_SIGMOID, K_TANH, K_EXP, K_LOG, K_SQRT, K_ABS,
  K_USER_SIGMOID_BWD,
  // stdlib (kernel_dispatch_v2)
  K_BC_ADD, K_BC_SUB, K_BC_MUL, K_BC_DIV,
  K_SOFTMAX, K_LAYERNORM, K_LAYERNORM_VAR,
  K_RED_SUM, K_RED_MEAN, K_RED_MAX, K_RED_VAR,
  K_EXPAND_AXIS, K_GELU, K_GELU_BWD, K_XENT_NLL, K_XENT_BWD,
  K_EMBED, K_EMBED_BWD, K_TRANSPOSE_2D, K_PERMUTE_3D, K_PERMUTE_ND,
  K_SCALE, K_FILL_LIKE, K_EQ, K_SIGMOID_BWD, K_RELU_BWD, K_TANH_BWD, K_SQRT_BWD, K_ABS_BWD,
  K_RSQRT_EPS,
};

const std::unordered_map<std::string, int>& names() {
  static const std::unordered_map<std::string, int> m = {
      {"malus_add", K_ADD}, {"malus_sub", K_SUB}, {"malus_mul", K_MUL}, {"malus_div", K_DIV},
      {"malus_add_scalar", K_ADD_S}, {"malus_sub_scalar", K_SUB_S},
      {"malus_rsub_scalar", K_RSUB_S}, {"malus_mul_scalar", K_MUL_S},
      {"malus_div_scalar", K_DIV_S}, {"malus_rdiv_scalar", K_RDIV_S},
      {"relu", K_RELU}, {"sigmoid", K_SIGMOID}, {"tanh", K_TANH}, {"exp", K_EXP},
      {"log", K_LOG}, {"sqrt", K_SQRT}, {"abs", K_ABS},
      {"sigmoid_backward", K_USER_SIGMOID_BWD},
      {"__broadcast_add_kernel", K_BC_ADD}, {"__broadcast_sub_kernel", K_BC_SUB},
      {"__broadcast_mul_kernel", K_BC_MUL}, {"__broadcast_div_kernel", K_BC_DIV},
      {"__softmax_kernel", K_SOFTMAX}, {"__layernorm_kernel", K_LAYERNORM},
      {"__layernorm_var_kernel", K_LAYERNORM_VAR},
      {"__reduce_sum_kernel", K_RED_SUM}, {"__reduce_mean_kernel", K_RED_MEAN},
      {"__reduce_max_kernel", K_RED_MAX}, {"__reduce_var_kernel", K_RED_VAR},
      {"__expand_axis_kernel", K_EXPAND_AXIS}, {"__gelu_kernel", K_GELU},
      {"__gelu_bwd_kernel", K_GELU_BWD}, {"__cross_entropy_nll_kernel", K_XENT_NLL},
      {"__cross_entropy_bwd_kernel", K_XENT_BWD}, {"__embedding_kernel", K_EMBED},
      {"__embedding_bwd_kernel", K_EMBED_BWD}, {"__transpose_2d_kernel", K_TRANSPOSE_2D},
      {"__permute_3d_kernel", K_PERMUTE_3D}, {"__permute_nd_kernel", K_PERMUTE_ND},
      {"__scale_kernel", K_SCALE}, {"__fill_like_kernel", K_FILL_LIKE}, {"__eq_kernel", K_EQ},
      {"__sigmoid_bwd_kernel", K_SIGMOID_BWD}, {"__relu_bwd_kernel", K_RELU_BWD},
      {"__tanh_bwd_kernel", K_TANH_BWD}, {"__sqrt_bwd_kernel", K_SQRT_BWD},
      {"__abs_bwd_kernel", K_ABS_BWD}, {"__rsqrt_eps_kernel", K_RSQRT_EPS},
  };
  return m;
}

std::mutex g_reg_mu;
std::unordered_map<uint64_t, int> g_registry;
std::unordered_map<uint64_t, JitKernel*> g_jit;   // ids bound to compiled user kernels

JitKernel* jit_of(uint64_t id) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_jit.find(id);
  return it == g_jit.end() ? nullptr : it->second;
}

int lookup(uint64_t id) {
  std::lock_guard<std::mutex> lk(g_reg_mu);
  auto it = g_registry.find(id);
  if (it == g_registry.end()) panic("kernel_dispatch: kernel_id %llu not registered", (unsigned long long)id);
  return it->second;
}

int32_t ui(const void* u, size_t bytes, int k) {
  if ((size_t)(k + 1) * 4 > bytes) panic("kernel_dispatch_v2: uniform %d missing", k);
  int32_t v;
  memcpy(&v, (const char*)u + 4 * k, 4);
  return v;
}
float uf(const void* u, size_t bytes, int k) {
  if ((size_t)(k + 1) * 4 > bytes) panic("kernel_dispatch_v2: uniform %d missing", k);
  float v;
  memcpy(&v, (const char*)u + 4 * k, 4);
  return v;
}

// Kernels that read an (outer, axis, inner) decomposition from uniforms and
// one group per grid.x entry: outer = groups / inner.
void groups_of(const size_t* grid, int32_t axis, int32_t inner, size_t* outer) {
  size_t g = grid[0] * grid[1] * grid[2];
  *outer = inner > 0 ? g / (size_t)inner : 0;
  (void)axis;
}

}  // namespace

extern "C" {

void malus_runtime_init(const uint64_t* ids, const char* const* nm, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    if (looks_like_msl(nm[i])) {           // a kernel body: translate + NVRTC
      JitKernel* k = jit_compile(nm[i]);
      std::lock_guard<std::mutex> lk(g_reg_mu);
      g_jit[ids[i]] = k;
      g_registry.erase(ids[i]);
      continue;
    }
    std::lock_guard<std::mutex> lk(g_reg_mu);
    auto it = names().find(nm[i]);
    if (it == names().end()) panic("runtime_init: no native kernel named '%s'", nm[i]);
    g_registry[ids[i]] = it->second;
    g_jit.erase(ids[i]);
  }
}

int64_t kernel_dispatch(uint64_t kernel_id, const int64_t* h, size_t count) {
  if (count == 0) panic("kernel_dispatch: no inputs");
  if (JitKernel* jk = jit_of(kernel_id)) {
    plane_cache_clear();   // a user kernel may write any buffer it is given
    int64_t o = alloc_like(h[0]);
    jit_dispatch_implicit(jk, h, count, o);
    return o;
  }
  int k = lookup(kernel_id);
  int64_t out = alloc_like(h[0]);
  size_t n = tb(h[0])->len;
  auto need = [&](size_t c) { if (count < c) panic("kernel_dispatch: kernel needs %zu inputs", c); };
  switch (k) {
    case K_ADD: case K_SUB: case K_MUL: case K_DIV:
      need(2);
      if (tb(h[1])->len != n) panic("kernel_dispatch: elementwise builtin needs equal lengths");
      binary_same(k - K_ADD, fptr(h[0]), fptr(h[1]), fptr(out), n);
      break;
    case K_ADD_S: need(2); scalar_op_dev(kSAdd, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_SUB_S: need(2); scalar_op_dev(kSSub, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_RSUB_S: need(2); scalar_op_dev(kSRSub, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_MUL_S: need(2); scalar_op_dev(kSMul, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_DIV_S: need(2); scalar_op_dev(kSDiv, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_RDIV_S: need(2); scalar_op_dev(kSRDiv, fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    case K_RELU: unary_op(kRelu, fptr(h[0]), fptr(out), n); break;
    case K_SIGMOID: unary_op(kSigmoid, fptr(h[0]), fptr(out), n); break;
    case K_TANH: unary_op(kTanh, fptr(h[0]), fptr(out), n); break;
    case K_EXP: unary_op(kExp, fptr(h[0]), fptr(out), n); break;
    case K_LOG: unary_op(kLog, fptr(h[0]), fptr(out), n); break;
    case K_SQRT: unary_op(kSqrt, fptr(h[0]), fptr(out), n); break;
    case K_ABS: unary_op(kAbs, fptr(h[0]), fptr(out), n); break;
    case K_USER_SIGMOID_BWD: need(2); sigmoid_backward_user(fptr(h[0]), fptr(h[1]), fptr(out), n); break;
    default:
      panic("kernel_dispatch: kernel %llu is an explicit kernel; use kernel_dispatch_v2",
            (unsigned long long)kernel_id);
  }
  return out;
}

int64_t kernel_dispatch_v2(uint64_t kernel_id, const int64_t* h, size_t hc, const size_t* grid,
                           const size_t* tg, const size_t* out_shape, size_t out_ndim,
                           int32_t out_dtype, const void* u, size_t ub) {
  if (!grid || !tg) panic("kernel_dispatch_v2 grid/tg must not be null");
  JitKernel* jk = jit_of(kernel_id);
  int k = jk ? -1 : lookup(kernel_id);
  int64_t out;
  if (out_ndim == 0) {
    if (hc == 0) panic("kernel_dispatch_v2: out_ndim==0 but no tensor inputs");
    auto* f = tb(h[0]);
    out = alloc(out_dtype >= 0 ? out_dtype : f->dtype, f->shape, f->ndim);
  } else {
    out = alloc(out_dtype, out_shape, (int)out_ndim);
  }
  if (jk) {
    plane_cache_clear();   // a user kernel may write any buffer it is given
    jit_dispatch_explicit(jk, h, hc, grid, tg, out, u, ub);
    return out;
  }
  size_t on = tb(out)->len;
  if (on == 0) return out;
  float* o = fptr(out);
  auto need = [&](size_t c) { if (hc < c) panic("kernel_dispatch_v2: kernel needs %zu inputs", c); };
  switch (k) {
    case K_BC_ADD: case K_BC_SUB: case K_BC_MUL: case K_BC_DIV:
      need(2);
      binary_project_into_a(k - K_BC_ADD, h[0], h[1], o);
      break;
    case K_SOFTMAX: case K_LAYERNORM: case K_LAYERNORM_VAR: {
      need(1);
      int32_t axis = ui(u, ub, 0), inner = ui(u, ub, 1);
      size_t outer;
      groups_of(grid, axis, inner, &outer);
      if (k == K_SOFTMAX) softmax_fwd(fptr(h[0]), o, outer, (size_t)axis, (size_t)inner);
      else {
        float eps = uf(u, ub, 2);
        float* var = (float*)scratch_alloc(outer * inner * 4 + 4);
        if (k == K_LAYERNORM) {
          layernorm_fwd(fptr(h[0]), o, var, outer, (size_t)axis, (size_t)inner, eps);
        } else {
          float* y = (float*)scratch_alloc(on * 4);
          layernorm_fwd(fptr(h[0]), y, var, outer, (size_t)axis, (size_t)inner, eps);
          // layernorm.ml:40-58: the variance broadcast back over the axis
          expand_axis(var, o, outer, (size_t)axis, (size_t)inner);
          scratch_free(y);
        }
        scratch_free(var);
      }
      break;
    }
    case K_RED_SUM: case K_RED_MEAN: case K_RED_MAX: case K_RED_VAR: {
      need(1);
      int32_t axis = ui(u, ub, 0), inner = ui(u, ub, 1);
      size_t outer;
      groups_of(grid, axis, inner, &outer);
      reduce_axis(k - K_RED_SUM, fptr(h[0]), o, outer, (size_t)axis, (size_t)inner);
      break;
    }
    case K_EXPAND_AXIS: {
      need(1);
      int32_t axis = ui(u, ub, 0), inner = ui(u, ub, 1);
      size_t outer = on / ((size_t)axis * (size_t)inner);
      expand_axis(fptr(h[0]), o, outer, (size_t)axis, (size_t)inner);
      break;
    }
    case K_GELU: need(1); unary_op(kGelu, fptr(h[0]), o, on); break;
    case K_GELU_BWD: need(2); unary_bwd(kGeluBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_XENT_NLL: {
      // out[i] = -log(probs[i*vocab + t_i])  (cross_entropy.ml:13-16)
      need(2);
      int32_t vocab = ui(u, ub, 0);
      xent_nll_gather(fptr(h[0]), vptr(h[1]), tb(h[1])->dtype, o, on, (size_t)vocab);
      break;
    }
    case K_XENT_BWD: {
      // (p - onehot) * scale with the host-computed scale uniform
      // (transformer_bwd.ml:56-75)
      need(2);
      int32_t vocab = ui(u, ub, 0);
      float scale = uf(u, ub, 1);
      xent_bwd_scaled(fptr(h[0]), vptr(h[1]), tb(h[1])->dtype, scale, o, on / (size_t)vocab, (size_t)vocab);
      break;
    }
    case K_EMBED: {
      need(2);
      int32_t dim = ui(u, ub, 0);
      size_t n = on / (size_t)dim;
      embedding_fwd(fptr(h[0]), vptr(h[1]), tb(h[1])->dtype, o, n, tb(h[0])->len / (size_t)dim,
                    (size_t)dim);
      break;
    }
    case K_EMBED_BWD: {
      need(2);
      int32_t seq = ui(u, ub, 0), dim = ui(u, ub, 1);
      size_t V = on / (size_t)dim;
      embedding_bwd(fptr(h[0]), vptr(h[1]), tb(h[1])->dtype, o, (size_t)seq, V, (size_t)dim);
      break;
    }
    case K_TRANSPOSE_2D: {
      need(1);
      Shape s = shape_of(h[0]);
      int p[2] = {1, 0};
      permute_nd(fptr(h[0]), o, s, p);
      break;
    }
    case K_PERMUTE_3D: case K_PERMUTE_ND: {
      need(1);
      Shape s = shape_of(h[0]);
      int p[kMaxRank];
      for (int d = 0; d < s.ndim; ++d) p[d] = ui(u, ub, d);
      permute_nd(fptr(h[0]), o, s, p);
      break;
    }
    case K_SCALE: need(1); scalar_op_imm(kSMul, fptr(h[0]), uf(u, ub, 0), o, on); break;
    case K_FILL_LIKE: scalar_op_imm(kSFill, nullptr, uf(u, ub, 0), o, on); break;
    case K_EQ: need(2); unary_bwd(kEq, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_SIGMOID_BWD: need(2); unary_bwd(kSigmoidBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_RELU_BWD: need(2); unary_bwd(kReluBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_TANH_BWD: need(2); unary_bwd(kTanhBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_SQRT_BWD: need(2); unary_bwd(kSqrtBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_ABS_BWD: need(2); unary_bwd(kAbsBwd, fptr(h[0]), fptr(h[1]), o, on); break;
    case K_RSQRT_EPS: need(1); unary_op(kRsqrtEps, fptr(h[0]), o, on, uf(u, ub, 0)); break;
    default:
      // builtins may also come through v2 with out_ndim == 0
      tensor_release(out);
      return kernel_dispatch(kernel_id, h, hc);
  }
  return out;
}

}  // extern "C"
