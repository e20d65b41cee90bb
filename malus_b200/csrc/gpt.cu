// The nanoGPT training step.
//
// Mode 0 ("tape") replays, call for call, what the Cranelift JIT emits for
// examples/nanogpt_modular.ml (forward :37-90, step loop :166-192) through
// this runtime's C ABI: stdlib host functions, tape_record_* after each
// grad-tracked op, backward(loss), and the AdamW update of :100-110 (fused
// into one launch with the identical f32 operation order).  Generalised to
// n_layer blocks, n_head heads and scale 1/sqrt(head_size); with tied=1 the
// LM head is transpose(wte).
//
// Mode 1 ("fused") is the B200-native compiled step: the same math with
// fused kernels, preallocated activations and transposed-operand GEMMs; see
// gpt_fused.cu.
//
// Parameters, first and second moments live in three fused device buffers
// (256-byte aligned slices wrapped as handles), so the optimizer is one
// launch and the data-parallel all-reduce can run on one buffer.
#include "common.cuh"

#include <cmath>
#include <vector>

namespace malus {
int dp_allreduce_async(float* ptr, size_t count);
void dp_join();
int dp_world();
struct FusedStep;
FusedStep* fused_create(const malus_gpt_config& cfg, const std::vector<float*>& params,
                        const std::vector<size_t>& sizes, float* gbuf,
                        const std::vector<size_t>& goff, float* pbuf, float* mbuf, float* vbuf,
                        size_t total_elems);
void fused_destroy(FusedStep* f);
void fused_train_step(FusedStep* f, const int32_t* x_dev, const int32_t* y_dev, float* loss_dev);
}  // namespace malus

using namespace malus;

namespace {

enum { T_MATMUL = 0, T_ADD = 1, T_MUL = 3, T_TRANSPOSE = 13, T_RESHAPE = 19, T_SOFTMAX = 20,
       T_LAYERNORM = 21, T_GELU = 22, T_XENT = 23, T_EMBED = 24 };

struct Model {
  malus_gpt_config cfg;
  int C, H, hs, T, B, V, L, C4;
  size_t M;
  std::vector<int64_t> params, ms, vs, gradv;   // gradv: views of the gradient buffer
  std::vector<size_t> offs;   // element offsets into the fused buffers
  std::vector<size_t> sizes;
  size_t total = 0;
  float *pbuf = nullptr, *mbuf = nullptr, *vbuf = nullptr, *gbuf = nullptr;
  int64_t x_h = 0, y_h = 0, pos_h = 0;
  int32_t *x_dev = nullptr, *y_dev = nullptr;
  int32_t *x_pin = nullptr, *y_pin = nullptr;
  float* loss_dev = nullptr;
  float* loss_pin = nullptr;
  int64_t step = 0;
  FusedStep* fused = nullptr;
  // tape mode: AdamW's step counter on the device and the bias-correction
  // table it indexes (so a captured step replays as a new step); the graph
  int64_t* step_dev = nullptr;
  float* bc_tab = nullptr;
  int64_t bc_cap = 0;
  int64_t graph = 0;
  bool dp_registered = false;
};

int64_t wrap(float* p, std::initializer_list<size_t> shape) {
  size_t s[kMaxRank];
  int n = 0;
  for (size_t d : shape) s[n++] = d;
  return malus_tensor_wrap(MALUS_F32, p, s, n);
}

int64_t rsh(int64_t h, std::initializer_list<size_t> shape) {
  size_t s[kMaxRank];
  int n = 0;
  for (size_t d : shape) s[n++] = d;
  return tensor_reshape(h, s, n);
}

// ---- tape-mode ops: the JIT's lowering of each builtin (codegen-cpu lib.rs) ----
int64_t op_binop(int tag, int64_t a, int64_t b) {
  int64_t out;
  switch (tag) {
    case T_ADD: out = __broadcast_add_fwd(a, b); break;
    case T_MUL: out = __broadcast_mul_fwd(a, b); break;
    default: out = tensor_matmul(a, b); break;
  }
  tape_record_binop(tag, a, b, out);
  return out;
}
int64_t op_layernorm(int64_t x) {
  int64_t box = __layernorm_fwd(x, 1);
  int64_t* f = reinterpret_cast<int64_t*>(box);
  int64_t y = f[1], var = f[2];
  free(f);  // aggregate_release of the 1-ref tuple box
  tape_record_layernorm(T_LAYERNORM, x, y, var, 1);
  return y;
}
int64_t op_reshape(int64_t x, std::initializer_list<size_t> shape) {
  int64_t out = rsh(x, shape);
  tape_record_unary(T_RESHAPE, x, out);
  return out;
}
int64_t op_permute(int64_t x, std::initializer_list<size_t> perm) {
  std::vector<size_t> p(perm);
  int64_t out = tensor_permute(x, p.data(), p.size());
  tape_record_perm(T_TRANSPOSE, x, out, p.data(), p.size());
  return out;
}

// forward of one Block (nanogpt_modular.ml:37-67); returns x3, releases nothing it doesn't own
int64_t block_forward(Model& m, int l, int64_t x) {
  const int64_t* P = &m.params[(size_t)l * 8];
  size_t B = m.B, T = m.T, H = m.H, hs = m.hs, C = m.C;
  int64_t y1 = op_layernorm(x);
  int64_t xn1 = op_binop(T_MUL, y1, P[0]);
  tensor_release(y1);
  int64_t qkv[3];
  for (int j = 0; j < 3; ++j) {
    int64_t q = op_binop(T_MATMUL, xn1, P[1 + j]);
    int64_t r1 = op_reshape(q, {B, T, H, hs});
    int64_t p1 = op_permute(r1, {0, 2, 1, 3});
    qkv[j] = op_reshape(p1, {B * H, T, hs});
    tensor_release(q);
    tensor_release(r1);
    tensor_release(p1);
  }
  tensor_release(xn1);
  int64_t Kt = op_permute(qkv[1], {0, 2, 1});
  // scale = variable(ones(1, 1) * (1/sqrt(hs)))
  size_t s11[2] = {1, 1};
  int64_t ones11 = tensor_alloc_ones_gpu(s11, 2);
  int64_t scale = alloc_f32({1, 1});
  scalar_op_imm(kSMul, fptr(ones11), 1.0f / sqrtf((float)hs), fptr(scale), 1);
  tensor_release(ones11);
  tape_register_leaf(scale);
  int64_t qk = op_binop(T_MATMUL, qkv[0], Kt);
  int64_t scores = op_binop(T_MUL, qk, scale);
  int64_t mask = tensor_causal_mask((int64_t)T);
  tape_register_leaf(mask);
  int64_t masked = op_binop(T_ADD, scores, mask);
  int64_t attn = __softmax_fwd(masked, 2);
  tape_record_reduce(T_SOFTMAX, masked, attn, 2, 0);
  int64_t av = op_binop(T_MATMUL, attn, qkv[2]);
  int64_t r2 = op_reshape(av, {B, H, T, hs});
  int64_t p2 = op_permute(r2, {0, 2, 1, 3});
  int64_t ao = op_reshape(p2, {B * T, C});
  int64_t proj = op_binop(T_MATMUL, ao, P[4]);
  int64_t x2 = op_binop(T_ADD, x, proj);
  for (int64_t h : {qkv[0], qkv[1], qkv[2], Kt, scale, qk, scores, mask, masked, attn, av, r2, p2,
                    ao, proj})
    tensor_release(h);
  int64_t y2 = op_layernorm(x2);
  int64_t xn2 = op_binop(T_MUL, y2, P[5]);
  int64_t hpre = op_binop(T_MATMUL, xn2, P[6]);
  int64_t hid = __gelu_fwd(hpre);
  tape_record_unary(T_GELU, hpre, hid);
  int64_t mlp = op_binop(T_MATMUL, hid, P[7]);
  int64_t x3 = op_binop(T_ADD, x2, mlp);
  for (int64_t h : {y2, xn2, hpre, hid, mlp, x2}) tensor_release(h);
  return x3;
}

void tape_step(Model& m) {
  size_t nparam = m.params.size();
  // Under data parallelism the parameters are the tape's registered leaves:
  // backward averages each bucket of their gradients across ranks as soon as
  // the walk has finished them (buckets of about one layer).
  if (dp_world() > 1 && !m.dp_registered) {
    if (malus_dp_register_leaves(m.params.data(), nparam, (size_t)4 << 20) <= 0)
      panic("data parallelism: registering the parameters failed");
    m.dp_registered = true;
  }
  tape_zero_grad(m.params.data(), nparam);
  const int64_t* top = &m.params[(size_t)m.L * 8];
  int64_t wte = top[0], wpe = top[1], lnf = top[2];
  int64_t te = __embedding_fwd(wte, m.x_h);
  tape_record_embedding(T_EMBED, wte, m.x_h, te);
  int64_t pe = __embedding_fwd(wpe, m.pos_h);
  tape_record_embedding(T_EMBED, wpe, m.pos_h, pe);
  int64_t x = op_binop(T_ADD, te, pe);
  tensor_release(te);
  tensor_release(pe);
  for (int l = 0; l < m.L; ++l) {
    int64_t nx = block_forward(m, l, x);
    tensor_release(x);
    x = nx;
  }
  int64_t yf = op_layernorm(x);
  int64_t xf = op_binop(T_MUL, yf, lnf);
  int64_t head;
  if (m.cfg.tied) {
    head = tensor_permute(wte, nullptr, 0);
    tape_record_perm(T_TRANSPOSE, wte, head, nullptr, 0);
  } else {
    head = top[3];
    tensor_retain(head);
  }
  int64_t logits = op_binop(T_MATMUL, xf, head);
  int64_t box = __cross_entropy_fwd(logits, m.y_h);
  int64_t* f = reinterpret_cast<int64_t*>(box);
  int64_t loss = f[1], probs = f[2];
  free(f);
  tape_record_cross_entropy(T_XENT, logits, loss, probs, m.y_h);
  for (int64_t h : {x, yf, xf, head, logits}) tensor_release(h);
  backward(loss);
  MALUS_CUDA(cudaMemcpyAsync(m.loss_dev, fptr(loss), 4, cudaMemcpyDeviceToDevice, stream()));
  tensor_release(loss);

  // gradients -> (DP all-reduce) -> fused AdamW
  std::vector<int64_t> grads(nparam);
  for (size_t i = 0; i < nparam; ++i) grads[i] = tape_get_grad(m.params[i]);
  // gather into the fused gradient buffer (readable with malus_gpt_grad; one
  // all-reduce over it under data parallelism)
  for (size_t i = 0; i < nparam; ++i) {
    MALUS_CUDA(cudaMemcpyAsync(m.gbuf + m.offs[i], fptr(grads[i]), m.sizes[i] * 4,
                               cudaMemcpyDeviceToDevice, stream()));
    tensor_release(grads[i]);
    grads[i] = wrap(m.gbuf + m.offs[i], {m.sizes[i]});
  }
  const float gscale = 1.0f;   // gradients are already averaged across ranks
  // the fused multi-tensor AdamW (malus_adamw_multi's kernel) with the bias
  // corrections read from the table at the device step counter
  std::vector<AdamSeg> segs(nparam);
  for (size_t i = 0; i < nparam; ++i)
    segs[i] = AdamSeg{fptr(m.params[i]), fptr(grads[i]), fptr(m.ms[i]), fptr(m.vs[i]), (int64_t)m.sizes[i]};
  step_advance(m.step_dev);
  adamw_multi_tab(segs.data(), (int)nparam, m.cfg.lr, m.cfg.beta1, m.cfg.beta2, m.cfg.eps, m.cfg.wd, 0.0f,
                  0.0f, gscale, m.bc_tab, m.step_dev);
  for (int64_t g : grads) tensor_release(g);
}

void tape_bc_table(Model& m, int64_t cap) {
  const std::vector<float> h = adam_bc_table(m.cfg.beta1, m.cfg.beta2, cap);
  if (m.bc_tab) {
    MALUS_CUDA(cudaStreamSynchronize(stream()));
    MALUS_CUDA(cudaFree(m.bc_tab));
  }
  MALUS_CUDA(cudaMalloc(&m.bc_tab, h.size() * sizeof(float)));
  MALUS_CUDA(cudaMemcpy(m.bc_tab, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
  m.bc_cap = cap;
}

// Under data parallelism, wait (bounded) for this step's collectives before a
// blocking host read: a lost peer aborts the communicator (its NCCL kernels
// end) and the process reports the failure instead of blocking forever.
void dp_drain_or_die() {
  if (dp_world() <= 1) return;
  int r = malus_dp_finish();
  if (r != 0) panic("data-parallel step failed: a peer was lost or timed out (%d)", r);
}

}  // namespace

namespace malus {

// Parameter layout of the fused buffers (nanogpt_modular.ml:112-125, 150-162):
// per block [ln1, wq, wk, wv, wo, ln2, w1, w2], then [wte, wpe, ln_f, (lm_head)],
// each slice 256-byte aligned.  Returns the buffer length in elements.
size_t gpt_layout(const malus_gpt_config& c, std::vector<std::vector<size_t>>& shapes,
                  std::vector<size_t>& offs, std::vector<size_t>& sizes) {
  const size_t C = c.n_embd, C4 = 4 * (size_t)c.n_embd, V = c.vocab, T = c.block_size;
  shapes.clear();
  offs.clear();
  sizes.clear();
  for (int l = 0; l < c.n_layer; ++l) {
    shapes.push_back({C});
    for (int j = 0; j < 4; ++j) shapes.push_back({C, C});
    shapes.push_back({C});
    shapes.push_back({C, C4});
    shapes.push_back({C4, C});
  }
  shapes.push_back({V, C});
  shapes.push_back({T, C});
  shapes.push_back({C});
  if (!c.tied) shapes.push_back({C, V});
  size_t off = 0;
  for (auto& s : shapes) {
    size_t n = 1;
    for (size_t d : s) n *= d;
    offs.push_back(off);
    sizes.push_back(n);
    off += (n + 63) & ~size_t(63);
  }
  return off;
}

// All-reduce buckets of the fused step in issue order: each layer's slice as soon
// as its backward is done (last layer first), then embeddings, final norm, head.
std::vector<std::pair<size_t, size_t>> gpt_dp_buckets(int n_layer, const std::vector<size_t>& offs,
                                                      const std::vector<size_t>& sizes) {
  std::vector<std::pair<size_t, size_t>> b;
  for (int l = n_layer - 1; l >= 0; --l) {
    size_t first = (size_t)l * 8, last = first + 7;
    b.push_back({offs[first], offs[last] + sizes[last]});
  }
  size_t top = (size_t)n_layer * 8;
  b.push_back({offs[top], offs.back() + sizes.back()});
  return b;
}

}  // namespace malus

extern "C" {

int32_t malus_gpt_layout(const malus_gpt_config* cfg, int64_t* offsets, int64_t* sizes, int32_t n,
                         int64_t* total) {
  std::vector<std::vector<size_t>> shapes;
  std::vector<size_t> o, z;
  size_t t = gpt_layout(*cfg, shapes, o, z);
  for (size_t i = 0; i < o.size() && (int32_t)i < n; ++i) {
    if (offsets) offsets[i] = (int64_t)o[i];
    if (sizes) sizes[i] = (int64_t)z[i];
  }
  if (total) *total = (int64_t)t;
  return (int32_t)o.size();
}

int32_t malus_gpt_dp_buckets(const malus_gpt_config* cfg, int64_t* lo, int64_t* hi, int32_t n) {
  std::vector<std::vector<size_t>> shapes;
  std::vector<size_t> o, z;
  gpt_layout(*cfg, shapes, o, z);
  auto b = gpt_dp_buckets(cfg->n_layer, o, z);
  for (size_t i = 0; i < b.size() && (int32_t)i < n; ++i) {
    if (lo) lo[i] = (int64_t)b[i].first;
    if (hi) hi[i] = (int64_t)b[i].second;
  }
  return (int32_t)b.size();
}

int64_t malus_gpt_create(const malus_gpt_config* cfgp) {
  auto* m = new Model();
  m->cfg = *cfgp;
  auto& c = m->cfg;
  m->C = c.n_embd; m->H = c.n_head; m->T = c.block_size; m->B = c.batch; m->V = c.vocab;
  m->L = c.n_layer; m->C4 = 4 * c.n_embd;
  if (m->C % m->H) panic("n_embd %d not divisible by n_head %d", m->C, m->H);
  m->hs = m->C / m->H;
  m->M = (size_t)m->B * m->T;
  std::vector<std::vector<size_t>> shapes;
  size_t off = gpt_layout(c, shapes, m->offs, m->sizes);
  m->total = off;
  MALUS_CUDA(cudaMalloc(&m->pbuf, off * 4));
  MALUS_CUDA(cudaMalloc(&m->mbuf, off * 4));
  MALUS_CUDA(cudaMalloc(&m->vbuf, off * 4));
  MALUS_CUDA(cudaMalloc(&m->gbuf, off * 4));
  MALUS_CUDA(cudaMemsetAsync(m->pbuf, 0, off * 4, stream()));
  MALUS_CUDA(cudaMemsetAsync(m->mbuf, 0, off * 4, stream()));
  MALUS_CUDA(cudaMemsetAsync(m->vbuf, 0, off * 4, stream()));
  MALUS_CUDA(cudaMemsetAsync(m->gbuf, 0, off * 4, stream()));
  for (size_t i = 0; i < shapes.size(); ++i) {
    size_t s[kMaxRank];
    for (size_t k = 0; k < shapes[i].size(); ++k) s[k] = shapes[i][k];
    m->params.push_back(malus_tensor_wrap(MALUS_F32, m->pbuf + m->offs[i], s, shapes[i].size()));
    m->ms.push_back(malus_tensor_wrap(MALUS_F32, m->mbuf + m->offs[i], s, shapes[i].size()));
    m->vs.push_back(malus_tensor_wrap(MALUS_F32, m->vbuf + m->offs[i], s, shapes[i].size()));
    m->gradv.push_back(malus_tensor_wrap(MALUS_F32, m->gbuf + m->offs[i], s, shapes[i].size()));
  }
  // initialisation in the reference's RNG call order: per block wq,wk,wv,wo,w1,w2,
  // then wte, wpe, (lm_head); LN gains are ones
  malus_rng_reset(c.seed);
  auto init_randn = [&](size_t i) {
    int64_t r = tensor_randn(tb(m->params[i])->shape, tb(m->params[i])->ndim);
    scalar_op_imm(kSMul, fptr(r), c.init_std, fptr(m->params[i]), m->sizes[i]);
    tensor_release(r);
  };
  auto init_ones = [&](size_t i) { scalar_op_imm(kSFill, nullptr, 1.0f, fptr(m->params[i]), m->sizes[i]); };
  for (int l = 0; l < m->L; ++l) {
    size_t b = (size_t)l * 8;
    init_ones(b + 0);
    for (int j = 1; j <= 4; ++j) init_randn(b + j);
    init_ones(b + 5);
    init_randn(b + 6);
    init_randn(b + 7);
  }
  size_t top = (size_t)m->L * 8;
  init_randn(top + 0);
  init_randn(top + 1);
  init_ones(top + 2);
  if (!c.tied) init_randn(top + 3);
  for (int64_t p : m->params) tape_register_leaf(p);
  // device token buffers, pinned staging, positions
  MALUS_CUDA(cudaMalloc(&m->x_dev, m->M * 4));
  MALUS_CUDA(cudaMalloc(&m->y_dev, m->M * 4));
  MALUS_CUDA(cudaMalloc(&m->loss_dev, 256));
  MALUS_CUDA(cudaMallocHost(&m->x_pin, m->M * 4));
  MALUS_CUDA(cudaMallocHost(&m->y_pin, m->M * 4));
  MALUS_CUDA(cudaMallocHost(&m->loss_pin, 256));
  size_t sm[1] = {m->M};
  m->x_h = malus_tensor_wrap(MALUS_I32, m->x_dev, sm, 1);
  m->y_h = malus_tensor_wrap(MALUS_I32, m->y_dev, sm, 1);
  std::vector<int32_t> pos(m->M);
  for (size_t i = 0; i < m->M; ++i) pos[i] = (int32_t)(i % m->T);
  m->pos_h = tensor_alloc_gpu(MALUS_I32, sm, 1, reinterpret_cast<const float*>(pos.data()));
  MALUS_CUDA(cudaMalloc(&m->step_dev, sizeof(int64_t)));
  MALUS_CUDA(cudaMemsetAsync(m->step_dev, 0, sizeof(int64_t), stream()));
  tape_bc_table(*m, 1 << 16);
  if (c.mode == 1) {
    std::vector<float*> ps;
    for (size_t i = 0; i < m->params.size(); ++i) ps.push_back(m->pbuf + m->offs[i]);
    m->fused = fused_create(c, ps, m->sizes, m->gbuf, m->offs, m->pbuf, m->mbuf, m->vbuf, m->total);
  }
  gpu_barrier();
  return reinterpret_cast<int64_t>(m);
}

void malus_gpt_destroy(int64_t h) {
  auto* m = reinterpret_cast<Model*>(h);
  gpu_barrier();
  if (m->graph) malus_graph_destroy(m->graph);
  cudaFree(m->step_dev);
  cudaFree(m->bc_tab);
  if (m->fused) fused_destroy(m->fused);
  for (int64_t p : m->params) tensor_release(p);
  for (int64_t p : m->ms) tensor_release(p);
  for (int64_t p : m->vs) tensor_release(p);
  for (int64_t p : m->gradv) tensor_release(p);
  tensor_release(m->x_h);
  tensor_release(m->y_h);
  tensor_release(m->pos_h);
  cudaFree(m->pbuf); cudaFree(m->mbuf); cudaFree(m->vbuf); cudaFree(m->gbuf);
  cudaFree(m->x_dev); cudaFree(m->y_dev); cudaFree(m->loss_dev);
  cudaFreeHost(m->x_pin); cudaFreeHost(m->y_pin); cudaFreeHost(m->loss_pin);
  delete m;
}

void malus_gpt_step_device(int64_t h, const int32_t* x_dev, const int32_t* y_dev) {
  auto* m = reinterpret_cast<Model*>(h);
  plane_cache_clear();   // the step rewrites its parameters in place
  if (x_dev != m->x_dev)
    MALUS_CUDA(cudaMemcpyAsync(m->x_dev, x_dev, m->M * 4, cudaMemcpyDeviceToDevice, stream()));
  if (y_dev != m->y_dev)
    MALUS_CUDA(cudaMemcpyAsync(m->y_dev, y_dev, m->M * 4, cudaMemcpyDeviceToDevice, stream()));
  if (m->cfg.mode == 1) {
    m->step++;
    fused_train_step(m->fused, m->x_dev, m->y_dev, m->loss_dev);
  } else {
    m->step++;
    if (m->step > m->bc_cap) {   // a new table (new address): the captured step is stale
      if (m->graph) malus_graph_destroy(m->graph);
      m->graph = 0;
      tape_bc_table(*m, m->bc_cap * 4);
    }
    // The reference's call sequence captured once (after one eager step sized
    // every workspace) as a CUDA graph through the runtime's graph API and
    // replayed: the caller side of the boundary, one launch per step.
    if (m->cfg.use_graph && !prof_on() && !sync_dispatch() && m->step > 1) {
      if (!m->graph) {
        malus_graph_begin();
        tape_step(*m);
        m->graph = malus_graph_end();
      }
      malus_graph_replay(m->graph);
    } else {
      tape_step(*m);
    }
  }
}

float malus_gpt_step(int64_t h, const int32_t* x, const int32_t* y) {
  auto* m = reinterpret_cast<Model*>(h);
  memcpy(m->x_pin, x, m->M * 4);
  memcpy(m->y_pin, y, m->M * 4);
  MALUS_CUDA(cudaMemcpyAsync(m->x_dev, m->x_pin, m->M * 4, cudaMemcpyHostToDevice, stream()));
  MALUS_CUDA(cudaMemcpyAsync(m->y_dev, m->y_pin, m->M * 4, cudaMemcpyHostToDevice, stream()));
  malus_gpt_step_device(h, m->x_dev, m->y_dev);
  MALUS_CUDA(cudaMemcpyAsync(m->loss_pin, m->loss_dev, 4, cudaMemcpyDeviceToHost, stream()));
  dp_drain_or_die();
  gpu_barrier();
  return m->loss_pin[0];
}

float malus_gpt_last_loss(int64_t h) {
  auto* m = reinterpret_cast<Model*>(h);
  float v;
  MALUS_CUDA(cudaMemcpyAsync(&v, m->loss_dev, 4, cudaMemcpyDeviceToHost, stream()));
  dp_drain_or_die();
  gpu_barrier();
  return v;
}

int32_t malus_gpt_num_params(int64_t h) { return (int32_t)reinterpret_cast<Model*>(h)->params.size(); }
int64_t malus_gpt_param(int64_t h, int32_t i) { return reinterpret_cast<Model*>(h)->params.at((size_t)i); }
int64_t malus_gpt_grad(int64_t h, int32_t i) { return reinterpret_cast<Model*>(h)->gradv.at((size_t)i); }
int64_t malus_gpt_moment(int64_t h, int32_t i, int32_t which) {
  auto* m = reinterpret_cast<Model*>(h);
  return (which ? m->vs : m->ms).at((size_t)i);
}
int64_t malus_gpt_num_elements(int64_t h) {
  auto* m = reinterpret_cast<Model*>(h);
  int64_t n = 0;
  for (size_t s : m->sizes) n += (int64_t)s;
  return n;
}

}  // extern "C"
