// Define-by-run autograd tape with the semantics of
// crates/malus-runtime/src/tape.rs: thread-local node list, leaf registry,
// persistent accumulate-until-zero_grad leaf gradients, a 30-entry BwdSlot
// table of VJP function pointers, and the same retain/release rules.
//
// Two additions that change no observable value: before the reverse walk the
// tape marks which handles can reach a registered leaf, and skips VJPs whose
// result could only flow into gradients that are dropped at the end of
// backward() (the reference computes and then releases them, tape.rs:714-717);
// and the gradient of a registered leaf that only a multiply or an add reads
// (the attention scale and mask leaves of nanogpt_modular.ml:52-56) is
// deferred to the end of backward(), where it is evaluated, with the same
// VJP and arguments, only if the leaf outlives the tape (a leaf released
// with the tape has its gradient dropped unevaluated, as the reference drops
// the one it computed).
#include "common.cuh"

#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace malus {

enum OpTag : int32_t {
  kMatmul = 0, kTAdd = 1, kTSub = 2, kTMul = 3, kTDiv = 4, kTSigmoid = 5, kTRelu = 6, kTTanh = 7,
  kTExp = 8, kTLog = 9, kTSqrt = 10, kTAbs = 11, kTSum = 12, kTranspose = 13, kTNeg = 14,
  kRedSum = 15, kRedMean = 16, kRedMax = 17, kRedVar = 18, kReshape = 19, kSoftmax = 20,
  kLayernorm = 21, kGeluTag = 22, kCrossEntropy = 23, kEmbedding = 24,
};

enum BwdSlot : int32_t {
  sAddA = 0, sAddB, sSubA, sSubB, sMulA, sMulB, sDivA, sDivB, sSigmoid, sRelu, sTanh, sExp, sLog,
  sSqrt, sAbs, sNeg, sSum, sPermuteNd, sRedSum, sRedMean, sRedMax, sRedVar, sSoftmax, sLayernorm,
  sGelu, sXent, sEmbedding, sMatmulA, sMatmulB, sGradAcc, kNumSlots
};

namespace {

struct Node {
  int32_t op;
  std::vector<int64_t> saved;
  int64_t output;
  std::vector<int64_t> meta;
};

// A leaf gradient not yet evaluated: VJP slot `slot` applied to (dout, a, b),
// all three retained.
struct Thunk {
  int slot;
  int64_t dout, a, b;
};

struct TapeState {
  bool recording = true;
  std::unordered_map<int64_t, Thunk> pending;   // leaf -> deferred gradient (during backward)
  std::vector<Node> nodes;
  std::unordered_set<int64_t> leaves;
  std::unordered_map<int64_t, int64_t> leaf_grad;
  size_t slots[kNumSlots] = {0};
  bool slots_init = false;
};
thread_local TapeState t_tape;

void init_slots() {
  auto& s = t_tape.slots;
  s[sAddA] = (size_t)&__add_bwd_a;
  s[sAddB] = (size_t)&__add_bwd_b;
  s[sSubA] = (size_t)&__sub_bwd_a;
  s[sSubB] = (size_t)&__sub_bwd_b;
  s[sMulA] = (size_t)&__mul_bwd_a;
  s[sMulB] = (size_t)&__mul_bwd_b;
  s[sDivA] = (size_t)&__div_bwd_a;
  s[sDivB] = (size_t)&__div_bwd_b;
  s[sSigmoid] = (size_t)&__sigmoid_bwd;
  s[sRelu] = (size_t)&__relu_bwd;
  s[sTanh] = (size_t)&__tanh_bwd;
  s[sExp] = (size_t)&__broadcast_mul_fwd;   // dx = dout * e
  s[sLog] = (size_t)&__broadcast_div_fwd;   // dx = dout / x
  s[sSqrt] = (size_t)&__sqrt_bwd;
  s[sAbs] = (size_t)&__abs_bwd;
  s[sNeg] = (size_t)&__scale_fwd;           // dx = dout * -1
  s[sSum] = (size_t)&__sum_bwd;
  s[sPermuteNd] = (size_t)&__permute_nd_fwd;
  s[sRedSum] = (size_t)&__reduce_sum_axis_bwd;
  s[sRedMean] = (size_t)&__reduce_mean_axis_bwd;
  s[sRedMax] = (size_t)&__reduce_max_axis_bwd;
  s[sRedVar] = (size_t)&__reduce_var_axis_bwd;
  s[sSoftmax] = (size_t)&__softmax_bwd;
  s[sLayernorm] = (size_t)&__layernorm_bwd;
  s[sGelu] = (size_t)&__gelu_bwd;
  s[sXent] = (size_t)&__cross_entropy_bwd;
  s[sEmbedding] = (size_t)&__embedding_bwd;
  s[sMatmulA] = (size_t)&__matmul_bwd_a;
  s[sMatmulB] = (size_t)&__matmul_bwd_b;
  s[sGradAcc] = (size_t)&__broadcast_add_fwd;
  t_tape.slots_init = true;
}

size_t slot(int s) {
  if (!t_tape.slots_init) init_slots();
  size_t p = t_tape.slots[s];
  if (!p) panic("backward kernel slot %d not registered", s);
  return p;
}

typedef int64_t (*F2)(int64_t, int64_t);
typedef int64_t (*F3)(int64_t, int64_t, int64_t);
typedef int64_t (*F4)(int64_t, int64_t, int64_t, int64_t);
typedef int64_t (*FScale)(int64_t, float);
typedef int64_t (*FPerm)(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t);

void check_op(int32_t tag) {
  if (tag < 0 || tag > kEmbedding) panic("unknown op tag %d", tag);
}

int64_t grad_acc(int64_t old, int64_t nw) { return ((F2)slot(sGradAcc))(old, nw); }

int64_t run_thunk(const Thunk& k) {
  if (k.slot == sMulB || k.slot == sDivB) return ((F3)slot(k.slot))(k.dout, k.a, k.b);
  return ((F2)slot(k.slot))(k.dout, k.b);   // sAddB, sSubB
}

void drop_thunk(const Thunk& k) {
  tensor_release(k.dout);
  tensor_release(k.a);
  tensor_release(k.b);
}

void accumulate(std::unordered_map<int64_t, int64_t>& grads, int64_t input, int64_t g) {
  auto it = grads.find(input);
  if (it == grads.end()) {
    grads.emplace(input, g);
    return;
  }
  int64_t old = it->second;
  int64_t summed = grad_acc(old, g);
  tensor_release(old);
  tensor_release(g);
  it->second = summed;
}

}  // namespace

void tape_on_release(int64_t h) {
  // tape.rs:781-789: the leaf registry never outlives its tensor
  auto& T = t_tape;
  int64_t g = 0;
  auto it = T.leaf_grad.find(h);
  if (it != T.leaf_grad.end()) {
    g = it->second;
    T.leaf_grad.erase(it);
  }
  T.leaves.erase(h);
  if (g) tensor_release(g);
}

}  // namespace malus

using namespace malus;

extern "C" {

void tape_register_backward_fn(int32_t s, size_t fnptr) {
  if (s < 0 || s >= kNumSlots) panic("backward slot %d out of range", s);
  if (!t_tape.slots_init) init_slots();
  t_tape.slots[s] = fnptr;
}

void tape_record_binop(int32_t op, int64_t a, int64_t b, int64_t out) {
  if (!t_tape.recording) return;
  check_op(op);
  tensor_retain(a);
  tensor_retain(b);
  tensor_retain(out);
  t_tape.nodes.push_back(Node{op, {a, b}, out, {}});
}

void tape_record_unary(int32_t op, int64_t x, int64_t out) {
  if (!t_tape.recording) return;
  check_op(op);
  tensor_retain(x);
  tensor_retain(out);
  t_tape.nodes.push_back(Node{op, {x}, out, {}});
}

void tape_record_reduce(int32_t op, int64_t x, int64_t out, int64_t axis, int64_t keepdim) {
  if (!t_tape.recording) return;
  check_op(op);
  tensor_retain(x);
  tensor_retain(out);
  t_tape.nodes.push_back(Node{op, {x}, out, {axis, keepdim}});
}

void tape_record_perm(int32_t op, int64_t x, int64_t out, const size_t* dims, size_t ndims) {
  if (!t_tape.recording) return;
  check_op(op);
  tensor_retain(x);
  tensor_retain(out);
  std::vector<int64_t> meta;
  if (dims)
    for (size_t i = 0; i < ndims; ++i) meta.push_back((int64_t)dims[i]);
  t_tape.nodes.push_back(Node{op, {x}, out, meta});
}

void tape_record_layernorm(int32_t op, int64_t x, int64_t out, int64_t var_h, int64_t axis) {
  if (!t_tape.recording) {
    tensor_release(var_h);
    return;
  }
  check_op(op);
  tensor_retain(x);
  tensor_retain(out);
  t_tape.nodes.push_back(Node{op, {x, var_h}, out, {axis}});
}

void tape_record_cross_entropy(int32_t op, int64_t logits, int64_t out, int64_t softmax_h,
                               int64_t targets) {
  if (!t_tape.recording) {
    tensor_release(softmax_h);
    return;
  }
  check_op(op);
  tensor_retain(logits);
  tensor_retain(out);
  tensor_retain(targets);
  t_tape.nodes.push_back(Node{op, {logits, softmax_h, targets}, out, {}});
}

void tape_record_embedding(int32_t op, int64_t w, int64_t idx, int64_t out) {
  if (!t_tape.recording) return;
  check_op(op);
  tensor_retain(w);
  tensor_retain(idx);
  tensor_retain(out);
  t_tape.nodes.push_back(Node{op, {w, idx}, out, {}});
}

void tape_register_leaf(int64_t h) { t_tape.leaves.insert(h); }
void tape_pause(void) { t_tape.recording = false; }
void tape_resume(void) { t_tape.recording = true; }

void tape_clear(void) {
  auto nodes = std::move(t_tape.nodes);
  t_tape.nodes.clear();
  for (auto& n : nodes) {
    for (int64_t h : n.saved) tensor_release(h);
    tensor_release(n.output);
  }
}

int64_t tape_get_grad(int64_t h) {
  auto it = t_tape.leaf_grad.find(h);
  if (it != t_tape.leaf_grad.end()) {
    tensor_retain(it->second);
    return it->second;
  }
  auto* t = tb(h);
  return tensor_alloc_zeros_gpu(t->shape, t->ndim);
}

void backward(int64_t loss) {
  auto& T = t_tape;
  std::vector<Node> nodes = T.nodes;  // snapshot (handles only)

  // Which handles can reach a leaf: leaves, and outputs of nodes with such an input.
  std::unordered_set<int64_t> live(T.leaves.begin(), T.leaves.end());
  for (auto& n : nodes) {
    bool any = false;
    size_t nin = n.saved.size();
    if (n.op == kLayernorm) nin = 1;        // var_h is not a differentiable input
    if (n.op == kCrossEntropy) nin = 1;     // probs, targets are not
    if (n.op == kEmbedding) nin = 1;        // indices are not
    for (size_t i = 0; i < nin; ++i) any |= live.count(n.saved[i]) > 0;
    if (any) live.insert(n.output);
  }
  auto need = [&](int64_t h) { return live.count(h) > 0; };

  // Data parallelism (malus_dp_register_leaves): a registered leaf's gradient
  // is final once the earliest node (in forward order) that reads it has been
  // processed by this reverse walk; it is reported then, so its bucket's
  // all-reduce overlaps the rest of the backward pass.
  const bool dp = dp_leaves_registered();
  std::unordered_map<size_t, std::vector<int64_t>> final_after;
  if (dp) {
    std::unordered_set<int64_t> seen;
    for (size_t i = 0; i < nodes.size(); ++i) {
      const Node& n = nodes[i];
      size_t nin = n.saved.size();
      if (n.op == kLayernorm || n.op == kCrossEntropy || n.op == kEmbedding) nin = 1;
      for (size_t k = 0; k < nin; ++k)
        if (dp_is_leaf(n.saved[k]) && seen.insert(n.saved[k]).second) final_after[i].push_back(n.saved[k]);
    }
  }

  std::unordered_map<int64_t, int64_t> grads;
  {
    auto* t = tb(loss);
    grads.emplace(loss, tensor_alloc_ones_gpu(t->shape, t->ndim));
  }

  // A leaf read by exactly one node (and in no data-parallel bucket) gets its
  // gradient as a thunk, which holds the leaf; after the tape is cleared the
  // thunk is evaluated only if something besides it still holds the leaf.
  std::unordered_map<int64_t, int> reads;
  for (auto& n : nodes) {
    size_t nin = n.saved.size();
    if (n.op == kLayernorm || n.op == kCrossEntropy || n.op == kEmbedding) nin = 1;
    for (size_t i = 0; i < nin; ++i)
      if (T.leaves.count(n.saved[i])) reads[n.saved[i]]++;
  }
  auto defer = [&](int64_t leaf, int slot_id, int64_t dout, int64_t a) -> bool {
    if (!T.leaves.count(leaf) || reads[leaf] != 1 || (dp && dp_is_leaf(leaf)) || grads.count(leaf) ||
        T.pending.count(leaf))
      return false;
    tensor_retain(dout);
    tensor_retain(a);
    tensor_retain(leaf);
    T.pending.emplace(leaf, Thunk{slot_id, dout, a, leaf});
    return true;
  };

  for (auto it = nodes.rbegin(); it != nodes.rend(); ++it) {
    const Node& n = *it;
    if (dp) {
      // leaves whose earliest reader is the node after this one are final now
      const size_t after = nodes.size() - (size_t)(it - nodes.rbegin());
      auto fa = final_after.find(after);
      if (fa != final_after.end())
        for (int64_t leaf : fa->second) {
          auto g = grads.find(leaf);
          if (dp_leaf_ready(leaf, g == grads.end() ? 0 : g->second) != 0)
            panic("data-parallel gradient all-reduce failed (peer lost or timed out)");
        }
    }
    auto gi = grads.find(n.output);
    if (gi == grads.end()) continue;
    int64_t dout = gi->second;
    switch (n.op) {
      case kMatmul: {
        int64_t a = n.saved[0], b = n.saved[1];
        if (need(a)) accumulate(grads, a, ((F3)slot(sMatmulA))(a, b, dout));
        if (need(b)) accumulate(grads, b, ((F3)slot(sMatmulB))(a, b, dout));
        break;
      }
      case kTAdd: case kTSub: {
        int64_t a = n.saved[0], b = n.saved[1];
        int sa = n.op == kTAdd ? sAddA : sSubA, sb = n.op == kTAdd ? sAddB : sSubB;
        if (need(a)) accumulate(grads, a, ((F2)slot(sa))(dout, a));
        if (need(b) && !defer(b, sb, dout, a)) accumulate(grads, b, ((F2)slot(sb))(dout, b));
        break;
      }
      case kTMul: case kTDiv: {
        int64_t a = n.saved[0], b = n.saved[1];
        int sa = n.op == kTMul ? sMulA : sDivA, sb = n.op == kTMul ? sMulB : sDivB;
        if (need(a)) accumulate(grads, a, ((F3)slot(sa))(dout, a, b));
        if (need(b) && !defer(b, sb, dout, a)) accumulate(grads, b, ((F3)slot(sb))(dout, a, b));
        break;
      }
      case kTSigmoid: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sSigmoid))(n.output, dout)); break;
      case kTRelu: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sRelu))(n.saved[0], dout)); break;
      case kTTanh: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sTanh))(n.output, dout)); break;
      case kTExp: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sExp))(dout, n.output)); break;
      case kTLog: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sLog))(dout, n.saved[0])); break;
      case kTSqrt: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sSqrt))(n.output, dout)); break;
      case kTAbs: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sAbs))(n.saved[0], dout)); break;
      case kTSum: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sSum))(n.saved[0], dout)); break;
      case kTNeg: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((FScale)slot(sNeg))(dout, -1.0f)); break;
      case kTranspose: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        int rank = tb(x)->ndim;
        std::vector<size_t> raw(n.meta.begin(), n.meta.end());
        // normalise like tensor_permute, then invert (tape.rs:573-587)
        std::vector<int> perm;
        if (raw.empty()) perm = {1, 0};
        else if (raw.size() == 2) {
          for (int k = 0; k < rank; ++k) perm.push_back(k);
          std::swap(perm[raw[0]], perm[raw[1]]);
        } else for (size_t v : raw) perm.push_back((int)v);
        int64_t inv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i < rank; ++i) inv[perm[i]] = i;
        accumulate(grads, x, ((FPerm)slot(sPermuteNd))(dout, inv[0], inv[1], inv[2], inv[3], inv[4],
                                                        inv[5], inv[6], inv[7]));
        break;
      }
      case kReshape: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        auto* t = tb(x);
        accumulate(grads, x, tensor_reshape(dout, t->shape, t->ndim));
        break;
      }
      case kRedSum: case kRedMean: case kRedVar: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        int s = n.op == kRedSum ? sRedSum : (n.op == kRedMean ? sRedMean : sRedVar);
        accumulate(grads, x, ((F3)slot(s))(x, dout, n.meta[0]));
        break;
      }
      case kRedMax: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        accumulate(grads, x, ((F4)slot(sRedMax))(x, n.output, dout, n.meta[0]));
        break;
      }
      case kSoftmax: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        int64_t axis = n.meta.empty() ? -1 : n.meta[0];
        accumulate(grads, x, ((F3)slot(sSoftmax))(n.output, dout, axis));
        break;
      }
      case kLayernorm: {
        int64_t x = n.saved[0];
        if (!need(x)) break;
        accumulate(grads, x, ((F4)slot(sLayernorm))(n.output, n.saved[1], dout, n.meta[0]));
        break;
      }
      case kGeluTag: if (need(n.saved[0])) accumulate(grads, n.saved[0], ((F2)slot(sGelu))(n.saved[0], dout)); break;
      case kCrossEntropy: {
        int64_t logits = n.saved[0];
        if (!need(logits)) break;
        accumulate(grads, logits, ((F3)slot(sXent))(n.saved[1], n.saved[2], dout));
        break;
      }
      case kEmbedding: {
        int64_t w = n.saved[0];
        if (!need(w)) break;
        accumulate(grads, w, ((F3)slot(sEmbedding))(w, n.saved[1], dout));
        break;
      }
      default: panic("backward: unhandled op tag %d", n.op);
    }
  }

  if (dp) {
    auto fa = final_after.find(0);   // leaves first read by node 0
    if (fa != final_after.end())
      for (int64_t leaf : fa->second) {
        auto g = grads.find(leaf);
        if (dp_leaf_ready(leaf, g == grads.end() ? 0 : g->second) != 0)
          panic("data-parallel gradient all-reduce failed (peer lost or timed out)");
      }
    if (dp_leaves_join() != 0) panic("data-parallel gradient all-reduce failed (peer lost or timed out)");
  }

  // Fold leaf grads into the persistent registry (accumulate semantics).
  std::vector<int64_t> to_release;
  for (int64_t leaf : T.leaves) {
    auto gi = grads.find(leaf);
    if (gi == grads.end()) continue;
    int64_t ng = gi->second;
    grads.erase(gi);
    // a leaf's gradient is kept as plain data: a deferred product would hold
    // its operands (possibly other leaves) alive as long as the gradient
    if (tb(ng)->lazy) materialize(ng);
    auto li = T.leaf_grad.find(leaf);
    if (li == T.leaf_grad.end()) {
      T.leaf_grad.emplace(leaf, ng);
    } else {
      int64_t old = li->second;
      li->second = grad_acc(old, ng);
      to_release.push_back(old);
      to_release.push_back(ng);
    }
  }
  for (int64_t h : to_release) tensor_release(h);
  for (auto& kv : grads) tensor_release(kv.second);
  // The thunks hold their leaves, so every pending leaf is alive here.  The
  // tape's references go first; a leaf then held by its thunk alone needs no
  // gradient (dropping the thunk releases it and its registry entry).  A
  // thunk's arguments can hold another pending leaf (the mask's thunk holds
  // the deferred scores, which hold the scale leaf), so thunks are dropped
  // until none is left whose leaf nothing else holds, and only then are the
  // remaining ones evaluated.
  tape_clear();
  std::vector<std::pair<int64_t, Thunk>> due(T.pending.begin(), T.pending.end());
  T.pending.clear();
  for (bool dropped = true; dropped;) {
    dropped = false;
    for (size_t i = 0; i < due.size();) {
      if (tb(due[i].first)->rc.load() == 1) {
        Thunk k = due[i].second;
        due.erase(due.begin() + (ptrdiff_t)i);
        drop_thunk(k);   // releases the leaf (and with it its registry entry)
        dropped = true;
      } else {
        ++i;
      }
    }
  }
  for (auto& kv : due) {
    const int64_t leaf = kv.first;
    const Thunk& k = kv.second;
    {   // held by someone besides the thunks: evaluate now
      int64_t ng = run_thunk(k);
      auto li = T.leaf_grad.find(leaf);
      if (li == T.leaf_grad.end()) {
        T.leaf_grad.emplace(leaf, ng);
      } else {
        int64_t old = li->second;
        li->second = grad_acc(old, ng);
        tensor_release(old);
        tensor_release(ng);
      }
    }
    drop_thunk(k);
  }
  plane_cache_clear();   // a step boundary: parameters are about to change in place
}

void tape_zero_grad(const int64_t* handles, size_t count) {
  plane_cache_clear();   // a step boundary (the optimizer has written the parameters)
  if (!handles || !count) return;
  std::vector<int64_t> rel;
  for (size_t i = 0; i < count; ++i) {
    auto it = t_tape.leaf_grad.find(handles[i]);
    if (it != t_tape.leaf_grad.end()) {
      rel.push_back(it->second);
      t_tape.leaf_grad.erase(it);
    }
  }
  for (int64_t g : rel) tensor_release(g);
}

void malus_tape_reset(void) {
  t_tape.leaves.clear();
  std::vector<int64_t> rel;
  for (auto& kv : t_tape.leaf_grad) rel.push_back(kv.second);
  t_tape.leaf_grad.clear();
  for (int64_t g : rel) tensor_release(g);
  tape_clear();
  t_tape.recording = true;
}

void malus_tape_registry_lens(int64_t* leaves, int64_t* grads) {
  if (leaves) *leaves = (int64_t)t_tape.leaves.size();
  if (grads) *grads = (int64_t)t_tape.leaf_grad.size();
}

}  // extern "C"
