/*
 * malus_runtime.h — C ABI of libmalus_runtime_cuda.so, the sm_100a (B200)
 * runtime behind malus's Cranelift-emitted host code.
 *
 * Every entry point in section 1 has the signature of the symbol the
 * reference injects into its JIT through `RuntimeSymbols`
 * (crates/malus-codegen-cpu/src/lib.rs:116-184); Rust `usize` is `size_t`,
 * tensor handles are `int64_t` (an opaque pointer, 0 = none).  Section 2 is
 * the non-JIT Rust API the CLI and tests call (crates/malus-runtime/src/
 * lib.rs, bench.rs, metal.rs).  Section 3 holds the stdlib host functions the
 * JIT would otherwise compile from crates/malus-stdlib/stdlib/*.ml; they keep
 * the .ml names and signatures, so the BwdSlot table (codegen-cpu
 * lib.rs:189-220) points at them directly.  Section 4 is new in this build:
 * fused optimizer, data parallelism, the compiled nanoGPT step, and
 * diagnostics.
 *
 * Conventions (same as the reference):
 *  - every op returns a NEW handle with refcount 1 owned by the caller; inputs
 *    are borrowed;
 *  - all work is asynchronous on one CUDA stream; host reads synchronise;
 *  - errors print "malus: ..." to stderr and abort() (panic-only model,
 *    reference docs/adr/0006-panic-only-error-model.md).
 */
#ifndef MALUS_RUNTIME_H
#define MALUS_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Dtype tags: crates/malus-runtime/src/metal.rs:18-60.  Only F32 (0), I32 (5)
 * and I64 (6) are allocatable (metal.rs:375-378). */
enum { MALUS_F32 = 0, MALUS_I32 = 5, MALUS_I64 = 6 };

/* ===================== 1. RuntimeSymbols (JIT-injected) ================== */

/* metal.rs:340-347 tensor_alloc_gpu: shape[ndims] row-major; data may be NULL
 * (uninitialised) or point to len*elem_size host bytes copied to the device. */
int64_t tensor_alloc_gpu(int32_t dtype, const size_t* shape, size_t ndims, const float* data);
/* metal.rs:458-484 */
int64_t tensor_alloc_zeros_gpu(const size_t* shape, size_t ndims);
/* metal.rs:486-492 */
int64_t tensor_alloc_ones_gpu(const size_t* shape, size_t ndims);
/* metal.rs:555-558: tensor_free == tensor_release. All accept 0. */
void tensor_free(int64_t h);
/* metal.rs:498-507 */
void tensor_retain(int64_t h);
/* metal.rs:509-551: decrement; aborts on over-release. */
void tensor_release(int64_t h);
/* metal.rs:560-588 */
void tensor_print(int64_t h);
/* metal.rs:651-672 (tensor_dim accepts negative i) */
int64_t tensor_len(int64_t h);
int64_t tensor_ndim(int64_t h);
int64_t tensor_dim(int64_t h, int64_t i);
/* metal.rs:1860-1931: launch a registered builtin kernel; out has the shape of
 * handles[0]. */
int64_t kernel_dispatch(uint64_t kernel_id, const int64_t* handles, size_t count);
/* metal.rs:1944-2065: launch a registered explicit kernel with caller
 * grid/tg, explicit out shape (out_ndim 0 = inherit handles[0]), uniforms. */
int64_t kernel_dispatch_v2(uint64_t kernel_id, const int64_t* handles, size_t hc,
                           const size_t* grid, const size_t* tg, const size_t* out_shape,
                           size_t out_ndim, int32_t out_dtype, const void* uniforms,
                           size_t uniforms_bytes);
/* metal.rs:676-694: wait for all queued work; abort on a device error. */
void gpu_barrier(void);
/* metal.rs:820-962: (2,2), (3,3) batched and (3,2) broadcast f32 matmul. */
int64_t tensor_matmul(int64_t a, int64_t b);
/* metal.rs:1419-1435 zero-copy reshape; metal.rs:1407-1417 permute (0 args =
 * 2-D transpose, 2 args = swap, rank args = full permutation). */
int64_t tensor_reshape(int64_t h, const size_t* dims, size_t ndims);
int64_t tensor_permute(int64_t h, const size_t* perm, size_t ndims);
/* metal.rs:1601-1612: [T,T], 0 on/below the diagonal, -1e9 above. */
int64_t tensor_causal_mask(int64_t t);
/* metal.rs:1715-1737: Philox4x32-10 + Box-Muller N(0,1), per-call key. */
int64_t tensor_randn(const size_t* shape, size_t ndims);
/* metal.rs:1741-1749 / 1751-1759: share the randn call counter. */
float malus_rand_uniform(void);
int64_t malus_rand_int(int64_t n);
/* metal.rs:1763-1769: flat f32 read (synchronises). */
float malus_tensor_get_f32(int64_t h, int64_t idx);

/* Tape: crates/malus-runtime/src/tape.rs:208-774. op_tag values follow
 * OpTag (tape.rs:14-44); slots follow BwdSlot (tape.rs:92-125). */
void tape_record_binop(int32_t op_tag, int64_t a, int64_t b, int64_t out);
void tape_record_unary(int32_t op_tag, int64_t x, int64_t out);
void tape_record_reduce(int32_t op_tag, int64_t x, int64_t out, int64_t axis, int64_t keepdim);
void tape_record_perm(int32_t op_tag, int64_t x, int64_t out, const size_t* dims, size_t ndims);
/* var_h / softmax_h ownership is transferred to the tape (tape.rs:289-336). */
void tape_record_layernorm(int32_t op_tag, int64_t x, int64_t out, int64_t var_h, int64_t axis);
void tape_record_cross_entropy(int32_t op_tag, int64_t logits, int64_t out, int64_t softmax_h,
                               int64_t targets);
void tape_record_embedding(int32_t op_tag, int64_t weight, int64_t indices, int64_t out);
void tape_register_leaf(int64_t h);
void tape_pause(void);
void tape_resume(void);
void tape_clear(void);
int64_t tape_get_grad(int64_t h);
void backward(int64_t loss);
void tape_zero_grad(const int64_t* handles, size_t count);
void tape_register_backward_fn(int32_t slot, size_t fnptr);

/* buffer.rs:11-50: host i32 staging buffer; freeze uploads an i32 tensor. */
int64_t malus_buffer_i32(int64_t len);
int64_t malus_buffer_get_i32(int64_t buf, int64_t idx);
void malus_buffer_set_i32(int64_t buf, int64_t idx, int64_t val);
void malus_buffer_free(int64_t buf);
int64_t malus_buffer_freeze_i32(int64_t buf);

/* lib.rs:33 gradient-check recorder; bench.rs:22-38 warm-median step timer. */
void malus_record_diff(float v);
void bench_step_begin(void);
void bench_step_end(void);

/* strio.rs (out of scope for the training hot path, whose workloads use
 * synthetic token ids).  Provided so a JIT link table resolves: strings are host byte
 * boxes, read_file reads a whole file. */
int64_t malus_str_box(const uint8_t* bytes, size_t len);
int64_t malus_read_file(int64_t path_box);
int64_t malus_str_len(int64_t s);
int64_t malus_str_char_at(int64_t s, int64_t i);
int64_t malus_str_from_char(int64_t c);

/* ===================== 2. Runtime API used by the CLI / tests ============ */

/* metal.rs:309-336 runtime_init(id -> source).  This runtime has no MSL
 * compiler: each id is bound to a native kernel by NAME (the builtin names of
 * crates/malus-syntax/src/ast.rs:59-81 and codegen-gpu lib.rs:373-418, or a
 * stdlib kernel name such as "__softmax_kernel").  Unknown names abort. */
void malus_runtime_init(const uint64_t* ids, const char* const* names, size_t n);
int64_t malus_cpu_compute_count(void);          /* lib.rs:14 (always 0 here) */
void malus_cpu_compute_reset(void);             /* lib.rs:19 */
float malus_gradcheck_max_diff(void);           /* lib.rs:48 */
void malus_gradcheck_reset(void);               /* lib.rs:53 */
void malus_rc_counts(int64_t* retains, int64_t* releases, int64_t* allocs); /* lib.rs:81 */
void malus_rc_reset(void);                      /* lib.rs:90 */
/* metal.rs:149-183: hits, misses, pooled bytes, peak device bytes. */
void malus_pool_stats(int64_t* hits, int64_t* misses, int64_t* pooled_bytes, int64_t* peak_bytes);
void malus_pool_reset(void);                    /* metal.rs:175 */
void malus_set_mem_budget(int64_t bytes);       /* metal.rs:148 */
void bench_enable(void);                        /* bench.rs:18 */
/* bench.rs:51-70: warm median (host clock, ms) over the steps after 3 warm-up
 * steps; -1 if fewer than 4 steps were recorded.  n_steps receives the timed
 * count.  bench_report_range gives the same steps' min and max (BenchReport's
 * min / max; -1 when there are none). */
double bench_report(int64_t* n_steps);
void bench_report_range(double* min_ms, double* max_ms);
void bench_reset(void);                         /* bench.rs:72: disables and clears */
/* Test helper mirroring tape.rs:733-750 tape_reset: drops leaves, grads, tape. */
void malus_tape_reset(void);
/* Number of live leaves / leaf grads (tape.rs:791-797 registry_lens). */
void malus_tape_registry_lens(int64_t* leaves, int64_t* grads);

/* Raw device pointer of a handle (for zero-copy interop: the data of a
 * handle lives in HBM on the current device). */
void* malus_tensor_data(int64_t h);
int32_t malus_tensor_dtype(int64_t h);
/* Copy a tensor to / from host memory (synchronous). */
void malus_tensor_read(int64_t h, void* dst, size_t bytes);
void malus_tensor_write(int64_t h, const void* src, size_t bytes);
/* Wrap caller-owned device memory as a handle (not pooled; never freed). */
int64_t malus_tensor_wrap(int32_t dtype, void* dev_ptr, const size_t* shape, size_t ndims);
/* Reset the Philox call counter (metal.rs:1713-1715 is thread-local; the
 * reference resets it only per thread start). */
void malus_rng_reset(uint64_t counter);
/* Host-only: the Philox4x32-10 block function of metal.rs:1692-1711 (Salmon
 * et al., SC'11) applied in place to a 4-word counter under a 2-word key, for
 * known-answer tests of the generator behind tensor_randn / malus_rand_*. */
void malus_philox4x32_10(uint32_t ctr[4], const uint32_t key[2]);
/* Select the CUDA device for this process (default: LOCAL_RANK or 0). */
void malus_set_device(int32_t dev);
/* Device kernel launches issued by this runtime since the last reset; the
 * kernels of a captured graph count at each malus_graph_replay, not at capture. */
int64_t malus_launch_count(void);
void malus_launch_count_reset(void);
/* Current stream as a cudaStream_t (for callers that share the stream). */
void* malus_stream(void);

/* ===================== 3. Native stdlib host functions ==================== */
/* Each replaces the same-named `fn` in crates/malus-stdlib/stdlib/*.ml. */

/* broadcast_binop.ml:82-112 (NumPy right-aligned broadcasting) */
int64_t __broadcast_add_fwd(int64_t a, int64_t b);
int64_t __broadcast_sub_fwd(int64_t a, int64_t b);
int64_t __broadcast_mul_fwd(int64_t a, int64_t b);
int64_t __broadcast_div_fwd(int64_t a, int64_t b);
/* softmax.ml:30-40 */
int64_t __softmax_fwd(int64_t x, int64_t axis);
/* layernorm.ml:60-72: returns a tuple box (calloc'd, refcount 1 at +0,
 * normed handle at +8, variance handle (keepdim at axis) at +16). */
int64_t __layernorm_fwd(int64_t x, int64_t axis);
/* cross_entropy.ml:18-28: tuple box (loss [1] at +8, probs [N,C] at +16). */
int64_t __cross_entropy_fwd(int64_t logits, int64_t targets);
/* embedding.ml:18-23 */
int64_t __embedding_fwd(int64_t weight, int64_t indices);
/* gelu.ml:12-14 */
int64_t __gelu_fwd(int64_t x);
/* reduce_*.ml: axis reductions (any axis length: no 1024 cap). */
int64_t __reduce_sum_fwd(int64_t x, int64_t axis, int64_t keepdim);
int64_t __reduce_mean_fwd(int64_t x, int64_t axis, int64_t keepdim);
int64_t __reduce_max_fwd(int64_t x, int64_t axis, int64_t keepdim);
int64_t __reduce_var_fwd(int64_t x, int64_t axis, int64_t keepdim);
/* reduce_all.ml:9-12 (any length) */
int64_t __reduce_all_sum_fwd(int64_t x);
/* permute.ml: rank-generic permute (perm padded to 8 entries). */
int64_t __permute_nd_fwd(int64_t x, int64_t p0, int64_t p1, int64_t p2, int64_t p3,
                         int64_t p4, int64_t p5, int64_t p6, int64_t p7);
int64_t __transpose_2d_fwd(int64_t x);
/* unary_bwd.ml: scale / fill_like / eq */
int64_t __scale_fwd(int64_t x, float c);
int64_t __fill_like_fwd(int64_t x, float c);
int64_t __eq_fwd(int64_t a, int64_t b);
/* reduce_bwd.ml:22-38 */
int64_t __expand_axis_fwd(int64_t small, int64_t x_template, int64_t axis);
/* elementwise_bwd.ml:8-22 */
int64_t __sum_to_shape_bwd(int64_t dout, int64_t target);
/* transformer_bwd.ml:6-12 */
int64_t __rsqrt_eps_fwd(int64_t v, float eps);

/* The 30 BwdSlot functions (tape.rs:92-125 / codegen-cpu lib.rs:189-220). */
int64_t __add_bwd_a(int64_t dout, int64_t a);
int64_t __add_bwd_b(int64_t dout, int64_t b);
int64_t __sub_bwd_a(int64_t dout, int64_t a);
int64_t __sub_bwd_b(int64_t dout, int64_t b);
int64_t __mul_bwd_a(int64_t dout, int64_t a, int64_t b);
int64_t __mul_bwd_b(int64_t dout, int64_t a, int64_t b);
int64_t __div_bwd_a(int64_t dout, int64_t a, int64_t b);
int64_t __div_bwd_b(int64_t dout, int64_t a, int64_t b);
int64_t __sigmoid_bwd(int64_t s, int64_t dout);
int64_t __relu_bwd(int64_t x, int64_t dout);
int64_t __tanh_bwd(int64_t t, int64_t dout);
int64_t __sqrt_bwd(int64_t s, int64_t dout);
int64_t __abs_bwd(int64_t x, int64_t dout);
/* reduce_bwd.ml:73-76: reads dout[0] ON THE DEVICE (no host sync). */
int64_t __sum_bwd(int64_t x, int64_t dout);
int64_t __reduce_sum_axis_bwd(int64_t x, int64_t dout, int64_t axis);
int64_t __reduce_mean_axis_bwd(int64_t x, int64_t dout, int64_t axis);
int64_t __reduce_max_axis_bwd(int64_t x, int64_t y, int64_t dout, int64_t axis);
int64_t __reduce_var_axis_bwd(int64_t x, int64_t dout, int64_t axis);
/* transformer_bwd.ml:15-20, fused into one kernel */
int64_t __softmax_bwd(int64_t s, int64_t dout, int64_t axis);
/* transformer_bwd.ml:24-36 with the host-side (tape.rs:1162-1186) per-row
 * variance semantics; fused into one kernel */
int64_t __layernorm_bwd(int64_t y, int64_t var_h, int64_t dout, int64_t axis);
int64_t __gelu_bwd(int64_t x, int64_t dout);
/* transformer_bwd.ml:66-75; dout[0] read on the device */
int64_t __cross_entropy_bwd(int64_t probs, int64_t targets, int64_t dout);
/* transformer_bwd.ml:83-98; deterministic sort-then-segmented-sum */
int64_t __embedding_bwd(int64_t weight, int64_t indices, int64_t dout);
/* matmul_bwd.ml:15-29; transposed-operand GEMMs (no materialised transpose) */
int64_t __matmul_bwd_a(int64_t a, int64_t b, int64_t dout);
int64_t __matmul_bwd_b(int64_t a, int64_t b, int64_t dout);

/* ===================== 4. New in this build ============================== */

/* Fused multi-tensor AdamW, the exact f32 operation order of
 * examples/nanogpt.ml:80-91 (L2-coupled weight decay):
 *   g = grad*grad_scale + wd*p; m = b1*m + (1-b1)*g; v = b2*v + ((1-b2)*g)*g;
 *   p = p - (lr*(m/bc1)) / (sqrt(v/bc2) + eps),  bc = 1 - beta**step (f32 powf).
 * Updates params, ms, vs IN PLACE (the reference re-registers a new leaf per
 * step; observable values are identical).  grads[i] == 0 means "no grad
 * accumulated" (tape_get_grad returns zeros). grad_scale is 1/world for DP. */
void malus_adamw_multi(const int64_t* params, const int64_t* grads, const int64_t* ms,
                       const int64_t* vs, size_t n, float lr, float beta1, float beta2,
                       float eps, float wd, int64_t step, float grad_scale);

/* Data parallelism (one process per GPU, NCCL over NVLink).  nccl_id is the
 * 128-byte ncclUniqueId produced by malus_dp_unique_id on rank 0 and shared
 * out of band.  Returns 0 on success, a negative error otherwise. */
int32_t malus_dp_unique_id(uint8_t* out128);
int32_t malus_dp_init(int32_t rank, int32_t world, const uint8_t* nccl_id, int32_t timeout_ms);
/* In-place sum-allreduce of a contiguous f32 device buffer on the DP stream. */
int32_t malus_dp_allreduce_f32(void* dev_ptr, size_t count);
int32_t malus_dp_finish(void);   /* wait for outstanding collectives */
/* Per-leaf gradient readiness (overlaps the gradient all-reduce with the
 * backward pass).  Register the leaves (parameters) once, in order; they are
 * grouped into buckets of at least bucket_bytes (returns the bucket count,
 * -1 if a leaf is listed twice).  After that the tape's backward reports each
 * registered leaf as soon as its gradient is final and averages every
 * completed bucket in place across ranks (one grouped all-reduce on the DP
 * stream); callers that build gradients outside the tape report them with
 * malus_dp_grad_ready(leaf, grad) (grad 0: no gradient in this backward pass).  All
 * ranks must report the same leaves in the same order. */
int32_t malus_dp_register_leaves(const int64_t* leaves, size_t n, size_t bucket_bytes);
int32_t malus_dp_grad_ready(int64_t leaf, int64_t grad);
int32_t malus_dp_destroy(void);
/* User kernel bodies.  malus_runtime_init accepts, for any id, either a native
 * kernel name or the MSL text that malus-codegen-gpu emits for a `kernel`
 * (crates/malus-codegen-gpu/src/lib.rs:432-1006; the reference's runtime_init
 * takes exactly that id -> MSL map, crates/malus-runtime/src/metal.rs:300-336);
 * the text is translated to CUDA C++ and compiled with NVRTC for sm_100a, once
 * per distinct source.  Host-only helpers: the translation itself (returns its
 * length, or -1 with the reason in out) and a compile check (0 = compiled). */
int32_t malus_jit_translate(const char* msl, char* out, size_t cap);
int32_t malus_jit_compile_check(const char* msl, char* log, size_t cap);
/* Fused causal attention forward (tcgen05, 3xTF32): from the tf32 planes of
 * q|k|v laid out [3][B][H][T][hs], writes O = causal_softmax(q k^T * scale) v
 * as head-unfolded planes [B*T][H*hs]; optionally the planes of P
 * [B*H][T][T] (keys up to each query's 128-wide tile; p_hi = p_lo = NULL
 * skips them) and the per-row statistics `stats` [B*H*T][2] = (row max of the
 * scaled scores times log2 e, 1 / row sum) that malus_attn_bwd recomputes P
 * from as 2^(s*scale*log2 e - max) / sum (NULL
 * skips them).  Needs T % 128 == 0 and hs in {32, 64} (returns -1 otherwise).
 * New in this build; replaces the reference's bmm + scale + mask + softmax +
 * bmm sequence of the attention block. */
int32_t malus_attn_fwd(const float* qkv_hi, const float* qkv_lo, int32_t B, int32_t H, int32_t T,
                       int32_t hs, float scale, float* p_hi, float* p_lo, float* o_hi, float* o_lo,
                       float* stats);
/* Which kernel serves malus_attn_fwd for T <= 384: 1 (default) keeps the
 * tile's scores resident in tensor memory and computes them once; 0 recomputes
 * them in the second softmax pass (the kernel used for longer sequences).  Both
 * give the same bits.  Returns the previous setting.  Environment:
 * MALUS_ATTN_RS=0 starts with 0.  New in this build. */
int32_t malus_attn_set_resident(int32_t on);

/* ---- SafeTensors files (malus's interop spec, docs/spec/08-interop.md:
 * `load(path)` / `save(tensors, path)` of named tensor sets).  An 8-byte
 * little-endian header length, a JSON header mapping each name to its dtype
 * ("F32", "I32", "I64"), shape and [begin, end) byte offsets, then the data.
 * Negative codes: -1 I/O, -2 header length, -3 JSON, -4 a name or field
 * (empty, duplicate, "__metadata__", unsupported dtype, rank above 8), -5
 * offsets (outside the file, not matching the shape, overlapping), -6 no such
 * name.  New in this build. */
/* Write n tensors held in host memory (dtype codes 0, 5, 6). */
int32_t malus_safetensors_write_host(const char* path, size_t n, const char* const* names, const int32_t* dtypes,
                                     const size_t* const* shapes, const size_t* ndims, const void* const* data);
/* The names in header order, newline-separated (NUL-terminated, truncated at
 * cap); returns the length the whole list needs, or a negative code. */
int32_t malus_safetensors_names(const char* path, char* buf, int32_t cap);
/* One tensor into host memory: dtype, rank, shape (up to 8 dims) always, its
 * bytes when cap holds them; returns the byte count or a negative code. */
int64_t malus_safetensors_read_host(const char* path, const char* name, int32_t* dtype, size_t* shape,
                                    size_t* ndim, void* data, size_t cap);
/* Save device tensors under the given names (views and deferred results are
 * materialised); returns 0 or a negative code. */
int32_t malus_save_safetensors(const char* path, size_t n, const char* const* names, const int64_t* handles);
/* Load one tensor onto the GPU as a new handle (refcount 1); 0 when the name
 * is absent or the file invalid (the reason goes to stderr). */
int64_t malus_load_safetensors(const char* path, const char* name);
/* Fused causal attention backward (tcgen05, 3xTF32), the VJP of
 * malus_attn_fwd: from the q|k|v planes, the planes of dO (head-folded
 * [B][H][T][hs]) and of O (head-unfolded, as the forward wrote them) and the
 * forward's `stats`, writes the planes of dq | dk | dv head-unfolded into
 * dqkv [3][B*T][H*hs].  `D` is a workspace of B*H*T floats (rowsum(dO * O)).
 * P is recomputed; no [T][T] tensor is touched.  Same shape limits as the
 * forward (returns -1 otherwise).  New in this build; replaces the reference's
 * VJPs of that sequence (tape.rs matmul VJP, softmax.ml softmax VJP). */
int32_t malus_attn_bwd(const float* qkv_hi, const float* qkv_lo, const float* do_hi,
                       const float* do_lo, const float* o_hi, const float* o_lo, const float* stats,
                       float* D, int32_t B, int32_t H, int32_t T, int32_t hs, float scale,
                       float* dqkv_hi, float* dqkv_lo);
/* Graph capture of the runtime stream (the caller side of the boundary: one
 * launch per training step).  Between malus_graph_begin and malus_graph_end
 * every runtime call is recorded instead of executed; malus_graph_replay
 * launches the recording on the runtime stream.  Replays run on the buffers
 * of the capture: the pool keeps every buffer the graph touches out of reuse
 * until malus_graph_destroy, a replayed step must update its state in place
 * and read its inputs from tensors that stay alive (write new inputs with
 * malus_tensor_write between replays), and host reads inside the capture
 * abort with a message.  Run the sequence once before capturing it so that
 * grow-on-demand workspaces are sized.  New in this build (no reference
 * counterpart: Metal command buffers are re-encoded every step). */
int32_t malus_graph_begin(void);
int64_t malus_graph_end(void);            /* graph id (> 0) */
int32_t malus_graph_replay(int64_t graph);   /* -1 for an unknown id */
int32_t malus_graph_destroy(int64_t graph);
/* Abort the communicator without contacting peers (after one is known lost). */
int32_t malus_dp_abort(void);
int32_t malus_dp_world(void);

/* The compiled nanoGPT training step (replaces the per-step call sequence of
 * examples/nanogpt.ml:167-191 / nanogpt_modular.ml with one entry point). */
typedef struct malus_gpt_config {
  int32_t vocab, n_layer, n_head, n_embd, block_size, batch;
  int32_t tied;          /* 1: LM head is wte^T (GPT-2 weight tying) */
  float lr, beta1, beta2, eps, wd, init_std;
  int32_t mode;          /* 0: tape (reference call sequence), 1: fused B200 step */
  int32_t use_graph;     /* 1: capture the fused step in a CUDA graph */
  uint64_t seed;         /* Philox call counter start for the weight init */
} malus_gpt_config;
int64_t malus_gpt_create(const malus_gpt_config* cfg);
void malus_gpt_destroy(int64_t model);
/* One training step on host token ids x/y (int32, batch*block_size each).
 * Copies the ids to the device, runs forward, backward, (DP allreduce) and
 * AdamW, and returns the loss (synchronises). */
float malus_gpt_step(int64_t model, const int32_t* x, const int32_t* y);
/* Same step with ids already on the device; the loss stays on the device
 * (read it with malus_gpt_last_loss). */
void malus_gpt_step_device(int64_t model, const int32_t* x_dev, const int32_t* y_dev);
float malus_gpt_last_loss(int64_t model);
/* Number of parameter tensors and their handles (layout order of
 * nanogpt_modular.ml: per block [ln1,wq,wk,wv,wo,ln2,w1,w2], then
 * [wte,wpe,ln_f,lm_head]). */
int32_t malus_gpt_num_params(int64_t model);
int64_t malus_gpt_param(int64_t model, int32_t i);
/* Gradient of parameter i from the last step (before the update; summed over
 * data-parallel ranks), same shape; a borrowed handle like malus_gpt_param. */
int64_t malus_gpt_grad(int64_t model, int32_t i);
/* AdamW state of parameter i (which = 0: first moment m, 1: second moment v),
 * a borrowed handle like malus_gpt_param. */
int64_t malus_gpt_moment(int64_t model, int32_t i, int32_t which);
int64_t malus_gpt_num_elements(int64_t model);
/* Host-only (no device work): the fused parameter/gradient buffer layout for a
 * config.  Writes offsets[i] and sizes[i] (elements) for the first n tensors,
 * *total = buffer length in elements (slices 256-byte aligned); returns the
 * tensor count. */
int32_t malus_gpt_layout(const malus_gpt_config* cfg, int64_t* offsets, int64_t* sizes, int32_t n,
                         int64_t* total);
/* Host-only: the data-parallel all-reduce buckets of the fused step in issue
 * order ([lo, hi) element ranges of the gradient buffer: each layer, last
 * first, then embeddings / final norm / head); returns the bucket count. */
int32_t malus_gpt_dp_buckets(const malus_gpt_config* cfg, int64_t* lo, int64_t* hi, int32_t n);

/* tcgen05 3xTF32 GEMM on pre-split tf32 operand planes, with fused epilogues.
 * Each f32 operand x is given as two planes hi = tf32_rn(x), lo = tf32_rn(x -
 * hi) (malus_tf32_split makes them).  An operand is a stack of nz row-major
 * slices of rows x cols (row pitch in floats, multiple of 4; slice stride
 * zstride): K-major operands are stored {rows = M (or N), cols = K}, MN-major
 * ones {rows = K, cols = M (or N)}.  zmode picks the slice for each tile:
 * 0 none, 1 the problem batch index, 2 k / seg, 3 m-or-n / seg.  The output
 * element (z, m, n) lives at oz(z) + om(m) + on(n), each term
 * (i / div) * hi + (i % div) * lo (div 0: i * lo).  Epilogues: 0 store
 * (alpha, beta), 1 residual add (out = aux + acc), 2 GELU (out = acc, planes
 * of gelu(acc)), 3 GELU derivative (planes of acc * gelu'(aux)), 4 softmax
 * backward (planes of alpha * P * (acc - rowv[z*M + m]) with P = aux + aux_lo,
 * the hi/lo planes of the softmax output, acc = dP); out_hi/out_lo,
 * when set, receive the tf32 planes of the stored value.  causal (per batch
 * slice, for attention matrices): 0 none; 1 only output tiles that reach the
 * lower triangle n <= m are computed (the rest of the output is not written);
 * 2 A is lower-triangular (A(m,k) = 0 for k > m: the K range stops at the
 * diagonal); 3 A is upper-triangular (A(m,k) = 0 for k < m).  New in this build
 * (the reference's matmul is an MPS call, metal.rs:805-962). */
typedef struct malus_tc_operand {
  const float* hi; const float* lo;
  int64_t rows, cols, pitch;
  int32_t nz; int64_t zstride;
  int32_t mn_major, zmode, seg;
} malus_tc_operand;
typedef struct malus_tc_layout { int64_t d1, s1, d2, s2, s3; } malus_tc_layout;
typedef struct malus_tc_problem {
  int32_t M, N, K, batch;
  malus_tc_operand a, b;
  int32_t epi;
  malus_tc_layout oz, om, on;
  float* out; float* out_hi; float* out_lo;
  const float* aux;
  float alpha, beta;
  int32_t causal;
  const float* aux_lo;
  const float* rowv;
} malus_tc_problem;
void malus_tc_gemm(const malus_tc_problem* p);
/* CTA pairs the tcgen05 GEMM keeps resident when it runs a problem as 2-CTA
 * clusters (256-row tiles; problems with M a multiple of 256, unsplit and
 * non-causal); 0 when pairs are off or cannot be placed.  A diagnostic with
 * no counterpart in the reference. */
int32_t malus_gemm_pair_clusters(void);
/* Which eligible problems run as CTA pairs: -1 the measured rule (plain-store
 * and GELU epilogues with K >= 256), 0 none, 1 all.  Starts from the
 * environment variable MALUS_GEMM_CTA2 (unset: -1).  Returns the previous
 * mode.  A tuning and test hook with no counterpart in the reference. */
int32_t malus_gemm_pair_mode(int32_t mode);
void malus_tf32_split(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t batch,
                      int64_t sstride, float* hi, float* lo, int64_t pitch);

/* Device diagnostics: last asynchronous error word written by a kernel whose
 * bounded wait ran out (0 = none); cleared by reading. */
int32_t malus_device_error(void);

/* Live per-kernel-class timing with CUDA events (for roofline figures).
 * Classes: 0 tcgen05 GEMM, 1 GEMM operand split, 2 SIMT GEMM (on the runtime
 * stream); 3 data-parallel all-reduce (on the collective stream, bytes =
 * payload); 4 the runtime stream's wait for the all-reduces (the part the
 * backward pass does not hide).  Enabling resets the records; while enabled
 * the model step runs without its CUDA graph. */
void malus_prof_enable(int32_t on);
void malus_prof_report(int32_t cls, int64_t* count, double* ms, double* flops, double* bytes);
/* Class 5, the compiled step's other kernels, each timed with its algorithmic
 * bytes: one text line "label<TAB>launches<TAB>ms<TAB>bytes" per kernel label
 * (first-launch order) into buf (NUL-terminated, truncated at cap); returns
 * the length of the whole text. */
int32_t malus_prof_kernels(char* buf, int32_t cap);

/* Embedding backward that allocates nothing.  This entry point has no
 * counterpart in the reference.  It is for callers that cannot call cudaMalloc
 * where they need the op (inside a stream capture that must not gain memory
 * nodes, inside another framework's memory arena, or under a fully committed
 * memory budget).  It computes dweight[vocab, dim] from dout[n, dim] and
 * indices[n] (i32 when index_dtype is 5, i64 when 6) with the same
 * deterministic sort-then-segmented-sum as __embedding_bwd, on the caller's
 * stream (NULL = the legacy default stream).  All inputs and the output are
 * caller-owned device pointers; the scratch is a fixed 4,982,016-byte device array
 * inside this library, present on every GPU that loads it until the process
 * exits.  Limits: n <= 65536 and vocab * ceil(n / 1024) <= 524288; larger
 * sizes return a negative error with a message on stderr.  The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  All calls share the array, so
 * calls that overlap on the GPU race; ordered calls (one stream) are safe.
 * An id outside [0, vocab) is skipped without a report (its dout row adds to
 * no gradient row; the call still returns 0), because this entry point does
 * not touch the runtime's error word; validate ids first where that matters.
 * n = 0 writes zeros to dweight.  Returns 0 on success. */
int32_t malus_embedding_bwd_noalloc(const float* dout, const void* indices, int32_t index_dtype,
                                    size_t n, size_t vocab, size_t dim, float* dweight,
                                    void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MALUS_RUNTIME_H */
