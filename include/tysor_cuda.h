/*
 * tysor CUDA backend: the C ABI of libtysor_cuda.so (sm_100a).
 *
 * This library takes the place of the reference's Metal bridge
 * (native/metal_bridge.mm, bound from Rust in src/backend/metal/native.rs).
 * The per-op surface keeps the Metal bridge's entry points, argument order
 * and error convention; the graph surface (tysor_cuda_graph_*) is the
 * device-resident executor that replaces the host-side op loop.
 *
 * Conventions (same as the Metal bridge, native/metal_bridge.mm:14-16, 72-97):
 *   - handles are opaque pointers; buffers hold fp32 element counts;
 *   - every call that can fail returns bool (or NULL); on failure
 *     tysor_cuda_last_error() returns the message (thread-local);
 *   - no C++ exception crosses this boundary, nothing aborts the process.
 * Unlike the Metal bridge, dispatches are asynchronous on the context's
 * stream: tysor_cuda_buffer_read / tysor_cuda_synchronize wait for them and
 * report any error a kernel recorded (for example an embedding index out of
 * range).  There is no CPU fallback: a missing GPU is an error.
 */
#ifndef TYSOR_CUDA_H
#define TYSOR_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- errors, context ---------------------------------------------------- */

/* native.rs:17 tysor_metal_last_error */
const char* tysor_cuda_last_error(void);

/* native.rs:18 tysor_metal_context_new(source): kernels are precompiled for
 * sm_100a, so the context takes a device ordinal instead of MSL source. */
void* tysor_cuda_context_new(int device);
/* native.rs:19 tysor_metal_context_free */
void tysor_cuda_context_free(void* context);
/* Waits for all work on the context stream; false if a kernel recorded an
 * error (the Metal bridge waits inside every dispatch, bridge:89-90). */
bool tysor_cuda_synchronize(void* context);
/* Matmul arithmetic: 0 = strict (3xTF32, the default), 1 = fast (1xTF32),
 * 2 = exact (CUDA-core fp32 in k order), 3 = strict16 (the same three
 * products over fp16 halves with a power-of-two scale per operand row, on
 * the tensor core's fp16 rate; unbatched non-causal GEMMs with M >= 256 and
 * N > 128, the others as strict).  No reference counterpart. */
bool tysor_cuda_set_matmul_mode(void* context, int mode);
/* Tensor-core matmuls (strict and fast): how many k-blocks of 16 the tensor
 * core accumulates in tensor memory before the partial sum is added into
 * fp32 registers with round-to-nearest.  The tensor core adds each MMA into
 * its accumulator rounding toward zero, a systematic shrink of up to one
 * ulp per instruction (three instructions per k-slice in strict mode), so
 * shorter chunks are more accurate and read the accumulator more often.
 * 0 = the default, 8 (128 elements of K).  Measured on the Llama block,
 * the 4-layer LM and the MLP at full size (gradients against an f64 answer):
 * within 2.1e-5 at 8, 7.5e-6 at 2 (the step 9.6% slower), 5.3e-6 at 1 (19%
 * slower), the f32 reference's own arithmetic being 5.5e-6 away.  Graphs
 * re-plan at their next run.  No reference counterpart. */
bool tysor_cuda_set_matmul_accumulation(void* context, int kblocks);
/* Runs the tensor-core pipelines' bounded barrier wait on a barrier that
 * nothing arrives at, giving up after `limit_cycles` (1 to 4e9) SM cycles:
 * returns false with "a tensor-core pipeline wait timed out", and the context
 * stays usable.  Exercises the timeout path without a fault.  No reference
 * counterpart. */
bool tysor_cuda_probe_wait_timeout(void* context, int64_t limit_cycles);
/* The context's CUDA stream (a cudaStream_t), for callers that time or
 * order their own work against it.  No reference counterpart. */
void* tysor_cuda_context_stream(void* context);

/* ---- buffers ------------------------------------------------------------- */

/* native.rs:20 tysor_metal_buffer_new_with_data */
void* tysor_cuda_buffer_new_with_data(void* context, const float* data, size_t count);
/* native.rs:21 tysor_metal_buffer_new_zeroed */
void* tysor_cuda_buffer_new_zeroed(void* context, size_t count);
/* native.rs:22 tysor_metal_buffer_free (also frees views) */
void tysor_cuda_buffer_free(void* buffer);
/* native.rs:23 tysor_metal_buffer_read: waits for the stream first. */
bool tysor_cuda_buffer_read(void* buffer, float* out_data, size_t count);
/* Host -> device copy into an existing buffer.  No reference counterpart. */
bool tysor_cuda_buffer_write(void* buffer, const float* data, size_t count);
/* A view of `count` elements starting at element `offset` of `base`
 * (plan-once arenas).  No reference counterpart. */
void* tysor_cuda_buffer_view(void* base, size_t offset, size_t count);
/* Element count of a buffer or view. */
size_t tysor_cuda_buffer_count(void* buffer);

/* ---- forward dispatch (native.rs:24-136, same names and argument order;
 *      the Metal kernel-name string becomes an op code) -------------------- */

enum {
  TYSOR_UNARY_COPY = 0, /* reshape, flatten_heads (codegen.rs:101-105) */
  TYSOR_UNARY_RELU = 1, /* codegen.rs:95-99 */
  TYSOR_UNARY_SILU = 2, /* codegen.rs:226-228 */
  TYSOR_UNARY_SCALE = 3 /* x * param: scale(), Dropout keep factor */
};
enum { TYSOR_BINARY_ADD = 0, TYSOR_BINARY_SUB = 1, TYSOR_BINARY_MUL = 2, TYSOR_BINARY_DIV = 3 };

/* native.rs:24-33 */
bool tysor_cuda_dispatch_matmul(void* context, void* lhs, void* rhs, void* out, uint32_t m,
                                uint32_t n, uint32_t k);
/* native.rs:34-40; param is the scale factor for TYSOR_UNARY_SCALE. */
bool tysor_cuda_dispatch_unary(void* context, int op, void* input, void* out, uint32_t count,
                               float param);
/* native.rs:41-48 */
bool tysor_cuda_dispatch_binary_tt(void* context, int op, void* lhs, void* rhs, void* out,
                                   uint32_t count);
/* native.rs:49-55 (the Metal version bakes the scalar into the kernel text) */
bool tysor_cuda_dispatch_binary_ts(void* context, int op, void* input, void* out, uint32_t count,
                                   double scalar);
/* native.rs:56-62 */
bool tysor_cuda_dispatch_binary_st(void* context, int op, void* input, void* out, uint32_t count,
                                   double scalar);
/* native.rs:63-70 (eps 1e-5, no gain, layers.rs:275-299) */
bool tysor_cuda_dispatch_rms_norm(void* context, void* input, void* out, uint32_t rows,
                                  uint32_t width);
/* native.rs:71-78 */
bool tysor_cuda_dispatch_softmax(void* context, void* input, void* out, uint32_t rows,
                                 uint32_t width);
/* native.rs:79-87 (dense target of the logits' shape) */
bool tysor_cuda_dispatch_cross_entropy(void* context, void* logits, void* target, void* out,
                                       uint32_t rows, uint32_t width);
/* native.rs:88-99 */
bool tysor_cuda_dispatch_linear(void* context, void* input, void* weight, void* bias, void* out,
                                uint32_t m, uint32_t n, uint32_t k, bool with_bias);
/* native.rs:100-108, plus num_embeddings so indices are range-checked (the
 * Metal kernel reads out of bounds, codegen.rs:107-111; the CPU reference
 * raises "Embedding index out of range", layers.rs:147-149). */
bool tysor_cuda_dispatch_embedding(void* context, void* indices, void* weight, void* out,
                                   uint32_t index_count, uint32_t embedding_dim,
                                   uint32_t num_embeddings);
/* native.rs:109-118 */
bool tysor_cuda_dispatch_repeat_kv(void* context, void* input, void* out, uint32_t outer,
                                   uint32_t out_heads, uint32_t inner, uint32_t repeats);
/* native.rs:119-127 */
bool tysor_cuda_dispatch_causal_mask(void* context, void* input, void* out, uint32_t outer,
                                     uint32_t q, uint32_t k);
/* native.rs:128-136, with theta as an argument (codegen.rs:125-130 bakes it) */
bool tysor_cuda_dispatch_rope(void* context, void* input, void* out, uint32_t outer,
                              uint32_t seq_len, uint32_t half_dim, double theta);

/* ---- backward and update (the reference runs these on the CPU:
 *      src/runtime/layers.rs:326-549, src/training/executor.rs:563-762) ---- */

/* General matmul: C[b] = alpha*op(A[b]).op(B[b]) (+bias[n]) (relu) (+C_old).
 * A stored [m,k] (trans_a=0) or [k,m] (trans_a=1); B stored [k,n]
 * (trans_b=0) or [n,k] (trans_b=1); ld* are row pitches in elements;
 * stride* are batch strides in elements.  Covers backward_linear_input
 * (g.W^T, layers.rs:521-523) and backward_linear_weight (X^T.g, 525-527)
 * without materialised transposes. */
bool tysor_cuda_dispatch_matmul_ex(void* context, uint32_t batch, uint32_t m, uint32_t n,
                                   uint32_t k, void* a, bool trans_a, uint64_t lda,
                                   uint64_t stride_a, void* b, bool trans_b, uint64_t ldb,
                                   uint64_t stride_b, void* c, uint64_t ldc, uint64_t stride_c,
                                   void* bias, float alpha, bool accumulate, bool relu);
/* training/executor.rs:644-652: dx (+)= grad * (out > 0) */
bool tysor_cuda_dispatch_relu_backward(void* context, void* out_act, void* grad, void* dx,
                                       uint64_t count, bool accumulate);
/* layers.rs:330-348 */
bool tysor_cuda_dispatch_silu_backward(void* context, void* input, void* grad, void* dx,
                                       uint64_t count, bool accumulate);
/* layers.rs:350-364 (diagonal term only) */
bool tysor_cuda_dispatch_softmax_backward(void* context, void* output, void* grad, void* dx,
                                          uint64_t count, bool accumulate);
/* layers.rs:479-488: softmax(logits) - target */
bool tysor_cuda_dispatch_cross_entropy_backward(void* context, void* logits, void* target,
                                                void* grad, uint32_t rows, uint32_t width,
                                                bool accumulate);
/* layers.rs:438-477 */
bool tysor_cuda_dispatch_rope_backward(void* context, void* grad, void* dx, uint32_t outer,
                                       uint32_t seq_len, uint32_t half_dim, double theta,
                                       bool accumulate);
/* layers.rs:388-416 (heads = input heads) */
bool tysor_cuda_dispatch_repeat_kv_backward(void* context, void* grad, void* dx, uint32_t outer,
                                            uint32_t heads, uint32_t inner, uint32_t repeats,
                                            bool accumulate);
/* layers.rs:418-436 */
bool tysor_cuda_dispatch_causal_mask_backward(void* context, void* grad, void* dx, uint32_t outer,
                                              uint32_t q, uint32_t k, bool accumulate);
/* layers.rs:497-519: deterministic scatter-add in token order */
bool tysor_cuda_dispatch_embedding_backward(void* context, void* grad, void* indices,
                                            void* weight_grad, uint32_t index_count,
                                            uint32_t embedding_dim, uint32_t num_embeddings,
                                            bool accumulate);
/* layers.rs:529-549: column sums */
bool tysor_cuda_dispatch_bias_grad(void* context, void* grad, void* bias_grad, uint32_t rows,
                                   uint32_t width, bool accumulate);
/* tensor.rs:94-103 add_in_place: dst = dst + src */
bool tysor_cuda_dispatch_add_inplace(void* context, void* dst, void* src, uint64_t count);
/* training/executor.rs:745-762: p -= (float)lr * g */
bool tysor_cuda_dispatch_sgd_update(void* context, void* param, void* grad, uint64_t count,
                                    double lr);
/* training/executor.rs:109-111: sum of all elements into out[0] */
bool tysor_cuda_dispatch_reduce_sum(void* context, void* input, void* out, uint64_t count);

/* Extensions (no reference counterpart). */
/* RMSNorm with gain g[width] and eps: y = x * rsqrt(mean(x^2)+eps) * g */
bool tysor_cuda_dispatch_rms_norm_gain(void* context, void* input, void* gain, void* out,
                                       uint32_t rows, uint32_t width, float eps);
/* dx (+)= dy * g ; dgain (+)= sum_rows dy * x * rsqrt(mean(x^2)+eps) */
bool tysor_cuda_dispatch_rms_norm_gain_backward(void* context, void* input, void* gain, void* dy,
                                                void* dx, void* dgain, uint32_t rows,
                                                uint32_t width, float eps, bool accumulate);
/* Cross entropy against class labels stored as f32 ids: loss[r] */
bool tysor_cuda_dispatch_cross_entropy_labels(void* context, void* logits, void* labels,
                                              void* out, uint32_t rows, uint32_t width);
bool tysor_cuda_dispatch_cross_entropy_labels_backward(void* context, void* logits, void* labels,
                                                       void* grad, uint32_t rows, uint32_t width,
                                                       bool accumulate);
/* Exchange axes a and b of a row-major tensor of rank <= 8. */
bool tysor_cuda_dispatch_transpose(void* context, void* input, void* out, const int64_t* dims,
                                   int rank, int a, int b);

/* ---- device-resident graph executor -------------------------------------
 * Replaces the host interpreters (runtime/graph_executor.rs:249-356,
 * training/backward.rs:145-380, training/executor.rs:252-816) for one
 * graph: values stay on the device, buffers are planned once, every step
 * is a sequence of launches on the context stream. */

/* Parses the text form of a lowered graph (tysor_b200/graph.py). */
void* tysor_cuda_graph_new(void* context, const char* graph_text);
void tysor_cuda_graph_free(void* graph);
/* --shape name=AxB (main.rs:98-120) */
bool tysor_cuda_graph_set_shape(void* graph, const char* name, const int64_t* dims, int rank);
/* Optional: explicit input values instead of the pattern input
 * (tensor.rs:24-34).  Copied at the next run. */
bool tysor_cuda_graph_set_input(void* graph, const char* name, const float* data, size_t count);
/* Copies `count` floats from host memory (pinned memory makes it
 * asynchronous) straight into the device buffer of graph input `name`,
 * enqueued on the context stream; the input keeps that value for later
 * runs.  The graph must have been run, backpropagated or trained once so
 * that its buffers are planned. */
bool tysor_cuda_graph_upload_input(void* graph, const char* name, const float* data,
                                   size_t count);
/* Queues `count` floats from host memory (pinned memory makes the copy
 * asynchronous) as the next value of graph input `name`: the copy runs on
 * a separate copy stream into one of two device staging buffers, so it
 * overlaps kernels already queued, and the next run / backward / train call
 * copies the oldest queued value into the input's buffer before its first
 * step.  At most two values per input may wait.  The graph must have been
 * run, backpropagated or trained once.  (Prefetching the next step's inputs
 * the way a data loader does; the reference reads inputs once, at startup:
 * tensor.rs:24-34.) */
bool tysor_cuda_graph_prefetch_input(void* graph, const char* name, const float* data,
                                     size_t count);
/* Optional: initial value of a trainable parameter (e.g. "linear_5_weight")
 * instead of its pattern initialiser (layers.rs:39-75). */
bool tysor_cuda_graph_set_parameter(void* graph, const char* name, const float* data,
                                    size_t count);
/* --run: forward with pattern weights (graph_executor.rs). */
bool tysor_cuda_graph_run(void* graph);
/* --backward: forward + value gradients (backward.rs:145-380). */
bool tysor_cuda_graph_backward(void* graph);
/* --train: `iterations` SGD steps (executor.rs:764-816); losses[i] receives
 * the summed objective of step i (may be NULL). */
bool tysor_cuda_graph_train(void* graph, int iterations, double lr, float* losses);
/* The same steps enqueued on the context stream without waiting: each
 * step's loss is copied to host_losses[i] on the stream (pinned host memory
 * keeps the copies asynchronous; NULL: not copied), valid once
 * tysor_cuda_synchronize returns, which also reports any error a step's
 * kernels recorded.  A trainer that prefetches its next inputs
 * (tysor_cuda_graph_prefetch_input) and enqueues its next step while this
 * one runs keeps the device busy between steps.  Extension: the reference
 * trains synchronously (executor.rs:764-816). */
bool tysor_cuda_graph_train_enqueue(void* graph, int iterations, double lr, float* host_losses);
/* Extension (no reference counterpart): one train step launched op by op
 * with a CUDA event after each planned step item (forward, backward, update
 * order); item_ms[i] (i < capacity) receives item i's device time and
 * *n_items the item count.  A profiling aid: the step is not captured. */
bool tysor_cuda_graph_train_traced(void* graph, double lr, float* item_ms, int capacity,
                                   int* n_items);
/* Extension: label of traced item `item` ("fwd <op> #<value>", "bwd ...",
 * "update ..."), valid until the next traced step; NULL if out of range. */
const char* tysor_cuda_graph_trace_label(void* graph, int item);
/* Shape and value of any tensor value by id after a run. */
int tysor_cuda_graph_value_rank(void* graph, int value_id);
bool tysor_cuda_graph_value_shape(void* graph, int value_id, int64_t* dims);
bool tysor_cuda_graph_read_value(void* graph, int value_id, float* out, size_t count);
/* Gradient of a value after tysor_cuda_graph_backward (false if none).
 * After tysor_cuda_graph_train only graph parameters' gradients are
 * defined: training hands an intermediate value's dead gradient buffer on
 * to one of its inputs, which adds its own gradient into it. */
bool tysor_cuda_graph_read_value_grad(void* graph, int value_id, float* out, size_t count);
/* Trainable parameters after tysor_cuda_graph_train. */
int tysor_cuda_graph_num_parameters(void* graph);
const char* tysor_cuda_graph_parameter_name(void* graph, int index);
size_t tysor_cuda_graph_parameter_count(void* graph, const char* name);
bool tysor_cuda_graph_read_parameter(void* graph, const char* name, float* out, size_t count);
bool tysor_cuda_graph_read_parameter_grad(void* graph, const char* name, float* out,
                                          size_t count);
/* Number of kernel launches the last run/backward/train step enqueued. */
int64_t tysor_cuda_graph_launch_count(void* graph);
/* Capture one train step in a CUDA graph and replay it for later steps
 * (default on for train). */
bool tysor_cuda_graph_set_capture(void* graph, bool enable);
/* How a train step sums its objective into the loss.  0 (default): a
 * parallel tree sum in f32, typically closer to the exact sum.  1: the
 * reference's tensor_sum (training/executor.rs:109-111), one f32 accumulator
 * in index order, which reproduces the reference's rounding (over millions
 * of terms it can drift by 1e-3..1e-2 from the exact sum) at the cost of one
 * thread walking the objective (about 70 ms per 33.5M elements).  The loss
 * does not feed the gradients, so training is the same either way. */
bool tysor_cuda_graph_set_loss_order(void* graph, int order);

/* ---- matmul without allocation ---------------------------------------------
 * No counterpart in the reference.  For callers that must not allocate
 * device memory (code running inside another framework's reserved memory
 * pool, or a hot path where cudaMalloc's implicit synchronisation is not
 * allowed): C[m,n] = A[m,k] . B[k,n], row-major fp32 device pointers, strict
 * 3xTF32, enqueued on `stream` (a cudaStream_t; NULL = default stream).  It
 * needs no context and allocates nothing: the split operands live in a fixed
 * 32 MiB device array inside the library, so A and B together may span at
 * most 8,388,608 elements (larger calls fail with an error).  The runtime
 * claims those 32 MiB on a device when it loads the library's module there:
 * at the first call on that device under CUDA's default lazy module loading,
 * or when the process initialises the device with CUDA_MODULE_LOADING=EAGER.
 * A caller that reserves most of the GPU's memory for its own pool should
 * make the first call before reserving it.  The first call on each device
 * also looks up that array's address; make it before any stream capture.
 * All calls on a device share the array, so calls that overlap on the GPU
 * race; order them on one stream.  The call only enqueues the work: a
 * kernel-side failure is recorded on the device and reported by
 * tysor_cuda_matmul_noalloc_status. */
bool tysor_cuda_matmul_noalloc(void* stream, uint32_t m, uint32_t n, uint32_t k, const float* a,
                               const float* b, float* c);
/* Companion of tysor_cuda_matmul_noalloc (no counterpart in the reference):
 * waits for `stream`, then reads and clears the current device's no-alloc
 * error word.  False (with tysor_cuda_last_error naming the failure, e.g. a
 * tensor-core pipeline wait that timed out) if a call since the last check
 * recorded one; its output is then incomplete.  Allocates nothing. */
bool tysor_cuda_matmul_noalloc_status(void* stream);

/* ---- data-parallel gradient all-reduce (NCCL over NVLink) ----------------
 * No reference counterpart: the reference has no multi-device code. */
bool tysor_cuda_nccl_get_unique_id(uint8_t out_id[128]);
/* Non-blocking init with a deadline; aborts the communicator on timeout. */
bool tysor_cuda_comm_init(void* context, int nranks, int rank, const uint8_t id[128],
                          int timeout_ms);
bool tysor_cuda_comm_free(void* context);
/* In-place sum all-reduce of `count` floats on the context stream. */
bool tysor_cuda_allreduce_sum(void* context, void* buffer, uint64_t count);
/* Attach the context's communicator to a graph: train steps all-reduce the
 * parameter gradients (sum) and the loss before the update. */
bool tysor_cuda_graph_enable_allreduce(void* graph, bool enable);

#ifdef __cplusplus
}
#endif

#endif /* TYSOR_CUDA_H */
