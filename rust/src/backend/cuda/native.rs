//! FFI binding of libtysor_cuda (the C ABI declared in include/tysor_cuda.h),
//! the CUDA counterpart of the Metal bridge's `extern "C"` block
//! (src/backend/metal/native.rs:14-136).
//!
//! Conventions carried over from the Metal bridge: opaque `*mut c_void`
//! handles, fp32 element counts, `bool` (or NULL) returns with the message in
//! the thread-local `tysor_cuda_last_error()` (native.rs:148-157), and RAII
//! owners whose `Drop` frees the handle (native.rs:322-347).  The library is
//! only linked when build.rs found nvcc and set `cfg(tysor_cuda)`.
//!
//! `graph_text` serialises a `GraphFunction` (src/ir/graph.rs:6-45) into the
//! line format `tysor_cuda_graph_new` parses: one `value` line per value in
//! id order, one `node` line per node, then the outputs, the objective and
//! `end`.

#![allow(dead_code)]

use crate::compiler::frontend_ir::{FeTypeKind, FeValue};
use crate::compiler::lexer::TokenType;
use crate::ir::graph::{GraphFunction, GraphNodeKind};

/// Every function of include/tysor_cuda.h, same names, order and C types.
#[cfg(tysor_cuda)]
pub mod ffi {
    use std::os::raw::{c_char, c_int, c_void};

    #[link(name = "tysor_cuda")]
    unsafe extern "C" {
        pub fn tysor_cuda_last_error() -> *const c_char;
        pub fn tysor_cuda_context_new(device: c_int) -> *mut c_void;
        pub fn tysor_cuda_context_free(context: *mut c_void);
        pub fn tysor_cuda_synchronize(context: *mut c_void) -> bool;
        pub fn tysor_cuda_set_matmul_mode(context: *mut c_void, mode: c_int) -> bool;
        pub fn tysor_cuda_set_matmul_accumulation(context: *mut c_void, kblocks: c_int) -> bool;
        pub fn tysor_cuda_probe_wait_timeout(context: *mut c_void, limit_cycles: i64) -> bool;
        pub fn tysor_cuda_context_stream(context: *mut c_void) -> *mut c_void;
        pub fn tysor_cuda_buffer_new_with_data(context: *mut c_void, data: *const f32, count: usize) -> *mut c_void;
        pub fn tysor_cuda_buffer_new_zeroed(context: *mut c_void, count: usize) -> *mut c_void;
        pub fn tysor_cuda_buffer_free(buffer: *mut c_void);
        pub fn tysor_cuda_buffer_read(buffer: *mut c_void, out_data: *mut f32, count: usize) -> bool;
        pub fn tysor_cuda_buffer_write(buffer: *mut c_void, data: *const f32, count: usize) -> bool;
        pub fn tysor_cuda_buffer_view(base: *mut c_void, offset: usize, count: usize) -> *mut c_void;
        pub fn tysor_cuda_buffer_count(buffer: *mut c_void) -> usize;
        pub fn tysor_cuda_dispatch_matmul(context: *mut c_void, lhs: *mut c_void, rhs: *mut c_void, out: *mut c_void, m: u32, n: u32, k: u32) -> bool;
        pub fn tysor_cuda_dispatch_unary(context: *mut c_void, op: c_int, input: *mut c_void, out: *mut c_void, count: u32, param: f32) -> bool;
        pub fn tysor_cuda_dispatch_binary_tt(context: *mut c_void, op: c_int, lhs: *mut c_void, rhs: *mut c_void, out: *mut c_void, count: u32) -> bool;
        pub fn tysor_cuda_dispatch_binary_ts(context: *mut c_void, op: c_int, input: *mut c_void, out: *mut c_void, count: u32, scalar: f64) -> bool;
        pub fn tysor_cuda_dispatch_binary_st(context: *mut c_void, op: c_int, input: *mut c_void, out: *mut c_void, count: u32, scalar: f64) -> bool;
        pub fn tysor_cuda_dispatch_rms_norm(context: *mut c_void, input: *mut c_void, out: *mut c_void, rows: u32, width: u32) -> bool;
        pub fn tysor_cuda_dispatch_softmax(context: *mut c_void, input: *mut c_void, out: *mut c_void, rows: u32, width: u32) -> bool;
        pub fn tysor_cuda_dispatch_cross_entropy(context: *mut c_void, logits: *mut c_void, target: *mut c_void, out: *mut c_void, rows: u32, width: u32) -> bool;
        pub fn tysor_cuda_dispatch_linear(context: *mut c_void, input: *mut c_void, weight: *mut c_void, bias: *mut c_void, out: *mut c_void, m: u32, n: u32, k: u32, with_bias: bool) -> bool;
        pub fn tysor_cuda_dispatch_embedding(context: *mut c_void, indices: *mut c_void, weight: *mut c_void, out: *mut c_void, index_count: u32, embedding_dim: u32, num_embeddings: u32) -> bool;
        pub fn tysor_cuda_dispatch_repeat_kv(context: *mut c_void, input: *mut c_void, out: *mut c_void, outer: u32, out_heads: u32, inner: u32, repeats: u32) -> bool;
        pub fn tysor_cuda_dispatch_causal_mask(context: *mut c_void, input: *mut c_void, out: *mut c_void, outer: u32, q: u32, k: u32) -> bool;
        pub fn tysor_cuda_dispatch_rope(context: *mut c_void, input: *mut c_void, out: *mut c_void, outer: u32, seq_len: u32, half_dim: u32, theta: f64) -> bool;
        pub fn tysor_cuda_dispatch_matmul_ex(context: *mut c_void, batch: u32, m: u32, n: u32, k: u32, a: *mut c_void, trans_a: bool, lda: u64, stride_a: u64, b: *mut c_void, trans_b: bool, ldb: u64, stride_b: u64, c: *mut c_void, ldc: u64, stride_c: u64, bias: *mut c_void, alpha: f32, accumulate: bool, relu: bool) -> bool;
        pub fn tysor_cuda_dispatch_relu_backward(context: *mut c_void, out_act: *mut c_void, grad: *mut c_void, dx: *mut c_void, count: u64, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_silu_backward(context: *mut c_void, input: *mut c_void, grad: *mut c_void, dx: *mut c_void, count: u64, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_softmax_backward(context: *mut c_void, output: *mut c_void, grad: *mut c_void, dx: *mut c_void, count: u64, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_cross_entropy_backward(context: *mut c_void, logits: *mut c_void, target: *mut c_void, grad: *mut c_void, rows: u32, width: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_rope_backward(context: *mut c_void, grad: *mut c_void, dx: *mut c_void, outer: u32, seq_len: u32, half_dim: u32, theta: f64, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_repeat_kv_backward(context: *mut c_void, grad: *mut c_void, dx: *mut c_void, outer: u32, heads: u32, inner: u32, repeats: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_causal_mask_backward(context: *mut c_void, grad: *mut c_void, dx: *mut c_void, outer: u32, q: u32, k: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_embedding_backward(context: *mut c_void, grad: *mut c_void, indices: *mut c_void, weight_grad: *mut c_void, index_count: u32, embedding_dim: u32, num_embeddings: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_bias_grad(context: *mut c_void, grad: *mut c_void, bias_grad: *mut c_void, rows: u32, width: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_add_inplace(context: *mut c_void, dst: *mut c_void, src: *mut c_void, count: u64) -> bool;
        pub fn tysor_cuda_dispatch_sgd_update(context: *mut c_void, param: *mut c_void, grad: *mut c_void, count: u64, lr: f64) -> bool;
        pub fn tysor_cuda_dispatch_reduce_sum(context: *mut c_void, input: *mut c_void, out: *mut c_void, count: u64) -> bool;
        pub fn tysor_cuda_dispatch_rms_norm_gain(context: *mut c_void, input: *mut c_void, gain: *mut c_void, out: *mut c_void, rows: u32, width: u32, eps: f32) -> bool;
        pub fn tysor_cuda_dispatch_rms_norm_gain_backward(context: *mut c_void, input: *mut c_void, gain: *mut c_void, dy: *mut c_void, dx: *mut c_void, dgain: *mut c_void, rows: u32, width: u32, eps: f32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_cross_entropy_labels(context: *mut c_void, logits: *mut c_void, labels: *mut c_void, out: *mut c_void, rows: u32, width: u32) -> bool;
        pub fn tysor_cuda_dispatch_cross_entropy_labels_backward(context: *mut c_void, logits: *mut c_void, labels: *mut c_void, grad: *mut c_void, rows: u32, width: u32, accumulate: bool) -> bool;
        pub fn tysor_cuda_dispatch_transpose(context: *mut c_void, input: *mut c_void, out: *mut c_void, dims: *const i64, rank: c_int, a: c_int, b: c_int) -> bool;
        pub fn tysor_cuda_graph_new(context: *mut c_void, graph_text: *const c_char) -> *mut c_void;
        pub fn tysor_cuda_graph_free(graph: *mut c_void);
        pub fn tysor_cuda_graph_set_shape(graph: *mut c_void, name: *const c_char, dims: *const i64, rank: c_int) -> bool;
        pub fn tysor_cuda_graph_set_input(graph: *mut c_void, name: *const c_char, data: *const f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_upload_input(graph: *mut c_void, name: *const c_char, data: *const f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_prefetch_input(graph: *mut c_void, name: *const c_char, data: *const f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_set_parameter(graph: *mut c_void, name: *const c_char, data: *const f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_run(graph: *mut c_void) -> bool;
        pub fn tysor_cuda_graph_backward(graph: *mut c_void) -> bool;
        pub fn tysor_cuda_graph_train(graph: *mut c_void, iterations: c_int, lr: f64, losses: *mut f32) -> bool;
        pub fn tysor_cuda_graph_train_enqueue(graph: *mut c_void, iterations: c_int, lr: f64, host_losses: *mut f32) -> bool;
        pub fn tysor_cuda_graph_train_traced(graph: *mut c_void, lr: f64, item_ms: *mut f32, capacity: c_int, n_items: *mut c_int) -> bool;
        pub fn tysor_cuda_graph_trace_label(graph: *mut c_void, item: c_int) -> *const c_char;
        pub fn tysor_cuda_graph_value_rank(graph: *mut c_void, value_id: c_int) -> c_int;
        pub fn tysor_cuda_graph_value_shape(graph: *mut c_void, value_id: c_int, dims: *mut i64) -> bool;
        pub fn tysor_cuda_graph_read_value(graph: *mut c_void, value_id: c_int, out: *mut f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_read_value_grad(graph: *mut c_void, value_id: c_int, out: *mut f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_num_parameters(graph: *mut c_void) -> c_int;
        pub fn tysor_cuda_graph_parameter_name(graph: *mut c_void, index: c_int) -> *const c_char;
        pub fn tysor_cuda_graph_parameter_count(graph: *mut c_void, name: *const c_char) -> usize;
        pub fn tysor_cuda_graph_read_parameter(graph: *mut c_void, name: *const c_char, out: *mut f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_read_parameter_grad(graph: *mut c_void, name: *const c_char, out: *mut f32, count: usize) -> bool;
        pub fn tysor_cuda_graph_launch_count(graph: *mut c_void) -> i64;
        pub fn tysor_cuda_graph_set_capture(graph: *mut c_void, enable: bool) -> bool;
        pub fn tysor_cuda_graph_set_loss_order(graph: *mut c_void, order: c_int) -> bool;
        pub fn tysor_cuda_matmul_noalloc(stream: *mut c_void, m: u32, n: u32, k: u32, a: *const f32, b: *const f32, c: *mut f32) -> bool;
        pub fn tysor_cuda_matmul_noalloc_status(stream: *mut c_void) -> bool;
        pub fn tysor_cuda_nccl_get_unique_id(out_id: *mut u8) -> bool;
        pub fn tysor_cuda_comm_init(context: *mut c_void, nranks: c_int, rank: c_int, id: *const u8, timeout_ms: c_int) -> bool;
        pub fn tysor_cuda_comm_free(context: *mut c_void) -> bool;
        pub fn tysor_cuda_allreduce_sum(context: *mut c_void, buffer: *mut c_void, count: u64) -> bool;
        pub fn tysor_cuda_graph_enable_allreduce(graph: *mut c_void, enable: bool) -> bool;
    }
}

/// The graph's text form for `tysor_cuda_graph_new`; `objective` is the value
/// whose sum training minimises and whose gradient seed backward uses
/// (training/executor.rs:528-543, training/backward.rs:115-133).
pub fn graph_text(graph: &GraphFunction, objective: usize) -> Result<String, String> {
    let mut out = format!("graph {}\n", if graph.name.is_empty() { "model" } else { &graph.name });
    for value in &graph.values {
        let kind = match value.ty.kind {
            FeTypeKind::Tensor => "tensor",
            FeTypeKind::Int => "int",
            FeTypeKind::Float => "float",
            FeTypeKind::Bool => "bool",
            _ => "callable",
        };
        let name = if value.name.is_empty() || value.name.contains(char::is_whitespace) {
            "-"
        } else {
            value.name.as_str()
        };
        out.push_str(&format!("value {} {} {} {}\n", value.id, kind, value.is_parameter as i32, name));
    }
    for node in &graph.nodes {
        let inputs = node.inputs.iter().map(|id| id.to_string()).collect::<Vec<_>>().join(" ");
        let line = match node.kind {
            GraphNodeKind::Constant => match &node.constant {
                FeValue::Int(v) => format!("node const {} int {}", node.output, v),
                FeValue::Float(v) => format!("node const {} float {:e}", node.output, v),
                FeValue::Bool(v) => format!("node const {} bool {}", node.output, *v as i32),
                other => return Err(format!("CUDA backend cannot pass constant {other:?} to the device graph")),
            },
            GraphNodeKind::Binary => {
                let op = match node.binary_op {
                    TokenType::Plus => "+",
                    TokenType::Minus => "-",
                    TokenType::Star => "*",
                    TokenType::Slash => "/",
                    other => return Err(format!("Unsupported binary operator {} in CUDA graph", other.as_str())),
                };
                format!("node binary {} {} {}", node.output, op, inputs)
            }
            GraphNodeKind::PrimitiveCall => format!("node primitive {} {} {}", node.output, node.op, inputs),
            GraphNodeKind::LibraryCall => format!("node call {} {} {}", node.output, node.op, inputs),
            GraphNodeKind::LibraryCtor => format!("node ctor {} {} {}", node.output, node.op, inputs),
            GraphNodeKind::Apply => format!("node apply {} {}", node.output, inputs),
        };
        out.push_str(line.trim_end());
        out.push('\n');
    }
    for output in &graph.outputs {
        out.push_str(&format!("output {output}\n"));
    }
    out.push_str(&format!("objective {objective}\nend\n"));
    Ok(out)
}

#[cfg(tysor_cuda)]
pub use owners::{last_error, Context, Graph};

#[cfg(tysor_cuda)]
mod owners {
    use super::ffi;
    use std::ffi::{CStr, CString};
    use std::marker::PhantomData;
    use std::os::raw::{c_int, c_void};

    /// tysor_cuda_last_error() as a String (native.rs:148-157).
    pub fn last_error() -> String {
        unsafe {
            let ptr = ffi::tysor_cuda_last_error();
            if ptr.is_null() {
                "unknown tysor_cuda error".to_string()
            } else {
                CStr::from_ptr(ptr).to_string_lossy().into_owned()
            }
        }
    }

    fn check(ok: bool, what: &str) -> Result<(), String> {
        if ok {
            Ok(())
        } else {
            Err(format!("{what}: {}", last_error()))
        }
    }

    fn c_string(text: &str) -> Result<CString, String> {
        CString::new(text).map_err(|_| format!("'{text}' contains a NUL byte"))
    }

    /// Selects the matmul engine of new contexts: `strict` (3xTF32, the
    /// default), `strict16` (the same three products over scaled fp16
    /// halves), `fast` (1xTF32) or `exact` (CUDA cores in k order).
    pub const MATMUL_ENV: &str = "TYSOR_CUDA_MATMUL";

    /// A CUDA context (device, stream, error word) owned by Rust.
    pub struct Context(*mut c_void);

    impl Context {
        pub fn new(device: i32) -> Result<Self, String> {
            let ptr = unsafe { ffi::tysor_cuda_context_new(device as c_int) };
            if ptr.is_null() {
                return Err(format!("CUDA context on device {device}: {}", last_error()));
            }
            let context = Context(ptr);
            if let Ok(mode) = std::env::var(MATMUL_ENV) {
                let code: c_int = match mode.as_str() {
                    "strict" => 0,
                    "fast" => 1,
                    "exact" => 2,
                    "strict16" => 3,
                    other => {
                        return Err(format!("{MATMUL_ENV}={other}: expected strict, strict16, fast or exact"))
                    }
                };
                if !unsafe { ffi::tysor_cuda_set_matmul_mode(context.0, code) } {
                    return Err(format!("{MATMUL_ENV}: {}", last_error()));
                }
            }
            Ok(context)
        }

        pub fn raw(&self) -> *mut c_void {
            self.0
        }
    }

    impl Drop for Context {
        fn drop(&mut self) {
            if !self.0.is_null() {
                unsafe { ffi::tysor_cuda_context_free(self.0) };
            }
        }
    }

    /// One lowered graph planned on a context; dropped before its context.
    pub struct Graph<'a> {
        ptr: *mut c_void,
        _context: PhantomData<&'a Context>,
    }

    impl<'a> Graph<'a> {
        pub fn new(context: &'a Context, text: &str) -> Result<Self, String> {
            let text = c_string(text)?;
            let ptr = unsafe { ffi::tysor_cuda_graph_new(context.raw(), text.as_ptr()) };
            if ptr.is_null() {
                return Err(format!("graph_new: {}", last_error()));
            }
            Ok(Graph { ptr, _context: PhantomData })
        }

        pub fn set_shape(&self, name: &str, dims: &[i64]) -> Result<(), String> {
            let name = c_string(name)?;
            check(
                unsafe { ffi::tysor_cuda_graph_set_shape(self.ptr, name.as_ptr(), dims.as_ptr(), dims.len() as c_int) },
                "set_shape",
            )
        }

        pub fn run(&self) -> Result<(), String> {
            check(unsafe { ffi::tysor_cuda_graph_run(self.ptr) }, "run")
        }

        pub fn backward(&self) -> Result<(), String> {
            check(unsafe { ffi::tysor_cuda_graph_backward(self.ptr) }, "backward")
        }

        /// `iterations` SGD steps on the device; the summed objective of each.
        pub fn train(&self, iterations: usize, learning_rate: f64) -> Result<Vec<f32>, String> {
            let mut losses = vec![0.0f32; iterations.max(1)];
            check(
                unsafe { ffi::tysor_cuda_graph_train(self.ptr, iterations as c_int, learning_rate, losses.as_mut_ptr()) },
                "train",
            )?;
            losses.truncate(iterations);
            Ok(losses)
        }

        pub fn shape(&self, value_id: usize) -> Result<Vec<i64>, String> {
            let rank = unsafe { ffi::tysor_cuda_graph_value_rank(self.ptr, value_id as c_int) };
            if rank < 0 {
                return Err(format!("value_rank: {}", last_error()));
            }
            let mut dims = vec![0i64; (rank as usize).max(1)];
            check(
                unsafe { ffi::tysor_cuda_graph_value_shape(self.ptr, value_id as c_int, dims.as_mut_ptr()) },
                "value_shape",
            )?;
            dims.truncate(rank as usize);
            Ok(dims)
        }

        fn count(dims: &[i64]) -> usize {
            dims.iter().product::<i64>().max(0) as usize
        }

        /// Shape and values of a tensor value after run / backward / train.
        pub fn value(&self, value_id: usize) -> Result<(Vec<i64>, Vec<f32>), String> {
            let dims = self.shape(value_id)?;
            let mut data = vec![0.0f32; Self::count(&dims)];
            check(
                unsafe { ffi::tysor_cuda_graph_read_value(self.ptr, value_id as c_int, data.as_mut_ptr(), data.len()) },
                "read_value",
            )?;
            Ok((dims, data))
        }

        /// The gradient of a value after backward; None when it has none.
        pub fn value_grad(&self, value_id: usize) -> Result<Option<Vec<f32>>, String> {
            let dims = self.shape(value_id)?;
            let mut data = vec![0.0f32; Self::count(&dims)];
            let ok = unsafe {
                ffi::tysor_cuda_graph_read_value_grad(self.ptr, value_id as c_int, data.as_mut_ptr(), data.len())
            };
            Ok(if ok { Some(data) } else { None })
        }

        pub fn num_parameters(&self) -> Result<usize, String> {
            let n = unsafe { ffi::tysor_cuda_graph_num_parameters(self.ptr) };
            if n < 0 {
                Err(format!("num_parameters: {}", last_error()))
            } else {
                Ok(n as usize)
            }
        }
    }

    impl Drop for Graph<'_> {
        fn drop(&mut self) {
            if !self.ptr.is_null() {
                unsafe { ffi::tysor_cuda_graph_free(self.ptr) };
            }
        }
    }
}
