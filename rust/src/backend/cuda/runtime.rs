//! `--backend cuda` entry points: `--run`, `--backward` and `--train` through
//! libtysor_cuda's device-resident graph executor.
//!
//! The reference's non-local backends run only the forward pass on the device
//! and hand every value back to the shared Rust reverse walk and SGD
//! (training/backward.rs:145-380, training/executor.rs:563-816).  Here the
//! whole step stays on the device: the lowered graph is handed to the library
//! once (`tysor_cuda_graph_new`), which plans its buffers, runs the forward,
//! the same reverse walk (value gradients for `--backward`, parameter
//! gradients for `--train`) and the update, and only what is printed comes
//! back.  The printed text is the reference's: `print_tensor`
//! (runtime/tensor.rs:36-69), the gradient section of backward.rs:382-399 and
//! the training section of executor.rs:794-814.
//!
//! There is no fallback: without a device (or without the library, when nvcc
//! was missing at build time) every entry point returns an error, the policy
//! TYSOR_METAL_REQUIRE_NATIVE=1 sets for Metal (metal/runtime.rs:347-360).
//! `TYSOR_CUDA_DEVICE` picks the device ordinal (default 0), `TYSOR_CUDA_MATMUL`
//! the matmul engine (native.rs::MATMUL_ENV).

#![cfg_attr(not(tysor_cuda), allow(dead_code, unused_imports))]

use std::collections::BTreeMap;

use crate::compiler::frontend_ir::{FeExecutionRun, FeFunction, FeTypeKind, FeValue, LoweredModule};
use crate::ir::builder::build_graph_function;
use crate::ir::graph::{GraphFunction, GraphNodeKind};
use crate::runtime::interpreter::RuntimeRunOptions;
use crate::training::backward::BackwardRunOptions;
use crate::training::executor::TrainRunOptions;

#[cfg(tysor_cuda)]
use super::native::{graph_text, Context, Graph};
#[cfg(tysor_cuda)]
use crate::runtime::tensor::{print_named_tensor, print_tensor, SimpleTensor};

const DEVICE_ENV: &str = "TYSOR_CUDA_DEVICE";

fn find_entry_function<'a>(lowered: &'a LoweredModule, entry: &str) -> Result<&'a FeFunction, String> {
    lowered
        .functions
        .iter()
        .find(|function| function.name == entry)
        .ok_or_else(|| format!("Entry function '{}' not found in lowered module", entry))
}

fn find_run<'a>(lowered: &'a LoweredModule, entry: &str) -> Option<&'a FeExecutionRun> {
    lowered
        .execution_plan
        .as_ref()
        .and_then(|plan| plan.runs.iter().find(|run| run.model_name == entry))
}

/// The `train model:` objective if one is named, else the first output
/// (training/backward.rs:115-133, training/executor.rs:528-543).
fn objective_id(run: Option<&FeExecutionRun>, graph: &GraphFunction) -> Result<usize, String> {
    if let Some(symbol) = run.and_then(|run| run.objective_symbol.as_ref()) {
        return graph
            .named_values
            .get(symbol)
            .copied()
            .ok_or_else(|| format!("Could not resolve objective '{}' in graph", symbol));
    }
    graph.outputs
        .first()
        .copied()
        .ok_or_else(|| "Entry function did not return a value".to_string())
}

/// The dtype string each tensor value carries in the reference's local
/// executor: a parameter its annotation (graph_executor.rs:90-93); an
/// embedding lookup its constructor's declared return dtype
/// (graph_executor.rs:208-213, layers.rs:147); `scalar op tensor` the
/// tensor's (tensor.rs:149); every other op its first tensor operand's
/// (tensor.rs:121-258, layers.rs:127-322).  The device computes in fp32
/// whatever the string says, as the reference does.
fn value_dtypes(graph: &GraphFunction) -> BTreeMap<usize, String> {
    let mut dtypes: BTreeMap<usize, String> = BTreeMap::new();
    let mut ctor_dtypes: BTreeMap<usize, (String, String)> = BTreeMap::new();
    for value in &graph.values {
        if value.is_parameter && value.ty.kind == FeTypeKind::Tensor {
            dtypes.insert(value.id, value.ty.tensor_dtype.clone().unwrap_or_else(|| "float32".to_string()));
        }
    }
    for node in &graph.nodes {
        let first_tensor = node.inputs.iter().find_map(|id| dtypes.get(id).cloned());
        let dtype = match node.kind {
            GraphNodeKind::Constant => None,
            GraphNodeKind::LibraryCtor => {
                let declared = graph.values[node.output]
                    .ty
                    .callable_return
                    .as_deref()
                    .and_then(|ty| ty.tensor_dtype.clone())
                    .unwrap_or_else(|| "float32".to_string());
                ctor_dtypes.insert(node.output, (node.op.clone(), declared));
                None
            }
            GraphNodeKind::Apply => match node.inputs.first().and_then(|callee| ctor_dtypes.get(callee)) {
                Some((op, declared)) if op == "Embedding" => Some(declared.clone()),
                _ => node.inputs.get(1).and_then(|id| dtypes.get(id).cloned()),
            },
            GraphNodeKind::Binary => {
                let lhs = node.inputs.first().and_then(|id| dtypes.get(id).cloned());
                let rhs = node.inputs.get(1).and_then(|id| dtypes.get(id).cloned());
                lhs.or(rhs)
            }
            GraphNodeKind::PrimitiveCall | GraphNodeKind::LibraryCall => first_tensor,
        };
        if let Some(dtype) = dtype {
            dtypes.insert(node.output, dtype);
        }
    }
    dtypes
}

fn number(value: &Option<FeValue>) -> Option<f64> {
    match value {
        Some(FeValue::Float(v)) => Some(*v),
        Some(FeValue::Int(v)) => Some(*v as f64),
        _ => None,
    }
}

#[cfg(tysor_cuda)]
fn device() -> i32 {
    std::env::var(DEVICE_ENV).ok().and_then(|v| v.trim().parse().ok()).unwrap_or(0)
}

/// Builds the entry's graph on a fresh context with every `--shape` applied.
#[cfg(tysor_cuda)]
fn planned<'c>(
    context: &'c Context,
    graph: &GraphFunction,
    objective: usize,
    shapes: &BTreeMap<String, Vec<i64>>,
) -> Result<Graph<'c>, String> {
    let device_graph = Graph::new(context, &graph_text(graph, objective)?)?;
    for (name, dims) in shapes {
        device_graph.set_shape(name, dims)?;
    }
    Ok(device_graph)
}

/// `tysor f.ty --run --backend cuda` (main.rs:269-283).
#[cfg(tysor_cuda)]
pub fn run_cuda_module(lowered: &LoweredModule, options: &RuntimeRunOptions) -> Result<(), String> {
    let graph = build_graph_function(find_entry_function(lowered, &options.entry)?)?;
    if graph.outputs.is_empty() {
        return Err("Entry function did not return a value".to_string());
    }
    if graph.outputs.len() != 1 {
        return Err("Runtime interpreter currently supports a single return value".to_string());
    }
    let output = graph.outputs[0];
    let context = Context::new(device())?;
    let device_graph = planned(&context, &graph, output, &options.tensor_shapes)?;
    device_graph.run()?;
    let (shape, data) = device_graph.value(output)?;
    let dtype = value_dtypes(&graph).remove(&output).unwrap_or_else(|| "float32".to_string());
    print_tensor(&SimpleTensor { shape, data, dtype });
    Ok(())
}

/// `tysor f.ty --backward --backend cuda` (backward.rs:382-399): the gradient
/// of every graph parameter, zeros for a parameter the objective does not
/// reach.  Gradients carry the objective's dtype (the ones seed's,
/// backward.rs:178, which every backward helper passes on).
#[cfg(tysor_cuda)]
pub fn run_cuda_backward_module(lowered: &LoweredModule, options: &BackwardRunOptions) -> Result<(), String> {
    let graph = build_graph_function(find_entry_function(lowered, &options.entry)?)?;
    let objective = objective_id(find_run(lowered, &options.entry), &graph)?;
    let context = Context::new(device())?;
    let device_graph = planned(&context, &graph, objective, &options.tensor_shapes)?;
    device_graph.backward()?;
    let dtypes = value_dtypes(&graph);
    let grad_dtype = dtypes.get(&objective).cloned().unwrap_or_else(|| "float32".to_string());
    println!("\n--- Gradient Output ---");
    for value in &graph.values {
        if !value.is_parameter || value.ty.kind != FeTypeKind::Tensor {
            continue;
        }
        let shape = device_graph.shape(value.id)?;
        let (data, dtype) = match device_graph.value_grad(value.id)? {
            Some(data) => (data, grad_dtype.clone()),
            None => (
                vec![0.0; shape.iter().product::<i64>().max(0) as usize],
                dtypes.get(&value.id).cloned().unwrap_or_else(|| "float32".to_string()),
            ),
        };
        print_named_tensor(&format!("{}_grad", value.name), &SimpleTensor { shape, data, dtype });
    }
    println!("-----------------------");
    Ok(())
}

/// `tysor f.ty --train --backend cuda` (executor.rs:764-816): the same
/// `train model:` settings (sgd only, lr default 0.01, 1 iteration by
/// default), every step (forward, parameter gradients, SGD in parameter-name
/// order) on the device, and the same report.
#[cfg(tysor_cuda)]
pub fn run_cuda_train_module(lowered: &LoweredModule, options: &TrainRunOptions) -> Result<(), String> {
    let entry = find_entry_function(lowered, &options.entry)?;
    let run = find_run(lowered, &options.entry)
        .ok_or_else(|| "Train executor requires a resolved 'train model' execution run".to_string())?;
    let graph = build_graph_function(entry)?;
    let optimizer = match &run.optimizer {
        Some(FeValue::String(value)) => value.as_str(),
        _ => "sgd",
    };
    if optimizer != "sgd" {
        return Err("Train executor currently supports only optimizer='sgd'".to_string());
    }
    let learning_rate = number(&run.learning_rate).unwrap_or(0.01);
    let iterations = match &run.iteration {
        Some(FeValue::Int(value)) => (*value).max(0) as usize,
        _ => 1,
    };
    let objective = objective_id(Some(run), &graph)?;
    let context = Context::new(device())?;
    let device_graph = planned(&context, &graph, objective, &options.tensor_shapes)?;
    let losses = device_graph.train(iterations, learning_rate)?;
    let parameters = device_graph.num_parameters()?;
    println!("\n--- Training Output ---");
    println!("backend={}", options.backend.as_str());
    for (step, loss) in losses.iter().enumerate() {
        println!("step={} loss={:.6} params={}", step + 1, loss, parameters);
    }
    println!("-----------------------");
    Ok(())
}

#[cfg(not(tysor_cuda))]
fn not_built() -> String {
    format!(
        "CUDA backend is not available: libtysor_cuda was not built (nvcc was not found when tysor was compiled; \
         {DEVICE_ENV} selects the device once it is)"
    )
}

#[cfg(not(tysor_cuda))]
pub fn run_cuda_module(_lowered: &LoweredModule, _options: &RuntimeRunOptions) -> Result<(), String> {
    Err(not_built())
}

#[cfg(not(tysor_cuda))]
pub fn run_cuda_backward_module(_lowered: &LoweredModule, _options: &BackwardRunOptions) -> Result<(), String> {
    Err(not_built())
}

#[cfg(not(tysor_cuda))]
pub fn run_cuda_train_module(_lowered: &LoweredModule, _options: &TrainRunOptions) -> Result<(), String> {
    Err(not_built())
}
