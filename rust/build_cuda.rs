// Build step for `--backend cuda`, included by build.rs (`include!("build_cuda.rs")`)
// and called first thing in its `main`, before the macOS-only Metal block.
//
// It compiles libtysor_cuda from the CUDA sources of the tysor B200 backend
// for sm_100a and links the tysor binaries against it, the way the Metal
// block compiles native/metal_bridge.mm (build.rs:8-53).  Where the sources
// are: `TYSOR_CUDA_DIR` (a checkout of the backend, holding
// tysor_b200/csrc/*.cu and include/tysor_cuda.h), else native/cuda in this
// crate with the same two subfolders.  Where nvcc is: `NVCC`, else
// /usr/local/cuda/bin/nvcc, else `nvcc` on PATH.  Without nvcc or the
// sources nothing is built and `cfg(tysor_cuda)` stays off, so
// `--backend cuda` reports that the backend is not available.

fn build_cuda() {
    use std::path::PathBuf;
    use std::process::Command;

    println!("cargo:rustc-check-cfg=cfg(tysor_cuda)");
    println!("cargo:rerun-if-env-changed=TYSOR_CUDA_DIR");
    println!("cargo:rerun-if-env-changed=NVCC");

    let root = std::env::var("TYSOR_CUDA_DIR")
        .map(PathBuf::from)
        .unwrap_or_else(|_| PathBuf::from("native/cuda"));
    let csrc = root.join("tysor_b200").join("csrc");
    let include = root.join("include");
    if !csrc.is_dir() || !include.join("tysor_cuda.h").is_file() {
        println!("cargo:warning=tysor: CUDA sources not found under {}; --backend cuda disabled", root.display());
        return;
    }
    let nvcc = std::env::var("NVCC")
        .ok()
        .map(PathBuf::from)
        .or_else(|| Some(PathBuf::from("/usr/local/cuda/bin/nvcc")).filter(|p| p.is_file()))
        .unwrap_or_else(|| PathBuf::from("nvcc"));
    if Command::new(&nvcc).arg("--version").output().map(|o| !o.status.success()).unwrap_or(true) {
        println!("cargo:warning=tysor: nvcc not found; --backend cuda disabled");
        return;
    }
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", include.display());

    let out_dir = PathBuf::from(std::env::var("OUT_DIR").expect("OUT_DIR"));
    // The same units, flags and per-file options as the backend's own build
    // (tysor_b200/build.py): ops.cu rounds every product and sum separately.
    let units = ["gemm.cu", "ops.cu", "bridge.cu", "executor.cu", "comm.cu", "noalloc.cu"];
    let run = |args: &[String], what: &str| {
        let status = Command::new(&nvcc).args(args).status().unwrap_or_else(|e| panic!("{what}: {e}"));
        if !status.success() {
            panic!("{what} failed");
        }
    };
    let mut objects = Vec::new();
    for unit in units {
        let source = csrc.join(unit);
        let object = out_dir.join(unit.replace(".cu", ".o"));
        let mut args: Vec<String> = [
            "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC",
            "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr",
        ]
        .iter()
        .map(|s| s.to_string())
        .collect();
        args.push(format!("-I{}", include.display()));
        if unit == "ops.cu" {
            args.push("--fmad=false".to_string());
        }
        args.extend(["-c".to_string(), source.display().to_string(), "-o".to_string(), object.display().to_string()]);
        run(&args, &format!("nvcc {unit}"));
        objects.push(object.display().to_string());
    }
    let library = out_dir.join("libtysor_cuda.so");
    let mut args: Vec<String> = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o"]
        .iter()
        .map(|s| s.to_string())
        .collect();
    args.push(library.display().to_string());
    args.extend(objects);
    args.extend(["-ldl".to_string(), "-lpthread".to_string()]);
    run(&args, "nvcc -shared libtysor_cuda.so");

    println!("cargo:rustc-link-search=native={}", out_dir.display());
    println!("cargo:rustc-link-lib=dylib=tysor_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out_dir.display());
    println!("cargo:rustc-cfg=tysor_cuda");
}
