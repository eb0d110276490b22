//! `--backend cuda`: tysor's graph executor on an NVIDIA B200 (sm_100a)
//! through libtysor_cuda's C ABI (include/tysor_cuda.h), the counterpart of
//! the Metal backend (src/backend/metal/).  `native` binds the library,
//! `runtime` holds the `--run`, `--backward` and `--train` entry points that
//! main.rs, training/backward.rs and training/executor.rs dispatch to.
pub mod native;
pub mod runtime;
