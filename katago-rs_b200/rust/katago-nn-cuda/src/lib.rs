//! katago-rs's `cuda` backend: the `NeuralNet` trait (katago-core) over libkatago_cuda.so, the B200 (sm_100a)
//! forward pass, and the NNEvaluatorHost that katago-cli selects with `-backend cuda`.
//!
//! Unlike the burn backend, whose networks are compiled in per NetId (crates/katago-cli/src/host.rs:58-60), any
//! KataGo model file loads at run time: the library parses `.bin` / `.bin.gz` / `.txt` / `.txt.gz` itself.

pub mod backend;
pub mod ffi;
pub mod host;

pub use backend::CudaNeuralNet;
pub use host::CudaHost;
