//! The cuda backend as Setup's NNEvaluatorHost (the counterpart of katago-cli's BurnHost,
//! crates/katago-cli/src/host.rs:64-130). katago-cli's `compiled_backends()` (args.rs:130-137) lists "cuda" behind
//! a `cuda` feature and builds `CudaHost::new(spawner)` for it. Config keys use the prefix "cuda" (cudaUseFP16,
//! cudaGpuToUseThread<k>), which Setup reads (setup.rs:456-517): one NN server thread, one handle and one weight
//! replica per GPU.

use std::cell::RefCell;
use std::rc::Rc;

use katago_core::core::config_parser::ConfigParser;
use katago_core::core::global::KataError;
use katago_core::neuralnet::nninterface::BatchPolicy;
use katago_core::neuralnet::nninterface::NeuralNet;
use katago_core::port::executor::Spawner;
use katago_core::program::setup::NNEvaluatorHost;

use crate::backend;
use crate::CudaNeuralNet;

pub struct CudaHost {
  pub spawner: Rc<dyn Spawner>,
  /// Model files loaded so far (for tests and diagnostics).
  pub loaded: RefCell<Vec<String>>,
}

impl CudaHost {
  pub fn new(spawner: Rc<dyn Spawner>) -> CudaHost {
    CudaHost { spawner, loaded: RefCell::new(Vec::new()) }
  }
}

impl NNEvaluatorHost for CudaHost {
  fn backend_prefix(&self) -> String {
    "cuda".to_string()
  }
  fn global_initialize(&self) {}
  fn global_cleanup(&self) {}
  /// The model file's bytes, read here (katago-core has no file IO); the backend parses them.
  fn load_model(&self, _nn_model_name: &str, nn_model_file: &str) -> Result<(Rc<dyn NeuralNet>, Vec<u8>), KataError> {
    self.loaded.borrow_mut().push(nn_model_file.to_string());
    let bytes = std::fs::read(nn_model_file).map_err(|e| {
      KataError::StringError(format!(
        "Error loading or parsing model file {nn_model_file}: Could not open file {nn_model_file} - does not exist or invalid permissions? ({e})"
      ))
    })?;
    Ok((Rc::new(CudaNeuralNet::new()), bytes))
  }
  fn spawner(&self) -> Rc<dyn Spawner> {
    self.spawner.clone()
  }
  fn get_batch_policy(&self, cfg: &mut ConfigParser) -> BatchPolicy {
    backend::get_batch_policy(cfg)
  }
  fn get_num_effective_devices(&self, cfg: &mut ConfigParser, gpu_idx_by_server_thread: &[i32]) -> i32 {
    backend::get_num_effective_devices(cfg, gpu_idx_by_server_thread)
  }
}
