//! `NeuralNet` over libkatago_cuda: the reference's burn backend (crates/katago-nn-burn/src/backend.rs) with the
//! generated network replaced by the B200 forward pass. The structure follows it: get_output in three parts,
//! copy_inputs (:497-546), run_network (:549-619, the wait on a helper OS thread as read_on_helper_thread :743-753)
//! and copy_outputs (:622-731). The library does the symmetry of the inputs and copy_outputs on the device when the
//! rows can travel bit-packed (every fill_row_v7 spatial feature is 0 or 1); otherwise the rows go as floats moved
//! by SymmetryHelpers here and copy_outputs runs here, as in the reference.

use std::any::Any;
use std::collections::BTreeSet;
use std::ffi::CString;
use std::rc::Rc;

use katago_core::core::commontypes::enabled_t;
use katago_core::core::config_parser::ConfigParser;
use katago_core::core::global::KataError;
use katago_core::neuralnet::desc::ModelDesc;
use katago_core::neuralnet::modelversion::NNModelVersion;
use katago_core::neuralnet::nneval::NNResultBuf;
use katago_core::neuralnet::nninputs::NNOutput;
use katago_core::neuralnet::nninputs::SymmetryHelpers;
use katago_core::neuralnet::nninterface;
use katago_core::port::executor::LocalBoxFuture;

use crate::ffi;

fn check(status: std::os::raw::c_int) -> Result<(), KataError> {
  if status == ffi::KC_OK {
    Ok(())
  } else {
    Err(KataError::StringError(ffi::last_error()))
  }
}

/// The backend object the host injects into NNEvaluator (one per process).
pub struct CudaNeuralNet {}

impl CudaNeuralNet {
  pub fn new() -> CudaNeuralNet {
    CudaNeuralNet {}
  }
}

/// upstream: LoadedModel. The parsed model (weights on the host until a handle uploads them) and its ModelDesc.
pub struct CudaLoadedModel {
  model: *mut ffi::KcModel,
  pub model_desc: ModelDesc,
}

impl Drop for CudaLoadedModel {
  fn drop(&mut self) {
    unsafe {
      ffi::kc_model_destroy(self.model);
    }
  }
}

impl nninterface::LoadedModel for CudaLoadedModel {
  fn as_any(&self) -> &dyn Any {
    self
  }
}

/// upstream: ComputeContext. Shared by the handles of every server thread (the library's context is immutable
/// once made).
pub struct CudaComputeContext {
  ctx: *mut ffi::KcContext,
  use_fp16: bool,
}

impl Drop for CudaComputeContext {
  fn drop(&mut self) {
    unsafe {
      ffi::kc_context_destroy(self.ctx);
    }
  }
}

impl nninterface::ComputeContext for CudaComputeContext {
  fn as_any(&self) -> &dyn Any {
    self
  }
}

/// upstream: ComputeHandle. One weight replica, stream and set of pinned staging buffers on one GPU, used by one
/// server thread.
pub struct CudaComputeHandle {
  h: *mut ffi::KcHandle,
  max_batch: usize,
  use_fp16: bool,
  model_version: i32,
  num_input_channels: usize,
  num_global: usize,
  num_meta: usize,
  num_policy_channels: usize,
  // packed staging (kc_handle_packed_input_ptrs)
  pk_bits: *mut u32,
  pk_global: *mut f32,
  pk_meta: *mut f32,
  pk_sym: *mut i32,
  pk_opt: *mut f32,
  // float staging (kc_handle_input_ptrs) and the raw output row layout, for rows that cannot be packed
  f_spatial: *mut f32,
  f_global: *mut f32,
  f_meta: *mut f32,
  row_len: usize,
  policy_off: usize,
  value_off: usize,
  score_off: usize,
  own_off: usize,
}

impl Drop for CudaComputeHandle {
  fn drop(&mut self) {
    unsafe {
      ffi::kc_handle_destroy(self.h);
    }
  }
}

impl nninterface::ComputeHandle for CudaComputeHandle {
  fn as_any_mut(&mut self) -> &mut dyn Any {
    self
  }
  fn as_any(&self) -> &dyn Any {
    self
  }
}

/// upstream: InputBuffers. The staging buffers belong to the handle (pinned memory of its GPU); this keeps the
/// sizes NNEvaluator asks for.
pub struct CudaInputBuffers {
  pub max_batch_size: i32,
  pub single_input_elts: usize,
  pub single_input_global_elts: usize,
  pub single_input_meta_elts: usize,
}

impl nninterface::InputBuffers for CudaInputBuffers {
  fn as_any_mut(&mut self) -> &mut dyn Any {
    self
  }
}

/// The handle's wait, moved to a helper thread (the handle is not touched by the serve task meanwhile).
struct PendingWait(*mut ffi::KcHandle);
unsafe impl Send for PendingWait {}
struct RowsPtr(*const f32);
unsafe impl Send for RowsPtr {}

/// kc_wait on a fresh OS thread, awaited without blocking the search thread (read_on_helper_thread,
/// backend.rs:743-753).
async fn wait_on_helper_thread(h: *mut ffi::KcHandle) -> Result<*const f32, KataError> {
  let (tx, rx) = futures::channel::oneshot::channel::<Result<RowsPtr, String>>();
  let pending = PendingWait(h);
  std::thread::Builder::new()
    .name("cuda-readback".to_string())
    .spawn(move || {
      let pending = pending;
      let mut rows: *const f32 = std::ptr::null();
      let st = unsafe { ffi::kc_wait(pending.0, -1, &mut rows) };
      let _ = tx.send(if st == ffi::KC_OK { Ok(RowsPtr(rows)) } else { Err(ffi::last_error()) });
    })
    .map_err(|e| KataError::StringError(format!("CUDA backend: could not start the readback thread: {e}")))?;
  match rx.await {
    Ok(Ok(rows)) => Ok(rows.0),
    Ok(Err(msg)) => Err(KataError::StringError(msg)),
    Err(_) => Err(KataError::StringError("CUDA backend: the readback thread died".to_string())),
  }
}

fn downcast_model(loaded_model: &dyn nninterface::LoadedModel) -> &CudaLoadedModel {
  loaded_model.as_any().downcast_ref::<CudaLoadedModel>().expect("LoadedModel created by CudaNeuralNet")
}

/// NeuralNet::getBatchPolicy: any batch size (the forward pass is captured per batch size).
pub fn get_batch_policy(cfg: &mut ConfigParser) -> nninterface::BatchPolicy {
  let _ = cfg;
  nninterface::BatchPolicy::Dynamic
}

/// NeuralNet::getNumEffectiveDevices: devices are selected by gpu index.
pub fn get_num_effective_devices(cfg: &mut ConfigParser, gpu_idx_by_server_thread: &[i32]) -> i32 {
  let _ = cfg;
  let distinct: BTreeSet<i32> = gpu_idx_by_server_thread.iter().copied().collect();
  std::cmp::max(1, distinct.len() as i32)
}

impl nninterface::NeuralNet for CudaNeuralNet {
  fn global_initialize(&self) {}
  fn global_cleanup(&self) {}

  fn print_devices(&self) {
    let mut count = 0;
    let st = unsafe { ffi::kc_device_count(&mut count) };
    if st == ffi::KC_OK {
      tracing::info!("CUDA backend: {} sm_100 device(s)", count);
    } else {
      tracing::info!("CUDA backend: {}", ffi::last_error());
    }
  }

  fn get_runtime_backend_detail(&self, cfg: &mut ConfigParser) -> String {
    let _ = cfg;
    String::new()
  }

  fn get_batch_policy(&self, cfg: &mut ConfigParser) -> nninterface::BatchPolicy {
    get_batch_policy(cfg)
  }

  fn get_num_effective_devices(&self, cfg: &mut ConfigParser, gpu_idx_by_server_thread: &[i32]) -> i32 {
    get_num_effective_devices(cfg, gpu_idx_by_server_thread)
  }

  /// upstream: NeuralNet::loadModelFile. A KataGo .bin / .bin.gz / .txt / .txt.gz, parsed by the library.
  fn load_model_file(&self, file: &str, model_bytes: Vec<u8>, expected_sha256: &str) -> Result<Box<dyn nninterface::LoadedModel>, KataError> {
    if !expected_sha256.is_empty() {
      return Err(KataError::StringError(
        "Error loading or parsing model file ".to_string() + file + ": expectedSha256 is not supported by the cuda backend",
      ));
    }
    let name = CString::new(file).map_err(|_| KataError::StringError(format!("bad model file name {file}")))?;
    let mut model: *mut ffi::KcModel = std::ptr::null_mut();
    check(unsafe { ffi::kc_model_load(model_bytes.as_ptr() as *const _, model_bytes.len(), name.as_ptr(), &mut model) })?;
    let mut d: ffi::KcDesc = unsafe { std::mem::zeroed() };
    let st = unsafe { ffi::kc_model_desc(model, &mut d) };
    if st != ffi::KC_OK {
      unsafe {
        ffi::kc_model_destroy(model);
      }
      return Err(KataError::StringError(ffi::last_error()));
    }
    let loaded = CudaLoadedModel { model, model_desc: model_desc_of(&d) };
    ModelDesc::check_name_valid(&loaded.model_desc.name)?;
    if loaded.model_desc.model_version > NNModelVersion::latestModelVersionImplemented {
      return Err(KataError::StringError(
        "This neural net requires a newer KataGo version. Model version: ".to_string() + &loaded.model_desc.model_version.to_string(),
      ));
    }
    Ok(Box::new(loaded))
  }

  fn get_model_desc<'a>(&self, loaded_model: &'a dyn nninterface::LoadedModel) -> &'a ModelDesc {
    &downcast_model(loaded_model).model_desc
  }

  /// upstream: NeuralNet::createComputeContext. useFP16 true: f16 for convolution nets and bf16 for transformer
  /// nets (tensor cores); false or auto: float32 (the parity tier, as the reference's default).
  fn create_compute_context(
    &self,
    gpu_idxs: &[i32],
    nn_x_len: i32,
    nn_y_len: i32,
    home_data_dir_override: &str,
    use_fp16_mode: enabled_t,
    loaded_model: &dyn nninterface::LoadedModel,
    cfg: &mut ConfigParser,
  ) -> Result<Box<dyn nninterface::ComputeContext>, KataError> {
    let _ = home_data_dir_override;
    let _ = cfg;
    let use_fp16 = use_fp16_mode == enabled_t::True;
    let precision = if use_fp16 { ffi::KC_PRECISION_AUTO } else { ffi::KC_PRECISION_F32 };
    let model = downcast_model(loaded_model);
    let mut ctx: *mut ffi::KcContext = std::ptr::null_mut();
    check(unsafe {
      ffi::kc_context_create(gpu_idxs.as_ptr(), gpu_idxs.len() as i32, nn_x_len, nn_y_len, precision, model.model, &mut ctx)
    })?;
    Ok(Box::new(CudaComputeContext { ctx, use_fp16 }))
  }

  /// upstream: NeuralNet::createComputeHandle. Uploads the packed weights to `gpu_idx_for_this_thread` (the
  /// server thread's cudaGpuToUseThread<k>) and prepares the forward pass for batches up to max_batch_size.
  fn create_compute_handle(
    &self,
    context: &dyn nninterface::ComputeContext,
    loaded_model: &dyn nninterface::LoadedModel,
    max_batch_size: i32,
    require_exact_nn_len: bool,
    inputs_use_nhwc: bool,
    gpu_idx_for_this_thread: i32,
    server_thread_idx: i32,
  ) -> Result<Box<dyn nninterface::ComputeHandle>, KataError> {
    let _ = require_exact_nn_len; // the on-board mask is always applied
    let context = context.as_any().downcast_ref::<CudaComputeContext>().expect("ComputeContext created by CudaNeuralNet");
    let m = &downcast_model(loaded_model).model_desc;
    tracing::info!("CUDA backend thread {}: Model version {}, gpu {}", server_thread_idx, m.model_version, gpu_idx_for_this_thread);
    let mut h: *mut ffi::KcHandle = std::ptr::null_mut();
    check(unsafe { ffi::kc_handle_create(context.ctx, gpu_idx_for_this_thread, max_batch_size, inputs_use_nhwc as i32, &mut h) })?;
    let mut ch = CudaComputeHandle {
      h,
      max_batch: max_batch_size as usize,
      use_fp16: context.use_fp16,
      model_version: m.model_version,
      num_input_channels: m.num_input_channels as usize,
      num_global: m.num_input_global_channels as usize,
      num_meta: m.num_input_meta_channels as usize,
      num_policy_channels: m.num_policy_channels as usize,
      pk_bits: std::ptr::null_mut(),
      pk_global: std::ptr::null_mut(),
      pk_meta: std::ptr::null_mut(),
      pk_sym: std::ptr::null_mut(),
      pk_opt: std::ptr::null_mut(),
      f_spatial: std::ptr::null_mut(),
      f_global: std::ptr::null_mut(),
      f_meta: std::ptr::null_mut(),
      row_len: 0,
      policy_off: 0,
      value_off: 0,
      score_off: 0,
      own_off: 0,
    };
    check(unsafe { ffi::kc_handle_packed_input_ptrs(h, &mut ch.pk_bits, &mut ch.pk_global, &mut ch.pk_meta, &mut ch.pk_sym, &mut ch.pk_opt) })?;
    check(unsafe { ffi::kc_handle_input_ptrs(h, &mut ch.f_spatial, &mut ch.f_global, &mut ch.f_meta) })?;
    let (mut rl, mut po, mut vo, mut so, mut oo) = (0, 0, 0, 0, 0);
    check(unsafe { ffi::kc_handle_output_layout(h, &mut rl, &mut po, &mut vo, &mut so, &mut oo) })?;
    ch.row_len = rl as usize;
    ch.policy_off = po as usize;
    ch.value_off = vo as usize;
    ch.score_off = so as usize;
    ch.own_off = oo as usize;
    Ok(Box::new(ch))
  }

  fn set_is_warmup(&self, compute_handle: &dyn nninterface::ComputeHandle, is_warmup: bool) -> bool {
    let _ = compute_handle;
    let _ = is_warmup;
    false
  }

  fn is_using_fp16(&self, compute_handle: &dyn nninterface::ComputeHandle) -> bool {
    compute_handle.as_any().downcast_ref::<CudaComputeHandle>().expect("ComputeHandle created by CudaNeuralNet").use_fp16
  }

  fn create_input_buffers(&self, loaded_model: &dyn nninterface::LoadedModel, max_batch_size: i32, nn_x_len: i32, nn_y_len: i32) -> Box<dyn nninterface::InputBuffers> {
    let m = &downcast_model(loaded_model).model_desc;
    Box::new(CudaInputBuffers {
      max_batch_size,
      single_input_elts: (m.num_input_channels * nn_x_len * nn_y_len) as usize,
      single_input_global_elts: m.num_input_global_channels as usize,
      single_input_meta_elts: m.num_input_meta_channels as usize,
    })
  }

  /// upstream: NeuralNet::getOutput.
  fn get_output<'a>(
    &'a self,
    compute_handle: &'a mut dyn nninterface::ComputeHandle,
    buffers: &'a mut dyn nninterface::InputBuffers,
    num_batch_elts_filled: i32,
    input_bufs: &'a [Rc<NNResultBuf>],
    outputs: &'a mut [NNOutput],
  ) -> LocalBoxFuture<'a, Result<(), KataError>> {
    Box::pin(async move {
      let h = compute_handle.as_any_mut().downcast_mut::<CudaComputeHandle>().expect("ComputeHandle created by CudaNeuralNet");
      let _ = buffers;
      get_output_impl(h, num_batch_elts_filled as usize, input_bufs, outputs).await
    })
  }
}

fn model_desc_of(d: &ffi::KcDesc) -> ModelDesc {
  let mut m = ModelDesc::new();
  m.name = unsafe { std::ffi::CStr::from_ptr(d.name.as_ptr()) }.to_string_lossy().into_owned();
  m.model_version = d.model_version;
  m.num_input_channels = d.num_input_channels;
  m.num_input_global_channels = d.num_input_global_channels;
  m.num_input_meta_channels = d.num_input_meta_channels;
  m.num_policy_channels = d.num_policy_channels;
  m.num_value_channels = d.num_value_channels;
  m.num_score_value_channels = d.num_score_value_channels;
  m.num_ownership_channels = d.num_ownership_channels;
  m.meta_encoder_version = d.meta_encoder_version;
  m.prefer_pass_alive_under_suicide_rules = d.prefer_pass_alive_under_suicide_rules != 0;
  m.prefer_exclude_territory_adjacent_to_atari = d.prefer_exclude_territory_adjacent_to_atari != 0;
  let p = &mut m.post_process_params;
  p.td_score_multiplier = d.post_process[0] as f64;
  p.score_mean_multiplier = d.post_process[1] as f64;
  p.score_stdev_multiplier = d.post_process[2] as f64;
  p.lead_multiplier = d.post_process[3] as f64;
  p.variance_time_multiplier = d.post_process[4] as f64;
  p.shortterm_value_error_multiplier = d.post_process[5] as f64;
  p.shortterm_score_error_multiplier = d.post_process[6] as f64;
  p.output_scale_multiplier = d.post_process[7];
  // the layer structure stays in the library: the summary values come from its parser
  m.arch_summary.present = true;
  m.arch_summary.trunk_spatial_conv_depth = d.trunk_spatial_conv_depth;
  m.arch_summary.num_parameters = d.num_parameters;
  m.arch_summary.has_any_transformer_blocks = d.has_any_transformer_blocks != 0;
  m.arch_summary.has_any_nested_bottleneck_blocks = d.has_any_nested_bottleneck_blocks != 0;
  m
}

/// get_output: copy_inputs, run_network, copy_outputs (backend.rs:410-731).
async fn get_output_impl(h: &mut CudaComputeHandle, n: usize, input_bufs: &[Rc<NNResultBuf>], outputs: &mut [NNOutput]) -> Result<(), KataError> {
  debug_assert!(n > 0 && n <= h.max_batch && outputs.len() == n);
  let c = h.num_input_channels;
  let words = c * ffi::KC_PACKED_WORDS_PER_PLANE;
  // copy_inputs: the symmetry and optimism of every row are read now, before the first await
  let mut symmetry_by_row = Vec::with_capacity(n);
  let mut optimism_by_row = Vec::with_capacity(n);
  let mut packed = true;
  for (row, buf) in input_bufs.iter().take(n).enumerate() {
    symmetry_by_row.push(buf.symmetry.get());
    optimism_by_row.push(buf.policy_optimism.get() as f32);
    if packed {
      let spatial = buf.row_spatial_buf.borrow();
      let st = unsafe { ffi::kc_pack_spatial(spatial.as_ptr(), c as i32, h.pk_bits.add(row * words)) };
      if st == ffi::KC_ERR_INVALID {
        packed = false; // a feature that is neither 0 nor 1: this batch goes as floats
      } else {
        check(st)?;
      }
    }
  }
  let (glob, meta) = if packed { (h.pk_global, h.pk_meta) } else { (h.f_global, h.f_meta) };
  for (row, buf) in input_bufs.iter().take(n).enumerate() {
    let g = buf.row_global_buf.borrow();
    unsafe { std::ptr::copy_nonoverlapping(g.as_ptr(), glob.add(row * h.num_global), h.num_global) };
    if h.num_meta > 0 {
      let m = buf.row_meta_buf.borrow();
      unsafe { std::ptr::copy_nonoverlapping(m.as_ptr(), meta.add(row * h.num_meta), h.num_meta) };
    }
    if packed {
      unsafe {
        *h.pk_sym.add(row) = symmetry_by_row[row];
        *h.pk_opt.add(row) = optimism_by_row[row];
      }
    } else {
      let spatial = buf.row_spatial_buf.borrow();
      let elts = c * 361;
      let dst = unsafe { std::slice::from_raw_parts_mut(h.f_spatial.add(row * elts), elts) };
      SymmetryHelpers::copy_inputs_with_symmetry(&spatial[..elts], dst, 1, 19, 19, c as i32, false, symmetry_by_row[row]);
    }
  }
  // run_network: enqueue, then wait on a helper thread
  if packed {
    check(unsafe { ffi::kc_enqueue_packed(h.h, n as i32, 1) })?;
  } else {
    check(unsafe { ffi::kc_enqueue(h.h, n as i32) })?;
  }
  let rows = wait_on_helper_thread(h.h).await?;
  // copy_outputs
  if packed {
    let fin = unsafe { std::slice::from_raw_parts(rows, n * ffi::KC_FINISHED_ROW_LEN) };
    for (row, output) in outputs.iter_mut().enumerate().take(n) {
      let f = &fin[row * ffi::KC_FINISHED_ROW_LEN..(row + 1) * ffi::KC_FINISHED_ROW_LEN];
      output.policy_probs[..362].copy_from_slice(&f[ffi::KC_FINISHED_POLICY..ffi::KC_FINISHED_POLICY + 362]);
      let v = &f[ffi::KC_FINISHED_VALUE..];
      output.white_win_prob = v[0];
      output.white_loss_prob = v[1];
      output.white_no_result_prob = v[2];
      let s = &f[ffi::KC_FINISHED_MISC..];
      output.white_score_mean = s[0];
      output.white_score_mean_sq = s[1];
      output.white_lead = s[2];
      output.var_time_left = s[3];
      output.shortterm_winloss_error = s[4];
      output.shortterm_score_error = s[5];
      if let Some(own) = output.white_owner_map.as_mut() {
        own[..361].copy_from_slice(&f[ffi::KC_FINISHED_OWNERSHIP..ffi::KC_FINISHED_OWNERSHIP + 361]);
      }
    }
  } else {
    let data = unsafe { std::slice::from_raw_parts(rows, n * h.row_len) };
    copy_outputs_raw(h, data, &symmetry_by_row, &optimism_by_row, outputs);
  }
  Ok(())
}

/// copy_outputs on raw rows (backend.rs:622-731), for batches that went as floats.
fn copy_outputs_raw(h: &CudaComputeHandle, data: &[f32], symmetry_by_row: &[i32], optimism_by_row: &[f32], outputs: &mut [NNOutput]) {
  let hw = 361usize;
  let mut tmp = [0.0f32; 361];
  for (row, output) in outputs.iter_mut().enumerate() {
    let rd = &data[row * h.row_len..(row + 1) * h.row_len];
    let pol = &rd[h.policy_off..];
    let sym = symmetry_by_row[row];
    let o = optimism_by_row[row];
    if h.num_policy_channels == 2 || (h.num_policy_channels == 4 && h.model_version >= 16) {
      for i in 0..hw {
        let p = pol[i];
        let p_opt = pol[(hw + 1) + i];
        tmp[i] = p + (p_opt - p) * o;
      }
      SymmetryHelpers::copy_outputs_with_symmetry(&tmp, &mut output.policy_probs, 1, 19, 19, sym);
      output.policy_probs[hw] = pol[hw] + (pol[(hw + 1) + hw] - pol[hw]) * o;
    } else {
      SymmetryHelpers::copy_outputs_with_symmetry(&pol[..hw], &mut output.policy_probs, 1, 19, 19, sym);
      output.policy_probs[hw] = pol[hw];
    }
    let v = &rd[h.value_off..];
    output.white_win_prob = v[0];
    output.white_loss_prob = v[1];
    output.white_no_result_prob = v[2];
    if let Some(own) = output.white_owner_map.as_mut() {
      SymmetryHelpers::copy_outputs_with_symmetry(&rd[h.own_off..h.own_off + hw], own, 1, 19, 19, sym);
    }
    let s = &rd[h.score_off..];
    let ver = h.model_version;
    if ver >= 9 {
      output.white_score_mean = s[0];
      output.white_score_mean_sq = s[1];
      output.white_lead = s[2];
      output.var_time_left = s[3];
      output.shortterm_winloss_error = s[4];
      output.shortterm_score_error = s[5];
    } else if ver >= 8 {
      output.white_score_mean = s[0];
      output.white_score_mean_sq = s[1];
      output.white_lead = s[2];
      output.var_time_left = s[3];
      output.shortterm_winloss_error = 0.0;
      output.shortterm_score_error = 0.0;
    } else if ver >= 4 {
      output.white_score_mean = s[0];
      output.white_score_mean_sq = s[1];
      output.white_lead = s[0];
      output.var_time_left = 0.0;
      output.shortterm_winloss_error = 0.0;
      output.shortterm_score_error = 0.0;
    } else {
      output.white_score_mean = s[0];
      output.white_score_mean_sq = s[0] * s[0];
      output.white_lead = s[0];
      output.var_time_left = 0.0;
      output.shortterm_winloss_error = 0.0;
      output.shortterm_score_error = 0.0;
    }
  }
}
