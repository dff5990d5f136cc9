//! The C ABI of libkatago_cuda.so (include/katago_cuda.h), declared for Rust. Every function returns a status
//! (KC_OK = 0); kc_last_error() holds the message of the last failure on the calling thread.

use std::os::raw::{c_char, c_float, c_int, c_void};

#[repr(C)]
pub struct KcModel {
  _p: [u8; 0],
}
#[repr(C)]
pub struct KcContext {
  _p: [u8; 0],
}
#[repr(C)]
pub struct KcHandle {
  _p: [u8; 0],
}

#[repr(C)]
pub struct KcDesc {
  pub name: [c_char; 128],
  pub model_version: i32,
  pub num_input_channels: i32,
  pub num_input_global_channels: i32,
  pub num_input_meta_channels: i32,
  pub meta_encoder_version: i32,
  pub num_policy_channels: i32,
  pub num_value_channels: i32,
  pub num_score_value_channels: i32,
  pub num_ownership_channels: i32,
  pub trunk_num_blocks: i32,
  pub trunk_num_channels: i32,
  pub trunk_norm_kind: i32,
  pub has_any_transformer_blocks: i32,
  pub has_any_nested_bottleneck_blocks: i32,
  pub post_process_from_header: i32,
  pub prefer_pass_alive_under_suicide_rules: i32,
  pub prefer_exclude_territory_adjacent_to_atari: i32,
  pub num_parameters: i64,
  pub trunk_spatial_conv_depth: f64,
  pub post_process: [c_float; 8],
}

pub const KC_OK: c_int = 0;
pub const KC_ERR_INVALID: c_int = 1;
pub const KC_ERR_TIMEOUT: c_int = 4;
pub const KC_PRECISION_F32: c_int = 0;
pub const KC_PRECISION_AUTO: c_int = 3;

pub const KC_PACKED_WORDS_PER_PLANE: usize = 12;
pub const KC_FINISHED_ROW_LEN: usize = 732;
pub const KC_FINISHED_POLICY: usize = 0;
pub const KC_FINISHED_VALUE: usize = 362;
pub const KC_FINISHED_MISC: usize = 365;
pub const KC_FINISHED_OWNERSHIP: usize = 371;

extern "C" {
  pub fn kc_last_error() -> *const c_char;
  pub fn kc_device_count(count: *mut c_int) -> c_int;
  pub fn kc_model_load(bytes: *const c_void, n: usize, file_name: *const c_char, out: *mut *mut KcModel) -> c_int;
  pub fn kc_model_desc(model: *const KcModel, out: *mut KcDesc) -> c_int;
  pub fn kc_model_destroy(model: *mut KcModel) -> c_int;
  pub fn kc_context_create(
    gpu_idxs: *const c_int,
    n_gpu_idxs: c_int,
    nn_x_len: c_int,
    nn_y_len: c_int,
    precision: c_int,
    model: *const KcModel,
    out: *mut *mut KcContext,
  ) -> c_int;
  pub fn kc_context_precision(ctx: *const KcContext, precision: *mut c_int) -> c_int;
  pub fn kc_context_destroy(ctx: *mut KcContext) -> c_int;
  pub fn kc_handle_create(ctx: *mut KcContext, gpu_idx: c_int, max_batch: c_int, inputs_use_nhwc: c_int, out: *mut *mut KcHandle)
    -> c_int;
  pub fn kc_handle_destroy(h: *mut KcHandle) -> c_int;
  pub fn kc_handle_input_ptrs(h: *mut KcHandle, spatial: *mut *mut f32, global: *mut *mut f32, meta: *mut *mut f32) -> c_int;
  pub fn kc_handle_packed_input_ptrs(
    h: *mut KcHandle,
    spatial_bits: *mut *mut u32,
    global: *mut *mut f32,
    meta: *mut *mut f32,
    symmetry: *mut *mut i32,
    policy_optimism: *mut *mut f32,
  ) -> c_int;
  pub fn kc_handle_output_layout(
    h: *const KcHandle,
    row_len: *mut c_int,
    policy_off: *mut c_int,
    value_off: *mut c_int,
    score_off: *mut c_int,
    ownership_off: *mut c_int,
  ) -> c_int;
  pub fn kc_pack_spatial(planes: *const f32, n_planes: c_int, bits: *mut u32) -> c_int;
  pub fn kc_enqueue(h: *mut KcHandle, n: c_int) -> c_int;
  pub fn kc_enqueue_packed(h: *mut KcHandle, n: c_int, finish: c_int) -> c_int;
  pub fn kc_wait(h: *mut KcHandle, timeout_ms: c_int, out_rows: *mut *const f32) -> c_int;
}

/// The message of the last failed call on this thread.
pub fn last_error() -> String {
  unsafe {
    let p = kc_last_error();
    if p.is_null() {
      return String::new();
    }
    std::ffi::CStr::from_ptr(p).to_string_lossy().into_owned()
  }
}
