//! Links libkatago_cuda.so. KATAGO_CUDA_LIB_DIR names the directory that holds it (the `lib/` directory that
//! `make -C katago-rs_b200` builds); the same directory is added to the binary's rpath.

fn main() {
  println!("cargo:rerun-if-env-changed=KATAGO_CUDA_LIB_DIR");
  if let Ok(dir) = std::env::var("KATAGO_CUDA_LIB_DIR") {
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
  }
  println!("cargo:rustc-link-lib=dylib=katago_cuda");
}
