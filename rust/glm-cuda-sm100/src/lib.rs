//! glm-cuda backend for libglmaxx_sm100: the B200 (sm_100a) routed-MoE library.
//!
//! Drop-in for the reference's `crates/glm-cuda` (`glmaxx_sm120`):
//! - [`abi`]: the C structs and constants of `include/glmaxx_kernel.h` beyond the
//!   reference's three descriptors (router, layer, EXL3 experts, finish, peer);
//! - [`ffi`]: the whole `extern "C"` surface, the reference's block
//!   (`crates/glm-cuda/src/ffi.rs:21-151`) plus the v3 entry points;
//! - [`rank`]: the thread-affine rank context (`NativeRankContext::bind`
//!   generalised to compute capability 10.x and 1/2/4/8 devices) and one rank's
//!   routed-MoE step;
//! - [`tp`]: an N-rank tensor-parallel group (one thread per rank) whose step is
//!   the layer on every rank plus the peer-memory finish.

pub mod abi;
pub mod ffi;
pub mod rank;
pub mod tp;

pub use abi::{check, KernelError, KERNEL_ABI};
pub use rank::{DeviceBuffer, LayerGeometry, RankContext, RankLayerWeights, RoutedMoeStep};
pub use tp::{StepOutput, TpMoeGroup};

/// Checks that the loaded library is this ABI (`glmaxx_kernel_abi()`).
pub fn validate_native_library() -> Result<(), KernelError> {
    // SAFETY: the library returns a static NUL-terminated string.
    let s = unsafe { core::ffi::CStr::from_ptr(ffi::glmaxx_kernel_abi()) };
    if s.to_bytes() == KERNEL_ABI.as_bytes() { Ok(()) } else { Err(KernelError::Abi) }
}
