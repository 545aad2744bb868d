//! Rust binding of libb200attn, the B200 (sm_100a) joint-attention path of the
//! Qwen-Image-2.1 MMDiT blocks.
//!
//! `ffi` mirrors `include/b200_attn.h` field for field and function for function (the
//! C ABI is the boundary).  The safe layer maps status codes to [`Error`]; the optional
//! `candle` feature adds a tensor-level call for the engine's two attention call sites
//! (`src/transformer.rs:179-193`, `src/quantized_transformer.rs:139-151` of the
//! engine), which replaces norm_q/norm_k -> apply_rope -> cat(prefix K/V) ->
//! chunked_attention -> head merge with one `b200_attn_fwd`.
//!
//! No Rust toolchain was available where this crate was written: it follows the header
//! exactly (a test of the C-side repository diffs the `#[repr(C)]` structs and the
//! `extern "C"` block against the header), but it has not been compiled.

use std::ffi::{c_char, c_int, c_void, CStr};
use std::fmt;

pub mod ffi {
    use std::ffi::{c_char, c_int, c_void};

    pub const B200_ATTN_HEAD_DIM: i32 = 128;
    pub const B200_ATTN_ABI_VERSION: i32 = 4;
    pub const B200_ATTN_SPLIT_WORKSPACE_BYTES: usize = 21299968;
    pub const B200_NOALLOC_SCRATCH_BYTES: usize = 64 << 20;

    /// `b200_dtype`: element types of the entry points that take more than one.
    pub const B200_DTYPE_BF16: i32 = 0;
    pub const B200_DTYPE_F32: i32 = 1;
    pub const B200_DTYPE_F16: i32 = 2;

    pub const B200_OK: c_int = 0;
    pub const B200_ERR_INVALID: c_int = -1;
    pub const B200_ERR_UNSUPPORTED: c_int = -2;
    pub const B200_ERR_CUDA: c_int = -3;
    pub const B200_ERR_WORKSPACE: c_int = -4;
    pub const B200_ERR_LAYOUT: c_int = -5;
    pub const B200_ERR_DEVICE_TIMEOUT: c_int = -6;

    /// `b200_kv_desc`: keys [0, prefix_valid) of the cache and [0, target_valid) of the
    /// call are attended (replaces the key_valid mask).
    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
    pub struct KvDesc {
        pub prefix_valid: i32,
        pub target_valid: i32,
    }

    /// `b200_attn_args` (ABI version 3).  Device pointers are the caller's.
    #[repr(C)]
    #[derive(Clone, Copy, Debug)]
    pub struct AttnArgs {
        pub batch: i32,
        pub heads: i32,
        pub head_dim: i32,
        pub target_len: i32,
        pub prefix_len: i32,
        pub q: *const c_void,
        pub k: *const c_void,
        pub v: *const c_void,
        pub prefix_k: *const c_void,
        pub prefix_v: *const c_void,
        pub norm_q_w: *const f32,
        pub norm_k_w: *const f32,
        pub norm_eps: f32,
        pub pe: *const f32,
        pub desc: *const KvDesc,
        pub scale: f32,
        pub out: *mut c_void,
        pub k_rot_out: *mut c_void,
        pub v_out: *mut c_void,
        pub workspace: *mut c_void,
        pub workspace_bytes: usize,
        pub status: *mut i32,
        pub row_limit: *const i32,
        pub pe_batch_stride: i64,
    }

    extern "C" {
        pub fn b200_attn_workspace_bytes(args: *const AttnArgs, bytes: *mut usize) -> c_int;
        pub fn b200_attn_fwd(args: *const AttnArgs, stream: *mut c_void) -> c_int;
        pub fn b200_attn_fwd_noalloc(args: *const AttnArgs, stream: *mut c_void) -> c_int;
        pub fn b200_joint_attention(q_rot: *const c_void, k_rot: *const c_void, v: *const c_void,
            prefix_k: *const c_void, prefix_v: *const c_void, batch: i32, heads: i32,
            target_len: i32, prefix_len: i32, head_dim: i32, desc: *const KvDesc, scale: f32,
            out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
            status: *mut i32, stream: *mut c_void) -> c_int;
        pub fn b200_flash_attention(q: *const c_void, k: *const c_void, v: *const c_void,
            out: *mut c_void, batch: i32, sq: i32, skv: i32, heads: i32, head_dim: i32,
            scale: f32, key_len: *const i32, status: *mut i32, stream: *mut c_void) -> c_int;
        pub fn b200_flash_attention_ex(q: *const c_void, k: *const c_void, v: *const c_void,
            out: *mut c_void, batch: i32, sq: i32, skv: i32, heads: i32, head_dim: i32,
            scale: f32, key_len: *const i32, dtype: i32, status: *mut i32,
            stream: *mut c_void) -> c_int;
        pub fn b200_chunked_attention(q: *const c_void, k: *const c_void, v: *const c_void,
            out: *mut c_void, batch: i32, heads: i32, sq: i32, skv: i32, head_dim: i32,
            scale: f32, key_len: *const i32, status: *mut i32, stream: *mut c_void) -> c_int;
        pub fn b200_norm_rope(x: *const c_void, y: *mut c_void, batch: i32, tokens: i32,
            heads: i32, head_dim: i32, norm_w: *const f32, eps: f32, pe: *const f32,
            stream: *mut c_void) -> c_int;
        pub fn b200_qk_norm_rope(q: *const c_void, k: *const c_void, q_rot: *mut c_void,
            k_rot: *mut c_void, batch: i32, tokens: i32, heads: i32, head_dim: i32,
            norm_q_w: *const f32, norm_k_w: *const f32, eps: f32, pe: *const f32,
            stream: *mut c_void) -> c_int;
        pub fn b200_joint_layout(text_len: i32, text_image_mask: *const u8,
            cond_shapes: *const i32, n_cond: i32, target_h: i32, target_w: i32, cap: i32,
            image_ids: *mut i64, image_pad_mask: *mut u8, img_shapes: *mut i32,
            len_out: *mut i32, prefix_len_out: *mut i32, target_len_out: *mut i32) -> c_int;
        pub fn b200_rope_positions(img_shapes: *const i32, n_shapes: i32,
            image_pad_mask: *const u8, seq_len: i32, pos_out: *mut i64) -> c_int;
        pub fn b200_rope_pe(img_shapes: *const i32, n_shapes: i32, image_pad_mask: *const u8,
            seq_len: i32, axes: *const i32, theta: f32, pe_out: *mut f32) -> c_int;
        pub fn b200_key_valid_to_desc(key_valid: *const u8, batch: i32, prefix_len: i32,
            target_len: i32, desc_out: *mut KvDesc) -> c_int;
        pub fn b200_block_causal_limits(image_ids: *const i64, len: i32,
            limits_out: *mut i32) -> c_int;
        pub fn b200_strerror(status: c_int) -> *const c_char;
        pub fn b200_attn_strerror(status: c_int) -> *const c_char;
        pub fn b200_abi_version() -> c_int;
        pub fn b200_wait_selftest(status: *mut i32, limit_us: u32, stream: *mut c_void) -> c_int;
    }
}

/// A non-zero status of a library call, with the library's message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Error {
    pub status: i32,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "b200-attn: {} (status {})", self.message, self.status)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn message(rc: c_int) -> String {
    // SAFETY: b200_strerror returns a static NUL-terminated string for every code.
    unsafe {
        let p: *const c_char = ffi::b200_strerror(rc);
        if p.is_null() { format!("status {rc}") } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    }
}

/// Ok for B200_OK, else the library's error.
pub fn check(rc: c_int) -> Result<()> {
    if rc == ffi::B200_OK { Ok(()) } else { Err(Error { status: rc, message: message(rc) }) }
}

/// The ABI version the loaded library was built with (4 for this binding).
pub fn abi_version() -> i32 {
    unsafe { ffi::b200_abi_version() }
}

/// Scratch bytes `attn_fwd` wants for `args`.
pub fn workspace_bytes(args: &ffi::AttnArgs) -> Result<usize> {
    let mut n = 0usize;
    check(unsafe { ffi::b200_attn_workspace_bytes(args, &mut n) })?;
    Ok(n)
}

/// One joint-attention layer on `stream` (a CUstream, null = legacy default stream).
///
/// # Safety
/// Every pointer in `args` must be a live device allocation of the documented shape on
/// the current device, and `stream` a stream of that device.
pub unsafe fn attn_fwd(args: &ffi::AttnArgs, stream: *mut c_void) -> Result<()> {
    check(ffi::b200_attn_fwd(args, stream))
}

/// `attn_fwd` with the library's fixed scratch array instead of `args.workspace`, for
/// callers that cannot allocate device memory when they call.  Calls must not overlap
/// on the GPU.
///
/// # Safety
/// As [`attn_fwd`].
pub unsafe fn attn_fwd_noalloc(args: &ffi::AttnArgs, stream: *mut c_void) -> Result<()> {
    check(ffi::b200_attn_fwd_noalloc(args, stream))
}

/// `JointLayout::new` (engine `src/joint_layout.rs:52-103`) on the host.
pub struct JointLayout {
    pub image_ids: Vec<i64>,
    pub image_pad_mask: Vec<u8>,
    pub img_shapes: Vec<[i32; 3]>,
    pub prefix_len: i32,
    pub target_len: i32,
}

pub fn joint_layout(text_len: i32, text_image_mask: Option<&[u8]>, cond_shapes: &[(i32, i32)],
                    target: (i32, i32)) -> Result<JointLayout> {
    let cond: Vec<i32> = cond_shapes.iter().flat_map(|&(h, w)| [h, w]).collect();
    let cap = text_len + cond_shapes.iter().map(|&(h, w)| h * w / 4).sum::<i32>() * 4
        + target.0 * target.1 + 4;
    let mut ids = vec![0i64; cap as usize];
    let mut pad = vec![0u8; cap as usize];
    let mut shapes = vec![0i32; 3 * (cond_shapes.len() + 1)];
    let (mut len, mut prefix, mut tgt) = (0i32, 0i32, 0i32);
    check(unsafe {
        ffi::b200_joint_layout(text_len, text_image_mask.map_or(std::ptr::null(), |m| m.as_ptr()),
            cond.as_ptr(), cond_shapes.len() as i32, target.0, target.1, cap, ids.as_mut_ptr(),
            pad.as_mut_ptr(), shapes.as_mut_ptr(), &mut len, &mut prefix, &mut tgt)
    })?;
    ids.truncate(len as usize);
    pad.truncate(len as usize);
    Ok(JointLayout {
        image_ids: ids,
        image_pad_mask: pad,
        img_shapes: shapes.chunks(3).map(|c| [c[0], c[1], c[2]]).collect(),
        prefix_len: prefix,
        target_len: tgt,
    })
}

/// `EmbedNd::forward` rows (engine `src/rope.rs:37-211`): f32 [seq_len, 128], interleaved
/// (cos, sin), axes {16, 56, 56}, theta 1e4.
pub fn rope_pe(layout: &JointLayout) -> Result<Vec<f32>> {
    let n = layout.image_pad_mask.len();
    let shapes: Vec<i32> = layout.img_shapes.iter().flatten().copied().collect();
    let axes = [16i32, 56, 56];
    let mut pe = vec![0f32; n * 128];
    check(unsafe {
        ffi::b200_rope_pe(shapes.as_ptr(), layout.img_shapes.len() as i32,
                          layout.image_pad_mask.as_ptr(), n as i32, axes.as_ptr(), 1e4,
                          pe.as_mut_ptr())
    })?;
    Ok(pe)
}

/// The key_valid mask [B, P+T] (engine `src/transformer.rs:736-745`) as descriptors.
pub fn key_valid_to_desc(key_valid: &[u8], batch: i32, prefix_len: i32, target_len: i32)
                         -> Result<Vec<ffi::KvDesc>> {
    let mut d = vec![ffi::KvDesc::default(); batch as usize];
    check(unsafe {
        ffi::b200_key_valid_to_desc(key_valid.as_ptr(), batch, prefix_len, target_len, d.as_mut_ptr())
    })?;
    Ok(d)
}

/// Per-row key limits of the block-causal prefix pass (replaces
/// `build_block_causal_mask`, engine `src/attention_mask.rs:18-66`).
pub fn block_causal_limits(image_ids: &[i64]) -> Result<Vec<i32>> {
    let mut lim = vec![0i32; image_ids.len()];
    check(unsafe {
        ffi::b200_block_causal_limits(image_ids.as_ptr(), image_ids.len() as i32, lim.as_mut_ptr())
    })?;
    Ok(lim)
}

#[cfg(feature = "candle")]
pub mod candle_op {
    //! `Attention::forward`'s middle for candle 0.11 CUDA tensors (written against
    //! candle 0.11 / cudarc 0.17 as candle-flash-attn uses them; not compiled here).
    use super::{check, ffi};
    use candle_core::cuda_backend::cudarc::driver::DevicePtr;
    use candle_core::{DType, Device, Result, Storage, Tensor};
    use std::ffi::c_void;

    fn ptr(t: &Tensor) -> Result<u64> {
        let (st, layout) = t.storage_and_layout();
        let Storage::Cuda(cs) = &*st else { candle_core::bail!("b200-attn: tensor is not on a CUDA device") };
        if !t.is_contiguous() {
            candle_core::bail!("b200-attn: tensor must be contiguous");
        }
        let stream = cs.device().cuda_stream();
        let off = layout.start_offset() * t.dtype().size_in_bytes();
        let base = match t.dtype() {
            DType::BF16 => { let (p, _g) = cs.as_cuda_slice::<half::bf16>()?.device_ptr(&stream); p }
            DType::F32 => { let (p, _g) = cs.as_cuda_slice::<f32>()?.device_ptr(&stream); p }
            DType::I32 => { let (p, _g) = cs.as_cuda_slice::<i32>()?.device_ptr(&stream); p }
            DType::U8 => { let (p, _g) = cs.as_cuda_slice::<u8>()?.device_ptr(&stream); p }
            dt => candle_core::bail!("b200-attn: unsupported dtype {dt:?}"),
        };
        Ok(base + off as u64)
    }

    /// q/k/v [B,T,H*D] bf16 (the projections), prefix (K, V) [B,H,P,D] bf16 post-RoPE,
    /// norm weights [D] f32, pe [T,D] f32, desc [B,2] i32 or None, out [B,T,H*D] bf16,
    /// optional k_rot_out / v_out [B,H,T,D] bf16 (the cache slots), workspace u8 of
    /// `workspace_bytes` bytes.  Errors follow the engine's `bail!` convention.
    #[allow(clippy::too_many_arguments)]
    pub fn attn_fwd(q: &Tensor, k: &Tensor, v: &Tensor, heads: usize,
                    prefix: Option<(&Tensor, &Tensor)>, norm_q_w: &Tensor, norm_k_w: &Tensor,
                    eps: f32, pe: &Tensor, desc: Option<&Tensor>, scale: f32, out: &Tensor,
                    k_rot_out: Option<&Tensor>, v_out: Option<&Tensor>, workspace: &Tensor)
                    -> Result<()> {
        let (b, t, hd) = q.dims3()?;
        let Device::Cuda(dev) = q.device() else { candle_core::bail!("b200-attn: not a CUDA tensor") };
        let p = prefix.map(|(pk, _)| pk.dims4().map(|d| d.2)).transpose()?.unwrap_or(0);
        let opt = |x: Option<&Tensor>| -> Result<u64> { x.map(ptr).transpose().map(|p| p.unwrap_or(0)) };
        let args = ffi::AttnArgs {
            batch: b as i32, heads: heads as i32, head_dim: (hd / heads) as i32,
            target_len: t as i32, prefix_len: p as i32,
            q: ptr(q)? as *const c_void, k: ptr(k)? as *const c_void, v: ptr(v)? as *const c_void,
            prefix_k: opt(prefix.map(|x| x.0))? as *const c_void,
            prefix_v: opt(prefix.map(|x| x.1))? as *const c_void,
            norm_q_w: ptr(norm_q_w)? as *const f32, norm_k_w: ptr(norm_k_w)? as *const f32,
            norm_eps: eps, pe: ptr(pe)? as *const f32,
            desc: opt(desc)? as *const ffi::KvDesc, scale,
            out: ptr(out)? as *mut c_void,
            k_rot_out: opt(k_rot_out)? as *mut c_void, v_out: opt(v_out)? as *mut c_void,
            workspace: ptr(workspace)? as *mut c_void,
            workspace_bytes: workspace.elem_count(),
            status: std::ptr::null_mut(), row_limit: std::ptr::null(), pe_batch_stride: 0,
        };
        let stream = dev.cuda_stream();
        // SAFETY: every pointer above comes from a live contiguous CUDA tensor on `dev`.
        let rc = unsafe { ffi::b200_attn_fwd(&args, stream.cu_stream() as *mut c_void) };
        check(rc).map_err(|e| candle_core::Error::Msg(e.to_string()))
    }
}

#[cfg(test)]
mod tests {
    use super::ffi::*;
    use std::mem::{align_of, offset_of, size_of};

    #[test]
    fn layout_matches_header() {
        assert_eq!(size_of::<KvDesc>(), 8);
        assert_eq!(offset_of!(AttnArgs, q), 24);
        assert_eq!(offset_of!(AttnArgs, norm_eps), 80);
        assert_eq!(offset_of!(AttnArgs, workspace_bytes), 144);
        assert_eq!(offset_of!(AttnArgs, pe_batch_stride), 168);
        assert_eq!(size_of::<AttnArgs>(), 176);
        assert_eq!(align_of::<AttnArgs>(), 8);
    }
}
