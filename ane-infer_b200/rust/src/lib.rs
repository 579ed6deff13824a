//! Rust binding of the B200 decode backend: the C ABI of `include/ab2.h`, implemented by
//! `libab2.so`, and a safe [`Decoder`] over it.
//!
//! [`Decoder`] stands in for the reference's Metal decode path:
//! * `GpuContext::new`, `upload_model_weights`, `GpuLayerScratch::new` and
//!   `GpuConstantPool::new` (crates/engine/src/metal_graph.rs:79, gpu_decode.rs:152,
//!   gpu_full_decode.rs:175, :104) are [`Decoder::new`];
//! * `encode_full_token_gpu` (crates/engine/src/gpu_full_decode.rs:221) is
//!   [`Decoder::decode_token`], and its batched form is [`Decoder::decode_step`];
//! * `greedy_sample` (crates/cli/src/main.rs:1767) is the `next` output of the same call.
//!
//! Errors carry the library's negative status code and its message instead of panicking.
//! A decoder owns one CUDA context's worth of state on one GPU. It may move between
//! threads, but it is not shared between them.

use std::ffi::CStr;
use std::fmt;
use std::os::raw::{c_char, c_int};
use std::ptr::NonNull;

/// Raw declarations of `include/ab2.h` (same names, same layouts).
#[allow(non_camel_case_types)]
pub mod ffi {
    use std::os::raw::{c_char, c_int, c_void};

    pub const AB2_OK: c_int = 0;
    pub const AB2_ERR_ARG: c_int = -1;
    pub const AB2_ERR_FORMAT: c_int = -2;
    pub const AB2_ERR_SHAPE: c_int = -3;
    pub const AB2_ERR_OOM: c_int = -4;
    pub const AB2_ERR_CUDA: c_int = -5;
    pub const AB2_ERR_CAPACITY: c_int = -6;
    pub const AB2_ERR_DEVICE: c_int = -7;

    #[repr(C)]
    pub struct ab2_ctx {
        _private: [u8; 0],
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct ab2_options {
        pub kv_bf16: i32,
        pub rope_dims: i32,
        pub exact_max_batch: i32,
        pub reserved: [i32; 5],
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct ab2_config {
        pub dim: i64,
        pub ffn: i64,
        pub n_layers: i64,
        pub vocab: i64,
        pub n_heads: i64,
        pub n_kv_heads: i64,
        pub head_dim: i64,
        pub dn_heads: i64,
        pub dn_state: i64,
        pub conv_kernel: i64,
        pub n_dn: i64,
        pub n_attn: i64,
        pub max_batch: i64,
        pub max_ctx: i64,
        pub context_length: i64,
        pub rope_base: f32,
        pub eps: f32,
        pub kv_bf16: i32,
        pub rope_dims: i32,
    }

    #[link(name = "ab2")]
    extern "C" {
        pub fn ab2_last_error() -> *const c_char;
        pub fn ab2_gguf_inspect(gguf: *const u8, len: u64, out: *mut ab2_config) -> c_int;
        pub fn ab2_create(gguf: *const u8, len: u64, device: c_int, max_batch: c_int, max_ctx: c_int,
                          opt: *const ab2_options, out: *mut *mut ab2_ctx) -> c_int;
        pub fn ab2_destroy(ctx: *mut ab2_ctx);
        pub fn ab2_get_config(ctx: *mut ab2_ctx, out: *mut ab2_config) -> c_int;
        pub fn ab2_layer_is_deltanet(ctx: *mut ab2_ctx, layer: c_int) -> c_int;
        pub fn ab2_reset_slot(ctx: *mut ab2_ctx, slot: c_int) -> c_int;
        pub fn ab2_set_pos(ctx: *mut ab2_ctx, slot: c_int, pos: i64) -> c_int;
        pub fn ab2_get_pos(ctx: *mut ab2_ctx, slot: c_int, pos: *mut i64) -> c_int;
        pub fn ab2_set_dn_state(ctx: *mut ab2_ctx, layer: c_int, slot: c_int, rec: *const f32,
                                conv: *const f32) -> c_int;
        pub fn ab2_get_dn_state(ctx: *mut ab2_ctx, layer: c_int, slot: c_int, rec: *mut f32,
                                conv: *mut f32) -> c_int;
        pub fn ab2_set_kv(ctx: *mut ab2_ctx, layer: c_int, slot: c_int, k: *const f32, v: *const f32,
                          n_tokens: i64) -> c_int;
        pub fn ab2_get_kv(ctx: *mut ab2_ctx, layer: c_int, slot: c_int, k: *mut f32, v: *mut f32,
                          n_tokens: i64) -> c_int;
        pub fn ab2_decode_step(ctx: *mut ab2_ctx, tokens: *const i32, batch: c_int, logits: *mut f32,
                               next_tokens: *mut i32) -> c_int;
        pub fn ab2_prefill(ctx: *mut ab2_ctx, slot: c_int, tokens: *const i32, n: i64, logits: *mut f32,
                           next_token: *mut i32) -> c_int;
        pub fn ab2_decode_step_device(ctx: *mut ab2_ctx, tokens_dev: *const i32, batch: c_int,
                                      logits_dev: *mut f32, next_dev: *mut i32, stream: *mut c_void) -> c_int;
        pub fn ab2_sync(ctx: *mut ab2_ctx) -> c_int;
        pub fn ab2_step_graph(ctx: *mut ab2_ctx, enable: c_int) -> c_int;
        pub fn ab2_mixer_layer(ctx: *mut ab2_ctx, layer: c_int, slot: c_int, x: *const f32, out: *mut f32) -> c_int;
        pub fn ab2_ffn_layer(ctx: *mut ab2_ctx, layer: c_int, x: *const f32, out: *mut f32) -> c_int;
    }
}

/// A failed call: the library's negative status code (`ffi::AB2_ERR_*`) and its message.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Error {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for Error {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "ab2 error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

fn last_error() -> String {
    // SAFETY: ab2_last_error returns a NUL-terminated thread-local string ("" when none).
    let p: *const c_char = unsafe { ffi::ab2_last_error() };
    if p.is_null() {
        return String::new();
    }
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}

fn check(rc: c_int) -> Result<()> {
    if rc == ffi::AB2_OK {
        Ok(())
    } else {
        Err(Error { code: rc, message: last_error() })
    }
}

fn arg_error(message: String) -> Error {
    Error { code: ffi::AB2_ERR_ARG, message }
}

/// Model configuration read from a GGUF (`Qwen35Config::from_gguf`, crates/engine/src/model.rs:70).
pub type Config = ffi::ab2_config;

/// Parse GGUF bytes on the host and derive the model configuration (no GPU needed).
pub fn inspect(gguf: &[u8]) -> Result<Config> {
    let mut cfg = Config::default();
    check(unsafe { ffi::ab2_gguf_inspect(gguf.as_ptr(), gguf.len() as u64, &mut cfg) })?;
    Ok(cfg)
}

/// Context options: the KV cache type and the rotated dims per head.
#[derive(Clone, Copy, Debug)]
pub struct Options {
    /// bf16 KV cache (default); false stores f32 like the reference.
    pub kv_bf16: bool,
    /// Rotated dims per head; 0 means all of head_dim, as the reference does.
    pub rope_dims: i32,
}

impl Default for Options {
    fn default() -> Self {
        Options { kv_bf16: true, rope_dims: 0 }
    }
}

/// Decode state for up to `max_batch` sequences (slots) of up to `max_ctx` tokens on one GPU.
pub struct Decoder {
    ctx: NonNull<ffi::ab2_ctx>,
    cfg: Config,
}

// SAFETY: a context may be driven from any one thread at a time (include/ab2.h, Threading).
unsafe impl Send for Decoder {}

impl Decoder {
    /// Load a qwen35 GGUF (Q8_0 weights) onto `device` and allocate state for `max_batch`
    /// sequences of up to `max_ctx` tokens.
    pub fn new(gguf: &[u8], device: i32, max_batch: i32, max_ctx: i32, opt: &Options) -> Result<Self> {
        let o = ffi::ab2_options { kv_bf16: opt.kv_bf16 as i32, rope_dims: opt.rope_dims, exact_max_batch: 0, reserved: [0; 5] };
        let mut raw: *mut ffi::ab2_ctx = std::ptr::null_mut();
        check(unsafe { ffi::ab2_create(gguf.as_ptr(), gguf.len() as u64, device, max_batch, max_ctx, &o, &mut raw) })?;
        let ctx = NonNull::new(raw).ok_or_else(|| arg_error("ab2_create returned no context".into()))?;
        // owned from here on: an error below drops it, which destroys the context
        let mut d = Decoder { ctx, cfg: Config::default() };
        check(unsafe { ffi::ab2_get_config(d.ctx.as_ptr(), &mut d.cfg) })?;
        Ok(d)
    }

    /// The model configuration, with this context's max_batch, max_ctx and KV type.
    pub fn config(&self) -> &Config {
        &self.cfg
    }

    fn raw(&mut self) -> *mut ffi::ab2_ctx {
        self.ctx.as_ptr()
    }

    /// Replay each decode step from a captured CUDA graph (one capture per launch plan).
    pub fn set_step_graph(&mut self, enable: bool) -> Result<()> {
        check(unsafe { ffi::ab2_step_graph(self.raw(), enable as c_int) })
    }

    /// Start a fresh sequence in `slot` (`HybridCache::new`, crates/engine/src/deltanet_cache.rs:76).
    pub fn reset_slot(&mut self, slot: i32) -> Result<()> {
        check(unsafe { ffi::ab2_reset_slot(self.raw(), slot) })
    }

    /// Position of the next token of `slot`.
    pub fn pos(&mut self, slot: i32) -> Result<i64> {
        let mut p = 0i64;
        check(unsafe { ffi::ab2_get_pos(self.raw(), slot, &mut p) })?;
        Ok(p)
    }

    pub fn set_pos(&mut self, slot: i32, pos: i64) -> Result<()> {
        check(unsafe { ffi::ab2_set_pos(self.raw(), slot, pos) })
    }

    /// One greedy decode step for slots 0..tokens.len(): each slot takes its token and
    /// advances one position. `logits` gets [batch][vocab], `next` the greedy ids.
    pub fn decode_step(&mut self, tokens: &[i32], logits: Option<&mut [f32]>, next: Option<&mut [i32]>) -> Result<()> {
        let b = tokens.len();
        let vocab = self.cfg.vocab as usize;
        if let Some(l) = logits.as_ref() {
            if l.len() != b * vocab {
                return Err(arg_error(format!("logits holds {} floats, expected {}", l.len(), b * vocab)));
            }
        }
        if let Some(n) = next.as_ref() {
            if n.len() != b {
                return Err(arg_error(format!("next holds {} ids, expected {}", n.len(), b)));
            }
        }
        let lp = logits.map_or(std::ptr::null_mut(), |l| l.as_mut_ptr());
        let np = next.map_or(std::ptr::null_mut(), |n| n.as_mut_ptr());
        check(unsafe { ffi::ab2_decode_step(self.raw(), tokens.as_ptr(), b as c_int, lp, np) })
    }

    /// The prompt loop of `cmd_bench` (`crates/cli/src/main.rs:358-362`) on the GPU: every
    /// prompt token of `slot` in one call; returns the last token's logits and greedy id.
    pub fn prefill(&mut self, slot: usize, tokens: &[u32]) -> Result<(Vec<f32>, u32)> {
        let ids: Vec<i32> = tokens.iter().map(|&t| t as i32).collect();
        let mut logits = vec![0f32; self.cfg.vocab as usize];
        let mut next = 0i32;
        check(unsafe {
            ffi::ab2_prefill(self.raw(), slot as c_int, ids.as_ptr(), ids.len() as i64, logits.as_mut_ptr(), &mut next)
        })?;
        Ok((logits, next as u32))
    }

    /// `encode_full_token_gpu` for one sequence (slot 0): token in, logits out.
    pub fn decode_token(&mut self, token_id: u32) -> Result<Vec<f32>> {
        let mut logits = vec![0f32; self.cfg.vocab as usize];
        self.decode_step(&[token_id as i32], Some(logits.as_mut_slice()), None)?;
        Ok(logits)
    }

    /// Batched greedy step: the next id of every slot; the logits stay on the device.
    pub fn decode_greedy(&mut self, tokens: &[i32]) -> Result<Vec<i32>> {
        let mut next = vec![0i32; tokens.len()];
        self.decode_step(tokens, None, Some(next.as_mut_slice()))?;
        Ok(next)
    }

    /// Recurrent state [dn_heads][dn_state][dn_state] and conv state [3·dim][conv_kernel] of
    /// a DeltaNet layer (`DeltaNetLayerState`, crates/engine/src/deltanet_cache.rs:5-65);
    /// either may be left out.
    pub fn set_dn_state(&mut self, layer: i32, slot: i32, rec: Option<&[f32]>, conv: Option<&[f32]>) -> Result<()> {
        let c = self.cfg;
        let (nr, nc) = ((c.dn_heads * c.dn_state * c.dn_state) as usize, (3 * c.dim * c.conv_kernel) as usize);
        if rec.map_or(false, |r| r.len() != nr) || conv.map_or(false, |v| v.len() != nc) {
            return Err(arg_error(format!("DeltaNet state sizes: recurrent {nr}, conv {nc} floats")));
        }
        let rp = rec.map_or(std::ptr::null(), |r| r.as_ptr());
        let cp = conv.map_or(std::ptr::null(), |v| v.as_ptr());
        check(unsafe { ffi::ab2_set_dn_state(self.raw(), layer, slot, rp, cp) })
    }

    /// K and V of an attention layer for positions 0..n_tokens, each [n_kv_heads][n_tokens]
    /// [head_dim] (`LayerKvCache::write_range`, crates/engine/src/kv_cache.rs:43-67).
    pub fn set_kv(&mut self, layer: i32, slot: i32, k: &[f32], v: &[f32], n_tokens: i64) -> Result<()> {
        let n = (self.cfg.n_kv_heads * n_tokens * self.cfg.head_dim) as usize;
        if n_tokens < 0 || k.len() != n || v.len() != n {
            return Err(arg_error(format!("K and V must hold {n} floats each")));
        }
        check(unsafe { ffi::ab2_set_kv(self.raw(), layer, slot, k.as_ptr(), v.as_ptr(), n_tokens) })
    }

    /// Wait for queued device work and report a timed-out device pipeline wait, if any.
    pub fn sync(&mut self) -> Result<()> {
        check(unsafe { ffi::ab2_sync(self.raw()) })
    }
}

impl Drop for Decoder {
    fn drop(&mut self) {
        unsafe { ffi::ab2_destroy(self.ctx.as_ptr()) }
    }
}

#[cfg(test)]
mod tests {
    use super::*;

    #[test]
    fn layouts_match_the_header() {
        assert_eq!(std::mem::size_of::<ffi::ab2_options>(), 32);
        assert_eq!(std::mem::size_of::<ffi::ab2_config>(), 15 * 8 + 4 * 4);
    }

    #[test]
    fn inspect_rejects_a_non_gguf_buffer() {
        let e = inspect(b"NOPE\0\0\0\0\0\0\0\0").unwrap_err();
        assert_eq!(e.code, ffi::AB2_ERR_FORMAT);
        assert!(e.message.contains("magic"), "{}", e.message);
    }

    #[test]
    fn create_rejects_a_zero_batch_before_touching_a_gpu() {
        let e = Decoder::new(b"", 0, 0, 16, &Options::default()).err().expect("max_batch 0 must fail");
        assert_eq!(e.code, ffi::AB2_ERR_ARG);
    }
}
