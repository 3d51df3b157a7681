//! Safe wrapper over `qora-mixer-sys` for the reference engine
//! (qora-protocol/QORA-LLM-4B).
//!
//! The handle types stand in for the reference's per-layer caches:
//! * [`DnStateHandle`] for `DeltaNetState` (src/gemv.rs:133-157) — B sequences'
//!   S [32,128,128] f32, conv history and conv_pos on the device;
//! * [`KvHandle`] for `KvCacheEntry` (src/gemv.rs:164-168) — a preallocated
//!   bf16 K/V cache [B,4,capacity,256] appended in place;
//! * [`HybridCache`] for the reference's `HybridCache` (src/gemv.rs:171-231)
//!   with `snapshot` / `restore_from`; a layer-kind mismatch is
//!   `QM_E_MISMATCH` instead of the reference's `panic!` (gemv.rs:228).
//!
//! Every handle owns its device storage and destroys it in `Drop`.  Calls
//! return `Result<(), QmError>` built from the status and `qm_last_error`.
//! `Mixer` methods taking slices are the `_host` entry points (host memory,
//! synchronous, like the reference's `Vec<f32>` functions); the `unsafe`
//! `*_device` methods take device pointers on the context's stream.
use core::ffi::{c_int, c_void, CStr};
use core::marker::PhantomData;
use core::ptr::{null, null_mut};
use qora_mixer_sys as sys;

/// A non-zero status of the library and the context's description of it.
#[derive(Debug, Clone)]
pub struct QmError {
    pub code: i32,
    pub message: String,
}

impl core::fmt::Display for QmError {
    fn fmt(&self, f: &mut core::fmt::Formatter<'_>) -> core::fmt::Result {
        write!(f, "qora_mixer status {}: {}", self.code, self.message)
    }
}

impl std::error::Error for QmError {}

pub type Result<T> = core::result::Result<T, QmError>;

fn status_text(code: c_int) -> String {
    // SAFETY: qm_status_string returns a static NUL-terminated string.
    unsafe { CStr::from_ptr(sys::qm_status_string(code)) }.to_string_lossy().into_owned()
}

fn plain(code: c_int) -> Result<()> {
    if code == sys::QM_OK {
        Ok(())
    } else {
        Err(QmError { code, message: status_text(code) })
    }
}

/// Mixer shape constants (`Qor4bConfig::default_4b`, src/config.rs:42-79).
pub fn shape() -> Result<sys::qm_shape> {
    let mut s = sys::qm_shape::default();
    plain(unsafe { sys::qm_shape_get(&mut s) })?;
    Ok(s)
}

/// The RoPE tables of src/convert.rs:161-176 (same f32 formula) for
/// `max_pos` positions; the reference stops at 8192.
pub fn rope_table(theta: f32, rope_dim: i32, max_pos: i32) -> Result<(Vec<f32>, Vec<f32>)> {
    let n = (max_pos.max(0) as usize) * (rope_dim.max(0) as usize / 2);
    let (mut c, mut s) = (vec![0.0f32; n], vec![0.0f32; n]);
    plain(unsafe { sys::qm_rope_table(theta, rope_dim, max_pos, c.as_mut_ptr(), s.as_mut_ptr()) })?;
    Ok((c, s))
}

/// One device and one CUDA stream (the reference drives its GPU from one
/// thread, src/gpu_inference.rs:946-953).  Not `Sync`: calls on a context
/// must be serialised.
pub struct Context {
    raw: *mut sys::qm_ctx,
}

impl Context {
    /// Fails with `QM_E_UNSUPPORTED` unless the device is compute capability 10.x.
    pub fn new(device: i32) -> Result<Self> {
        let mut raw = null_mut();
        plain(unsafe { sys::qm_ctx_create(device, &mut raw) })?;
        Ok(Self { raw })
    }

    pub fn as_raw(&self) -> *mut sys::qm_ctx {
        self.raw
    }

    fn check(&self, code: c_int) -> Result<()> {
        if code == sys::QM_OK {
            return Ok(());
        }
        // SAFETY: the context is alive; the string is copied before any other call.
        let msg = unsafe { CStr::from_ptr(sys::qm_last_error(self.raw)) }.to_string_lossy().into_owned();
        Err(QmError { code, message: if msg.is_empty() { status_text(code) } else { msg } })
    }

    /// Runs later calls on `stream` (a `cudaStream_t`; null = legacy default stream).
    ///
    /// # Safety
    /// `stream` must be a live stream on the context's device.
    pub unsafe fn set_stream(&self, stream: *mut c_void) -> Result<()> {
        self.check(sys::qm_ctx_set_stream(self.raw, stream))
    }

    pub fn stream(&self) -> *mut c_void {
        unsafe { sys::qm_ctx_get_stream(self.raw) }
    }

    /// Waits for the stream; a device-side wait that gave up is `QM_E_TIMEOUT`.
    pub fn sync(&self) -> Result<()> {
        self.check(unsafe { sys::qm_sync(self.raw) })
    }

    /// Grows the workspace now so later calls never allocate (CUDA graphs).
    pub fn reserve(&self, bytes: usize) -> Result<()> {
        self.check(unsafe { sys::qm_ctx_reserve(self.raw, bytes) })
    }

    pub fn set_host_parts(&self, dn_parts: i32, gqa_parts: i32) -> Result<()> {
        self.check(unsafe { sys::qm_ctx_set_host_parts(self.raw, dn_parts, gqa_parts) })
    }

    pub fn set_host_direct(&self, on: bool) -> Result<()> {
        self.check(unsafe { sys::qm_ctx_set_host_direct(self.raw, on as c_int) })
    }

    /// (`_host` calls that ran in place on page-locked memory, calls that were staged).
    pub fn host_calls(&self) -> Result<(i64, i64)> {
        let (mut a, mut b) = (0i64, 0i64);
        self.check(unsafe { sys::qm_ctx_host_calls(self.raw, &mut a, &mut b) })?;
        Ok((a, b))
    }

    pub fn launch_count(&self) -> i64 {
        unsafe { sys::qm_ctx_launch_count(self.raw) }
    }

    pub fn set_timing(&self, on: bool) -> Result<()> {
        self.check(unsafe { sys::qm_ctx_set_timing(self.raw, on as c_int) })
    }

    /// Summed device time (ms) and launch count of kernel `name` while timing was on.
    pub fn kernel_time(&self, name: &CStr) -> Result<(f64, i64)> {
        let (mut ms, mut n) = (0.0f64, 0i64);
        self.check(unsafe { sys::qm_ctx_kernel_time(self.raw, name.as_ptr(), &mut ms, &mut n) })?;
        Ok((ms, n))
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            sys::qm_ctx_destroy(self.raw);
        }
    }
}

/// `DeltaNetState` for `batch` sequences advancing together
/// (`DeltaNetState::new`, src/gemv.rs:144-157: all zero).
pub struct DnStateHandle<'c> {
    raw: *mut sys::qm_dn_state,
    ctx: &'c Context,
}

impl<'c> DnStateHandle<'c> {
    pub fn new(ctx: &'c Context, batch: i32) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(unsafe { sys::qm_dn_state_create(ctx.raw, batch, &mut raw) })?;
        Ok(Self { raw, ctx })
    }

    /// The V heads [vh_lo, vh_lo + nvh) of every sequence (head-sharded decode).
    pub fn new_heads(ctx: &'c Context, batch: i32, vh_lo: i32, nvh: i32) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(unsafe { sys::qm_dn_state_create_heads(ctx.raw, batch, vh_lo, nvh, &mut raw) })?;
        Ok(Self { raw, ctx })
    }

    /// Over caller-owned device storage: s [B,32,128,128] f32, conv [B,4,8192] f32.
    ///
    /// # Safety
    /// Both pointers must stay valid device memory for the handle's lifetime.
    pub unsafe fn wrap(ctx: &'c Context, batch: i32, s: *mut f32, conv: *mut f32) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(sys::qm_dn_state_wrap(ctx.raw, batch, s, conv, &mut raw))?;
        Ok(Self { raw, ctx })
    }

    /// # Safety
    /// As [`DnStateHandle::wrap`], for the V heads [vh_lo, vh_lo + nvh).
    pub unsafe fn wrap_heads(
        ctx: &'c Context,
        batch: i32,
        vh_lo: i32,
        nvh: i32,
        s: *mut f32,
        conv: *mut f32,
    ) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(sys::qm_dn_state_wrap_heads(ctx.raw, batch, vh_lo, nvh, s, conv, &mut raw))?;
        Ok(Self { raw, ctx })
    }

    pub fn as_raw(&self) -> *mut sys::qm_dn_state {
        self.raw
    }

    pub fn batch(&self) -> i32 {
        unsafe { sys::qm_dn_state_batch(self.raw) }
    }

    pub fn heads(&self) -> Result<(i32, i32)> {
        let (mut lo, mut n) = (0, 0);
        self.ctx.check(unsafe { sys::qm_dn_state_heads(self.raw, &mut lo, &mut n) })?;
        Ok((lo, n))
    }

    pub fn conv_pos(&self) -> i64 {
        unsafe { sys::qm_dn_state_conv_pos(self.raw) }
    }

    pub fn set_conv_pos(&mut self, conv_pos: i64) -> Result<()> {
        self.ctx.check(unsafe { sys::qm_dn_state_set_conv_pos(self.raw, conv_pos) })
    }

    pub fn reset(&mut self) -> Result<()> {
        self.ctx.check(unsafe { sys::qm_dn_state_reset(self.ctx.raw, self.raw) })
    }

    /// Deep copy (`HybridCache::snapshot`, src/gemv.rs:198-212).
    pub fn snapshot(&self) -> Result<DnStateHandle<'c>> {
        let mut raw = null_mut();
        self.ctx.check(unsafe { sys::qm_dn_state_snapshot(self.ctx.raw, self.raw, &mut raw) })?;
        Ok(Self { raw, ctx: self.ctx })
    }

    /// Copy `src` in (`HybridCache::restore_from`, src/gemv.rs:215-231).
    pub fn restore_from(&mut self, src: &DnStateHandle<'_>) -> Result<()> {
        self.ctx.check(unsafe { sys::qm_dn_state_restore(self.ctx.raw, self.raw, src.raw) })
    }

    /// Sequence `b` in the reference layout: s [nvh*128*128], conv_buf [8192*3].
    pub fn read(&self, b: i32, s: &mut [f32], conv_buf: &mut [f32]) -> Result<()> {
        let (_, nvh) = self.heads()?;
        if s.len() < nvh as usize * 128 * 128 || conv_buf.len() < 8192 * 3 {
            return Err(QmError { code: sys::QM_E_SHAPE, message: "read: buffers too small".into() });
        }
        self.ctx.check(unsafe {
            sys::qm_dn_state_read(self.ctx.raw, self.raw, b, s.as_mut_ptr(), conv_buf.as_mut_ptr())
        })
    }

    pub fn write(&mut self, b: i32, s: Option<&[f32]>, conv_buf: Option<&[f32]>) -> Result<()> {
        let (_, nvh) = self.heads()?;
        if s.map_or(false, |x| x.len() < nvh as usize * 128 * 128)
            || conv_buf.map_or(false, |x| x.len() < 8192 * 3)
        {
            return Err(QmError { code: sys::QM_E_SHAPE, message: "write: buffers too small".into() });
        }
        self.ctx.check(unsafe {
            sys::qm_dn_state_write(
                self.ctx.raw,
                self.raw,
                b,
                s.map_or(null(), |x| x.as_ptr()),
                conv_buf.map_or(null(), |x| x.as_ptr()),
            )
        })
    }

    /// Raw device storage (S, conv ring of 4 slots).
    pub fn data(&self) -> Result<(*mut f32, *mut f32)> {
        let (mut s, mut c) = (null_mut(), null_mut());
        self.ctx.check(unsafe { sys::qm_dn_state_data(self.raw, &mut s, &mut c) })?;
        Ok((s, c))
    }
}

impl Drop for DnStateHandle<'_> {
    fn drop(&mut self) {
        unsafe {
            sys::qm_dn_state_destroy(self.raw);
        }
    }
}

/// `KvCacheEntry` for `batch` sequences: bf16 K/V [B,4,capacity,256].
pub struct KvHandle<'c> {
    raw: *mut sys::qm_kv,
    ctx: &'c Context,
}

impl<'c> KvHandle<'c> {
    pub fn new(ctx: &'c Context, batch: i32, capacity: i32) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(unsafe { sys::qm_kv_create(ctx.raw, batch, capacity, &mut raw) })?;
        Ok(Self { raw, ctx })
    }

    /// KV heads [kv_lo, kv_lo + nkv) (head-sharded decode).
    pub fn new_heads(ctx: &'c Context, batch: i32, capacity: i32, kv_lo: i32, nkv: i32) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(unsafe { sys::qm_kv_create_heads(ctx.raw, batch, capacity, kv_lo, nkv, &mut raw) })?;
        Ok(Self { raw, ctx })
    }

    /// # Safety
    /// `k` and `v` must stay valid device memory of bf16 [batch,4,capacity,256].
    pub unsafe fn wrap(ctx: &'c Context, batch: i32, capacity: i32, k: *mut u16, v: *mut u16) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(sys::qm_kv_wrap(ctx.raw, batch, capacity, k, v, &mut raw))?;
        Ok(Self { raw, ctx })
    }

    /// # Safety
    /// As [`KvHandle::wrap`], for KV heads [kv_lo, kv_lo + nkv).
    pub unsafe fn wrap_heads(
        ctx: &'c Context,
        batch: i32,
        capacity: i32,
        kv_lo: i32,
        nkv: i32,
        k: *mut u16,
        v: *mut u16,
    ) -> Result<Self> {
        let mut raw = null_mut();
        ctx.check(sys::qm_kv_wrap_heads(ctx.raw, batch, capacity, kv_lo, nkv, k, v, &mut raw))?;
        Ok(Self { raw, ctx })
    }

    pub fn as_raw(&self) -> *mut sys::qm_kv {
        self.raw
    }

    pub fn seq_len(&self) -> i64 {
        unsafe { sys::qm_kv_seq_len(self.raw) }
    }

    pub fn set_seq_len(&mut self, seq_len: i64) -> Result<()> {
        self.ctx.check(unsafe { sys::qm_kv_set_seq_len(self.raw, seq_len) })
    }

    pub fn capacity(&self) -> i32 {
        unsafe { sys::qm_kv_capacity(self.raw) }
    }

    pub fn batch(&self) -> i32 {
        unsafe { sys::qm_kv_batch(self.raw) }
    }

    pub fn heads(&self) -> Result<(i32, i32)> {
        let (mut lo, mut n) = (0, 0);
        self.ctx.check(unsafe { sys::qm_kv_heads(self.raw, &mut lo, &mut n) })?;
        Ok((lo, n))
    }

    pub fn data(&self) -> Result<(*mut u16, *mut u16)> {
        let (mut k, mut v) = (null_mut(), null_mut());
        self.ctx.check(unsafe { sys::qm_kv_data(self.raw, &mut k, &mut v) })?;
        Ok((k, v))
    }

    pub fn snapshot(&self) -> Result<KvHandle<'c>> {
        let mut raw = null_mut();
        self.ctx.check(unsafe { sys::qm_kv_snapshot(self.ctx.raw, self.raw, &mut raw) })?;
        Ok(Self { raw, ctx: self.ctx })
    }

    pub fn restore_from(&mut self, src: &KvHandle<'_>) -> Result<()> {
        self.ctx.check(unsafe { sys::qm_kv_restore(self.ctx.raw, self.raw, src.raw) })
    }
}

impl Drop for KvHandle<'_> {
    fn drop(&mut self) {
        unsafe {
            sys::qm_kv_destroy(self.raw);
        }
    }
}

/// One layer's cache (`CacheEntry`, src/gemv.rs:177-180).
pub enum CacheEntry<'c> {
    DeltaNet(DnStateHandle<'c>),
    KvCache(KvHandle<'c>),
}

/// `HybridCache` (src/gemv.rs:171-231): one entry per layer.
pub struct HybridCache<'c> {
    pub entries: Vec<CacheEntry<'c>>,
}

impl<'c> HybridCache<'c> {
    /// `is_attn[i]` selects a KV cache for layer i (LayerType::FullAttn), else a DeltaNet state.
    pub fn new(ctx: &'c Context, is_attn: &[bool], batch: i32, capacity: i32) -> Result<Self> {
        let mut entries = Vec::with_capacity(is_attn.len());
        for &attn in is_attn {
            entries.push(if attn {
                CacheEntry::KvCache(KvHandle::new(ctx, batch, capacity)?)
            } else {
                CacheEntry::DeltaNet(DnStateHandle::new(ctx, batch)?)
            });
        }
        Ok(Self { entries })
    }

    pub fn snapshot(&self) -> Result<HybridCache<'c>> {
        let mut entries = Vec::with_capacity(self.entries.len());
        for e in &self.entries {
            entries.push(match e {
                CacheEntry::DeltaNet(d) => CacheEntry::DeltaNet(d.snapshot()?),
                CacheEntry::KvCache(k) => CacheEntry::KvCache(k.snapshot()?),
            });
        }
        Ok(Self { entries })
    }

    /// `QM_E_MISMATCH` where the reference panics (src/gemv.rs:228).
    pub fn restore_from(&mut self, src: &HybridCache<'_>) -> Result<()> {
        if self.entries.len() != src.entries.len() {
            return Err(QmError { code: sys::QM_E_MISMATCH, message: "layer count differs".into() });
        }
        for (d, s) in self.entries.iter_mut().zip(src.entries.iter()) {
            match (d, s) {
                (CacheEntry::DeltaNet(d), CacheEntry::DeltaNet(s)) => d.restore_from(s)?,
                (CacheEntry::KvCache(d), CacheEntry::KvCache(s)) => d.restore_from(s)?,
                _ => {
                    return Err(QmError {
                        code: sys::QM_E_MISMATCH,
                        message: "cache type mismatch during restore".into(),
                    })
                }
            }
        }
        Ok(())
    }
}

/// DeltaNet layer parameters: device pointers kept alive by the caller.
#[derive(Clone, Copy)]
pub struct DnParams<'a> {
    raw: sys::qm_dn_params,
    _life: PhantomData<&'a ()>,
}

impl<'a> DnParams<'a> {
    /// # Safety
    /// Device pointers on the context's device: conv_w [8192*4], a_log [32],
    /// dt_bias [32], norm_gamma [128] (may be null when no call fuses the gate).
    pub unsafe fn new(conv_w: *const f32, a_log: *const f32, dt_bias: *const f32, norm_gamma: *const f32) -> Self {
        Self { raw: sys::qm_dn_params { conv_w, a_log, dt_bias, norm_gamma }, _life: PhantomData }
    }
}

/// GQA layer parameters: device pointers kept alive by the caller.
#[derive(Clone, Copy)]
pub struct GqaParams<'a> {
    raw: sys::qm_gqa_params,
    _life: PhantomData<&'a ()>,
}

impl<'a> GqaParams<'a> {
    /// # Safety
    /// Device pointers: q_norm, k_norm [256]; rope_cos, rope_sin [max_pos*32].
    pub unsafe fn new(
        q_norm: *const f32,
        k_norm: *const f32,
        rope_cos: *const f32,
        rope_sin: *const f32,
        max_pos: i32,
    ) -> Self {
        Self { raw: sys::qm_gqa_params { q_norm, k_norm, rope_cos, rope_sin, max_pos }, _life: PhantomData }
    }
}

fn need(buf_len: usize, want: usize, what: &str) -> Result<()> {
    if buf_len < want {
        Err(QmError { code: sys::QM_E_SHAPE, message: format!("{what}: {buf_len} < {want} elements") })
    } else {
        Ok(())
    }
}

/// The mixer calls of one context.
pub struct Mixer<'c> {
    ctx: &'c Context,
}

impl<'c> Mixer<'c> {
    pub fn new(ctx: &'c Context) -> Self {
        Self { ctx }
    }

    /// `forward_deltanet_decode`'s mixer region (src/gemv.rs:744-883) on host
    /// buffers: qkv [B*8192], a, b [B*32]; with `z` [B*4096], `out` [B*4096]
    /// receives the gated output (the input of out_proj), else `y` [B*4096].
    pub fn dn_decode_host(
        &self,
        p: &DnParams<'_>,
        st: &mut DnStateHandle<'_>,
        qkv: &[f32],
        a: &[f32],
        b: &[f32],
        z: Option<&[f32]>,
        out: &mut [f32],
    ) -> Result<()> {
        let bsz = st.batch() as usize;
        need(qkv.len(), bsz * 8192, "qkv")?;
        need(a.len(), bsz * 32, "a")?;
        need(b.len(), bsz * 32, "b")?;
        need(out.len(), bsz * 4096, "out")?;
        if let Some(z) = z {
            need(z.len(), bsz * 4096, "z")?;
        }
        let (y, zp, o) = match z {
            Some(z) => (null_mut(), z.as_ptr(), out.as_mut_ptr()),
            None => (out.as_mut_ptr(), null(), null_mut()),
        };
        self.ctx.check(unsafe {
            sys::qm_dn_decode_host(self.ctx.raw, &p.raw, st.raw, qkv.as_ptr(), a.as_ptr(), b.as_ptr(), y, zp, o)
        })
    }

    /// Device-pointer form of [`Mixer::dn_decode_host`], asynchronous on the context stream.
    ///
    /// # Safety
    /// Every pointer is device memory of the documented size (or null where allowed).
    pub unsafe fn dn_decode_device(
        &self,
        p: &DnParams<'_>,
        st: &mut DnStateHandle<'_>,
        qkv: *const f32,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> Result<()> {
        self.ctx.check(sys::qm_dn_decode(self.ctx.raw, &p.raw, st.raw, qkv, a, b, y, z, out))
    }

    /// `prefill_deltanet_layer`'s loop (src/gemv.rs:1119-1219) for `t` tokens.
    ///
    /// # Safety
    /// Device pointers: qkv bf16 [B*t*8192], a, b [B*t*32], y [B*t*4096];
    /// z and out [B*t*4096] or both null.
    pub unsafe fn dn_prefill_device(
        &self,
        p: &DnParams<'_>,
        st: &mut DnStateHandle<'_>,
        t: i32,
        qkv_bf16: *const u16,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> Result<()> {
        self.ctx.check(sys::qm_dn_prefill(self.ctx.raw, &p.raw, st.raw, t, qkv_bf16, a, b, y, z, out))
    }

    /// `prefill_deltanet_layer`'s loop on host buffers (the reference's GPU
    /// prefill flow, src/gpu_inference.rs:464-604): qkv bf16 bits
    /// [B*t*8192], a, b [B*t*32], y [B*t*4096]; with `z_out`, the gated
    /// output (z [B*t*4096] in, out [B*t*4096]).
    pub fn dn_prefill_host(
        &self,
        p: &DnParams<'_>,
        st: &mut DnStateHandle<'_>,
        t: i32,
        qkv_bf16: &[u16],
        a: &[f32],
        b: &[f32],
        y: &mut [f32],
        z_out: Option<(&[f32], &mut [f32])>,
    ) -> Result<()> {
        let n = st.batch() as usize * t.max(0) as usize;
        need(qkv_bf16.len(), n * 8192, "qkv")?;
        need(a.len(), n * 32, "a")?;
        need(b.len(), n * 32, "b")?;
        need(y.len(), n * 4096, "y")?;
        let (zp, op) = match z_out {
            Some((z, out)) => {
                need(z.len(), n * 4096, "z")?;
                need(out.len(), n * 4096, "out")?;
                (z.as_ptr(), out.as_mut_ptr())
            }
            None => (null(), null_mut()),
        };
        self.ctx.check(unsafe {
            sys::qm_dn_prefill_host(
                self.ctx.raw,
                &p.raw,
                st.raw,
                t,
                qkv_bf16.as_ptr(),
                a.as_ptr(),
                b.as_ptr(),
                y.as_mut_ptr(),
                zp,
                op,
            )
        })
    }

    /// `forward_attn_decode`'s attention region (src/gemv.rs:927-1011) on
    /// host buffers: q_gate [B*16*512], k_new, v_new [B*4*256], out [B*16*256].
    pub fn gqa_decode_host(
        &self,
        p: &GqaParams<'_>,
        kv: &mut KvHandle<'_>,
        q_gate: &[f32],
        k_new: &[f32],
        v_new: &[f32],
        out: &mut [f32],
    ) -> Result<()> {
        let bsz = kv.batch() as usize;
        need(q_gate.len(), bsz * 16 * 512, "q_gate")?;
        need(k_new.len(), bsz * 4 * 256, "k_new")?;
        need(v_new.len(), bsz * 4 * 256, "v_new")?;
        need(out.len(), bsz * 16 * 256, "out")?;
        self.ctx.check(unsafe {
            sys::qm_gqa_decode_host(
                self.ctx.raw,
                &p.raw,
                kv.raw,
                q_gate.as_ptr(),
                k_new.as_ptr(),
                v_new.as_ptr(),
                out.as_mut_ptr(),
            )
        })
    }

    /// # Safety
    /// Device pointers of the sizes of [`Mixer::gqa_decode_host`].
    pub unsafe fn gqa_decode_device(
        &self,
        p: &GqaParams<'_>,
        kv: &mut KvHandle<'_>,
        q_gate: *const f32,
        k_new: *const f32,
        v_new: *const f32,
        out: *mut f32,
    ) -> Result<()> {
        self.ctx.check(sys::qm_gqa_decode(self.ctx.raw, &p.raw, kv.raw, q_gate, k_new, v_new, out))
    }

    /// `prefill_attn_layer`'s attention region on host buffers (bf16 bits):
    /// q_gate [B*t*16*512], k, v [B*t*4*256]; out [B*t*16*256] f32.
    pub fn gqa_prefill_host(
        &self,
        p: &GqaParams<'_>,
        kv: &mut KvHandle<'_>,
        t: i32,
        q_gate_bf16: &[u16],
        k_bf16: &[u16],
        v_bf16: &[u16],
        out: &mut [f32],
    ) -> Result<()> {
        let n = kv.batch() as usize * t.max(0) as usize;
        need(q_gate_bf16.len(), n * 16 * 512, "q_gate")?;
        need(k_bf16.len(), n * 4 * 256, "k")?;
        need(v_bf16.len(), n * 4 * 256, "v")?;
        need(out.len(), n * 16 * 256, "out")?;
        self.ctx.check(unsafe {
            sys::qm_gqa_prefill_host(
                self.ctx.raw,
                &p.raw,
                kv.raw,
                t,
                q_gate_bf16.as_ptr(),
                k_bf16.as_ptr(),
                v_bf16.as_ptr(),
                out.as_mut_ptr(),
            )
        })
    }

    /// T sequential decode steps in one launch (device pointers; see `qm_dn_decode_seq`).
    ///
    /// # Safety
    /// Device pointers: qkv [B*t*8192] (16-byte aligned), a, b [B*t*32],
    /// y [B*t*nvh*128] or null when out is given; z [B*t*4096] and out, or both null.
    pub unsafe fn dn_decode_seq_device(
        &self,
        p: &DnParams<'_>,
        st: &mut DnStateHandle<'_>,
        t: i32,
        qkv: *const f32,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> Result<()> {
        self.ctx.check(sys::qm_dn_decode_seq(self.ctx.raw, &p.raw, st.raw, t, qkv, a, b, y, z, out))
    }

    /// `prefill_attn_layer`'s attention region (src/gemv.rs:1364-1444); it
    /// replaces the cache contents with the prompt's K/V.
    ///
    /// # Safety
    /// Device pointers: q_gate bf16 [B*t*16*512], k, v bf16 [B*t*4*256], out [B*t*16*256].
    pub unsafe fn gqa_prefill_device(
        &self,
        p: &GqaParams<'_>,
        kv: &mut KvHandle<'_>,
        t: i32,
        q_gate_bf16: *const u16,
        k_bf16: *const u16,
        v_bf16: *const u16,
        out: *mut f32,
    ) -> Result<()> {
        self.ctx.check(sys::qm_gqa_prefill(self.ctx.raw, &p.raw, kv.raw, t, q_gate_bf16, k_bf16, v_bf16, out))
    }
}

/// GQA decode without any device allocation and without a context, for
/// callers whose allocator owns all device memory.  Returns the raw status
/// (no context exists to describe it).
///
/// # Safety
/// Device pointers of the sizes of `qm_gqa_decode`; `stream` a live
/// `cudaStream_t` on the current device; calls that overlap on the GPU race.
pub unsafe fn gqa_decode_noalloc(
    p: &GqaParams<'_>,
    k_cache: *mut u16,
    v_cache: *mut u16,
    batch: i32,
    capacity: i32,
    seq_len: i64,
    q_gate: *const f32,
    k_new: *const f32,
    v_new: *const f32,
    out: *mut f32,
    stream: *mut c_void,
) -> Result<()> {
    plain(sys::qm_gqa_decode_noalloc(
        &p.raw, k_cache, v_cache, batch, capacity, seq_len, q_gate, k_new, v_new, out, stream,
    ))
}
