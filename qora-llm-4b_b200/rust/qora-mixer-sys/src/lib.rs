//! Raw declarations of the C ABI in `include/qora_mixer.h` (libqora_mixer.so,
//! the B200 token-mixer library), one `extern "C"` item per header function,
//! in header order.  Every function returns a status (`QM_OK` or a `QM_E_*`
//! code) unless its C declaration returns something else.  Pointers to
//! tensors are device pointers on the context's device except in the `_host`
//! entry points.  The safe wrapper is the `qora-mixer` crate.
//!
//! The reference (qora-protocol/QORA-LLM-4B) keeps its mixers as inline
//! regions of `forward_deltanet_decode` (src/gemv.rs:719), `forward_attn_decode`
//! (907), `prefill_deltanet_layer` (1086), `prefill_attn_layer` (1339) and
//! their wgpu twins (src/gpu_inference.rs:125, 247, 436, 670); each region
//! becomes one call declared here.
#![allow(non_camel_case_types)]
#![no_std]

use core::ffi::{c_char, c_int, c_uchar, c_void};

// ---- status codes ---------------------------------------------------------
pub const QM_OK: c_int = 0;
pub const QM_E_ARG: c_int = 1;
pub const QM_E_SHAPE: c_int = 2;
pub const QM_E_OOM: c_int = 3;
pub const QM_E_CUDA: c_int = 4;
pub const QM_E_NCCL: c_int = 5;
pub const QM_E_TIMEOUT: c_int = 6;
pub const QM_E_RANGE: c_int = 7;
/// Takes the place of the reference's `panic!` on a layer/cache mismatch
/// (src/gemv.rs:228, 1049; src/gpu_inference.rs:418).
pub const QM_E_MISMATCH: c_int = 8;
pub const QM_E_UNSUPPORTED: c_int = 9;
pub const QM_E_CAPTURE: c_int = 10;

/// Bytes of the fixed device array `qm_gqa_decode_noalloc` uses (16 MiB).
pub const QM_NOALLOC_SCRATCH_BYTES: u32 = 16u32 << 20;

/// Weight formats of `qm_weight::kind`.
pub const QM_W_F16: c_int = 0; // f16 [k][n] (gemv_f16, src/gemv.rs:338-368)
pub const QM_W_Q4: c_int = 1; // packed [k][n/2] + f16 scales [k][n/32] (src/gemv.rs:411-450)
pub const QM_W_F16_ROWS: c_int = 2; // one row per output, f16 [n][k] (lm_head, src/gemv.rs:664-676)
pub const QM_W_Q4_ROWS: c_int = 3; // one row per output, [n][k/2] + scales [n][k/32] (src/gemv.rs:677-707)

pub const QM_COMM_ID_BYTES: usize = 128;

/// `qm_build_flags` bit: device-side bounds self-checks compiled in.
pub const QM_BUILD_BOUNDS_CHECKS: c_int = 1;

// ---- opaque handles -------------------------------------------------------
#[repr(C)]
pub struct qm_ctx {
    _private: [u8; 0],
}
#[repr(C)]
pub struct qm_dn_state {
    _private: [u8; 0],
}
#[repr(C)]
pub struct qm_kv {
    _private: [u8; 0],
}
#[repr(C)]
pub struct qm_comm {
    _private: [u8; 0],
}

// ---- plain structs (field order and types as in the header) ----------------
/// Mixer fields of `Qor4bConfig::default_4b` (src/config.rs:42-79).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct qm_shape {
    pub num_qk_heads: c_int,
    pub num_v_heads: c_int,
    pub dn_head_dim: c_int,
    pub conv_kernel: c_int,
    pub num_attn_heads: c_int,
    pub num_kv_heads: c_int,
    pub attn_head_dim: c_int,
    pub rope_dim: c_int,
    pub rope_theta: f32,
    pub rms_eps: f32,
}

/// DeltaNet layer parameters (device pointers): conv1d_weight [8192,4],
/// A_log [32], dt_bias [32], attn_norm_weight [128] widened from f16
/// (src/gemv.rs:68-71).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qm_dn_params {
    pub conv_w: *const f32,
    pub a_log: *const f32,
    pub dt_bias: *const f32,
    pub norm_gamma: *const f32,
}

/// GQA layer parameters (device pointers): q_norm / k_norm [256] widened
/// from f16 (applied as 1 + g, src/gemv.rs:86, 594) and the RoPE tables
/// [max_pos, 32] (src/convert.rs:161-176).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qm_gqa_params {
    pub q_norm: *const f32,
    pub k_norm: *const f32,
    pub rope_cos: *const f32,
    pub rope_sin: *const f32,
    pub max_pos: c_int,
}

/// A projection weight in one of the four `QM_W_*` formats (device pointers;
/// `scales` only for the Q4 kinds).
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct qm_weight {
    pub kind: c_int,
    pub k: c_int,
    pub n: c_int,
    pub data: *const c_void,
    pub scales: *const c_void,
}

/// Head-sharded layout of one rank (`qm_shard_plan`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct qm_shard {
    pub world: c_int,
    pub rank: c_int,
    pub vh_lo: c_int,
    pub nvh: c_int,
    pub kv_lo: c_int,
    pub nkv: c_int,
    pub seq_part: c_int,
    pub seq_parts: c_int,
}

extern "C" {
    // ---- build, shape, status ------------------------------------------------
    pub fn qm_build_flags() -> c_int;
    pub fn qm_shape_get(out: *mut qm_shape) -> c_int;
    pub fn qm_status_string(status: c_int) -> *const c_char;

    // ---- context ------------------------------------------------------------
    pub fn qm_ctx_create(device: c_int, out: *mut *mut qm_ctx) -> c_int;
    pub fn qm_ctx_destroy(ctx: *mut qm_ctx) -> c_int;
    pub fn qm_ctx_set_stream(ctx: *mut qm_ctx, stream: *mut c_void) -> c_int;
    pub fn qm_ctx_get_stream(ctx: *const qm_ctx) -> *mut c_void;
    pub fn qm_sync(ctx: *mut qm_ctx) -> c_int;
    pub fn qm_last_error(ctx: *const qm_ctx) -> *const c_char;
    pub fn qm_ctx_reserve(ctx: *mut qm_ctx, bytes: usize) -> c_int;
    pub fn qm_ctx_set_host_parts(ctx: *mut qm_ctx, dn_parts: c_int, gqa_parts: c_int) -> c_int;
    pub fn qm_ctx_set_host_direct(ctx: *mut qm_ctx, on: c_int) -> c_int;
    pub fn qm_ctx_host_calls(ctx: *const qm_ctx, in_place: *mut i64, staged: *mut i64) -> c_int;
    pub fn qm_ctx_launch_count(ctx: *const qm_ctx) -> i64;
    pub fn qm_ctx_set_timing(ctx: *mut qm_ctx, on: c_int) -> c_int;
    pub fn qm_ctx_kernel_time(
        ctx: *mut qm_ctx,
        name: *const c_char,
        total_ms: *mut f64,
        launches: *mut i64,
    ) -> c_int;

    // ---- RoPE tables (src/convert.rs:161-176, any length) -------------------
    pub fn qm_rope_table(
        theta: f32,
        rope_dim: c_int,
        max_pos: c_int,
        cos_host: *mut f32,
        sin_host: *mut f32,
    ) -> c_int;

    // ---- DeltaNet recurrent state (DeltaNetState, src/gemv.rs:133-157) ------
    pub fn qm_dn_state_create(ctx: *mut qm_ctx, batch: c_int, out: *mut *mut qm_dn_state) -> c_int;
    pub fn qm_dn_state_wrap(
        ctx: *mut qm_ctx,
        batch: c_int,
        s: *mut f32,
        conv: *mut f32,
        out: *mut *mut qm_dn_state,
    ) -> c_int;
    pub fn qm_dn_state_destroy(st: *mut qm_dn_state) -> c_int;
    pub fn qm_dn_state_reset(ctx: *mut qm_ctx, st: *mut qm_dn_state) -> c_int;
    pub fn qm_dn_state_snapshot(
        ctx: *mut qm_ctx,
        src: *const qm_dn_state,
        out: *mut *mut qm_dn_state,
    ) -> c_int;
    pub fn qm_dn_state_restore(ctx: *mut qm_ctx, dst: *mut qm_dn_state, src: *const qm_dn_state) -> c_int;
    pub fn qm_dn_state_read(
        ctx: *mut qm_ctx,
        st: *const qm_dn_state,
        b: c_int,
        s_host: *mut f32,
        conv_buf_host: *mut f32,
    ) -> c_int;
    pub fn qm_dn_state_write(
        ctx: *mut qm_ctx,
        st: *mut qm_dn_state,
        b: c_int,
        s_host: *const f32,
        conv_buf_host: *const f32,
    ) -> c_int;
    pub fn qm_dn_state_conv_pos(st: *const qm_dn_state) -> i64;
    pub fn qm_dn_state_set_conv_pos(st: *mut qm_dn_state, conv_pos: i64) -> c_int;
    pub fn qm_dn_state_batch(st: *const qm_dn_state) -> c_int;
    pub fn qm_dn_state_data(st: *const qm_dn_state, s: *mut *mut f32, conv: *mut *mut f32) -> c_int;

    // ---- DeltaNet mixer ---------------------------------------------------------
    /// src/gemv.rs:744-883 (decode, one token per sequence).
    pub fn qm_dn_decode(
        ctx: *mut qm_ctx,
        p: *const qm_dn_params,
        st: *mut qm_dn_state,
        qkv: *const f32,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> c_int;
    pub fn qm_dn_decode_host(
        ctx: *mut qm_ctx,
        p: *const qm_dn_params,
        st: *mut qm_dn_state,
        qkv: *const f32,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> c_int;
    /// T sequential decode steps in one launch (src/gemv.rs:1129-1203), f32, state on chip.
    pub fn qm_dn_decode_seq(
        ctx: *mut qm_ctx,
        p: *const qm_dn_params,
        st: *mut qm_dn_state,
        t: c_int,
        qkv: *const f32,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> c_int;
    /// src/gemv.rs:1119-1219 (prefill, chunked on the tensor cores).
    pub fn qm_dn_prefill(
        ctx: *mut qm_ctx,
        p: *const qm_dn_params,
        st: *mut qm_dn_state,
        t: c_int,
        qkv: *const u16,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> c_int;
    pub fn qm_dn_prefill_host(
        ctx: *mut qm_ctx,
        p: *const qm_dn_params,
        st: *mut qm_dn_state,
        t: c_int,
        qkv: *const u16,
        a: *const f32,
        b: *const f32,
        y: *mut f32,
        z: *const f32,
        out: *mut f32,
    ) -> c_int;
    pub fn qm_dn_state_create_heads(
        ctx: *mut qm_ctx,
        batch: c_int,
        vh_lo: c_int,
        nvh: c_int,
        out: *mut *mut qm_dn_state,
    ) -> c_int;
    pub fn qm_dn_state_wrap_heads(
        ctx: *mut qm_ctx,
        batch: c_int,
        vh_lo: c_int,
        nvh: c_int,
        s: *mut f32,
        conv: *mut f32,
        out: *mut *mut qm_dn_state,
    ) -> c_int;
    pub fn qm_dn_state_heads(st: *const qm_dn_state, vh_lo: *mut c_int, nvh: *mut c_int) -> c_int;

    // ---- GQA KV cache (KvCacheEntry, src/gemv.rs:164-168) ---------------------
    pub fn qm_kv_create(ctx: *mut qm_ctx, batch: c_int, capacity: c_int, out: *mut *mut qm_kv) -> c_int;
    pub fn qm_kv_wrap(
        ctx: *mut qm_ctx,
        batch: c_int,
        capacity: c_int,
        k: *mut u16,
        v: *mut u16,
        out: *mut *mut qm_kv,
    ) -> c_int;
    pub fn qm_kv_destroy(kv: *mut qm_kv) -> c_int;
    pub fn qm_kv_snapshot(ctx: *mut qm_ctx, src: *const qm_kv, out: *mut *mut qm_kv) -> c_int;
    pub fn qm_kv_restore(ctx: *mut qm_ctx, dst: *mut qm_kv, src: *const qm_kv) -> c_int;
    pub fn qm_kv_seq_len(kv: *const qm_kv) -> i64;
    pub fn qm_kv_set_seq_len(kv: *mut qm_kv, seq_len: i64) -> c_int;
    pub fn qm_kv_capacity(kv: *const qm_kv) -> c_int;
    pub fn qm_kv_batch(kv: *const qm_kv) -> c_int;
    pub fn qm_kv_data(kv: *const qm_kv, k: *mut *mut u16, v: *mut *mut u16) -> c_int;
    pub fn qm_kv_create_heads(
        ctx: *mut qm_ctx,
        batch: c_int,
        capacity: c_int,
        kv_lo: c_int,
        nkv: c_int,
        out: *mut *mut qm_kv,
    ) -> c_int;
    pub fn qm_kv_wrap_heads(
        ctx: *mut qm_ctx,
        batch: c_int,
        capacity: c_int,
        kv_lo: c_int,
        nkv: c_int,
        k: *mut u16,
        v: *mut u16,
        out: *mut *mut qm_kv,
    ) -> c_int;
    pub fn qm_kv_heads(kv: *const qm_kv, kv_lo: *mut c_int, nkv: *mut c_int) -> c_int;

    // ---- GQA mixer ----------------------------------------------------------------
    /// src/gemv.rs:927-1011 (decode, one token per sequence).
    pub fn qm_gqa_decode(
        ctx: *mut qm_ctx,
        p: *const qm_gqa_params,
        kv: *mut qm_kv,
        q_gate: *const f32,
        k_new: *const f32,
        v_new: *const f32,
        out: *mut f32,
    ) -> c_int;
    pub fn qm_gqa_decode_host(
        ctx: *mut qm_ctx,
        p: *const qm_gqa_params,
        kv: *mut qm_kv,
        q_gate: *const f32,
        k_new: *const f32,
        v_new: *const f32,
        out: *mut f32,
    ) -> c_int;
    /// src/gemv.rs:1364-1444 (causal prefill; replaces the cache contents).
    pub fn qm_gqa_prefill(
        ctx: *mut qm_ctx,
        p: *const qm_gqa_params,
        kv: *mut qm_kv,
        t: c_int,
        q_gate: *const u16,
        k: *const u16,
        v: *const u16,
        out: *mut f32,
    ) -> c_int;
    pub fn qm_gqa_prefill_host(
        ctx: *mut qm_ctx,
        p: *const qm_gqa_params,
        kv: *mut qm_kv,
        t: c_int,
        q_gate: *const u16,
        k: *const u16,
        v: *const u16,
        out: *mut f32,
    ) -> c_int;
    /// GQA decode that allocates nothing (no counterpart in the reference).
    pub fn qm_gqa_decode_noalloc(
        p: *const qm_gqa_params,
        k_cache: *mut u16,
        v_cache: *mut u16,
        batch: c_int,
        capacity: c_int,
        seq_len: i64,
        q_gate: *const f32,
        k_new: *const f32,
        v_new: *const f32,
        out: *mut f32,
        stream: *mut c_void,
    ) -> c_int;

    // ---- projections around the mixers (src/gemv.rs:286-300, 390, 529) --------------
    pub fn qm_gemv(ctx: *mut qm_ctx, w: *const qm_weight, batch: c_int, x: *const f32, y: *mut f32) -> c_int;
    pub fn qm_gemv_multi(
        ctx: *mut qm_ctx,
        ws: *const qm_weight,
        count: c_int,
        batch: c_int,
        x: *const f32,
        ys: *const *mut f32,
    ) -> c_int;
    pub fn qm_gemm(ctx: *mut qm_ctx, w: *const qm_weight, t: c_int, x: *const u16, y: *mut f32) -> c_int;
    pub fn qm_gemm_bf16(ctx: *mut qm_ctx, w: *const qm_weight, t: c_int, x: *const u16, y: *mut u16) -> c_int;

    // ---- the decode loop's tail (src/generate.rs:185-198, 334-384) --------------------
    pub fn qm_logits_penalize(
        ctx: *mut qm_ctx,
        logits: *mut f32,
        batch: c_int,
        vocab: c_int,
        tokens: *const c_int,
        lens: *const c_int,
        stride: c_int,
        repetition_penalty: f32,
        presence_penalty: f32,
        ban_token: c_int,
    ) -> c_int;
    pub fn qm_sample(
        ctx: *mut qm_ctx,
        logits: *const f32,
        batch: c_int,
        vocab: c_int,
        temperature: f32,
        top_p: f32,
        top_k: c_int,
        r: *const f32,
        ids: *mut c_int,
    ) -> c_int;

    // ---- several GPUs (no reference counterpart: it drives one device) -------------------
    pub fn qm_shard_plan(world: c_int, rank: c_int, out: *mut qm_shard) -> c_int;
    pub fn qm_comm_unique_id(id: *mut c_uchar) -> c_int;
    pub fn qm_comm_create(
        ctx: *mut qm_ctx,
        id: *const c_uchar,
        world: c_int,
        rank: c_int,
        timeout_ms: c_int,
        out: *mut *mut qm_comm,
    ) -> c_int;
    pub fn qm_comm_allgather(
        comm: *mut qm_comm,
        send: *const c_void,
        recv: *mut c_void,
        bytes_per_rank: usize,
    ) -> c_int;
    pub fn qm_comm_enable_peer(comm: *mut qm_comm, max_bytes_per_rank: usize, wait_ms: c_int) -> c_int;
    pub fn qm_comm_destroy(comm: *mut qm_comm) -> c_int;
}
