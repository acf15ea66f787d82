// Rust binding of the B200 attention / DeltaNet backend (include/vxg_attn_cuda.h), as a
// vxg-tensor maintainer would add it: crates/vxg-tensor/src/cuda_b200_ffi.rs (new), in the
// style of the Metal runner's FFI (crates/vxg-tensor/src/metal_cb4_fast_ffi.rs:134-235):
// extern "C" declarations (one per entry point of the header; pointers typed *const where the
// header says const), RAII handles, errors as (err, cap) strings.  No Rust toolchain exists in
// this build's image, so this file is not compiled here; a CPU test checks that it declares
// every entry point of the header.

use std::ffi::{c_char, c_void, CStr};
use std::ptr::NonNull;

#[link(name = "vxg_attn_cuda")]
extern "C" {
    fn vxg_attn_cuda_create(err: *mut c_char, cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_destroy(ctx: *mut c_void);
    fn vxg_attn_cuda_kv_create(ctx: *mut c_void, n_seq: u32, n_head_kv: u32, head_dim: u32,
                               cap_tokens: u32, err: *mut c_char, cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_kv_destroy(kv: *mut c_void);
    fn vxg_attn_cuda_kv_bytes(kv: *mut c_void) -> usize;
    fn vxg_attn_cuda_kv_reserve(kv: *mut c_void, cap_tokens: u32, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_step_full_gqa_q8(
        ctx: *mut c_void, kv: *mut c_void, seq: u32, q_raw: *const f32, k_cur: *mut f32,
        v_cur: *const f32, q_norm: *const f32, k_norm: *const f32, gated_q: i32, n_head: u32,
        n_head_kv: u32, head_dim: u32, pos: u32, rope_pos: u32, rope_dim: u32,
        rope_freq_base: f32, rope_neox: i32, eps: f32, attn_out: *mut f32,
        err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_deltanet_step(
        ctx: *mut c_void, n_batch: u32, n_kh: u32, n_vh: u32, dk: u32, dv: u32,
        q: *const f32, k: *const f32, v: *const f32, beta_raw: *const f32,
        alpha_raw: *const f32, ssm_a: *const f32, dt_bias: *const f32, q_scale: f32, eps: f32,
        state: *mut f32, o: *mut f32, memkind: i32, stream: *mut c_void,
        err: *mut c_char, cap: usize) -> i32;
}

pub(crate) struct B200Ctx(NonNull<c_void>);
impl Drop for B200Ctx { fn drop(&mut self) { unsafe { vxg_attn_cuda_destroy(self.0.as_ptr()) } } }

pub(crate) struct B200Kv(NonNull<c_void>);   // one per full-attention layer
impl Drop for B200Kv { fn drop(&mut self) { unsafe { vxg_attn_cuda_kv_destroy(self.0.as_ptr()) } } }

fn msg(buf: &[c_char]) -> String {
    unsafe { CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned()
}

impl B200Ctx {
    pub fn new() -> crate::Result<Self> {
        let mut e = [0 as c_char; 512];
        NonNull::new(unsafe { vxg_attn_cuda_create(e.as_mut_ptr(), e.len()) })
            .map(B200Ctx).ok_or_else(|| crate::Error::msg(msg(&e)))
    }
    /// Same arguments and in-place effects as llm_prefill.rs:259-278, with the layer's device
    /// KV pool + sequence id in place of `&mut Vec<KvQ8Block>`.
    #[allow(clippy::too_many_arguments)]
    pub fn step_full_gqa_q8(&self, kv: &B200Kv, seq: u32, q_raw: &[f32], k_cur: &mut [f32],
                            v_cur: &[f32], q_norm: Option<&[f32]>, k_norm: Option<&[f32]>,
                            gated_q: bool, n_head: usize, n_head_kv: usize, head_dim: usize,
                            pos: usize, rope_pos: usize, rope_dim: usize, rope_freq_base: f32,
                            rope_neox: bool, eps: f32, attn_out: &mut [f32]) -> crate::Result<()> {
        let mut e = [0 as c_char; 512];
        let opt = |o: Option<&[f32]>| o.map_or(std::ptr::null(), |s| s.as_ptr());
        let rc = unsafe { vxg_attn_cuda_step_full_gqa_q8(
            self.0.as_ptr(), kv.0.as_ptr(), seq, q_raw.as_ptr(), k_cur.as_mut_ptr(),
            v_cur.as_ptr(), opt(q_norm), opt(k_norm), gated_q as i32, n_head as u32,
            n_head_kv as u32, head_dim as u32, pos as u32, rope_pos as u32, rope_dim as u32,
            rope_freq_base, rope_neox as i32, eps, attn_out.as_mut_ptr(), e.as_mut_ptr(), e.len()) };
        if rc < 0 { return Err(crate::Error::msg(msg(&e))); }
        Ok(())
    }
}

extern "C" {
    fn vxg_attn_cuda_q8_prefill(ctx: *mut c_void, kv: *mut c_void, n_batch: u32, n_tok: u32,
                                n_head: u32, seq_ids: *const i32, pos: *const i32,
                                q: *const c_void, k_new: *const c_void, v_new: *const c_void,
                                q_gate: *const c_void, dtype: i32, scale: f32, max_ctx: u32,
                                out: *mut f32, memkind: i32, stream: *mut c_void,
                                err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_state_checkpoint(ctx: *mut c_void, n: u32, states: *const *mut c_void,
                                      backups: *const *mut c_void, bytes: *const usize,
                                      restore: u32, stream: *mut c_void, err: *mut c_char,
                                      cap: usize) -> i32;
}

extern "C" {
    fn vxg_attn_cuda_q8_decode_host_async(ctx: *mut c_void, kv: *mut c_void, n_batch: u32,
        n_head: u32, seq_ids: *const i32, pos: *const i32, q: *const f32, k_new: *const f32,
        v_new: *const f32, q_gate: *const f32, scale: f32, max_ctx: u32, out: *mut f32,
        ticket: *mut u64, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_ticket_wait(ctx: *mut c_void, ticket: u64, err: *mut c_char,
                                 cap: usize) -> i32;
}
// inputs / outputs in pinned memory (vxg_attn_cuda_host_alloc); the inputs of a step must not
// change, and its output must not be read, until its ticket has been waited for

extern "C" {
    fn vxg_attn_cuda_version() -> *const c_char;
    fn vxg_attn_cuda_sync(ctx: *mut c_void, stream: *mut c_void, err: *mut c_char,
        cap: usize) -> i32;
    fn vxg_attn_cuda_sm_count(ctx: *mut c_void) -> i32;
    fn vxg_attn_cuda_set_timing(ctx: *mut c_void, enable: i32) -> i32;
    fn vxg_attn_cuda_last_split_ms(ctx: *mut c_void) -> f64;
    fn vxg_attn_cuda_force_generic(ctx: *mut c_void, enable: i32) -> i32;
    fn vxg_attn_cuda_malloc(ctx: *mut c_void, bytes: usize, err: *mut c_char,
        cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_free(ctx: *mut c_void, dptr: *mut c_void);
    fn vxg_attn_cuda_host_alloc(ctx: *mut c_void, bytes: usize, err: *mut c_char,
        cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_host_free(ctx: *mut c_void, hptr: *mut c_void);
    fn vxg_attn_cuda_memcpy(ctx: *mut c_void, dst: *mut c_void, src: *const c_void, bytes: usize,
        kind: i32, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_kv_capacity(kv: *mut c_void) -> u32;
    fn vxg_attn_cuda_kv_device_ptrs(kv: *mut c_void, k_pool: *mut *mut c_void,
        v_pool: *mut *mut c_void, seq_stride: *mut usize) -> i32;
    fn vxg_attn_cuda_kv_import(ctx: *mut c_void, kv: *mut c_void, seq: u32, tok_begin: u32,
        n_tok: u32, k_blocks: *const c_void, v_blocks: *const c_void, memkind: i32,
        err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_kv_export(ctx: *mut c_void, kv: *mut c_void, seq: u32, tok_begin: u32,
        n_tok: u32, k_blocks: *mut c_void, v_blocks: *mut c_void, memkind: i32, err: *mut c_char,
        cap: usize) -> i32;
    fn vxg_attn_cuda_kv_create_f32(ctx: *mut c_void, n_seq: u32, n_head_kv: u32, head_dim: u32,
        cap_tokens: u32, err: *mut c_char, cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_q8_append(ctx: *mut c_void, kv: *mut c_void, n_batch: u32, n_tok: u32,
        seq_ids: *const i32, pos: *const i32, k_new: *const f32, v_new: *const f32, memkind: i32,
        stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_q8_decode(ctx: *mut c_void, kv: *mut c_void, n_batch: u32, n_head: u32,
        seq_ids: *const i32, pos: *const i32, q: *const f32, k_new: *const f32,
        v_new: *const f32, q_gate: *const f32, scale: f32, max_ctx: u32, out: *mut f32,
        memkind: i32, stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_q8_decode_noalloc(k_pool: *mut c_void, v_pool: *mut c_void, n_seq: u32,
        cap_tokens: u32, n_head_kv: u32, head_dim: u32, n_batch: u32, n_head: u32,
        seq_ids: *const i32, pos: *const i32, q: *const f32, k_new: *const f32,
        v_new: *const f32, q_gate: *const f32, scale: f32, out: *mut f32, stream: *mut c_void,
        err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_f32_append(ctx: *mut c_void, kv: *mut c_void, n_batch: u32, n_tok: u32,
        seq_ids: *const i32, pos: *const i32, k_new: *const f32, v_new: *const f32, memkind: i32,
        stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_f32_decode(ctx: *mut c_void, kv: *mut c_void, n_batch: u32, n_head: u32,
        seq_ids: *const i32, pos: *const i32, q: *const f32, k_new: *const f32,
        v_new: *const f32, q_gate: *const f32, scale: f32, max_ctx: u32, out: *mut f32,
        memkind: i32, stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_q8_decode_partial(ctx: *mut c_void, kv: *mut c_void, n_batch: u32,
        n_head: u32, seq_ids: *const i32, kv_begin: *const i32, kv_end: *const i32,
        q: *const f32, scale: f32, max_ctx: u32, m: *mut f32, l: *mut f32, o: *mut f32,
        memkind: i32, stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_lse_combine(ctx: *mut c_void, n_parts: u32, n_rows: u32, head_dim: u32,
        m: *const f32, l: *const f32, o: *const f32, gate: *const f32, out: *mut f32,
        memkind: i32, stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_lse_combine_packed(ctx: *mut c_void, n_parts: u32, n_rows: u32,
        head_dim: u32, packed: *const f32, gate: *const f32, out: *mut f32, memkind: i32,
        stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_peer_buffer_bytes(world: u32, n_rows: u32, head_dim: u32) -> usize;
    fn vxg_attn_cuda_peer_close(ctx: *mut c_void, mapped: *mut c_void);
    fn vxg_attn_cuda_peer_free(ctx: *mut c_void, buf: *mut c_void);
    fn vxg_attn_cuda_step_full_gqa(ctx: *mut c_void, kv: *mut c_void, seq: u32,
        q_raw: *const f32, k_cur: *mut f32, v_cur: *const f32, q_norm: *const f32,
        k_norm: *const f32, gated_q: i32, n_head: u32, n_head_kv: u32, head_dim: u32, pos: u32,
        rope_dim: u32, rope_freq_base: f32, rope_neox: i32, eps: f32, att_cat: *mut f32,
        err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_deltanet_prefill(ctx: *mut c_void, n_batch: u32, n_tok: u32, n_kh: u32,
        n_vh: u32, dk: u32, dv: u32, q: *const f32, k: *const f32, v: *const f32,
        beta_raw: *const f32, alpha_raw: *const f32, ssm_a: *const f32, dt_bias: *const f32,
        q_scale: f32, eps: f32, state: *mut f32, o: *mut f32, memkind: i32, stream: *mut c_void,
        err: *mut c_char, cap: usize) -> i32;
    fn vxg_attn_cuda_step_deltanet_recurrent(ctx: *mut c_void, n_batch: u32,
        qkv_mixed: *const f32, conv_ch: u32, z: *const f32, alpha_raw: *const f32,
        beta_raw: *const f32, ssm_conv1d: *const f32, ssm_a: *const f32, ssm_dt_bias: *const f32,
        ssm_norm: *const f32, conv_state: *mut f32, ssm_state: *mut f32, n_kh: u32, n_vh: u32,
        dk: u32, dv: u32, k_sz: u32, eps: f32, y_concat: *mut f32, memkind: i32,
        stream: *mut c_void, err: *mut c_char, cap: usize) -> i32;
}

extern "C" {
    fn vxg_attn_cuda_peer_alloc(ctx: *mut c_void, world: u32, n_rows: u32, head_dim: u32,
                                ipc_handle: *mut u8, err: *mut c_char, cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_peer_open(ctx: *mut c_void, ipc_handle: *const u8, err: *mut c_char,
                               cap: usize) -> *mut c_void;
    fn vxg_attn_cuda_peer_step(ctx: *mut c_void, bufs: *const *mut c_void, world: u32,
                               rank: u32, n_rows: u32, head_dim: u32, send: *const f32,
                               gate: *const f32, out: *mut f32, stream: *mut c_void,
                               err: *mut c_char, cap: usize) -> i32;
}
