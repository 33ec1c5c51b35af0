//! Raw bindings of include/arctic_cuda.h (one `extern "C"` declaration per C function, same order
//! and parameter types; tests/test_rust_ffi.py checks the two against each other).
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void};

pub const AE_HIDDEN: usize = 384;
pub const AE_MAX_POSITIONS: usize = 512;

pub const AE_OK: c_int = 0;
pub const AE_ERR_INVALID_ARG: c_int = -1;
pub const AE_ERR_CUDA: c_int = -2;
pub const AE_ERR_NO_MODEL: c_int = -3;
pub const AE_ERR_BAD_PACK: c_int = -4;
pub const AE_ERR_TOKEN_RANGE: c_int = -5;
pub const AE_ERR_DEVICE: c_int = -6;
pub const AE_ERR_CAPACITY: c_int = -7;

pub const AE_ATTENTION_EXACT: c_int = 0;
pub const AE_ATTENTION_INT8: c_int = 1;

pub const AE_TRACE_EMBED: c_int = 0;
pub const AE_TRACE_ATTN0: c_int = 1;

pub const AE_KERNEL_KINDS: usize = 9;

/// Opaque context: one GPU, its copy of the model, workspace, stream and graphs.
#[repr(C)]
pub struct ae_ctx {
    _opaque: [u8; 0],
}

/// Opaque WordPiece tokenizer (host only).
#[repr(C)]
pub struct ae_tokenizer {
    _opaque: [u8; 0],
}

/// QuantizedLinearRaw as host pointers (n_out == 0: pruned, only inv_smooth is read).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct ae_linear_desc {
    pub n_out: u64,
    pub k_in: u64,
    pub w_q: *const i8,
    pub w_scale: *const f32,
    pub bias: *const f32,
    pub inv_smooth: *const f32,
}

/// QuantizedLayerRaw as host pointers.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct ae_layer_desc {
    pub qkv: ae_linear_desc,
    pub has_split: i32,
    pub q_only: ae_linear_desc,
    pub kv_only: ae_linear_desc,
    pub attn_out: ae_linear_desc,
    pub ln1_weight: *const f32,
    pub ln1_bias: *const f32,
    pub ffn_inter: ae_linear_desc,
    pub ffn_out: ae_linear_desc,
    pub ln2_weight: *const f32,
    pub ln2_bias: *const f32,
}

/// QuantizedModelRaw as host pointers.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct ae_model_desc {
    pub word_emb_q: *const i8,
    pub word_emb_scale: *const f32,
    pub pos_emb_q: *const i8,
    pub pos_emb_scale: *const f32,
    pub type_emb_q: *const i8,
    pub type_emb_scale: *const f32,
    pub emb_ln_weight: *const f32,
    pub emb_ln_bias: *const f32,
    pub layers: [ae_layer_desc; 12],
}

extern "C" {
    pub fn ae_ctx_create(device: c_int, out: *mut *mut ae_ctx) -> c_int;
    pub fn ae_ctx_destroy(ctx: *mut ae_ctx) -> c_int;
    pub fn ae_last_error(ctx: *const ae_ctx) -> *const c_char;
    pub fn ae_ctx_set_stream(ctx: *mut ae_ctx, cuda_stream: *mut c_void) -> c_int;
    pub fn ae_ctx_device(ctx: *const ae_ctx) -> c_int;
    pub fn ae_model_load(ctx: *mut ae_ctx, desc: *const ae_model_desc) -> c_int;
    pub fn ae_model_load_file(ctx: *mut ae_ctx, path: *const c_char) -> c_int;
    pub fn ae_reserve(ctx: *mut ae_ctx, max_tokens: u32, max_seqs: u32) -> c_int;
    pub fn ae_forward_cls(ctx: *mut ae_ctx, ids: *const u16, len: u32, out384: *mut f32) -> c_int;
    pub fn ae_forward_ragged(ctx: *mut ae_ctx, ids: *const u16, cu_seqlens: *const u32, n_seqs: u32,
                             out: *mut f32) -> c_int;
    pub fn ae_forward_ragged_device(ctx: *mut ae_ctx, d_ids: *const u16, d_cu_seqlens: *const u32, n_seqs: u32,
                                    total_tokens: u32, max_len: u32, d_out: *mut f32) -> c_int;
    pub fn ae_embed_batch_multi(ctxs: *const *mut ae_ctx, n_ctx: c_int, ids: *const u16, cu_seqlens: *const u32,
                                n_seqs: u32, max_batch_tokens: u32, out: *mut f32) -> c_int;
    pub fn ae_plan_shards(cu_seqlens: *const u32, n_seqs: u32, n_shards: c_int, shard_of: *mut i32) -> c_int;
    pub fn ae_gemm_i8(ctx: *mut ae_ctx, epi: c_int, m: u32, n: u32, k: u32, d_a: *const i8, d_a_scale: *const f32,
                      d_w: *const i8, d_w_scale: *const f32, d_bias: *const f32, d_res: *const f32,
                      d_gamma: *const f32, d_beta: *const f32, d_inv_smooth: *const f32, d_out: *mut f32,
                      d_out_q: *mut i8, d_out_scale: *mut f32, d_acc: *mut i32) -> c_int;
    pub fn ae_attention_f32(ctx: *mut ae_ctx, d_qkv: *const f32, d_cu_seqlens: *const u32, n_seqs: u32,
                            max_len: u32, d_ctx: *mut f32) -> c_int;
    pub fn ae_set_attention_mode(ctx: *mut ae_ctx, mode: c_int) -> c_int;
    pub fn ae_get_attention_mode(ctx: *const ae_ctx) -> c_int;
    pub fn ae_attention_i8(ctx: *mut ae_ctx, d_qkv: *const f32, d_cu_seqlens: *const u32, n_seqs: u32,
                           max_len: u32, d_ctx: *mut f32) -> c_int;
    pub fn ae_forward_cls_noalloc(ctx: *mut ae_ctx, d_ids: *const u16, len: u32, d_out384: *mut f32) -> c_int;
    pub fn ae_trace_forward(ctx: *mut ae_ctx, ids: *const u16, cu_seqlens: *const u32, n_seqs: u32, stage: c_int,
                            f32_rows: *mut f32, q: *mut i8, scale: *mut f32) -> c_int;
    pub fn ae_profile(ctx: *mut ae_ctx, enable: c_int) -> c_int;
    pub fn ae_profile_read(ctx: *mut ae_ctx, total_ms: *mut f32, launches: *mut u32) -> c_int;
    pub fn ae_kernel_launches(ctx: *const ae_ctx) -> u64;
    pub fn ae_sync(ctx: *mut ae_ctx) -> c_int;
    pub fn ae_measure_int8_peak(ctx: *mut ae_ctx, iters: u32, ms: *mut f32, tops: *mut f64) -> c_int;
    pub fn ae_selftest_wait_timeout(ctx: *mut ae_ctx, limit_us: u32) -> c_int;
    pub fn ae_tokenizer_create_from_file(vocab_path: *const c_char, out: *mut *mut ae_tokenizer) -> c_int;
    pub fn ae_tokenizer_create_from_vocab(vocab_text: *const c_char, len: usize, out: *mut *mut ae_tokenizer)
        -> c_int;
    pub fn ae_tokenizer_destroy(tok: *mut ae_tokenizer) -> c_int;
    pub fn ae_tokenizer_vocab_size(tok: *const ae_tokenizer) -> u32;
    pub fn ae_tokenizer_last_error() -> *const c_char;
    pub fn ae_tokenize(tok: *const ae_tokenizer, text: *const c_char, len: usize, is_query: c_int, ids: *mut u16,
                       cap: u32, n_ids: *mut u32) -> c_int;
    pub fn ae_tokenize_batch(tok: *const ae_tokenizer, texts: *const *const c_char, lens: *const usize, n: u32,
                             is_query: c_int, ids: *mut u16, ids_cap: usize, cu_seqlens: *mut u32) -> c_int;
}
