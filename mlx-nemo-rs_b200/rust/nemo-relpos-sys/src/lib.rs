//! Raw FFI to libnemo_relpos (`include/nemo_relpos.h`): the B200 (sm_100a)
//! relative-position multi-head attention of the FastConformer encoder, a
//! drop-in for the `internals` attention API of mlx-voice
//! (src/asr/modules/encoders/attention.rs, src/core/quantization.rs,
//! src/asr/streaming/core.rs).  One `extern "C"` declaration per function of
//! the header, with the same names and argument order; `build.rs` compiles
//! the CUDA sources with nvcc (through `cc`) and links them statically.
//!
//! Every function returns an `int` status (`NRP_OK` or a negative
//! `NRP_ERR_*`); `nrp_last_error` gives the calling thread's last message.
//! Device pointers are CUDA memory on the context's device; work is queued on
//! the given stream (`*mut c_void` = `cudaStream_t`).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_float, c_int, c_void};

pub const NRP_OK: c_int = 0;
pub const NRP_DTYPE_F32: c_int = 0;
pub const NRP_DTYPE_BF16: c_int = 1;
pub const NRP_ABI_VERSION: c_int = 1;
pub const NRP_ERR_INVALID: c_int = -1;
pub const NRP_ERR_CUDA: c_int = -2;
pub const NRP_ERR_UNSUPPORTED: c_int = -3;
pub const NRP_ERR_NOMEM: c_int = -4;
pub const NRP_ERR_DEVICE: c_int = -5;
pub const NRP_HALO_ID_BYTES: usize = 128;
pub const NRP_LINEAR_Q: c_int = 0;
pub const NRP_LINEAR_K: c_int = 1;
pub const NRP_LINEAR_V: c_int = 2;
pub const NRP_LINEAR_OUT: c_int = 3;
pub const NRP_LINEAR_POS: c_int = 4;
pub const NRP_BLOCK_FF1_LINEAR1: c_int = 0;
pub const NRP_BLOCK_FF1_LINEAR2: c_int = 1;
pub const NRP_BLOCK_CONV_PW1: c_int = 2;
pub const NRP_BLOCK_CONV_PW2: c_int = 3;
pub const NRP_BLOCK_FF2_LINEAR1: c_int = 4;
pub const NRP_BLOCK_FF2_LINEAR2: c_int = 5;
pub const NRP_BLOCK_NORM_FF1: c_int = 0;
pub const NRP_BLOCK_NORM_ATT: c_int = 1;
pub const NRP_BLOCK_NORM_CONV: c_int = 2;
pub const NRP_BLOCK_NORM_FF2: c_int = 3;
pub const NRP_BLOCK_NORM_OUT: c_int = 4;
pub const NRP_KERNEL_GEMM_BF16: c_int = 0;
pub const NRP_KERNEL_GEMM_Q8: c_int = 1;
pub const NRP_KERNEL_QGEMV: c_int = 2;
pub const NRP_KERNEL_GEMM_F32: c_int = 3;
pub const NRP_KERNEL_ATTN_SM100: c_int = 4;
pub const NRP_KERNEL_ATTN_SIMT: c_int = 5;
pub const NRP_KERNEL_ATTN_STREAM: c_int = 6;
pub const NRP_KERNEL_RING_APPEND: c_int = 7;
pub const NRP_KERNEL_LAYERNORM: c_int = 8;
pub const NRP_KERNEL_DWCONV: c_int = 9;
pub const NRP_KERNEL_ELEMENTWISE: c_int = 10;
pub const NRP_KERNEL_DEQUANT: c_int = 11;
pub const NRP_KERNEL_SUBSAMPLE: c_int = 12;
pub const NRP_KERNEL_KINDS: c_int = 13;

#[repr(C)] pub struct nrp_context { _p: [u8; 0] }
#[repr(C)] pub struct nrp_attn { _p: [u8; 0] }
#[repr(C)] pub struct nrp_cache { _p: [u8; 0] }
#[repr(C)] pub struct nrp_halo { _p: [u8; 0] }
#[repr(C)] pub struct nrp_block { _p: [u8; 0] }
#[repr(C)] pub struct nrp_encoder { _p: [u8; 0] }
#[repr(C)] pub struct nrp_subsampling { _p: [u8; 0] }
#[repr(C)] pub struct nrp_encoder_cache { _p: [u8; 0] }
pub const NRP_FEATURES_BFT: c_int = 0;
pub const NRP_FEATURES_BTF: c_int = 1;
#[repr(C)] #[derive(Clone, Copy)]
pub struct nrp_att_context { pub left: i32, pub right: i32, pub chunked: i32 }
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct nrp_streaming_config {
    pub chunk_size: [i32; 2], pub shift_size: [i32; 2], pub cache_drop_size: i32,
    pub last_channel_cache_size: i32, pub last_time_cache_size: i32, pub valid_out_len: i32,
    pub pre_encode_cache_size: [i32; 2], pub drop_extra_pre_encoded: i32,
    pub lookahead_frames: i32, pub mode_idx: i32, pub left_context: i32, pub right_context: i32,
}
#[repr(C)] #[derive(Clone, Copy, Default)]
pub struct nrp_seq_plan {
    pub start: c_int, pub len: c_int, pub halo_left: c_int, pub halo_right: c_int,
    pub send_prev: c_int, pub send_next: c_int,
}

extern "C" {
    pub fn nrp_abi_version() -> c_int;
    pub fn nrp_last_error() -> *const c_char;
    pub fn nrp_block_mask_host(context: *const nrp_att_context, start: c_int, end: c_int,
                               seq_len: c_int, vis: *mut u8) -> c_int;
    pub fn nrp_key_padding_mask_host(lengths: *const i32, batch: c_int, seq_len: c_int,
                                     mask: *mut c_float) -> c_int;
    pub fn nrp_streaming_mask_host(context: *const nrp_att_context, max_audio_length: c_int,
                                   cache_len: c_int, filled_cache_len: c_int,
                                   tensor_seq_len: c_int, valid_seq_len: c_int,
                                   vis: *mut u8) -> c_int;
    pub fn nrp_streaming_config_compute(left: c_int, right: c_int, chunked: c_int,
                                        n_layers: c_int, subsampling_factor: c_int,
                                        conv_kernel_size: c_int, causal_conv: c_int,
                                        mode_idx: c_int, max_context: c_int,
                                        out: *mut nrp_streaming_config) -> c_int;
    pub fn nrp_attn_forward_noalloc(attn: *mut nrp_attn, stream: *mut c_void, x: *const c_void,
                                    batch: c_int, seq_len: c_int, pos_emb: *const c_void,
                                    lengths: *const i32, context: *const nrp_att_context,
                                    out: *mut c_void) -> c_int;
    pub fn nrp_cache_reset(cache: *mut nrp_cache, stream: *mut c_void) -> c_int;
    pub fn nrp_seq_shard_plan(seq_len: c_int, nranks: c_int, rank: c_int,
                              context: *const nrp_att_context, out: *mut nrp_seq_plan) -> c_int;
    pub fn nrp_encoder_destroy(enc: *mut nrp_encoder) -> c_int;
    pub fn nrp_linear(ctx: *mut nrp_context, stream: *mut c_void, dtype: c_int, x: *const c_void,
                      m: c_int, k: c_int, w: *const c_void, n: c_int, bias: *const c_void,
                      y: *mut c_void) -> c_int;
    pub fn nrp_profile_enable(ctx: *mut nrp_context, enable: c_int) -> c_int;
    pub fn nrp_profile_reset(ctx: *mut nrp_context) -> c_int;
    pub fn nrp_profile_read(ctx: *mut nrp_context, kind: c_int, launches: *mut i64,
                            total_ms: *mut f64) -> c_int;
    pub fn nrp_profile_launches(ctx: *mut nrp_context, kinds: *mut c_int, ms: *mut f32,
                                capacity: i64, count: *mut i64) -> c_int;
    pub fn nrp_pe_encoding_host(d_model: c_int, max_len: c_int, seq_len: c_int, out: *mut c_float) -> c_int;
    pub fn nrp_pe_xscale(d_model: c_int, xscaling: c_int) -> c_float;
    pub fn nrp_att_context_new(left: c_int, right: c_int, style: *const c_char, out: *mut nrp_att_context) -> c_int;
    pub fn nrp_context_create(device: c_int, out: *mut *mut nrp_context) -> c_int;
    pub fn nrp_context_destroy(ctx: *mut nrp_context) -> c_int;
    pub fn nrp_context_check(ctx: *mut nrp_context, stream: *mut c_void) -> c_int;
    pub fn nrp_context_selftest_wait_expiry(ctx: *mut nrp_context, stream: *mut c_void,
                                            budget_us: c_int) -> c_int;
    pub fn nrp_pe_encoding(ctx: *mut nrp_context, d_model: c_int, max_len: c_int, seq_len: c_int,
                           dtype: c_int, dev_out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn nrp_attn_create(ctx: *mut nrp_context, d_model: c_int, n_heads: c_int, use_bias: c_int,
                           out: *mut *mut nrp_attn) -> c_int;
    pub fn nrp_attn_destroy(a: *mut nrp_attn) -> c_int;
    pub fn nrp_attn_set_dtype(a: *mut nrp_attn, dtype: c_int) -> c_int;
    pub fn nrp_attn_set_cache_drop_size(a: *mut nrp_attn, n: c_int) -> c_int;
    pub fn nrp_attn_load_linear(a: *mut nrp_attn, which: c_int, w: *const c_float, b: *const c_float) -> c_int;
    pub fn nrp_attn_load_linear_quantized(a: *mut nrp_attn, which: c_int, bits: c_int, group: c_int,
                                          wq: *const u32, scales: *const c_float, biases: *const c_float,
                                          bias: *const c_float) -> c_int;
    pub fn nrp_attn_load_pos_bias(a: *mut nrp_attn, u: *const c_float, v: *const c_float) -> c_int;
    pub fn nrp_attn_forward(a: *mut nrp_attn, stream: *mut c_void, x: *const c_void, batch: c_int,
                            seq_len: c_int, pos_emb: *const c_void, lengths: *const i32,
                            context: *const nrp_att_context, out: *mut c_void) -> c_int;
    pub fn nrp_cache_create(a: *mut nrp_attn, batch: c_int, cache_len: c_int, out: *mut *mut nrp_cache) -> c_int;
    pub fn nrp_cache_destroy(c: *mut nrp_cache) -> c_int;
    pub fn nrp_cache_import_h(c: *mut nrp_cache, h: *const c_float, stream: *mut c_void) -> c_int;
    pub fn nrp_cache_export_h(c: *mut nrp_cache, h: *mut c_float, stream: *mut c_void) -> c_int;
    pub fn nrp_cache_get_head(c: *const nrp_cache, head: *mut c_int) -> c_int;
    pub fn nrp_cache_set_head(c: *mut nrp_cache, head: c_int) -> c_int;
    pub fn nrp_attn_forward_with_cache(a: *mut nrp_attn, stream: *mut c_void, x: *const c_void,
                                       batch: c_int, seq_len: c_int, pos_emb: *const c_void,
                                       cache: *mut nrp_cache, filled: c_int, valid: c_int,
                                       context: *const nrp_att_context, out: *mut c_void) -> c_int;
    // sequence split over several GPUs (no reference counterpart)
    pub fn nrp_seq_shard(seq_len: c_int, nranks: c_int, rank: c_int, start: *mut c_int,
                         len: *mut c_int) -> c_int;
    pub fn nrp_halo_unique_id(id: *mut u8) -> c_int;  // 128 bytes
    pub fn nrp_halo_comm_create(ctx: *mut nrp_context, id: *const u8, rank: c_int, nranks: c_int,
                                timeout_ms: c_int, out: *mut *mut nrp_halo) -> c_int;
    pub fn nrp_halo_comm_destroy(h: *mut nrp_halo) -> c_int;
    pub fn nrp_halo_comm_check(h: *mut nrp_halo, stream: *mut c_void) -> c_int;
    pub fn nrp_attn_forward_seq_sharded(a: *mut nrp_attn, h: *mut nrp_halo, stream: *mut c_void,
                                        x_local: *const c_void, batch: c_int, seq_len: c_int,
                                        pos_emb: *const c_void, lengths: *const i32,
                                        context: *const nrp_att_context,
                                        out_local: *mut c_void) -> c_int;
    // Conformer block / encoder (conformer.rs:694-722, 1617-2437)
    pub fn nrp_block_create(ctx: *mut nrp_context, d_model: c_int, n_heads: c_int, ff_dim: c_int,
                            conv_kernel: c_int, causal_conv: c_int, conv_norm: c_int,
                            use_bias: c_int, out: *mut *mut nrp_block) -> c_int;
    pub fn nrp_block_destroy(b: *mut nrp_block) -> c_int;
    pub fn nrp_block_set_dtype(b: *mut nrp_block, dtype: c_int) -> c_int;
    pub fn nrp_block_attn(b: *mut nrp_block, attn: *mut *mut nrp_attn) -> c_int;
    pub fn nrp_block_load_linear(b: *mut nrp_block, which: c_int, w: *const c_float,
                                 bias: *const c_float) -> c_int;
    pub fn nrp_block_load_linear_quantized(b: *mut nrp_block, which: c_int, bits: c_int,
                                           group: c_int, wq: *const u32, scales: *const c_float,
                                           biases: *const c_float, bias: *const c_float) -> c_int;
    pub fn nrp_block_load_norm(b: *mut nrp_block, which: c_int, gamma: *const c_float,
                               beta: *const c_float) -> c_int;
    pub fn nrp_block_load_depthwise(b: *mut nrp_block, w: *const c_float, bias: *const c_float) -> c_int;
    pub fn nrp_block_load_conv_norm(b: *mut nrp_block, gamma: *const c_float, beta: *const c_float,
                                    mean: *const c_float, var: *const c_float) -> c_int;
    pub fn nrp_block_forward(b: *mut nrp_block, stream: *mut c_void, x: *const c_void, batch: c_int,
                             seq_len: c_int, pos_emb: *const c_void, lengths: *const i32,
                             context: *const nrp_att_context, out: *mut c_void) -> c_int;
    pub fn nrp_encoder_create(ctx: *mut nrp_context, n_layers: c_int, d_model: c_int,
                              n_heads: c_int, ff_dim: c_int, conv_kernel: c_int,
                              causal_conv: c_int, conv_norm: c_int, use_bias: c_int,
                              xscaling: c_int, max_len: c_int, out: *mut *mut nrp_encoder) -> c_int;
    pub fn nrp_encoder_block(e: *mut nrp_encoder, layer: c_int, out: *mut *mut nrp_block) -> c_int;
    pub fn nrp_encoder_set_dtype(e: *mut nrp_encoder, dtype: c_int) -> c_int;
    pub fn nrp_encoder_forward_from_embeddings(e: *mut nrp_encoder, stream: *mut c_void,
                                               x: *const c_void, batch: c_int, seq_len: c_int,
                                               lengths: *const i32,
                                               context: *const nrp_att_context,
                                               out: *mut c_void) -> c_int;
    pub fn nrp_encoder_add_subsampling(e: *mut nrp_encoder, feat_in: c_int, factor: c_int,
                                       conv_channels: c_int, causal_downsampling: c_int,
                                       sub: *mut *mut nrp_subsampling) -> c_int;
    pub fn nrp_encoder_forward(e: *mut nrp_encoder, stream: *mut c_void, features: *const c_float,
                               batch: c_int, frames: c_int, lengths: *const i32,
                               context: *const nrp_att_context, out: *mut c_void,
                               out_lengths: *mut i32) -> c_int;
    pub fn nrp_block_forward_with_cache(b: *mut nrp_block, stream: *mut c_void, x: *const c_void,
                                        batch: c_int, seq_len: c_int, pos_emb: *const c_void,
                                        attn_cache: *mut nrp_cache, conv_cache: *mut c_void,
                                        filled: c_int, valid: c_int,
                                        context: *const nrp_att_context, out: *mut c_void) -> c_int;
    pub fn nrp_encoder_cache_create(e: *mut nrp_encoder, batch: c_int, cache_len: c_int,
                                    out: *mut *mut nrp_encoder_cache) -> c_int;
    pub fn nrp_encoder_cache_destroy(c: *mut nrp_encoder_cache) -> c_int;
    pub fn nrp_encoder_cache_reset(c: *mut nrp_encoder_cache, stream: *mut c_void) -> c_int;
    pub fn nrp_encoder_cache_get_filled(c: *const nrp_encoder_cache, filled: *mut c_int) -> c_int;
    pub fn nrp_encoder_cache_set_filled(c: *mut nrp_encoder_cache, filled: c_int) -> c_int;
    pub fn nrp_encoder_cache_layer(c: *mut nrp_encoder_cache, layer: c_int,
                                   attn_cache: *mut *mut nrp_cache,
                                   conv_cache: *mut *mut c_void) -> c_int;
    pub fn nrp_encoder_cache_copy_conv(c: *mut nrp_encoder_cache, layer: c_int, data: *mut c_void,
                                       to_cache: c_int, stream: *mut c_void) -> c_int;
    pub fn nrp_encoder_forward_streaming(e: *mut nrp_encoder, stream: *mut c_void,
                                         features: *const c_float, batch: c_int, frames: c_int,
                                         lengths: *const i32, cache: *mut nrp_encoder_cache,
                                         drop_extra_pre_encoded: c_int,
                                         context: *const nrp_att_context, out: *mut c_void,
                                         out_lengths: *mut i32, out_frames: *mut c_int) -> c_int;
    pub fn nrp_context_set_weight_cache(ctx: *mut nrp_context, enable: c_int) -> c_int;
    pub fn nrp_partition_utterances(lengths: *const i32, n: c_int, nranks: c_int, d_model: c_int,
                                    rank_of: *mut i32, rank_cost: *mut f64) -> c_int;
    pub fn nrp_copy_frames(dst: *mut c_void, src: *const c_void, lengths: *const i32,
                           batch: c_int, frames: c_int, row_bytes: i64, stream: *mut c_void,
                           bytes: *mut i64) -> c_int;
    pub fn nrp_unpack_frames(dst: *mut c_void, src: *const c_void, lengths: *const i32,
                             batch: c_int, frames: c_int, row_bytes: i64, staging: *mut c_void,
                             dev_lengths: *mut i32, stream: *mut c_void, bytes: *mut i64)
                             -> c_int;
    pub fn nrp_pack_frames(dst: *mut c_void, src: *const c_void, lengths: *const i32,
                           batch: c_int, frames: c_int, row_bytes: i64, staging: *mut c_void,
                           stream: *mut c_void, bytes: *mut i64) -> c_int;
    pub fn nrp_subsampling_create(ctx: *mut nrp_context, feat_in: c_int, d_model: c_int,
                                  factor: c_int, conv_channels: c_int, causal_downsampling: c_int,
                                  out: *mut *mut nrp_subsampling) -> c_int;
    pub fn nrp_subsampling_destroy(s: *mut nrp_subsampling) -> c_int;
    pub fn nrp_subsampling_set_dtype(s: *mut nrp_subsampling, dtype: c_int) -> c_int;
    pub fn nrp_subsampling_feat_out(s: *const nrp_subsampling, feat_out: *mut c_int) -> c_int;
    pub fn nrp_subsampling_output_length(s: *const nrp_subsampling, frames: c_int,
                                         out_frames: *mut c_int) -> c_int;
    pub fn nrp_subsampling_load_conv(s: *mut nrp_subsampling, index: c_int, weight: *const c_float,
                                     bias: *const c_float) -> c_int;
    pub fn nrp_subsampling_load_out(s: *mut nrp_subsampling, weight: *const c_float,
                                    bias: *const c_float) -> c_int;
    pub fn nrp_subsampling_load_out_quantized(s: *mut nrp_subsampling, bits: c_int, group: c_int,
                                              wq: *const u32, scales: *const c_float,
                                              biases: *const c_float, bias: *const c_float) -> c_int;
    pub fn nrp_subsampling_forward(s: *mut nrp_subsampling, stream: *mut c_void,
                                   features: *const c_float, layout: c_int, batch: c_int,
                                   frames: c_int, lengths: *const i32, out: *mut c_void) -> c_int;
    pub fn nrp_subsampling_set_chunk_frames(s: *mut nrp_subsampling, frames: c_int) -> c_int;
    pub fn nrp_qlinear(ctx: *mut nrp_context, stream: *mut c_void, x: *const c_void, m: c_int, k: c_int,
                       wq: *const u32, scales: *const c_void, biases: *const c_void, n: c_int,
                       group: c_int, bits: c_int, bias: *const c_void, y: *mut c_void) -> c_int;
}

/// The few CUDA runtime entry points the safe wrapper uses for its device
/// arrays (the runtime is linked statically with the library).
pub mod cuda {
    use std::os::raw::{c_int, c_void};
    pub const MEMCPY_HOST_TO_DEVICE: c_int = 1;
    pub const MEMCPY_DEVICE_TO_HOST: c_int = 2;
    pub const MEMCPY_DEVICE_TO_DEVICE: c_int = 3;
    extern "C" {
        pub fn cudaSetDevice(device: c_int) -> c_int;
        pub fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> c_int;
        pub fn cudaFree(ptr: *mut c_void) -> c_int;
        pub fn cudaMemcpy(dst: *mut c_void, src: *const c_void, bytes: usize, kind: c_int) -> c_int;
        pub fn cudaMemsetAsync(ptr: *mut c_void, value: c_int, bytes: usize,
                               stream: *mut c_void) -> c_int;
        pub fn cudaStreamSynchronize(stream: *mut c_void) -> c_int;
    }
}
