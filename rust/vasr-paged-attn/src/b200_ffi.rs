// b200_ffi.rs — the extern "C" block of libvasr_pa.so (include/vasr_pa.h),
// one declaration per exported function, for the vasr-paged-attn crate.
//
// UNVERIFIED HERE: this container has no Rust toolchain, so this file has
// not been compiled. It is the binding a maintainer adds next to
// vasr-paged-attn/src/lib.rs; every signature mirrors include/vasr_pa.h
// (plain pointers and sizes, cudaStream_t as a raw pointer, i32 status).
use std::ffi::c_void;
pub type CuStream = *mut c_void; // cudaStream_t
#[repr(i32)] pub enum VasrPaDtype { F32 = 0, Bf16 = 1, F16 = 2, Fp8E4m3 = 3 }
extern "C" {
    pub fn vasr_pa_reshape_and_cache(key: *const c_void, value: *const c_void,
        key_cache: *mut c_void, value_cache: *mut c_void, slot_mapping: *const i64,
        num_tokens: i64, num_kv_heads: i32, head_dim: i32, block_size: i32, num_blocks: i64,
        key_token_stride: i64, value_token_stride: i64, dtype: i32,
        k_scale: *const f32, v_scale: *const f32, stream: CuStream) -> i32;
    pub fn vasr_pa_paged_attention_workspace_size(num_seqs: i32, num_heads: i32,
        num_kv_heads: i32, head_dim: i32, block_size: i32, max_context_len: i32, dtype: i32) -> usize;
    pub fn vasr_pa_paged_attention(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, num_seqs: i32, num_heads: i32, num_kv_heads: i32,
        head_dim: i32, block_size: i32, num_blocks: i64, max_num_blocks_per_seq: i32,
        max_context_len: i32, scale: f32, softcapping: f32, q_seq_stride: i64, dtype: i32,
        workspace: *mut c_void, workspace_bytes: usize, stream: CuStream) -> i32;
    pub fn vasr_pa_paged_attention_after_append(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, num_seqs: i32, num_heads: i32, num_kv_heads: i32,
        head_dim: i32, block_size: i32, num_blocks: i64, max_num_blocks_per_seq: i32,
        max_context_len: i32, scale: f32, softcapping: f32, q_seq_stride: i64, dtype: i32,
        workspace: *mut c_void, workspace_bytes: usize, stream: CuStream) -> i32;
    pub fn vasr_pa_gather_kv_cache(key_out: *mut c_void, value_out: *mut c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        cu_seqlens_kv: *const u32, num_seqs: i32, max_num_blocks_per_seq: i32, total_tokens: i64,
        num_kv_heads: i32, head_dim: i32, block_size: i32, num_blocks: i64, dtype: i32,
        stream: CuStream) -> i32;
    pub fn vasr_pa_paged_attention_varlen_prefill(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, cu_seqlens_q: *const u32, num_seqs: i32, total_q_tokens: i64,
        max_query_len: i32, num_heads: i32, num_kv_heads: i32, head_dim: i32, block_size: i32,
        num_blocks: i64, max_num_blocks_per_seq: i32, scale: f32, softcapping: f32,
        q_token_stride: i64, dtype: i32, stream: CuStream) -> i32;
    pub fn vasr_pa_copy_blocks(key_caches: *const *mut c_void, value_caches: *const *mut c_void,
        num_layers: i32, block_mapping: *const i64, num_pairs: i64, num_blocks: i64,
        block_bytes: i64, stream: CuStream) -> i32;
    pub fn vasr_pa_swap_blocks(dst: *mut c_void, src: *const c_void, block_mapping: *const i64,
        num_pairs: i64, src_num_blocks: i64, dst_num_blocks: i64, block_bytes: i64,
        stream: CuStream) -> i32;
    // fp8 (E4M3) pages with per-tensor scales (the k_scale / v_scale arguments)
    pub fn vasr_pa_reshape_and_cache_fp8(key: *const c_void, value: *const c_void,
        key_cache: *mut c_void, value_cache: *mut c_void, slot_mapping: *const i64,
        num_tokens: i64, num_kv_heads: i32, head_dim: i32, block_size: i32, num_blocks: i64,
        key_token_stride: i64, value_token_stride: i64, src_dtype: i32,
        k_scale: *const f32, v_scale: *const f32, stream: CuStream) -> i32;
    pub fn vasr_pa_gather_kv_cache_fp8(key_out: *mut c_void, value_out: *mut c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        cu_seqlens_kv: *const u32, num_seqs: i32, max_num_blocks_per_seq: i32,
        total_tokens: i64, num_kv_heads: i32, head_dim: i32, block_size: i32,
        num_blocks: i64, out_dtype: i32, k_scale: *const f32, v_scale: *const f32,
        stream: CuStream) -> i32;
    pub fn vasr_pa_paged_attention_varlen_prefill_fp8(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, cu_seqlens_q: *const u32, num_seqs: i32, total_q_tokens: i64,
        max_query_len: i32, num_heads: i32, num_kv_heads: i32, head_dim: i32, block_size: i32,
        num_blocks: i64, max_num_blocks_per_seq: i32, scale: f32, softcapping: f32,
        q_token_stride: i64, dtype: i32, k_scale: *const f32, v_scale: *const f32,
        workspace: *mut c_void, workspace_bytes: usize, stream: CuStream) -> i32;
    pub fn vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size(num_seqs: i32,
        num_kv_heads: i32, head_dim: i32, block_size: i32, max_num_blocks_per_seq: i32) -> usize;
    pub fn vasr_pa_paged_attention_fp8(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, num_seqs: i32, num_heads: i32, num_kv_heads: i32,
        head_dim: i32, block_size: i32, num_blocks: i64, max_num_blocks_per_seq: i32,
        max_context_len: i32, scale: f32, softcapping: f32, q_seq_stride: i64, dtype: i32,
        k_scale: *const f32, v_scale: *const f32, workspace: *mut c_void,
        workspace_bytes: usize, stream: CuStream) -> i32;
    // device decode loop (no reference counterpart call: replaces host work of
    // paged_batch_engine.rs:634-728)
    pub fn vasr_pa_decode_step_prepare(next_ids: *const u32, eos_ids: *const u32, num_eos: i32,
        prompt_lens: *const u32, step: *const u32, block_tables: *const u32,
        block_table_lens: *const u32, max_num_blocks_per_seq: i32, block_size: i32,
        num_blocks: i64, num_seqs: i32, finished: *mut u8, generated: *mut u32,
        history: *mut u32, history_cols: i32, input_ids: *mut i64, positions: *mut i64,
        slot_mapping: *mut i64, context_lens: *mut u32, stream: CuStream) -> i32;
    pub fn vasr_pa_greedy_argmax_workspace_size(num_seqs: i32, vocab: i64) -> usize;
    pub fn vasr_pa_greedy_argmax(next_ids: *mut u32, logits: *const c_void, num_seqs: i32,
        vocab: i64, row_stride: i64, dtype: i32, finished: *const u8, step: *mut u32,
        workspace: *mut c_void, workspace_bytes: usize, stream: CuStream) -> i32;
    // fused q/k RMSNorm + RoPE + K/V append of one layer (replaces the
    // thinker_text.rs:1041-1109 chain before reshape_and_cache)
    pub fn vasr_pa_fused_qk_norm_rope_append(q_out: *mut c_void, qkv: *const c_void,
        qkv_token_stride: i64, q_norm_weight: *const c_void, k_norm_weight: *const c_void,
        eps: f32, cos_table: *const f32, sin_table: *const f32, max_position: i64,
        positions: *const i64, key_cache: *mut c_void, value_cache: *mut c_void,
        slot_mapping: *const i64, num_tokens: i64, num_heads: i32, num_kv_heads: i32,
        head_dim: i32, block_size: i32, num_blocks: i64, dtype: i32, stream: CuStream) -> i32;
    // decode without a caller workspace (fixed library scratch; see below)
    pub fn vasr_pa_paged_attention_noalloc(out: *mut c_void, query: *const c_void,
        key_cache: *const c_void, value_cache: *const c_void, block_tables: *const u32,
        context_lens: *const u32, num_seqs: i32, num_heads: i32, num_kv_heads: i32,
        head_dim: i32, block_size: i32, num_blocks: i64, max_num_blocks_per_seq: i32,
        max_context_len: i32, scale: f32, softcapping: f32, q_seq_stride: i64, dtype: i32,
        stream: CuStream) -> i32;
    pub fn vasr_pa_noalloc_scratch_bytes() -> usize;
    pub fn vasr_pa_abi_version() -> i32;
    pub fn vasr_pa_status_string(status: i32) -> *const std::os::raw::c_char;
}
