// b200.rs — `mistralrs_paged_attn` for vasr-paged-attn on B200, over the C ABI
// of libvasr_pa.so (include/vasr_pa.h, declared in b200_ffi.rs).
//
// UNVERIFIED HERE: this container has no Rust toolchain (no cargo / rustc)
// and the Candle fork is not vendored, so this file has not been compiled.
// It is the drop-in a maintainer wires into the crate in place of the
// third-party re-export at vasr-paged-attn/src/lib.rs:20-21:
//
//     #[cfg(feature = "paged-attn")]
//     pub use mistralrs_paged_attn;            // removed
//     mod b200_ffi;                            // added
//     #[path = "b200.rs"] pub mod mistralrs_paged_attn;   // added
//
// so that `use vasr_paged_attn::mistralrs_paged_attn;`
// (vasr-models/src/model/thinker_text.rs:21) and every call site
// (:190-198, :1101-1109, :1126-1139, :1324-1332, :1344-1352) compile
// unchanged. Every function keeps the argument order of those calls.
//
// Conventions:
//  - Device pointers come from Candle tensors the way cuda_graph.rs:498-595
//    obtains them: storage_and_layout -> as_cuda_slice -> device_ptr(stream)
//    + start_offset * element size.
//  - Outputs and workspaces are allocated by Candle on the tensors' device
//    before the C call; the C ABI itself never allocates or synchronises.
//  - fp8 (E4M3) caches route to the *_fp8 entry points with the per-tensor
//    k_scale / v_scale (PagedAttentionHandle, thinker_text.rs:23-28). For a
//    16-bit cache the scales the call sites pass (both 1.0) are not used.
//  - A non-zero status becomes candle_core::Error::Msg with the library's
//    status text.
use std::collections::HashMap;
use std::ffi::{c_void, CStr};
use std::sync::Mutex;

use candle_core::cuda_backend::cudarc::driver::{CudaStream, DevicePtr};
use candle_core::{DType, Device, Result, Storage, Tensor};

use super::b200_ffi as ffi;

// ------------------------------------------------------------------ helpers
fn fail(what: &str, status: i32) -> candle_core::Error {
    let text = unsafe { CStr::from_ptr(ffi::vasr_pa_status_string(status)) };
    candle_core::Error::Msg(format!("{what}: {} (status {status})", text.to_string_lossy()))
}

fn check(what: &str, status: i32) -> Result<()> {
    if status == 0 { Ok(()) } else { Err(fail(what, status)) }
}

/// vasr_pa_dtype code of a model dtype (the cache's, or the query's).
fn dtype_code(dt: DType) -> Result<i32> {
    match dt {
        DType::F32 => Ok(ffi::VasrPaDtype::F32 as i32),
        DType::BF16 => Ok(ffi::VasrPaDtype::Bf16 as i32),
        DType::F16 => Ok(ffi::VasrPaDtype::F16 as i32),
        other => candle_core::bail!("paged attention: unsupported dtype {other:?}"),
    }
}

fn is_fp8(t: &Tensor) -> bool {
    t.dtype() == DType::F8E4M3
}

/// The CUDA stream of the tensor's device (one stream per device in the
/// reference, bench_text_decode.rs:295).
fn stream_of(t: &Tensor) -> Result<std::sync::Arc<CudaStream>> {
    match t.device() {
        Device::Cuda(d) => Ok(d.cuda_stream()),
        _ => candle_core::bail!("paged attention tensors must live on a CUDA device"),
    }
}

fn raw_stream(s: &CudaStream) -> ffi::CuStream {
    s.cu_stream() as ffi::CuStream
}

/// Device address of the tensor's first element.
fn dev_ptr(t: &Tensor, stream: &CudaStream) -> Result<*mut c_void> {
    let (storage, layout) = t.storage_and_layout();
    let Storage::Cuda(cs) = &*storage else {
        candle_core::bail!("expected a CUDA tensor");
    };
    macro_rules! base {
        ($ty:ty) => {{
            let slice = cs.as_cuda_slice::<$ty>()?;
            let (ptr, _guard) = slice.device_ptr(stream);
            ptr + (layout.start_offset() * std::mem::size_of::<$ty>()) as u64
        }};
    }
    let addr = match t.dtype() {
        DType::F32 => base!(f32),
        DType::BF16 => base!(half::bf16),
        DType::F16 => base!(half::f16),
        DType::U32 => base!(u32),
        DType::I64 => base!(i64),
        DType::U8 => base!(u8),
        DType::F8E4M3 => base!(float8::F8E4M3),
        other => candle_core::bail!("paged attention: no device pointer for dtype {other:?}"),
    };
    Ok(addr as *mut c_void)
}

fn opt_ptr(t: Option<&Tensor>, stream: &CudaStream) -> Result<*const f32> {
    match t {
        Some(t) => Ok(dev_ptr(t, stream)? as *const f32),
        None => Ok(std::ptr::null()),
    }
}

fn scales<'a>(k: Option<&'a Tensor>, v: Option<&'a Tensor>) -> Result<(&'a Tensor, &'a Tensor)> {
    match (k, v) {
        (Some(k), Some(v)) => Ok((k, v)),
        _ => candle_core::bail!("fp8 paged caches need k_scale and v_scale"),
    }
}

/// (num_blocks, num_kv_heads, head_dim, block_size) of a vLLM-layout pair:
/// K [nb, Hkv, D/x, bs, x], V [nb, Hkv, D, bs] (paged_kv_cache.rs:285-294).
fn geometry(key_cache: &Tensor, value_cache: &Tensor) -> Result<(usize, usize, usize, usize)> {
    let (nb, hkv, dx, bs, x) = key_cache.dims5()?;
    let (nbv, hkvv, d, bsv) = value_cache.dims4()?;
    if (nb, hkv, bs) != (nbv, hkvv, bsv) || dx * x != d {
        candle_core::bail!(
            "paged cache shape mismatch: key={:?} value={:?}",
            key_cache.shape(),
            value_cache.shape()
        );
    }
    Ok((nb, hkv, d, bs))
}

// Decode workspaces: one zero-filled buffer per (device, stream), grown when a
// call needs more. The kernels leave their counters at zero after every call,
// so a buffer is zero-filled only when it is (re)allocated; grow it before a
// CUDA graph capture (the reference prewarms graphs, cuda_graph.rs:204-211).
struct Workspace {
    tensor: Tensor,
    bytes: usize,
}

static WORKSPACES: Mutex<Option<HashMap<(usize, usize), Workspace>>> = Mutex::new(None);

fn workspace_for(
    like: &Tensor,
    stream: &CudaStream,
    bytes: usize,
) -> Result<(*mut c_void, usize)> {
    let ordinal = match like.device() {
        Device::Cuda(d) => d.ordinal(),
        _ => candle_core::bail!("workspace wants a CUDA device"),
    };
    let key = (ordinal, stream.cu_stream() as usize);
    let mut guard = WORKSPACES.lock().unwrap();
    let map = guard.get_or_insert_with(HashMap::new);
    let grow = map.get(&key).map_or(true, |w| w.bytes < bytes);
    if grow {
        let n = bytes.max(1 << 20);
        let tensor = Tensor::zeros(n, DType::U8, like.device())?;
        map.insert(key, Workspace { tensor, bytes: n });
    }
    let w = &map[&key];
    Ok((dev_ptr(&w.tensor, stream)?, w.bytes))
}

// ------------------------------------------------------------- KV append
/// Scatter key/value [T, Hkv, D] into the pages at slot_mapping (i64 [T],
/// -1 = skip): thinker_text.rs:1101-1109 and :1324-1332.
pub fn reshape_and_cache(
    key: &Tensor,
    value: &Tensor,
    k_scale: Option<&Tensor>,
    v_scale: Option<&Tensor>,
    key_cache: &Tensor,
    value_cache: &Tensor,
    slot_mapping: &Tensor,
) -> Result<()> {
    let (nb, hkv, d, bs) = geometry(key_cache, value_cache)?;
    let (t, kh, kd) = key.dims3()?;
    if (kh, kd) != (hkv, d) || value.dims() != key.dims() {
        candle_core::bail!("reshape_and_cache: key/value must be [T, {hkv}, {d}]");
    }
    if slot_mapping.dtype() != DType::I64 || slot_mapping.dims1()? != t {
        candle_core::bail!("reshape_and_cache: slot_mapping must be i64 [T]");
    }
    let s = stream_of(key)?;
    let (kp, vp) = (dev_ptr(key, &s)?, dev_ptr(value, &s)?);
    let (kc, vc) = (dev_ptr(key_cache, &s)?, dev_ptr(value_cache, &s)?);
    let slots = dev_ptr(slot_mapping, &s)? as *const i64;
    let (ks, vs) = (key.stride()[0] as i64, value.stride()[0] as i64);
    let st = if is_fp8(key_cache) {
        let (k_sc, v_sc) = scales(k_scale, v_scale)?;
        unsafe {
            ffi::vasr_pa_reshape_and_cache_fp8(
                kp, vp, kc, vc, slots, t as i64, hkv as i32, d as i32, bs as i32, nb as i64, ks, vs,
                dtype_code(key.dtype())?, opt_ptr(Some(k_sc), &s)?, opt_ptr(Some(v_sc), &s)?,
                raw_stream(&s),
            )
        }
    } else {
        unsafe {
            ffi::vasr_pa_reshape_and_cache(
                kp, vp, kc, vc, slots, t as i64, hkv as i32, d as i32, bs as i32, nb as i64, ks, vs,
                dtype_code(key_cache.dtype())?, opt_ptr(k_scale, &s)?, opt_ptr(v_scale, &s)?,
                raw_stream(&s),
            )
        }
    };
    check("reshape_and_cache", st)
}

// --------------------------------------------------------- decode attention
/// Single-token decode attention over the pages, [B, Hq, D] in q's dtype:
/// thinker_text.rs:1126-1139. max_context_len is an upper bound (the graph
/// bucket, cuda_graph.rs:141); the kernels read the true context_lens.
#[allow(clippy::too_many_arguments)]
pub fn paged_attention(
    q: &Tensor,
    k_scale: Option<&Tensor>,
    v_scale: Option<&Tensor>,
    key_cache: &Tensor,
    value_cache: &Tensor,
    block_tables: &Tensor,
    context_lens: &Tensor,
    alibi: Option<&Tensor>,
    max_context_len: usize,
    softmax_scale: f32,
    softcapping: f32,
    sinks: Option<&Tensor>,
) -> Result<Tensor> {
    if alibi.is_some() || sinks.is_some() {
        candle_core::bail!("paged_attention: alibi / attention sinks are not used by Qwen3-ASR");
    }
    let (nb, hkv, d, bs) = geometry(key_cache, value_cache)?;
    let (b, hq, qd) = q.dims3()?;
    if qd != d {
        candle_core::bail!("paged_attention: q must be [B, Hq, {d}]");
    }
    let (tb, cols) = block_tables.dims2()?;
    if tb != b || context_lens.dims1()? != b {
        candle_core::bail!("paged_attention: block_tables [B, cols] / context_lens [B] mismatch");
    }
    let s = stream_of(q)?;
    // callee-allocated output in Candle's pool, as the reference's crate returns it
    let out = Tensor::zeros((b, hq, d), q.dtype(), q.device())?;
    let code = dtype_code(q.dtype())?;
    let need = unsafe {
        ffi::vasr_pa_paged_attention_workspace_size(
            b as i32, hq as i32, hkv as i32, d as i32, bs as i32, max_context_len.max(1) as i32, code,
        )
    };
    let (ws, ws_bytes) = workspace_for(q, &s, need)?;
    let args = (
        dev_ptr(&out, &s)?,
        dev_ptr(q, &s)? as *const c_void,
        dev_ptr(key_cache, &s)? as *const c_void,
        dev_ptr(value_cache, &s)? as *const c_void,
        dev_ptr(block_tables, &s)? as *const u32,
        dev_ptr(context_lens, &s)? as *const u32,
    );
    let st = if is_fp8(key_cache) {
        let (k_sc, v_sc) = scales(k_scale, v_scale)?;
        unsafe {
            ffi::vasr_pa_paged_attention_fp8(
                args.0, args.1, args.2, args.3, args.4, args.5, b as i32, hq as i32, hkv as i32,
                d as i32, bs as i32, nb as i64, cols as i32, max_context_len as i32, softmax_scale,
                softcapping, q.stride()[0] as i64, code, opt_ptr(Some(k_sc), &s)?,
                opt_ptr(Some(v_sc), &s)?, ws, ws_bytes, raw_stream(&s),
            )
        }
    } else {
        unsafe {
            ffi::vasr_pa_paged_attention(
                args.0, args.1, args.2, args.3, args.4, args.5, b as i32, hq as i32, hkv as i32,
                d as i32, bs as i32, nb as i64, cols as i32, max_context_len as i32, softmax_scale,
                softcapping, q.stride()[0] as i64, code, ws, ws_bytes, raw_stream(&s),
            )
        }
    };
    check("paged_attention", st)?;
    Ok(out)
}

// ------------------------------------------------------------------ gather
/// Packed [sum kv, Hkv, D] K and V of each sequence's first kv_len tokens:
/// thinker_text.rs:190-198 and :1344-1352. fp8 pages give byte x scale in
/// out_dtype (the model dtype the call sites pass); 16-bit pages keep theirs.
pub fn gather_kv_cache(
    key_cache: &Tensor,
    value_cache: &Tensor,
    k_scale: Option<&Tensor>,
    v_scale: Option<&Tensor>,
    block_tables: &Tensor,
    cu_seqlens_kv: &Tensor,
    out_dtype: DType,
) -> Result<(Tensor, Tensor)> {
    let (nb, hkv, d, bs) = geometry(key_cache, value_cache)?;
    let (b, cols) = block_tables.dims2()?;
    if cu_seqlens_kv.dims1()? != b + 1 {
        candle_core::bail!("gather_kv_cache: cu_seqlens_kv must be [B + 1]");
    }
    // the output size is the last cumulative length (a host read, as the
    // reference's crate sizes its outputs)
    let total = cu_seqlens_kv.narrow(0, b, 1)?.to_dtype(DType::U32)?.to_vec1::<u32>()?[0] as usize;
    let fp8 = is_fp8(key_cache);
    let dt = if fp8 { out_dtype } else { key_cache.dtype() };
    let k_out = Tensor::zeros((total, hkv, d), dt, key_cache.device())?;
    let v_out = Tensor::zeros((total, hkv, d), dt, key_cache.device())?;
    let s = stream_of(key_cache)?;
    let (ko, vo) = (dev_ptr(&k_out, &s)?, dev_ptr(&v_out, &s)?);
    let (kc, vc) = (dev_ptr(key_cache, &s)? as *const c_void, dev_ptr(value_cache, &s)? as *const c_void);
    let bt = dev_ptr(block_tables, &s)? as *const u32;
    let cu = dev_ptr(cu_seqlens_kv, &s)? as *const u32;
    let st = if fp8 {
        let (k_sc, v_sc) = scales(k_scale, v_scale)?;
        unsafe {
            ffi::vasr_pa_gather_kv_cache_fp8(
                ko, vo, kc, vc, bt, cu, b as i32, cols as i32, total as i64, hkv as i32, d as i32,
                bs as i32, nb as i64, dtype_code(dt)?, opt_ptr(Some(k_sc), &s)?, opt_ptr(Some(v_sc), &s)?,
                raw_stream(&s),
            )
        }
    } else {
        if out_dtype != key_cache.dtype() {
            candle_core::bail!("gather_kv_cache: 16-bit pages keep their dtype");
        }
        unsafe {
            ffi::vasr_pa_gather_kv_cache(
                ko, vo, kc, vc, bt, cu, b as i32, cols as i32, total as i64, hkv as i32, d as i32,
                bs as i32, nb as i64, dtype_code(dt)?, raw_stream(&s),
            )
        }
    };
    check("gather_kv_cache", st)?;
    Ok((k_out, v_out))
}

// ------------------------------------------------------ varlen prefill
/// Causal chunked prefill of packed q [T, Hq, D] straight from the pages
/// (replaces gather_kv_cache + flash_attn_varlen at thinker_text.rs:1344-1365;
/// argument order of the Metal entry point, metal/varlen_prefill.rs:291-427).
/// Sequence b's rows are cu_seqlens_q[b] .. cu_seqlens_q[b + 1]; row i sits at
/// position context_lens[b] - qlen_b + i and sees keys up to that position.
#[allow(clippy::too_many_arguments)]
pub fn paged_attention_varlen_prefill(
    q: &Tensor,
    key_cache: &Tensor,
    value_cache: &Tensor,
    block_tables: &Tensor,
    context_lens: &Tensor,
    cu_seqlens_q: &Tensor,
    k_scale: Option<&Tensor>,
    v_scale: Option<&Tensor>,
    max_query_len: usize,
    softmax_scale: f32,
    softcapping: f32,
) -> Result<Tensor> {
    let (nb, hkv, d, bs) = geometry(key_cache, value_cache)?;
    let (t, hq, qd) = q.dims3()?;
    let (b, cols) = block_tables.dims2()?;
    if qd != d || cu_seqlens_q.dims1()? != b + 1 || context_lens.dims1()? != b {
        candle_core::bail!("paged_attention_varlen_prefill: q / metadata shape mismatch");
    }
    let s = stream_of(q)?;
    let out = Tensor::zeros((t, hq, d), q.dtype(), q.device())?;
    let code = dtype_code(q.dtype())?;
    let args = (
        dev_ptr(&out, &s)?,
        dev_ptr(q, &s)? as *const c_void,
        dev_ptr(key_cache, &s)? as *const c_void,
        dev_ptr(value_cache, &s)? as *const c_void,
        dev_ptr(block_tables, &s)? as *const u32,
        dev_ptr(context_lens, &s)? as *const u32,
        dev_ptr(cu_seqlens_q, &s)? as *const u32,
    );
    let st = if is_fp8(key_cache) {
        // the library needs the workspace only for page sizes its tcgen05
        // kernel does not read directly (it converts 16-token fp8 pages
        // itself); the entry point asks for it in every case
        let (k_sc, v_sc) = scales(k_scale, v_scale)?;
        let need = unsafe {
            ffi::vasr_pa_paged_attention_varlen_prefill_fp8_workspace_size(
                b as i32, hkv as i32, d as i32, bs as i32, cols as i32,
            )
        };
        let scratch = Tensor::zeros(need.max(1), DType::U8, q.device())?;
        unsafe {
            ffi::vasr_pa_paged_attention_varlen_prefill_fp8(
                args.0, args.1, args.2, args.3, args.4, args.5, args.6, b as i32, t as i64,
                max_query_len as i32, hq as i32, hkv as i32, d as i32, bs as i32, nb as i64,
                cols as i32, softmax_scale, softcapping, q.stride()[0] as i64, code,
                opt_ptr(Some(k_sc), &s)?, opt_ptr(Some(v_sc), &s)?, dev_ptr(&scratch, &s)?, need,
                raw_stream(&s),
            )
        }
    } else {
        unsafe {
            ffi::vasr_pa_paged_attention_varlen_prefill(
                args.0, args.1, args.2, args.3, args.4, args.5, args.6, b as i32, t as i64,
                max_query_len as i32, hq as i32, hkv as i32, d as i32, bs as i32, nb as i64,
                cols as i32, softmax_scale, softcapping, q.stride()[0] as i64, code, raw_stream(&s),
            )
        }
    };
    check("paged_attention_varlen_prefill", st)?;
    Ok(out)
}

// ------------------------------------------------------------- block ops
/// For every layer and (src, dst) pair of block_mapping (i64 [N, 2]): page
/// dst <- page src, K and V (fork / compaction; the allocator events of
/// paged_cache_runtime.rs:320-357). vLLM's name and argument order.
pub fn copy_blocks(key_caches: &[Tensor], value_caches: &[Tensor], block_mapping: &Tensor) -> Result<()> {
    if key_caches.is_empty() || key_caches.len() != value_caches.len() {
        candle_core::bail!("copy_blocks: one K and one V cache per layer");
    }
    let (nb, hkv, d, bs) = geometry(&key_caches[0], &value_caches[0])?;
    let (n, two) = block_mapping.dims2()?;
    if two != 2 || block_mapping.dtype() != DType::I64 {
        candle_core::bail!("copy_blocks: block_mapping must be i64 [N, 2]");
    }
    let s = stream_of(&key_caches[0])?;
    let mut k = Vec::with_capacity(key_caches.len());
    let mut v = Vec::with_capacity(value_caches.len());
    for (kc, vc) in key_caches.iter().zip(value_caches) {
        if geometry(kc, vc)? != (nb, hkv, d, bs) || kc.dtype() != key_caches[0].dtype() {
            candle_core::bail!("copy_blocks: all layers must share one cache geometry");
        }
        k.push(dev_ptr(kc, &s)?);
        v.push(dev_ptr(vc, &s)?);
    }
    let block_bytes = hkv * d * bs * key_caches[0].dtype().size_in_bytes();
    let st = unsafe {
        ffi::vasr_pa_copy_blocks(
            k.as_ptr(), v.as_ptr(), k.len() as i32, dev_ptr(block_mapping, &s)? as *const i64,
            n as i64, nb as i64, block_bytes as i64, raw_stream(&s),
        )
    };
    check("copy_blocks", st)
}

/// One side of a swap: a device cache tensor, or a pool of pinned host pages
/// (cudaHostAlloc'd, mapped, so the device addresses it directly). Candle has
/// no pinned host tensor, so the engine owns such a pool as a raw allocation
/// of `num_blocks` pages of the device cache's page geometry.
pub enum SwapSide<'a> {
    Device(&'a Tensor),
    PinnedHost { ptr: *mut c_void, num_blocks: usize },
}

/// dst[pair.1] <- src[pair.0] between a device cache and a pinned host pool
/// of one page geometry (eviction and restore); block_mapping is i64 [N, 2]
/// on the device. vLLM's name; the reference has no call site for it.
pub fn swap_blocks(src: SwapSide<'_>, dst: SwapSide<'_>, block_mapping: &Tensor) -> Result<()> {
    let (n, two) = block_mapping.dims2()?;
    if two != 2 || block_mapping.dtype() != DType::I64 {
        candle_core::bail!("swap_blocks: block_mapping must be i64 [N, 2]");
    }
    let s = stream_of(block_mapping)?;
    let page_bytes = |t: &Tensor| -> usize {
        let nb = t.dims()[0];
        if nb == 0 { 0 } else { t.elem_count() / nb * t.dtype().size_in_bytes() }
    };
    let block_bytes = match (&src, &dst) {
        (SwapSide::Device(a), SwapSide::Device(b)) => {
            if a.dtype() != b.dtype() || a.dims()[1..] != b.dims()[1..] {
                candle_core::bail!("swap_blocks: caches differ in geometry");
            }
            page_bytes(a)
        }
        (SwapSide::Device(t), _) | (_, SwapSide::Device(t)) => page_bytes(t),
        _ => candle_core::bail!("swap_blocks: one side must be a device cache"),
    };
    let side = |x: &SwapSide<'_>| -> Result<(*mut c_void, usize)> {
        match x {
            SwapSide::Device(t) => Ok((dev_ptr(t, &s)?, t.dims()[0])),
            SwapSide::PinnedHost { ptr, num_blocks } => Ok((*ptr, *num_blocks)),
        }
    };
    let (sp, sn) = side(&src)?;
    let (dp, dn) = side(&dst)?;
    let st = unsafe {
        ffi::vasr_pa_swap_blocks(
            dp, sp as *const c_void, dev_ptr(block_mapping, &s)? as *const i64, n as i64, sn as i64,
            dn as i64, block_bytes as i64, raw_stream(&s),
        )
    };
    check("swap_blocks", st)
}
