//! Safe wrapper over `nemo-relpos-sys` that keeps the signatures of the
//! mlx-voice `internals` attention API it replaces
//! (src/asr/modules/encoders/attention.rs, src/core/quantization.rs,
//! src/asr/streaming/core.rs), so the encoder's call sites
//! (`ConformerBlock::forward{,_with_cache}`, conformer.rs:1767-1769,
//! 1927-1933) change only their imports.
//!
//! `Array` plays the role of `mlx_rs::Array` on this path: a row-major tensor
//! in CUDA memory on one device, f32 or bf16.  Work is queued on the legacy
//! default stream; reading an `Array` back (`to_vec_f32`) synchronises.
//! Errors keep the reference's kinds (src/core/error.rs:7-60).
#![allow(clippy::missing_safety_doc)]

use nemo_relpos_sys as sys;
use std::collections::HashMap;
use std::ffi::{CStr, CString};
use std::os::raw::{c_int, c_void};
use std::ptr;
use std::sync::{Arc, Mutex, OnceLock};

// ------------------------------------------------------------------ errors
#[derive(Debug, Clone)]
pub enum Error {
    /// bad argument or shape (the reference's Error::Model / ShapeMismatch)
    Model(String),
    /// CUDA runtime or driver error (the role of Error::Mlx)
    Cuda(String),
    /// configuration the library does not implement (Error::NotImplemented)
    NotImplemented(String),
    /// a kernel gave up on a bounded wait (reported by nrp_context_check)
    Device(String),
}

pub type Result<T> = std::result::Result<T, Error>;

fn last_error() -> String {
    unsafe {
        let p = sys::nrp_last_error();
        if p.is_null() {
            String::new()
        } else {
            CStr::from_ptr(p).to_string_lossy().into_owned()
        }
    }
}

fn check(rc: c_int) -> Result<()> {
    match rc {
        sys::NRP_OK => Ok(()),
        sys::NRP_ERR_INVALID => Err(Error::Model(last_error())),
        sys::NRP_ERR_UNSUPPORTED => Err(Error::NotImplemented(last_error())),
        sys::NRP_ERR_DEVICE => Err(Error::Device(last_error())),
        _ => Err(Error::Cuda(last_error())),
    }
}

fn cuda(rc: c_int, what: &str) -> Result<()> {
    if rc == 0 {
        Ok(())
    } else {
        Err(Error::Cuda(format!("{what}: CUDA error {rc}")))
    }
}

// ----------------------------------------------------------------- context
/// One device's library context (error word, profiling, weight cache).
pub struct Context {
    raw: *mut sys::nrp_context,
    device: i32,
}

unsafe impl Send for Context {}
unsafe impl Sync for Context {}

impl Context {
    pub fn new(device: i32) -> Result<Arc<Self>> {
        let mut raw = ptr::null_mut();
        check(unsafe { sys::nrp_context_create(device, &mut raw) })?;
        Ok(Arc::new(Context { raw, device }))
    }

    /// The shared context of `device` (the reference has no context object:
    /// modules created without one use this).
    pub fn default_for(device: i32) -> Result<Arc<Self>> {
        static CTXS: OnceLock<Mutex<HashMap<i32, Arc<Context>>>> = OnceLock::new();
        let map = CTXS.get_or_init(|| Mutex::new(HashMap::new()));
        let mut m = map.lock().unwrap();
        if let Some(c) = m.get(&device) {
            return Ok(c.clone());
        }
        let c = Context::new(device)?;
        m.insert(device, c.clone());
        Ok(c)
    }

    /// Synchronises the default stream and reports a kernel's expired wait.
    pub fn check(&self) -> Result<()> {
        check(unsafe { sys::nrp_context_check(self.raw, ptr::null_mut()) })
    }

    pub fn device(&self) -> i32 {
        self.device
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        unsafe {
            sys::nrp_context_destroy(self.raw);
        }
    }
}

// ------------------------------------------------------------------- dtype
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum Dtype {
    Float32,
    Bfloat16,
}

impl Dtype {
    fn raw(self) -> c_int {
        match self {
            Dtype::Float32 => sys::NRP_DTYPE_F32,
            Dtype::Bfloat16 => sys::NRP_DTYPE_BF16,
        }
    }
    fn size(self) -> usize {
        match self {
            Dtype::Float32 => 4,
            Dtype::Bfloat16 => 2,
        }
    }
}

fn bf16_bits(x: f32) -> u16 {
    // round to nearest even (finite inputs)
    let b = x.to_bits();
    ((b + 0x7fff + ((b >> 16) & 1)) >> 16) as u16
}

// ------------------------------------------------------------------- array
/// A row-major tensor in CUDA memory (the role of `mlx_rs::Array`).
pub struct Array {
    ptr: *mut c_void,
    shape: Vec<i32>,
    dtype: Dtype,
    /// Per-utterance valid lengths, when this array is a key padding mask
    /// made by `key_padding_mask` (the forward then needs no read-back).
    lengths: Option<Vec<i32>>,
}

unsafe impl Send for Array {}

impl Array {
    fn alloc(shape: &[i32], dtype: Dtype) -> Result<Self> {
        let n: usize = shape.iter().map(|&d| d.max(0) as usize).product();
        let mut p = ptr::null_mut();
        cuda(unsafe { sys::cuda::cudaMalloc(&mut p, (n * dtype.size()).max(16)) }, "cudaMalloc")?;
        Ok(Array { ptr: p, shape: shape.to_vec(), dtype, lengths: None })
    }

    pub fn zeros(shape: &[i32], dtype: Dtype) -> Result<Self> {
        let a = Self::alloc(shape, dtype)?;
        cuda(unsafe { sys::cuda::cudaMemsetAsync(a.ptr, 0, a.bytes(), ptr::null_mut()) },
             "cudaMemsetAsync")?;
        Ok(a)
    }

    /// Host f32 data to the device in `dtype` (bf16: rounded to nearest even).
    pub fn from_f32(data: &[f32], shape: &[i32], dtype: Dtype) -> Result<Self> {
        let n: usize = shape.iter().map(|&d| d as usize).product();
        if n != data.len() {
            return Err(Error::Model(format!("{} values for shape {:?}", data.len(), shape)));
        }
        let a = Self::alloc(shape, dtype)?;
        let kind = sys::cuda::MEMCPY_HOST_TO_DEVICE;
        let rc = match dtype {
            Dtype::Float32 => unsafe {
                sys::cuda::cudaMemcpy(a.ptr, data.as_ptr() as *const c_void, a.bytes(), kind)
            },
            Dtype::Bfloat16 => {
                let h: Vec<u16> = data.iter().map(|&x| bf16_bits(x)).collect();
                unsafe { sys::cuda::cudaMemcpy(a.ptr, h.as_ptr() as *const c_void, a.bytes(), kind) }
            }
        };
        cuda(rc, "cudaMemcpy")?;
        Ok(a)
    }

    /// The values as f32 on the host (synchronises).
    pub fn to_vec_f32(&self) -> Result<Vec<f32>> {
        let n = self.len();
        let kind = sys::cuda::MEMCPY_DEVICE_TO_HOST;
        match self.dtype {
            Dtype::Float32 => {
                let mut v = vec![0f32; n];
                cuda(unsafe { sys::cuda::cudaMemcpy(v.as_mut_ptr() as *mut c_void, self.ptr,
                                                    self.bytes(), kind) }, "cudaMemcpy")?;
                Ok(v)
            }
            Dtype::Bfloat16 => {
                let mut v = vec![0u16; n];
                cuda(unsafe { sys::cuda::cudaMemcpy(v.as_mut_ptr() as *mut c_void, self.ptr,
                                                    self.bytes(), kind) }, "cudaMemcpy")?;
                Ok(v.into_iter().map(|b| f32::from_bits((b as u32) << 16)).collect())
            }
        }
    }

    pub fn shape(&self) -> &[i32] {
        &self.shape
    }
    pub fn dtype(&self) -> Dtype {
        self.dtype
    }
    pub fn len(&self) -> usize {
        self.shape.iter().map(|&d| d.max(0) as usize).product()
    }
    pub fn is_empty(&self) -> bool {
        self.len() == 0
    }
    fn bytes(&self) -> usize {
        self.len() * self.dtype.size()
    }
    pub fn as_ptr(&self) -> *const c_void {
        self.ptr
    }
}

impl Drop for Array {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe {
                sys::cuda::cudaFree(self.ptr);
            }
        }
    }
}

/// Device int32 buffer (per-utterance lengths handed to the kernels).
struct Lengths {
    ptr: *mut c_void,
    cap: usize,
}

impl Lengths {
    fn upload(&mut self, v: &[i32]) -> Result<*const i32> {
        if v.len() > self.cap {
            if !self.ptr.is_null() {
                unsafe { sys::cuda::cudaFree(self.ptr) };
                self.ptr = ptr::null_mut();
            }
            cuda(unsafe { sys::cuda::cudaMalloc(&mut self.ptr, v.len() * 4) }, "cudaMalloc")?;
            self.cap = v.len();
        }
        cuda(unsafe { sys::cuda::cudaMemcpy(self.ptr, v.as_ptr() as *const c_void, v.len() * 4,
                                            sys::cuda::MEMCPY_HOST_TO_DEVICE) }, "cudaMemcpy")?;
        Ok(self.ptr as *const i32)
    }
}

impl Drop for Lengths {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe { sys::cuda::cudaFree(self.ptr) };
        }
    }
}

// ------------------------------------------------------ positional encoding
/// RelPositionalEncoding (attention.rs:35-188).
pub struct RelPositionalEncoding {
    d_model: i32,
    max_len: i32,
    xscaling: bool,
    dtype: Dtype,
    ctx: Arc<Context>,
}

impl RelPositionalEncoding {
    /// attention.rs:35-51.
    pub fn new(d_model: i32, max_len: i32, xscaling: bool) -> Self {
        let ctx = Context::default_for(0).expect("CUDA device 0");
        RelPositionalEncoding { d_model, max_len, xscaling, dtype: Dtype::Float32, ctx }
    }
    /// get_encoding (attention.rs:131-177): [1, 2 seq_len - 1, d_model].
    pub fn get_encoding(&self, seq_len: i32) -> Result<Array> {
        let out = Array::alloc(&[1, 2 * seq_len - 1, self.d_model], self.dtype)?;
        check(unsafe {
            sys::nrp_pe_encoding(self.ctx.raw, self.d_model, self.max_len, seq_len,
                                 self.dtype.raw(), out.ptr, ptr::null_mut())
        })?;
        Ok(out)
    }
    /// set_dtype (attention.rs:180-183).
    pub fn set_dtype(&mut self, dtype: Dtype) {
        self.dtype = dtype;
    }
    /// xscale (attention.rs:186-188).
    pub fn xscale(&self) -> f32 {
        unsafe { sys::nrp_pe_xscale(self.d_model, self.xscaling as c_int) }
    }
    pub fn d_model(&self) -> i32 {
        self.d_model
    }
}

// ---------------------------------------------------------------- contexts
/// AttentionContext (attention.rs:210-273).
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub struct AttentionContext {
    pub left: i32,
    pub right: i32,
    pub chunked: bool,
}

impl AttentionContext {
    /// attention.rs:220-227: None when both bounds are negative.
    pub fn new(size: (i32, i32), style: &str) -> Option<Self> {
        let s = CString::new(style).ok()?;
        let mut c = sys::nrp_att_context { left: 0, right: 0, chunked: 0 };
        let rc = unsafe { sys::nrp_att_context_new(size.0, size.1, s.as_ptr(), &mut c) };
        if rc == 1 {
            Some(AttentionContext { left: c.left, right: c.right, chunked: c.chunked != 0 })
        } else {
            None
        }
    }
    fn raw(&self) -> sys::nrp_att_context {
        sys::nrp_att_context { left: self.left, right: self.right, chunked: self.chunked as i32 }
    }
}

/// key_padding_mask (attention.rs:280-294): the additive mask [B, 1, 1, T]
/// (0 or -inf, each row keeping max(len, 1) keys), or None when no frame is
/// padding.  The returned array remembers `lengths`, so a forward given it
/// reads nothing back.
pub fn key_padding_mask(lengths: &[i32], max_len: i32) -> Result<Option<Array>> {
    let b = lengths.len() as i32;
    let mut host = vec![0f32; lengths.len() * max_len as usize];
    let rc = unsafe {
        sys::nrp_key_padding_mask_host(lengths.as_ptr(), b, max_len, host.as_mut_ptr())
    };
    if rc < 0 {
        return Err(check(rc).unwrap_err());
    }
    if rc == 0 {
        return Ok(None);
    }
    let mut a = Array::from_f32(&host, &[b, 1, 1, max_len], Dtype::Float32)?;
    a.lengths = Some(lengths.to_vec());
    Ok(Some(a))
}

/// The lengths an additive key mask [B, 1, 1, T] encodes (keys at and past
/// the length are -inf); a mask that is not of that form is an error.
fn mask_lengths(mask: &Array) -> Result<Vec<i32>> {
    if let Some(l) = &mask.lengths {
        return Ok(l.clone());
    }
    let s = mask.shape();
    let t = *s.last().unwrap_or(&0) as usize;
    let v = mask.to_vec_f32()?;
    let rows = if t == 0 { 0 } else { v.len() / t };
    let mut out = Vec::with_capacity(rows);
    for r in 0..rows {
        let row = &v[r * t..(r + 1) * t];
        let len = row.iter().take_while(|&&m| m == 0.0).count();
        if row[len..].iter().any(|&m| m != f32::NEG_INFINITY) {
            return Err(Error::NotImplemented(
                "key masks other than a padding suffix per utterance".into()));
        }
        out.push(len as i32);
    }
    Ok(out)
}

// ------------------------------------------------------------ quantisation
/// QuantizationConfig (quantization.rs:14-31): MLX affine, 8 bits, group 64
/// on this path.
#[derive(Clone, Copy, Debug)]
pub struct QuantizationConfig {
    pub bits: i32,
    pub group_size: i32,
}

impl Default for QuantizationConfig {
    fn default() -> Self {
        QuantizationConfig { bits: 8, group_size: 64 }
    }
}

/// A host tensor of a checkpoint: f32 values, or packed u32 codes.
pub enum HostTensor {
    F32 { data: Vec<f32>, shape: Vec<usize> },
    U32 { data: Vec<u32>, shape: Vec<usize> },
}

/// Named checkpoint tensors (the role of core::Weights, loading.rs).
#[derive(Default)]
pub struct Weights {
    pub tensors: HashMap<String, HostTensor>,
}

impl Weights {
    fn f32(&self, key: &str) -> Option<&[f32]> {
        match self.tensors.get(key) {
            Some(HostTensor::F32 { data, .. }) => Some(data),
            _ => None,
        }
    }
    fn u32(&self, key: &str) -> Option<&[u32]> {
        match self.tensors.get(key) {
            Some(HostTensor::U32 { data, .. }) => Some(data),
            _ => None,
        }
    }
}

// --------------------------------------------------------------- attention
/// The module's ring of cached attention inputs (and their K/V projections)
/// behind forward_with_cache, with the cache array it last returned.
struct Ring {
    raw: *mut sys::nrp_cache,
    batch: i32,
    cache_len: i32,
    last: Option<*const c_void>,
}

/// RelPositionMultiHeadAttention (attention.rs:328-893).
pub struct RelPositionMultiHeadAttention {
    raw: *mut sys::nrp_attn,
    ctx: Arc<Context>,
    d_model: i32,
    n_heads: i32,
    dtype: Dtype,
    /// attention.rs:349-350 (set by ConformerEncoder::setup_streaming)
    pub cache_drop_size: i32,
    /// attention.rs:351-354
    pub att_context_size: Option<AttentionContext>,
    lengths: Lengths,
    ring: Option<Ring>,
}

unsafe impl Send for RelPositionMultiHeadAttention {}

const LINEARS: [(&str, c_int); 5] = [
    ("linear_q", sys::NRP_LINEAR_Q),
    ("linear_k", sys::NRP_LINEAR_K),
    ("linear_v", sys::NRP_LINEAR_V),
    ("linear_out", sys::NRP_LINEAR_OUT),
    ("linear_pos", sys::NRP_LINEAR_POS),
];

impl RelPositionMultiHeadAttention {
    /// attention.rs:367-406 (zero parameters, f32).
    pub fn new(d_model: i32, n_heads: i32, use_bias: bool) -> Result<Self> {
        let ctx = Context::default_for(0)?;
        let mut raw = ptr::null_mut();
        check(unsafe { sys::nrp_attn_create(ctx.raw, d_model, n_heads, use_bias as c_int,
                                            &mut raw) })?;
        Ok(RelPositionMultiHeadAttention {
            raw, ctx, d_model, n_heads, dtype: Dtype::Float32, cache_drop_size: 0,
            att_context_size: None, lengths: Lengths { ptr: ptr::null_mut(), cap: 0 },
            ring: None,
        })
    }

    pub fn head_dim(&self) -> i32 {
        self.d_model / self.n_heads
    }
    pub fn n_heads(&self) -> i32 {
        self.n_heads
    }

    /// set_dtype (attention.rs:409-423).
    pub fn set_dtype(&mut self, dtype: Dtype) -> Result<()> {
        check(unsafe { sys::nrp_attn_set_dtype(self.raw, dtype.raw()) })?;
        self.dtype = dtype;
        Ok(())
    }

    /// load_weights (attention.rs:863-893): `{prefix}.linear_{q,k,v,out,pos}`
    /// (`.weight`, `.bias`; quantised: `.scales`, `.biases`, u32 `.weight`)
    /// and `{prefix}.pos_bias_{u,v}`.  A layer is quantised when its
    /// `.scales` is present (load_linear_layer, quantization.rs:327-345).
    pub fn load_weights(&mut self, weights: &Weights, prefix: &str,
                        quant: Option<&QuantizationConfig>) -> Result<()> {
        for (name, which) in LINEARS {
            let key = format!("{prefix}.{name}");
            let bias = weights.f32(&format!("{key}.bias")).map_or(ptr::null(), |b| b.as_ptr());
            if let Some(scales) = weights.f32(&format!("{key}.scales")) {
                let q = quant.copied().unwrap_or_default();
                let wq = weights.u32(&format!("{key}.weight"))
                    .ok_or_else(|| Error::Model(format!("{key}.weight: u32 codes missing")))?;
                let biases = weights.f32(&format!("{key}.biases"))
                    .ok_or_else(|| Error::Model(format!("{key}.biases missing")))?;
                check(unsafe {
                    sys::nrp_attn_load_linear_quantized(self.raw, which, q.bits, q.group_size,
                                                        wq.as_ptr(), scales.as_ptr(),
                                                        biases.as_ptr(), bias)
                })?;
            } else {
                let w = weights.f32(&format!("{key}.weight"))
                    .ok_or_else(|| Error::Model(format!("{key}.weight missing")))?;
                check(unsafe { sys::nrp_attn_load_linear(self.raw, which, w.as_ptr(), bias) })?;
            }
        }
        let u = weights.f32(&format!("{prefix}.pos_bias_u"))
            .ok_or_else(|| Error::Model(format!("{prefix}.pos_bias_u missing")))?;
        let v = weights.f32(&format!("{prefix}.pos_bias_v"))
            .ok_or_else(|| Error::Model(format!("{prefix}.pos_bias_v missing")))?;
        check(unsafe { sys::nrp_attn_load_pos_bias(self.raw, u.as_ptr(), v.as_ptr()) })
    }

    fn check_input(&self, x: &Array) -> Result<(i32, i32)> {
        let s = x.shape();
        if s.len() != 3 || s[2] != self.d_model || x.dtype() != self.dtype {
            return Err(Error::Model(format!(
                "x {:?} {:?}: expected [B, T, {}] in the module dtype {:?}", s, x.dtype(),
                self.d_model, self.dtype)));
        }
        Ok((s[0], s[1]))
    }

    /// forward (attention.rs:446-573): x [B, T, d_model], pos_emb from
    /// RelPositionalEncoding::get_encoding(T); key_mask from
    /// key_padding_mask (its lengths are used; any other additive suffix
    /// mask is read back once).  Rows past an utterance's length are
    /// unspecified, as in the reference (conformer.rs:1590-1593).
    pub fn forward(&mut self, x: &Array, pos_emb: &Array, context: Option<AttentionContext>,
                   key_mask: Option<&Array>) -> Result<Array> {
        let (b, t) = self.check_input(x)?;
        let lengths = match key_mask {
            Some(m) => {
                let l = mask_lengths(m)?;
                if l.len() != b as usize {
                    return Err(Error::Model(format!("{} mask rows for batch {b}", l.len())));
                }
                self.lengths.upload(&l)?
            }
            None => ptr::null(),
        };
        let ctx = context.map(|c| c.raw());
        let out = Array::alloc(&[b, t, self.d_model], self.dtype)?;
        check(unsafe {
            sys::nrp_attn_forward(self.raw, ptr::null_mut(), x.ptr, b, t, pos_emb.ptr, lengths,
                                  ctx.as_ref().map_or(ptr::null(), |c| c as *const _), out.ptr)
        })?;
        Ok(out)
    }

    /// forward_with_cache (attention.rs:606-816) as
    /// ConformerEncoder::forward_streaming drives it: cache is the layer's
    /// `EncoderCache.last_channel` slice [B, cache_len, d_model] (f32);
    /// returns the output and the next cache.  The library keeps the cache
    /// as a device ring with its K/V projections, so a cache array this
    /// module returned is used in place; any other is imported (and its K/V
    /// re-projected).  att_mask is create_attention_mask's bool mask
    /// [1, T, cache_len + T] or None; only the number of query rows that
    /// see keys (the valid frames) is read from it, as the library builds
    /// the mask itself from `filled` and `att_context_size`
    /// (conformer.rs:97-221).  A call without a cache is the offline forward.
    pub fn forward_with_cache(&mut self, x: &Array, pos_emb: &Array, cache: Option<&Array>,
                              filled: i32, att_mask: Option<&Array>)
                              -> Result<(Array, Option<Array>)> {
        let (b, t) = self.check_input(x)?;
        let cache = match cache {
            None => return Ok((self.forward(x, pos_emb, self.att_context_size, None)?, None)),
            Some(c) => c,
        };
        let cs = cache.shape();
        if cs.len() != 3 || cs[0] != b || cs[2] != self.d_model || cache.dtype() != Dtype::Float32 {
            return Err(Error::Model(format!("cache {cs:?}: expected [{b}, C, {}] f32",
                                            self.d_model)));
        }
        let valid = match att_mask {
            None => t,
            Some(m) => {
                let v = m.to_vec_f32()?;
                let tk = *m.shape().last().unwrap_or(&0) as usize;
                (0..t as usize).filter(|&r| v[r * tk..(r + 1) * tk].iter().any(|&e| e != 0.0))
                    .count() as i32
            }
        };
        self.ensure_ring(b, cs[1])?;
        let ring = self.ring.as_mut().unwrap();
        if ring.last != Some(cache.ptr as *const c_void) {
            check(unsafe { sys::nrp_cache_import_h(ring.raw, cache.ptr as *const f32,
                                                   ptr::null_mut()) })?;
        }
        check(unsafe { sys::nrp_attn_set_cache_drop_size(self.raw, self.cache_drop_size) })?;
        let ctx = self.att_context_size.map(|c| c.raw());
        let out = Array::alloc(&[b, t, self.d_model], self.dtype)?;
        check(unsafe {
            sys::nrp_attn_forward_with_cache(self.raw, ptr::null_mut(), x.ptr, b, t, pos_emb.ptr,
                                             ring.raw, filled, valid,
                                             ctx.as_ref().map_or(ptr::null(), |c| c as *const _),
                                             out.ptr)
        })?;
        let next = Array::alloc(&[b, ring.cache_len, self.d_model], Dtype::Float32)?;
        check(unsafe { sys::nrp_cache_export_h(ring.raw, next.ptr as *mut f32, ptr::null_mut()) })?;
        ring.last = Some(next.ptr as *const c_void);
        Ok((out, Some(next)))
    }

    fn ensure_ring(&mut self, batch: i32, cache_len: i32) -> Result<()> {
        if let Some(r) = &self.ring {
            if r.batch == batch && r.cache_len == cache_len {
                return Ok(());
            }
            unsafe { sys::nrp_cache_destroy(r.raw) };
            self.ring = None;
        }
        let mut raw = ptr::null_mut();
        check(unsafe { sys::nrp_cache_create(self.raw, batch, cache_len, &mut raw) })?;
        self.ring = Some(Ring { raw, batch, cache_len, last: None });
        Ok(())
    }

    /// The forward with its intermediates in the library's static device
    /// array (nrp_attn_forward_noalloc): for a caller that cannot let the
    /// library allocate.  key_mask must come from key_padding_mask.
    pub fn forward_noalloc(&mut self, x: &Array, pos_emb: &Array, context: Option<AttentionContext>,
                           key_mask: Option<&Array>, out: &mut Array) -> Result<()> {
        let (b, t) = self.check_input(x)?;
        let lengths = match key_mask {
            Some(m) => self.lengths.upload(&mask_lengths(m)?)?,
            None => ptr::null(),
        };
        let ctx = context.map(|c| c.raw());
        check(unsafe {
            sys::nrp_attn_forward_noalloc(self.raw, ptr::null_mut(), x.ptr, b, t, pos_emb.ptr,
                                          lengths, ctx.as_ref().map_or(ptr::null(), |c| c as *const _),
                                          out.ptr)
        })
    }

    pub fn context(&self) -> &Arc<Context> {
        &self.ctx
    }
}

impl Drop for RelPositionMultiHeadAttention {
    fn drop(&mut self) {
        unsafe {
            if let Some(r) = self.ring.take() {
                sys::nrp_cache_destroy(r.raw);
            }
            sys::nrp_attn_destroy(self.raw);
        }
    }
}

// --------------------------------------------------------------- streaming
/// StreamingConfig (src/asr/streaming/core.rs:27-67).
pub type StreamingConfig = sys::nrp_streaming_config;

/// compute_streaming_config (src/asr/streaming/core.rs:247-362).
#[allow(clippy::too_many_arguments)]
pub fn compute_streaming_config(att_context_size: (i32, i32), chunked_limited: bool,
                                n_layers: i32, subsampling_factor: i32, conv_kernel_size: i32,
                                causal_conv: bool, mode_idx: i32, max_context: i32)
                                -> Result<StreamingConfig> {
    let mut out = StreamingConfig::default();
    check(unsafe {
        sys::nrp_streaming_config_compute(att_context_size.0, att_context_size.1,
                                          chunked_limited as c_int, n_layers, subsampling_factor,
                                          conv_kernel_size, causal_conv as c_int, mode_idx,
                                          max_context, &mut out)
    })?;
    Ok(out)
}

/// EncoderCache (src/asr/streaming/core.rs:117-185): one
/// `last_channel` array [B, cache_len, d_model] per layer (f32, zeroed),
/// the conv caches [B, d_model, conv_kernel - 1] per layer, and the fill
/// level of each stream.
pub struct EncoderCache {
    pub last_channel: Vec<Array>,
    pub last_time: Vec<Array>,
    pub last_channel_len: Vec<i64>,
}

impl EncoderCache {
    pub fn new(n_layers: usize, batch: i32, cache_len: i32, d_model: i32, conv_kernel: i32)
               -> Result<Self> {
        let mut last_channel = Vec::with_capacity(n_layers);
        let mut last_time = Vec::with_capacity(n_layers);
        for _ in 0..n_layers {
            last_channel.push(Array::zeros(&[batch, cache_len, d_model], Dtype::Float32)?);
            last_time.push(Array::zeros(&[batch, d_model, conv_kernel - 1], Dtype::Float32)?);
        }
        Ok(EncoderCache { last_channel, last_time, last_channel_len: vec![0; batch as usize] })
    }
}
