//! arctic-embed-s int8 embeddings on B200 GPUs, with the public API of the reference crate
//! `arctic_embed_s_int8` (mdlockyer/snowflake-arctic-embed-s-rust): `ArcticEmbedS::from_dir`,
//! `embed_document` / `embed_query` / `embed_tokens` with a `Workspace`, the `*_parallel` variants
//! with a `ParallelContext`, `embed_batch`, `cosine_similarity` (src/lib.rs:18-271,
//! src/parallel.rs:137-254, src/model.rs:123-179). The forward pass, the `.ae8` loader and the
//! WordPiece tokenizer run in libarctic_cuda.so behind the C ABI of include/arctic_cuda.h
//! (`cuda_ffi`); there is no CPU fallback.
//!
//! Differences a caller sees:
//! * `GpuModel` takes the place of `PackedModel`: one context per GPU, each behind a mutex (a
//!   context is not thread-safe), so `ArcticEmbedS` stays `Sync` and is shared across threads as the
//!   reference's is. `Workspace` keeps only the token-id buffer; the device workspace lives in the
//!   context.
//! * `embed_batch` shards the texts over every GPU the model was loaded on
//!   (`ae_embed_batch_multi`); `num_threads` sets the tokenizer's host threads only.
//! * Errors: loading returns `io::Result` (a malformed pack is `ErrorKind::InvalidData`); the embed
//!   calls panic with the library's message where the reference panics (empty input, token ids out
//!   of range) and on a CUDA failure.

pub mod cuda_ffi;

use cuda_ffi as ffi;
use std::ffi::{c_int, CStr, CString};
use std::io;
use std::os::unix::ffi::OsStrExt;
use std::path::{Path, PathBuf};
use std::sync::Mutex;

pub const HIDDEN_SIZE: usize = ffi::AE_HIDDEN;
pub const MAX_POSITIONS: usize = ffi::AE_MAX_POSITIONS;
/// File names inside a model directory and the environment variable naming it (src/lib.rs:18-23).
pub const MODEL_FILE: &str = "model.ae8";
pub const VOCAB_FILE: &str = "vocab.txt";
pub const MODEL_DIR_ENV_VAR: &str = "ARCTIC_EMBED_MODEL_DIR";
/// Prefix of search queries (src/tokenizer.rs:23).
pub const QUERY_PREFIX: &str = "Represent this sentence for searching relevant passages: ";

/// `$ARCTIC_EMBED_MODEL_DIR` if set, otherwise `./model` (src/lib.rs:27-31).
pub fn default_model_dir() -> PathBuf {
    std::env::var_os(MODEL_DIR_ENV_VAR).map(PathBuf::from).unwrap_or_else(|| PathBuf::from("model"))
}

fn error_of(code: c_int, msg: String) -> io::Error {
    let kind = match code {
        ffi::AE_ERR_BAD_PACK => io::ErrorKind::InvalidData,
        ffi::AE_ERR_INVALID_ARG | ffi::AE_ERR_TOKEN_RANGE => io::ErrorKind::InvalidInput,
        ffi::AE_ERR_CAPACITY => io::ErrorKind::OutOfMemory,
        _ => io::ErrorKind::Other,
    };
    io::Error::new(kind, msg)
}

fn check(ctx: *const ffi::ae_ctx, code: c_int) -> io::Result<()> {
    if code == ffi::AE_OK {
        return Ok(());
    }
    // SAFETY: ae_last_error returns a NUL-terminated string owned by the context (or by the library
    // for a null context) that stays valid until the next call on that context.
    let msg = unsafe { CStr::from_ptr(ffi::ae_last_error(ctx)) }.to_string_lossy().into_owned();
    Err(error_of(code, msg))
}

fn c_path(p: &Path) -> io::Result<CString> {
    CString::new(p.as_os_str().as_bytes()).map_err(|_| io::Error::new(io::ErrorKind::InvalidInput, "NUL in path"))
}

/// One GPU context with the model uploaded (`ae_ctx`).
struct Ctx(*mut ffi::ae_ctx);

// SAFETY: a context may be driven from any thread as long as one thread at a time does so; GpuModel
// keeps every Ctx behind a Mutex.
unsafe impl Send for Ctx {}

impl Ctx {
    fn new(device: i32) -> io::Result<Self> {
        let mut h = std::ptr::null_mut();
        // SAFETY: `h` is a valid out-pointer.
        check(std::ptr::null(), unsafe { ffi::ae_ctx_create(device, &mut h) })?;
        Ok(Self(h))
    }
}

impl Drop for Ctx {
    fn drop(&mut self) {
        // SAFETY: the handle came from ae_ctx_create and is destroyed once.
        unsafe { ffi::ae_ctx_destroy(self.0) };
    }
}

/// The borrowed arrays of one int8 linear layer (the fields of the reference's
/// `QuantizedLinearRaw`, src/quantize.rs:22-30). `n_out == 0` marks the pruned layer-11 QKV.
#[derive(Clone, Copy)]
pub struct LinearView<'a> {
    pub n_out: usize,
    pub k_in: usize,
    pub w_q: &'a [i8],
    pub w_scale: &'a [f32],
    pub bias: &'a [f32],
    pub inv_smooth: &'a [f32],
}

/// One encoder layer (`QuantizedLayerRaw`, src/quantize.rs:46-58).
#[derive(Clone, Copy)]
pub struct LayerView<'a> {
    pub qkv: LinearView<'a>,
    pub q_only: Option<LinearView<'a>>,
    pub kv_only: Option<LinearView<'a>>,
    pub attn_out: LinearView<'a>,
    pub ln1_weight: &'a [f32],
    pub ln1_bias: &'a [f32],
    pub ffn_inter: LinearView<'a>,
    pub ffn_out: LinearView<'a>,
    pub ln2_weight: &'a [f32],
    pub ln2_bias: &'a [f32],
}

/// The whole quantized model (`QuantizedModelRaw`, src/quantize.rs:60-72), borrowed: a crate that
/// keeps the reference's `.ae8` loader fills this from its `QuantizedModelRaw` field by field.
pub struct ModelView<'a> {
    pub word_emb_q: &'a [i8],
    pub word_emb_scale: &'a [f32],
    pub pos_emb_q: &'a [i8],
    pub pos_emb_scale: &'a [f32],
    pub type_emb_q: &'a [i8],
    pub type_emb_scale: &'a [f32],
    pub emb_ln_weight: &'a [f32],
    pub emb_ln_bias: &'a [f32],
    pub layers: Vec<LayerView<'a>>,
}

fn linear_desc(l: &LinearView<'_>) -> ffi::ae_linear_desc {
    let ptr_or_null = |s: &[i8]| if s.is_empty() { std::ptr::null() } else { s.as_ptr() };
    ffi::ae_linear_desc {
        n_out: l.n_out as u64,
        k_in: l.k_in as u64,
        w_q: ptr_or_null(l.w_q),
        w_scale: l.w_scale.as_ptr(),
        bias: l.bias.as_ptr(),
        inv_smooth: l.inv_smooth.as_ptr(),
    }
}

const EMPTY_LINEAR: ffi::ae_linear_desc = ffi::ae_linear_desc {
    n_out: 0,
    k_in: 0,
    w_q: std::ptr::null(),
    w_scale: std::ptr::null(),
    bias: std::ptr::null(),
    inv_smooth: std::ptr::null(),
};

impl ModelView<'_> {
    fn desc(&self) -> io::Result<ffi::ae_model_desc> {
        if self.layers.len() != 12 {
            return Err(io::Error::new(io::ErrorKind::InvalidData, "expected 12 layers"));
        }
        let layer = |l: &LayerView<'_>| ffi::ae_layer_desc {
            qkv: linear_desc(&l.qkv),
            has_split: (l.q_only.is_some() && l.kv_only.is_some()) as i32,
            q_only: l.q_only.as_ref().map(linear_desc).unwrap_or(EMPTY_LINEAR),
            kv_only: l.kv_only.as_ref().map(linear_desc).unwrap_or(EMPTY_LINEAR),
            attn_out: linear_desc(&l.attn_out),
            ln1_weight: l.ln1_weight.as_ptr(),
            ln1_bias: l.ln1_bias.as_ptr(),
            ffn_inter: linear_desc(&l.ffn_inter),
            ffn_out: linear_desc(&l.ffn_out),
            ln2_weight: l.ln2_weight.as_ptr(),
            ln2_bias: l.ln2_bias.as_ptr(),
        };
        let layers: Vec<ffi::ae_layer_desc> = self.layers.iter().map(layer).collect();
        Ok(ffi::ae_model_desc {
            word_emb_q: self.word_emb_q.as_ptr(),
            word_emb_scale: self.word_emb_scale.as_ptr(),
            pos_emb_q: self.pos_emb_q.as_ptr(),
            pos_emb_scale: self.pos_emb_scale.as_ptr(),
            type_emb_q: self.type_emb_q.as_ptr(),
            type_emb_scale: self.type_emb_scale.as_ptr(),
            emb_ln_weight: self.emb_ln_weight.as_ptr(),
            emb_ln_bias: self.emb_ln_bias.as_ptr(),
            layers: layers.try_into().map_err(|_| io::Error::new(io::ErrorKind::InvalidData, "expected 12 layers"))?,
        })
    }
}

/// `PackedModel` on one or more GPUs: the model uploaded into one context per device.
pub struct GpuModel {
    ctxs: Vec<Mutex<Ctx>>,
    devices: Vec<i32>,
}

impl GpuModel {
    /// `QuantizedModelRaw::load_ae8` + `PackedModel::from_raw` (src/quantize.rs:76-137,
    /// src/model.rs:49-84) on each device: the pack is parsed and validated by the library.
    pub fn load_ae8<P: AsRef<Path>>(path: P, devices: &[i32]) -> io::Result<Self> {
        let p = c_path(path.as_ref())?;
        let mut ctxs = Vec::with_capacity(devices.len());
        for &d in devices {
            let c = Ctx::new(d)?;
            // SAFETY: valid context and NUL-terminated path.
            check(c.0, unsafe { ffi::ae_model_load_file(c.0, p.as_ptr()) })?;
            ctxs.push(Mutex::new(c));
        }
        Ok(Self { ctxs, devices: devices.to_vec() })
    }

    /// Uploads a model held in host memory (the reference's `QuantizedModelRaw`, as a view).
    pub fn from_view(view: &ModelView<'_>, devices: &[i32]) -> io::Result<Self> {
        let desc = view.desc()?;
        let mut ctxs = Vec::with_capacity(devices.len());
        for &d in devices {
            let c = Ctx::new(d)?;
            // SAFETY: every pointer in `desc` borrows from `view`, alive for the call.
            check(c.0, unsafe { ffi::ae_model_load(c.0, &desc) })?;
            ctxs.push(Mutex::new(c));
        }
        Ok(Self { ctxs, devices: devices.to_vec() })
    }

    pub fn devices(&self) -> &[i32] {
        &self.devices
    }

    /// `PackedModel::forward_cls` (src/model.rs:185-513) on the first device: one sequence,
    /// truncated to 512 ids, replayed from a CUDA graph per length.
    pub fn forward_cls(&self, input_ids: &[u16], out: &mut [f32; HIDDEN_SIZE]) -> io::Result<()> {
        let c = self.ctxs[0].lock().unwrap_or_else(|e| e.into_inner());
        // SAFETY: `input_ids` and `out` are valid for the lengths passed.
        check(c.0, unsafe { ffi::ae_forward_cls(c.0, input_ids.as_ptr(), input_ids.len() as u32, out.as_mut_ptr()) })
    }

    /// `PackedModel::forward_ragged_cls` (src/model.rs:521-914) on the first device, without its
    /// 64-sequence and 512-row limits.
    pub fn forward_ragged_cls(&self, seqs: &[&[u16]], out: &mut [[f32; HIDDEN_SIZE]]) -> io::Result<()> {
        assert_eq!(seqs.len(), out.len(), "one output row per sequence");
        let (ids, cu) = pack(seqs.iter().copied());
        let c = self.ctxs[0].lock().unwrap_or_else(|e| e.into_inner());
        // SAFETY: ids / cu / out hold cu[n] ids, n + 1 offsets and n rows.
        check(c.0, unsafe {
            ffi::ae_forward_ragged(c.0, ids.as_ptr(), cu.as_ptr(), seqs.len() as u32, out.as_mut_ptr() as *mut f32)
        })
    }

    /// `embed_batch`'s device part over every context (`ae_embed_batch_multi`): token-weighted
    /// shards, one host thread per GPU, results in input order.
    pub fn embed_batch_tokens(&self, ids: &[u16], cu_seqlens: &[u32], out: &mut [[f32; HIDDEN_SIZE]]) -> io::Result<()> {
        let n = cu_seqlens.len().saturating_sub(1);
        assert_eq!(out.len(), n, "one output row per sequence");
        let guards: Vec<_> = self.ctxs.iter().map(|m| m.lock().unwrap_or_else(|e| e.into_inner())).collect();
        let handles: Vec<*mut ffi::ae_ctx> = guards.iter().map(|g| g.0).collect();
        // SAFETY: every context is locked for the call; buffers hold what cu_seqlens describes.
        check(handles[0], unsafe {
            ffi::ae_embed_batch_multi(handles.as_ptr(), handles.len() as c_int, ids.as_ptr(), cu_seqlens.as_ptr(),
                                      n as u32, 0, out.as_mut_ptr() as *mut f32)
        })
    }
}

fn pack<'a>(seqs: impl Iterator<Item = &'a [u16]>) -> (Vec<u16>, Vec<u32>) {
    let mut ids = Vec::new();
    let mut cu = vec![0u32];
    for s in seqs {
        ids.extend_from_slice(s);
        cu.push(ids.len() as u32);
    }
    (ids, cu)
}

/// `BertTokenizer` (src/tokenizer.rs:25-327) in the library: same ids, immutable, shareable.
pub struct BertTokenizer(*mut ffi::ae_tokenizer);

// SAFETY: the tokenizer is immutable after creation (include/arctic_cuda.h).
unsafe impl Send for BertTokenizer {}
unsafe impl Sync for BertTokenizer {}

fn tokenizer_error() -> io::Error {
    // SAFETY: a NUL-terminated thread-local message of the library.
    let msg = unsafe { CStr::from_ptr(ffi::ae_tokenizer_last_error()) }.to_string_lossy().into_owned();
    io::Error::new(io::ErrorKind::InvalidData, msg)
}

impl BertTokenizer {
    pub fn from_vocab_file<P: AsRef<Path>>(path: P) -> io::Result<Self> {
        let p = c_path(path.as_ref())?;
        let mut t = std::ptr::null_mut();
        // SAFETY: valid path and out-pointer.
        if unsafe { ffi::ae_tokenizer_create_from_file(p.as_ptr(), &mut t) } != ffi::AE_OK {
            return Err(tokenizer_error());
        }
        Ok(Self(t))
    }

    pub fn from_vocab_str(vocab: &str) -> io::Result<Self> {
        let mut t = std::ptr::null_mut();
        // SAFETY: the text is passed with its length (no NUL needed).
        if unsafe { ffi::ae_tokenizer_create_from_vocab(vocab.as_ptr().cast(), vocab.len(), &mut t) } != ffi::AE_OK {
            return Err(tokenizer_error());
        }
        Ok(Self(t))
    }

    pub fn vocab_size(&self) -> usize {
        // SAFETY: valid tokenizer.
        unsafe { ffi::ae_tokenizer_vocab_size(self.0) as usize }
    }

    /// `encode_into` (src/tokenizer.rs:90-101): [CLS] (+ query prefix) + WordPiece ids + [SEP],
    /// at most 512 ids.
    pub fn encode_into(&self, text: &str, is_query: bool, ids: &mut Vec<u16>) {
        ids.clear();
        ids.resize(MAX_POSITIONS, 0);
        let mut n = 0u32;
        // SAFETY: `ids` has room for 512 ids; text is passed with its length.
        let code = unsafe {
            ffi::ae_tokenize(self.0, text.as_ptr().cast(), text.len(), is_query as c_int, ids.as_mut_ptr(),
                             MAX_POSITIONS as u32, &mut n)
        };
        assert_eq!(code, ffi::AE_OK, "tokenizer failed with code {code}");
        ids.truncate(n as usize);
    }

    pub fn encode(&self, text: &str) -> Vec<u16> {
        let mut v = Vec::new();
        self.encode_into(text, false, &mut v);
        v
    }

    pub fn encode_query(&self, query: &str) -> Vec<u16> {
        let mut v = Vec::new();
        self.encode_into(query, true, &mut v);
        v
    }

    /// The tokenization step of `embed_batch` on the library's host threads: packed ids and
    /// cu_seqlens.
    pub fn encode_batch<S: AsRef<str>>(&self, texts: &[S], is_query: bool) -> (Vec<u16>, Vec<u32>) {
        let ptrs: Vec<*const std::ffi::c_char> = texts.iter().map(|t| t.as_ref().as_ptr().cast()).collect();
        let lens: Vec<usize> = texts.iter().map(|t| t.as_ref().len()).collect();
        let cap = texts.len() * MAX_POSITIONS;
        let mut ids = vec![0u16; cap];
        let mut cu = vec![0u32; texts.len() + 1];
        // SAFETY: ids has room for 512 ids per text; cu for n + 1 offsets.
        let code = unsafe {
            ffi::ae_tokenize_batch(self.0, ptrs.as_ptr(), lens.as_ptr(), texts.len() as u32, is_query as c_int,
                                   ids.as_mut_ptr(), cap, cu.as_mut_ptr())
        };
        assert_eq!(code, ffi::AE_OK, "tokenizer failed with code {code}");
        ids.truncate(*cu.last().unwrap_or(&0) as usize);
        (ids, cu)
    }
}

impl Drop for BertTokenizer {
    fn drop(&mut self) {
        // SAFETY: created by ae_tokenizer_create_*, destroyed once.
        unsafe { ffi::ae_tokenizer_destroy(self.0) };
    }
}

/// Per-caller reusable buffers (src/model.rs:123-179). The device workspace is owned by the GPU
/// context; this keeps the token-id buffer the embed calls reuse.
#[derive(Default)]
pub struct Workspace {
    pub token_ids: Vec<u16>,
}

impl Workspace {
    pub fn new() -> Self {
        Self { token_ids: Vec::with_capacity(MAX_POSITIONS) }
    }
}

/// Latency mode (src/parallel.rs:137-254): one sequence on all SMs of one GPU. The reference splits
/// a sequence over CPU threads; on the GPU every kernel is already parallel, so `n_threads` is
/// recorded (for `num_threads`) and does not change the computation.
pub struct ParallelContext {
    n: usize,
}

impl ParallelContext {
    pub fn new(n_threads: usize) -> Self {
        Self { n: n_threads.clamp(1, 8) }
    }

    pub fn recommended(_engine: &ArcticEmbedS) -> Self {
        Self::new(1)
    }

    pub fn num_threads(&self) -> usize {
        self.n
    }

    /// Embeds `input_ids` (truncated to 512) into `out_emb`.
    pub fn forward_cls(&mut self, model: &GpuModel, input_ids: &[u16], out_emb: &mut [f32; HIDDEN_SIZE]) {
        assert!(!input_ids.is_empty(), "input_ids must not be empty");
        model.forward_cls(input_ids, out_emb).unwrap_or_else(|e| panic!("forward_cls: {e}"));
    }
}

/// The embedding engine (src/lib.rs:34-260).
pub struct ArcticEmbedS {
    pub tokenizer: BertTokenizer,
    pub model: GpuModel,
    pub raw_size_bytes: usize,
}

impl ArcticEmbedS {
    /// Loads `vocab.txt` and `model.ae8` from `dir` onto GPU 0.
    pub fn from_dir<P: AsRef<Path>>(dir: P) -> io::Result<Self> {
        Self::from_dir_on_devices(dir, &[0])
    }

    /// Loads the model onto each of `devices` (one context per GPU); `embed_batch` shards over them.
    pub fn from_dir_on_devices<P: AsRef<Path>>(dir: P, devices: &[i32]) -> io::Result<Self> {
        let dir = dir.as_ref();
        let tokenizer = BertTokenizer::from_vocab_file(dir.join(VOCAB_FILE))?;
        let pack = dir.join(MODEL_FILE);
        let raw_size_bytes = std::fs::metadata(&pack)?.len() as usize;
        let model = GpuModel::load_ae8(&pack, devices)?;
        Ok(Self { tokenizer, model, raw_size_bytes })
    }

    /// `[CLS] + text + [SEP]`, embedded with the reusable `Workspace`.
    pub fn embed_document(&self, text: &str, ws: &mut Workspace) -> [f32; HIDDEN_SIZE] {
        let mut ids = std::mem::take(&mut ws.token_ids);
        self.tokenizer.encode_into(text, false, &mut ids);
        let out = self.embed_tokens(&ids, ws);
        ws.token_ids = ids;
        out
    }

    /// `[CLS] + QUERY_PREFIX + query + [SEP]`.
    pub fn embed_query(&self, query: &str, ws: &mut Workspace) -> [f32; HIDDEN_SIZE] {
        let mut ids = std::mem::take(&mut ws.token_ids);
        self.tokenizer.encode_into(query, true, &mut ids);
        let out = self.embed_tokens(&ids, ws);
        ws.token_ids = ids;
        out
    }

    /// Pre-tokenised `input_ids`.
    pub fn embed_tokens(&self, input_ids: &[u16], _ws: &mut Workspace) -> [f32; HIDDEN_SIZE] {
        let mut out = [0.0f32; HIDDEN_SIZE];
        self.model.forward_cls(input_ids, &mut out).unwrap_or_else(|e| panic!("embed_tokens: {e}"));
        out
    }

    pub fn embed_query_parallel(&self, query: &str, par: &mut ParallelContext) -> [f32; HIDDEN_SIZE] {
        let ids = self.tokenizer.encode_query(query);
        self.embed_tokens_parallel(&ids, par)
    }

    pub fn embed_document_parallel(&self, text: &str, par: &mut ParallelContext) -> [f32; HIDDEN_SIZE] {
        let ids = self.tokenizer.encode(text);
        self.embed_tokens_parallel(&ids, par)
    }

    pub fn embed_tokens_parallel(&self, input_ids: &[u16], par: &mut ParallelContext) -> [f32; HIDDEN_SIZE] {
        let mut out = [0.0f32; HIDDEN_SIZE];
        par.forward_cls(&self.model, input_ids, &mut out);
        out
    }

    /// src/lib.rs:138-260: texts tokenised on the library's host threads, then packed without
    /// padding and sharded over the model's GPUs; results in input order.
    pub fn embed_batch<S: AsRef<str> + Sync>(&self, texts: &[S], is_query: bool, _num_threads: usize)
        -> Vec<[f32; HIDDEN_SIZE]> {
        if texts.is_empty() {
            return Vec::new();
        }
        let (ids, cu) = self.tokenizer.encode_batch(texts, is_query);
        let mut out = vec![[0.0f32; HIDDEN_SIZE]; texts.len()];
        self.model.embed_batch_tokens(&ids, &cu, &mut out).unwrap_or_else(|e| panic!("embed_batch: {e}"));
        out
    }
}

/// Dot product of two L2-normalised embeddings, summed in order (src/lib.rs:263-271).
pub fn cosine_similarity(a: &[f32; HIDDEN_SIZE], b: &[f32; HIDDEN_SIZE]) -> f32 {
    let mut s = 0.0f32;
    for i in 0..HIDDEN_SIZE {
        s += a[i] * b[i];
    }
    s
}
