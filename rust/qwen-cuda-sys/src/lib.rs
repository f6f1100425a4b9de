//! Rust bindings of `libqwen_cuda.so`, the B200 (sm_100a) decode engine for Qwen3-MoE GGUF
//! models, declared in `include/qwen_cuda.h`.
//!
//! The reference crate (qwen-rust 0.1.0) computes every matvec through its per-matvec plugin
//! trait `Backend` (src/backend.rs:14-23), called 29 x layers + 1 times per token by
//! `Model::forward_inner` (src/model.rs:217-302).  The engine behind these bindings runs the whole
//! token on the device, so the boundary is one call per token (`qc_forward`); the per-matrix calls
//! (`qc_matrix_*`) remain for the reference's matvec interface.
//!
//! Two layers:
//! * `ffi`: the C ABI as declared in the header, `#[repr(C)]` structs field for field;
//! * `safe`: owning handles (`Engine`, `Sampler`, `Matrix`) that free themselves on drop and turn
//!   status codes into `Error` (implements `std::error::Error`, so `?` converts it into
//!   `anyhow::Error` inside qwen-rust).

#![allow(non_camel_case_types)]

pub mod ffi {
    use std::os::raw::{c_char, c_float, c_int, c_void};

    pub const QC_OK: c_int = 0;
    pub const QC_ERR_INVALID: c_int = 1;
    pub const QC_ERR_CUDA: c_int = 2;
    pub const QC_ERR_CONTEXT: c_int = 3;
    pub const QC_ERR_TOKEN: c_int = 4;
    pub const QC_ERR_NONFINITE: c_int = 5;
    pub const QC_ERR_NOMEM: c_int = 6;

    #[repr(C)]
    pub struct qc_engine {
        _opaque: [u8; 0],
    }
    #[repr(C)]
    pub struct qc_matrix {
        _opaque: [u8; 0],
    }
    #[repr(C)]
    pub struct qc_sampler {
        _opaque: [u8; 0],
    }
    #[repr(C)]
    pub struct qc_batch {
        _opaque: [u8; 0],
    }

    /// model.rs:5-19 `Config`, with fixed-width fields.
    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default, PartialEq)]
    pub struct qc_config {
        pub hidden: u32,
        pub layers: u32,
        pub heads: u32,
        pub kvheads: u32,
        pub head_dim: u32,
        pub experts: u32,
        pub top: u32,
        pub intermediate: u32,
        pub vocab: u32,
        pub max_context: u32,
        pub eps: f32,
        pub theta: f32,
    }

    /// gguf.rs:14-21 `Tensor`: dims in GGUF order (dims[0] = columns), `offset` absolute in `base`.
    #[repr(C)]
    #[derive(Clone, Copy, Debug)]
    pub struct qc_tensor_desc {
        pub name: *const c_char,
        pub kind: u32,
        pub n_dims: u32,
        pub dims: [u64; 3],
        pub offset: u64,
        pub len: u64,
    }

    /// backend.rs:7-13 `Stats` (first four fields) plus engine counters.
    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qc_stats {
        pub matvecs: u64,
        pub uploaded_bytes: u64,
        pub cache_hits: u64,
        pub matvec_ms: f64,
        pub tokens: u64,
        pub weight_bytes: u64,
        pub kv_bytes: u64,
    }

    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct qc_phase_times {
        pub embed_ms: f64,
        pub attn_in_ms: f64,
        pub attention_ms: f64,
        pub oproj_ms: f64,
        pub router_ms: f64,
        pub gateup_ms: f64,
        pub down_ms: f64,
        pub output_ms: f64,
        pub launches: u32,
        pub token_ms: f64,
    }

    extern "C" {
        pub fn qc_engine_create(
            tensors: *const qc_tensor_desc,
            n_tensors: usize,
            base: *const u8,
            base_len: usize,
            cfg: *const qc_config,
            context: u32,
            device: c_int,
            out: *mut *mut qc_engine,
        ) -> c_int;
        pub fn qc_engine_create_gguf(
            image: *const u8,
            len: usize,
            context: u32,
            device: c_int,
            out: *mut *mut qc_engine,
        ) -> c_int;
        pub fn qc_engine_create_gguf_ep(
            image: *const u8,
            len: usize,
            context: u32,
            device: c_int,
            rank: u32,
            world: u32,
            out: *mut *mut qc_engine,
        ) -> c_int;
        pub fn qc_engine_ep_handle(e: *mut qc_engine, handle: *mut c_void, device_id: *mut c_int) -> c_int;
        pub fn qc_engine_ep_connect(e: *mut qc_engine, handles: *const c_void, device_ids: *const c_int) -> c_int;
        pub fn qc_engine_open(path: *const c_char, context: u32, device: c_int, out: *mut *mut qc_engine) -> c_int;
        pub fn qc_engine_destroy(e: *mut qc_engine);
        pub fn qc_engine_error(e: *const qc_engine) -> *const c_char;
        pub fn qc_last_error() -> *const c_char;
        pub fn qc_engine_config(e: *const qc_engine, out: *mut qc_config) -> c_int;
        pub fn qc_engine_set_stream(e: *mut qc_engine, stream: *mut c_void) -> c_int;

        pub fn qc_forward(e: *mut qc_engine, token: u32, logits: *mut c_float) -> c_int;
        pub fn qc_forward_tokens(e: *mut qc_engine, tokens: *const u32, n: usize, logits: *mut c_float) -> c_int;
        pub fn qc_decode_greedy(e: *mut qc_engine, n: u32, tokens_out: *mut u32, logits: *mut c_float) -> c_int;
        pub fn qc_decode_enqueue(e: *mut qc_engine, n: u32) -> c_int;
        pub fn qc_moe_layer(
            e: *mut qc_engine,
            layer: u32,
            x: *const c_float,
            n_tokens: u32,
            out: *mut c_float,
            path: c_int,
            device_ms: *mut c_float,
        ) -> c_int;

        pub fn qc_sampler_create(
            seed: u64,
            temperature: c_float,
            top_k: u32,
            top_p: c_float,
            device: c_int,
            out: *mut *mut qc_sampler,
        ) -> c_int;
        pub fn qc_sampler_destroy(s: *mut qc_sampler);
        pub fn qc_sampler_sample(
            s: *mut qc_sampler,
            device_logits: *const c_float,
            n: u32,
            stream: *mut c_void,
            token: *mut u32,
        ) -> c_int;
        pub fn qc_sampler_words(s: *mut qc_sampler, n: u32, out: *mut u32) -> c_int;
        pub fn qc_engine_sample(e: *mut qc_engine, s: *mut qc_sampler, token: *mut u32) -> c_int;
        pub fn qc_decode_sample(
            e: *mut qc_engine,
            s: *mut qc_sampler,
            n: u32,
            tokens_out: *mut u32,
            logits: *mut c_float,
        ) -> c_int;
        pub fn qc_sync(e: *mut qc_engine) -> c_int;

        pub fn qc_batch_create(e: *mut qc_engine, n_seqs: u32, context: u32, out: *mut *mut qc_batch) -> c_int;
        pub fn qc_batch_destroy(b: *mut qc_batch);
        pub fn qc_batch_forward(
            b: *mut qc_batch,
            seq_ids: *const u32,
            tokens: *const u32,
            n: u32,
            logits: *mut c_float,
        ) -> c_int;
        pub fn qc_batch_reset(b: *mut qc_batch, seq: u32) -> c_int;
        pub fn qc_batch_position(b: *const qc_batch, seq: u32, pos: *mut u32) -> c_int;
        pub fn qc_batch_logits_device(b: *const qc_batch, seq: u32, out: *mut *const c_float) -> c_int;
        pub fn qc_batch_sample(
            b: *mut qc_batch,
            samplers: *const *mut qc_sampler,
            seq_ids: *const u32,
            n: u32,
            tokens_out: *mut u32,
        ) -> c_int;
        pub fn qc_batch_decode_sample(
            b: *mut qc_batch,
            samplers: *const *mut qc_sampler,
            seq_ids: *const u32,
            n: u32,
            steps: u32,
            tokens_out: *mut u32,
        ) -> c_int;
        pub fn qc_batch_stats(b: *const qc_batch, out: *mut qc_stats) -> c_int;
        pub fn qc_batch_ep_handle(b: *mut qc_batch, handle: *mut c_void, device_id: *mut c_int) -> c_int;
        pub fn qc_batch_ep_connect(b: *mut qc_batch, handles: *const c_void, device_ids: *const c_int) -> c_int;

        pub fn qc_reset(e: *mut qc_engine) -> c_int;
        pub fn qc_position(e: *const qc_engine, pos: *mut u32) -> c_int;
        pub fn qc_get_stats(e: *const qc_engine, out: *mut qc_stats) -> c_int;
        pub fn qc_profile_step(e: *mut qc_engine, out: *mut qc_phase_times) -> c_int;
        pub fn qc_engine_set_decode_mode(e: *mut qc_engine, mode: c_int) -> c_int;
        pub fn qc_engine_decode_path(e: *const qc_engine, path: *mut c_int, why: *mut *const c_char) -> c_int;
        pub fn qc_logits_device(e: *const qc_engine, out: *mut *const c_float) -> c_int;

        pub fn qc_row_bytes(kind: u32, cols: u64, out: *mut u64) -> c_int;
        pub fn qc_matrix_create(
            kind: u32,
            rows: u64,
            cols: u64,
            experts: u64,
            blocks: *const u8,
            len: u64,
            device: c_int,
            out: *mut *mut qc_matrix,
        ) -> c_int;
        pub fn qc_matrix_matvec(
            m: *const qc_matrix,
            expert: u32,
            x: *const c_float,
            y: *mut c_float,
            stream: *mut c_void,
        ) -> c_int;
        pub fn qc_matrix_dequant(m: *const qc_matrix, expert: u32, out: *mut c_float, stream: *mut c_void) -> c_int;
        pub fn qc_matrix_bytes(m: *const qc_matrix, device_bytes: *mut u64, packed_bytes: *mut u64) -> c_int;
        pub fn qc_matrix_destroy(m: *mut qc_matrix);
        pub fn qc_packed_matvec(
            kind: u32,
            rows: u64,
            cols: u64,
            blocks: *const u8,
            len: u64,
            x: *const c_float,
            y: *mut c_float,
        ) -> c_int;
        pub fn qc_packed_matvec_noalloc(
            kind: u32,
            rows: u64,
            cols: u64,
            blocks: *const u8,
            len: u64,
            x: *const c_float,
            y: *mut c_float,
        ) -> c_int;
    }
}

pub mod safe {
    //! Owning wrappers.  Each engine belongs to one thread at a time (`Send`, not `Sync`), as the
    //! reference's `&mut self` backend does.
    use super::ffi;
    use std::ffi::{CStr, CString};
    use std::fmt;
    use std::os::raw::{c_char, c_int};
    use std::ptr;

    /// A failed call: the status code (ffi::QC_ERR_*) and the engine's message.
    #[derive(Debug, Clone)]
    pub struct Error {
        pub code: i32,
        pub message: String,
    }
    impl fmt::Display for Error {
        fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
            write!(f, "{} (qwen_cuda status {})", self.message, self.code)
        }
    }
    impl std::error::Error for Error {}
    pub type Result<T> = std::result::Result<T, Error>;

    fn text(p: *const c_char) -> String {
        if p.is_null() {
            String::new()
        } else {
            unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
        }
    }
    fn global(rc: c_int) -> Result<()> {
        if rc == ffi::QC_OK {
            Ok(())
        } else {
            Err(Error { code: rc, message: text(unsafe { ffi::qc_last_error() }) })
        }
    }

    /// Bytes of one GGUF row (quant.rs:12-21).
    pub fn row_bytes(kind: u32, cols: u64) -> Result<u64> {
        let mut out = 0u64;
        global(unsafe { ffi::qc_row_bytes(kind, cols, &mut out) })?;
        Ok(out)
    }

    /// One tensor of a parsed GGUF (the reference's `gguf::Tensor`), offset absolute in `base`.
    pub struct TensorRef<'a> {
        pub name: &'a str,
        pub kind: u32,
        pub dims: &'a [usize],
        pub offset: usize,
        pub len: usize,
    }

    pub struct Engine {
        h: *mut ffi::qc_engine,
        pub config: ffi::qc_config,
    }
    unsafe impl Send for Engine {}

    impl Engine {
        fn wrap(h: *mut ffi::qc_engine) -> Result<Self> {
            let mut config = ffi::qc_config::default();
            let mut e = Engine { h, config };
            e.check(unsafe { ffi::qc_engine_config(h, &mut config) })?;
            e.config = config;
            Ok(e)
        }
        fn check(&self, rc: c_int) -> Result<()> {
            if rc == ffi::QC_OK {
                Ok(())
            } else {
                Err(Error { code: rc, message: text(unsafe { ffi::qc_engine_error(self.h) }) })
            }
        }

        /// `Model::new` (model.rs:173-201) from the caller's parsed tensor table over its mapped
        /// file; the engine copies the weights to device `device` and never reads `base` again.
        pub fn from_tensors(
            tensors: &[TensorRef<'_>],
            base: &[u8],
            config: &ffi::qc_config,
            context: u32,
            device: i32,
        ) -> Result<Self> {
            let names: Vec<CString> = tensors
                .iter()
                .map(|t| CString::new(t.name).map_err(|_| Error { code: ffi::QC_ERR_INVALID, message: "tensor name".into() }))
                .collect::<Result<_>>()?;
            let mut descs = Vec::with_capacity(tensors.len());
            for (t, n) in tensors.iter().zip(&names) {
                if t.dims.len() > 3 {
                    return Err(Error { code: ffi::QC_ERR_INVALID, message: format!("tensor {} has rank > 3", t.name) });
                }
                let mut dims = [0u64; 3];
                for (d, &v) in dims.iter_mut().zip(t.dims) {
                    *d = v as u64;
                }
                descs.push(ffi::qc_tensor_desc {
                    name: n.as_ptr(),
                    kind: t.kind,
                    n_dims: t.dims.len() as u32,
                    dims,
                    offset: t.offset as u64,
                    len: t.len as u64,
                });
            }
            let mut h = ptr::null_mut();
            global(unsafe {
                ffi::qc_engine_create(descs.as_ptr(), descs.len(), base.as_ptr(), base.len(), config, context, device, &mut h)
            })?;
            Engine::wrap(h)
        }

        /// Parse a GGUF image in memory (gguf.rs:102-195) and build the engine.
        pub fn from_gguf(image: &[u8], context: u32, device: i32) -> Result<Self> {
            let mut h = ptr::null_mut();
            global(unsafe { ffi::qc_engine_create_gguf(image.as_ptr(), image.len(), context, device, &mut h) })?;
            Engine::wrap(h)
        }

        /// Map a GGUF file and build the engine.
        pub fn open(path: &str, context: u32, device: i32) -> Result<Self> {
            let p = CString::new(path).map_err(|_| Error { code: ffi::QC_ERR_INVALID, message: "path".into() })?;
            let mut h = ptr::null_mut();
            global(unsafe { ffi::qc_engine_open(p.as_ptr(), context, device, &mut h) })?;
            Engine::wrap(h)
        }

        /// `Model::forward` (model.rs:210-216): the logits of `token` at the current position.
        /// On error the engine has reset its KV cache and position, as the reference does.
        pub fn forward(&mut self, token: u32) -> Result<Vec<f32>> {
            let mut logits = vec![0f32; self.config.vocab as usize];
            self.check(unsafe { ffi::qc_forward(self.h, token, logits.as_mut_ptr()) })?;
            Ok(logits)
        }
        /// Forwards of every token; the logits of the last one (the `logits` command's loop).
        pub fn forward_tokens(&mut self, tokens: &[u32]) -> Result<Vec<f32>> {
            let mut logits = vec![0f32; self.config.vocab as usize];
            self.check(unsafe { ffi::qc_forward_tokens(self.h, tokens.as_ptr(), tokens.len(), logits.as_mut_ptr()) })?;
            Ok(logits)
        }
        /// Greedy decode of n tokens on the device (the chat loop at temperature 0).
        pub fn decode_greedy(&mut self, n: u32) -> Result<Vec<u32>> {
            let mut out = vec![0u32; n as usize];
            self.check(unsafe { ffi::qc_decode_greedy(self.h, n, out.as_mut_ptr(), ptr::null_mut()) })?;
            Ok(out)
        }
        /// The chat loop with sampling on the device: n (sample, step) pairs.
        pub fn decode_sample(&mut self, sampler: &mut Sampler, n: u32) -> Result<Vec<u32>> {
            let mut out = vec![0u32; n as usize];
            self.check(unsafe { ffi::qc_decode_sample(self.h, sampler.h, n, out.as_mut_ptr(), ptr::null_mut()) })?;
            Ok(out)
        }
        /// `Sampler::sample` on the last step's logits, on the device.
        pub fn sample(&mut self, sampler: &mut Sampler) -> Result<u32> {
            let mut t = 0u32;
            self.check(unsafe { ffi::qc_engine_sample(self.h, sampler.h, &mut t) })?;
            Ok(t)
        }
        /// `Model::reset` (model.rs:202-208).
        pub fn reset(&mut self) -> Result<()> {
            self.check(unsafe { ffi::qc_reset(self.h) })
        }
        pub fn position(&self) -> Result<u32> {
            let mut p = 0u32;
            self.check(unsafe { ffi::qc_position(self.h, &mut p) })?;
            Ok(p)
        }
        pub fn stats(&self) -> Result<ffi::qc_stats> {
            let mut s = ffi::qc_stats::default();
            self.check(unsafe { ffi::qc_get_stats(self.h, &mut s) })?;
            Ok(s)
        }
        pub fn raw(&self) -> *mut ffi::qc_engine {
            self.h
        }

        /// Expert parallelism: this rank's share (experts [rank E / world, (rank + 1) E / world)) of
        /// the model in `image`, one process and GPU per rank.  Usable after `ep_connect`.
        pub fn expert_parallel(image: &[u8], context: u32, device: i32, rank: u32, world: u32) -> Result<Self> {
            let mut h = ptr::null_mut();
            global(unsafe {
                ffi::qc_engine_create_gguf_ep(image.as_ptr(), image.len(), context, device, rank, world, &mut h)
            })?;
            Engine::wrap(h)
        }
        /// This rank's exchange-buffer handle and GPU id, to be given to every rank.
        pub fn ep_handle(&self) -> Result<([u8; 64], i32)> {
            let mut h = [0u8; 64];
            let mut dev: c_int = 0;
            self.check(unsafe { ffi::qc_engine_ep_handle(self.h, h.as_mut_ptr().cast(), &mut dev) })?;
            Ok((h, dev))
        }
        /// Every rank's `ep_handle()`, in rank order.
        pub fn ep_connect(&mut self, handles: &[([u8; 64], i32)]) -> Result<()> {
            let (flat, ids) = flatten_handles(handles);
            self.check(unsafe { ffi::qc_engine_ep_connect(self.h, flat.as_ptr().cast(), ids.as_ptr()) })
        }
    }
    /// (handles: n x 64 bytes, device ids: n) of a list of (handle, id) pairs.
    fn flatten_handles(handles: &[([u8; 64], i32)]) -> (Vec<u8>, Vec<c_int>) {
        let flat = handles.iter().flat_map(|(h, _)| h.iter().copied()).collect();
        let ids = handles.iter().map(|(_, d)| *d as c_int).collect();
        (flat, ids)
    }
    impl Drop for Engine {
        fn drop(&mut self) {
            unsafe { ffi::qc_engine_destroy(self.h) }
        }
    }

    /// `Sampler::new(seed, temperature, top_k, top_p)` (sampling.rs:9-25) living on `device`.
    pub struct Sampler {
        h: *mut ffi::qc_sampler,
    }
    unsafe impl Send for Sampler {}
    impl Sampler {
        pub fn new(seed: u64, temperature: f32, top_k: u32, top_p: f32, device: i32) -> Result<Self> {
            let mut h = ptr::null_mut();
            global(unsafe { ffi::qc_sampler_create(seed, temperature, top_k, top_p, device, &mut h) })?;
            Ok(Sampler { h })
        }
    }
    impl Drop for Sampler {
        fn drop(&mut self) {
            unsafe { ffi::qc_sampler_destroy(self.h) }
        }
    }

    /// Several sequences on one engine (`qc_batch_*`): per-sequence KV caches and positions, any mix
    /// of their tokens per step.  Borrows the engine, which must outlive it.
    pub struct Batch<'e> {
        h: *mut ffi::qc_batch,
        engine: &'e mut Engine,
    }
    impl<'e> Batch<'e> {
        pub fn new(engine: &'e mut Engine, n_seqs: u32, context: u32) -> Result<Self> {
            let mut h = ptr::null_mut();
            engine.check(unsafe { ffi::qc_batch_create(engine.h, n_seqs, context, &mut h) })?;
            Ok(Batch { h, engine })
        }
        /// One step: token i to sequence seq_ids[i]; one logits row per sequence of the call (its
        /// last token), in call order.
        pub fn forward(&mut self, seq_ids: &[u32], tokens: &[u32]) -> Result<Vec<Vec<f32>>> {
            if seq_ids.len() != tokens.len() {
                return Err(Error { code: ffi::QC_ERR_INVALID, message: "seq_ids and tokens differ in length".into() });
            }
            let mut seen = std::collections::HashSet::new();
            let rows = seq_ids.iter().rev().filter(|s| seen.insert(**s)).count();
            let v = self.engine.config.vocab as usize;
            let mut flat = vec![0f32; rows * v];
            self.engine.check(unsafe {
                ffi::qc_batch_forward(self.h, seq_ids.as_ptr(), tokens.as_ptr(), seq_ids.len() as u32, flat.as_mut_ptr())
            })?;
            Ok(flat.chunks(v).map(|c| c.to_vec()).collect())
        }
        /// The chat loop for distinct sequences: `steps` x n sampled ids, step-major.
        pub fn decode_sample(&mut self, samplers: &mut [&mut Sampler], seq_ids: &[u32], steps: u32) -> Result<Vec<u32>> {
            let sp: Vec<*mut ffi::qc_sampler> = samplers.iter_mut().map(|s| s.h).collect();
            let mut out = vec![0u32; steps as usize * seq_ids.len()];
            self.engine.check(unsafe {
                ffi::qc_batch_decode_sample(self.h, sp.as_ptr(), seq_ids.as_ptr(), seq_ids.len() as u32, steps, out.as_mut_ptr())
            })?;
            Ok(out)
        }
        pub fn reset(&mut self, seq: u32) -> Result<()> {
            self.engine.check(unsafe { ffi::qc_batch_reset(self.h, seq) })
        }
        /// Batches of an expert-parallel engine: this rank's exchange-region handle and GPU id.
        pub fn ep_handle(&self) -> Result<([u8; 64], i32)> {
            let mut h = [0u8; 64];
            let mut dev: c_int = 0;
            self.engine.check(unsafe { ffi::qc_batch_ep_handle(self.h, h.as_mut_ptr().cast(), &mut dev) })?;
            Ok((h, dev))
        }
        /// Every rank's batch `ep_handle()`, in rank order; then every rank makes the same calls
        /// with the same token counts.
        pub fn ep_connect(&mut self, handles: &[([u8; 64], i32)]) -> Result<()> {
            let (flat, ids) = flatten_handles(handles);
            self.engine.check(unsafe { ffi::qc_batch_ep_connect(self.h, flat.as_ptr().cast(), ids.as_ptr()) })
        }
    }
    impl Drop for Batch<'_> {
        fn drop(&mut self) {
            unsafe { ffi::qc_batch_destroy(self.h) }
        }
    }

    /// `experts` stacked (rows x cols) GGUF matrices resident on the device, for the reference's
    /// per-matvec `Backend::matvec` (backend.rs:14-23).
    pub struct Matrix {
        h: *mut ffi::qc_matrix,
        pub rows: usize,
        pub cols: usize,
    }
    unsafe impl Send for Matrix {}
    impl Matrix {
        pub fn new(kind: u32, rows: usize, cols: usize, experts: usize, blocks: &[u8], device: i32) -> Result<Self> {
            let mut h = ptr::null_mut();
            global(unsafe {
                ffi::qc_matrix_create(kind, rows as u64, cols as u64, experts as u64, blocks.as_ptr(), blocks.len() as u64, device, &mut h)
            })?;
            Ok(Matrix { h, rows, cols })
        }
        /// y = W_expert x with device pointers on `stream` (null: the default stream).
        ///
        /// # Safety
        /// `x` and `y` must be device pointers to `cols` and `rows` floats.
        pub unsafe fn matvec_device(&self, expert: u32, x: *const f32, y: *mut f32, stream: *mut std::ffi::c_void) -> Result<()> {
            global(ffi::qc_matrix_matvec(self.h, expert, x, y, stream))
        }
    }
    impl Drop for Matrix {
        fn drop(&mut self) {
            unsafe { ffi::qc_matrix_destroy(self.h) }
        }
    }

    /// Host-to-host matvec of one packed matrix (`Vulkan::packed_matvec`, backend.rs:174-261).
    pub fn packed_matvec(kind: u32, rows: usize, cols: usize, blocks: &[u8], x: &[f32]) -> Result<Vec<f32>> {
        if x.len() != cols {
            return Err(Error { code: ffi::QC_ERR_INVALID, message: "matvec shape mismatch".into() });
        }
        let mut y = vec![0f32; rows];
        global(unsafe {
            ffi::qc_packed_matvec(kind, rows as u64, cols as u64, blocks.as_ptr(), blocks.len() as u64, x.as_ptr(), y.as_mut_ptr())
        })?;
        Ok(y)
    }
}
