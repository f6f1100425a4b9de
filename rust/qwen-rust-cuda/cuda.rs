//! `--device cuda` for qwen-rust: the CUDA backend over libqwen_cuda.so (B200, sm_100a).
//!
//! This file is added to the qwen-rust crate as `src/cuda.rs` (see `device-cuda.patch` beside it,
//! which also adds the `cuda` cargo feature, `Device::Cuda` and the whole-token hook).
//!
//! Two paths, both behind the reference's own `Backend` trait (src/backend.rs:14-23):
//! * `forward_token` (the hook the patch adds to `Backend`, called first by `Model::forward`):
//!   the whole token on the device — embedding, every layer's attention and experts, the output
//!   norm and vocabulary projection — with the KV cache held by the engine.  `Model::forward`
//!   keeps its contract (src/model.rs:210-216): the same logits, the position advances by one,
//!   and any error resets both the engine and the model.
//! * `matvec` (the per-matvec trait method): `qc_packed_matvec`, for callers that drive the
//!   reference's own loop, e.g. its matvec tests; it uploads the matrix per call.
use crate::{
    backend::{Backend, Stats},
    gguf::Gguf,
    model::Config,
};
use anyhow::{ensure, Context, Result};
use qwen_cuda_sys::{ffi, safe};
use std::time::Instant;

pub struct CudaBackend {
    device: i32,
    /// The engine of the model being run: (Gguf id, context) it was built for, and the engine.
    engine: Option<(usize, usize, safe::Engine)>,
    stats: Stats,
}

impl CudaBackend {
    /// A backend on CUDA device `device`; the engine is built at the first token of a model.
    pub fn new(device: i32) -> Result<Self> {
        ensure!(device >= 0, "invalid CUDA device {device}");
        Ok(Self { device, engine: None, stats: Stats::default() })
    }

    fn engine_for(&mut self, model: &Gguf, config: &Config, context: usize) -> Result<&mut safe::Engine> {
        let fresh = !matches!(&self.engine, Some((id, ctx, _)) if *id == model.id && *ctx == context);
        if fresh {
            self.engine = None; // frees the previous model's device memory first
            // The tensor offsets are absolute in the mapped file; recover the mapping's start
            // from any tensor's data slice and hand the engine the whole mapped range.
            let first = model.tensors.values().next().context("GGUF has no tensors")?;
            let end = model.tensors.values().map(|t| t.offset + t.len).max().unwrap_or(0);
            let base = model.data(first).as_ptr().wrapping_sub(first.offset);
            // SAFETY: [base, base + end) lies inside the file mapping that `model` owns and keeps
            // alive for this call; the engine copies the weights and keeps no pointer into it.
            let bytes = unsafe { std::slice::from_raw_parts(base, end) };
            let tensors: Vec<safe::TensorRef<'_>> = model
                .tensors
                .values()
                .map(|t| safe::TensorRef { name: &t.name, kind: t.kind, dims: &t.dims, offset: t.offset, len: t.len })
                .collect();
            let u = |v: usize, what: &str| u32::try_from(v).with_context(|| format!("{what} exceeds u32"));
            let cfg = ffi::qc_config {
                hidden: u(config.hidden, "hidden")?,
                layers: u(config.layers, "layers")?,
                heads: u(config.heads, "heads")?,
                kvheads: u(config.kvheads, "kvheads")?,
                head_dim: u(config.head_dim, "head_dim")?,
                experts: u(config.experts, "experts")?,
                top: u(config.top, "top")?,
                intermediate: u(config.intermediate, "intermediate")?,
                vocab: u(config.vocab, "vocab")?,
                max_context: u(config.max_context, "max_context")?,
                eps: config.eps,
                theta: config.theta,
            };
            let t0 = Instant::now();
            let e = safe::Engine::from_tensors(&tensors, bytes, &cfg, u(context, "context")?, self.device)?;
            let st = e.stats()?;
            self.stats.uploaded_bytes += st.uploaded_bytes;
            eprintln!(
                "CUDA engine: device {} | {:.1} GiB weights, {:.1} GiB KV | built in {:.1} s",
                self.device,
                st.weight_bytes as f64 / (1u64 << 30) as f64,
                st.kv_bytes as f64 / (1u64 << 30) as f64,
                t0.elapsed().as_secs_f64()
            );
            self.engine = Some((model.id, context, e));
        }
        Ok(&mut self.engine.as_mut().unwrap().2)
    }
}

impl Backend for CudaBackend {
    fn matvec(&mut self, model: &Gguf, name: &str, expert: Option<usize>, x: &[f32]) -> Result<Vec<f32>> {
        // the reference's matrix() rules (backend.rs:57-75): rank 2, or rank 3 with an expert index
        let t = model.tensor(name)?;
        ensure!(t.dims.len() == if expert.is_some() { 3 } else { 2 }, "matrix rank mismatch: {name}");
        let (cols, rows) = (t.dims[0], t.dims[1]);
        let len = safe::row_bytes(t.kind, cols as u64)? as usize * rows;
        let e = expert.unwrap_or(0);
        ensure!(expert.is_none() || e < t.dims[2], "expert out of bounds");
        let data = &model.data(t)[e * len..(e + 1) * len];
        let t0 = Instant::now();
        let y = safe::packed_matvec(t.kind, rows, cols, data, x)?;
        self.stats.matvecs += 1;
        self.stats.uploaded_bytes += len as u64;
        self.stats.matvec_ms += t0.elapsed().as_secs_f64() * 1e3;
        Ok(y)
    }

    fn stats(&self) -> &Stats {
        &self.stats
    }

    fn forward_token(
        &mut self,
        model: &Gguf,
        config: &Config,
        context: usize,
        position: usize,
        token: u32,
    ) -> Option<Result<Vec<f32>>> {
        let per_token = ((5 + 3 * config.top) * config.layers + 1) as u64;
        Some((|| {
            let e = self.engine_for(model, config, context)?;
            if e.position()? as usize != position {
                // the model was reset without this backend (Model::reset): follow it
                ensure!(position == 0, "CUDA engine is out of step with the model");
                e.reset()?;
            }
            let t0 = Instant::now();
            let logits = e.forward(token)?;
            self.stats.matvecs += per_token;
            self.stats.matvec_ms += t0.elapsed().as_secs_f64() * 1e3;
            Ok(logits)
        })())
    }
}
