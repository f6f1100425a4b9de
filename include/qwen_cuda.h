/* qwen_cuda.h — C ABI of the B200 decode engine for Qwen3-MoE GGUF models.
 *
 * Library: qwen-30brust_b200/libqwen_cuda.so (sm_100a kernels, CUDA runtime linked statically).
 *
 * This is the drop-in boundary for the reference crate K410Sh4/QWEN-30BRust
 * (qwen-rust 0.1.0).  Its plugin API is the per-matvec trait
 *     trait Backend { fn matvec(&mut self, model: &Gguf, name: &str,
 *                               expert: Option<usize>, x: &[f32]) -> Result<Vec<f32>>;
 *                     fn stats(&self) -> &Stats; }            (src/backend.rs:14-23)
 * called 29*layers+1 times per token by Model::forward_inner (src/model.rs:217-302).
 * Here the boundary moves up to the whole token: qc_forward replaces
 * Model::forward + every Backend::matvec of that token, so activations never
 * leave the device between matvecs.  The per-matvec entry points
 * (qc_matrix_*, qc_packed_matvec) remain for the reference's matvec tests
 * and microbenchmarks.
 *
 * Conventions (mirroring the Rust side):
 *   - every call returns an int status, QC_OK (0) on success;
 *   - the message of the last failure is qc_engine_error(engine) or, for calls
 *     without an engine, qc_last_error() (thread-local);
 *   - a failed qc_forward / qc_forward_tokens / qc_decode_greedy resets the KV
 *     cache and position, as Model::forward does (src/model.rs:210-216);
 *   - one engine is used by one thread at a time (the reference takes &mut self);
 *   - the caller keeps ownership of every host buffer; the engine copies the
 *     weights to the device at creation and never reads `base` afterwards.
 */
#ifndef QWEN_CUDA_H
#define QWEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  QC_OK = 0,
  QC_ERR_INVALID = 1,   /* bad argument, shape, type or metadata */
  QC_ERR_CUDA = 2,      /* a CUDA runtime call failed */
  QC_ERR_CONTEXT = 3,   /* "context limit reached" (model.rs:219-223) */
  QC_ERR_TOKEN = 4,     /* "token outside vocabulary" (model.rs:224) */
  QC_ERR_NONFINITE = 5, /* "nonfinite model output" (model.rs:296-299) or non-finite router logits (ops.rs:50-52) */
  QC_ERR_NOMEM = 6      /* device allocation failed */
};

typedef struct qc_engine qc_engine;
typedef struct qc_matrix qc_matrix;
typedef struct qc_sampler qc_sampler;
typedef struct qc_batch qc_batch;

/* Model hyper-parameters; same fields and meaning as model.rs:5-19 Config. */
typedef struct qc_config {
  uint32_t hidden, layers, heads, kvheads, head_dim, experts, top, intermediate, vocab, max_context;
  float eps, theta;
} qc_config;

/* One GGUF tensor; same fields as gguf.rs:14-21 Tensor.  dims are in GGUF order
 * (dims[0] = columns).  `offset` is the absolute byte offset of the tensor data
 * in the caller's buffer (gguf.rs:175-178 after adding the data start). */
typedef struct qc_tensor_desc {
  const char* name;
  uint32_t kind;
  uint32_t n_dims;
  uint64_t dims[3];
  uint64_t offset;
  uint64_t len;
} qc_tensor_desc;

/* Counters; the first four fields are backend.rs:7-13 Stats. */
typedef struct qc_stats {
  uint64_t matvecs;        /* matvecs the reference would have issued: (5+3*top)*layers+1 per token */
  uint64_t uploaded_bytes; /* host->device weight bytes (at creation only) */
  uint64_t cache_hits;     /* always 0: every weight stays resident, there is no cache */
  double matvec_ms;        /* device time of the forward steps run so far (CUDA events) */
  uint64_t tokens;         /* forward steps run */
  uint64_t weight_bytes;   /* device bytes holding weights */
  uint64_t kv_bytes;       /* device bytes of the fp32 KV cache */
} qc_stats;

/* ---- engine life cycle ------------------------------------------------- */

/* Build an engine from an already parsed GGUF: the tensor table and the mapped
 * file (replaces Model::new, model.rs:173-201, plus the reference's weight
 * upload in Vulkan::packed_matvec, backend.rs:174-261).  Validates the config
 * and tensor shapes like Config::from_gguf/validate_tensors (model.rs:58-149)
 * and context in 1..=max_context (model.rs:176-180). */
int qc_engine_create(const qc_tensor_desc* tensors, size_t n_tensors, const uint8_t* base, size_t base_len,
                     const qc_config* cfg, uint32_t context, int device, qc_engine** out);

/* Parse a GGUF image held in memory (gguf.rs:102-195, model.rs:21-90) and build the engine. */
int qc_engine_create_gguf(const uint8_t* image, size_t len, uint32_t context, int device, qc_engine** out);

/* Expert parallelism (no counterpart in the reference): as qc_engine_create_gguf, but this engine
 * holds only experts [rank*E/world, (rank+1)*E/world) of the `world` ranks (world <= 8, one process
 * and one GPU per rank) and replicates everything else.  Every rank computes the router and the
 * top-k itself, runs the selected experts it holds, and adds its partial MoE vector straight into
 * the other ranks' exchange buffers over NVLink (8-byte tagged values, system scope), so one token
 * is one launch on every rank with no separate collective.  Before the first forward each rank
 * exports a handle with qc_engine_ep_handle, the host gathers all `world` handles and device ids
 * (rank order) and passes them to qc_engine_ep_connect on every rank.  All ranks must then run the
 * same forward / decode calls in the same order.  If one rank stops, the others' next step ends
 * with QC_ERR_CUDA ("a wait between thread blocks timed out", after 2 s) and resets them; after
 * any error the ranks' token tags no longer agree, so every rank must be destroyed and created
 * again.  Ranks on the same GPU are refused. */
int qc_engine_create_gguf_ep(const uint8_t* image, size_t len, uint32_t context, int device, uint32_t rank,
                             uint32_t world, qc_engine** out);
/* 64-byte CUDA IPC handle of this rank's exchange buffer and an id of its GPU (PCI location). */
int qc_engine_ep_handle(qc_engine* e, void* handle, int* device_id);
/* handles: world x 64 bytes, device_ids: world ints, both in rank order. */
int qc_engine_ep_connect(qc_engine* e, const void* handles, const int* device_ids);

/* Map a GGUF file read-only and build the engine (Gguf::open + Model::new). */
int qc_engine_open(const char* path, uint32_t context, int device, qc_engine** out);

void qc_engine_destroy(qc_engine* e);
const char* qc_engine_error(const qc_engine* e);
const char* qc_last_error(void);
int qc_engine_config(const qc_engine* e, qc_config* out);

/* Run subsequent work on the caller's CUDA stream (a cudaStream_t; NULL = the engine's own stream). */
int qc_engine_set_stream(qc_engine* e, void* stream);

/* ---- decode ------------------------------------------------------------ */

/* One causal single-token forward at the current position: Model::forward
 * (model.rs:210-216).  Writes `vocab` logits to `logits` (host memory; may be
 * NULL to keep them on the device).  On error the cache and position are reset. */
int qc_forward(qc_engine* e, uint32_t token, float* logits);

/* Sequential forwards of n tokens (the `logits` command's loop, main.rs:144-146);
 * the logits of the last token go to `logits` (may be NULL). */
int qc_forward_tokens(qc_engine* e, const uint32_t* tokens, size_t n, float* logits);

/* Greedy decode of n tokens entirely on the device.  Step i feeds the argmax
 * (ties to the lower id, sampling.rs:31-35) of the previous logits and records
 * it in tokens_out[i] (host, may be NULL); requires a previous forward.  The
 * last step's logits go to `logits` (may be NULL).  Fails before running when
 * position + n exceeds the context (main.rs:219-227). */
int qc_decode_greedy(qc_engine* e, uint32_t n, uint32_t* tokens_out, float* logits);

/* As qc_decode_greedy, but only enqueues the n steps on the engine's stream and
 * returns; qc_sync waits and reports a non-finite output or a bad token. */
int qc_decode_enqueue(qc_engine* e, uint32_t n);

/* The MoE half of layer `layer` (model.rs:245-287: RMSNorm(ffn_norm), router, top-k, expert
 * SwiGLU, weighted combine, residual) for n_tokens independent token vectors at once.
 * x, out: n_tokens x hidden floats in host memory.  path 1 runs the per-token decode kernels
 * once per token (matvecs); path 2 the batched kernels: tokens grouped per expert, gate/up and
 * down as tcgen05 tensor-core GEMMs (gate/up and down in Q4_K or Q6_K; other formats are refused
 * on this path).  The first path-2 call makes the engine's GEMM-layout copy of the Q4_K/Q6_K
 * weights (about their size again in device memory).  device_ms (may be NULL) receives the device
 * time of the layer, copies excluded.  The KV cache and position are not touched.  Not available on
 * expert-parallel engines. */
int qc_moe_layer(qc_engine* e, uint32_t layer, const float* x, uint32_t n_tokens, float* out, int path,
                 float* device_ms);

/* ---- Sampler (sampling.rs:3-65) on the device ---------------------------------------------------
 * qc_sampler_create ~ Sampler::new(seed, temperature, top_k, top_p): "invalid sampling parameters"
 * unless temperature is finite and >= 0 and 0 < top_p <= 1; top_k 0 = off.  The random source is
 * rand 0.8's StdRng (ChaCha12 keyed by seed_from_u64), one keystream word per non-greedy draw.
 * The sampler lives on `device` and is used with engines on that device. */
int qc_sampler_create(uint64_t seed, float temperature, uint32_t top_k, float top_p, int device, qc_sampler** out);
void qc_sampler_destroy(qc_sampler* s);
/* Sampler::sample on n logits in DEVICE memory (stream: a cudaStream_t or NULL for the sampler's
 * own); "invalid logits" (QC_ERR_INVALID) when empty or not all finite.  Errors: qc_last_error(). */
int qc_sampler_sample(qc_sampler* s, const float* device_logits, uint32_t n, void* stream, uint32_t* token);
/* The next n keystream words of the sampler's StdRng (advances it): reproducibility checks. */
int qc_sampler_words(qc_sampler* s, uint32_t n, uint32_t* out);
/* Sampler::sample on the logits of the engine's last step (no step is run). */
int qc_engine_sample(qc_engine* e, qc_sampler* s, uint32_t* token);
/* The chat loop with sampling (main.rs:261-282) on the device: n times, sample the current
 * logits and feed the id to the next step.  tokens_out (n ids) and logits (of the last step) may
 * be NULL.  Argument errors leave the engine as it was; a failed step resets it. */
int qc_decode_sample(qc_engine* e, qc_sampler* s, uint32_t n, uint32_t* tokens_out, float* logits);
int qc_sync(qc_engine* e);

/* ---- several sequences per step (no counterpart in the reference) --------------------------------
 * The reference decodes one sequence, one token per Model::forward (model.rs:210-216).  A batch keeps
 * n_seqs independent sequences (KV cache and position each, `context` positions at most, <= the
 * engine's context) beside an engine's weights, and runs any mix of their tokens as one step: a
 * decode step (one token of each of many sequences) and a prompt chunk (consecutive tokens of one
 * sequence, each attending to the ones before it) are the same call.  The dense matrices read each
 * weight once per step for all its tokens (tcgen05 tensor-core GEMMs for Q4_K/Q6_K matrices, a
 * CUDA-core batched matvec for other formats); the MoE half groups the step's tokens per expert and
 * runs gate/up and down as tensor-core GEMMs (Q4_K or Q6_K experts; other formats run the per-token
 * kernels).  Creating a batch makes the engine's GEMM-layout copy of the Q4_K/Q6_K weights (about
 * their size again in device memory) if it does not exist yet.  Logits agree with Model::forward on each sequence within the decode path's
 * tolerance.  Error messages: qc_engine_error(engine).  Argument errors (unknown sequence, token
 * outside the vocabulary, a sequence past its context) change nothing; a call that fails on the
 * device (non-finite output) resets the sequences it carried.  The engine's own decode state is not
 * touched, and the engine must outlive the batch. */
int qc_batch_create(qc_engine* e, uint32_t n_seqs, uint32_t context, qc_batch** out);
void qc_batch_destroy(qc_batch* b);
/* Token i goes to sequence seq_ids[i] at that sequence's next position (a sequence may appear several
 * times: its tokens take consecutive positions in call order).  logits (host, may be NULL) receives
 * one row of vocab floats per sequence of the call, for the last of its tokens, in call order; the
 * latest row of every sequence also stays on the device (qc_batch_logits_device) for sampling. */
int qc_batch_forward(qc_batch* b, const uint32_t* seq_ids, const uint32_t* tokens, uint32_t n, float* logits);
/* Model::reset for one sequence, or for all with seq = 0xffffffff. */
int qc_batch_reset(qc_batch* b, uint32_t seq);
int qc_batch_position(const qc_batch* b, uint32_t seq, uint32_t* pos);
int qc_batch_logits_device(const qc_batch* b, uint32_t seq, const float** out);
/* Sampler::sample (sampling.rs:26-65) of samplers[i] on the latest logits of sequence seq_ids[i],
 * all n draws in one launch; ids to tokens_out (host).  The samplers live on the engine's device. */
int qc_batch_sample(qc_batch* b, qc_sampler* const* samplers, const uint32_t* seq_ids, uint32_t n, uint32_t* tokens_out);
/* The chat loop (main.rs:261-282) for n distinct sequences at once, on the device: `steps` times,
 * sample every sequence's latest logits with its sampler and run the n ids as one step.
 * tokens_out (host, may be NULL): steps x n ids, step-major. */
int qc_batch_decode_sample(qc_batch* b, qc_sampler* const* samplers, const uint32_t* seq_ids, uint32_t n, uint32_t steps,
                           uint32_t* tokens_out);
/* Tokens run, device time of the steps (matvec_ms), KV and weight bytes. */
int qc_batch_stats(const qc_batch* b, qc_stats* out);
/* Expert parallelism of a batch (BASELINE config 5 over 2-8 GPUs: dispatch and combine of the MoE
 * half; no counterpart in the reference, which runs one sequence on one device): a batch of an expert-parallel engine (qc_engine_create_gguf_ep)
 * holds this rank's own sequences (attention, dense rows and vocabulary run data-parallel) and, per
 * layer, exchanges the MoE half with the other ranks through their exchange regions over NVLink:
 * every rank publishes its tokens' normalized inputs and router selections, each rank runs its
 * experts' GEMMs over the pairs of all ranks' tokens routed to them, and each token's home rank sums
 * its experts' outputs in selection order (the same arithmetic as one GPU).  Two barriers per layer
 * (system-scope flags, waits bounded at 2 s).  The batch needs the tensor-core MoE path (Q4_K/Q6_K
 * experts).  Before the first forward each rank exports qc_batch_ep_handle, the host gathers the
 * handles in rank order and passes them to qc_batch_ep_connect on every rank.  All ranks must then
 * make the same forward / decode calls with the same token counts, in the same order; a rank that
 * stops or a count mismatch ends the others' call with an error, after which every rank's batch
 * must be destroyed and created again. */
int qc_batch_ep_handle(qc_batch* b, void* handle, int* device_id);
int qc_batch_ep_connect(qc_batch* b, const void* handles, const int* device_ids);

/* model.rs:202-208: clear the KV cache and set the position to 0. */
int qc_reset(qc_engine* e);
int qc_position(const qc_engine* e, uint32_t* pos);
int qc_get_stats(const qc_engine* e, qc_stats* out);
/* Device time of each kernel kind over one decode step, from CUDA events
 * recorded between the kernels of a captured step graph (each span also holds
 * the launch gap before its kernel).  Runs one real step: it feeds the argmax
 * of the previous step (token 0 at position 0) and advances the position. */
typedef struct qc_phase_times {
  double embed_ms, attn_in_ms, attention_ms, oproj_ms, router_ms, gateup_ms, down_ms, output_ms;
  uint32_t launches; /* kernels in one step: 1 (whole-token kernel) or 2 + 6*layers (per-phase kernels) */
  double token_ms;   /* the whole step; with the whole-token kernel the per-kernel fields stay 0 */
} qc_phase_times;
int qc_profile_step(qc_engine* e, qc_phase_times* out);

/* Decode path (no counterpart in the reference, which has one CPU path per token).
 * mode 0 (default): the whole-token persistent kernel, one launch per token,
 * whenever the model's per-SM weight slices fit in shared memory, else the
 * per-phase kernels; mode 1: always the per-phase kernels (2 + 6*layers
 * launches per token).  Both compute the same forward. */
int qc_engine_set_decode_mode(qc_engine* e, int mode);
/* The path in use (0 whole-token kernel, 1 per-phase kernels) and, when the
 * whole-token kernel cannot be used, why (`why` may be NULL; "" when it fits). */
int qc_engine_decode_path(const qc_engine* e, int* path, const char** why);

/* Device pointer of the logits of the latest step (vocab floats). */
int qc_logits_device(const qc_engine* e, const float** out);

/* ---- per-matrix boundary (backend.rs:14-23 Backend::matvec, 174-261 packed_matvec) ---- */

/* Bytes of one GGUF row (quant.rs:12-21). */
int qc_row_bytes(uint32_t kind, uint64_t cols, uint64_t* out);

/* Upload `experts` stacked (rows x cols) matrices of GGML type `kind` from host
 * blocks (len = experts*rows*row_bytes) into the device layout. */
int qc_matrix_create(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t experts, const uint8_t* blocks,
                     uint64_t len, int device, qc_matrix** out);
/* y = W_expert x with device pointers on `stream` (cudaStream_t, NULL = default stream). */
int qc_matrix_matvec(const qc_matrix* m, uint32_t expert, const float* x, float* y, void* stream);
/* Dequantize expert `expert` to out[rows*cols] (device), bit-exact with quant.rs:36-80. */
int qc_matrix_dequant(const qc_matrix* m, uint32_t expert, float* out, void* stream);
/* Device bytes held, and packed GGUF bytes represented. */
int qc_matrix_bytes(const qc_matrix* m, uint64_t* device_bytes, uint64_t* packed_bytes);
void qc_matrix_destroy(qc_matrix* m);

/* Host-to-host matvec of one packed matrix: Vulkan::packed_matvec (backend.rs:174-261)
 * without the cache key: uploads, computes, copies y back. */
int qc_packed_matvec(uint32_t kind, uint64_t rows, uint64_t cols, const uint8_t* blocks, uint64_t len,
                     const float* x, float* y);

/* Allocation-free variant of qc_packed_matvec; it has no counterpart in the
 * reference.  For callers that may not allocate device memory: a host whose
 * own allocator has reserved the GPU's memory, or code that must not call
 * cudaFree (it may synchronize the whole device).  All device working memory
 * (raw blocks, the repacked matrix, x and y) lives in one static 32 MiB
 * __device__ array per GPU; larger matrices are rejected with QC_ERR_INVALID.
 * CUDA loads device code lazily, so the 32 MiB are reserved on a device at the
 * first call there (the current device), which also looks up the array's
 * address and sets kernel attributes: make that first call on each device
 * before the host's allocator claims the GPU's memory and before any stream
 * capture.  The array is then held until the process exits.  Calls share the
 * array: calls that overlap on the GPU race. */
int qc_packed_matvec_noalloc(uint32_t kind, uint64_t rows, uint64_t cols, const uint8_t* blocks, uint64_t len,
                             const float* x, float* y);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_CUDA_H */
