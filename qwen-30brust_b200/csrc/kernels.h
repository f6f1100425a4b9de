// Kernel launch interface shared by the host engine (engine.cu) and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "layout.h"

namespace qc {

// Device-resident step state (one per engine).
struct DevState {
  uint32_t pos;        // position of the token being processed
  uint32_t token;      // input token of the next step
  uint32_t nonfinite;  // sticky: a router logit or an output logit was not finite
  uint32_t bad_token;  // sticky: an input token was outside the vocabulary
  unsigned long long best;  // packed argmax of the current step: (total-order key << 32) | ~index
  uint32_t gen_count;  // tokens appended to gen_tokens
  uint32_t gen_cap;
  uint32_t* gen_tokens;
  uint32_t attn_done[64];  // last-block counters, one per KV head
  uint32_t router_done;
  uint32_t output_done;
  uint32_t abort;  // sticky: a wait of the whole-token kernel timed out
  // Tag of the whole-token kernel's inter-block values: one per token, never
  // reset (an engine reset keeps it, so values of earlier tokens never match).
  uint32_t seq;
};

// Per-layer weights in the device layout.
struct LayerDev {
  MatDesc q, k, v, o, router, gate, up, down;
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* ffn_norm;
  float* kc;  // [kvheads][ctx][head_dim]
  float* vc;
};

static_assert(sizeof(LayerDev) % 16 == 0, "LayerDev is copied in 16-byte pieces");

// Model dimensions and scratch buffers used by the decode kernels.
struct DecodeDims {
  uint32_t hidden, heads, kvheads, head_dim, experts, top, inter, vocab, ctx;
  uint32_t nsplit;  // attention splits per KV head
  float eps;
};
struct Scratch {
  float* x;       // [hidden] residual stream
  float* qkv;     // [heads*D + 2*kvheads*D] raw projections
  float* attn;    // [heads*D] attention output
  float* part;    // [kvheads][nsplit][G][D + 2] attention partials
  float* rlogit;  // [experts] router logits
  uint32_t* sel;  // [top] selected experts
  float* selw;    // [top] their weights
  float* h;       // [top][inter] SwiGLU activations
  float* logits;  // [vocab]
  const float2* rope;  // [ctx][D/2] (cos, sin)
};

void launch_repack(const uint8_t* src, uint64_t flat0, uint64_t n_rows, uint32_t rows, uint64_t raw_row, uint32_t kind,
                   uint64_t cols, uint8_t* dst, const DevLayout& l, uint64_t expert_stride, cudaStream_t s);
void launch_dequant(const MatDesc& m, uint32_t e, float* out, cudaStream_t s);
void launch_matvec(const MatDesc& m, uint32_t e, const float* x, float* y, int sms, cudaStream_t s);
size_t matvec_smem(const MatDesc& m);
cudaError_t matvec_prepare(int max_smem);

// ---- decode step ---------------------------------------------------------------------------
constexpr uint32_t kMinChunk = 64;                // attention positions per split, at least
constexpr uint32_t kWeightBudget = 160 * 1024;    // shared-memory weight bytes per block
constexpr uint32_t kOutStageBudget = 48 * 1024;   // shared-memory bytes per vocab-projection stage

// Positions per attention split held in shared memory, and the kernel's dynamic shared memory.
__host__ __device__ inline uint32_t attn_cmax(const DecodeDims& d) {
  const uint32_t c = (d.ctx + d.nsplit - 1) / d.nsplit;
  return c < kMinChunk ? kMinChunk : c;
}
inline size_t attn_smem(const DecodeDims& d) {
  const uint32_t G = d.heads / d.kvheads, c = attn_cmax(d), kp = d.head_dim + 4;
  return (size_t)(2 * c * kp + G * kp + G * c + d.head_dim) * sizeof(float);
}

struct StepArgs {
  DecodeDims dims;
  Scratch sc;
  DevState* st;
  const LayerDev* layers;      // host array
  const LayerDev* layers_dev;  // the same array in device memory (whole-token kernel)
  uint32_t n_layers;
  // expert parallelism (whole-token kernel): shard ep_rank of ep_world holds experts [e_lo, e_lo + e_n)
  uint32_t ep_rank, ep_world, e_lo, e_n;
  unsigned long long* const* peers;  // device array: exchange buffers of the ranks (own included)
  MatDesc embd, out;
  const float* out_norm;
  int sms;
};
// Grid and per-block work of the per-layer kernels (the same for every layer).
struct KernelSplit {
  uint32_t grid, gper, wbytes;  // blocks, row groups per block, shared-memory weight bytes per block
};
struct StepPlan {
  KernelSplit attn_in, oproj, router, gateup, down;
  uint32_t gateup_bpe;        // gate/up blocks per selected expert
  uint32_t out_grid, out_sg;  // vocab projection: blocks, groups per pipeline stage
};
StepPlan plan_step(const StepArgs& a);
size_t step_smem_max(const StepArgs& a, const StepPlan& p);

// Kernel kinds of a step, in launch order within a layer.
enum StepKernel { K_EMBED = 0, K_ATTN_IN, K_ATTENTION, K_OPROJ, K_ROUTER, K_GATEUP, K_DOWN, K_OUTPUT, K_COUNT };
// Called before each launch of a step with the kernel kind, and once more with K_COUNT after the last.
typedef void (*StepHook)(void* ctx, int kind, cudaStream_t s);
void launch_step(const StepArgs& a, const StepPlan& p, cudaStream_t s, StepHook hook = nullptr, void* ctx = nullptr);
inline uint32_t step_launches(uint32_t layers) { return 2 + 6 * layers; }
cudaError_t decode_prepare(int max_smem);

// ---- whole-token persistent kernel (token.cu) ---------------------------------------------
constexpr uint32_t kMaxTokenLayers = 256;
constexpr uint32_t kMaxTokenSlots = 12;  // vocab-projection pipeline stages

// Work layout of the whole-token kernel: shared-memory regions and the offsets
// (in 8-byte tagged values) of its per-layer exchange buffers.
struct TokenPlan {
  uint32_t nb;                          // thread blocks (one per SM)
  uint32_t p_bytes, q_bytes;            // weight regions P and Q
  uint32_t stage_off, misc_off, smem;   // staging area, small arrays, dynamic total
  uint32_t smax;                        // attention splits per KV head, at most
  uint32_t out_sg, nsp, nsq;            // vocab stage groups; stage slots in P and Q
  uint32_t nsegs;                       // row-run descriptors in shared memory
  uint32_t part_floats;                 // unit-group partial sums of the row engine
  uint64_t ll_qkv, ll_part, ll_attn, ll_xmid, ll_rl, ll_h, ll_xout, ll_moe, ll_layer;  // exchange buffer offsets
};
// Fills *p and returns nullptr if the model fits the whole-token kernel, else the reason it does not.
const char* plan_token(const StepArgs& a, int max_smem, TokenPlan* p);
// One token: the whole forward of StepArgs as one launch.  `ll` holds a.n_layers * p.ll_layer values.
void launch_token(const StepArgs& a, const TokenPlan& p, unsigned long long* ll, bool cooperative, cudaStream_t s);
cudaError_t token_prepare(int max_smem);

// A matrix (or expert stack) in the tensor-core GEMM's layout: 64-row tiles, a tile's super-blocks
// back to back, each (tile, super-block) one contiguous block of its 64 rows, Q4_K [64][144] or Q6_K
// [64][208] followed by the 64 rows' f16 d values, so that a GEMM stage is two contiguous copies.
// Rows past `rows` are zeros.
struct GemmMat {
  const uint8_t* w;
  uint32_t kind, rows, cols;
  uint32_t tiles;           // ceil(rows / 64)
  uint32_t blockb;          // bytes of one (tile, super-block) block
  uint64_t tile_bytes;      // cols / 256 blocks
  uint64_t expert_stride;   // tiles * tile_bytes
};
inline GemmMat gemm_mat(const MatDesc& m, const uint8_t* w) {
  GemmMat g{};
  g.w = w;
  g.kind = m.kind;
  g.rows = m.rows;
  g.cols = m.cols;
  g.tiles = (m.rows + 63) / 64;
  g.blockb = 64 * (m.kind == Q4_K ? 144 : 210);
  g.tile_bytes = (uint64_t)(m.cols / 256) * g.blockb;
  g.expert_stride = g.tiles * g.tile_bytes;
  return g;
}
// Device bytes of an expert stack in the GEMM layout.
inline uint64_t gemm_bytes(const MatDesc& m, uint32_t experts) { return (uint64_t)experts * gemm_mat(m, nullptr).expert_stride; }
// src (engine layout, `experts` matrices) -> dst (GEMM layout, dst.w sized by gemm_bytes).
void launch_qg_relayout(const MatDesc& src, uint32_t experts, const GemmMat& dst, cudaStream_t s);

// The MoE half of one layer for a batch of tokens (moe.cu).
struct QgGroup;
struct MoeArgs {
  MatDesc router, gate, up, down;  // one layer's router and expert stacks, device layout
  GemmMat ggate, gup, gdown;       // the expert stacks in the GEMM layout
  const float* ffn_norm;
  uint32_t H, I, E, top, T;
  float eps;
  float smin_g, smin_u, smin_d;  // Q4_K min-block scales of the tensor-core GEMM (qgemm.cu)
  uint32_t NPgu, NPdn, SSgu, SSdn;  // vectors per GEMM pass and stages (qgemm_shape)
  int sms;
  uint32_t e_lo, e_n;  // experts the GEMM weights hold: [e_lo, e_lo + e_n) (e_n 0: all E)
  // scratch
  float* h;          // [T][H] normalized inputs
  float* hscale;     // [T] power-of-two scale of each token's h
  float* rlg;        // [T][E] router logits
  uint32_t* sel;     // [T][top] selected experts, selection order
  float* selw;       // [T][top] their weights
  uint32_t* cnt;     // [E] pairs per expert
  uint32_t* off;     // [E] first grouped pair of each expert
  uint32_t* ptok;    // [T*top] grouped pairs: token
  uint32_t* ppair;   // [T*top] grouped pairs: pair id t*top + slot
  QgGroup* groups;   // [2E] GEMM groups: gate/up, then down
  uint32_t* nitems;  // [2] their work items
  uint4* imgrows;    // [moe_image_rows] rows of the gate/up activation image
  uint32_t* nrows;   // [1] image rows in use
  uint8_t* img_gu;   // gate/up activation image (hidden columns)
  uint8_t* img_dn;   // down activation image (intermediate columns), written by the SwiGLU epilogue
  float* y;          // [T*top][H] down outputs by pair id
  uint32_t* err;     // bit 0: non-finite router logit; bit 1: a tensor-core wait timed out; bit 2: fp16 range;
                     // bit 3: an expert-parallel barrier timed out; bit 4: ranks with different token counts
};
const char* moe_tc_supported(const MoeArgs& a);
// Rows of the activation images for T tokens (pairs rounded up to 16 per expert), at most.
uint32_t moe_image_rows(uint32_t T, uint32_t top, uint32_t E);
// x [T][H] -> out [T][H]: route, plan, tensor-core gate/up + SwiGLU, down, combine.
// (null, or why it could not launch)
const char* launch_moe_tc(const MoeArgs& a, const float* x, float* out, cudaStream_t s);

// Expert parallelism of the batched MoE layer: `world` ranks, one GPU each, every rank with T tokens
// of its own sequences and experts [rank * e_n, (rank + 1) * e_n).  Each rank's exchange region
// (device memory of that rank, mapped into every other rank) holds, at the byte offsets below:
//   flags [8] u64   flags[q]: the latest barrier number rank q has passed (written by rank q)
//   hdr   u32       this layer's T
//   h     [T][H]    the tokens' normalized inputs; hs [T] their scales; sel [T][top] their experts
//   y     [world * T * top][H]  down outputs of the pairs routed here, by global pair id
//                   (global token g = rank * T + t, pair g * top + slot)
// hdr .. y are double-buffered by the caller (one set per parity of a running layer count).
struct MoeEp {
  uint32_t rank, world, e_n, T;
  uint8_t* const* peers;  // [world] every rank's exchange region (device array; own included)
  uint8_t* own;           // this rank's region
  uint64_t o_flags, o_hdr, o_h, o_hs, o_sel, o_y;
};
// Bytes of one rank's exchange region and the offsets of the two buffer sets (b = 0, 1).
uint64_t moe_ep_layout(uint32_t cap, uint32_t H, uint32_t top, uint32_t world, MoeEp* set0, MoeEp* set1);
// As launch_moe_tc, over all ranks' tokens for this rank's experts: route and select into the
// exchange, barrier `seq`, gather every rank's inputs and selections, plan / image / GEMMs over the
// pairs of the local experts (down outputs into the exchange), barrier `seq + 1`, then the combine
// of this rank's tokens from the ranks that hold their experts, in selection order.  a.T = ep.T
// (this rank's tokens); a's scratch holds world * T tokens.  Barrier waits give up after 2 s
// (err bit 3); ranks with different T set err bit 4.
const char* launch_moe_tc_ep(const MoeArgs& a, const MoeEp& ep, unsigned long long seq, const float* x, float* out,
                             cudaStream_t s);
// The per-token MoE kernels of the decode step (router, gate/up, down) on the vector c.x, in place.
StepPlan plan_moe(const DecodeDims& d, const LayerDev& L, int sms);
void launch_moe_token(const DecodeDims& d, const StepPlan& p, const LayerDev& L, const Scratch& c, DevState* st,
                      cudaStream_t s);

// Device state of one sampler (sampling.rs:3-8): the StdRng keystream position and the parameters.
struct SamplerDev {
  uint32_t key[8];          // ChaCha12 key (from seed_from_u64)
  unsigned long long word;  // next keystream word
  float temperature, top_p;
  uint32_t top_k;           // 0 = off
  uint32_t err;             // sticky: the logits held a non-finite value
  uint32_t token;           // the last sampled id
};
// Sampler::sample on n device logits: one block; the id goes to s->token and, if given, *token_dst.
// Device scratch of a sample over more than sample_exact_max() ids (a set too large for shared
// memory): the sort's ping-pong (key, index) arrays and the probabilities, their quotients by the
// total and the total's running sums, n words each (sample_scratch_bytes(n) in all).
struct SampleScratch {
  uint32_t *key0, *key1, *idx0, *idx1;
  float *p, *q, *run;
};
inline size_t sample_scratch_bytes(uint32_t n) { return (size_t)n * 4 * 7; }
inline SampleScratch sample_scratch_at(void* base, uint32_t n) {
  uint32_t* w = static_cast<uint32_t*>(base);
  return SampleScratch{w, w + n, w + 2 * (size_t)n, w + 3 * (size_t)n, reinterpret_cast<float*>(w + 4 * (size_t)n),
                       reinterpret_cast<float*>(w + 5 * (size_t)n), reinterpret_cast<float*>(w + 6 * (size_t)n)};
}
uint32_t sample_exact_max();
// Once per device (the dynamic shared-memory attribute of the sampler kernel), before launch_sample.
cudaError_t sample_prepare();
cudaError_t launch_sample(const float* logits, uint32_t n, SamplerDev* s, uint32_t* token_dst,
                          const SampleScratch& scr, cudaStream_t st);
// `draws` samples at once, one block each: logits row rows[b] (n floats) with sampler sv[b] (both
// device arrays of device pointers), id to tokens[b] (device).  scratch: draws x
// sample_scratch_bytes(n) bytes (needed when a sampler's top-k set exceeds sample_exact_max()), or null.
cudaError_t launch_sample_batch(const float* const* rows, uint32_t n, uint32_t draws, SamplerDev* const* sv,
                                uint32_t* tokens, void* scratch, cudaStream_t st);

// ---- several sequences per step (batch.cu) --------------------------------------------------
struct BatchTok {
  uint32_t seq, pos;  // the token's sequence and its position there
};
struct BatchArgs {
  const BatchTok* tok;  // [T] device
  float* kv;            // [seq][layer][K, V][kvheads][ctx][head_dim]
  uint64_t kv_floats;   // floats of one K (or V) block of one layer: kvheads * ctx * head_dim
  uint32_t n_layers, heads, kvheads, D, ctx;
  float eps;
  const float2* rope;   // [ctx][D/2] (cos, sin)
};
cudaError_t batch_prepare(int max_smem);
size_t batch_matvec_smem(const MatDesc& m);
size_t batch_attention_smem(uint32_t heads, uint32_t kvheads, uint32_t D);
// x[t] = embedding row ids[t]
void launch_batch_embed(const MatDesc& embd, const BatchTok* tok, const uint32_t* ids, uint32_t T, uint32_t H, float* x,
                        cudaStream_t s);
// XView t (at xv + t * xb) of rms(x[src ? src[t] : t], w), or of the vector itself when w is null
void launch_batch_stage(const float* x, const uint32_t* src, uint32_t T, uint32_t n, uint32_t units, bool with_float,
                        const float* w, float eps, uint8_t* xv, uint32_t xb, cudaStream_t s);
// y[v * ystride + r] = (add ? add[v * ystride + r] : 0) + (W x_v)[r] for the T XViews
void launch_batch_matvec(const MatDesc& m, const uint8_t* xv, uint32_t xb, uint32_t T, float* y, uint64_t ystride,
                         const float* add, int sms, cudaStream_t s);
void launch_batch_qkprep(const BatchArgs& a, uint32_t layer, const float* q_norm, const float* k_norm, float* q,
                         const float* k, const float* v, uint32_t T, cudaStream_t s);
void launch_batch_attention(const BatchArgs& a, uint32_t layer, const float* q, float* out, uint32_t T, cudaStream_t s);
void launch_batch_finite(const float* v, uint64_t n, uint32_t* flag, cudaStream_t s);
// n keystream words of the sampler (advancing it), for reproducibility checks.
void launch_sampler_words(SamplerDev* s, uint32_t n, uint32_t* out, cudaStream_t st);

// ---- tensor-core GEMM over Q4_K / Q6_K rows (qgemm.cu) ---------------------------------------
// A group: some rows of a matrix (or, in pair mode, of two matrices side by side) times `cnt`
// vectors of the B image (rows imgoff .. imgoff + nimg of it, nimg a multiple of 16, rows past cnt
// zero).  Its work items are (128-row tile, pass of up to NP vectors), items item0 .. of the launch.
struct QgGroup {
  uint32_t item0, cnt, nimg, imgoff;
  uint32_t mat;  // rows from mats[mat] (pair mode: tile rows 0-63 from mats[mat], 64-127 from mats[mat + 1])
  uint32_t e;    // expert index in those matrices
  float* y;      // plain epilogue: y[row(n) * ystride + r] (+ add[same]), row(n) = ymap ? ymap[n] : n
  const float* add;
  const uint32_t* ymap;
  const uint32_t* hsmap;  // the scale of image vector n is hs[hsmap ? hsmap[n] : n] (hs null: 1)
  uint64_t ystride;
};
struct QgArgs {
  GemmMat mats[4];
  float smin[4];        // Q4_K: power-of-two scale of the min block (dmin * mn * smin < 2^14)
  uint32_t pair;        // pair mode (SwiGLU: gate rows then up rows of each 128-row tile)
  uint32_t K, NP, SS;   // columns (a multiple of 256); vectors per pass; stages (qgemm_shape)
  uint32_t img_hasmin;  // the image carries the Q4_K min chunks
  const uint8_t* img;
  const float* hs;
  const QgGroup* groups;  // device array of ngroups, or null: inl
  uint32_t ngroups;
  const uint32_t* nitems_dev;  // device item count, or null: nitems
  uint32_t nitems;
  QgGroup inl[3];
  uint8_t* img2;  // SwiGLU epilogue: the image of the next GEMM (K = K2, K step = tile)
  uint32_t K2, img2_hasmin;
  uint32_t* err;  // bit 1: a wait timed out; bit 2: a SwiGLU output outside the fp16 range
};
// B image rows: either `rows` (device, *nrows of them: {source row or ~0, imgoff, nimg, 0}) or the
// dense form: rows 0 .. round16(T), source src[i] (or i) for i < T.
struct QgImageArgs {
  const float* x;
  uint64_t xstride;
  uint32_t K, T;
  const uint32_t* src;
  const uint4* rows;
  const uint32_t* nrows;
  const float* w;  // RMSNorm weight, or null
  float eps;
  const float* hs_in;  // per source row, or null: computed (pow2 of max |x|) and written to hs_out[i]
  float* hs_out;
  uint32_t hasmin;
  uint8_t* img;
};
__host__ __device__ inline float qg_pow2_scale(float maxabs) {  // 2^k with maxabs * 2^k < 2^14
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 1.f;
  int ex;
  frexpf(maxabs, &ex);
  return ldexpf(1.f, 14 - ex);
}
const char* qgemm_supported(uint32_t kind, uint32_t cols);
// Vectors per pass and B stages of a GEMM over `cols` columns of `kind` rows (after qgemm_prepare),
// or the reason it cannot run.
const char* qgemm_shape(uint32_t kind, uint32_t cols, bool img_hasmin, uint32_t* np, uint32_t* ss);
uint64_t qg_image_row_bytes(uint32_t cols, bool hasmin);
size_t qgemm_smem(uint32_t kind, uint32_t cols, uint32_t np, uint32_t ss, bool img_hasmin);
cudaError_t qgemm_prepare();  // once per device
size_t qgemm_smem_cap();      // dynamic shared memory available to the GEMM kernels (after qgemm_prepare)
void launch_qgemm(const QgArgs& a, uint32_t kind, bool swiglu, uint32_t grid, cudaStream_t s);
void launch_qg_image(const QgImageArgs& a, uint32_t grid, cudaStream_t s);
void launch_qg_dmin(const MatDesc& m, uint32_t experts, uint32_t* out, cudaStream_t s);

}  // namespace qc
