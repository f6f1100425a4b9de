// Kernel launch interface shared by the host engine (engine.cu) and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

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

// Model dimensions and scratch buffers used by the decode kernels.
struct DecodeDims {
  uint32_t hidden, heads, kvheads, head_dim, experts, top, inter, vocab, ctx;
  uint32_t nsplit;  // attention splits per KV head
  float eps;
};
struct Scratch {
  float* x;       // [hidden] residual stream
  float* xn;      // [hidden] ffn-normalised x (router -> experts)
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

void launch_repack(const uint8_t* src, uint64_t n_rows, uint64_t raw_row, uint32_t kind, uint64_t cols, uint8_t* dst,
                   uint64_t row_stride, __half* dplane, uint64_t d_stride, cudaStream_t s);
void launch_dequant(const MatDesc& m, uint32_t e, float* out, cudaStream_t s);
void launch_matvec(const MatDesc& m, uint32_t e, const float* x, float* y, int sms, cudaStream_t s);
size_t matvec_smem(const MatDesc& m);
cudaError_t matvec_prepare(int max_smem);

// One decode step (all kernels of one token) enqueued on `s`.
struct StepArgs {
  DecodeDims dims;
  Scratch sc;
  DevState* st;
  const LayerDev* layers;  // host array
  uint32_t n_layers;
  MatDesc embd, out;
  const float* out_norm;
  int sms;
};
// Kernel kinds of a step, in launch order within a layer.
enum StepKernel { K_EMBED = 0, K_ATTN_IN, K_ATTENTION, K_OPROJ, K_ROUTER, K_GATEUP, K_DOWN, K_OUTPUT, K_COUNT };
// Called before each launch of a step with the kernel kind, and once more with K_COUNT after the last.
typedef void (*StepHook)(void* ctx, int kind, cudaStream_t s);
void launch_step(const StepArgs& a, cudaStream_t s, StepHook hook = nullptr, void* ctx = nullptr);
inline uint32_t step_launches(uint32_t layers) { return 2 + 6 * layers; }
cudaError_t decode_prepare(int max_smem);

}  // namespace qc
