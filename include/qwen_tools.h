/* qwen_tools.h — host-side model tooling for the Qwen3-MoE CUDA engine.
 *
 * The reference crate (qwen-rust 0.1.0) reads GGUF files but never writes
 * quantized ones: quant.rs only decodes, and tools/reference_fixture.py:21-66
 * writes F32 tensors only.  These entry points add the missing encoders and a
 * synthetic-model writer so that every benchmark configuration can be built
 * without network access.  They run on the host only (no CUDA).
 *
 * Library: qwen-30brust_b200/libqwen_tools.so
 */
#ifndef QWEN_TOOLS_H
#define QWEN_TOOLS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids (quant.rs:5-11). */
enum {
  QC_F32 = 0,
  QC_F16 = 1,
  QC_Q4_0 = 2,
  QC_Q8_0 = 8,
  QC_Q4_K = 12,
  QC_Q5_K = 13,
  QC_Q6_K = 14
};

/* A synthetic qwen3moe model: architecture, tensor types and weight law. */
typedef struct qct_spec {
  uint32_t hidden, layers, heads, kvheads, head_dim, experts, top, intermediate, vocab;
  uint32_t context_length;
  float eps, theta;
  uint32_t kind_embd, kind_attn, kind_attn_out, kind_router, kind_gate_up, kind_down, kind_output;
  uint32_t tied_output; /* 1: omit output.weight (model.rs:290-294 falls back to token_embd) */
  float weight_std;     /* random weights are N(0, weight_std) */
  float norm_value;     /* every norm weight is this constant */
  uint64_t seed;
} qct_spec;

/* Quantize n floats (a multiple of the block size) into GGML blocks.
 * Returns 0, -1 for an unsupported kind or ragged n, -2 if out_len is short. */
int qct_quantize(uint32_t kind, const float* x, size_t n, uint8_t* out, size_t out_len);

/* Elements [first, first+n) of the N(mean, std) stream (seed, stream). */
void qct_normal(uint64_t seed, uint64_t stream, uint64_t first, float mean, float std, float* out, size_t n);

/* The stream id used for a tensor name (FNV-1a of the name). */
uint64_t qct_stream_of(const char* name);

/* rows x cols random N(0, std) weights, quantized row by row into out. */
int qct_random_matrix(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t seed, uint64_t stream, float std,
                      uint8_t* out, size_t out_len, int threads);

/* Size in bytes of the GGUF image for a spec, then the image itself. */
int qct_synth_size(const qct_spec* spec, uint64_t* total);
int qct_synth_write(const qct_spec* spec, uint8_t* out, uint64_t len, int threads);

float qct_f16_to_f32(uint16_t v);
uint16_t qct_f32_to_f16(float v);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_TOOLS_H */
