// Several sequences per step: the forward of model.rs:217-302 for a batch of T
// tokens, each appended to its own sequence's KV cache at that sequence's next position.
//
// The reference runs one token of one sequence at a time (Model::forward, src/model.rs:210-216);
// here one step carries T tokens from any mix of sequences: decode (one token of each of many
// sequences) and prefill chunks (consecutive tokens of one sequence, each attending to the ones
// before it) are the same call.  Per layer:
//   k_b_stage     per token: rms(x, attn_norm) quantized to the activation digit planes (XView) in
//                 global memory, the same staging the decode kernels use in shared memory
//   k_b_matvec    Q, K, V rows: a block streams a run of weight row groups through shared memory
//                 (cp.async, 3 stages) and applies every stage to all T activation vectors, so each
//                 weight byte is read from HBM once per step however many tokens the step carries
//   k_b_qkprep    per token: QK-norm, NeoX RoPE at the token's position, K and V rows appended to
//                 its sequence's cache (model.rs:233-243)
//   k_b_attention per (token, KV head): the GQA heads over the token's sequence, positions
//                 0..pos, online softmax over tiles of 32 positions (ops.rs:57-98)
//   k_b_matvec    O rows + residual (model.rs:245-248)
//   MoE           moe.cu's batched path: router and top-k per token, the tokens grouped per expert,
//                 gate/up + SwiGLU and down as tcgen05 tensor-core GEMMs, weighted combine
// then the output norm and vocabulary rows for the tokens whose logits are wanted (model.rs:289-301),
// and a finiteness check.
#include "kernels.h"

namespace qc {
namespace {

constexpr int kBStages = 3;
constexpr uint32_t kAttTile = 32;  // attention positions per tile

__device__ __forceinline__ float* seq_kv(const BatchArgs& a, uint32_t seq, uint32_t layer, uint32_t which) {
  return a.kv + ((uint64_t)seq * a.n_layers + layer) * 2 * a.kv_floats + which * a.kv_floats;
}

__global__ void __launch_bounds__(256) k_b_embed(MatDesc embd, const uint32_t* __restrict__ ids, uint32_t H,
                                                  float* __restrict__ x) {
  const uint32_t t = blockIdx.x, id = ids[t];
  const uint8_t* row = row_ptr(embd, embd.w, id);
  const __half* drow = drow_ptr(embd, embd.w, id);
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) x[(uint64_t)t * H + i] = dequant_one(embd, row, drow, i);
}

// XView of rms(x[src[t]], w) (w null: of x[src[t]] itself) for t < gridDim.x, at xv + t * xb.
__global__ void __launch_bounds__(512) k_b_stage(const float* __restrict__ x, const uint32_t* __restrict__ src,
                                                  uint32_t n, uint32_t units, bool with_float, const float* __restrict__ w,
                                                  float eps, uint8_t* __restrict__ xv, uint32_t xb) {
  __shared__ float red[32];
  const uint32_t t = blockIdx.x;
  const float* xr = x + (uint64_t)(src ? src[t] : t) * n;
  if (w)
    stage_vectors<true>(xv + (uint64_t)t * xb, 1, n, units, with_float, [&](uint32_t, uint32_t i) { return xr[i]; }, w,
                        eps, red);
  else
    stage_vectors<false>(xv + (uint64_t)t * xb, 1, n, units, with_float, [&](uint32_t, uint32_t i) { return xr[i]; },
                         nullptr, 0.f, red);
}

// y[v][r] = (add ? add[v][r] : 0) + W x_v for v < T: a block's run of row groups streamed through
// shared memory, each stage applied to every activation vector (XViews in global memory).
template <uint32_t KIND>
__global__ void __launch_bounds__(512) k_b_matvec(MatDesc m, const uint8_t* __restrict__ xv, uint32_t xb, uint32_t T,
                                                   float* y, uint64_t ystride, const float* add, uint32_t sg) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t groups = (m.rows + 7) / 8;
  const uint32_t per = (groups + gridDim.x - 1) / gridDim.x;
  const uint32_t g0 = min(groups, blockIdx.x * per), g1 = min(groups, g0 + per);
  const uint32_t nst = (g1 - g0 + sg - 1) / sg;
  const uint64_t stage_bytes = (uint64_t)sg * m.group_bytes;
  for (uint32_t k = 0; k < kBStages - 1; k++) {
    if (k < nst) copy_groups(smem + (k % kBStages) * stage_bytes, m, 0, g0 + k * sg, min(g1, g0 + (k + 1) * sg));
    cp_commit();
  }
  const bool flt = uses_float_x(KIND);
  for (uint32_t k = 0; k < nst; k++) {
    const uint32_t kn = k + kBStages - 1;
    if (kn < nst) copy_groups(smem + (kn % kBStages) * stage_bytes, m, 0, g0 + kn * sg, min(g1, g0 + (kn + 1) * sg));
    cp_commit();
    cp_wait<kBStages - 1>();
    __syncthreads();
    const uint8_t* sb = smem + (k % kBStages) * stage_bytes;
    const uint32_t r0 = (g0 + k * sg) * 8, r1 = min(m.rows, min(g1, g0 + (k + 1) * sg) * 8);
    for (uint32_t v = 0; v < T; v++) {
      float* yv = y + v * ystride;
      const float* av = add ? add + v * ystride : nullptr;
      warp_rows_k<KIND, true>(m, r0, r1, xview_at(xv + (uint64_t)v * xb, m.units, flt), SmemRows{&m, sb, r0},
                              [&](uint32_t r, float s) { yv[r] = av ? __fadd_rn(av[r], s) : s; }, threadIdx.x >> 5,
                              blockDim.x >> 5);
    }
    __syncthreads();
  }
}

// Per token (one block): QK-norm and RoPE at its position for the query heads (in place) and the
// key heads; the key and value rows appended to its sequence's cache (model.rs:233-243).
__global__ void __launch_bounds__(256) k_b_qkprep(BatchArgs a, uint32_t layer, const float* __restrict__ q_norm,
                                                   const float* __restrict__ k_norm, float* __restrict__ q,
                                                   const float* __restrict__ k, const float* __restrict__ v) {
  extern __shared__ __align__(16) float hv[];  // [8 warps][D]
  const uint32_t t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const BatchTok tk = a.tok[t];
  const uint32_t D = a.D, QH = a.heads, KH = a.kvheads;
  const float2* cs = a.rope + (uint64_t)tk.pos * (D / 2);
  float* buf = hv + warp * D;
  float* kc = seq_kv(a, tk.seq, layer, 0);
  float* vc = seq_kv(a, tk.seq, layer, 1);
  // block (t, y): heads nw y .. nw y + nw - 1 of token t (query heads, then KV heads), one per warp
  for (uint32_t h = blockIdx.y * nw + warp; h < min(QH + KH, (blockIdx.y + 1) * nw); h += nw) {
    const bool isq = h < QH;
    const float* src = isq ? q + ((uint64_t)t * QH + h) * D : k + ((uint64_t)t * KH + (h - QH)) * D;
    for (uint32_t i = lane; i < D; i += 32) buf[i] = src[i];
    __syncwarp();
    head_norm_rope(buf, isq ? q_norm : k_norm, D, a.eps, cs);
    if (isq)
      for (uint32_t i = lane; i < D; i += 32) q[((uint64_t)t * QH + h) * D + i] = buf[i];
    else {
      const uint32_t kh = h - QH;
      for (uint32_t i = lane; i < D; i += 32) {
        kc[((uint64_t)kh * a.ctx + tk.pos) * D + i] = buf[i];
        vc[((uint64_t)kh * a.ctx + tk.pos) * D + i] = v[((uint64_t)t * KH + kh) * D + i];
      }
    }
    __syncwarp();
  }
}

// Per (token, KV head): out = softmax(q k^T / sqrt(D)) v over positions 0..pos of the token's
// sequence for the G query heads of the KV head; warp w handles heads w, w + 8, ...; lane l
// scores position l of each tile and sums dimensions l, l + 32, ... (D <= 128).
__global__ void __launch_bounds__(256) k_b_attention(BatchArgs a, uint32_t layer, const float* __restrict__ q,
                                                      float* __restrict__ out) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t t = blockIdx.x / a.kvheads, kh = blockIdx.x % a.kvheads;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const BatchTok tk = a.tok[t];
  const uint32_t D = a.D, G = a.heads / a.kvheads, KP = D + 1, time = tk.pos + 1;
  float* qs = sm;                       // [G][D]
  float* kt = qs + G * D;               // [32][D + 1]
  float* vt = kt + kAttTile * KP;       // [32][D]
  const float* kc = seq_kv(a, tk.seq, layer, 0) + (uint64_t)kh * a.ctx * D;
  const float* vc = seq_kv(a, tk.seq, layer, 1) + (uint64_t)kh * a.ctx * D;
  for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) qs[i] = q[((uint64_t)t * a.heads + kh * G) * D + i];
  const float sd = sqrtf((float)D);
  constexpr int kMaxHeadsPerWarp = 4, kDims = 4;  // G <= 32, D <= 128
  float mrun[kMaxHeadsPerWarp], lrun[kMaxHeadsPerWarp], acc[kMaxHeadsPerWarp][kDims];
#pragma unroll
  for (int j = 0; j < kMaxHeadsPerWarp; j++) {
    mrun[j] = -INFINITY;
    lrun[j] = 0.f;
#pragma unroll
    for (int i = 0; i < kDims; i++) acc[j][i] = 0.f;
  }
  for (uint32_t s0 = 0; s0 < time; s0 += kAttTile) {
    const uint32_t n = min(kAttTile, time - s0);
    __syncthreads();  // the previous tile is consumed (and qs is written)
    for (uint32_t i = threadIdx.x; i < n * D; i += blockDim.x) {
      const uint32_t p = i / D, d = i % D;
      kt[p * KP + d] = kc[(uint64_t)(s0 + p) * D + d];
      vt[p * D + d] = vc[(uint64_t)(s0 + p) * D + d];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kMaxHeadsPerWarp; j++) {
      const uint32_t g = warp + j * nw;
      if (g >= G) break;
      float sc = -INFINITY;
      if (lane < n) {
        float dot = 0.f;
        for (uint32_t d = 0; d < D; d++) dot = fmaf(qs[g * D + d], kt[lane * KP + d], dot);
        sc = dot / sd;
      }
      const float mt = warp_max(sc), mn = fmaxf(mrun[j], mt);
      const float f = expf(mrun[j] - mn), p = lane < n ? expf(sc - mn) : 0.f;
      lrun[j] = lrun[j] * f + warp_sum(p);
      mrun[j] = mn;
#pragma unroll
      for (int i = 0; i < kDims; i++) acc[j][i] *= f;
      for (uint32_t pp = 0; pp < n; pp++) {
        const float w = __shfl_sync(0xffffffffu, p, pp);
#pragma unroll
        for (int i = 0; i < kDims; i++) {
          const uint32_t d = lane + 32 * i;
          if (d < D) acc[j][i] = fmaf(w, vt[pp * D + d], acc[j][i]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxHeadsPerWarp; j++) {
    const uint32_t g = warp + j * nw;
    if (g >= G) break;
    const float inv = 1.f / lrun[j];
#pragma unroll
    for (int i = 0; i < kDims; i++) {
      const uint32_t d = lane + 32 * i;
      if (d < D) out[((uint64_t)t * a.heads + kh * G + g) * D + d] = acc[j][i] * inv;
    }
  }
}

// Sticky flag when any of n values is not finite.
// 16-byte loads, four in flight per thread (v is 16-byte aligned; the n % 4 tail is read singly).
__global__ void __launch_bounds__(512) k_b_finite(const float* __restrict__ v, uint64_t n, uint32_t* flag) {
  bool bad = false;
  const uint64_t n4 = n / 4, step = (uint64_t)gridDim.x * blockDim.x;
  const float4* v4 = reinterpret_cast<const float4*>(v);
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += 4 * step) {
    float4 f[4];
#pragma unroll
    for (int k = 0; k < 4; k++) f[k] = i + k * step < n4 ? __ldg(v4 + i + k * step) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; k++) bad |= !isfinite(f[k].x) || !isfinite(f[k].y) || !isfinite(f[k].z) || !isfinite(f[k].w);
  }
  if (blockIdx.x == 0 && threadIdx.x < n % 4) bad |= !isfinite(v[n4 * 4 + threadIdx.x]);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

uint32_t b_stage_groups(const MatDesc& m) {
  const uint64_t sg = (56 * 1024) / m.group_bytes;
  return (uint32_t)(sg < 1 ? 1 : (sg > 8 ? 8 : sg));
}

}  // namespace

size_t batch_matvec_smem(const MatDesc& m) { return (size_t)kBStages * b_stage_groups(m) * m.group_bytes; }

cudaError_t batch_prepare(int max_smem) {
  cudaError_t err = cudaSuccess;
#define QC_ATTR(K)                                                                                      \
  if (err == cudaSuccess)                                                                               \
    err = cudaFuncSetAttribute(k_b_matvec<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  QC_ATTR(Q4_K) QC_ATTR(Q5_K) QC_ATTR(Q6_K) QC_ATTR(Q8_0) QC_ATTR(Q4_0) QC_ATTR(F16) QC_ATTR(F32)
#undef QC_ATTR
  if (err == cudaSuccess) err = cudaFuncSetAttribute(k_b_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  return err;
}

void launch_batch_embed(const MatDesc& embd, const BatchTok* tok, const uint32_t* ids, uint32_t T, uint32_t H, float* x,
                        cudaStream_t s) {
  k_b_embed<<<T, 256, 0, s>>>(embd, ids, H, x);
}

void launch_batch_stage(const float* x, const uint32_t* src, uint32_t T, uint32_t n, uint32_t units, bool with_float,
                        const float* w, float eps, uint8_t* xv, uint32_t xb, cudaStream_t s) {
  k_b_stage<<<T, 512, 0, s>>>(x, src, n, units, with_float, w, eps, xv, xb);
}

void launch_batch_matvec(const MatDesc& m, const uint8_t* xv, uint32_t xb, uint32_t T, float* y, uint64_t ystride,
                         const float* add, int sms, cudaStream_t s) {
  const uint32_t groups = (m.rows + 7) / 8, sg = b_stage_groups(m);
  uint32_t grid = (groups + sg - 1) / sg;
  grid = grid < (uint32_t)sms ? grid : (uint32_t)sms;
  grid = grid < 1 ? 1 : grid;
  const size_t smem = batch_matvec_smem(m);
  switch (m.kind) {
    case Q4_K: k_b_matvec<Q4_K><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    case Q5_K: k_b_matvec<Q5_K><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    case Q6_K: k_b_matvec<Q6_K><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    case Q8_0: k_b_matvec<Q8_0><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    case Q4_0: k_b_matvec<Q4_0><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    case F16: k_b_matvec<F16><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
    default: k_b_matvec<F32><<<grid, 512, smem, s>>>(m, xv, xb, T, y, ystride, add, sg); break;
  }
}

void launch_batch_qkprep(const BatchArgs& a, uint32_t layer, const float* q_norm, const float* k_norm, float* q,
                         const float* k, const float* v, uint32_t T, cudaStream_t s) {
  k_b_qkprep<<<dim3(T, (a.heads + a.kvheads + 7) / 8), 256, 8 * a.D * sizeof(float), s>>>(a, layer, q_norm, k_norm, q,
                                                                                          k, v);
}

size_t batch_attention_smem(uint32_t heads, uint32_t kvheads, uint32_t D) {
  return ((size_t)(heads / kvheads) * D + kAttTile * (D + 1) + kAttTile * D) * sizeof(float);
}

void launch_batch_attention(const BatchArgs& a, uint32_t layer, const float* q, float* out, uint32_t T, cudaStream_t s) {
  k_b_attention<<<T * a.kvheads, 256, batch_attention_smem(a.heads, a.kvheads, a.D), s>>>(a, layer, q, out);
}

void launch_batch_finite(const float* v, uint64_t n, uint32_t* flag, cudaStream_t s) {
  k_b_finite<<<148 * 4, 512, 0, s>>>(v, n, flag);
}

}  // namespace qc
