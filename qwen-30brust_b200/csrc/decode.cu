// Whole-token decode kernels: one token of reference model.rs:217-302 with
// every activation kept on the device.
//
// Per layer, six launches:
//   k_attn_in   RMSNorm(attn_norm) fused into the Q/K/V matvecs      (model.rs:228-232)
//   k_attention QK-norm, NeoX RoPE, KV append, split GQA attention   (model.rs:233-244, ops.rs:17-98)
//   k_oproj     O projection + residual                               (model.rs:245-248)
//   k_router    RMSNorm(ffn_norm) + router matvec + top-k + softmax   (model.rs:249-257, ops.rs:45-56)
//   k_gateup    gate/up matvecs of the selected experts + SwiGLU      (model.rs:259-274)
//   k_down      down matvecs, weighted combine, residual              (model.rs:275-287)
// then k_output: RMSNorm(output_norm), vocab matvec, finiteness check and
// greedy argmax (model.rs:289-301, sampling.rs:31-35).
//
// Launch chaining: every kernel is launched with programmatic stream
// serialization.  A kernel first issues L2 bulk prefetches of the weight rows
// its block will read (these do not depend on earlier kernels), then waits for
// the previous kernel (griddepcontrol.wait), then lets the next kernel launch
// (griddepcontrol.launch_dependents) and does its work.  The weight stream of
// kernel k+1 therefore overlaps the tail of kernel k.
#include <utility>

#include "kernels.h"

namespace qc {

constexpr int NT = 256;

QC_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QC_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Prefetch [p, p + bytes) into L2 (16-byte aligned start; whole 16-byte granules).
QC_DEV void prefetch_l2(const void* p, uint64_t bytes) {
  const uint64_t a = reinterpret_cast<uint64_t>(p) & ~15ull;
  const uint64_t end = (reinterpret_cast<uint64_t>(p) + bytes + 15) & ~15ull;
  for (uint64_t o = a + threadIdx.x * 65536ull; o < end; o += blockDim.x * 65536ull) {
    const uint32_t n = (uint32_t)(end - o < 65536ull ? end - o : 65536ull);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(o), "r"(n) : "memory");
  }
}
// Prefetch rows [r0, r1) of expert e of m (main plane and d plane).
QC_DEV void prefetch_rows(const MatDesc& m, uint32_t e, uint32_t r0, uint32_t r1) {
  if (r1 <= r0) return;
  prefetch_l2(m.w + e * m.expert_stride + (uint64_t)r0 * m.row_stride, (uint64_t)(r1 - r0) * m.row_stride);
  if (m.d) prefetch_l2(m.d + e * m.d_expert_stride + (uint64_t)r0 * m.d_stride, (uint64_t)(r1 - r0) * m.d_stride * 2);
}

// rms scale 1/sqrt(mean(x^2) + eps) of x[0..n) (reference ops.rs:3-15), block-wide.
QC_DEV float rms_scale(const float* __restrict__ x, uint32_t n, float eps, float* red) {
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  return 1.0f / sqrtf(ss / (float)n + eps);
}

// Rows [r0, r1) of this block for `rows` rows split over the grid in row groups of G.
struct RowChunk {
  uint32_t r0, r1;
};
QC_DEV RowChunk my_rows(uint32_t rows, uint32_t G) {
  const uint32_t groups = (rows + G - 1) / G;
  const uint32_t per = (groups + gridDim.x - 1) / gridDim.x;
  const uint32_t g0 = blockIdx.x * per, g1 = min(groups, g0 + per);
  return {min(rows, g0 * G), min(rows, g1 * G)};
}

// The block's warps walk row groups of its chunk; lpr lanes per row.
template <class F>
QC_DEV void for_rows(const MatDesc& m, RowChunk c, F&& body) {
  const uint32_t lpr = m.lpr, G = 32 / lpr, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (uint32_t base = c.r0 + warp * G; base < c.r1; base += nw * G) {
    const uint32_t r = base + lane / lpr, lr = lane % lpr;
    const bool ok = r < c.r1;
    body(r, lr, ok);
  }
}

// ---------------------------------------------------------------------------
// Embedding row, dequantized exactly as gguf.rs:204-213 (model.rs:225).
// Block 0 records the token fed at this step in gen_tokens (the greedy sequence
// when steps are chained on the device) and clears the argmax slot.
__global__ void k_embed(MatDesc embd, DevState* st, float* __restrict__ x, uint32_t vocab) {
  pdl_wait();
  pdl_trigger();
  uint32_t tok = st->token;
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    if (st->gen_tokens && st->gen_count < st->gen_cap) st->gen_tokens[st->gen_count] = tok;
    st->gen_count = st->gen_count + 1;
    st->best = 0ull;
  }
  if (tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) st->bad_token = 1;
    tok = 0;
  }
  const uint8_t* row = embd.w + (uint64_t)tok * embd.row_stride;
  const __half* drow = embd.d ? embd.d + (uint64_t)tok * embd.d_stride : nullptr;
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < embd.cols; c += gridDim.x * blockDim.x)
    x[c] = dequant_one(embd, row, drow, c);
}

// ---------------------------------------------------------------------------
// Q, K, V = W_{q,k,v} * rms(x).  The three matrices share lpr; the block's
// row chunk runs over the concatenated rows [Q | K | V].
__global__ void __launch_bounds__(NT) k_attn_in(MatDesc mq, MatDesc mk, MatDesc mv, const float* __restrict__ x,
                                                const float* __restrict__ norm, uint32_t hidden, float eps,
                                                float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t nq = mq.rows, nk = mk.rows, total = nq + nk + mv.rows;
  const uint32_t G = 32 / mq.lpr;
  const RowChunk c = my_rows(total, G);
  // prefetch this block's rows of each matrix
  prefetch_rows(mq, 0, min(c.r0, nq), min(c.r1, nq));
  prefetch_rows(mk, 0, min(max(c.r0, nq), nq + nk) - nq, min(max(c.r1, nq), nq + nk) - nq);
  prefetch_rows(mv, 0, max(c.r0, nq + nk) - nq - nk, max(c.r1, nq + nk) - nq - nk);
  pdl_wait();
  pdl_trigger();
  const float s = rms_scale(x, hidden, eps, red);
  const bool fl = uses_float_x(mq.kind) || uses_float_x(mk.kind) || uses_float_x(mv.kind);
  const XView xv = stage_x(smem, hidden, mq.units, fl, [&](uint32_t i) { return __fmul_rn(x[i], __fmul_rn(s, norm[i])); });
  for_rows(mq, c, [&](uint32_t r, uint32_t lr, bool ok) {
    const MatDesc& m = r < nq ? mq : (r < nq + nk ? mk : mv);
    const uint32_t rr = r < nq ? r : (r < nq + nk ? r - nq : r - nq - nk);
    float p = ok ? row_partial(m, 0, rr, lr, xv) : 0.f;
    p = group_sum(p, mq.lpr);
    if (lr == 0 && ok) out[r] = p;
  });
}

// ---------------------------------------------------------------------------
// Per-head RMSNorm + NeoX RoPE of one head vector held in shared memory by one warp.
QC_DEV void head_norm_rope(float* v, const float* __restrict__ w, uint32_t D, float eps, const float2* __restrict__ cs) {
  const uint32_t lane = threadIdx.x & 31;
  float ss = 0.f;
  for (uint32_t i = lane; i < D; i += 32) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float s = 1.0f / sqrtf(ss / (float)D + eps);
  for (uint32_t i = lane; i < D; i += 32) v[i] = __fmul_rn(v[i], __fmul_rn(s, w[i]));
  __syncwarp();
  // ops.rs:17-28: (a, b) -> (a c - b s, a s + b c) for pairs (i, i + D/2)
  for (uint32_t i = lane; i < D / 2; i += 32) {
    const float a = v[i], b = v[i + D / 2];
    const float2 t = cs[i];
    v[i] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
    v[i + D / 2] = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(b, t.x));
  }
  __syncwarp();
}

constexpr uint32_t kMinChunk = 64;  // positions per attention split, at least

// Split GQA decode attention.  Block (h, s) owns KV head h and positions
// [s*chunk, (s+1)*chunk) of [0, pos], chunk = max(64, ceil((pos+1)/nsplit)); it
// handles the G query heads of that KV head.  The block whose range holds `pos`
// appends the new K/V row.  The last active block of head h merges the partial
// softmax states.
__global__ void __launch_bounds__(NT) k_attention(DecodeDims dd, const float* __restrict__ qkv,
                                                  const float* __restrict__ qn_w, const float* __restrict__ kn_w,
                                                  float* __restrict__ kc, float* __restrict__ vc,
                                                  const float2* __restrict__ rope, float* __restrict__ part,
                                                  float* __restrict__ attn, DevState* st) {
  pdl_wait();
  pdl_trigger();
  const uint32_t h = blockIdx.x, s = blockIdx.y, D = dd.head_dim, G = dd.heads / dd.kvheads;
  const uint32_t pos = st->pos, time = pos + 1;
  uint32_t chunk = (time + dd.nsplit - 1) / dd.nsplit;
  chunk = chunk < kMinChunk ? kMinChunk : chunk;
  const uint32_t active = (time + chunk - 1) / chunk;
  if (s >= active) return;
  const uint32_t cmax = max(kMinChunk, (dd.ctx + dd.nsplit - 1) / dd.nsplit);
  const uint32_t t0 = s * chunk, t1 = min(time, t0 + chunk);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;             // [G][D]
  float* sc = qs + G * D;     // [G][cmax]
  float* kn = sc + G * cmax;  // [D] the new key row
  __shared__ float ml[2 * 64];
  __shared__ int last;
  const float2* cs = rope + (uint64_t)pos * (D / 2);
  const uint32_t QD = dd.heads * D, KD = dd.kvheads * D;
  float* kc_h = kc + (uint64_t)h * dd.ctx * D;
  float* vc_h = vc + (uint64_t)h * dd.ctx * D;

  for (uint32_t g = warp; g < G; g += nw) {
    for (uint32_t i = lane; i < D; i += 32) qs[g * D + i] = qkv[(h * G + g) * D + i];
    __syncwarp();
    head_norm_rope(qs + g * D, qn_w, D, dd.eps, cs);
  }
  if (t0 <= pos && pos < t1 && warp == nw - 1) {  // model.rs:241-243: append k (normed, rotated) and v
    for (uint32_t i = lane; i < D; i += 32) kn[i] = qkv[QD + h * D + i];
    __syncwarp();
    head_norm_rope(kn, kn_w, D, dd.eps, cs);
    for (uint32_t i = lane; i < D; i += 32) {
      kc_h[(uint64_t)pos * D + i] = kn[i];
      vc_h[(uint64_t)pos * D + i] = qkv[QD + KD + h * D + i];
    }
  }
  __syncthreads();

  // scores s[g][t] = (q_g . k_t) / sqrt(D)  (ops.rs:84-91)
  const float sd = sqrtf((float)D);
  for (uint32_t t = t0 + warp; t < t1; t += nw) {
    const float* kr = kc_h + (uint64_t)t * D;
    float kv[8];
#pragma unroll
    for (int j = 0; j < 8; j++) kv[j] = (lane + 32 * j < D) ? kr[lane + 32 * j] : 0.f;
    for (uint32_t g = 0; g < G; g++) {
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (lane + 32 * j < D) p = fmaf(qs[g * D + lane + 32 * j], kv[j], p);
      p = warp_sum(p);
      if (lane == 0) sc[g * cmax + (t - t0)] = p / sd;
    }
  }
  __syncthreads();
  // partial softmax state per head: m = max, p_t = exp(s_t - m), l = sum p_t
  for (uint32_t g = warp; g < G; g += nw) {
    float m = -INFINITY;
    for (uint32_t t = lane; t < t1 - t0; t += 32) m = fmaxf(m, sc[g * cmax + t]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t t = lane; t < t1 - t0; t += 32) {
      const float p = expf(sc[g * cmax + t] - m);
      sc[g * cmax + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      ml[2 * g] = m;
      ml[2 * g + 1] = l;
    }
  }
  __syncthreads();
  float* pb = part + ((uint64_t)(h * dd.nsplit + s) * G) * (D + 2);
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const uint32_t g = idx / D, d = idx % D;
    float acc = 0.f;
    for (uint32_t t = t0; t < t1; t++) acc = fmaf(sc[g * cmax + (t - t0)], vc_h[(uint64_t)t * D + d], acc);
    pb[g * (D + 2) + d] = acc;
  }
  for (uint32_t g = threadIdx.x; g < G; g += blockDim.x) {
    pb[g * (D + 2) + D] = ml[2 * g];
    pb[g * (D + 2) + D + 1] = ml[2 * g + 1];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&st->attn_done[h], 1u) == active - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge: weights f_k = exp(m_k - M) per (split, head) computed once into shared memory
  const float* ph = part + (uint64_t)h * dd.nsplit * G * (D + 2);
  float* fw = sc;  // [active][G]
  for (uint32_t g = warp; g < G; g += nw) {
    float M = -INFINITY;
    for (uint32_t k = lane; k < active; k += 32) M = fmaxf(M, __ldcg(ph + (k * G + g) * (D + 2) + D));
    M = warp_max(M);
    float L = 0.f;
    for (uint32_t k = lane; k < active; k += 32) {
      const float f = expf(__ldcg(ph + (k * G + g) * (D + 2) + D) - M);
      fw[k * G + g] = f;
      L = fmaf(__ldcg(ph + (k * G + g) * (D + 2) + D + 1), f, L);
    }
    L = warp_sum(L);
    if (lane == 0) ml[g] = 1.f / L;
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const uint32_t g = idx / D, d = idx % D;
    float o = 0.f;
    for (uint32_t k = 0; k < active; k++) o = fmaf(__ldcg(ph + (k * G + g) * (D + 2) + d), fw[k * G + g], o);
    attn[(h * G + g) * D + d] = o * ml[g];
  }
  if (threadIdx.x == 0) st->attn_done[h] = 0;
}

// ---------------------------------------------------------------------------
// x += W_o * attn (model.rs:245-248).
__global__ void __launch_bounds__(NT) k_oproj(MatDesc mo, const float* __restrict__ a, float* __restrict__ x) {
  extern __shared__ __align__(16) uint8_t smem[];
  const RowChunk c = my_rows(mo.rows, 32 / mo.lpr);
  prefetch_rows(mo, 0, c.r0, c.r1);
  pdl_wait();
  pdl_trigger();
  const XView xv = stage_x(smem, mo.cols, mo.units, uses_float_x(mo.kind), [&](uint32_t i) { return a[i]; });
  for_rows(mo, c, [&](uint32_t r, uint32_t lr, bool ok) {
    float p = ok ? row_partial(mo, 0, r, lr, xv) : 0.f;
    p = group_sum(p, mo.lpr);
    if (lr == 0 && ok) x[r] = __fadd_rn(x[r], p);
  });
}

// ---------------------------------------------------------------------------
// Router logits, then (last block) top-k with ties to the lower index and a
// softmax over the kept logits (ops.rs:45-56, 29-44).
__global__ void __launch_bounds__(NT) k_router(MatDesc mr, const float* __restrict__ x, const float* __restrict__ norm,
                                               uint32_t hidden, float eps, uint32_t top, float* __restrict__ rlogit,
                                               uint32_t* __restrict__ sel, float* __restrict__ selw, DevState* st) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  __shared__ int last;
  const RowChunk c = my_rows(mr.rows, 32 / mr.lpr);
  prefetch_rows(mr, 0, c.r0, c.r1);
  pdl_wait();
  pdl_trigger();
  const float s = rms_scale(x, hidden, eps, red);
  const XView xv = stage_x(smem, hidden, mr.units, uses_float_x(mr.kind),
                           [&](uint32_t i) { return __fmul_rn(x[i], __fmul_rn(s, norm[i])); });
  for_rows(mr, c, [&](uint32_t r, uint32_t lr, bool ok) {
    float p = ok ? row_partial(mr, 0, r, lr, xv) : 0.f;
    p = group_sum(p, mr.lpr);
    if (lr == 0 && ok) rlogit[r] = p;
  });
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&st->router_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const uint32_t E = mr.rows;
  unsigned long long* key = reinterpret_cast<unsigned long long*>(smem);  // [E] (reuses the staging space)
  for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) {
    const float v = __ldcg(rlogit + e);
    if (!isfinite(v)) atomicOr(&st->nonfinite, 1u);
    key[e] = ((unsigned long long)total_key_u(v) << 32) | (0xffffffffu - e);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const uint32_t lane = threadIdx.x;
    float kept[64];
    uint32_t ids[64];
    for (uint32_t k = 0; k < top; k++) {
      unsigned long long best = 0ull;
      for (uint32_t e = lane; e < E; e += 32) best = key[e] > best ? key[e] : best;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const uint32_t e = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
      __syncwarp();
      if (lane == 0) key[e] = 0ull;
      __syncwarp();
      ids[k] = e;
      kept[k] = __ldcg(rlogit + e);
    }
    if (lane == 0) {  // ops.rs:29-44, sequential in selection order
      float mx = -INFINITY;
      for (uint32_t k = 0; k < top; k++) mx = fmaxf(mx, kept[k]);
      float sum = 0.f;
      for (uint32_t k = 0; k < top; k++) {
        kept[k] = expf(kept[k] - mx);
        sum = __fadd_rn(sum, kept[k]);
      }
      for (uint32_t k = 0; k < top; k++) {
        sel[k] = ids[k];
        selw[k] = kept[k] / sum;
      }
      st->router_done = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// h[s][r] = silu(gate_e[r] . xn) * (up_e[r] . xn) for the selected experts
// (model.rs:259-274); xn = rms(x, ffn_norm) is recomputed from x.  Block b owns
// a contiguous chunk of the (slot, row group) task space.
__global__ void __launch_bounds__(NT) k_gateup(MatDesc mg, MatDesc mu, const float* __restrict__ x,
                                               const float* __restrict__ norm, uint32_t hidden, float eps,
                                               uint32_t top, const uint32_t* __restrict__ sel,
                                               float* __restrict__ hout) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t I = mg.rows, G = 32 / mg.lpr;
  const uint32_t groups = (I + G - 1) / G;
  const uint32_t tasks = top * groups, per = (tasks + gridDim.x - 1) / gridDim.x;
  const uint32_t t0 = blockIdx.x * per, t1 = min(tasks, t0 + per);
  pdl_wait();
  pdl_trigger();
  for (uint32_t t = t0; t < t1;) {  // prefetch this block's expert rows (sel is ready after the wait)
    const uint32_t s = t / groups, g0 = t % groups, g1 = min(groups, g0 + (t1 - t));
    const uint32_t e = sel[s];
    prefetch_rows(mg, e, g0 * G, min(I, g1 * G));
    prefetch_rows(mu, e, g0 * G, min(I, g1 * G));
    t += g1 - g0;
  }
  const float sc = rms_scale(x, hidden, eps, red);
  const bool fl = uses_float_x(mg.kind) || uses_float_x(mu.kind);
  const XView xv = stage_x(smem, hidden, mg.units, fl, [&](uint32_t i) { return __fmul_rn(x[i], __fmul_rn(sc, norm[i])); });
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, lpr = mg.lpr;
  for (uint32_t t = t0 + warp; t < t1; t += nw) {
    const uint32_t s = t / groups, grp = t % groups, e = sel[s];
    const uint32_t r = grp * G + lane / lpr, lr = lane % lpr;
    float g = 0.f, u = 0.f;
    if (r < I) {
      g = row_partial(mg, e, r, lr, xv);
      u = row_partial(mu, e, r, lr, xv);
    }
    g = group_sum(g, lpr);
    u = group_sum(u, lpr);
    if (lr == 0 && r < I) hout[s * I + r] = __fmul_rn(g / (1.f + expf(-g)), u);
  }
}

// ---------------------------------------------------------------------------
// x[r] += sum_s w_s * (down_{e_s}[r] . h_s), summed in selection order (model.rs:275-287).
// Block b owns a contiguous chunk of row groups; warp w computes slots w, w+8, ...
__global__ void __launch_bounds__(NT) k_down(MatDesc md, const float* __restrict__ hin, uint32_t top,
                                             const uint32_t* __restrict__ sel, const float* __restrict__ selw,
                                             float* __restrict__ x) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t I = md.cols, lpr = md.lpr, G = 32 / lpr, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nw = blockDim.x >> 5;
  const RowChunk c = my_rows(md.rows, G);
  // sel was written by the router two launches back: complete before the previous kernel started its work
  for (uint32_t s = 0; s < top; s++) prefetch_rows(md, __ldcg(sel + s), c.r0, c.r1);
  pdl_wait();
  pdl_trigger();
  const bool fl = uses_float_x(md.kind);
  const uint32_t xb = xview_bytes(md.units, fl);
  XView xs0;
  for (uint32_t s = 0; s < top; s++) {  // one XView per slot; all threads take part in each
    const XView v = stage_x(smem + s * xb, I, md.units, fl, [&](uint32_t i) { return hin[s * I + i]; });
    if (s == 0) xs0 = v;
  }
  float* pp = reinterpret_cast<float*>(smem + top * xb);  // [top][G] partials
  for (uint32_t grp = c.r0; grp < c.r1; grp += G) {
    const uint32_t r = grp + lane / lpr, lr = lane % lpr;
    for (uint32_t s = warp; s < top; s += nw) {
      const uint64_t off = (uint64_t)s * xb;  // the slot's XView is xs0 shifted by s*xb bytes
      XView xv;
      xv.dig = xs0.dig + off;
      xv.sx = reinterpret_cast<const int*>(reinterpret_cast<const uint8_t*>(xs0.sx) + off);
      xv.sb = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(xs0.sb) + off);
      xv.xf = xs0.xf ? reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(xs0.xf) + off) : nullptr;
      float p = r < c.r1 ? row_partial(md, sel[s], r, lr, xv) : 0.f;
      p = group_sum(p, lpr);
      if (lr == 0) pp[s * G + lane / lpr] = p;
    }
    __syncthreads();
    if (threadIdx.x < G) {
      const uint32_t rr = grp + threadIdx.x;
      if (rr < c.r1) {
        float acc = 0.f;
        for (uint32_t s = 0; s < top; s++) acc = __fadd_rn(acc, __fmul_rn(selw[s], pp[s * G + threadIdx.x]));
        x[rr] = __fadd_rn(x[rr], acc);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// logits = W_out * rms(x, output_norm); finiteness flag; greedy argmax (ties to
// the lower index); the last block advances the step state.
__global__ void __launch_bounds__(NT) k_output(MatDesc mo, const float* __restrict__ x, const float* __restrict__ norm,
                                               uint32_t hidden, float eps, float* __restrict__ logits, DevState* st) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  __shared__ int last;
  const RowChunk c = my_rows(mo.rows, 32 / mo.lpr);
  prefetch_rows(mo, 0, c.r0, c.r1);
  pdl_wait();
  pdl_trigger();
  const float s = rms_scale(x, hidden, eps, red);
  const XView xv = stage_x(smem, hidden, mo.units, uses_float_x(mo.kind),
                           [&](uint32_t i) { return __fmul_rn(x[i], __fmul_rn(s, norm[i])); });
  unsigned long long best = 0ull;
  bool bad = false;
  for_rows(mo, c, [&](uint32_t r, uint32_t lr, bool ok) {
    float p = ok ? row_partial(mo, 0, r, lr, xv) : 0.f;
    p = group_sum(p, mo.lpr);
    if (lr == 0 && ok) {
      logits[r] = p;
      bad |= !isfinite(p);
      const unsigned long long key = ((unsigned long long)total_key_u(p) << 32) | (0xffffffffu - r);
      best = key > best ? key : best;
    }
  });
  const uint32_t lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&st->nonfinite, 2u);
  if (lane == 0 && best) atomicMax(&st->best, best);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&st->output_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const unsigned long long b = atomicAdd(&st->best, 0ull);
  const uint32_t idx = 0xffffffffu - (uint32_t)(b & 0xffffffffu);
  st->token = idx;
  st->pos = st->pos + 1;
  st->output_done = 0;
}

// ---------------------------------------------------------------------------
// Launch with programmatic stream serialization (PDL); inside a captured graph
// this becomes a programmatic dependency edge.
template <typename... KArgs, typename... Args>
static void launch(void (*k)(KArgs...), dim3 grid, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

static uint32_t grid_rows(uint32_t rows, uint32_t lpr, int sms, uint32_t per_sm) {
  const uint32_t groups = (rows + 32 / lpr - 1) / (32 / lpr);
  const uint32_t need = (groups + 7) / 8;  // at least one row group per warp
  const uint32_t cap = (uint32_t)sms * per_sm;
  return need < 1 ? 1 : (need < cap ? need : cap);
}

void launch_step(const StepArgs& a, cudaStream_t s, StepHook hook, void* ctx) {
  const DecodeDims& d = a.dims;
  const Scratch& c = a.sc;
  auto H = [&](int kind) {
    if (hook) hook(ctx, kind, s);
  };
  H(K_EMBED);
  launch(k_embed, dim3((d.hidden + NT - 1) / NT), 0, s, a.embd, a.st, c.x, d.vocab);
  const uint32_t G = d.heads / d.kvheads;
  const uint32_t cmax = max(kMinChunk, (d.ctx + d.nsplit - 1) / d.nsplit);
  const size_t attn_smem = (size_t)(G * d.head_dim + G * cmax + d.head_dim) * sizeof(float);
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const LayerDev& L = a.layers[l];
    {
      const bool fl = uses_float_x(L.q.kind) || uses_float_x(L.k.kind) || uses_float_x(L.v.kind);
      const size_t smem = xview_bytes(L.q.units, fl);
      H(K_ATTN_IN);
      launch(k_attn_in, dim3(grid_rows(L.q.rows + L.k.rows + L.v.rows, L.q.lpr, a.sms, 1)), smem, s, L.q, L.k, L.v,
             c.x, L.attn_norm, d.hidden, d.eps, c.qkv);
    }
    H(K_ATTENTION);
    launch(k_attention, dim3(d.kvheads, d.nsplit), attn_smem, s, d, c.qkv, L.q_norm, L.k_norm, L.kc, L.vc, c.rope,
           c.part, c.attn, a.st);
    H(K_OPROJ);
    launch(k_oproj, dim3(grid_rows(L.o.rows, L.o.lpr, a.sms, 1)), xview_bytes(L.o.units, uses_float_x(L.o.kind)), s,
           L.o, c.attn, c.x);
    {
      uint32_t grid = grid_rows(L.router.rows, L.router.lpr, a.sms, 1);
      grid = grid > 32 ? 32 : grid;
      size_t smem = xview_bytes(L.router.units, uses_float_x(L.router.kind));
      const size_t keys = (size_t)L.router.rows * 8;
      smem = smem > keys ? smem : keys;
      H(K_ROUTER);
      launch(k_router, dim3(grid), smem, s, L.router, c.x, L.ffn_norm, d.hidden, d.eps, d.top, c.rlogit, c.sel, c.selw,
             a.st);
    }
    {
      const bool fl = uses_float_x(L.gate.kind) || uses_float_x(L.up.kind);
      const uint32_t Gg = 32 / L.gate.lpr;
      const uint32_t tasks = (L.gate.rows + Gg - 1) / Gg * d.top;
      uint32_t grid = (tasks + 7) / 8;
      grid = grid > (uint32_t)a.sms * 2 ? (uint32_t)a.sms * 2 : grid;
      H(K_GATEUP);
      launch(k_gateup, dim3(grid), xview_bytes(L.gate.units, fl), s, L.gate, L.up, c.x, L.ffn_norm, d.hidden, d.eps,
             d.top, c.sel, c.h);
    }
    {
      const uint32_t Gd = 32 / L.down.lpr;
      const size_t smem = (size_t)d.top * xview_bytes(L.down.units, uses_float_x(L.down.kind)) + (size_t)d.top * Gd * 4;
      const uint32_t groups = (L.down.rows + Gd - 1) / Gd;
      const uint32_t grid = groups < (uint32_t)a.sms * 2 ? groups : (uint32_t)a.sms * 2;
      H(K_DOWN);
      launch(k_down, dim3(grid), smem, s, L.down, c.h, d.top, c.sel, c.selw, c.x);
    }
  }
  H(K_OUTPUT);
  launch(k_output, dim3(grid_rows(a.out.rows, a.out.lpr, a.sms, 4)), xview_bytes(a.out.units, uses_float_x(a.out.kind)),
         s, a.out, c.x, a.out_norm, d.hidden, d.eps, c.logits, a.st);
  H(K_COUNT);
}

cudaError_t decode_prepare(int max_smem) {
  cudaError_t e = cudaSuccess;
#define QC_ATTR(K) \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  QC_ATTR(k_attn_in) QC_ATTR(k_attention) QC_ATTR(k_oproj) QC_ATTR(k_router) QC_ATTR(k_gateup) QC_ATTR(k_down)
  QC_ATTR(k_output)
#undef QC_ATTR
  return e;
}

}  // namespace qc
