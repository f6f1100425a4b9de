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
#include "kernels.h"

namespace qc {

constexpr int NT = 256;

// xs[i] = x[i] * (s * w[i]) with s = 1/sqrt(mean(x^2) + eps) (reference ops.rs:3-15), zero padded.
QC_DEV void stage_rms(float* xs, const float* __restrict__ x, const float* __restrict__ w, uint32_t n, uint32_t padded,
                      float eps, float* red) {
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float s = 1.0f / sqrtf(ss / (float)n + eps);
  for (uint32_t i = threadIdx.x; i < padded; i += blockDim.x) xs[i] = i < n ? __fmul_rn(x[i], __fmul_rn(s, w[i])) : 0.f;
  __syncthreads();
}

QC_DEV void stage_copy(float* xs, const float* __restrict__ x, uint32_t n, uint32_t padded) {
  for (uint32_t i = threadIdx.x; i < padded; i += blockDim.x) xs[i] = i < n ? x[i] : 0.f;
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Embedding row, dequantized exactly as gguf.rs:204-213 (model.rs:225).
// Block 0 also records the token fed at this step in gen_tokens (the greedy
// sequence when steps are chained on the device) and clears the argmax slot.
__global__ void k_embed(MatDesc embd, DevState* st, float* __restrict__ x, uint32_t vocab) {
  uint32_t tok = st->token;
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    if (st->gen_tokens && st->gen_count < st->gen_cap) st->gen_tokens[st->gen_count] = tok;
    st->gen_count = st->gen_count + 1;
  }
  if (tok >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) st->bad_token = 1;
    tok = 0;
  }
  const uint8_t* row = embd.w + (uint64_t)tok * embd.row_stride;
  const __half* drow = embd.d ? embd.d + (uint64_t)tok * embd.d_stride : nullptr;
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < embd.cols; c += gridDim.x * blockDim.x)
    x[c] = dequant_one(embd, row, drow, c);
  if (blockIdx.x == 0 && threadIdx.x == 0) st->best = 0ull;
}

// ---------------------------------------------------------------------------
// Q, K, V = W_{q,k,v} * rms(x); rows of the three matrices form one task space.
__global__ void __launch_bounds__(NT) k_attn_in(MatDesc mq, MatDesc mk, MatDesc mv, const float* __restrict__ x,
                                                const float* __restrict__ norm, uint32_t hidden, uint32_t padded,
                                                float eps, float* __restrict__ out) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  stage_rms(xs, x, norm, hidden, padded, eps, red);
  const uint32_t lpr = mq.lpr, G = 32 / lpr, lane = threadIdx.x & 31;
  const uint32_t gq = (mq.rows + G - 1) / G, gk = (mk.rows + G - 1) / G, gv = (mv.rows + G - 1) / G;
  const uint32_t total = gq + gk + gv, wpb = blockDim.x >> 5;
  for (uint32_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < total; t += gridDim.x * wpb) {
    const MatDesc* m;
    uint32_t grp, off;
    if (t < gq) { m = &mq; grp = t; off = 0; }
    else if (t < gq + gk) { m = &mk; grp = t - gq; off = mq.rows; }
    else { m = &mv; grp = t - gq - gk; off = mq.rows + mk.rows; }
    const uint32_t r = grp * G + lane / lpr, lr = lane % lpr;
    float p = r < m->rows ? row_partial(*m, 0, r, lr, xs) : 0.f;
    p = group_sum(p, lpr);
    if (lr == 0 && r < m->rows) out[off + r] = p;
  }
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

// Split GQA decode attention.  Block (h, s) owns KV head h and time range s of
// [0, pos]; it handles the G query heads of that KV head.  The block whose
// range holds `pos` appends the new K/V row.  The last block of head h merges
// the nsplit partial softmax states.
__global__ void __launch_bounds__(NT) k_attention(DecodeDims dd, const float* __restrict__ qkv,
                                                  const float* __restrict__ qn_w, const float* __restrict__ kn_w,
                                                  float* __restrict__ kc, float* __restrict__ vc,
                                                  const float2* __restrict__ rope, float* __restrict__ part,
                                                  float* __restrict__ attn, DevState* st) {
  const uint32_t h = blockIdx.x, s = blockIdx.y, D = dd.head_dim, G = dd.heads / dd.kvheads;
  const uint32_t pos = st->pos, time = pos + 1;
  const uint32_t chunk = (time + dd.nsplit - 1) / dd.nsplit, cmax = (dd.ctx + dd.nsplit - 1) / dd.nsplit;
  const uint32_t t0 = min(time, s * chunk), t1 = min(time, t0 + chunk);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;            // [G][D]
  float* sc = qs + G * D;    // [G][cmax]
  float* kn = sc + G * cmax; // [D] the new key row
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
  if (threadIdx.x == 0) last = atomicAdd(&st->attn_done[h], 1u) == dd.nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* ph = part + (uint64_t)h * dd.nsplit * G * (D + 2);
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const uint32_t g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (uint32_t k = 0; k < dd.nsplit; k++) M = fmaxf(M, __ldcg(ph + (k * G + g) * (D + 2) + D));
    float L = 0.f, o = 0.f;
    for (uint32_t k = 0; k < dd.nsplit; k++) {
      const float* q = ph + (k * G + g) * (D + 2);
      const float l = __ldcg(q + D + 1);
      if (l == 0.f) continue;  // empty split
      const float f = expf(__ldcg(q + D) - M);
      L = fmaf(l, f, L);
      o = fmaf(__ldcg(q + d), f, o);
    }
    attn[(h * G + g) * D + d] = o / L;
  }
  if (threadIdx.x == 0) st->attn_done[h] = 0;
}

// ---------------------------------------------------------------------------
// x += W_o * attn (model.rs:245-248).
__global__ void __launch_bounds__(NT) k_oproj(MatDesc mo, const float* __restrict__ a, uint32_t padded,
                                              float* __restrict__ x) {
  extern __shared__ __align__(16) float xs[];
  stage_copy(xs, a, mo.cols, padded);
  const uint32_t lpr = mo.lpr, G = 32 / lpr, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const uint32_t total = (mo.rows + G - 1) / G;
  for (uint32_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < total; t += gridDim.x * wpb) {
    const uint32_t r = t * G + lane / lpr, lr = lane % lpr;
    float p = r < mo.rows ? row_partial(mo, 0, r, lr, xs) : 0.f;
    p = group_sum(p, lpr);
    if (lr == 0 && r < mo.rows) x[r] = __fadd_rn(x[r], p);
  }
}

// ---------------------------------------------------------------------------
// Router logits, then (last block) top-k with ties to the lower index and a
// softmax over the kept logits (ops.rs:45-56, 29-44).
__global__ void __launch_bounds__(NT) k_router(MatDesc mr, const float* __restrict__ x, const float* __restrict__ norm,
                                               uint32_t hidden, uint32_t padded, float eps, uint32_t top,
                                               float* __restrict__ xn, float* __restrict__ rlogit,
                                               uint32_t* __restrict__ sel, float* __restrict__ selw, DevState* st) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  __shared__ int last;
  __shared__ uint8_t taken[1024];
  stage_rms(xs, x, norm, hidden, padded, eps, red);
  if (blockIdx.x == 0)
    for (uint32_t i = threadIdx.x; i < hidden; i += blockDim.x) xn[i] = xs[i];
  const uint32_t lpr = mr.lpr, G = 32 / lpr, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const uint32_t total = (mr.rows + G - 1) / G;
  for (uint32_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < total; t += gridDim.x * wpb) {
    const uint32_t r = t * G + lane / lpr, lr = lane % lpr;
    float p = r < mr.rows ? row_partial(mr, 0, r, lr, xs) : 0.f;
    p = group_sum(p, lpr);
    if (lr == 0 && r < mr.rows) rlogit[r] = p;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&st->router_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const uint32_t E = mr.rows;
  for (uint32_t i = threadIdx.x; i < E; i += blockDim.x) taken[i] = 0;
  __syncthreads();
  if (threadIdx.x < 32) {
    __shared__ float kept[64];
    for (uint32_t k = 0; k < top; k++) {
      unsigned long long best = 0ull;
      for (uint32_t e = lane; e < E; e += 32) {
        if (taken[e]) continue;
        const float v = __ldcg(rlogit + e);
        if (k == 0 && !isfinite(v)) atomicOr(&st->nonfinite, 1u);
        const unsigned long long key = ((unsigned long long)total_key_u(v) << 32) | (0xffffffffu - e);
        best = key > best ? key : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const uint32_t e = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
      if (lane == 0) {
        taken[e] = 1;
        sel[k] = e;
        kept[k] = __ldcg(rlogit + e);
      }
      __syncwarp();
    }
    if (lane == 0) {  // ops.rs:29-44, sequential in selection order
      float mx = -INFINITY;
      for (uint32_t k = 0; k < top; k++) mx = fmaxf(mx, kept[k]);
      float sum = 0.f;
      for (uint32_t k = 0; k < top; k++) {
        kept[k] = expf(kept[k] - mx);
        sum = __fadd_rn(sum, kept[k]);
      }
      for (uint32_t k = 0; k < top; k++) selw[k] = kept[k] / sum;
      st->router_done = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// h[s][r] = silu(gate_e[r] . xn) * (up_e[r] . xn) for the selected experts (model.rs:259-274).
__global__ void __launch_bounds__(NT) k_gateup(MatDesc mg, MatDesc mu, const float* __restrict__ xn, uint32_t hidden,
                                               uint32_t padded, uint32_t top, const uint32_t* __restrict__ sel,
                                               float* __restrict__ hout) {
  extern __shared__ __align__(16) float xs[];
  stage_copy(xs, xn, hidden, padded);
  const uint32_t lpr = mg.lpr, G = 32 / lpr, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const uint32_t I = mg.rows, groups = (I + G - 1) / G, total = groups * top;
  for (uint32_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < total; t += gridDim.x * wpb) {
    const uint32_t s = t / groups, grp = t % groups, e = sel[s];
    const uint32_t r = grp * G + lane / lpr, lr = lane % lpr;
    float g = 0.f, u = 0.f;
    if (r < I) {
      g = row_partial(mg, e, r, lr, xs);
      u = row_partial(mu, e, r, lr, xs);
    }
    g = group_sum(g, lpr);
    u = group_sum(u, lpr);
    if (lr == 0 && r < I) hout[s * I + r] = __fmul_rn(g / (1.f + expf(-g)), u);
  }
}

// ---------------------------------------------------------------------------
// x[r] += sum_s w_s * (down_{e_s}[r] . h_s), summed in selection order (model.rs:275-287).
// Block b owns rows [b*G, b*G+G); warp w computes slots w, w+8, ...
__global__ void __launch_bounds__(NT) k_down(MatDesc md, const float* __restrict__ hin, uint32_t padded, uint32_t top,
                                             const uint32_t* __restrict__ sel, const float* __restrict__ selw,
                                             float* __restrict__ x) {
  extern __shared__ __align__(16) float hs[];  // [top][padded] then [top][G] partials
  const uint32_t I = md.cols, lpr = md.lpr, G = 32 / lpr, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nw = blockDim.x >> 5;
  for (uint32_t i = threadIdx.x; i < top * padded; i += blockDim.x) {
    const uint32_t s = i / padded, c = i % padded;
    hs[i] = c < I ? hin[s * I + c] : 0.f;
  }
  __syncthreads();
  float* pp = hs + top * padded;
  const uint32_t groups = (md.rows + G - 1) / G;
  for (uint32_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const uint32_t r = grp * G + lane / lpr, lr = lane % lpr;
    for (uint32_t s = warp; s < top; s += nw) {
      float p = r < md.rows ? row_partial(md, sel[s], r, lr, hs + s * padded) : 0.f;
      p = group_sum(p, lpr);
      if (lr == 0) pp[s * G + lane / lpr] = p;
    }
    __syncthreads();
    if (threadIdx.x < G) {
      const uint32_t rr = grp * G + threadIdx.x;
      if (rr < md.rows) {
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
                                               uint32_t hidden, uint32_t padded, float eps,
                                               float* __restrict__ logits, DevState* st) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[32];
  __shared__ int last;
  stage_rms(xs, x, norm, hidden, padded, eps, red);
  const uint32_t lpr = mo.lpr, G = 32 / lpr, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
  const uint32_t total = (mo.rows + G - 1) / G;
  unsigned long long best = 0ull;
  bool bad = false;
  for (uint32_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < total; t += gridDim.x * wpb) {
    const uint32_t r = t * G + lane / lpr, lr = lane % lpr;
    float p = r < mo.rows ? row_partial(mo, 0, r, lr, xs) : 0.f;
    p = group_sum(p, lpr);
    if (lr == 0 && r < mo.rows) {
      logits[r] = p;
      bad |= !isfinite(p);
      const unsigned long long key = ((unsigned long long)total_key_u(p) << 32) | (0xffffffffu - r);
      best = key > best ? key : best;
    }
  }
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
static uint32_t padded_of(const MatDesc& m) { return m.units * unit_elems(m.kind); }

static uint32_t grid_for(uint32_t tasks_warps, int sms) {
  const uint32_t need = (tasks_warps + 7) / 8;
  const uint32_t cap = (uint32_t)sms * 4;
  return need < 1 ? 1 : (need < cap ? need : cap);
}

void launch_step(const StepArgs& a, cudaStream_t s, StepHook hook, void* ctx) {
  const DecodeDims& d = a.dims;
  const Scratch& c = a.sc;
  auto H = [&](int kind) {
    if (hook) hook(ctx, kind, s);
  };
  H(K_EMBED);
  k_embed<<<(d.hidden + NT - 1) / NT, NT, 0, s>>>(a.embd, a.st, c.x, d.vocab);
  const uint32_t G = d.heads / d.kvheads;
  const uint32_t cmax = (d.ctx + d.nsplit - 1) / d.nsplit;
  const size_t attn_smem = (size_t)(G * d.head_dim + G * cmax + d.head_dim) * sizeof(float);
  float* qkv = c.qkv;
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const LayerDev& L = a.layers[l];
    {
      uint32_t pad = padded_of(L.q);
      pad = pad > padded_of(L.k) ? pad : padded_of(L.k);
      pad = pad > padded_of(L.v) ? pad : padded_of(L.v);
      const uint32_t Gq = 32 / L.q.lpr;
      const uint32_t warps = (L.q.rows + Gq - 1) / Gq + (L.k.rows + Gq - 1) / Gq + (L.v.rows + Gq - 1) / Gq;
      H(K_ATTN_IN);
      k_attn_in<<<grid_for(warps, a.sms), NT, pad * sizeof(float), s>>>(L.q, L.k, L.v, c.x, L.attn_norm, d.hidden,
                                                                         pad, d.eps, qkv);
    }
    H(K_ATTENTION);
    k_attention<<<dim3(d.kvheads, d.nsplit), NT, attn_smem, s>>>(d, qkv, L.q_norm, L.k_norm, L.kc, L.vc, c.rope,
                                                                 c.part, c.attn, a.st);
    {
      const uint32_t pad = padded_of(L.o), Go = 32 / L.o.lpr;
      H(K_OPROJ);
      k_oproj<<<grid_for((L.o.rows + Go - 1) / Go, a.sms), NT, pad * sizeof(float), s>>>(L.o, c.attn, pad, c.x);
    }
    {
      const uint32_t pad = padded_of(L.router), Gr = 32 / L.router.lpr;
      const uint32_t warps = (L.router.rows + Gr - 1) / Gr;
      uint32_t grid = (warps + 7) / 8;
      if (grid > 32) grid = 32;
      H(K_ROUTER);
      k_router<<<grid, NT, pad * sizeof(float), s>>>(L.router, c.x, L.ffn_norm, d.hidden, pad, d.eps, d.top, c.xn,
                                                      c.rlogit, c.sel, c.selw, a.st);
    }
    {
      uint32_t pad = padded_of(L.gate);
      pad = pad > padded_of(L.up) ? pad : padded_of(L.up);
      const uint32_t Gg = 32 / L.gate.lpr;
      const uint32_t warps = (L.gate.rows + Gg - 1) / Gg * d.top;
      H(K_GATEUP);
      k_gateup<<<grid_for(warps, a.sms), NT, pad * sizeof(float), s>>>(L.gate, L.up, c.xn, d.hidden, pad, d.top,
                                                                        c.sel, c.h);
    }
    {
      const uint32_t pad = padded_of(L.down), Gd = 32 / L.down.lpr;
      const uint32_t groups = (L.down.rows + Gd - 1) / Gd;
      const size_t smem = ((size_t)d.top * pad + (size_t)d.top * Gd) * sizeof(float);
      H(K_DOWN);
      k_down<<<groups, NT, smem, s>>>(L.down, c.h, pad, d.top, c.sel, c.selw, c.x);
    }
  }
  {
    const uint32_t pad = padded_of(a.out), Go = 32 / a.out.lpr;
    const uint32_t warps = (a.out.rows + Go - 1) / Go;
    H(K_OUTPUT);
    k_output<<<grid_for(warps, a.sms), NT, pad * sizeof(float), s>>>(a.out, c.x, a.out_norm, d.hidden, pad, d.eps,
                                                                      c.logits, a.st);
  }
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
