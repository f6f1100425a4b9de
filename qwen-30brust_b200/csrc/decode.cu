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
// Every kernel is launched with programmatic stream serialization (PDL).  A
// block first copies the weight rows it owns (and, in attention, the cached
// K/V rows) into shared memory with cp.async — inputs that do not depend on
// the previous kernel — then waits for the previous kernel
// (griddepcontrol.wait), lets the next one launch (launch_dependents), stages
// its activation vector in one pass and computes from shared memory.  The
// weight stream of each kernel thus overlaps the tail of the one before.
#include <algorithm>

#include "kernels.h"

namespace qc {

constexpr int NT = 512;

QC_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QC_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

#ifdef QC_TRACE
// Phase timestamps of block-level progress (diagnostic builds only).
struct TraceRec {
  unsigned long long t[6];
};
__device__ TraceRec g_trace[K_COUNT][1024];
QC_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define QC_TRACE_AT(kind, i)                                                                                   \
  do {                                                                                                         \
    if (threadIdx.x == 0 && blockIdx.y == 0 && blockIdx.x < 1024) g_trace[kind][blockIdx.x].t[i] = gtimer(); \
  } while (0)
#else
#define QC_TRACE_AT(kind, i) \
  do {                       \
  } while (0)
#endif

// Stage RMSNorm(x, w) (n elements) as an XView at mem; ends with __syncthreads().
QC_DEV XView stage_rms(uint8_t* mem, const float* __restrict__ x, const float* __restrict__ w, uint32_t n,
                       uint32_t units, bool with_float, float eps, float* red) {
  stage_vectors<true>(mem, 1, n, units, with_float, [&](uint32_t, uint32_t i) { return x[i]; }, w, eps, red);
  return xview_at(mem, units, with_float);
}

// The part of one matrix (a segment of a concatenated group space) held by a block.
struct Part {
  uint32_t g0, g1;  // groups [g0, g1) of the matrix
  uint32_t off;     // shared-memory byte offset of group g0
};
// Block groups [B0, B1) of a concatenation in which this segment occupies
// [seg_begin, seg_begin + seg_groups); advances *off by the bytes taken.
QC_DEV Part take_part(uint32_t seg_begin, uint32_t seg_groups, uint32_t B0, uint32_t B1, uint32_t group_bytes,
                      uint32_t* off) {
  const uint32_t lo = max(B0, seg_begin), hi = min(B1, seg_begin + seg_groups);
  Part p;
  p.g0 = lo - seg_begin;
  p.g1 = hi > lo ? hi - seg_begin : p.g0;
  p.off = *off;
  *off += (p.g1 - p.g0) * group_bytes;
  return p;
}
QC_DEV void copy_part(uint8_t* smem, const MatDesc& m, uint32_t e, const Part& p) {
  copy_groups(smem + p.off, m, e, p.g0, p.g1);
}
// All warps over the rows of a part held in shared memory; emit(r, sum).
template <class Emit>
QC_DEV void part_rows(const MatDesc& m, const Part& p, const uint8_t* smem, const XView& xv, Emit emit) {
  const uint32_t r0 = p.g0 * 8, r1 = min(m.rows, p.g1 * 8);
  if (r1 > r0) warp_rows<true>(m, r0, r1, xv, SmemRows{&m, smem + p.off, r0}, emit);
}

// ---------------------------------------------------------------------------
// Embedding row, dequantized exactly as gguf.rs:204-213 (model.rs:225).
// Block 0 records the token fed at this step in gen_tokens (the greedy sequence
// when steps are chained on the device) and clears the argmax slot.
__global__ void k_embed(const __grid_constant__ MatDesc embd, DevState* st, float* __restrict__ x, uint32_t vocab) {
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
  const uint8_t* row = row_ptr(embd, embd.w, tok);
  const __half* drow = drow_ptr(embd, embd.w, tok);
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < embd.cols; c += gridDim.x * blockDim.x)
    x[c] = dequant_one(embd, row, drow, c);
}

// ---------------------------------------------------------------------------
// Q, K, V = W_{q,k,v} * rms(x).  The row groups of Q, K and V form one group
// space; block b owns groups [b*gper, (b+1)*gper) of it.
__global__ void __launch_bounds__(NT) k_attn_in(const __grid_constant__ MatDesc mq, const __grid_constant__ MatDesc mk,
                                                const __grid_constant__ MatDesc mv, const float* __restrict__ x,
                                                const float* __restrict__ norm, uint32_t hidden, float eps,
                                                float* __restrict__ out, uint32_t gper, uint32_t wbytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t gq = (mq.rows + 7) / 8, gk = (mk.rows + 7) / 8, gv = (mv.rows + 7) / 8;
  const uint32_t B0 = min(gq + gk + gv, blockIdx.x * gper), B1 = min(gq + gk + gv, B0 + gper);
  uint32_t off = 0;
  const Part pq = take_part(0, gq, B0, B1, mq.group_bytes, &off);
  const Part pk = take_part(gq, gk, B0, B1, mk.group_bytes, &off);
  const Part pv = take_part(gq + gk, gv, B0, B1, mv.group_bytes, &off);
  copy_part(smem, mq, 0, pq);
  copy_part(smem, mk, 0, pk);
  copy_part(smem, mv, 0, pv);
  cp_commit();
  QC_TRACE_AT(K_ATTN_IN, 0);
  pdl_wait();
  pdl_trigger();
  QC_TRACE_AT(K_ATTN_IN, 1);
  const bool fl = uses_float_x(mq.kind) || uses_float_x(mk.kind) || uses_float_x(mv.kind);
  const XView xv = stage_rms(smem + wbytes, x, norm, hidden, mq.units, fl, eps, red);
  QC_TRACE_AT(K_ATTN_IN, 2);
  cp_wait_all();
  __syncthreads();
  QC_TRACE_AT(K_ATTN_IN, 3);
  part_rows(mq, pq, smem, xv, [&](uint32_t r, float v) { out[r] = v; });
  part_rows(mk, pk, smem, xv, [&](uint32_t r, float v) { out[mq.rows + r] = v; });
  part_rows(mv, pv, smem, xv, [&](uint32_t r, float v) { out[mq.rows + mk.rows + r] = v; });
  QC_TRACE_AT(K_ATTN_IN, 4);
}

// Split GQA decode attention.  Block (h, s) owns KV head h and positions
// [s*chunk, (s+1)*chunk) of [0, pos], chunk = max(kMinChunk, ceil((pos+1)/nsplit));
// it handles the G query heads of that KV head.  The cached K/V rows of its
// range are copied to shared memory (rows padded to D+4 floats) before the
// wait; the block whose range holds `pos` computes and appends the new K/V row.
// Scores: one thread per (position, head) dot product; values: one thread per
// (head, 4 dims).  With one split the block writes the output directly;
// otherwise the last active block of head h merges the partial softmax states.
__global__ void __launch_bounds__(NT) k_attention(DecodeDims dd, const float* __restrict__ qkv,
                                                  const float* __restrict__ qn_w, const float* __restrict__ kn_w,
                                                  float* __restrict__ kc, float* __restrict__ vc,
                                                  const float2* __restrict__ rope, float* __restrict__ part,
                                                  float* __restrict__ attn, DevState* st) {
  const uint32_t h = blockIdx.x, s = blockIdx.y, D = dd.head_dim, G = dd.heads / dd.kvheads, KP = D + 4;
  // pos is written only by the last kernel of a step, so it is final before this step's first kernel
  const uint32_t pos = st->pos, time = pos + 1;
  uint32_t chunk = (time + dd.nsplit - 1) / dd.nsplit;
  chunk = chunk < kMinChunk ? kMinChunk : chunk;
  const uint32_t active = (time + chunk - 1) / chunk;
  const uint32_t cmax = attn_cmax(dd);
  const uint32_t t0 = s * chunk, t1 = min(time, t0 + chunk);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  extern __shared__ __align__(16) float sm[];
  float* ks = sm;              // [cmax][KP] cached keys of the range
  float* vs = ks + cmax * KP;  // [cmax][KP] cached values
  float* qs = vs + cmax * KP;  // [G][KP]
  float* sc = qs + G * KP;     // [G][cmax]
  float* kn = sc + G * cmax;   // [D] the new key row
  __shared__ float ml[2 * 64];
  __shared__ int last;
  float* kc_h = kc + (uint64_t)h * dd.ctx * D;
  float* vc_h = vc + (uint64_t)h * dd.ctx * D;
  const bool act = s < active;
  if (act) {  // rows written by earlier steps: [t0, min(t1, pos)), 16-byte granules into padded rows
    const uint32_t te = min(t1, pos), gpr = D / 4;
    for (uint32_t i = threadIdx.x; i < (te > t0 ? te - t0 : 0) * gpr; i += blockDim.x) {
      const uint32_t t = i / gpr, j = i % gpr;
      cp16(ks + t * KP + 4 * j, kc_h + (uint64_t)(t0 + t) * D + 4 * j);
      cp16(vs + t * KP + 4 * j, vc_h + (uint64_t)(t0 + t) * D + 4 * j);
    }
    cp_commit();
  }
  QC_TRACE_AT(K_ATTENTION, 0);
  pdl_wait();
  pdl_trigger();
  QC_TRACE_AT(K_ATTENTION, 1);
  if (!act) return;
  const float2* cs = rope + (uint64_t)pos * (D / 2);
  const uint32_t QD = dd.heads * D, KD = dd.kvheads * D;
  for (uint32_t g = warp; g < G; g += nw) {
    for (uint32_t i = lane; i < D; i += 32) qs[g * KP + i] = qkv[(h * G + g) * D + i];
    __syncwarp();
    head_norm_rope(qs + g * KP, qn_w, D, dd.eps, cs);
  }
  if (t0 <= pos && pos < t1 && warp == nw - 1) {  // model.rs:241-243: append k (normed, rotated) and v
    for (uint32_t i = lane; i < D; i += 32) kn[i] = qkv[QD + h * D + i];
    __syncwarp();
    head_norm_rope(kn, kn_w, D, dd.eps, cs);
    for (uint32_t i = lane; i < D; i += 32) {
      const float v = qkv[QD + KD + h * D + i];
      kc_h[(uint64_t)pos * D + i] = kn[i];
      vc_h[(uint64_t)pos * D + i] = v;
      ks[(pos - t0) * KP + i] = kn[i];
      vs[(pos - t0) * KP + i] = v;
    }
  }
  QC_TRACE_AT(K_ATTENTION, 2);
  cp_wait_all();
  __syncthreads();
  QC_TRACE_AT(K_ATTENTION, 3);

  // scores s[g][t] = (q_g . k_t) / sqrt(D)  (ops.rs:84-91); thread per (t, g), t fastest
  const float sd = sqrtf((float)D);
  const uint32_t n = t1 - t0;
  for (uint32_t i = threadIdx.x; i < n * G; i += blockDim.x) {
    const uint32_t t = i % n, g = i / n;
    const float4* kr = reinterpret_cast<const float4*>(ks + t * KP);
    const float4* qr = reinterpret_cast<const float4*>(qs + g * KP);
    float p = 0.f;
    for (uint32_t j = 0; j < D / 4; j++) {
      const float4 a = kr[j], b = qr[j];
      p = fmaf(a.x, b.x, p);
      p = fmaf(a.y, b.y, p);
      p = fmaf(a.z, b.z, p);
      p = fmaf(a.w, b.w, p);
    }
    sc[g * cmax + t] = p / sd;
  }
  __syncthreads();
  // partial softmax state per head: m = max, p_t = exp(s_t - m), l = sum p_t
  for (uint32_t g = warp; g < G; g += nw) {
    float m = -INFINITY;
    for (uint32_t t = lane; t < n; t += 32) m = fmaxf(m, sc[g * cmax + t]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t t = lane; t < n; t += 32) {
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
  // acc[g][d..d+3] = sum_t p[g][t] v_t[d..d+3]; thread per (g, 4 dims)
  float* pb = part + ((uint64_t)(h * dd.nsplit + s) * G) * (D + 2);
  for (uint32_t i = threadIdx.x; i < G * (D / 4); i += blockDim.x) {
    const uint32_t g = i / (D / 4), d4 = i % (D / 4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t t = 0; t < n; t++) {
      const float p = sc[g * cmax + t];
      const float4 v = *reinterpret_cast<const float4*>(vs + t * KP + 4 * d4);
      acc.x = fmaf(p, v.x, acc.x);
      acc.y = fmaf(p, v.y, acc.y);
      acc.z = fmaf(p, v.z, acc.z);
      acc.w = fmaf(p, v.w, acc.w);
    }
    if (active == 1) {  // single split: normalize and write the output directly
      const float inv = 1.f / ml[2 * g + 1];
      float* o = attn + (h * G + g) * D + 4 * d4;
      o[0] = acc.x * inv;
      o[1] = acc.y * inv;
      o[2] = acc.z * inv;
      o[3] = acc.w * inv;
    } else {
      float* o = pb + g * (D + 2) + 4 * d4;
      o[0] = acc.x;
      o[1] = acc.y;
      o[2] = acc.z;
      o[3] = acc.w;
    }
  }
  QC_TRACE_AT(K_ATTENTION, 4);
  if (active == 1) return;
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
    float mk[2], lk[2];
    float M = -INFINITY;
    for (uint32_t k = lane; k < active; k += 32) M = fmaxf(M, __ldcg(ph + (k * G + g) * (D + 2) + D));
    M = warp_max(M);
    float L = 0.f;
    for (uint32_t k = lane; k < active; k += 32) {
      mk[0] = __ldcg(ph + (k * G + g) * (D + 2) + D);
      lk[0] = __ldcg(ph + (k * G + g) * (D + 2) + D + 1);
      const float f = expf(mk[0] - M);
      fw[k * G + g] = f;
      L = fmaf(lk[0], f, L);
    }
    L = warp_sum(L);
    if (lane == 0) ml[g] = 1.f / L;
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const uint32_t g = idx / D, d = idx % D;
    float o = 0.f;
#pragma unroll 8
    for (uint32_t k = 0; k < active; k++) o = fmaf(__ldcg(ph + (k * G + g) * (D + 2) + d), fw[k * G + g], o);
    attn[(h * G + g) * D + d] = o * ml[g];
  }
  if (threadIdx.x == 0) st->attn_done[h] = 0;
  QC_TRACE_AT(K_ATTENTION, 5);
}

// ---------------------------------------------------------------------------
// x += W_o * attn (model.rs:245-248).
__global__ void __launch_bounds__(NT) k_oproj(const __grid_constant__ MatDesc mo, const float* __restrict__ a,
                                              float* __restrict__ x, uint32_t gper, uint32_t wbytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t groups = (mo.rows + 7) / 8;
  uint32_t off = 0;
  const Part p = take_part(0, groups, min(groups, blockIdx.x * gper), min(groups, blockIdx.x * gper + gper),
                           mo.group_bytes, &off);
  copy_part(smem, mo, 0, p);
  cp_commit();
  pdl_wait();
  pdl_trigger();
  const bool fl = uses_float_x(mo.kind);
  stage_vectors<false>(smem + wbytes, 1, mo.cols, mo.units, fl, [&](uint32_t, uint32_t i) { return a[i]; }, nullptr,
                       0.f, red);
  const XView xv = xview_at(smem + wbytes, mo.units, fl);
  cp_wait_all();
  __syncthreads();
  part_rows(mo, p, smem, xv, [&](uint32_t r, float v) { x[r] = __fadd_rn(x[r], v); });
}

// ---------------------------------------------------------------------------
// Router logits, then (last block) top-k with ties to the lower index and a
// softmax over the kept logits (ops.rs:45-56, 29-44).
__global__ void __launch_bounds__(NT) k_router(const __grid_constant__ MatDesc mr, const float* __restrict__ x,
                                               const float* __restrict__ norm, uint32_t hidden, float eps, uint32_t top,
                                               float* __restrict__ rlogit, uint32_t* __restrict__ sel,
                                               float* __restrict__ selw, DevState* st, uint32_t gper, uint32_t wbytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  __shared__ int last;
  const uint32_t groups = (mr.rows + 7) / 8;
  uint32_t off = 0;
  const Part p = take_part(0, groups, min(groups, blockIdx.x * gper), min(groups, blockIdx.x * gper + gper),
                           mr.group_bytes, &off);
  copy_part(smem, mr, 0, p);
  cp_commit();
  QC_TRACE_AT(K_ROUTER, 0);
  pdl_wait();
  pdl_trigger();
  QC_TRACE_AT(K_ROUTER, 1);
  const XView xv = stage_rms(smem + wbytes, x, norm, hidden, mr.units, uses_float_x(mr.kind), eps, red);
  QC_TRACE_AT(K_ROUTER, 2);
  cp_wait_all();
  __syncthreads();
  QC_TRACE_AT(K_ROUTER, 3);
  part_rows(mr, p, smem, xv, [&](uint32_t r, float v) { rlogit[r] = v; });
  QC_TRACE_AT(K_ROUTER, 4);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&st->router_done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const uint32_t E = mr.rows;
  // keys and logits in shared memory (reusing the staging space): [E] u64 then [E] f32
  unsigned long long* key = reinterpret_cast<unsigned long long*>(smem + wbytes);
  float* lg = reinterpret_cast<float*>(key + E);
  for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) {
    const float v = __ldcg(rlogit + e);
    if (!isfinite(v)) atomicOr(&st->nonfinite, 1u);
    lg[e] = v;
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
      kept[k] = lg[e];
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
      QC_TRACE_AT(K_ROUTER, 5);
    }
  }
}

// ---------------------------------------------------------------------------
// h[s][r] = silu(gate_e[r] . xn) * (up_e[r] . xn) for the selected experts
// (model.rs:259-274); xn = rms(x, ffn_norm) is recomputed from x.  Block b
// serves slot b / bpe and row groups [(b % bpe) * gper, ...) of its expert.
__global__ void __launch_bounds__(NT) k_gateup(const __grid_constant__ MatDesc mg, const __grid_constant__ MatDesc mu,
                                               const float* __restrict__ x, const float* __restrict__ norm,
                                               uint32_t hidden, float eps, const uint32_t* __restrict__ sel,
                                               float* __restrict__ hout, uint32_t bpe, uint32_t gper, uint32_t wbytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t I = mg.rows, groups = (I + 7) / 8;
  const uint32_t slot = blockIdx.x / bpe, j = blockIdx.x % bpe;
  const uint32_t B0 = min(groups, j * gper), B1 = min(groups, B0 + gper);
  uint32_t off = 0;
  const Part pg = take_part(0, groups, B0, B1, mg.group_bytes, &off);
  const Part pu = take_part(0, groups, B0, B1, mu.group_bytes, &off);
  QC_TRACE_AT(K_GATEUP, 0);
  pdl_wait();  // the router (previous kernel) writes sel
  pdl_trigger();
  QC_TRACE_AT(K_GATEUP, 1);
  const uint32_t e = sel[slot];
  copy_part(smem, mg, e, pg);
  copy_part(smem, mu, e, pu);
  cp_commit();
  const bool fl = uses_float_x(mg.kind) || uses_float_x(mu.kind);
  const XView xv = stage_rms(smem + wbytes, x, norm, hidden, mg.units, fl, eps, red);
  QC_TRACE_AT(K_GATEUP, 2);
  cp_wait_all();
  __syncthreads();
  QC_TRACE_AT(K_GATEUP, 3);
  // gate and up partial sums to shared memory, then SwiGLU
  float* gu = reinterpret_cast<float*>(smem + wbytes + xview_bytes(mg.units, fl));  // [2][8*gper]
  const uint32_t r0 = B0 * 8, nr = 8 * gper;
  part_rows(mg, pg, smem, xv, [&](uint32_t r, float v) { gu[r - r0] = v; });
  part_rows(mu, pu, smem, xv, [&](uint32_t r, float v) { gu[nr + r - r0] = v; });
  __syncthreads();
  for (uint32_t r = r0 + threadIdx.x; r < min(I, B1 * 8); r += blockDim.x) {
    const float g = gu[r - r0], u = gu[nr + r - r0];
    hout[slot * I + r] = __fmul_rn(g / (1.f + expf(-g)), u);
  }
  QC_TRACE_AT(K_GATEUP, 4);
}

// ---------------------------------------------------------------------------
// x[r] += sum_s w_s * (down_{e_s}[r] . h_s), summed in selection order (model.rs:275-287).
// Block b owns row groups [b*gper, (b+1)*gper) of all selected experts; warp w
// computes slots w, w+nw, ... of them.
__global__ void __launch_bounds__(NT) k_down(const __grid_constant__ MatDesc md, const float* __restrict__ hin,
                                             uint32_t top, const uint32_t* __restrict__ sel,
                                             const float* __restrict__ selw, float* __restrict__ x, uint32_t gper,
                                             uint32_t wbytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  const uint32_t I = md.cols, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, groups = (md.rows + 7) / 8;
  const uint32_t B0 = min(groups, blockIdx.x * gper), B1 = min(groups, B0 + gper);
  const uint32_t pbytes = (B1 - B0) * md.group_bytes;
  QC_TRACE_AT(K_DOWN, 0);
  // sel was written by the router two launches back: final before the previous kernel started its work
  for (uint32_t s = 0; s < top; s++) copy_groups(smem + s * pbytes, md, __ldcg(sel + s), B0, B1);
  cp_commit();
  pdl_wait();
  pdl_trigger();
  QC_TRACE_AT(K_DOWN, 1);
  const bool fl = uses_float_x(md.kind);
  const uint32_t xb = xview_bytes(md.units, fl);
  uint8_t* xmem = smem + wbytes;
  stage_vectors<false>(xmem, top, I, md.units, fl, [&](uint32_t s, uint32_t i) { return hin[s * I + i]; }, nullptr,
                       0.f, red);
  const uint32_t r0 = B0 * 8, r1 = min(md.rows, B1 * 8), nr = 8 * gper;
  float* pp = reinterpret_cast<float*>(xmem + top * xb);  // [top][8*gper] partials
  QC_TRACE_AT(K_DOWN, 2);
  cp_wait_all();
  __syncthreads();
  QC_TRACE_AT(K_DOWN, 3);
  {  // warps split evenly over the slots (nw a multiple of top) or take slots in turn
    const uint32_t per = nw >= top ? nw / top : 1;
    for (uint32_t s = warp / per; s < top; s += nw / per) {
      const XView xv = xview_at(xmem + s * xb, md.units, fl);
      warp_rows<true>(md, r0, r1, xv, SmemRows{&md, smem + s * pbytes, r0},
                      [&](uint32_t r, float v) { pp[s * nr + r - r0] = v; }, warp % per, per);
    }
  }
  __syncthreads();
  for (uint32_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    float acc = 0.f;
    for (uint32_t s = 0; s < top; s++) acc = __fadd_rn(acc, __fmul_rn(selw[s], pp[s * nr + r - r0]));
    x[r] = __fadd_rn(x[r], acc);
  }
  QC_TRACE_AT(K_DOWN, 4);
}

// ---------------------------------------------------------------------------
// logits = W_out * rms(x, output_norm); finiteness flag; greedy argmax (ties to
// the lower index); the last block advances the step state.  The block's rows
// stream through shared memory in stages of `sg` groups (kOutStages deep).
constexpr int kOutStages = 3;

__global__ void __launch_bounds__(NT) k_output(const __grid_constant__ MatDesc mo, const float* __restrict__ x,
                                               const float* __restrict__ norm, uint32_t hidden, float eps,
                                               float* __restrict__ logits, DevState* st, uint32_t sg) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[32];
  __shared__ int last;
  __shared__ unsigned long long wbest[NT / 32];
  __shared__ int wbad[NT / 32];
  const uint32_t groups = (mo.rows + 7) / 8;
  const uint32_t per = (groups + gridDim.x - 1) / gridDim.x;
  const uint32_t g0 = min(groups, blockIdx.x * per), g1 = min(groups, g0 + per);
  const uint32_t nst = (g1 - g0 + sg - 1) / sg;
  const uint64_t stage_bytes = (uint64_t)sg * mo.group_bytes;
  for (uint32_t k = 0; k < kOutStages - 1; k++) {
    if (k < nst) copy_groups(smem + (k % kOutStages) * stage_bytes, mo, 0, g0 + k * sg, min(g1, g0 + (k + 1) * sg));
    cp_commit();
  }
  pdl_wait();
  pdl_trigger();
  const XView xv = stage_rms(smem + kOutStages * stage_bytes, x, norm, hidden, mo.units, uses_float_x(mo.kind), eps, red);
  const uint32_t lane = threadIdx.x & 31;
  unsigned long long best = 0ull;
  bool bad = false;
  for (uint32_t k = 0; k < nst; k++) {
    const uint32_t kn = k + kOutStages - 1;
    if (kn < nst)
      copy_groups(smem + (kn % kOutStages) * stage_bytes, mo, 0, g0 + kn * sg, min(g1, g0 + (kn + 1) * sg));
    cp_commit();
    cp_wait<kOutStages - 1>();
    __syncthreads();
    const uint8_t* sb = smem + (k % kOutStages) * stage_bytes;
    const uint32_t r0 = (g0 + k * sg) * 8, r1 = min(mo.rows, min(g1, g0 + (k + 1) * sg) * 8);
    warp_rows<true>(mo, r0, r1, xv, SmemRows{&mo, sb, r0}, [&](uint32_t r, float p) {
      logits[r] = p;
      bad |= !isfinite(p);
      const unsigned long long key = ((unsigned long long)total_key_u(p) << 32) | (0xffffffffu - r);
      best = key > best ? key : best;
    });
    __syncthreads();
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  const int anybad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    wbest[threadIdx.x >> 5] = best;
    wbad[threadIdx.x >> 5] = anybad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // one atomic per block
    unsigned long long b = 0ull;
    int bb = 0;
    for (uint32_t w = 0; w < blockDim.x / 32; w++) {
      b = wbest[w] > b ? wbest[w] : b;
      bb |= wbad[w];
    }
    if (bb) atomicOr(&st->nonfinite, 2u);
    if (b) atomicMax(&st->best, b);
    __threadfence();
    last = atomicAdd(&st->output_done, 1u) == gridDim.x - 1;
  }
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

// Blocks and groups per block so that each block's weights fit in `budget` bytes
// and the grid covers about `blocks` blocks.
struct Split {
  uint32_t grid, gper;
};
static Split split_groups(uint32_t groups, uint32_t group_bytes, uint32_t blocks, uint32_t budget) {
  uint32_t gper = (groups + blocks - 1) / blocks;
  const uint32_t cap = budget / group_bytes;
  if (gper > cap) gper = cap < 1 ? 1 : cap;
  if (gper < 1) gper = 1;
  return {(groups + gper - 1) / gper, gper};
}

// Router, gate/up and down splits (the MoE kernels).
static void plan_moe_part(StepPlan& p, const DecodeDims& d, const LayerDev& L, uint32_t sms) {
  {
    const Split s = split_groups((L.router.rows + 7) / 8, L.router.group_bytes, sms, kWeightBudget);
    p.router = {s.grid, s.gper, s.gper * L.router.group_bytes};
  }
  {  // gate/up: bpe blocks per selected expert
    const uint32_t groups = (L.gate.rows + 7) / 8, gb = L.gate.group_bytes + L.up.group_bytes;
    const uint32_t per_expert = std::max(1u, (2 * sms + d.top - 1) / d.top);
    const Split s = split_groups(groups, gb, per_expert, kWeightBudget);
    p.gateup = {s.grid * d.top, s.gper, s.gper * gb};
    p.gateup_bpe = s.grid;
  }
  {  // down: row groups of all selected experts
    const uint32_t gb = L.down.group_bytes * d.top;
    const Split s = split_groups((L.down.rows + 7) / 8, gb, sms, kWeightBudget);
    p.down = {s.grid, s.gper, s.gper * gb};
  }
}

StepPlan plan_moe(const DecodeDims& d, const LayerDev& L, int sms) {
  StepPlan p{};
  plan_moe_part(p, d, L, (uint32_t)sms);
  return p;
}

StepPlan plan_step(const StepArgs& a) {
  StepPlan p{};
  const DecodeDims& d = a.dims;
  const uint32_t sms = (uint32_t)a.sms;
  const LayerDev& L = a.layers[0];
  {  // attn_in: the group space of Q, K and V
    const uint32_t gb = std::max(L.q.group_bytes, std::max(L.k.group_bytes, L.v.group_bytes));
    const uint32_t groups = (L.q.rows + 7) / 8 + (L.k.rows + 7) / 8 + (L.v.rows + 7) / 8;
    const Split s = split_groups(groups, gb, sms, kWeightBudget);
    p.attn_in = {s.grid, s.gper, s.gper * gb};
  }
  {
    const Split s = split_groups((L.o.rows + 7) / 8, L.o.group_bytes, sms, kWeightBudget);
    p.oproj = {s.grid, s.gper, s.gper * L.o.group_bytes};
  }
  plan_moe_part(p, d, L, sms);
  {
    const uint32_t sg = std::max(1u, std::min(8u, kOutStageBudget / a.out.group_bytes));
    p.out_sg = sg;
    p.out_grid = std::min<uint32_t>(sms, ((a.out.rows + 7) / 8 + sg - 1) / sg);
  }
  return p;
}

// Dynamic shared memory of each kernel.
static size_t smem_attn_in(const LayerDev& L, const StepPlan& p) {
  return p.attn_in.wbytes +
         xview_bytes(L.q.units, uses_float_x(L.q.kind) || uses_float_x(L.k.kind) || uses_float_x(L.v.kind));
}
static size_t smem_oproj(const LayerDev& L, const StepPlan& p) {
  return p.oproj.wbytes + xview_bytes(L.o.units, uses_float_x(L.o.kind));
}
static size_t smem_router(const LayerDev& L, const StepPlan& p) {
  return p.router.wbytes + std::max<size_t>(xview_bytes(L.router.units, uses_float_x(L.router.kind)), L.router.rows * 12);
}
static size_t smem_gateup(const LayerDev& L, const StepPlan& p) {
  return p.gateup.wbytes + xview_bytes(L.gate.units, uses_float_x(L.gate.kind) || uses_float_x(L.up.kind)) +
         2 * 8 * p.gateup.gper * sizeof(float);
}
static size_t smem_down(const LayerDev& L, const StepPlan& p, uint32_t top) {
  return p.down.wbytes + top * xview_bytes(L.down.units, uses_float_x(L.down.kind)) + top * 8 * p.down.gper * sizeof(float);
}
static size_t smem_output(const StepArgs& a, const StepPlan& p) {
  return (size_t)kOutStages * p.out_sg * a.out.group_bytes + xview_bytes(a.out.units, uses_float_x(a.out.kind));
}

size_t step_smem_max(const StepArgs& a, const StepPlan& p) {
  const LayerDev& L = a.layers[0];
  size_t m = std::max(smem_attn_in(L, p), smem_oproj(L, p));
  m = std::max(m, std::max(smem_router(L, p), smem_gateup(L, p)));
  m = std::max(m, std::max(smem_down(L, p, a.dims.top), attn_smem(a.dims)));
  return std::max(m, smem_output(a, p));
}

void launch_step(const StepArgs& a, const StepPlan& p, cudaStream_t s, StepHook hook, void* ctx) {
  const DecodeDims& d = a.dims;
  const Scratch& c = a.sc;
  auto H = [&](int kind) {
    if (hook) hook(ctx, kind, s);
  };
  H(K_EMBED);
  launch(k_embed, dim3((d.hidden + NT - 1) / NT), 0, s, a.embd, a.st, c.x, d.vocab);
  for (uint32_t l = 0; l < a.n_layers; l++) {
    const LayerDev& L = a.layers[l];
    H(K_ATTN_IN);
    launch(k_attn_in, dim3(p.attn_in.grid), smem_attn_in(L, p), s, L.q, L.k, L.v, c.x, L.attn_norm, d.hidden, d.eps,
           c.qkv, p.attn_in.gper, p.attn_in.wbytes);
    H(K_ATTENTION);
    launch(k_attention, dim3(d.kvheads, d.nsplit), attn_smem(d), s, d, c.qkv, L.q_norm, L.k_norm, L.kc, L.vc, c.rope,
           c.part, c.attn, a.st);
    H(K_OPROJ);
    launch(k_oproj, dim3(p.oproj.grid), smem_oproj(L, p), s, L.o, c.attn, c.x, p.oproj.gper, p.oproj.wbytes);
    H(K_ROUTER);
    launch(k_router, dim3(p.router.grid), smem_router(L, p), s, L.router, c.x, L.ffn_norm, d.hidden, d.eps, d.top,
           c.rlogit, c.sel, c.selw, a.st, p.router.gper, p.router.wbytes);
    H(K_GATEUP);
    launch(k_gateup, dim3(p.gateup.grid), smem_gateup(L, p), s, L.gate, L.up, c.x, L.ffn_norm, d.hidden, d.eps, c.sel,
           c.h, p.gateup_bpe, p.gateup.gper, p.gateup.wbytes);
    H(K_DOWN);
    launch(k_down, dim3(p.down.grid), smem_down(L, p, d.top), s, L.down, c.h, d.top, c.sel, c.selw, c.x, p.down.gper,
           p.down.wbytes);
  }
  H(K_OUTPUT);
  launch(k_output, dim3(p.out_grid), smem_output(a, p), s, a.out, c.x, a.out_norm, d.hidden, d.eps, c.logits, a.st,
         p.out_sg);
  H(K_COUNT);
}

void launch_moe_token(const DecodeDims& d, const StepPlan& p, const LayerDev& L, const Scratch& c, DevState* st,
                      cudaStream_t s) {
  launch(k_router, dim3(p.router.grid), smem_router(L, p), s, L.router, c.x, L.ffn_norm, d.hidden, d.eps, d.top,
         c.rlogit, c.sel, c.selw, st, p.router.gper, p.router.wbytes);
  launch(k_gateup, dim3(p.gateup.grid), smem_gateup(L, p), s, L.gate, L.up, c.x, L.ffn_norm, d.hidden, d.eps, c.sel,
         c.h, p.gateup_bpe, p.gateup.gper, p.gateup.wbytes);
  launch(k_down, dim3(p.down.grid), smem_down(L, p, d.top), s, L.down, c.h, d.top, c.sel, c.selw, c.x, p.down.gper,
         p.down.wbytes);
}

#ifdef QC_TRACE
cudaError_t trace_read(void* host, size_t bytes) { return cudaMemcpyFromSymbol(host, g_trace, bytes); }
#endif

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
