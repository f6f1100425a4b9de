// The MoE half of a layer (model.rs:245-287) for a batch of T tokens at once, on the 5th-generation
// tensor cores.
//
//   k_moe_route    per token: RMSNorm(ffn_norm), router matvec (F16), top-k with ties to the lower
//                  index, softmax over the kept logits in selection order (ops.rs:3-15, 29-56)
//   k_moe_plan     the (token, slot) pairs grouped by expert, tokens ascending within an expert
//   k_qg_image     the gate/up activation image: each expert's tokens' normalized inputs
//   k_qgemm (pair) per (expert, 64 gate + 64 up rows): the expert's rows times its tokens' inputs,
//                  then SwiGLU  g / (1 + exp(-g)) * u  (model.rs:259-274) into the down image
//   k_qgemm        per (expert, 128 down rows): down rows times the expert's SwiGLU outputs
//   k_moe_combine  x + (w_0 y_0 + w_1 y_1 + ...) in selection order (model.rs:275-287)
//
// The GEMMs run on the tensor-core kernel of qgemm.cu (exact K-quant integer operands, one TMEM
// accumulator per super-block): gate/up as one GEMM over 128-row tiles of 64 gate + 64 up rows with
// the SwiGLU epilogue writing the down GEMM's activation image, then down.  Each expert's pairs are
// a group of the GEMM; k_moe_plan writes the groups and the rows of the gate/up activation image.
#include <cuda_fp16.h>

#include "kernels.h"

namespace qc {
namespace {

// ---- per-token routing ---------------------------------------------------------------------
// Block (t, g): RMSNorm of token t (every block of the token computes it; block g = 0 keeps it, with
// its power-of-two scale), then the router logits of experts 16 g .. 16 g + 15 into rlg[t][e].
constexpr uint32_t kRouteRows = 16;
__global__ void __launch_bounds__(256) k_moe_route(MoeArgs a, const float* __restrict__ x) {
  __shared__ float red[32];
  extern __shared__ __align__(16) float hsm[];  // [H] the normalized input, for the router rows
  const uint32_t t = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* xr = x + (uint64_t)t * a.H;
  float ss = 0.f;
  for (uint32_t i = tid; i < a.H; i += 256) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
  ss = block_sum(ss, red);
  // ops.rs:3-15: s = 1 / sqrt(sum / n + eps); x_i * (s * w_i)
  const float s = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.H), a.eps)));
  float* hr = a.h + (uint64_t)t * a.H;
  float mx = 0.f;
  for (uint32_t i = tid; i < a.H; i += 256) {
    const float v = __fmul_rn(xr[i], __fmul_rn(s, a.ffn_norm[i]));
    if (g == 0) hr[i] = v;
    hsm[i] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  __syncthreads();
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0 && g == 0) {
    float m = 0.f;
    for (int w = 0; w < 8; w++) m = fmaxf(m, red[w]);
    a.hscale[t] = qg_pow2_scale(m);
  }
  // router logits: one warp per expert row (F16), 16-byte loads of 8 weights per lane
  const uint32_t e1 = min(a.E, (g + 1) * kRouteRows);
  for (uint32_t e = g * kRouteRows + warp; e < e1; e += 8) {
    const uint4* wr = reinterpret_cast<const uint4*>(row_ptr(a.router, a.router.w, e));
    float acc = 0.f, acc2 = 0.f;
    for (uint32_t c = lane; c < a.H / 8; c += 32) {
      const uint4 v = ldg16(wr + c);
      const float4 h0 = *reinterpret_cast<const float4*>(hsm + 8 * c), h1 = *reinterpret_cast<const float4*>(hsm + 8 * c + 4);
      const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&v.x)),
                   w1 = __half22float2(*reinterpret_cast<const __half2*>(&v.y)),
                   w2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z)),
                   w3 = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
      acc = fmaf(w0.x, h0.x, acc);
      acc2 = fmaf(w0.y, h0.y, acc2);
      acc = fmaf(w1.x, h0.z, acc);
      acc2 = fmaf(w1.y, h0.w, acc2);
      acc = fmaf(w2.x, h1.x, acc);
      acc2 = fmaf(w2.y, h1.y, acc2);
      acc = fmaf(w3.x, h1.z, acc);
      acc2 = fmaf(w3.y, h1.w, acc2);
    }
    acc = warp_sum(acc + acc2);
    if (lane == 0) {
      a.rlg[(uint64_t)t * a.E + e] = acc;
      if (!isfinite(acc)) atomicOr(a.err, 1u);
    }
  }
}

// Token t: the rank of each logit (ties to the lower index) gives the selection in order, then
// ops.rs:29-44 (softmax) over the kept logits in selection order.
__global__ void __launch_bounds__(128) k_moe_select(MoeArgs a) {
  __shared__ float lg[1024];
  const uint32_t t = blockIdx.x, tid = threadIdx.x;
  for (uint32_t e = tid; e < a.E; e += 128) lg[e] = a.rlg[(uint64_t)t * a.E + e];
  __syncthreads();
  for (uint32_t e = tid; e < a.E; e += 128) {
    const uint32_t ke = total_key_u(lg[e]);
    uint32_t rank = 0;
    for (uint32_t j = 0; j < a.E; j++) {
      const uint32_t kj = total_key_u(lg[j]);
      rank += kj > ke || (kj == ke && j < e);
    }
    if (rank < a.top) a.sel[(uint64_t)t * a.top + rank] = e;
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t* sl = a.sel + (uint64_t)t * a.top;
    float* w = a.selw + (uint64_t)t * a.top;
    float m = -INFINITY;
    for (uint32_t k = 0; k < a.top; k++) m = fmaxf(m, lg[sl[k]]);
    float sum = 0.f;
    for (uint32_t k = 0; k < a.top; k++) {
      w[k] = expf(__fsub_rn(lg[sl[k]], m));
      sum = __fadd_rn(sum, w[k]);
    }
    for (uint32_t k = 0; k < a.top; k++) w[k] = __fdiv_rn(w[k], sum);
  }
}

// ---- pairs grouped by expert, and the two GEMMs' groups -----------------------------------------
// Expert e's pairs are rows imgoff_e .. imgoff_e + nimg_e of the activation images (nimg_e = its pair
// count rounded up to 16); its gate/up group has ceil(I / 64) tiles and its down group ceil(H / 128),
// each times ceil(nimg_e / NP) passes.
__global__ void __launch_bounds__(1024) k_moe_plan(MoeArgs a) {
  __shared__ uint32_t cnt[1024], off[1025], igu[1025], idn[1025], img[1025];
  const uint32_t tid = threadIdx.x, P = a.T * a.top, lane = tid & 31, warp = tid >> 5;
  for (uint32_t e = tid; e < a.E; e += 1024) cnt[e] = 0;
  __syncthreads();
  for (uint32_t p = tid; p < P; p += 1024) atomicAdd(&cnt[a.sel[p]], 1u);
  __syncthreads();
  if (tid == 0) {
    const uint32_t tgu = (a.I + 63) / 64, tdn = (a.H + 127) / 128;
    off[0] = igu[0] = idn[0] = img[0] = 0;
    for (uint32_t e = 0; e < a.E; e++) {
      const uint32_t c = cnt[e], n = (c + 15) & ~15u;
      off[e + 1] = off[e] + c;
      img[e + 1] = img[e] + n;
      igu[e + 1] = igu[e] + tgu * ((n + a.NPgu - 1) / a.NPgu);
      idn[e + 1] = idn[e] + tdn * ((n + a.NPdn - 1) / a.NPdn);
    }
    a.nitems[0] = igu[a.E];
    a.nitems[1] = idn[a.E];
    *a.nrows = img[a.E];
  }
  __syncthreads();
  for (uint32_t e = tid; e < a.E; e += 1024) {
    a.cnt[e] = cnt[e];
    a.off[e] = off[e];
    const uint32_t n = (cnt[e] + 15) & ~15u;
    a.groups[e] = QgGroup{igu[e], cnt[e], n, img[e], 0, e, nullptr, nullptr, nullptr, a.ptok + off[e], 0};
    a.groups[a.E + e] = QgGroup{idn[e], cnt[e], n, img[e], 0, e, a.y, nullptr, a.ppair + off[e], nullptr, a.H};
  }
  // (the order of an expert's pairs does not change any result: each is its own GEMM column; the
  // loop above handles expert e in the same thread, so the count can be reset here)
  for (uint32_t e = tid; e < a.E; e += 1024) cnt[e] = 0;
  __syncthreads();
  for (uint32_t p = tid; p < P; p += 1024) {
    const uint32_t e = a.sel[p];
    const uint32_t pos = off[e] + atomicAdd(&cnt[e], 1u);
    a.ptok[pos] = p / a.top;
    a.ppair[pos] = p;
  }
  __syncthreads();
  for (uint32_t e = warp; e < a.E; e += 32) {  // image rows: source token, or none past the pairs
    const uint32_t c = off[e + 1] - off[e], n = (c + 15) & ~15u;
    for (uint32_t i = lane; i < n; i += 32)
      a.imgrows[img[e] + i] = make_uint4(i < c ? a.ptok[off[e] + i] : 0xffffffffu, img[e], n, 0);
  }
}

// ---- combine in selection order + residual ---------------------------------------------------
__global__ void __launch_bounds__(256) k_moe_combine(MoeArgs a, const float* __restrict__ x, float* __restrict__ out) {
  const uint32_t t = blockIdx.x;
  for (uint32_t r = threadIdx.x; r < a.H; r += 256) {
    float acc = 0.f;
    for (uint32_t k = 0; k < a.top; k++) {
      const uint32_t p = t * a.top + k;
      acc = __fadd_rn(acc, __fmul_rn(a.selw[p], a.y[(uint64_t)p * a.H + r]));
    }
    out[(uint64_t)t * a.H + r] = __fadd_rn(x[(uint64_t)t * a.H + r], acc);
  }
}

}  // namespace

const char* moe_tc_supported(const MoeArgs& a) {
  if (a.gate.kind != a.up.kind) return "the tensor-core MoE path needs gate and up rows of one format";
  if (const char* why = qgemm_supported(a.gate.kind, a.H)) return why;
  if (const char* why = qgemm_supported(a.down.kind, a.I)) return why;
  if (a.I % 64) return "the tensor-core MoE path needs an intermediate size in multiples of 64";
  if (a.router.kind != F16) return "the batched MoE path takes an F16 router";
  if (a.E > 1024) return "the batched MoE path takes at most 1024 experts";
  if (!a.ggate.w || !a.gup.w || !a.gdown.w) return "the GEMM-layout copy of the experts is missing";
  uint32_t np, ss;
  if (const char* why = qgemm_shape(a.gate.kind, a.H, a.gate.kind == Q4_K, &np, &ss)) return why;
  if (const char* why = qgemm_shape(a.down.kind, a.I, a.down.kind == Q4_K, &np, &ss)) return why;
  return nullptr;
}

uint32_t moe_image_rows(uint32_t T, uint32_t top, uint32_t E) {
  const uint32_t P = T * top;
  return P + 15 * (E < P ? E : P);
}

const char* launch_moe_tc(const MoeArgs& a, const float* x, float* out, cudaStream_t s) {
  const uint32_t rmax = moe_image_rows(a.T, a.top, a.E);
  k_moe_route<<<dim3(a.T, (a.E + kRouteRows - 1) / kRouteRows), 256, a.H * sizeof(float), s>>>(a, x);
  k_moe_select<<<a.T, 128, 0, s>>>(a);
  k_moe_plan<<<1, 1024, 0, s>>>(a);
  QgImageArgs ia{};
  ia.x = a.h;
  ia.xstride = a.H;
  ia.K = a.H;
  ia.rows = a.imgrows;
  ia.nrows = a.nrows;
  ia.hs_in = a.hscale;
  ia.hasmin = a.gate.kind == Q4_K;
  ia.img = a.img_gu;
  launch_qg_image(ia, rmax, s);
  QgArgs g{};
  g.mats[0] = a.ggate;
  g.mats[1] = a.gup;
  g.smin[0] = a.smin_g;
  g.smin[1] = a.smin_u;
  g.pair = 1;
  g.K = a.H;
  g.NP = a.NPgu;
  g.SS = a.SSgu;
  g.img_hasmin = a.gate.kind == Q4_K;
  g.img = a.img_gu;
  g.hs = a.hscale;
  g.groups = a.groups;
  g.ngroups = a.E;
  g.nitems_dev = a.nitems;
  g.img2 = a.img_dn;
  g.K2 = a.I;
  g.img2_hasmin = a.down.kind == Q4_K;
  g.err = a.err;
  launch_qgemm(g, a.gate.kind, true, a.sms, s);
  QgArgs d{};
  d.mats[0] = a.gdown;
  d.smin[0] = a.smin_d;
  d.K = a.I;
  d.NP = a.NPdn;
  d.SS = a.SSdn;
  d.img_hasmin = a.down.kind == Q4_K;
  d.img = a.img_dn;
  d.groups = a.groups + a.E;
  d.ngroups = a.E;
  d.nitems_dev = a.nitems + 1;
  d.err = a.err;
  launch_qgemm(d, a.down.kind, false, a.sms, s);
  k_moe_combine<<<a.T, 256, 0, s>>>(a, x, out);
  return nullptr;
}

}  // namespace qc
