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
  __shared__ uint32_t key[1024];  // total-order keys of the logits, computed once
  const uint32_t t = blockIdx.x, tid = threadIdx.x;
  for (uint32_t e = tid; e < a.E; e += 128) {
    lg[e] = a.rlg[(uint64_t)t * a.E + e];
    key[e] = total_key_u(lg[e]);
  }
  __syncthreads();
  for (uint32_t e = tid; e < a.E; e += 128) {
    const uint32_t ke = key[e];
    uint32_t rank = 0;
    for (uint32_t j = 0; j < a.E; j++) {
      const uint32_t kj = key[j];
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
// Only pairs of the experts the weights hold ([e_lo, e_lo + e_n)) are planned; group expert ids are
// relative to e_lo.
__global__ void __launch_bounds__(1024) k_moe_plan(MoeArgs a) {
  __shared__ uint32_t cnt[1024], off[1025], igu[1025], idn[1025], img[1025];
  const uint32_t tid = threadIdx.x, P = a.T * a.top, lane = tid & 31, warp = tid >> 5;
  const uint32_t elo = a.e_n ? a.e_lo : 0, en = a.e_n ? a.e_n : a.E;
  auto held = [&](uint32_t e) { return e - elo < en; };
  for (uint32_t e = tid; e < a.E; e += 1024) cnt[e] = 0;
  __syncthreads();
  for (uint32_t p = tid; p < P; p += 1024) {
    const uint32_t e = a.sel[p];
    if (held(e)) atomicAdd(&cnt[e], 1u);
  }
  __syncthreads();
  {  // per expert (thread e; E <= 1024): pairs, image rows, gate/up and down items, scanned together
    __shared__ uint4 wsum[32];
    const uint32_t tgu = (a.I + 63) / 64, tdn = (a.H + 127) / 128;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (tid < a.E) {
      const uint32_t c = cnt[tid], n = (c + 15) & ~15u;
      v = make_uint4(c, n, tgu * ((n + a.NPgu - 1) / a.NPgu), tdn * ((n + a.NPdn - 1) / a.NPdn));
    }
    auto scan = [&](uint4 x) {  // inclusive over the warp's lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint4 y = make_uint4(__shfl_up_sync(0xffffffffu, x.x, o), __shfl_up_sync(0xffffffffu, x.y, o),
                                   __shfl_up_sync(0xffffffffu, x.z, o), __shfl_up_sync(0xffffffffu, x.w, o));
        if (lane >= (uint32_t)o) x = make_uint4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
      }
      return x;
    };
    uint4 inc = scan(v);
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {  // the warps' totals, exclusive
      const uint4 w = wsum[lane], wi = scan(w);
      wsum[lane] = make_uint4(wi.x - w.x, wi.y - w.y, wi.z - w.z, wi.w - w.w);
    }
    __syncthreads();
    const uint4 base = wsum[warp];
    inc = make_uint4(inc.x + base.x, inc.y + base.y, inc.z + base.z, inc.w + base.w);
    if (tid < a.E) {
      off[tid + 1] = inc.x;
      img[tid + 1] = inc.y;
      igu[tid + 1] = inc.z;
      idn[tid + 1] = inc.w;
    }
    if (tid == 0) off[0] = img[0] = igu[0] = idn[0] = 0;
    if (tid == a.E - 1) {
      a.nitems[0] = inc.z;
      a.nitems[1] = inc.w;
      *a.nrows = inc.y;
    }
  }
  __syncthreads();
  for (uint32_t e = tid; e < a.E; e += 1024) {
    a.cnt[e] = cnt[e];
    a.off[e] = off[e];
    const uint32_t n = (cnt[e] + 15) & ~15u;
    const uint32_t le = held(e) ? e - elo : 0;
    a.groups[e] = QgGroup{igu[e], cnt[e], n, img[e], 0, le, nullptr, nullptr, nullptr, a.ptok + off[e], 0};
    a.groups[a.E + e] = QgGroup{idn[e], cnt[e], n, img[e], 0, le, a.y, nullptr, a.ppair + off[e], nullptr, a.H};
  }
  // (the order of an expert's pairs does not change any result: each is its own GEMM column; the
  // loop above handles expert e in the same thread, so the count can be reset here)
  for (uint32_t e = tid; e < a.E; e += 1024) cnt[e] = 0;
  __syncthreads();
  for (uint32_t p = tid; p < P; p += 1024) {
    const uint32_t e = a.sel[p];
    if (!held(e)) continue;
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
// Block (t, c): elements 1024 c .. 1024 c + 1023 of token t, four per thread (H is a multiple of 4).
__global__ void __launch_bounds__(256) k_moe_combine(MoeArgs a, const float* __restrict__ x, float* __restrict__ out) {
  const uint32_t t = blockIdx.x, r = blockIdx.y * 256 + threadIdx.x;
  if (r >= a.H / 4) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t k = 0; k < a.top; k++) {
    const uint32_t p = t * a.top + k;
    const float w = a.selw[p];
    const float4 y = reinterpret_cast<const float4*>(a.y)[(uint64_t)p * (a.H / 4) + r];
    acc.x = __fadd_rn(acc.x, __fmul_rn(w, y.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(w, y.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(w, y.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(w, y.w));
  }
  const float4 xv = reinterpret_cast<const float4*>(x)[(uint64_t)t * (a.H / 4) + r];
  reinterpret_cast<float4*>(out)[(uint64_t)t * (a.H / 4) + r] =
      make_float4(__fadd_rn(xv.x, acc.x), __fadd_rn(xv.y, acc.y), __fadd_rn(xv.z, acc.z), __fadd_rn(xv.w, acc.w));
}

// ---- expert parallelism: barriers, gather, combine across the ranks' exchange regions ---------------
// Peer data is read with ld.global.cv (fetched again, never a stale cached line); the barrier flags
// with system-scope release / acquire.
__device__ __forceinline__ unsigned long long ep_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Rank `rank` passes barrier `seq`: this layer's T into its header, then flags[rank] = seq in every
// rank's region, after a system-scope fence (the earlier kernels' writes of h, hs, sel or y first).
__global__ void k_ep_signal(MoeEp ep, unsigned long long seq) {
  if (threadIdx.x != 0) return;
  *reinterpret_cast<volatile uint32_t*>(ep.peers[ep.rank] + ep.o_hdr) = ep.T;
  __threadfence_system();
  for (uint32_t q = 0; q < ep.world; q++) {
    unsigned long long* f = reinterpret_cast<unsigned long long*>(ep.peers[q] + ep.o_flags) + ep.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
}

// Waits until every rank has passed barrier `seq` (lane q polls flags[q] of this rank's region), at
// most 2 s; then err bit 3 and no further waiting (a barrier that timed out stays failed until the
// host has read the error).
__global__ void k_ep_wait(MoeEp ep, unsigned long long seq, uint32_t* err) {
  const uint32_t q = threadIdx.x;
  if (q >= ep.world) return;
  const unsigned long long* f = reinterpret_cast<const unsigned long long*>(ep.peers[ep.rank] + ep.o_flags) + q;
  const unsigned long long t0 = ep_now();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
    if (v >= seq) return;
    if (*reinterpret_cast<volatile uint32_t*>(err) & 8u) return;
    if (ep_now() - t0 > 2000000000ull) {
      atomicOr(err, 8u);
      return;
    }
    __nanosleep(200);
  }
}

// Block g = (rank q, token t): token t of rank q becomes global token g of this rank's scratch (its
// normalized input, scale and selected experts).  Block 0 checks every rank's T.
__global__ void __launch_bounds__(256) k_ep_gather(MoeArgs a, MoeEp ep) {
  const uint32_t g = blockIdx.x, q = g / ep.T, t = g % ep.T, tid = threadIdx.x;
  const uint8_t* src = ep.peers[q];
  if (g == 0 && tid < ep.world && __ldcv(reinterpret_cast<const unsigned int*>(ep.peers[tid] + ep.o_hdr)) != ep.T)
    atomicOr(a.err, 16u);
  const float4* hs = reinterpret_cast<const float4*>(src + ep.o_h) + (uint64_t)t * (a.H / 4);
  float4* hd = reinterpret_cast<float4*>(a.h) + (uint64_t)g * (a.H / 4);
  for (uint32_t i = tid; i < a.H / 4; i += 256) hd[i] = __ldcv(hs + i);
  if (tid == 0) a.hscale[g] = __ldcv(reinterpret_cast<const float*>(src + ep.o_hs) + t);
  if (tid < a.top)
    a.sel[(uint64_t)g * a.top + tid] = __ldcv(reinterpret_cast<const unsigned int*>(src + ep.o_sel) + (uint64_t)t * a.top + tid);
}

// x + (w_0 y_0 + w_1 y_1 + ...) in selection order for this rank's token t, each y read from the rank
// that holds the expert (model.rs:275-287).  Block (t, c): elements 1024 c .. 1024 c + 1023.
__global__ void __launch_bounds__(256) k_moe_combine_ep(MoeArgs a, MoeEp ep, const float* __restrict__ x,
                                                        float* __restrict__ out) {
  const uint32_t t = blockIdx.x, g = ep.rank * ep.T + t;
  const uint32_t* sl = reinterpret_cast<const uint32_t*>(ep.peers[ep.rank] + ep.o_sel) + (uint64_t)t * a.top;
  for (uint32_t r = blockIdx.y * 256 + threadIdx.x; r < min(a.H / 4, (blockIdx.y + 1) * 256); r += 256) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t k = 0; k < a.top; k++) {
      const uint32_t e = sl[k];
      const float w = a.selw[(uint64_t)t * a.top + k];
      const float4 y = __ldcv(reinterpret_cast<const float4*>(ep.peers[e / ep.e_n] + ep.o_y) +
                              ((uint64_t)g * a.top + k) * (a.H / 4) + r);
      acc.x = __fadd_rn(acc.x, __fmul_rn(w, y.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w, y.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w, y.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w, y.w));
    }
    const float4 xv = reinterpret_cast<const float4*>(x)[(uint64_t)t * (a.H / 4) + r];
    reinterpret_cast<float4*>(out)[(uint64_t)t * (a.H / 4) + r] =
        make_float4(__fadd_rn(xv.x, acc.x), __fadd_rn(xv.y, acc.y), __fadd_rn(xv.z, acc.z), __fadd_rn(xv.w, acc.w));
  }
}

// Plan, activation image and the two GEMMs over the pairs of a.sel (down outputs into a.y).
void launch_moe_groups(const MoeArgs& a, cudaStream_t s) {
  const uint32_t rmax = moe_image_rows(a.T, a.top, a.E);
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
  k_moe_route<<<dim3(a.T, (a.E + kRouteRows - 1) / kRouteRows), 256, a.H * sizeof(float), s>>>(a, x);
  k_moe_select<<<a.T, 128, 0, s>>>(a);
  launch_moe_groups(a, s);
  k_moe_combine<<<dim3(a.T, (a.H / 4 + 255) / 256), 256, 0, s>>>(a, x, out);
  return nullptr;
}

uint64_t moe_ep_layout(uint32_t cap, uint32_t H, uint32_t top, uint32_t world, MoeEp* set0, MoeEp* set1) {
  uint64_t o = 256;  // flags
  auto take = [&](uint64_t bytes) {
    const uint64_t at = o;
    o = (o + bytes + 255) & ~255ull;
    return at;
  };
  for (MoeEp* m : {set0, set1}) {
    m->o_flags = 0;
    m->o_hdr = take(16);
    m->o_h = take((uint64_t)cap * H * 4);
    m->o_hs = take((uint64_t)cap * 4);
    m->o_sel = take((uint64_t)cap * top * 4);
    m->o_y = take((uint64_t)world * cap * top * H * 4);
  }
  return o;
}

const char* launch_moe_tc_ep(const MoeArgs& a, const MoeEp& ep, unsigned long long seq, const float* x, float* out,
                             cudaStream_t s) {
  if (ep.T == 0 || a.T != ep.T || ep.world < 2 || ep.world > 8 || ep.e_n * ep.world != a.E || a.H % 4)
    return "invalid expert-parallel layer arguments";
  uint8_t* const own = ep.own;
  MoeArgs l = a;  // this rank's tokens: normalized inputs, scales and selections into the exchange
  l.h = reinterpret_cast<float*>(own + ep.o_h);
  l.hscale = reinterpret_cast<float*>(own + ep.o_hs);
  l.sel = reinterpret_cast<uint32_t*>(own + ep.o_sel);
  k_moe_route<<<dim3(l.T, (l.E + kRouteRows - 1) / kRouteRows), 256, l.H * sizeof(float), s>>>(l, x);
  k_moe_select<<<l.T, 128, 0, s>>>(l);
  k_ep_signal<<<1, 32, 0, s>>>(ep, seq);
  k_ep_wait<<<1, 32, 0, s>>>(ep, seq, a.err);
  MoeArgs g = a;  // every rank's tokens, this rank's experts
  g.T = ep.world * ep.T;
  g.e_lo = ep.rank * ep.e_n;
  g.e_n = ep.e_n;
  g.y = reinterpret_cast<float*>(own + ep.o_y);
  k_ep_gather<<<g.T, 256, 0, s>>>(g, ep);
  launch_moe_groups(g, s);
  k_ep_signal<<<1, 32, 0, s>>>(ep, seq + 1);
  k_ep_wait<<<1, 32, 0, s>>>(ep, seq + 1, a.err);
  k_moe_combine_ep<<<dim3(l.T, (l.H / 4 + 255) / 256), 256, 0, s>>>(l, ep, x, out);
  return nullptr;
}

}  // namespace qc
