// The MoE half of a layer (model.rs:245-287) for a batch of T tokens at once, on the 5th-generation
// tensor cores.
//
//   k_moe_route    per token: RMSNorm(ffn_norm), router matvec (F16), top-k with ties to the lower
//                  index, softmax over the kept logits in selection order (ops.rs:3-15, 29-56)
//   k_moe_plan     the (token, slot) pairs grouped by expert, tokens ascending within an expert
//   k_moe_gemm<0>  per (expert, 64-row tile): gate and up rows of the expert times its tokens'
//                  normalized inputs, then SwiGLU  g / (1 + exp(-g)) * u  (model.rs:259-274)
//   k_moe_gemm<1>  per (expert, 128-row tile): down rows times the expert's SwiGLU outputs
//   k_moe_combine  x + (w_0 y_0 + w_1 y_1 + ...) in selection order (model.rs:275-287)
//
// Tensor-core GEMM (tcgen05.mma, kind::f16, fp32 accumulator in TMEM, M = 128, N = tokens padded
// to 16): each weight is dequantized exactly as quant.rs does (separately rounded products),
// scaled by a power of two and split into two fp16 values hi + lo; each activation likewise
// (power-of-two scale per token).  hi*hi + hi*lo + lo*hi is accumulated by three MMAs per K step,
// so a product keeps ~22 significant bits and the only other rounding is the fp32 accumulation:
// results stay within the matvec tolerance of the reference's f32 fold.  Operands are written by
// the CTA's threads straight into the canonical no-swizzle K-major shared-memory layout (8-row x
// 16-byte core matrices) in two stages of K = 32, so dequantization of K step k+1 overlaps the
// MMAs of step k (two CTAs per SM); one thread issues the MMAs and commits them to the stage's
// mbarrier.  The bytes of the next K step are fetched into registers during the current one.
#include <cuda_fp16.h>

#include "kernels.h"

namespace qc {
namespace {

constexpr int kMT = 256;          // threads of a GEMM CTA
constexpr uint32_t kKS = 32;      // K elements per stage
constexpr uint32_t kKC = kKS / 8;  // 16-byte chunks of a row per stage
constexpr uint32_t kCPT = kKC / 2;  // A chunks per thread (two threads per row)
constexpr uint32_t kNMax = 128;   // tokens per accumulator pass
constexpr uint32_t kBPT = kNMax * kKC / kMT;  // B chunks per thread, at most
constexpr uint32_t kAStage = 128 * kKS * 2;         // one fp16 plane of A per stage: 8 KB
constexpr uint32_t kBStage = kNMax * kKS * 2;       // one fp16 plane of B per stage (N = 128): 8 KB
constexpr uint32_t kStage = 2 * kAStage + 2 * kBStage;
constexpr uint32_t kEpiBytes = 128 * (kNMax + 1) * 4;  // the epilogue's [128][N + 1] floats
constexpr uint32_t kSmem = 2 * kStage > kEpiBytes ? 2 * kStage : kEpiBytes;
constexpr uint32_t kTmemCols = 128;
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Canonical K-major layout without swizzle: 16-byte chunk kc (8 fp16 along K) of row r.
__device__ __forceinline__ uint32_t kmajor_off(uint32_t r, uint32_t kc, uint32_t rows) {
  return kc * rows * 16 + (r >> 3) * 128 + (r & 7) * 16;
}
// Shared-memory matrix descriptor: start, leading byte offset (between K chunks), stride byte offset
// (between 8-row groups), descriptor version 1, no swizzle.
__device__ __forceinline__ unsigned long long sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (unsigned long long)((addr >> 4) & 0x3fff) | ((unsigned long long)((lbo >> 4) & 0x3fff) << 16) |
         ((unsigned long long)((sbo >> 4) & 0x3fff) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mbar_init(uint64_t* m) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(m)) : "memory");
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Wait (at most 2 s) for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity) {
  const uint32_t a = smem_u32(m);
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; i++) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255) == 255 && now_ns() - t0 > kWaitNs) return false;
  }
}

__device__ __forceinline__ float pow2_scale(float maxabs) {  // 2^k with maxabs * 2^k < 2^14
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 1.f;
  int ex;
  frexpf(maxabs, &ex);  // maxabs < 2^ex
  return ldexpf(1.f, 14 - ex);
}

// v * s (s a power of two: exact) as fp16 hi + lo, two values per conversion.
__device__ __forceinline__ void split8(const float (&v)[8], float s, uint4* hi, uint4* lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float x0 = v[2 * j] * s, x1 = v[2 * j + 1] * s;
    const __half2 hh = __floats2half2_rn(x0, x1);
    const float2 back = __half22float2(hh);
    const __half2 ll = __floats2half2_rn(x0 - back.x, x1 - back.y);  // exact differences
    h[j] = *reinterpret_cast<const uint32_t*>(&hh);
    l[j] = *reinterpret_cast<const uint32_t*>(&ll);
  }
  *hi = make_uint4(h[0], h[1], h[2], h[3]);
  *lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---- per-token routing ---------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_moe_route(MoeArgs a, const float* __restrict__ x) {
  __shared__ float red[32];
  __shared__ float lg[1024];
  extern __shared__ __align__(16) float hsm[];  // [H] the normalized input, for the router rows
  const uint32_t t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    hr[i] = v;
    hsm[i] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  __syncthreads();
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = 0.f;
    for (int w = 0; w < 8; w++) m = fmaxf(m, red[w]);
    a.hscale[t] = pow2_scale(m);
  }
  // router logits: one warp per expert row (F16), 16-byte loads of 8 weights per lane
  for (uint32_t e = warp; e < a.E; e += 8) {
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
      lg[e] = acc;
      if (!isfinite(acc)) atomicOr(a.err, 1u);
    }
  }
  __syncthreads();
  // rank of each logit (ties to the lower index); the top ranks are the selection, in order
  for (uint32_t e = tid; e < a.E; e += 256) {
    const uint32_t ke = total_key_u(lg[e]);
    uint32_t rank = 0;
    for (uint32_t j = 0; j < a.E; j++) {
      const uint32_t kj = total_key_u(lg[j]);
      rank += kj > ke || (kj == ke && j < e);
    }
    if (rank < a.top) a.sel[(uint64_t)t * a.top + rank] = e;
  }
  __syncthreads();
  if (tid == 0) {  // ops.rs:29-44 over the kept logits, in selection order
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

// ---- pairs grouped by expert ---------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_moe_plan(MoeArgs a) {
  __shared__ uint32_t cnt[1024], off[1025];
  const uint32_t tid = threadIdx.x, P = a.T * a.top;
  for (uint32_t e = tid; e < a.E; e += 1024) cnt[e] = 0;
  __syncthreads();
  for (uint32_t p = tid; p < P; p += 1024) atomicAdd(&cnt[a.sel[p]], 1u);
  __syncthreads();
  if (tid == 0) {
    off[0] = 0;
    for (uint32_t e = 0; e < a.E; e++) off[e + 1] = off[e] + cnt[e];
  }
  __syncthreads();
  for (uint32_t e = tid; e < a.E; e += 1024) {
    a.cnt[e] = cnt[e];
    a.off[e] = off[e];
  }
  for (uint32_t p = tid; p < P; p += 1024) {
    const uint32_t e = a.sel[p];
    uint32_t before = 0;
    for (uint32_t q = 0; q < p; q++) before += a.sel[q] == e;
    const uint32_t pos = off[e] + before;
    a.ptok[pos] = p / a.top;
    a.ppair[pos] = p;
    a.gumax[p] = 0;
  }
}

// ---- A and B operands of one K step, fetched one step ahead -------------------------------------
// A: thread -> row tid/2 of the tile, chunks 4*(tid&1) .. +3 of the step (8 weights each, one
// quant.rs sub-block of Q4_K / one quarter of Q6_K).  The raw bytes of step k+1 are loaded into
// registers while step k is decoded and multiplied.
struct ARaw {
  uint4 hdr;            // Q4_K: d, dmin, 12 scale bytes.  Q6_K: the 16 scale bytes
  uint4 q[kCPT / 2];    // Q4_K: qs bytes of the chunks.  Q6_K: ql bytes
  uint4 h[kCPT / 2];    // Q6_K: qh bytes
  uint32_t d;           // Q6_K: f16 bits of d
};

template <int MODE>
__device__ __forceinline__ bool a_row(const MoeArgs& a, uint32_t tile, uint32_t r, const MatDesc** m, uint32_t* row) {
  if (MODE == 0) {
    *m = r < 64 ? &a.gate : &a.up;
    *row = tile * 64 + (r & 63);
    return *row < a.I;
  }
  *m = &a.down;
  *row = tile * 128 + r;
  return *row < a.H;
}

template <int MODE>
__device__ __forceinline__ void fetch_a(const MoeArgs& a, uint32_t e, uint32_t tile, uint32_t k0, ARaw& w) {
  const uint32_t r = threadIdx.x >> 1, kc0 = (threadIdx.x & 1) * kCPT;
  const MatDesc* m;
  uint32_t row;
  if (!a_row<MODE>(a, tile, r, &m, &row)) {
    w.hdr = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (uint32_t u = 0; u < kCPT / 2; u++) w.q[u] = w.h[u] = make_uint4(0, 0, 0, 0);
    w.d = 0;
    return;
  }
  const uint8_t* base = expert_base(*m, e);
  const uint32_t i = (k0 & 255) + 8 * kc0;  // first element of the thread's chunks in the super-block
  if (MODE == 0) {  // the chunks share one sub-block: 8 * kCPT consecutive qs bytes
    const uint8_t* b = row_ptr(*m, base, row) + (k0 >> 8) * 144;
    w.hdr = ldg16(b);
#pragma unroll
    for (uint32_t u = 0; u < kCPT / 2; u++) w.q[u] = ldg16(b + 16 + (i >> 6) * 32 + (i & 31) + 16 * u);
  } else {  // ... one quarter: 8 * kCPT consecutive ql and qh bytes
    const uint8_t* b = row_ptr(*m, base, row) + (k0 >> 8) * 208;
    const uint32_t chunk = i >> 7, quarter = (i & 127) >> 5, lane = i & 31;
    w.hdr = ldg16(b + 192);
#pragma unroll
    for (uint32_t u = 0; u < kCPT / 2; u++) {
      w.q[u] = ldg16(b + chunk * 64 + (quarter & 1) * 32 + lane + 16 * u);
      w.h[u] = ldg16(b + 128 + chunk * 32 + lane + 16 * u);
    }
    w.d = __ldg(reinterpret_cast<const unsigned short*>(drow_ptr(*m, base, row)) + (k0 >> 8));
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, uint32_t i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t byte_in(const uint4& v, uint32_t i) { return (word_of(v, i >> 2) >> (8 * (i & 3))) & 0xffu; }

// Chunk c (< kCPT) of the thread's A work for step k0: 8 weights, quant.rs arithmetic.
// The products are those of quant.rs times sw (a power of two, so the roundings are the same).
template <int MODE>
__device__ __forceinline__ void decode_a(const ARaw& w, uint32_t k0, uint32_t c, float sw, float (&out)[8]) {
  const uint32_t kc0 = (threadIdx.x & 1) * kCPT, i = (k0 & 255) + 8 * (kc0 + c);
  const uint4& q = w.q[c / 2];
  const uint32_t lo = word_of(q, (c & 1) * 2), hi = word_of(q, (c & 1) * 2 + 1);
  if (MODE == 0) {
    const uint32_t g = i >> 5;
    const uint4 h = w.hdr;
    int sc, mn;
    if (g < 4) {
      sc = byte_in(h, 4 + g) & 63;
      mn = byte_in(h, 8 + g) & 63;
    } else {
      sc = (byte_in(h, 8 + g) & 15) | ((byte_in(h, g) >> 6) << 4);
      mn = (byte_in(h, 8 + g) >> 4) | ((byte_in(h, 4 + g) >> 6) << 4);
    }
    const float d = h2f_bits(h.x), dmin = h2f_bits(h.x >> 16);
    const float ds = __fmul_rn(d, (float)sc) * sw, dm = __fmul_rn(dmin, (float)mn) * sw;
    const uint32_t sh = (g & 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t byte = ((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xffu;
      out[j] = __fsub_rn(__fmul_rn(ds, (float)((byte >> sh) & 15u)), dm);
    }
  } else {
    const uint32_t chunk = i >> 7, quarter = (i & 127) >> 5, lane = i & 31;
    const float sc = (float)(int8_t)byte_in(w.hdr, chunk * 8 + quarter * 2 + lane / 16);
    const float ds = __fmul_rn(h2f_bits(w.d), sc) * sw;
    const uint4& Hh = w.h[c / 2];
    const uint32_t h0 = word_of(Hh, (c & 1) * 2), h1 = word_of(Hh, (c & 1) * 2 + 1);
    const uint32_t sl = (quarter >> 1) * 4, shh = quarter * 2;
#pragma unroll
    for (int t = 0; t < 8; t++) {
      const uint32_t l = ((t < 4 ? lo : hi) >> (8 * (t & 3))) & 0xffu;
      const uint32_t h = ((t < 4 ? h0 : h1) >> (8 * (t & 3))) & 0xffu;
      const int qv = (int)(((l >> sl) & 15u) | (((h >> shh) & 3u) << 4)) - 32;
      out[t] = __fmul_rn(ds, (float)qv);
    }
  }
}

// B: items (token n, chunk kc) it = tid + 256 j, j < kBPT (N * kKC items).
struct BRaw {
  float4 v[kBPT][2];
};

template <int MODE>
__device__ __forceinline__ void fetch_b(const MoeArgs& a, const uint32_t* btok, const uint32_t* bpair, uint32_t nn,
                                        uint32_t N, uint32_t k0, BRaw& b) {
#pragma unroll
  for (uint32_t j = 0; j < kBPT; j++) {
    const uint32_t it = threadIdx.x + kMT * j, n = it / kKC, kc = it % kKC;
    if (it < N * kKC && n < nn) {
      const float* src = MODE == 0 ? a.h + (uint64_t)btok[n] * a.H + k0 + kc * 8
                                   : a.gu + (uint64_t)bpair[n] * a.I + k0 + kc * 8;
      b.v[j][0] = *reinterpret_cast<const float4*>(src);
      b.v[j][1] = *reinterpret_cast<const float4*>(src + 4);
    } else {
      b.v[j][0] = b.v[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

// ---- grouped GEMM on the tensor cores --------------------------------------------------------
// MODE 0: A rows 0-63 = gate rows [64 tile, +64), rows 64-127 = up rows; K = H; B = h of the tokens.
// MODE 1: A rows = down rows [128 tile, +128); K = I; B = SwiGLU outputs of the pairs.
template <int MODE>
__global__ void __launch_bounds__(kMT, 2) k_moe_gemm(MoeArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t mbar[2];
  __shared__ uint32_t tmem_base;
  __shared__ float bscale[kNMax];
  __shared__ uint32_t bpair[kNMax], btok[kNMax];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t e = blockIdx.y, tile = blockIdx.x;
  const uint32_t n_all = a.cnt[e];
  if (n_all == 0) return;
  const MatDesc& mA = MODE == 0 ? a.gate : a.down;
  const uint32_t K = MODE == 0 ? a.H : a.I, KS = K / kKS;
  const float sw = MODE == 0 ? a.sw_gu : a.sw_down;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&mbar[0]);
    mbar_init(&mbar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  uint32_t issued[2] = {0, 0};
  bool ok = true;

  for (uint32_t n0 = 0; n0 < n_all && ok; n0 += kNMax) {
    const uint32_t nn = min(kNMax, n_all - n0), N = max(16u, (nn + 15) & ~15u);
    for (uint32_t n = tid; n < N; n += kMT) {
      if (n < nn) {
        const uint32_t pos = a.off[e] + n0 + n;
        bpair[n] = a.ppair[pos];
        btok[n] = a.ptok[pos];
        bscale[n] = MODE == 0 ? a.hscale[btok[n]] : pow2_scale(__uint_as_float(a.gumax[bpair[n]]));
      } else {
        bpair[n] = btok[n] = 0xffffffffu;
        bscale[n] = 0.f;
      }
    }
    __syncthreads();
    // instruction descriptor: f32 accumulator, f16 A and B, both K-major, N, M = 128
    const uint32_t idesc = (1u << 4) | ((N >> 3) << 17) | ((128u >> 4) << 24);
    ARaw anx;
    BRaw bnx;
    fetch_a<MODE>(a, e, tile, 0, anx);
    fetch_b<MODE>(a, btok, bpair, nn, N, 0, bnx);
    for (uint32_t ks = 0; ks < KS; ks++) {
      const uint32_t s = ks & 1;
      const ARaw acur = anx;
      const BRaw bcur = bnx;
      const uint32_t k0 = ks * kKS;
      if (ks + 1 < KS) {  // the next step's bytes are in flight during this step
        fetch_a<MODE>(a, e, tile, k0 + kKS, anx);
        fetch_b<MODE>(a, btok, bpair, nn, N, k0 + kKS, bnx);
      }
      if (issued[s] && !mbar_wait(&mbar[s], (issued[s] - 1) & 1)) {
        ok = false;
        break;
      }
      uint8_t* st = sm + s * kStage;
      uint8_t *ahi = st, *alo = st + kAStage, *bhi = st + 2 * kAStage, *blo = bhi + kBStage;
      {
        const uint32_t r = tid >> 1, kc0 = (tid & 1) * kCPT;
#pragma unroll
        for (uint32_t c = 0; c < kCPT; c++) {
          float w[8];
          decode_a<MODE>(acur, k0, c, sw, w);
          uint4 h, l;
          split8(w, 1.f, &h, &l);
          *reinterpret_cast<uint4*>(ahi + kmajor_off(r, kc0 + c, 128)) = h;
          *reinterpret_cast<uint4*>(alo + kmajor_off(r, kc0 + c, 128)) = l;
        }
      }
#pragma unroll
      for (uint32_t j = 0; j < kBPT; j++) {
        const uint32_t it = tid + kMT * j, n = it / kKC, kc = it % kKC;
        if (it < N * kKC) {
          const float v[8] = {bcur.v[j][0].x, bcur.v[j][0].y, bcur.v[j][0].z, bcur.v[j][0].w,
                              bcur.v[j][1].x, bcur.v[j][1].y, bcur.v[j][1].z, bcur.v[j][1].w};
          uint4 h, l;
          split8(v, n < nn ? bscale[n] : 0.f, &h, &l);
          *reinterpret_cast<uint4*>(bhi + kmajor_off(n, kc, N)) = h;
          *reinterpret_cast<uint4*>(blo + kmajor_off(n, kc, N)) = l;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (tid == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_hi = smem_u32(ahi), a_lo = smem_u32(alo), b_hi = smem_u32(bhi), b_lo = smem_u32(blo);
#pragma unroll
        for (uint32_t j = 0; j < kKS / 16; j++) {  // K = 16 per MMA: chunks 2j, 2j+1
          const unsigned long long dah = sdesc(a_hi + 2 * j * 128 * 16, 128 * 16, 128);
          const unsigned long long dal = sdesc(a_lo + 2 * j * 128 * 16, 128 * 16, 128);
          const unsigned long long dbh = sdesc(b_hi + 2 * j * N * 16, N * 16, 128);
          const unsigned long long dbl = sdesc(b_lo + 2 * j * N * 16, N * 16, 128);
          const uint32_t acc0 = (ks > 0 || j > 0) ? 1u : 0u;
          asm volatile(
              "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
              "l"(dah), "l"(dbh), "r"(idesc), "r"(acc0)
              : "memory");
          asm volatile(
              "{\n.reg .pred p;\nsetp.ne.b32 p, 1, 0;\n"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
              "l"(dah), "l"(dbl), "r"(idesc)
              : "memory");
          asm volatile(
              "{\n.reg .pred p;\nsetp.ne.b32 p, 1, 0;\n"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
              "l"(dal), "l"(dbh), "r"(idesc)
              : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&mbar[s]))
                     : "memory");
      }
      issued[s]++;
    }
    if (!ok) break;
    {  // the last commit covers every MMA issued before it
      const uint32_t s = (KS - 1) & 1;
      if (!mbar_wait(&mbar[s], (issued[s] - 1) & 1)) {
        ok = false;
        break;
      }
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // epilogue: warp q < 4 reads TMEM lanes 32q..32q+31 (rows), N columns (tokens)
    float* E = reinterpret_cast<float*>(sm);  // [128][N + 1]
    if (warp < 4) {
      const uint32_t r = warp * 32 + lane;
      for (uint32_t c0 = 0; c0 < N; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
            "%14, %15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tmem + ((warp * 32u) << 16) + c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const uint32_t n = c0 + j;
          E[r * (N + 1) + n] = n < nn ? __uint_as_float(v[j]) / (sw * bscale[n]) : 0.f;
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (MODE == 0) {
      for (uint32_t it = tid; it < 64 * nn; it += kMT) {
        const uint32_t n = it / 64, j = it % 64, row = tile * 64 + j;
        if (row < a.I) {
          const float g = E[j * (N + 1) + n], u = E[(64 + j) * (N + 1) + n];
          const float act = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
          a.gu[(uint64_t)bpair[n] * a.I + row] = act;
          atomicMax(&a.gumax[bpair[n]], __float_as_uint(fabsf(act)));
        }
      }
    } else {
      for (uint32_t it = tid; it < 128 * nn; it += kMT) {
        const uint32_t n = it / 128, r = it % 128, row = tile * 128 + r;
        if (row < a.H) a.y[(uint64_t)bpair[n] * a.H + row] = E[r * (N + 1) + n];
      }
    }
    __syncthreads();
  }
  if (!ok && tid == 0) atomicOr(a.err, 2u);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (!ok) {  // let MMAs still in flight finish before the accumulator is released
    for (uint32_t s = 0; s < 2; s++)
      if (issued[s]) mbar_wait(&mbar[s], (issued[s] - 1) & 1);
  }
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
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

// Upper bound of |w| over a Q4_K or Q6_K expert stack, from the block scales (atomic max of bits).
__global__ void k_moe_wbound(MatDesc m, uint32_t experts, uint32_t* out) {
  const uint32_t blocks = m.cols / 256;
  const uint64_t n = (uint64_t)experts * m.rows * blocks;
  float mx = 0.f;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t e = (uint32_t)(i / ((uint64_t)m.rows * blocks)), rem = (uint32_t)(i % ((uint64_t)m.rows * blocks));
    const uint32_t r = rem / blocks, sb = rem % blocks;
    const uint8_t* base = expert_base(m, e);
    if (m.kind == Q4_K) {
      const uint8_t* b = row_ptr(m, base, r) + sb * 144;
      const float d = fabsf(h2f_bits(b[0] | (b[1] << 8))), dmin = fabsf(h2f_bits(b[2] | (b[3] << 8)));
      mx = fmaxf(mx, d * 63.f * 15.f + dmin * 63.f);
    } else {
      mx = fmaxf(mx, fabsf(__half2float(drow_ptr(m, base, r)[sb])) * 128.f * 32.f);
    }
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0 && isfinite(mx)) atomicMax(out, __float_as_uint(mx));
}

}  // namespace

const char* moe_tc_supported(const MoeArgs& a) {
  if (a.gate.kind != Q4_K || a.up.kind != Q4_K || a.down.kind != Q6_K)
    return "the tensor-core MoE path takes Q4_K gate/up and Q6_K down experts";
  if (a.H % 64 || a.I % 64) return "the tensor-core MoE path needs hidden and intermediate sizes in multiples of 64";
  if (a.router.kind != F16) return "the batched MoE path takes an F16 router";
  if (a.E > 1024) return "the batched MoE path takes at most 1024 experts";
  return nullptr;
}

size_t moe_gemm_smem() { return kSmem; }

cudaError_t moe_prepare() {
  cudaError_t e = cudaFuncSetAttribute(k_moe_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)moe_gemm_smem());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_moe_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)moe_gemm_smem());
  return e;
}

void launch_moe_wbound(const MatDesc& m, uint32_t experts, uint32_t* out, cudaStream_t s) {
  k_moe_wbound<<<296, 256, 0, s>>>(m, experts, out);
}

void launch_moe_tc(const MoeArgs& a, const float* x, float* out, cudaStream_t s) {
  k_moe_route<<<a.T, 256, a.H * sizeof(float), s>>>(a, x);
  k_moe_plan<<<1, 1024, 0, s>>>(a);
  k_moe_gemm<0><<<dim3((a.I + 63) / 64, a.E), kMT, moe_gemm_smem(), s>>>(a);
  k_moe_gemm<1><<<dim3((a.H + 127) / 128, a.E), kMT, moe_gemm_smem(), s>>>(a);
  k_moe_combine<<<a.T, 256, 0, s>>>(a, x, out);
}

}  // namespace qc
