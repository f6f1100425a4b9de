// Sampler::sample (sampling.rs:26-65) on the device, with its random source.
//
// One block of 1024 threads reads the logits (L2-resident after the output phase wrote them).
//  * argmax with ties to the lower index: temperature 0 returns it without drawing (sampling.rs:34-36);
//  * the top-k set (sampling.rs:37-39) is found by a radix select on the f32 total-order key
//    (descending key, then ascending index, the reference's sort order) without sorting;
//  * sets of at most kExact ids are gathered, sorted (bitonic) and then run through the reference's
//    own sequential f32 arithmetic by one thread: max-subtracted exp / temperature, total, the
//    cumulative top-p cut, the draw and the subtract loop, with the same roundings;
//  * larger sets (top_k 0 over a 151,936-token vocabulary) are put in the same order by a stable
//    single-block LSD radix sort of all n (key, index) pairs in device scratch, and one warp then
//    runs the reference's sequential f32 folds over them (total with its running sums, cumulative
//    top-p cut, draw, subtract loop): the same values and roundings as the reference, so the same
//    id, at the cost of three dependent chains of up to n additions (~0.3 ms each at n = 151,936).
//  * exp((l - max) / T) is exp in double rounded once to f32 (correctly rounded except in rare
//    double-rounding cases), so it agrees with the host libm's f32 exp wherever that is within
//    half an ulp.
// The random source is rand 0.8's StdRng: ChaCha12 keyed by rand_core's seed_from_u64 (PCG32),
// words consumed in keystream order, gen::<f32>() = (word >> 8) * 2^-24.
#include "kernels.h"

namespace qc {
namespace {

constexpr int kST = 1024;
constexpr uint32_t kExact = 16384;  // (key, index) and probability of each: 12 B in shared memory
constexpr int kSortE = 8;            // radix sort: elements per thread per tile (tile = kST * kSortE)

// exp(x) for the probabilities: double exp rounded once to f32.
__device__ __forceinline__ float exp_f32(float x) { return __double2float_rn(exp((double)x)); }

__device__ __forceinline__ uint32_t order_key(float f) {  // f32::total_cmp order as unsigned
  const uint32_t u = __float_as_uint(f);
  return u ^ ((u >> 31) ? 0xffffffffu : 0x80000000u);
}

__device__ __forceinline__ uint32_t warp_of() { return threadIdx.x >> 5; }

__device__ __forceinline__ uint32_t rotl(uint32_t v, int c) { return __funnelshift_l(v, v, c); }

// ChaCha block (RFC 7539 quarter rounds), 12 rounds, block counter in words 12-13, stream 0.
__device__ void chacha12(const uint32_t key[8], unsigned long long block, uint32_t out[16]) {
  uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
  for (int i = 0; i < 8; i++) in[4 + i] = key[i];
  in[12] = (uint32_t)block;
  in[13] = (uint32_t)(block >> 32);
  in[14] = in[15] = 0;
  uint32_t x[16];
  for (int i = 0; i < 16; i++) x[i] = in[i];
#define QC_QR(a, b, c, d)                  \
  x[a] += x[b]; x[d] = rotl(x[d] ^ x[a], 16); \
  x[c] += x[d]; x[b] = rotl(x[b] ^ x[c], 12); \
  x[a] += x[b]; x[d] = rotl(x[d] ^ x[a], 8);  \
  x[c] += x[d]; x[b] = rotl(x[b] ^ x[c], 7);
  for (int r = 0; r < 12; r += 2) {
    QC_QR(0, 4, 8, 12) QC_QR(1, 5, 9, 13) QC_QR(2, 6, 10, 14) QC_QR(3, 7, 11, 15)
    QC_QR(0, 5, 10, 15) QC_QR(1, 6, 11, 12) QC_QR(2, 7, 8, 13) QC_QR(3, 4, 9, 14)
  }
#undef QC_QR
  for (int i = 0; i < 16; i++) out[i] = x[i] + in[i];
}

__device__ uint32_t next_word(SamplerDev* s) {  // one thread
  const unsigned long long w = s->word;
  uint32_t out[16];
  chacha12(s->key, w / 16, out);
  s->word = w + 1;
  return out[w % 16];
}

struct Found {
  uint32_t key, idx;
  unsigned long long before;  // weight of the members ahead of it in sort order
  unsigned long long w;       // its own weight
};

struct Shared {
  unsigned long long hist[256];
  unsigned long long red[33];
  Found found;
  uint32_t sel_b, count, token;
  unsigned long long sel_acc;
};

__device__ unsigned long long block_sum(unsigned long long v, Shared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = sh.red[lane];
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh.red[32] = v;
  }
  __syncthreads();
  v = sh.red[32];
  __syncthreads();
  return v;
}

__device__ unsigned long long block_max(unsigned long long v, Shared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = sh.red[lane];
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
      v = t > v ? t : v;
    }
    if (lane == 0) sh.red[32] = v;
  }
  __syncthreads();
  v = sh.red[32];
  __syncthreads();
  return v;
}

// Exclusive prefix sum over the threads in thread order.
__device__ unsigned long long block_exclusive(unsigned long long v, Shared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = v;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) sh.red[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = sh.red[lane], wi = w;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    sh.red[lane] = wi - w;  // exclusive over warps
  }
  __syncthreads();
  const unsigned long long r = sh.red[warp] + inc - v;
  __syncthreads();
  return r;
}

// The first id in (key descending, index ascending) order whose inclusive cumulative weight reaches
// `target` (1 <= target <= total weight).  wf(i, key) is the weight of id i (0 = not counted).
template <class W>
__device__ Found select_first(const float* __restrict__ lg, uint32_t n, unsigned long long target, W wf, Shared& sh) {
  const uint32_t tid = threadIdx.x;
  uint32_t prefix = 0, mask = 0;
  unsigned long long before = 0;
  for (int shf = 24; shf >= 0; shf -= 8) {
    for (uint32_t b = tid; b < 256; b += kST) sh.hist[b] = 0;
    __syncthreads();
    for (uint32_t i = tid; i < n; i += kST) {
      const uint32_t k = order_key(lg[i]);
      if ((k & mask) != prefix) continue;
      const unsigned long long w = wf(i, k);
      if (w) atomicAdd(&sh.hist[(k >> shf) & 255u], w);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned long long acc = 0;
      uint32_t b = 0;
      for (int bb = 255; bb >= 0; bb--) {
        if (acc + sh.hist[bb] >= target) {
          b = (uint32_t)bb;
          break;
        }
        acc += sh.hist[bb];
      }
      sh.sel_b = b;
      sh.sel_acc = acc;
    }
    __syncthreads();
    target -= sh.sel_acc;
    before += sh.sel_acc;
    prefix |= sh.sel_b << shf;
    mask |= 255u << shf;
  }
  // ids with exactly this key, in index order: each thread scans one contiguous range
  const uint32_t ch = (n + kST - 1) / kST, i0 = min(n, tid * ch), i1 = min(n, i0 + ch);
  unsigned long long mine = 0;
  for (uint32_t i = i0; i < i1; i++) {
    const uint32_t k = order_key(lg[i]);
    if (k == prefix) mine += wf(i, k);
  }
  const unsigned long long ex = block_exclusive(mine, sh);
  if (ex < target && target <= ex + mine) {  // exactly one thread
    unsigned long long c = ex;
    for (uint32_t i = i0; i < i1; i++) {
      const uint32_t k = order_key(lg[i]);
      if (k != prefix) continue;
      const unsigned long long w = wf(i, k);
      if (w && c + w >= target) {
        sh.found = Found{prefix, i, before + c, w};
        break;
      }
      c += w;
    }
  }
  __syncthreads();
  const Found f = sh.found;
  __syncthreads();
  return f;
}

__device__ __forceinline__ bool ahead_or_at(uint32_t i, uint32_t k, const Found& f) {
  return k > f.key || (k == f.key && i <= f.idx);
}

// The lanes of the warp whose digit d (8 bits) equals this lane's, among the lanes with valid set:
// one ballot per digit bit (match.any costs far more per element at this rate).  0 for invalid lanes.
__device__ __forceinline__ uint32_t digit_peers(uint32_t d, bool valid) {
  uint32_t peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
  for (int b = 0; b < 8; b++) {
    const uint32_t bit = (d >> b) & 1u, bal = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? bal : ~bal;
  }
  return valid ? peers : 0u;
}

// Exclusive scan of v[0..256) in place, by one warp (8 per lane); returns the sum to every lane.
__device__ uint32_t warp_scan256(uint32_t* v) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t x[8], s = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    x[i] = v[lane * 8 + i];
    s += x[i];
  }
  uint32_t incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= (uint32_t)o) incl += t;
  }
  uint32_t run = incl - s;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    v[lane * 8 + i] = run;
    run += x[i];
  }
  return __shfl_sync(0xffffffffu, incl, 31);
}

constexpr uint32_t kTile = kST * kSortE;                          // ids per tile of the radix sort
constexpr uint32_t kSortWords = 32 * 256 + 2 * kTile + 4 * 256 + 2 * 256;  // its shared memory

// All n ids in (key descending, index ascending) order: a stable LSD radix sort of the inverted key
// (4 passes of 8 bits) from index order.  One read first counts all four digits (global start of
// each digit per pass).  Each pass then walks tiles of kTile ids: warp w takes 32 * kSortE
// consecutive ids in rounds of 32 and ranks each among the same digit in its warp (ballots; earlier
// rounds counted in cnt[w][digit]); a scan over the warps per digit and over the tile's digits gives
// every id its place in the tile sorted by digit (shared memory), and the sorted tile goes out in
// order, so each digit's run of the tile is one contiguous write at that digit's global position.
// Index order is kept within each digit.  Result in key[1], idx[1].  sm: kSortWords words of shared
// memory.
__device__ void sort_desc(const float* __restrict__ lg, uint32_t n, uint32_t* const key[2], uint32_t* const idx[2],
                          uint32_t* sm) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t* const cnt = sm;                // [32][256] per-warp digit counts, then their prefixes
  uint32_t* const tk = cnt + 32 * 256;     // [kTile] the tile's keys in digit order
  uint32_t* const ti = tk + kTile;         // [kTile] and their indices
  uint32_t* const gof = ti + kTile;        // [4][256] global start of each digit, per pass
  uint32_t* const lst = gof + 4 * 256;     // [256] the tile's digit starts
  uint32_t* const tot = lst + 256;         // [256] the tile's digit counts
  for (uint32_t b = tid; b < 4 * 256; b += kST) gof[b] = 0;
  for (uint32_t b = tid; b < 32 * 256; b += kST) cnt[b] = 0;
  __syncthreads();
  for (uint32_t base = 0; base < n; base += kTile) {  // the four digit histograms
    uint32_t kv[kSortE];
#pragma unroll
    for (int e = 0; e < kSortE; e++) {
      const uint32_t j = base + e * kST + tid;
      kv[e] = j < n ? ~order_key(lg[j]) : 0u;
    }
#pragma unroll
    for (int e = 0; e < kSortE; e++) {
      const bool valid = base + e * kST + tid < n;
      if (valid) {  // the mantissa digits are spread out: plain atomics
        atomicAdd(&gof[kv[e] & 255u], 1u);
        atomicAdd(&gof[256 + ((kv[e] >> 8) & 255u)], 1u);
        atomicAdd(&gof[512 + ((kv[e] >> 16) & 255u)], 1u);
      }
      // the sign and exponent digit bunches up: one atomic per distinct digit of a warp
      const uint32_t d = kv[e] >> 24, peers = digit_peers(d, valid);
      if (valid && (peers & lt) == 0) atomicAdd(&gof[768 + d], (uint32_t)__popc(peers));
    }
  }
  __syncthreads();
  if (warp < 4) warp_scan256(gof + warp * 256);
  __syncthreads();
  for (int pass = 0; pass < 4; pass++) {
    const int shf = 8 * pass;
    const uint32_t* ks = pass ? key[(pass - 1) & 1] : nullptr;  // pass 0 reads the logits
    const uint32_t* is = pass ? idx[(pass - 1) & 1] : nullptr;
    uint32_t* kd = key[pass & 1];
    uint32_t* id = idx[pass & 1];
    uint32_t* const go = gof + pass * 256;
    for (uint32_t base = 0; base < n; base += kTile) {
      const uint32_t w0 = base + warp * 32 * kSortE;
      uint32_t rank[kSortE], kv[kSortE], iv[kSortE];
#pragma unroll
      for (int e = 0; e < kSortE; e++) {  // the tile's keys and indices, loads all in flight together
        const uint32_t j = w0 + e * 32 + lane;
        kv[e] = j < n ? (ks ? ks[j] : ~order_key(lg[j])) : 0u;
        iv[e] = j < n ? (is ? is[j] : j) : 0u;
      }
#pragma unroll
      for (int e = 0; e < kSortE; e++) {
        const bool valid = w0 + e * 32 + lane < n;
        const uint32_t d = (kv[e] >> shf) & 255u, peers = digit_peers(d, valid);
        const int lead = valid ? __ffs(peers) - 1 : (int)lane;
        uint32_t r = 0;
        if (valid && lead == (int)lane) {
          r = cnt[warp * 256 + d];
          cnt[warp * 256 + d] = r + __popc(peers);
        }
        rank[e] = __shfl_sync(0xffffffffu, r, lead) + __popc(peers & lt);
        __syncwarp();
      }
      __syncthreads();
      if (tid < 256) {  // per digit: the warps' counts become their starting positions in the digit
        uint32_t run = 0;
#pragma unroll 8
        for (int w = 0; w < 32; w++) {
          const uint32_t c = cnt[w * 256 + tid];
          cnt[w * 256 + tid] = run;
          run += c;
        }
        tot[tid] = run;
        lst[tid] = run;
      }
      __syncthreads();
      if (warp == 0) warp_scan256(lst);
      __syncthreads();
#pragma unroll
      for (int e = 0; e < kSortE; e++) {  // the tile in digit order, in shared memory
        if (w0 + e * 32 + lane < n) {
          const uint32_t d = (kv[e] >> shf) & 255u, lp = lst[d] + cnt[warp * 256 + d] + rank[e];
          tk[lp] = kv[e];
          ti[lp] = iv[e];
        }
      }
      __syncthreads();
      const uint32_t m = min(kTile, n - base);
      for (uint32_t i = tid; i < m; i += kST) {  // out in order: runs of one digit are contiguous
        const uint32_t k = tk[i], d = (k >> shf) & 255u, g = go[d] + i - lst[d];
        kd[g] = k;
        id[g] = ti[i];
      }
      __syncthreads();
      if (tid < 256) go[tid] += tot[tid];
      for (uint32_t b = tid; b < 32 * 256; b += kST) cnt[b] = 0;
      __syncthreads();
    }
  }
}

// Thread 0 visits v[0..n) in order, a chunk at a time: visit(c0, buf, m) sees v[c0 .. c0 + m) in
// shared memory and returns how many of them it consumed before stopping (m: go on).  The whole block
// stages each chunk (buf: kChunk floats), so the serial chain reads shared memory instead of waiting on
// global loads.  Returns the index where the visit stopped, or n.  All threads of the block call it.
constexpr uint32_t kChunk = 16384;
template <class F>
__device__ uint32_t block_chunks(const float* __restrict__ v, uint32_t n, float* buf, Shared& sh, F visit) {
  if (threadIdx.x == 0) sh.count = n;
  for (uint32_t c0 = 0; c0 < n; c0 += kChunk) {
    __syncthreads();
    if (sh.count != n) break;
    const uint32_t m = min(kChunk, n - c0);
    for (uint32_t i = threadIdx.x; i < m; i += kST) buf[i] = v[c0 + i];
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t used = visit(c0, buf, m);
      if (used < m) sh.count = c0 + used;
    }
  }
  __syncthreads();
  const uint32_t stop = sh.count;
  __syncthreads();
  return stop;
}

// The three sequential f32 chains of the large-set path (sampling.rs:41-63), eight terms per step
// (each still one rounded operation after the other, exactly as the reference folds them):
// total = fold of p with every eighth running sum; the top-p cut (the cumulative sum of q never decreases,
// so if the eighth partial sum stays below top_p all eight do); the pick (draw < p_j exactly when
// draw - p_j rounds below zero, and once negative the remainder stays negative).
struct TotalChain {
  float total;
  float* run;
  __device__ uint32_t operator()(uint32_t c0, const float* b, uint32_t m) {
    uint32_t j = 0;
    for (; j + 8 <= m; j += 8) {
      const float4 x0 = *reinterpret_cast<const float4*>(b + j), x1 = *reinterpret_cast<const float4*>(b + j + 4);
      float t = total;
      t = __fadd_rn(t, x0.x); t = __fadd_rn(t, x0.y); t = __fadd_rn(t, x0.z); t = __fadd_rn(t, x0.w);
      t = __fadd_rn(t, x1.x); t = __fadd_rn(t, x1.y); t = __fadd_rn(t, x1.z); t = __fadd_rn(t, x1.w);
      run[c0 + j + 7] = t;  // one running sum per 8 terms (positions 7 mod 8; run_at recomputes the rest)
      total = t;
    }
    for (; j < m; j++) {
      total = __fadd_rn(total, b[j]);
      run[c0 + j] = total;
    }
    return m;
  }
};
struct CutChain {
  float cum, top_p;
  __device__ uint32_t operator()(uint32_t, const float* b, uint32_t m) {
    uint32_t j = 0;
    for (; j + 8 <= m; j += 8) {
      const float4 x0 = *reinterpret_cast<const float4*>(b + j), x1 = *reinterpret_cast<const float4*>(b + j + 4);
      float c[8];
      c[0] = __fadd_rn(cum, x0.x); c[1] = __fadd_rn(c[0], x0.y); c[2] = __fadd_rn(c[1], x0.z);
      c[3] = __fadd_rn(c[2], x0.w); c[4] = __fadd_rn(c[3], x1.x); c[5] = __fadd_rn(c[4], x1.y);
      c[6] = __fadd_rn(c[5], x1.z); c[7] = __fadd_rn(c[6], x1.w);
      if (c[7] >= top_p) {
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (c[k] >= top_p) return j + k;
      }
      cum = c[7];
    }
    for (; j < m; j++) {
      cum = __fadd_rn(cum, b[j]);
      if (cum >= top_p) return j;
    }
    return m;
  }
};
struct PickChain {
  float draw;
  __device__ uint32_t operator()(uint32_t, const float* b, uint32_t m) {
    uint32_t j = 0;
    for (; j + 8 <= m; j += 8) {
      const float4 x0 = *reinterpret_cast<const float4*>(b + j), x1 = *reinterpret_cast<const float4*>(b + j + 4);
      float e[8];
      e[0] = __fsub_rn(draw, x0.x); e[1] = __fsub_rn(e[0], x0.y); e[2] = __fsub_rn(e[1], x0.z);
      e[3] = __fsub_rn(e[2], x0.w); e[4] = __fsub_rn(e[3], x1.x); e[5] = __fsub_rn(e[4], x1.y);
      e[6] = __fsub_rn(e[5], x1.z); e[7] = __fsub_rn(e[6], x1.w);
      if (e[7] < 0.f) {
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (e[k] < 0.f) return j + k;
      }
      draw = e[7];
    }
    for (; j < m; j++) {
      if (draw < b[j]) return j;
      draw = __fsub_rn(draw, b[j]);
    }
    return m;
  }
};

// The running sum of the fold of p after term q, from the stored sums (positions 7 mod 8, and every
// position of a chunk's tail): the same additions as the fold, in the same order.
__device__ float run_at(const float* p, const float* run, uint32_t q, uint32_t n) {
  const uint32_t c0 = q / kChunk * kChunk, m = min(kChunk, n - c0), tail = c0 + (m & ~7u);
  if ((q & 7) == 7 || q >= tail) return run[q];
  const uint32_t j0 = q & ~7u;
  float t = j0 ? run[j0 - 1] : 0.f;
  for (uint32_t j = j0; j <= q; j++) t = __fadd_rn(t, p[j]);
  return t;
}

// The logit of a sorted key (the sort keeps ~order_key(logit)): order_key inverted.
__device__ __forceinline__ float key_value(uint32_t nk) {
  const uint32_t k = ~nk;
  return __uint_as_float((k >> 31) ? (k ^ 0x80000000u) : ~k);
}

// One block per draw: block b samples logits row b (lg_base + b * lg_stride) with sampler sv[b]
// (or s0 for a single draw), writing the id to dsts[b] (or dst0) and using scratch region b.
struct SampleBatch {
  const float* lg_base;
  const float* const* lgv;  // per-block logits rows (device array), or null: lg_base + b * lg_stride
  uint64_t lg_stride;
  SamplerDev* s0;
  SamplerDev* const* sv;
  uint32_t* dst0;
  uint32_t* dsts;
  SampleScratch scr;
  uint64_t scr_stride;  // words between the scratch regions of consecutive blocks
};

__global__ void __launch_bounds__(kST) k_sample(SampleBatch sb, uint32_t n) {
  const uint32_t b = blockIdx.x;
  const float* __restrict__ lg = sb.lgv ? sb.lgv[b] : sb.lg_base + b * sb.lg_stride;
  SamplerDev* const s = sb.sv ? sb.sv[b] : sb.s0;
  uint32_t* const token_dst = sb.dsts ? sb.dsts + b : sb.dst0;
  SampleScratch scr = sb.scr;
  if (scr.key0) {
    const uint64_t o = b * sb.scr_stride;
    scr = SampleScratch{scr.key0 + o, scr.key1 + o, scr.idx0 + o, scr.idx1 + o, scr.p + o, scr.q + o, scr.run + o};
  }
  __shared__ Shared sh;
  extern __shared__ __align__(16) unsigned char dyn[];
  const uint32_t tid = threadIdx.x;
  // exact path: [kExact] (~key << 32 | index), sorted ascending, and their probabilities
  unsigned long long* const ck = reinterpret_cast<unsigned long long*>(dyn);
  float* const probs = reinterpret_cast<float*>(dyn + kExact * 8);
  const float temp = s->temperature, top_p = s->top_p;
  // argmax (ties to the lower index) and the finiteness check (sampling.rs:27-30)
  unsigned long long best = 0, bad = 0;
  for (uint32_t i = tid; i < n; i += kST) {
    const float v = lg[i];
    if (!isfinite(v)) bad = 1;
    const unsigned long long c = ((unsigned long long)order_key(v) << 32) | (0xffffffffu - i);
    best = c > best ? c : best;
  }
  best = block_max(best, sh);
  bad = block_sum(bad, sh);
  if (bad || n == 0) {
    if (tid == 0) s->err = 1;
    return;
  }
  const uint32_t amax = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
  uint32_t token = amax;
  if (tid == 0) sh.found = Found{0u, amax, 0, 0};  // (always overwritten by a select)
  __syncthreads();
  if (temp != 0.f) {
    const float mx = lg[amax];
    const uint32_t Kset = s->top_k > 0 && s->top_k < n ? s->top_k : n;
    Found fk{0u, 0xffffffffu, 0, 0};  // last id of the top-k set (everything when Kset == n)
    if (Kset < n && Kset <= kExact) fk = select_first(lg, n, Kset, [](uint32_t, uint32_t) { return 1ull; }, sh);
    if (Kset <= kExact) {
      // gather the set, sort it, then the reference's arithmetic on one thread
      if (tid == 0) sh.count = 0;
      __syncthreads();
      for (uint32_t i = tid; i < n; i += kST) {
        const uint32_t k = order_key(lg[i]);
        if (ahead_or_at(i, k, fk)) {
          const uint32_t slot = atomicAdd(&sh.count, 1u);
          if (slot < kExact) ck[slot] = ((unsigned long long)(~k) << 32) | i;
        }
      }
      __syncthreads();
      const uint32_t K = min(Kset, min(sh.count, kExact));  // == Kset
      uint32_t P = 1;
      while (P < K) P <<= 1;
      for (uint32_t j = K + tid; j < P; j += kST) ck[j] = ~0ull;
      __syncthreads();
      for (uint32_t size = 2; size <= P; size <<= 1)
        for (uint32_t stride = size >> 1; stride; stride >>= 1) {
          for (uint32_t j = tid; j < P; j += kST) {
            const uint32_t o = j ^ stride;
            if (o > j) {
              const unsigned long long a = ck[j], b = ck[o];
              const bool up = (j & size) == 0;
              if ((a > b) == up) {
                ck[j] = b;
                ck[o] = a;
              }
            }
          }
          __syncthreads();
        }
      for (uint32_t j = tid; j < K; j += kST)
        probs[j] = exp_f32(__fdiv_rn(__fsub_rn(lg[(uint32_t)ck[j]], mx), temp));
      __syncthreads();
      if (tid == 0) {
        float total = 0.f;
        for (uint32_t j = 0; j < K; j++) total = __fadd_rn(total, probs[j]);
        float cum = 0.f;
        uint32_t keep = K;
        for (uint32_t j = 0; j < K; j++) {
          cum = __fadd_rn(cum, __fdiv_rn(probs[j], total));
          if (cum >= top_p) {
            keep = j + 1;
            break;
          }
        }
        float mass = 0.f;
        for (uint32_t j = 0; j < keep; j++) mass = __fadd_rn(mass, probs[j]);
        float draw = __fmul_rn((float)(next_word(s) >> 8) * (1.0f / 16777216.0f), mass);
        uint32_t pick = (uint32_t)ck[keep - 1];
        for (uint32_t j = 0; j < keep; j++) {
          if (draw < probs[j]) {
            pick = (uint32_t)ck[j];
            break;
          }
          draw = __fsub_rn(draw, probs[j]);
        }
        sh.token = pick;
      }
      __syncthreads();
      token = sh.token;
    } else {
      // all n ids sorted in scratch; the top-k set is the first Kset of them (sampling.rs:32-39)
      uint32_t* const key[2] = {scr.key0, scr.key1};
      uint32_t* const idx[2] = {scr.idx0, scr.idx1};
      sort_desc(lg, n, key, idx, reinterpret_cast<uint32_t*>(dyn));
      const uint32_t K = Kset, *const ids = scr.idx1;
      // probabilities in sorted order, from the sorted keys (no gather of the logits)
      for (uint32_t j = tid; j < K; j += kST) scr.p[j] = exp_f32(__fdiv_rn(__fsub_rn(key_value(scr.key1[j]), mx), temp));
      __syncthreads();
      float* const buf = reinterpret_cast<float*>(dyn);  // (the sort's counters are consumed)
      TotalChain tc{0.f, scr.run};  // thread 0: the total with its running sums (sampling.rs:44)
      block_chunks(scr.p, K, buf, sh, [&](uint32_t c0, const float* b, uint32_t m) { return tc(c0, b, m); });
      const float total = tc.total;
      if (tid == 0) sh.red[0] = __float_as_uint(total);
      __syncthreads();
      const float tot = __uint_as_float((uint32_t)sh.red[0]);
      for (uint32_t j = tid; j < K; j += kST) scr.q[j] = __fdiv_rn(scr.p[j], tot);
      __syncthreads();
      // top-p: the first j whose cumulative sum of p / total reaches top_p (sampling.rs:45-52)
      CutChain cc{0.f, top_p};
      const uint32_t cut = block_chunks(scr.q, K, buf, sh, [&](uint32_t c0, const float* b, uint32_t m) { return cc(c0, b, m); });
      const uint32_t keep = cut < K ? cut + 1 : K;
      // the draw over the kept probabilities; their mass is the total's running sum at keep - 1
      float draw = 0.f;
      if (tid == 0) {
        const float mass = run_at(scr.p, scr.run, keep - 1, K);
        draw = __fmul_rn((float)(next_word(s) >> 8) * (1.0f / 16777216.0f), mass);
      }
      PickChain pc{draw};  // sampling.rs:56-63
      const uint32_t hit = block_chunks(scr.p, keep, buf, sh, [&](uint32_t c0, const float* b, uint32_t m) { return pc(c0, b, m); });
      if (tid == 0) sh.token = ids[hit < keep ? hit : keep - 1];
      __syncthreads();
      token = sh.token;
    }
  }
  if (tid == 0) {
    s->token = token;
    if (token_dst) *token_dst = token;
  }
}

__global__ void k_sampler_words(SamplerDev* s, uint32_t n, uint32_t* out) {
  if (threadIdx.x == 0)
    for (uint32_t i = 0; i < n; i++) out[i] = next_word(s);
}

}  // namespace

constexpr int kSampleSmem = kExact * 12;  // also holds the radix sort's tiles and counters
static_assert(kExact * 12 >= kSortWords * 4, "the radix sort fits the exact path's shared memory");
static_assert(kExact * 12 >= kChunk * 4, "a chain chunk fits the exact path's shared memory");

uint32_t sample_exact_max() { return kExact; }

cudaError_t sample_prepare() {
  return cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampleSmem);
}

cudaError_t launch_sample(const float* logits, uint32_t n, SamplerDev* s, uint32_t* token_dst,
                          const SampleScratch& scr, cudaStream_t st) {
  k_sample<<<1, kST, kSampleSmem, st>>>(SampleBatch{logits, nullptr, 0, s, nullptr, token_dst, nullptr, scr, 0}, n);
  return cudaGetLastError();
}

cudaError_t launch_sample_batch(const float* const* rows, uint32_t n, uint32_t draws, SamplerDev* const* sv,
                                uint32_t* tokens, void* scratch, cudaStream_t st) {
  const SampleScratch scr = scratch ? sample_scratch_at(scratch, n) : SampleScratch{};
  k_sample<<<draws, kST, kSampleSmem, st>>>(
      SampleBatch{nullptr, rows, 0, nullptr, sv, nullptr, tokens, scr, scratch ? sample_scratch_bytes(n) / 4 : 0}, n);
  return cudaGetLastError();
}

void launch_sampler_words(SamplerDev* s, uint32_t n, uint32_t* out, cudaStream_t st) {
  k_sampler_words<<<1, 32, 0, st>>>(s, n, out);
}

}  // namespace qc
