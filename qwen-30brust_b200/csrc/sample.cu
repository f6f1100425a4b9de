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
constexpr int kSortE = 16;           // radix sort: elements per thread per tile (tile = kST * kSortE)

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
  uint32_t offs[256];
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

// All n ids in (key descending, index ascending) order: a stable LSD radix sort of the inverted key
// (4 passes of 8 bits) from index order.  Each pass counts the digits, then walks tiles of
// kST * kSortE ids: warp w takes 32 * kSortE consecutive ids in rounds of 32, ranks each id among
// the same digit in its warp (match_any; earlier rounds counted in cnt[w][digit]), and after a
// scan of the warps' counts per digit every id lands at offs[digit] + (ids of that digit in
// earlier warps) + its rank: index order is kept within each digit.  Result in key[1], idx[1].
// cnt: [32][256] words of shared memory.
__device__ void sort_desc(const float* __restrict__ lg, uint32_t n, uint32_t* const key[2], uint32_t* const idx[2],
                          uint32_t* cnt, Shared& sh) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  for (int pass = 0; pass < 4; pass++) {
    const int shf = 8 * pass;
    const uint32_t* ks = pass ? key[(pass - 1) & 1] : nullptr;  // pass 0 reads the logits
    const uint32_t* is = pass ? idx[(pass - 1) & 1] : nullptr;
    uint32_t* kd = key[pass & 1];
    uint32_t* id = idx[pass & 1];
    auto kget = [&](uint32_t j) { return ks ? ks[j] : ~order_key(lg[j]); };
    auto iget = [&](uint32_t j) { return is ? is[j] : j; };
    for (uint32_t b = tid; b < 256; b += kST) sh.offs[b] = 0;
    for (uint32_t b = tid; b < 32 * 256; b += kST) cnt[b] = 0;
    __syncthreads();
    for (uint32_t j = tid; j < n; j += kST) atomicAdd(&sh.offs[(kget(j) >> shf) & 255u], 1u);
    __syncthreads();
    if (tid == 0) {  // exclusive scan of the digit counts
      uint32_t run = 0;
      for (int b = 0; b < 256; b++) {
        const uint32_t c = sh.offs[b];
        sh.offs[b] = run;
        run += c;
      }
    }
    __syncthreads();
    for (uint32_t base = 0; base < n; base += kST * kSortE) {
      const uint32_t w0 = base + warp * 32 * kSortE;
      uint32_t rank[kSortE];
#pragma unroll
      for (int e = 0; e < kSortE; e++) {
        const uint32_t j = w0 + e * 32 + lane;
        const uint32_t d = j < n ? (kget(j) >> shf) & 255u : 256u + lane;  // past n: a class of its own
        const uint32_t m = __match_any_sync(0xffffffffu, d);
        uint32_t r = 0;
        if (d < 256) r = cnt[warp * 256 + d];
        __syncwarp();
        if (d < 256 && (m & lt) == 0) cnt[warp * 256 + d] = r + __popc(m);  // the group's first lane
        __syncwarp();
        rank[e] = r + __popc(m & lt);
      }
      __syncthreads();
      if (tid < 256) {  // per digit: the warps' counts become their starting positions
        uint32_t run = sh.offs[tid];
        for (int w = 0; w < 32; w++) {
          const uint32_t c = cnt[w * 256 + tid];
          cnt[w * 256 + tid] = run;
          run += c;
        }
        sh.offs[tid] = run;
      }
      __syncthreads();
#pragma unroll
      for (int e = 0; e < kSortE; e++) {
        const uint32_t j = w0 + e * 32 + lane;
        if (j < n) {
          const uint32_t k = kget(j);
          const uint32_t pos = cnt[warp * 256 + ((k >> shf) & 255u)] + rank[e];
          kd[pos] = k;
          id[pos] = iget(j);
        }
      }
      __syncthreads();
      for (uint32_t b = tid; b < 32 * 256; b += kST) cnt[b] = 0;
      __syncthreads();
    }
  }
}

// Thread 0 visits v[0..n) in order, calling step(j, v[j]) until it returns false; the whole block
// stages the values in shared memory (buf: kChunk floats) a chunk at a time, so the serial chain
// reads shared memory instead of waiting on global loads.  Returns the index where the visit
// stopped, or n.  All threads of the block call it.
constexpr uint32_t kChunk = 16384;
template <class F>
__device__ uint32_t block_serial(const float* __restrict__ v, uint32_t n, float* buf, Shared& sh, F step) {
  if (threadIdx.x == 0) sh.count = n;
  for (uint32_t c0 = 0; c0 < n; c0 += kChunk) {
    __syncthreads();
    if (sh.count != n) break;
    const uint32_t m = min(kChunk, n - c0);
    for (uint32_t i = threadIdx.x; i < m; i += kST) buf[i] = v[c0 + i];
    __syncthreads();
    if (threadIdx.x == 0) {  // 8 values per pass, the next 8 loaded while these are visited
      const float4* b4 = reinterpret_cast<const float4*>(buf);
      const uint32_t m8 = m & ~7u;
      bool go = true;
      float4 x0 = m8 ? b4[0] : make_float4(0.f, 0.f, 0.f, 0.f), x1 = m8 ? b4[1] : x0;
      for (uint32_t j = 0; j < m8 && go; j += 8) {
        float4 y0 = x0, y1 = x1;
        if (j + 8 < m8) {
          y0 = b4[(j + 8) / 4];
          y1 = b4[(j + 8) / 4 + 1];
        }
        const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int k = 0; k < 8; k++)
          if (go && !step(c0 + j + k, x[k])) {
            sh.count = c0 + j + k;
            go = false;
          }
        x0 = y0;
        x1 = y1;
      }
      for (uint32_t j = m8; j < m && go; j++)
        if (!step(c0 + j, buf[j])) {
          sh.count = c0 + j;
          go = false;
        }
    }
  }
  __syncthreads();
  const uint32_t stop = sh.count;
  __syncthreads();
  return stop;
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
      sort_desc(lg, n, key, idx, reinterpret_cast<uint32_t*>(dyn), sh);
      const uint32_t K = Kset, *const ids = scr.idx1;
      for (uint32_t j = tid; j < K; j += kST) scr.p[j] = exp_f32(__fdiv_rn(__fsub_rn(lg[ids[j]], mx), temp));
      __syncthreads();
      float* const buf = reinterpret_cast<float*>(dyn);  // (the sort's counters are consumed)
      float total = 0.f;  // thread 0: the total with its running sums (sampling.rs:44)
      block_serial(scr.p, K, buf, sh, [&](uint32_t j, float x) {
        total = __fadd_rn(total, x);
        scr.run[j] = total;
        return true;
      });
      if (tid == 0) sh.red[0] = __float_as_uint(total);
      __syncthreads();
      const float tot = __uint_as_float((uint32_t)sh.red[0]);
      for (uint32_t j = tid; j < K; j += kST) scr.q[j] = __fdiv_rn(scr.p[j], tot);
      __syncthreads();
      // top-p: the first j whose cumulative sum of p / total reaches top_p (sampling.rs:45-52)
      float cum = 0.f;
      const uint32_t cut = block_serial(scr.q, K, buf, sh, [&](uint32_t, float x) {
        cum = __fadd_rn(cum, x);
        return !(cum >= top_p);
      });
      const uint32_t keep = cut < K ? cut + 1 : K;
      // the draw over the kept probabilities; their mass is the total's running sum at keep - 1
      float draw = 0.f;
      if (tid == 0) {
        const float mass = scr.run[keep - 1];
        draw = __fmul_rn((float)(next_word(s) >> 8) * (1.0f / 16777216.0f), mass);
      }
      const uint32_t hit = block_serial(scr.p, keep, buf, sh, [&](uint32_t, float x) {  // sampling.rs:56-63
        if (draw < x) return false;
        draw = __fsub_rn(draw, x);
        return true;
      });
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

constexpr int kSampleSmem = kExact * 12;  // also holds the radix sort's [32][256] counters
static_assert(kExact * 12 >= 32 * 256 * 4, "sort counters fit the exact path's shared memory");

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
