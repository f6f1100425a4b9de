// Sampler::sample (sampling.rs:26-65) on the device, with its random source.
//
// One block of 1024 threads reads the logits (L2-resident after the output phase wrote them).
//  * argmax with ties to the lower index: temperature 0 returns it without drawing (sampling.rs:34-36);
//  * the top-k set (sampling.rs:37-39) is found by a radix select on the f32 total-order key
//    (descending key, then ascending index, the reference's sort order) without sorting;
//  * sets of at most kExact ids are gathered, sorted (bitonic) and then run through the reference's
//    own sequential f32 arithmetic by one thread: max-subtracted exp / temperature, total, the
//    cumulative top-p cut, the draw and the subtract loop, with the same roundings;
//  * larger sets (top_k 0 over a 151,936-token vocabulary) use the same order and rules in exact
//    2^-40 fixed point: the total, the top-p boundary (first id whose cumulative mass reaches
//    top_p * total) and the drawn id (first id whose cumulative mass exceeds draw * kept mass) are
//    each a radix select by mass.  Integer sums make the result independent of thread timing; it
//    can differ from the reference's f32 running sums only when the draw or the cut falls within
//    their rounding of a boundary.
// The random source is rand 0.8's StdRng: ChaCha12 keyed by rand_core's seed_from_u64 (PCG32),
// words consumed in keystream order, gen::<f32>() = (word >> 8) * 2^-24.
#include "kernels.h"

namespace qc {
namespace {

constexpr int kST = 1024;
constexpr uint32_t kExact = 16384;  // (key, index) and probability of each: 12 B in shared memory
constexpr double kFix = 1099511627776.0;  // 2^40

__device__ __forceinline__ uint32_t order_key(float f) {  // f32::total_cmp order as unsigned
  const uint32_t u = __float_as_uint(f);
  return u ^ ((u >> 31) ? 0xffffffffu : 0x80000000u);
}

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

__global__ void __launch_bounds__(kST) k_sample(const float* __restrict__ lg, uint32_t n, SamplerDev* s,
                                                uint32_t* token_dst) {
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
    if (Kset < n) fk = select_first(lg, n, Kset, [](uint32_t, uint32_t) { return 1ull; }, sh);
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
        probs[j] = expf(__fdiv_rn(__fsub_rn(lg[(uint32_t)ck[j]], mx), temp));
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
      // exact fixed-point masses: w = round(exp((l - max) / T) * 2^40) inside the top-k set
      auto fix = [&](uint32_t i) {
        return (unsigned long long)__double2ull_rn((double)expf(__fdiv_rn(__fsub_rn(lg[i], mx), temp)) * kFix);
      };
      auto in_k = [&](uint32_t i, uint32_t k) { return ahead_or_at(i, k, fk) ? fix(i) : 0ull; };
      unsigned long long tot = 0;
      for (uint32_t i = tid; i < n; i += kST) tot += in_k(i, order_key(lg[i]));
      tot = block_sum(tot, sh);
      // top-p: the first id whose cumulative mass reaches top_p * total
      unsigned long long tp = (unsigned long long)ceil((double)top_p * (double)tot);
      tp = tp < 1 ? 1 : (tp > tot ? tot : tp);
      const Found fp = select_first(lg, n, tp, in_k, sh);
      const unsigned long long kept = fp.before + fp.w;
      // the draw: the first kept id whose cumulative mass exceeds u * kept
      if (tid == 0) sh.red[0] = next_word(s) >> 8;
      __syncthreads();
      const unsigned long long u = sh.red[0];
      __syncthreads();
      const unsigned long long lo = u * kept, hi = __umul64hi(u, kept);
      const unsigned long long d = (hi << 40) | (lo >> 24);  // floor(u * kept / 2^24) < kept
      const Found fd = select_first(lg, n, d + 1, [&](uint32_t i, uint32_t k) {
        return ahead_or_at(i, k, fp) ? in_k(i, k) : 0ull;
      }, sh);
      token = fd.idx;
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

constexpr int kSampleSmem = kExact * 12;

cudaError_t sample_prepare() {
  return cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampleSmem);
}

cudaError_t launch_sample(const float* logits, uint32_t n, SamplerDev* s, uint32_t* token_dst, cudaStream_t st) {
  k_sample<<<1, kST, kSampleSmem, st>>>(logits, n, s, token_dst);
  return cudaGetLastError();
}

void launch_sampler_words(SamplerDev* s, uint32_t n, uint32_t* out, cudaStream_t st) {
  k_sampler_words<<<1, 32, 0, st>>>(s, n, out);
}

}  // namespace qc
