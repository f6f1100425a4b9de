// CPU ORACLE — test infrastructure only.
//
// This file restates, in C++, the CPU path of the reference Rust crate
// (qwen-rust 0.1.0) so that the CUDA engine can be checked against it on the
// same inputs.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline arm load it; the engine never links or calls it.
//
// Parity is pinned by tests/test_oracle.py against the reference's own golden
// vectors: the two-block dequant fixtures of tests/core.rs:50-151 (bit-exact),
// the rope / route / GQA known answers of tests/core.rs:3-27, and the 4x16
// expected logits of tests/data/expected-logits.json produced by
// tools/reference_fixture.py (abs 2e-5, tests/model.rs:48-69).
//
// Every function cites the reference file:line it follows.  Floating-point
// operations are written in the same order as the Rust source (sequential
// left folds, product of scale and weight first, division by sqrt(d), ...),
// and the file is compiled with -ffp-contract=off so no multiply-add is fused
// where Rust would round twice.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <condition_variable>
#include <exception>
#include <functional>
#include <mutex>
#include <thread>

namespace {

thread_local std::string g_err;

// Row-parallel loop over [0, n) on `threads` worker threads (0 = all hardware threads).  Each
// index is computed by exactly one thread with the same sequential arithmetic, so results do not
// depend on the thread count.  The workers persist between calls (a pool), so the many small
// matvecs of one token do not pay a thread start each.
class Pool {
 public:
  static Pool& get() {
    static Pool p;
    return p;
  }
  // Runs f(i) for i in [0, n) on min(nt, n) threads (the caller is one of them).
  void run(size_t n, size_t nt, const std::function<void(size_t)>& f) {
    std::lock_guard<std::mutex> serial(call_mu_);  // one parallel loop at a time
    nt = std::min(nt, n);
    if (nt <= 1) {
      for (size_t i = 0; i < n; i++) f(i);
      return;
    }
    grow(nt - 1);
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &f;
      n_ = n;
      nt_ = nt;
      pending_ = nt - 1;
      gen_++;
    }
    cv_.notify_all();
    slice(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
    if (err_) {  // the first failure of any slice, raised on the calling thread
      std::exception_ptr e = err_;
      err_ = nullptr;
      std::rethrow_exception(e);
    }
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }

 private:
  void slice(size_t t) {
    const size_t lo = n_ * t / nt_, hi = n_ * (t + 1) / nt_;
    try {
      for (size_t i = lo; i < hi; i++) (*job_)(i);
    } catch (...) {
      std::lock_guard<std::mutex> lk(err_mu_);
      if (!err_) err_ = std::current_exception();
    }
  }
  void grow(size_t want) {
    while (workers_.size() < want) {
      const size_t id = workers_.size() + 1;  // slice index of this worker
      workers_.emplace_back([this, id] {
        uint64_t seen = 0;
        for (;;) {
          {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return gen_ != seen; });
            seen = gen_;
            if (stop_) return;
            if (id >= nt_) continue;  // not needed by this loop
          }
          slice(id);
          std::lock_guard<std::mutex> lk(mu_);
          if (--pending_ == 0) done_cv_.notify_one();
        }
      });
    }
  }
  std::mutex call_mu_, mu_, err_mu_;
  std::exception_ptr err_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::thread> workers_;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t n_ = 0, nt_ = 1, pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

template <class F>
void parallel_for(size_t n, int threads, F&& f) {
  size_t nt = threads > 0 ? (size_t)threads : std::max(1u, std::thread::hardware_concurrency());
  const std::function<void(size_t)> fn = [&](size_t i) { f(i); };
  Pool::get().run(n, nt, fn);
}

struct Fail {
  std::string msg;
};
[[noreturn]] void fail(const std::string& m) { throw Fail{m}; }
#define ENSURE(c, m)       \
  do {                     \
    if (!(c)) fail(m);     \
  } while (0)

// ---------------------------------------------------------------- quant.rs
// quant.rs:5-11
bool layout(uint32_t kind, size_t* block, size_t* bytes) {
  switch (kind) {
    case 0: *block = 1; *bytes = 4; return true;
    case 1: *block = 1; *bytes = 2; return true;
    case 2: *block = 32; *bytes = 18; return true;
    case 8: *block = 32; *bytes = 34; return true;
    case 12: *block = 256; *bytes = 144; return true;
    case 13: *block = 256; *bytes = 176; return true;
    case 14: *block = 256; *bytes = 210; return true;
    default: return false;
  }
}
// quant.rs:12-21
size_t row_bytes(uint32_t kind, size_t cols) {
  size_t block, bytes;
  if (!layout(kind, &block, &bytes))
    fail("GGML tensor type " + std::to_string(kind) +
         " is not supported (supported: F32/F16/Q4_0/Q8_0/Q4_K/Q5_K/Q6_K)");
  ENSURE(cols > 0 && cols % block == 0,
         "row width " + std::to_string(cols) + " is not divisible by block size " +
             std::to_string(block));
  size_t n = cols / block;
  ENSURE(n == 0 || bytes <= SIZE_MAX / n, "row size overflow");
  return n * bytes;
}
// IEEE binary16 -> binary32, exact (the `half` crate's f16::to_f32, quant.rs:22-24).
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400));
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
inline float h(const uint8_t* b, size_t p) { return f16_to_f32((uint16_t)(b[p] | (b[p + 1] << 8))); }
// quant.rs:25-34
inline void scale(const uint8_t* b, size_t j, uint8_t* s, uint8_t* m) {
  if (j < 4) {
    *s = b[j] & 63;
    *m = b[j + 4] & 63;
  } else {
    *s = (uint8_t)((b[j + 4] & 15) | ((b[j - 4] >> 6) << 4));
    *m = (uint8_t)((b[j + 4] >> 4) | ((b[j] >> 6) << 4));
  }
}
// quant.rs:36-80 — one element of a validated row.
float value(const uint8_t* b, uint32_t kind, size_t col) {
  switch (kind) {
    case 0: {
      float f;
      memcpy(&f, b + col * 4, 4);
      return f;
    }
    case 1:
      return h(b, col * 2);
    case 2: {
      size_t p = col / 32 * 18, i = col % 32;
      uint8_t q = (uint8_t)((b[p + 2 + i % 16] >> (i < 16 ? 0 : 4)) & 15);
      return h(b, p) * (float)((int)q - 8);
    }
    case 8: {
      size_t p = col / 32 * 34;
      return h(b, p) * (float)(int8_t)b[p + 2 + col % 32];
    }
    case 12:
    case 13: {
      size_t size = kind == 12 ? 144 : 176;
      size_t p = col / 256 * size, i = col % 256, group = i / 32;
      uint8_t s, m;
      scale(b + p + 4, group, &s, &m);
      size_t qs = p + (kind == 12 ? 16 : 48);
      uint8_t q = (uint8_t)((b[qs + (i / 64) * 32 + i % 32] >> ((group % 2) * 4)) & 15);
      if (kind == 13 && (b[p + 16 + i % 32] & (1u << group)) != 0) q += 16;
      // h(b,p) * s as f32 * q as f32 - h(b,p+2) * m as f32  (left to right, no fusion)
      float a = h(b, p) * (float)s;
      a = a * (float)q;
      float c = h(b, p + 2) * (float)m;
      return a - c;
    }
    case 14: {
      size_t p = col / 256 * 210, i = col % 256, chunk = i / 128, j = i % 128;
      size_t quarter = j / 32, lane = j % 32;
      uint8_t low = b[p + chunk * 64 + (quarter % 2) * 32 + lane];
      uint8_t lo = (uint8_t)((low >> ((quarter / 2) * 4)) & 15);
      uint8_t hi = (uint8_t)((b[p + 128 + chunk * 32 + lane] >> (quarter * 2)) & 3);
      int q = (int)(lo | (hi << 4)) - 32;
      float a = h(b, p + 208) * (float)(int8_t)b[p + 192 + chunk * 8 + quarter * 2 + lane / 16];
      return a * (float)q;
    }
  }
  fail("tensor types validated by reader");
}

// Rust's `Iterator::sum::<f32>()` is a sequential left fold that starts from -0.0.
constexpr float kSumInit = -0.0f;

// All values of block `k` of a row (elements k*block .. +block), each computed with exactly the
// operations value() uses for it (quant.rs:36-80); only the per-block factors (d * sc, dmin * m,
// d * scale) are computed once per block or sub-block instead of once per element, which gives the
// same f32 results.  Used by the fast matvec below.
void decode_block(const uint8_t* b, uint32_t kind, size_t k, float* out) {
  switch (kind) {
    case 2: {
      const size_t p = k * 18;
      const float d = h(b, p);
      for (size_t i = 0; i < 32; i++) {
        const uint8_t q = (uint8_t)((b[p + 2 + i % 16] >> (i < 16 ? 0 : 4)) & 15);
        out[i] = d * (float)((int)q - 8);
      }
      return;
    }
    case 8: {
      const size_t p = k * 34;
      const float d = h(b, p);
      for (size_t i = 0; i < 32; i++) out[i] = d * (float)(int8_t)b[p + 2 + i];
      return;
    }
    case 12:
    case 13: {
      const size_t size = kind == 12 ? 144 : 176, p = k * size, qs = p + (kind == 12 ? 16 : 48);
      const float d = h(b, p), dmin = h(b, p + 2);
      for (size_t g = 0; g < 8; g++) {
        uint8_t s, m;
        scale(b + p + 4, g, &s, &m);
        const float ds = d * (float)s, c = dmin * (float)m;
        for (size_t t = 0; t < 32; t++) {
          const size_t i = g * 32 + t;
          uint8_t q = (uint8_t)((b[qs + (i / 64) * 32 + i % 32] >> ((g % 2) * 4)) & 15);
          if (kind == 13 && (b[p + 16 + i % 32] & (1u << g)) != 0) q += 16;
          out[i] = ds * (float)q - c;
        }
      }
      return;
    }
    case 14: {
      const size_t p = k * 210;
      const float d = h(b, p + 208);
      for (size_t i = 0; i < 256; i++) {
        const size_t chunk = i / 128, j = i % 128, quarter = j / 32, lane = j % 32;
        const uint8_t low = b[p + chunk * 64 + (quarter % 2) * 32 + lane];
        const uint8_t lo = (uint8_t)((low >> ((quarter / 2) * 4)) & 15);
        const uint8_t hi = (uint8_t)((b[p + 128 + chunk * 32 + lane] >> (quarter * 2)) & 3);
        const int q = (int)(lo | (hi << 4)) - 32;
        out[i] = (d * (float)(int8_t)b[p + 192 + chunk * 8 + quarter * 2 + lane / 16]) * (float)q;
      }
      return;
    }
    default:
      out[0] = value(b, kind, k);
  }
}

// backend.rs:28-52 (Cpu::matvec) — y[r] = sequential f32 fold of x[i] * value(row, i), each element
// decoded by value() as the reference does.  With `fast`, the same folds over values decoded a
// block at a time (decode_block), four rows interleaved per thread: identical results, for tests
// that need many tokens of a large model.
void matvec(const uint8_t* data, uint32_t kind, size_t rows, size_t cols, const float* x, float* y,
            int threads, bool fast = false) {
  size_t rb = row_bytes(kind, cols);
  if (!fast) {
    parallel_for(rows, threads, [&](size_t r) {
      const uint8_t* b = data + r * rb;
      float acc = kSumInit;
      for (size_t i = 0; i < cols; i++) acc = acc + x[i] * value(b, kind, i);
      y[r] = acc;
    });
    return;
  }
  size_t block, bytes;
  layout(kind, &block, &bytes);
  const size_t nq = (rows + 3) / 4;
  parallel_for(nq, threads, [&](size_t qi) {
    const size_t r0 = qi * 4, nr = std::min<size_t>(4, rows - r0);
    float acc[4] = {kSumInit, kSumInit, kSumInit, kSumInit};
    float v[4][256];
    for (size_t k = 0; k < cols / block; k++) {
      for (size_t j = 0; j < nr; j++) decode_block(data + (r0 + j) * rb, kind, k, v[j]);
      const float* xx = x + k * block;
      if (nr == 4) {
        for (size_t i = 0; i < block; i++) {
          acc[0] = acc[0] + xx[i] * v[0][i];
          acc[1] = acc[1] + xx[i] * v[1][i];
          acc[2] = acc[2] + xx[i] * v[2][i];
          acc[3] = acc[3] + xx[i] * v[3][i];
        }
      } else {
        for (size_t j = 0; j < nr; j++)
          for (size_t i = 0; i < block; i++) acc[j] = acc[j] + xx[i] * v[j][i];
      }
    }
    for (size_t j = 0; j < nr; j++) y[r0 + j] = acc[j];
  });
}

// Y[t][r] for n input vectors X[t] (t < n): the same sequential fold per (t, r) as matvec, each
// row decoded once (decode_block) and applied to kTile vectors at a time (independent folds, so
// the compiler runs them side by side in vector registers).  Used by Model::prefill.
constexpr size_t kTile = 32;
void matmul(const uint8_t* data, uint32_t kind, size_t rows, size_t cols, const float* X, size_t n, float* Y,
            int threads) {
  size_t rb = row_bytes(kind, cols);
  size_t block, bytes;
  layout(kind, &block, &bytes);
  // X transposed in tiles: XT[tile][i][k] = X[tile * kTile + k][i] (0 past n)
  const size_t tiles = (n + kTile - 1) / kTile;
  std::vector<float> XT(tiles * cols * kTile, 0.f);
  for (size_t t = 0; t < n; t++)
    for (size_t i = 0; i < cols; i++) XT[(t / kTile) * cols * kTile + i * kTile + t % kTile] = X[t * cols + i];
  parallel_for(rows, threads, [&](size_t r) {
    std::vector<float> w(cols);
    const uint8_t* b = data + r * rb;
    for (size_t k = 0; k < cols / block; k++) decode_block(b, kind, k, w.data() + k * block);
    for (size_t tile = 0; tile < tiles; tile++) {
      float acc[kTile];
      for (size_t k = 0; k < kTile; k++) acc[k] = kSumInit;
      const float* xt = XT.data() + tile * cols * kTile;
      for (size_t i = 0; i < cols; i++)
        for (size_t k = 0; k < kTile; k++) acc[k] = acc[k] + xt[i * kTile + k] * w[i];
      for (size_t k = 0; k < kTile && tile * kTile + k < n; k++) Y[(tile * kTile + k) * rows + r] = acc[k];
    }
  });
}

// ---------------------------------------------------------------- ops.rs
// ops.rs:3-15
void rms(float* x, const float* w, size_t n, float eps) {
  ENSURE(n > 0 && eps > 0.f, "RMSNorm shape/epsilon invalid");
  float ss = kSumInit;
  for (size_t i = 0; i < n; i++) ss = ss + x[i] * x[i];
  float s = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) x[i] *= s * w[i];
}
// ops.rs:17-28 (NeoX split-half rotation)
void rope(float* x, size_t n, size_t head, size_t pos, float theta) {
  for (size_t o = 0; o + head <= n; o += head) {
    float* hh = x + o;
    for (size_t i = 0; i < head / 2; i++) {
      float e = -2.0f * (float)i / (float)head;
      float angle = (float)pos * powf(theta, e);
      float s = sinf(angle), c = cosf(angle);
      float a = hh[i], b = hh[i + head / 2];
      hh[i] = a * c - b * s;
      hh[i + head / 2] = a * s + b * c;
    }
  }
}
// ops.rs:29-44
void softmax(float* x, size_t n) {
  ENSURE(n > 0, "invalid softmax logits");
  for (size_t i = 0; i < n; i++) ENSURE(std::isfinite(x[i]), "invalid softmax logits");
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = std::fmax(mx, x[i]);
  float sum = 0.f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf(x[i] - mx);
    sum += x[i];
  }
  for (size_t i = 0; i < n; i++) x[i] /= sum;
}
// f32::total_cmp key (IEEE totalOrder): larger key == larger value.
inline int32_t total_key(float f) {
  int32_t i;
  memcpy(&i, &f, 4);
  i ^= (int32_t)(((uint32_t)(i >> 31)) >> 1);
  return i;
}
// ops.rs:45-56 — descending by total_cmp, ties to the lower index, softmax of the kept logits.
void route(const float* logits, size_t n, size_t top, uint32_t* ids, float* weights) {
  ENSURE(top > 0 && top <= n, "invalid MoE router");
  for (size_t i = 0; i < n; i++) ENSURE(std::isfinite(logits[i]), "invalid MoE router");
  std::vector<uint32_t> idx(n);
  for (size_t i = 0; i < n; i++) idx[i] = (uint32_t)i;
  std::sort(idx.begin(), idx.end(), [&](uint32_t a, uint32_t b) {
    int32_t ka = total_key(logits[a]), kb = total_key(logits[b]);
    if (ka != kb) return ka > kb;
    return a < b;
  });
  for (size_t i = 0; i < top; i++) {
    ids[i] = idx[i];
    weights[i] = logits[idx[i]];
  }
  softmax(weights, top);
}
// ops.rs:57-98 — GQA causal attention over the whole cache, layout [t][kvhead][d].
void attention(const float* q, const float* k, const float* v, size_t heads, size_t kvheads, size_t d,
               size_t time, float* out, int threads = 1) {
  ENSURE(kvheads > 0 && heads > 0 && d > 0 && heads % kvheads == 0, "attention shape mismatch");
  ENSURE(time > 0, "empty KV cache");
  for (size_t i = 0; i < heads * d; i++) out[i] = 0.f;
  float sd = sqrtf((float)d);
  // heads are independent: one thread computes each head with the reference's arithmetic
  parallel_for(heads, time * d >= (1u << 16) ? threads : 1, [&](size_t hh) {
    std::vector<float> scores(time);
    size_t kh = hh / (heads / kvheads);
    const float* qs = q + hh * d;
    for (size_t t = 0; t < time; t++) {
      const float* kr = k + (t * kvheads + kh) * d;
      float acc = kSumInit;
      for (size_t j = 0; j < d; j++) acc = acc + qs[j] * kr[j];
      scores[t] = acc / sd;
    }
    softmax(scores.data(), time);
    for (size_t t = 0; t < time; t++) {
      float sc = scores[t];
      const float* vr = v + (t * kvheads + kh) * d;
      for (size_t j = 0; j < d; j++) out[hh * d + j] += sc * vr[j];
    }
  });
}

// ---------------------------------------------------------------- gguf.rs
struct Value {
  enum Kind { U, I, F, B, S, A } kind = U;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::vector<Value> arr;
  // serde_json::Value::as_u64
  bool as_u64(uint64_t* o) const {
    if (kind == U) { *o = u; return true; }
    if (kind == I && i >= 0) { *o = (uint64_t)i; return true; }
    return false;
  }
  // serde_json::Value::as_f64
  bool as_f64(double* o) const {
    if (kind == U) { *o = (double)u; return true; }
    if (kind == I) { *o = (double)i; return true; }
    if (kind == F) { *o = f; return true; }
    return false;
  }
};
struct Tensor {
  std::string name;
  std::vector<size_t> dims;
  uint32_t kind;
  size_t offset, len;
};
struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  size_t budget = 128u * 1024 * 1024;
  void take(void* out, size_t k) {
    ENSURE(k <= n - pos, "failed to fill whole buffer");
    memcpy(out, p + pos, k);
    pos += k;
  }
  uint8_t u8() { uint8_t v; take(&v, 1); return v; }
  uint32_t u32() { uint32_t v; take(&v, 4); return v; }
  uint64_t u64() { uint64_t v; take(&v, 8); return v; }
  size_t count(size_t max) {  // gguf.rs:44-48
    uint64_t c = u64();
    ENSURE(c <= max, "GGUF count " + std::to_string(c) + " exceeds limit " + std::to_string(max));
    return (size_t)c;
  }
  std::string str() {  // gguf.rs:49-56
    size_t c = count(16 * 1024 * 1024);
    ENSURE(c <= budget, "GGUF metadata budget exceeded");
    budget -= c;
    std::string s(c, '\0');
    take(s.data(), c);
    return s;
  }
  Value val(uint32_t t, size_t depth) {  // gguf.rs:57-99
    ENSURE(depth <= 4 && budget >= 8, "excessive metadata depth/size");
    budget -= 8;
    Value v;
    switch (t) {
      case 0: v.kind = Value::U; v.u = u8(); break;
      case 1: v.kind = Value::I; v.i = (int8_t)u8(); break;
      case 2: { uint16_t x; take(&x, 2); v.kind = Value::U; v.u = x; break; }
      case 3: { int16_t x; take(&x, 2); v.kind = Value::I; v.i = x; break; }
      case 4: v.kind = Value::U; v.u = u32(); break;
      case 5: { int32_t x; take(&x, 4); v.kind = Value::I; v.i = x; break; }
      case 6: {
        float x; take(&x, 4);
        ENSURE(std::isfinite(x), "nonfinite metadata");
        v.kind = Value::F; v.f = x; break;
      }
      case 7: {
        uint8_t x = u8();
        ENSURE(x <= 1, "invalid boolean");
        v.kind = Value::B; v.u = x; break;
      }
      case 8: v.kind = Value::S; v.s = str(); break;
      case 9: {
        uint32_t ty = u32();
        size_t c = count(1000000);
        v.kind = Value::A;
        for (size_t k = 0; k < c; k++) v.arr.push_back(val(ty, depth + 1));
        break;
      }
      case 10: v.kind = Value::U; v.u = u64(); break;
      case 11: { int64_t x; take(&x, 8); v.kind = Value::I; v.i = x; break; }
      case 12: {
        double x; take(&x, 8);
        ENSURE(std::isfinite(x), "nonfinite metadata");
        v.kind = Value::F; v.f = x; break;
      }
      default: fail("unknown GGUF metadata type " + std::to_string(t));
    }
    return v;
  }
};
struct Gguf {
  std::map<std::string, Value> meta;
  std::map<std::string, Tensor> tensors;
  const uint8_t* base = nullptr;
  size_t len = 0;
  void* map = nullptr;  // owned mmap, if any
  std::vector<uint8_t> owned;
  ~Gguf() {
    if (map) munmap(map, len);
  }
  // gguf.rs:102-195
  void parse() {
    Reader r{base, len};
    uint8_t magic[4];
    r.take(magic, 4);
    ENSURE(memcmp(magic, "GGUF", 4) == 0, "not a GGUF file");
    uint32_t ver = r.u32();
    ENSURE(ver == 2 || ver == 3, "GGUF version " + std::to_string(ver) + " unsupported");
    size_t nt = r.count(100000), nk = r.count(100000);
    for (size_t k = 0; k < nk; k++) {
      std::string key = r.str();
      uint32_t t = r.u32();
      Value v = r.val(t, 0);
      ENSURE(meta.emplace(key, std::move(v)).second, "duplicate metadata key");
    }
    auto sc = meta.find("split.count");
    uint64_t split = 1;
    if (sc != meta.end() && !sc->second.as_u64(&split)) split = 1;
    ENSURE(split == 1, "split GGUF not supported; merge shards first");
    for (size_t k = 0; k < nt; k++) {
      Tensor t;
      t.name = r.str();
      uint32_t nd = r.u32();
      ENSURE(nd >= 1 && nd <= 3, "unsupported tensor rank " + std::to_string(nd) + ": " + t.name);
      for (uint32_t d = 0; d < nd; d++) {
        uint64_t dd = r.u64();
        ENSURE(dd > 0, "zero tensor dimension");
        t.dims.push_back((size_t)dd);
      }
      t.kind = r.u32();
      t.offset = (size_t)r.u64();
      size_t l = row_bytes(t.kind, t.dims[0]);
      for (size_t d = 1; d < t.dims.size(); d++) {
        ENSURE(t.dims[d] == 0 || l <= SIZE_MAX / t.dims[d], "tensor length overflow");
        l *= t.dims[d];
      }
      t.len = l;
      std::string name = t.name;
      ENSURE(tensors.emplace(name, std::move(t)).second, "duplicate tensor name");
    }
    uint64_t alignment = 32;
    auto al = meta.find("general.alignment");
    if (al != meta.end() && !al->second.as_u64(&alignment)) alignment = 32;
    ENSURE(alignment && (alignment & (alignment - 1)) == 0 && alignment <= 4096, "invalid GGUF alignment");
    size_t start = (r.pos + alignment - 1) & ~(size_t)(alignment - 1);
    std::vector<std::pair<size_t, size_t>> ranges;
    for (auto& kv : tensors) {
      Tensor& t = kv.second;
      ENSURE(t.offset % alignment == 0, "unaligned tensor " + t.name);
      ENSURE(t.offset <= SIZE_MAX - start, "tensor offset overflow");
      t.offset += start;
      ENSURE(t.len <= SIZE_MAX - t.offset, "tensor end overflow");
      size_t end = t.offset + t.len;
      ENSURE(end <= len, "truncated tensor " + t.name);
      ranges.push_back({t.offset, end});
    }
    std::sort(ranges.begin(), ranges.end());
    for (size_t k = 1; k < ranges.size(); k++) ENSURE(ranges[k - 1].second <= ranges[k].first, "overlapping tensors");
  }
  const Tensor& tensor(const std::string& n) const {  // gguf.rs:196-200
    auto it = tensors.find(n);
    ENSURE(it != tensors.end(), "missing tensor " + n);
    return it->second;
  }
  const uint8_t* data(const Tensor& t) const { return base + t.offset; }
  std::vector<float> row(const std::string& n, size_t row) const {  // gguf.rs:204-213
    const Tensor& t = tensor(n);
    size_t size = row_bytes(t.kind, t.dims[0]);
    ENSURE(row < t.len / size, "row out of bounds: " + n);
    std::vector<float> out(t.dims[0]);
    const uint8_t* b = data(t) + row * size;
    for (size_t i = 0; i < t.dims[0]; i++) out[i] = value(b, t.kind, i);
    return out;
  }
  size_t uint(const std::string& key) const {  // gguf.rs:214-222
    auto it = meta.find(key);
    uint64_t v;
    ENSURE(it != meta.end() && it->second.as_u64(&v), "missing integer " + key);
    return (size_t)v;
  }
  float flt(const std::string& key, float def) const {  // gguf.rs:223-229
    auto it = meta.find(key);
    double v;
    if (it == meta.end() || !it->second.as_f64(&v)) return def;
    return (float)v;
  }
};

// ---------------------------------------------------------------- model.rs
struct Config {  // model.rs:5-19
  size_t hidden, layers, heads, kvheads, head_dim, experts, top, intermediate, vocab, max_context;
  float eps, theta;
};
Config config_from(const Gguf& m) {  // model.rs:21-90
  auto arch = m.meta.find("general.architecture");
  ENSURE(arch != m.meta.end() && arch->second.kind == Value::S && arch->second.s == "qwen3moe",
         "only qwen3moe architecture is implemented");
  auto get = [&](const std::string& k) { return m.uint("qwen3moe." + k); };
  auto has = [&](const std::string& k) {
    auto it = m.meta.find("qwen3moe." + k);
    uint64_t v;
    return it != m.meta.end() && it->second.as_u64(&v);
  };
  Config c{};
  c.hidden = get("embedding_length");
  c.heads = get("attention.head_count");
  c.top = get("expert_used_count");
  c.head_dim = has("attention.key_length") ? get("attention.key_length") : c.hidden / std::max<size_t>(c.heads, 1);
  size_t vl = has("attention.value_length") ? get("attention.value_length") : c.head_dim;
  ENSURE(vl == c.head_dim, "different key/value head sizes unsupported");
  c.layers = get("block_count");
  c.kvheads = get("attention.head_count_kv");
  c.experts = get("expert_count");
  c.intermediate = has("expert_feed_forward_length") ? get("expert_feed_forward_length")
                                                     : get("feed_forward_length") / std::max<size_t>(c.top, 1);
  const Tensor& te = m.tensor("token_embd.weight");
  ENSURE(te.dims.size() > 1, "invalid embedding rank");
  c.vocab = te.dims[1];
  c.max_context = get("context_length");
  c.eps = m.flt("qwen3moe.attention.layer_norm_rms_epsilon", 1e-6f);
  c.theta = m.flt("qwen3moe.rope.freq_base", 1000000.f);
  ENSURE(c.hidden > 0 && c.layers > 0 && c.layers <= 256 && c.kvheads > 0 && c.heads > 0 &&
             c.heads % c.kvheads == 0 && c.head_dim > 0 && c.head_dim % 2 == 0 && c.top > 0 &&
             c.top <= c.experts && c.experts <= 1024 && c.intermediate > 0 && std::isfinite(c.eps) &&
             c.eps > 0.f && std::isfinite(c.theta) && c.theta > 0.f,
         "invalid Qwen3 MoE config");
  size_t rd = has("rope.dimension_count") ? get("rope.dimension_count") : c.head_dim;
  ENSURE(rd == c.head_dim, "partial rotary dimensions unsupported");
  auto rs = m.meta.find("qwen3moe.rope.scaling.type");
  ENSURE(rs == m.meta.end() || rs->second.kind != Value::S || rs->second.s == "none",
         "RoPE scaling is not implemented; use the original native-context model");
  return c;
}
void validate_tensors(const Config& c, const Gguf& m) {  // model.rs:91-149
  auto check = [&](const std::string& n, std::vector<size_t> shape) {
    const Tensor& t = m.tensor(n);
    ENSURE(t.dims == shape, n + ": unexpected shape");
  };
  check("token_embd.weight", {c.hidden, c.vocab});
  check("output_norm.weight", {c.hidden});
  if (m.tensors.count("output.weight")) check("output.weight", {c.hidden, c.vocab});
  for (size_t i = 0; i < c.layers; i++) {
    std::string b = "blk." + std::to_string(i) + ".";
    check(b + "attn_norm.weight", {c.hidden});
    check(b + "ffn_norm.weight", {c.hidden});
    check(b + "attn_q_norm.weight", {c.head_dim});
    check(b + "attn_k_norm.weight", {c.head_dim});
    check(b + "attn_q.weight", {c.hidden, c.heads * c.head_dim});
    check(b + "attn_k.weight", {c.hidden, c.kvheads * c.head_dim});
    check(b + "attn_v.weight", {c.hidden, c.kvheads * c.head_dim});
    check(b + "attn_output.weight", {c.heads * c.head_dim, c.hidden});
    check(b + "ffn_gate_inp.weight", {c.hidden, c.experts});
    check(b + "ffn_gate_exps.weight", {c.hidden, c.intermediate, c.experts});
    check(b + "ffn_up_exps.weight", {c.hidden, c.intermediate, c.experts});
    check(b + "ffn_down_exps.weight", {c.intermediate, c.hidden, c.experts});
    for (auto& kv : m.tensors) {
      const std::string& n = kv.first;
      bool bias = n.size() >= 5 && n.compare(n.size() - 5, 5, ".bias") == 0;
      ENSURE(!(n.rfind(b, 0) == 0 && bias), "unexpected bias tensors");
    }
  }
}

struct Model {
  std::unique_ptr<Gguf> g;
  Config c;
  std::vector<std::vector<float>> kk, vv;  // per-layer fp32 KV, layout [t][kvhead][d]
  std::vector<std::vector<std::vector<float>>> norms;
  std::vector<float> output_norm;
  size_t position = 0, context = 0;
  int threads = 0;
  bool fast = false;  // block-decoding matvec (same results, for long test runs)
  uint64_t matvecs = 0;

  // backend.rs:57-75 (backend::matrix: rank check, expert slice) + Cpu::matvec
  std::vector<float> mv(const std::string& name, long expert, const std::vector<float>& x) {
    const Tensor& t = g->tensor(name);
    ENSURE(t.dims.size() == (expert >= 0 ? 3u : 2u), "matrix rank mismatch: " + name);
    size_t cols = t.dims[0], rows = t.dims[1];
    size_t len = row_bytes(t.kind, cols) * rows;
    size_t e = expert >= 0 ? (size_t)expert : 0;
    ENSURE(expert < 0 || e < t.dims[2], "expert out of bounds");
    ENSURE(cols == x.size(), "matvec shape mismatch " + name);
    std::vector<float> y(rows);
    matvec(g->data(t) + e * len, t.kind, rows, cols, x.data(), y.data(), threads, fast);
    matvecs++;
    return y;
  }
  void reset() {  // model.rs:202-208
    for (auto& k : kk) k.clear();
    for (auto& v : vv) v.clear();
    position = 0;
  }
  // model.rs:217-302.  With want_logits false the output projection (model.rs:289-301) is skipped
  // and an empty vector returned: a test-speed shortcut for prompt tokens whose logits nobody reads
  // (the KV cache and position advance exactly as in the full forward).
  std::vector<float> forward_inner(uint32_t token, bool want_logits = true) {
    ENSURE(position < context, "context limit " + std::to_string(context) + " reached");
    ENSURE(token < c.vocab, "token outside vocabulary");
    std::vector<float> x = g->row("token_embd.weight", token);
    size_t D = c.head_dim;
    for (size_t i = 0; i < c.layers; i++) {
      std::string base = "blk." + std::to_string(i);
      std::vector<float> xn = x;
      rms(xn.data(), norms[i][0].data(), xn.size(), c.eps);
      std::vector<float> q = mv(base + ".attn_q.weight", -1, xn);
      std::vector<float> k = mv(base + ".attn_k.weight", -1, xn);
      std::vector<float> v = mv(base + ".attn_v.weight", -1, xn);
      for (size_t o = 0; o + D <= q.size(); o += D) rms(q.data() + o, norms[i][1].data(), D, c.eps);
      for (size_t o = 0; o + D <= k.size(); o += D) rms(k.data() + o, norms[i][2].data(), D, c.eps);
      rope(q.data(), q.size(), D, position, c.theta);
      rope(k.data(), k.size(), D, position, c.theta);
      kk[i].insert(kk[i].end(), k.begin(), k.end());
      vv[i].insert(vv[i].end(), v.begin(), v.end());
      size_t time = kk[i].size() / (c.kvheads * D);
      std::vector<float> a(c.heads * D);
      ENSURE(q.size() == c.heads * D, "attention shape mismatch");
      attention(q.data(), kk[i].data(), vv[i].data(), c.heads, c.kvheads, D, time, a.data(), threads);
      std::vector<float> o = mv(base + ".attn_output.weight", -1, a);
      for (size_t j = 0; j < x.size(); j++) x[j] += o[j];
      xn = x;
      rms(xn.data(), norms[i][3].data(), xn.size(), c.eps);
      std::vector<float> logits = mv(base + ".ffn_gate_inp.weight", -1, xn);
      std::vector<uint32_t> ids(c.top);
      std::vector<float> w(c.top);
      route(logits.data(), logits.size(), c.top, ids.data(), w.data());
      std::vector<float> moe(c.hidden, 0.f);
      for (size_t s = 0; s < c.top; s++) {
        std::vector<float> gate = mv(base + ".ffn_gate_exps.weight", ids[s], xn);
        std::vector<float> up = mv(base + ".ffn_up_exps.weight", ids[s], xn);
        for (size_t j = 0; j < gate.size(); j++) {
          float gg = gate[j];
          gate[j] = (gg / (1.f + expf(-gg))) * up[j];
        }
        std::vector<float> down = mv(base + ".ffn_down_exps.weight", ids[s], gate);
        for (size_t j = 0; j < moe.size(); j++) moe[j] += w[s] * down[j];
      }
      for (size_t j = 0; j < x.size(); j++) x[j] += moe[j];
    }
    if (!want_logits) {
      position++;
      return {};
    }
    rms(x.data(), output_norm.data(), x.size(), c.eps);
    const char* out = g->tensors.count("output.weight") ? "output.weight" : "token_embd.weight";
    std::vector<float> logits = mv(out, -1, x);
    for (float f : logits) ENSURE(std::isfinite(f), "nonfinite model output");
    position++;
    return logits;
  }

  // forward_inner(token, false) for each of n tokens, computed layer by layer over all of them:
  // token t's layer-l step needs only the layer-l keys and values of tokens <= t, so this order
  // gives the same results as n sequential forwards, with each weight row decoded once per layer
  // instead of once per token.  Test and benchmark set-up only (a long prompt before the
  // positions a test checks); errors are raised before any state changes.
  void prefill(const uint32_t* toks, size_t n) {
    ENSURE(position + n <= context, "context limit " + std::to_string(context) + " reached");
    for (size_t t = 0; t < n; t++) ENSURE(toks[t] < c.vocab, "token outside vocabulary");
    if (n == 0) return;
    const size_t H = c.hidden, D = c.head_dim, QD = c.heads * D, KD = c.kvheads * D;
    std::vector<float> X(n * H), XN(n * H);
    for (size_t t = 0; t < n; t++) {
      std::vector<float> e = g->row("token_embd.weight", toks[t]);
      std::copy(e.begin(), e.end(), X.begin() + t * H);
    }
    auto mm = [&](const std::string& name, long expert, const float* in, size_t nin, size_t cols, float* out) {
      const Tensor& t = g->tensor(name);
      size_t rows = t.dims[1], len = row_bytes(t.kind, t.dims[0]) * rows;
      ENSURE(t.dims[0] == cols, "matvec shape mismatch " + name);
      matmul(g->data(t) + (expert >= 0 ? (size_t)expert : 0) * len, t.kind, rows, cols, in, nin, out, threads);
      matvecs += nin;
      return rows;
    };
    for (size_t i = 0; i < c.layers; i++) {
      std::string base = "blk." + std::to_string(i);
      XN = X;
      for (size_t t = 0; t < n; t++) rms(XN.data() + t * H, norms[i][0].data(), H, c.eps);
      std::vector<float> q(n * QD), k(n * KD), v(n * KD);
      mm(base + ".attn_q.weight", -1, XN.data(), n, H, q.data());
      mm(base + ".attn_k.weight", -1, XN.data(), n, H, k.data());
      mm(base + ".attn_v.weight", -1, XN.data(), n, H, v.data());
      for (size_t t = 0; t < n; t++) {
        float* qt = q.data() + t * QD;
        float* kt = k.data() + t * KD;
        for (size_t o = 0; o + D <= QD; o += D) rms(qt + o, norms[i][1].data(), D, c.eps);
        for (size_t o = 0; o + D <= KD; o += D) rms(kt + o, norms[i][2].data(), D, c.eps);
        rope(qt, QD, D, position + t, c.theta);
        rope(kt, KD, D, position + t, c.theta);
        kk[i].insert(kk[i].end(), kt, kt + KD);
        vv[i].insert(vv[i].end(), v.data() + t * KD, v.data() + (t + 1) * KD);
      }
      std::vector<float> a(n * QD, 0.f), o(n * H);
      for (size_t t = 0; t < n; t++)
        attention(q.data() + t * QD, kk[i].data(), vv[i].data(), c.heads, c.kvheads, D, position + t + 1,
                  a.data() + t * QD, threads);
      mm(base + ".attn_output.weight", -1, a.data(), n, QD, o.data());
      for (size_t j = 0; j < n * H; j++) X[j] += o[j];
      XN = X;
      for (size_t t = 0; t < n; t++) rms(XN.data() + t * H, norms[i][3].data(), H, c.eps);
      std::vector<float> rl(n * c.experts);
      mm(base + ".ffn_gate_inp.weight", -1, XN.data(), n, H, rl.data());
      std::vector<uint32_t> ids(n * c.top);
      std::vector<float> w(n * c.top);
      for (size_t t = 0; t < n; t++)
        route(rl.data() + t * c.experts, c.experts, c.top, ids.data() + t * c.top, w.data() + t * c.top);
      // every (token, slot) pair of an expert at once; down[t][s] kept for the combine in slot order
      const size_t I = c.intermediate;
      std::vector<float> down(n * c.top * H);
      for (uint32_t e = 0; e < c.experts; e++) {
        std::vector<size_t> pairs;
        for (size_t p = 0; p < n * c.top; p++)
          if (ids[p] == e) pairs.push_back(p);
        if (pairs.empty()) continue;
        const size_t np = pairs.size();
        std::vector<float> xin(np * H), gate(np * I), up(np * I), dn(np * H);
        for (size_t j = 0; j < np; j++)
          std::copy(XN.begin() + (pairs[j] / c.top) * H, XN.begin() + (pairs[j] / c.top + 1) * H, xin.begin() + j * H);
        mm(base + ".ffn_gate_exps.weight", e, xin.data(), np, H, gate.data());
        mm(base + ".ffn_up_exps.weight", e, xin.data(), np, H, up.data());
        for (size_t j = 0; j < np * I; j++) {
          float gg = gate[j];
          gate[j] = (gg / (1.f + expf(-gg))) * up[j];
        }
        mm(base + ".ffn_down_exps.weight", e, gate.data(), np, I, dn.data());
        for (size_t j = 0; j < np; j++) std::copy(dn.begin() + j * H, dn.begin() + (j + 1) * H, down.begin() + pairs[j] * H);
      }
      for (size_t t = 0; t < n; t++) {
        std::vector<float> moe(H, 0.f);
        for (size_t s2 = 0; s2 < c.top; s2++) {
          const float ws = w[t * c.top + s2];
          const float* d = down.data() + (t * c.top + s2) * H;
          for (size_t j = 0; j < H; j++) moe[j] += ws * d[j];
        }
        for (size_t j = 0; j < H; j++) X[t * H + j] += moe[j];
      }
    }
    position += n;
  }
};

Model* model_new(std::unique_ptr<Gguf> g, size_t context) {  // model.rs:173-201
  std::unique_ptr<Model> m(new Model);
  m->c = config_from(*g);
  validate_tensors(m->c, *g);
  ENSURE(context > 0 && context <= m->c.max_context,
         "context must be in 1..=" + std::to_string(m->c.max_context));
  for (size_t i = 0; i < m->c.layers; i++) {
    std::vector<std::vector<float>> n;
    for (const char* nm : {"attn_norm", "attn_q_norm", "attn_k_norm", "ffn_norm"})
      n.push_back(g->row("blk." + std::to_string(i) + "." + nm + ".weight", 0));
    m->norms.push_back(std::move(n));
  }
  m->output_norm = g->row("output_norm.weight", 0);
  m->kk.resize(m->c.layers);
  m->vv.resize(m->c.layers);
  m->context = context;
  m->g = std::move(g);
  return m.release();
}

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const Fail& e) {
    g_err = e.msg;
    return 1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

// ---- sampling.rs:9-65 with its random source ------------------------------------------------
// The reference draws from rand 0.8's StdRng seeded by SeedableRng::seed_from_u64.  Those crates
// (rand 0.8.5's StdRng = rand_chacha 0.3 ChaCha12Rng; rand_core 0.6.4 seed_from_u64) are not in the
// reference tree; their published algorithms are restated here:
//  * seed_from_u64: a PCG32 step per 4 seed bytes (state = state * 6364136223846793005 +
//    11634580027462260723, then the XSH-RR output of the new state, little-endian), 8 steps for the
//    32-byte ChaCha key;
//  * ChaCha12: the ChaCha block function (RFC 7539 quarter round) with 12 rounds over
//    ["expand 32-byte k", key, 64-bit block counter (words 12-13), 64-bit stream id 0 (words 14-15)],
//    the keystream read as consecutive little-endian u32 words from block 0;
//  * gen::<f32>(): (next_u32 >> 8) * 2^-24.
// The block function is pinned by the RFC 7539 block test vectors (20 rounds) in the tests; the
// rest has no golden in the reference (its test checks determinism only), so sampled ids are
// unpinned beyond greedy.
static inline uint32_t rotl32(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }
void chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]) {
  uint32_t x[16];
  memcpy(x, in, sizeof x);
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < rounds; r += 2) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; i++) out[i] = x[i] + in[i];
}
struct StdRngState {
  uint32_t key[8];
  uint64_t word = 0;  // position in the keystream, in u32 words
  void seed_from_u64(uint64_t state) {
    for (int i = 0; i < 8; i++) {
      state = state * 6364136223846793005ull + 11634580027462260723ull;
      const uint32_t xs = (uint32_t)(((state >> 18) ^ state) >> 27), rot = (uint32_t)(state >> 59);
      key[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
    word = 0;
  }
  uint32_t next_u32() {
    const uint64_t block = word / 16;
    uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u}, out[16];
    memcpy(in + 4, key, 32);
    in[12] = (uint32_t)block;
    in[13] = (uint32_t)(block >> 32);
    in[14] = in[15] = 0;
    chacha_block(in, 12, out);
    return out[word++ % 16];
  }
  float gen_f32() { return (float)(next_u32() >> 8) * (1.0f / 16777216.0f); }
};
struct Sampler {
  StdRngState rng;
  float temperature, top_p;
  size_t top_k;
};
// sampling.rs:26-65.  Sums are sequential left folds in sorted order, as in the Rust source.
uint32_t sample(Sampler& s, const float* logits, size_t n) {
  ENSURE(n > 0, "invalid logits");
  for (size_t i = 0; i < n; i++) ENSURE(std::isfinite(logits[i]), "invalid logits");
  std::vector<uint32_t> ids(n);
  for (size_t i = 0; i < n; i++) ids[i] = (uint32_t)i;
  std::sort(ids.begin(), ids.end(), [&](uint32_t a, uint32_t b) {
    int32_t ka = total_key(logits[a]), kb = total_key(logits[b]);
    if (ka != kb) return ka > kb;
    return a < b;
  });
  if (s.temperature == 0.f) return ids[0];
  if (s.top_k > 0) ids.resize(std::min(s.top_k, ids.size()));
  const float mx = logits[ids[0]];
  std::vector<float> probs(ids.size());
  for (size_t i = 0; i < ids.size(); i++) probs[i] = expf((logits[ids[i]] - mx) / s.temperature);
  float total = 0.f;
  for (float p : probs) total += p;
  float cumulative = 0.f;
  size_t keep = probs.size();
  for (size_t i = 0; i < probs.size(); i++) {
    cumulative += probs[i] / total;
    if (cumulative >= s.top_p) {
      keep = i + 1;
      break;
    }
  }
  probs.resize(keep);
  ids.resize(keep);
  float mass = 0.f;
  for (float p : probs) mass += p;
  float draw = s.rng.gen_f32() * mass;
  for (size_t i = 0; i < keep; i++) {
    if (draw < probs[i]) return ids[i];
    draw -= probs[i];
  }
  return ids.back();
}

}  // namespace

extern "C" {

const char* or_last_error(void) { return g_err.c_str(); }

int or_layout(uint32_t kind, size_t* block, size_t* bytes) {
  return guarded([&] { ENSURE(layout(kind, block, bytes), "GGML tensor type " + std::to_string(kind) + " is not supported"); });
}
int or_row_bytes(uint32_t kind, size_t cols, size_t* out) {
  return guarded([&] { *out = row_bytes(kind, cols); });
}
// quant.rs:81-84
int or_decode(const uint8_t* b, size_t len, uint32_t kind, size_t cols, float* out) {
  return guarded([&] {
    ENSURE(len >= row_bytes(kind, cols), "truncated quantized row");
    for (size_t i = 0; i < cols; i++) out[i] = value(b, kind, i);
  });
}
// Decodes `rows` consecutive rows (whole tensor or one expert slice).
int or_decode_rows(const uint8_t* b, uint32_t kind, size_t rows, size_t cols, float* out) {
  return guarded([&] {
    size_t rb = row_bytes(kind, cols);
    parallel_for(rows, 0, [&](size_t r) {
      for (size_t i = 0; i < cols; i++) out[r * cols + i] = value(b + r * rb, kind, i);
    });
  });
}
int or_matvec(const uint8_t* data, size_t len, uint32_t kind, size_t rows, size_t cols, const float* x, float* y,
              int threads) {
  return guarded([&] {
    ENSURE(rows > 0 && len >= row_bytes(kind, cols) * rows, "matvec shape mismatch");
    matvec(data, kind, rows, cols, x, y, threads);
  });
}
// The block-decoding form of or_matvec (identical results).
int or_matvec_fast(const uint8_t* data, size_t len, uint32_t kind, size_t rows, size_t cols, const float* x,
                   float* y, int threads) {
  return guarded([&] {
    ENSURE(rows > 0 && len >= row_bytes(kind, cols) * rows, "matvec shape mismatch");
    matvec(data, kind, rows, cols, x, y, threads, true);
  });
}
int or_rms(float* x, const float* w, size_t n, float eps) { return guarded([&] { rms(x, w, n, eps); }); }
void or_rope(float* x, size_t n, size_t head, size_t pos, float theta) { rope(x, n, head, pos, theta); }
int or_softmax(float* x, size_t n) { return guarded([&] { softmax(x, n); }); }
int or_route(const float* logits, size_t n, size_t top, uint32_t* ids, float* weights) {
  return guarded([&] { route(logits, n, top, ids, weights); });
}
int or_attention(const float* q, const float* k, const float* v, size_t heads, size_t kvheads, size_t d,
                 size_t time, float* out) {
  return guarded([&] { attention(q, k, v, heads, kvheads, d, time, out); });
}
// sampling.rs:26-35 — greedy: the first id after sorting by total_cmp descending, ties to the lower index.
int or_sample_greedy(const float* logits, size_t n, uint32_t* out) {
  return guarded([&] {
    ENSURE(n > 0, "invalid logits");
    for (size_t i = 0; i < n; i++) ENSURE(std::isfinite(logits[i]), "invalid logits");
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
      if (total_key(logits[i]) > total_key(logits[best])) best = i;
    *out = (uint32_t)best;
  });
}

void or_chacha_block(const uint32_t* in, int rounds, uint32_t* out) { chacha_block(in, rounds, out); }
// sampling.rs:10-25 (Sampler::new): parameter checks, then StdRng::seed_from_u64(seed).
void* or_sampler_new(uint64_t seed, float temperature, size_t top_k, float top_p) {
  Sampler* out = nullptr;
  int rc = guarded([&] {
    ENSURE(std::isfinite(temperature) && temperature >= 0.f && std::isfinite(top_p) && top_p > 0.f && top_p <= 1.f,
           "invalid sampling parameters");
    out = new Sampler;
    out->rng.seed_from_u64(seed);
    out->temperature = temperature;
    out->top_k = top_k;
    out->top_p = top_p;
  });
  return rc == 0 ? out : nullptr;
}
int or_sampler_sample(void* h, const float* logits, size_t n, uint32_t* out) {
  return guarded([&] { *out = sample(*static_cast<Sampler*>(h), logits, n); });
}
uint32_t or_sampler_next_u32(void* h) { return static_cast<Sampler*>(h)->rng.next_u32(); }
void or_sampler_key(void* h, uint32_t* key8) { memcpy(key8, static_cast<Sampler*>(h)->rng.key, 32); }
void or_sampler_free(void* h) { delete static_cast<Sampler*>(h); }
void* or_model_open(const char* path, size_t context, int threads) {
  Model* out = nullptr;
  int rc = guarded([&] {
    std::unique_ptr<Gguf> g(new Gguf);
    int fd = open(path, O_RDONLY);
    ENSURE(fd >= 0, std::string("open ") + path);
    struct stat st;
    fstat(fd, &st);
    g->len = (size_t)st.st_size;
    if (g->len) {
      g->map = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
      if (g->map == MAP_FAILED) g->map = nullptr;
    }
    close(fd);
    ENSURE(g->len == 0 || g->map, "mmap failed");
    g->base = (const uint8_t*)g->map;
    g->parse();
    out = model_new(std::move(g), context);
    out->threads = threads;
  });
  return rc == 0 ? out : nullptr;
}
// Borrows `buf` (the caller keeps it alive), like the reference's mmap.
void* or_model_from_memory(const uint8_t* buf, size_t len, size_t context, int threads) {
  Model* out = nullptr;
  int rc = guarded([&] {
    std::unique_ptr<Gguf> g(new Gguf);
    g->base = buf;
    g->len = len;
    g->parse();
    out = model_new(std::move(g), context);
    out->threads = threads;
  });
  return rc == 0 ? out : nullptr;
}
// model.rs:210-216 — on error the cache and position are reset.  logits == NULL skips the output
// projection (see forward_inner).
int or_model_forward(void* h, uint32_t token, float* logits) {
  Model* m = (Model*)h;
  std::vector<float> out;
  int rc = guarded([&] { out = m->forward_inner(token, logits != nullptr); });
  if (rc) {
    m->reset();
    return rc;
  }
  if (logits) memcpy(logits, out.data(), out.size() * sizeof(float));
  return 0;
}
// n forwards without logits (Model::prefill); on error the cache and position are reset.
int or_model_prefill(void* h, const uint32_t* tokens, size_t n) {
  Model* m = (Model*)h;
  int rc = guarded([&] { m->prefill(tokens, n); });
  if (rc) m->reset();
  return rc;
}
void or_model_reset(void* h) { ((Model*)h)->reset(); }
// Fast (block-decoding) matvecs on or off; results are identical either way.
void or_model_set_fast(void* h, int fast) { ((Model*)h)->fast = fast != 0; }
size_t or_model_position(void* h) { return ((Model*)h)->position; }
uint64_t or_model_matvecs(void* h) { return ((Model*)h)->matvecs; }
// hidden, layers, heads, kvheads, head_dim, experts, top, intermediate, vocab, max_context
void or_model_config(void* h, size_t* out10, float* eps_theta) {
  const Config& c = ((Model*)h)->c;
  size_t v[10] = {c.hidden, c.layers, c.heads, c.kvheads, c.head_dim, c.experts, c.top, c.intermediate, c.vocab, c.max_context};
  memcpy(out10, v, sizeof v);
  eps_theta[0] = c.eps;
  eps_theta[1] = c.theta;
}
void or_model_free(void* h) { delete (Model*)h; }
// Header parse only (gguf.rs:102-195); returns 0 when the file is accepted.
int or_gguf_check(const uint8_t* buf, size_t len) {
  return guarded([&] {
    Gguf g;
    g.base = buf;
    g.len = len;
    g.parse();
    g.base = nullptr;
  });
}
float or_f16_to_f32(uint16_t v) { return f16_to_f32(v); }

}  // extern "C"
