// Block quantizers and a synthetic Qwen3-MoE GGUF writer (host C++).
//
// The reference crate only decodes GGML blocks (quant.rs:36-80) and its only
// GGUF writer emits F32 tensors (tools/reference_fixture.py:21-66), so every
// quantized model used here is produced by this file.  Each encoder is derived
// from the reference decode formula of its format:
//   Q8_0  w = d * int8                                (quant.rs:46-49)
//   Q4_0  w = d * (nibble - 8)                        (quant.rs:40-45)
//   Q4_K  w = d*sc*q - dmin*m, 8 sub-blocks of 32     (quant.rs:50-62)
//   Q5_K  as Q4_K with a fifth bit from qh            (quant.rs:50-62)
//   Q6_K  w = d*sc*(q-32), 16 sub-blocks of 16        (quant.rs:63-77)
// The encoders pick scales from each sub-block's range; they are not tuned for
// quantization error, only for producing valid blocks that exercise every bit
// field.  Values come from a counter-based normal generator so a tensor is
// reproducible from (seed, tensor name) and can be generated in parallel.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qwen_tools.h"

namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
inline double unit(uint64_t h) { return ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

// Element i of the N(0,1) stream `key`: Box-Muller on pair i/2.
inline void normal_pair(uint64_t key, uint64_t pair, double* z0, double* z1) {
  double u1 = unit(mix64(key + 2 * pair)), u2 = unit(mix64(key + 2 * pair + 1));
  double r = std::sqrt(-2.0 * std::log(u1)), t = 6.283185307179586 * u2;
  *z0 = r * std::cos(t);
  *z1 = r * std::sin(t);
}

uint64_t stream_key(uint64_t seed, uint64_t stream) { return mix64(mix64(seed) ^ mix64(stream + 0x51ed270b)); }

template <class F>
void parallel_for(size_t n, int threads, F&& f) {
  size_t nt = threads > 0 ? (size_t)threads : std::max(1u, std::thread::hardware_concurrency());
  nt = std::min(nt, n ? n : 1);
  if (nt <= 1) {
    for (size_t i = 0; i < n; i++) f(i);
    return;
  }
  std::vector<std::thread> pool;
  for (size_t t = 0; t < nt; t++)
    pool.emplace_back([&, t] {
      size_t lo = n * t / nt, hi = n * (t + 1) / nt;
      for (size_t i = lo; i < hi; i++) f(i);
    });
  for (auto& th : pool) th.join();
}

// binary32 -> binary16, round to nearest even (overflow to inf, subnormals kept).
uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000u) {                                   // result subnormal or zero
    if (ax < 0x33000000u) return (uint16_t)sign;            // < 2^-25 rounds to 0
    uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126 - e;  // 14..24
    uint32_t v = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (v & 1))) v++;
    return (uint16_t)(sign | v);
  }
  uint32_t v = ((ax - 0x38000000u) >> 13);
  uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (v & 1))) v++;
  return (uint16_t)(sign | v);
}
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
inline void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}
inline int iround(float v) { return (int)std::nearbyint(v); }
inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void q8_0(const float* x, uint8_t* b) {
  float amax = 0;
  for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
  uint16_t d16 = f32_to_f16(amax / 127.f);
  float d = f16_to_f32(d16), id = d != 0 ? 1.f / d : 0.f;
  put16(b, d16);
  for (int i = 0; i < 32; i++) b[2 + i] = (uint8_t)(int8_t)clampi(iround(x[i] * id), -127, 127);
}
void q4_0(const float* x, uint8_t* b) {
  float amax = 0;
  for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
  uint16_t d16 = f32_to_f16(amax / 7.f);
  float d = f16_to_f32(d16), id = d != 0 ? 1.f / d : 0.f;
  put16(b, d16);
  for (int i = 0; i < 16; i++) {
    int lo = clampi(iround(x[i] * id) + 8, 0, 15), hi = clampi(iround(x[i + 16] * id) + 8, 0, 15);
    b[2 + i] = (uint8_t)(lo | (hi << 4));
  }
}
// Q4_K (levels=15) and Q5_K (levels=31).
void qk_45(const float* x, uint8_t* b, int levels) {
  float scale[8], mins[8];
  for (int j = 0; j < 8; j++) {
    float mn = x[j * 32], mx = x[j * 32];
    for (int i = 1; i < 32; i++) {
      mn = std::min(mn, x[j * 32 + i]);
      mx = std::max(mx, x[j * 32 + i]);
    }
    mn = std::min(mn, 0.f);
    mx = std::max(mx, 0.f);
    scale[j] = (mx - mn) / (float)levels;
    mins[j] = -mn;
  }
  float ms = 0, mm = 0;
  for (int j = 0; j < 8; j++) {
    ms = std::max(ms, scale[j]);
    mm = std::max(mm, mins[j]);
  }
  uint16_t d16 = f32_to_f16(ms / 63.f), m16 = f32_to_f16(mm / 63.f);
  float d = f16_to_f32(d16), dm = f16_to_f32(m16);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = (uint8_t)(d > 0 ? clampi((int)std::ceil(scale[j] / d), 0, 63) : 0);
    m[j] = (uint8_t)(dm > 0 ? clampi(iround(mins[j] / dm), 0, 63) : 0);
  }
  put16(b, d16);
  put16(b + 2, m16);
  uint8_t* s = b + 4;  // 12 packed bytes, inverse of quant.rs:25-34
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
  }
  uint8_t* qh = b + 16;
  uint8_t* qs = b + (levels == 15 ? 16 : 48);
  if (levels == 31) memset(qh, 0, 32);
  memset(qs, 0, 128);
  for (int i = 0; i < 256; i++) {
    int g = i / 32;
    float es = d * (float)sc[g], em = dm * (float)m[g];
    int q = es > 0 ? clampi(iround((x[i] + em) / es), 0, levels) : 0;
    qs[(i / 64) * 32 + i % 32] |= (uint8_t)((q & 15) << ((g % 2) * 4));
    if (levels == 31 && (q & 16)) qh[i % 32] |= (uint8_t)(1u << g);
  }
}
void q6_k(const float* x, uint8_t* b) {
  float scale[16];
  for (int j = 0; j < 16; j++) {
    float amax = 0;
    for (int i = 0; i < 16; i++) amax = std::max(amax, std::fabs(x[j * 16 + i]));
    scale[j] = amax / 31.f;
  }
  float ms = 0;
  for (int j = 0; j < 16; j++) ms = std::max(ms, scale[j]);
  uint16_t d16 = f32_to_f16(ms / 127.f);
  float d = f16_to_f32(d16);
  int8_t sc[16];
  for (int j = 0; j < 16; j++) sc[j] = (int8_t)(d > 0 ? clampi((int)std::ceil(scale[j] / d), -128, 127) : 0);
  memset(b, 0, 210);
  uint8_t *ql = b, *qh = b + 128;
  for (int i = 0; i < 256; i++) {
    float es = d * (float)sc[i / 16];
    int q = es != 0 ? clampi(iround(x[i] / es) + 32, 0, 63) : 32;
    int chunk = i / 128, j = i % 128, quarter = j / 32, lane = j % 32;
    ql[chunk * 64 + (quarter % 2) * 32 + lane] |= (uint8_t)((q & 15) << ((quarter / 2) * 4));
    qh[chunk * 32 + lane] |= (uint8_t)(((q >> 4) & 3) << (quarter * 2));
  }
  for (int j = 0; j < 16; j++) b[192 + j] = (uint8_t)sc[j];
  put16(b + 208, d16);
}

bool block_of(uint32_t kind, size_t* block, size_t* bytes) {
  switch (kind) {
    case QC_F32: *block = 1; *bytes = 4; return true;
    case QC_F16: *block = 1; *bytes = 2; return true;
    case QC_Q4_0: *block = 32; *bytes = 18; return true;
    case QC_Q8_0: *block = 32; *bytes = 34; return true;
    case QC_Q4_K: *block = 256; *bytes = 144; return true;
    case QC_Q5_K: *block = 256; *bytes = 176; return true;
    case QC_Q6_K: *block = 256; *bytes = 210; return true;
  }
  return false;
}

void quantize_blocks(uint32_t kind, const float* x, size_t n, uint8_t* out) {
  size_t block = 1, bytes = 0;
  if (!block_of(kind, &block, &bytes)) return;
  for (size_t k = 0; k < n / block; k++) {
    const float* xb = x + k * block;
    uint8_t* ob = out + k * bytes;
    switch (kind) {
      case QC_F32: memcpy(ob, xb, 4); break;
      case QC_F16: put16(ob, f32_to_f16(*xb)); break;
      case QC_Q4_0: q4_0(xb, ob); break;
      case QC_Q8_0: q8_0(xb, ob); break;
      case QC_Q4_K: qk_45(xb, ob, 15); break;
      case QC_Q5_K: qk_45(xb, ob, 31); break;
      case QC_Q6_K: q6_k(xb, ob); break;
    }
  }
}

// ---------------------------------------------------------------- GGUF image
struct TensorPlan {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order: dims[0] = columns
  uint32_t kind;
  float fill;      // norms: constant value; NaN = random N(0, std)
  float std;       // standard deviation of random weights
  uint64_t offset; // relative to the data section
  uint64_t bytes;
};

struct Writer {
  std::vector<uint8_t> h;
  void u32(uint32_t v) { h.insert(h.end(), (uint8_t*)&v, (uint8_t*)&v + 4); }
  void u64(uint64_t v) { h.insert(h.end(), (uint8_t*)&v, (uint8_t*)&v + 8); }
  void f32(float v) { h.insert(h.end(), (uint8_t*)&v, (uint8_t*)&v + 4); }
  void str(const std::string& s) {
    u64(s.size());
    h.insert(h.end(), s.begin(), s.end());
  }
  void kv_u32(const std::string& k, uint32_t v) { str(k); u32(4); u32(v); }
  void kv_f32(const std::string& k, float v) { str(k); u32(6); f32(v); }
  void kv_str(const std::string& k, const std::string& v) { str(k); u32(8); str(v); }
};

uint64_t name_stream(const std::string& s) {  // FNV-1a
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) h = (h ^ c) * 1099511628211ull;
  return h;
}

std::vector<TensorPlan> plan(const qct_spec& s) {
  std::vector<TensorPlan> t;
  const float nan = std::nanf("");
  uint64_t H = s.hidden, Q = (uint64_t)s.heads * s.head_dim, KV = (uint64_t)s.kvheads * s.head_dim;
  auto add = [&](std::string n, std::vector<uint64_t> d, uint32_t k, float fill) {
    t.push_back({std::move(n), std::move(d), k, fill, s.weight_std, 0, 0});
  };
  add("token_embd.weight", {H, s.vocab}, s.kind_embd, nan);
  add("output_norm.weight", {H}, QC_F32, s.norm_value);
  if (!s.tied_output) add("output.weight", {H, s.vocab}, s.kind_output, nan);
  for (uint32_t i = 0; i < s.layers; i++) {
    std::string b = "blk." + std::to_string(i) + ".";
    add(b + "attn_norm.weight", {H}, QC_F32, s.norm_value);
    add(b + "attn_q.weight", {H, Q}, s.kind_attn, nan);
    add(b + "attn_k.weight", {H, KV}, s.kind_attn, nan);
    add(b + "attn_v.weight", {H, KV}, s.kind_attn, nan);
    add(b + "attn_q_norm.weight", {s.head_dim}, QC_F32, s.norm_value);
    add(b + "attn_k_norm.weight", {s.head_dim}, QC_F32, s.norm_value);
    add(b + "attn_output.weight", {Q, H}, s.kind_attn_out ? s.kind_attn_out : s.kind_attn, nan);
    add(b + "ffn_norm.weight", {H}, QC_F32, s.norm_value);
    add(b + "ffn_gate_inp.weight", {H, s.experts}, s.kind_router, nan);
    add(b + "ffn_gate_exps.weight", {H, s.intermediate, s.experts}, s.kind_gate_up, nan);
    add(b + "ffn_up_exps.weight", {H, s.intermediate, s.experts}, s.kind_gate_up, nan);
    add(b + "ffn_down_exps.weight", {s.intermediate, H, s.experts}, s.kind_down, nan);
  }
  return t;
}

bool tensor_bytes(TensorPlan& p) {
  size_t block, bytes;
  if (!block_of(p.kind, &block, &bytes) || p.dims[0] % block) return false;
  uint64_t n = p.dims[0] / block * bytes;
  for (size_t d = 1; d < p.dims.size(); d++) n *= p.dims[d];
  p.bytes = n;
  return true;
}

Writer header(const qct_spec& s, std::vector<TensorPlan>& t) {
  Writer w;
  w.h.insert(w.h.end(), {'G', 'G', 'U', 'F'});
  w.u32(3);
  w.u64(t.size());
  size_t kv_count_at = w.h.size();
  w.u64(0);
  w.kv_str("general.architecture", "qwen3moe");
  w.kv_u32("qwen3moe.embedding_length", s.hidden);
  w.kv_u32("qwen3moe.block_count", s.layers);
  w.kv_u32("qwen3moe.attention.head_count", s.heads);
  w.kv_u32("qwen3moe.attention.head_count_kv", s.kvheads);
  w.kv_u32("qwen3moe.attention.key_length", s.head_dim);
  w.kv_u32("qwen3moe.attention.value_length", s.head_dim);
  w.kv_u32("qwen3moe.expert_count", s.experts);
  w.kv_u32("qwen3moe.expert_used_count", s.top);
  w.kv_u32("qwen3moe.expert_feed_forward_length", s.intermediate);
  w.kv_u32("qwen3moe.context_length", s.context_length);
  w.kv_f32("qwen3moe.rope.freq_base", s.theta);
  w.kv_f32("qwen3moe.attention.layer_norm_rms_epsilon", s.eps);
  uint64_t n_kv = 13;
  memcpy(w.h.data() + kv_count_at, &n_kv, 8);
  uint64_t off = 0;
  for (auto& p : t) {
    off = (off + 31) & ~31ull;
    p.offset = off;
    off += p.bytes;
    w.str(p.name);
    w.u32((uint32_t)p.dims.size());
    for (uint64_t d : p.dims) w.u64(d);
    w.u32(p.kind);
    w.u64(p.offset);
  }
  while (w.h.size() % 32) w.h.push_back(0);
  return w;
}

}  // namespace

extern "C" {

int qct_quantize(uint32_t kind, const float* x, size_t n, uint8_t* out, size_t out_len) {
  size_t block, bytes;
  if (!block_of(kind, &block, &bytes) || n % block) return -1;
  if (out_len < n / block * bytes) return -2;
  quantize_blocks(kind, x, n, out);
  return 0;
}

void qct_normal(uint64_t seed, uint64_t stream, uint64_t first, float mean, float std, float* out, size_t n) {
  uint64_t key = stream_key(seed, stream);
  for (size_t k = 0; k < n; k++) {
    uint64_t i = first + k;
    double z0, z1;
    normal_pair(key, i / 2, &z0, &z1);
    out[k] = (float)(mean + std * ((i & 1) ? z1 : z0));
  }
}

uint64_t qct_stream_of(const char* name) { return name_stream(name); }

float qct_f16_to_f32(uint16_t v) { return f16_to_f32(v); }
uint16_t qct_f32_to_f16(float v) { return f32_to_f16(v); }

// Random weights N(0, std) for `rows` rows of `cols`, quantized row by row.
// Element (r, c) is element r*cols + c of the (seed, stream) normal stream.
int qct_random_matrix(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t seed, uint64_t stream, float std,
                      uint8_t* out, size_t out_len, int threads) {
  size_t block, bytes;
  if (!block_of(kind, &block, &bytes) || cols % block) return -1;
  uint64_t rb = cols / block * bytes;
  if (out_len < rb * rows) return -2;
  uint64_t key = stream_key(seed, stream);
  const uint64_t chunk = 64;
  parallel_for((rows + chunk - 1) / chunk, threads, [&](size_t c) {
    std::vector<float> buf(cols);
    for (uint64_t r = c * chunk; r < std::min<uint64_t>(rows, (c + 1) * chunk); r++) {
      for (uint64_t k = 0; k < cols; k++) {
        uint64_t i = r * cols + k;
        double z0, z1;
        normal_pair(key, i / 2, &z0, &z1);
        buf[k] = (float)(std * ((i & 1) ? z1 : z0));
      }
      quantize_blocks(kind, buf.data(), cols, out + r * rb);
    }
  });
  return 0;
}

int qct_synth_size(const qct_spec* s, uint64_t* total) {
  auto t = plan(*s);
  for (auto& p : t)
    if (!tensor_bytes(p)) return -1;
  Writer w = header(*s, t);
  uint64_t end = 0;
  for (auto& p : t) end = p.offset + p.bytes;
  *total = w.h.size() + end;
  return 0;
}

int qct_synth_write(const qct_spec* s, uint8_t* out, uint64_t len, int threads) {
  auto t = plan(*s);
  for (auto& p : t)
    if (!tensor_bytes(p)) return -1;
  Writer w = header(*s, t);
  uint64_t data = w.h.size(), end = 0;
  for (auto& p : t) end = p.offset + p.bytes;
  if (len < data + end) return -2;
  memcpy(out, w.h.data(), data);
  memset(out + data, 0, end);
  for (auto& p : t) {
    uint8_t* dst = out + data + p.offset;
    uint64_t rows = 1;
    for (size_t d = 1; d < p.dims.size(); d++) rows *= p.dims[d];
    if (!std::isnan(p.fill)) {
      std::vector<float> v(p.dims[0] * rows, p.fill);
      quantize_blocks(p.kind, v.data(), v.size(), dst);
    } else {
      int rc = qct_random_matrix(p.kind, rows, p.dims[0], s->seed, name_stream(p.name), p.std, dst, p.bytes, threads);
      if (rc) return rc;
    }
  }
  return 0;
}

}  // extern "C"
