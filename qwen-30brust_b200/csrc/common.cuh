// Shared device code of the Qwen3-MoE decode engine (sm_100a): device layout
// descriptors, bit-exact dequant, and the dequant-fused dot products.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QC_DEV __device__ __forceinline__

namespace qc {

// GGML type ids (reference quant.rs:5-11).
enum Kind : uint32_t { F32 = 0, F16 = 1, Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

// Device layout of one matrix (or of expert 0 of an expert stack; expert e
// starts e*expert_stride bytes / e*d_expert_stride halves further).  A row is
// processed in "units" of 64 consecutive elements.
//
// Q4_K, Q5_K   raw GGUF super-blocks (144 / 176 bytes, already 16-aligned)
// Q6_K         per block: ql[128] qh[64] scales[16] (208 bytes); d in a plane
// Q8_0         per block: qs[32]; d in a plane; rows padded to an even block count
// Q4_0         per block: qs[16]; d in a plane; rows padded to an even block count
// F16, F32     raw rows padded with zeros to a multiple of 64 elements
struct MatDesc {
  const uint8_t* w;
  const __half* d;
  uint32_t kind, rows, cols;
  uint32_t units;  // ceil(cols / 64)
  uint32_t lpr;    // lanes cooperating on one row (power of two, divides units, <= 32)
  uint32_t upl;    // units per lane = units / lpr
  uint64_t row_stride;       // bytes between rows of the main plane
  uint64_t d_stride;         // halves between rows of the d plane
  uint64_t expert_stride;    // bytes between experts of the main plane
  uint64_t d_expert_stride;  // halves between experts of the d plane
};

__host__ __device__ inline bool uses_float_x(uint32_t kind) { return kind == F16 || kind == F32; }

QC_DEV uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
QC_DEV float h2f(__half h) { return __half2float(h); }
QC_DEV float h2f_bits(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffff))); }
QC_DEV uint32_t byte_of(uint32_t w, uint32_t i) { return (w >> (8 * i)) & 0xffu; }

// IEEE totalOrder key of f32::total_cmp (larger key == larger value), as an unsigned order.
QC_DEV uint32_t total_key_u(float f) {
  int32_t i = __float_as_int(f);
  i ^= (int32_t)(((uint32_t)(i >> 31)) >> 1);
  return (uint32_t)i ^ 0x80000000u;
}

QC_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QC_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over groups of `lpr` consecutive lanes (lpr a power of two <= 32); every lane gets its group's sum.
QC_DEV float group_sum(float v, uint32_t lpr) {
  for (uint32_t o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32; `red` holds >= 32 floats.  All threads get the result.
QC_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (w == 0) {
    t = l < nw ? red[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  t = red[0];
  return t;
}

// ---------------------------------------------------------------------------
// Per-element dequant, bit-exact with reference quant.rs:36-80.  Products are
// rounded separately (__fmul_rn / __fsub_rn) so the compiler cannot fuse
// d*sc*q - dmin*m into one multiply-add.
QC_DEV void kq_scale(const uint8_t* s, int j, int* sc, int* m) {  // quant.rs:25-34
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

QC_DEV float dequant_one(const MatDesc& m, const uint8_t* row, const __half* drow, uint32_t col) {
  switch (m.kind) {
    case F32: return reinterpret_cast<const float*>(row)[col];
    case F16: return h2f(reinterpret_cast<const __half*>(row)[col]);
    case Q4_0: {
      const uint8_t* b = row + (col / 32) * 16;
      uint32_t i = col % 32;
      int q = (b[i % 16] >> (i < 16 ? 0 : 4)) & 15;
      return __fmul_rn(h2f(drow[col / 32]), (float)(q - 8));
    }
    case Q8_0: {
      const int8_t* b = reinterpret_cast<const int8_t*>(row + (col / 32) * 32);
      return __fmul_rn(h2f(drow[col / 32]), (float)b[col % 32]);
    }
    case Q4_K:
    case Q5_K: {
      const uint32_t size = m.kind == Q4_K ? 144 : 176;
      const uint8_t* b = row + (col / 256) * size;
      uint32_t i = col % 256, g = i / 32;
      int sc, mn;
      kq_scale(b + 4, g, &sc, &mn);
      const uint8_t* qs = b + (m.kind == Q4_K ? 16 : 48);
      int q = (qs[(i / 64) * 32 + i % 32] >> ((g % 2) * 4)) & 15;
      if (m.kind == Q5_K && (b[16 + i % 32] & (1u << g))) q += 16;
      float d = h2f_bits(b[0] | (b[1] << 8)), dmin = h2f_bits(b[2] | (b[3] << 8));
      float a = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
      return __fsub_rn(a, __fmul_rn(dmin, (float)mn));
    }
    case Q6_K: {
      const uint8_t* b = row + (col / 256) * 208;
      uint32_t i = col % 256, chunk = i / 128, j = i % 128, quarter = j / 32, lane = j % 32;
      uint32_t lo = (b[chunk * 64 + (quarter % 2) * 32 + lane] >> ((quarter / 2) * 4)) & 15;
      uint32_t hi = (b[128 + chunk * 32 + lane] >> (quarter * 2)) & 3;
      int q = (int)(lo | (hi << 4)) - 32;
      float sc = (float)(int8_t)b[192 + chunk * 8 + quarter * 2 + lane / 16];
      return __fmul_rn(__fmul_rn(h2f(drow[col / 256]), sc), (float)q);
    }
  }
  return 0.f;
}

// ---------------------------------------------------------------------------
// Activation vector staged in shared memory for the fused dot products.
//
// x is quantized per block of 256 elements to 22-bit integers,
//   xi = rint(x * 2^21 / max|x_block|),  |xi| <= 2^21,
// and split into three signed byte digits, xi = d0 + 256 d1 + 65536 d2
// (d0, d1 in [-128, 127], |d2| <= 32).  Weight codes (nibbles, 6-bit, int8)
// then meet the activations in exact dp4a integer dot products; the only
// rounding is that of xi (2^-22 of the block maximum) and of the final float
// combination.  Per unit u (64 elements) the three digit planes are stored as
// [d0 x64][d1 x64][d2 x64][pad 16] = 208 bytes: the pad makes the 16-byte
// reads of 8 consecutive units fall in 8 different bank groups.
// F16/F32 matrices read a float copy instead: 64 floats + 4 pad per unit.
constexpr uint32_t kUnitDigitBytes = 208;
constexpr uint32_t kUnitFloats = 68;
constexpr float kXRange = 2097152.f;  // 2^21

struct XView {
  const uint8_t* dig;  // [units][208]
  const int* sx;       // [units][4]: sum of xi over each 16 elements
  const float* sb;     // [ceil(units/4)]: x scale of each 256-block (x = xi * sb)
  const float* xf;     // [units][68] padded float copy (F16/F32 only), may be null
};

// Shared-memory bytes of an XView for `units` units.
__host__ __device__ inline uint32_t xview_bytes(uint32_t units, bool with_float) {
  uint32_t b = units * kUnitDigitBytes + units * 16 + ((units + 3) / 4) * 4;
  b = (b + 15) & ~15u;
  if (with_float) b += units * kUnitFloats * 4;
  return b;
}

// Stage n values v(i) (i < n; zero beyond, up to units*64) into `mem` as an
// XView.  Called by all threads of the block; ends with __syncthreads().
// One warp per 256-block: max, scale, digits and sums in one pass.
template <class F>
QC_DEV XView stage_x(uint8_t* mem, uint32_t n, uint32_t units, bool with_float, F v) {
  uint8_t* dig = mem;
  int* sx = reinterpret_cast<int*>(mem + units * kUnitDigitBytes);
  float* sb = reinterpret_cast<float*>(sx + units * 4);
  float* xf = with_float ? reinterpret_cast<float*>(mem + ((units * kUnitDigitBytes + units * 16 + ((units + 3) / 4) * 4 + 15) & ~15u))
                         : nullptr;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const uint32_t nblk = (units + 3) / 4;
  for (uint32_t b = warp; b < nblk; b += nw) {
    // lane holds elements b*256 + lane*8 .. +7 (two groups of 4)
    float x[8];
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t i = b * 256 + lane * 8 + k;
      x[k] = (i < n) ? v(i) : 0.f;
      mx = fmaxf(mx, fabsf(x[k]));
    }
    mx = warp_max(mx);
    const float inv = mx > 0.f ? kXRange / mx : 0.f;
    if (lane == 0) sb[b] = mx > 0.f ? mx / kXRange : 0.f;
    const uint32_t u = b * 4 + lane / 8;  // unit of this lane's elements
    const uint32_t e = (lane % 8) * 8;    // element offset inside the unit
    int s = 0;
    uint32_t w0[2], w1[2], w2[2];
#pragma unroll
    for (int g = 0; g < 2; g++) {
      uint32_t p0 = 0, p1 = 0, p2 = 0;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        int xi = __float2int_rn(x[g * 4 + k] * inv);
        xi = max(-2097152, min(2097152, xi));
        s += xi;
        const int d0 = (int)(int8_t)(xi & 0xff);
        const int r1 = (xi - d0) >> 8;
        const int d1 = (int)(int8_t)(r1 & 0xff);
        const int d2 = (r1 - d1) >> 8;
        p0 |= (uint32_t)(d0 & 0xff) << (8 * k);
        p1 |= (uint32_t)(d1 & 0xff) << (8 * k);
        p2 |= (uint32_t)(d2 & 0xff) << (8 * k);
      }
      w0[g] = p0;
      w1[g] = p1;
      w2[g] = p2;
    }
    // sums over 16 elements: lanes (2j, 2j+1) of a unit hold one 16-group
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (u < units) {
      uint8_t* du = dig + u * kUnitDigitBytes + e;
      *reinterpret_cast<uint2*>(du) = make_uint2(w0[0], w0[1]);
      *reinterpret_cast<uint2*>(du + 64) = make_uint2(w1[0], w1[1]);
      *reinterpret_cast<uint2*>(du + 128) = make_uint2(w2[0], w2[1]);
      if ((lane & 1) == 0) sx[u * 4 + (lane % 8) / 2] = s;
      if (xf) {
        float* f = xf + u * kUnitFloats + e;
        *reinterpret_cast<float4*>(f) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(f + 4) = make_float4(x[4], x[5], x[6], x[7]);
      }
    }
  }
  __syncthreads();
  return XView{dig, sx, sb, xf};
}

QC_DEV int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// Dot of 32 codes (8 words of 4 bytes; codes are bytes: nibbles, 5/6-bit values
// or int8) with the 32 activation integers xi starting at element `e` of the
// unit: three exact dp4a sums, one per digit, combined in float (each digit sum
// is below 2^24 in magnitude, so only the final combination rounds).
struct Digits32 {
  uint4 p0[2], p1[2], p2[2];
};
QC_DEV Digits32 load_digits32(const uint8_t* du, uint32_t e) {
  Digits32 d;
  const uint4* a = reinterpret_cast<const uint4*>(du + e);
  d.p0[0] = a[0];
  d.p0[1] = a[1];
  d.p1[0] = a[4];
  d.p1[1] = a[5];
  d.p2[0] = a[8];
  d.p2[1] = a[9];
  return d;
}
QC_DEV uint32_t w4(const uint4 (&v)[2], int j) {
  const uint4& t = v[j >> 2];
  switch (j & 3) {
    case 0: return t.x;
    case 1: return t.y;
    case 2: return t.z;
    default: return t.w;
  }
}
QC_DEV float combine(int a0, int a1, int a2) { return (float)a0 + 256.f * (float)a1 + 65536.f * (float)a2; }
// codes[j] holds the 4 codes of elements 4j..4j+3.
QC_DEV float idot32(const uint32_t (&codes)[8], const Digits32& d) {
  int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    a0 = dp4a(codes[j], w4(d.p0, j), a0);
    a1 = dp4a(codes[j], w4(d.p1, j), a1);
    a2 = dp4a(codes[j], w4(d.p2, j), a2);
  }
  return combine(a0, a1, a2);
}
// As idot32 but split into the two 16-element halves (Q6_K scale groups).
QC_DEV void idot16x2(const uint32_t (&codes)[8], const Digits32& d, float* lo, float* hi) {
  int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    a0 = dp4a(codes[j], w4(d.p0, j), a0);
    a1 = dp4a(codes[j], w4(d.p1, j), a1);
    a2 = dp4a(codes[j], w4(d.p2, j), a2);
    b0 = dp4a(codes[j + 4], w4(d.p0, j + 4), b0);
    b1 = dp4a(codes[j + 4], w4(d.p1, j + 4), b1);
    b2 = dp4a(codes[j + 4], w4(d.p2, j + 4), b2);
  }
  *lo = combine(a0, a1, a2);
  *hi = combine(b0, b1, b2);
}

// 6-bit scale and min of sub-block j from the 12 packed bytes s0|s1|s2 (quant.rs:25-34).
QC_DEV void kq_scale_w(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t j, float* sc, float* m) {
  uint32_t a, b;
  if (j < 4) {
    a = byte_of(s0, j) & 63;
    b = byte_of(s1, j) & 63;
  } else {
    const uint32_t jj = j - 4;
    a = (byte_of(s2, jj) & 15) | ((byte_of(s0, jj) >> 6) << 4);
    b = (byte_of(s2, jj) >> 4) | ((byte_of(s1, jj) >> 6) << 4);
  }
  *sc = (float)a;
  *m = (float)b;
}

// ---- unit dot products: contribution of unit u (64 elements) of one row, in x units (times sb) ----

// Q4_K unit u = (block u/4, pair p = u%4): sub-blocks 2p (low nibbles) and 2p+1 (high nibbles).
QC_DEV float unit_q4k(const uint8_t* row, uint32_t u, const XView& xv) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 144;
  const uint4 hd = ldg16(blk);
  const uint4 q0 = ldg16(blk + 16 + 32 * p), q1 = ldg16(blk + 32 + 32 * p);
  const uint8_t* du = xv.dig + u * kUnitDigitBytes;
  const Digits32 dlo = load_digits32(du, 0), dhi = load_digits32(du, 32);
  const int4 s4 = *reinterpret_cast<const int4*>(xv.sx + u * 4);
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    lo[j] = w[j] & 0x0f0f0f0fu;
    hi[j] = (w[j] >> 4) & 0x0f0f0f0fu;
  }
  const float qlo = idot32(lo, dlo), qhi = idot32(hi, dhi);
  float sc0, m0, sc1, m1;
  kq_scale_w(hd.y, hd.z, hd.w, 2 * p, &sc0, &m0);
  kq_scale_w(hd.y, hd.z, hd.w, 2 * p + 1, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float r = sc0 * qlo + sc1 * qhi;
  const float mm = m0 * (float)(s4.x + s4.y) + m1 * (float)(s4.z + s4.w);
  return (d * r - dmin * mm) * xv.sb[b];
}

// Q5_K: as Q4_K plus the fifth bit: qh[t] bit g belongs to element 32g + t.
QC_DEV float unit_q5k(const uint8_t* row, uint32_t u, const XView& xv) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 176;
  const uint4 hd = ldg16(blk);
  const uint4 h0 = ldg16(blk + 16), h1 = ldg16(blk + 32);
  const uint4 q0 = ldg16(blk + 48 + 32 * p), q1 = ldg16(blk + 64 + 32 * p);
  const uint8_t* du = xv.dig + u * kUnitDigitBytes;
  const Digits32 dlo = load_digits32(du, 0), dhi = load_digits32(du, 32);
  const int4 s4 = *reinterpret_cast<const int4*>(xv.sx + u * 4);
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t h[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t g0 = 2 * p, g1 = 2 * p + 1;
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    lo[j] = (w[j] & 0x0f0f0f0fu) | (((h[j] >> g0) & 0x01010101u) << 4);
    hi[j] = ((w[j] >> 4) & 0x0f0f0f0fu) | (((h[j] >> g1) & 0x01010101u) << 4);
  }
  const float qlo = idot32(lo, dlo), qhi = idot32(hi, dhi);
  float sc0, m0, sc1, m1;
  kq_scale_w(hd.y, hd.z, hd.w, g0, &sc0, &m0);
  kq_scale_w(hd.y, hd.z, hd.w, g1, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float r = sc0 * qlo + sc1 * qhi;
  const float mm = m0 * (float)(s4.x + s4.y) + m1 * (float)(s4.z + s4.w);
  return (d * r - dmin * mm) * xv.sb[b];
}

// Q6_K unit u = (block u/4, chunk c = (u/2)%2, half h = u%2): quarters 2h (elements
// c*128+64h+t) and 2h+1 (c*128+64h+32+t), t < 32; four 16-element scale groups.
QC_DEV float unit_q6k(const uint8_t* row, const __half* drow, uint32_t u, const XView& xv) {
  const uint32_t b = u >> 2, c = (u >> 1) & 1, hh = u & 1;
  const uint8_t* blk = row + b * 208;
  const uint4 l0 = ldg16(blk + c * 64), l1 = ldg16(blk + c * 64 + 16);        // quarter 2h: ql[c*64 + t]
  const uint4 l2 = ldg16(blk + c * 64 + 32), l3 = ldg16(blk + c * 64 + 48);   // quarter 2h+1: ql[c*64+32+t]
  const uint4 qa = ldg16(blk + 128 + c * 32), qb = ldg16(blk + 128 + c * 32 + 16);
  const uint4 sc = ldg16(blk + 192);
  const uint8_t* du = xv.dig + u * kUnitDigitBytes;
  const Digits32 d0 = load_digits32(du, 0), d1 = load_digits32(du, 32);
  const int4 s4 = *reinterpret_cast<const int4*>(xv.sx + u * 4);
  const uint32_t la[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  const uint32_t lb[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
  const uint32_t qh[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  const uint32_t ns = 4 * hh, s0 = 2 * (2 * hh), s1 = 2 * (2 * hh + 1);
  uint32_t ca[8], cb[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    ca[j] = ((la[j] >> ns) & 0x0f0f0f0fu) | (((qh[j] >> s0) & 0x03030303u) << 4);
    cb[j] = ((lb[j] >> ns) & 0x0f0f0f0fu) | (((qh[j] >> s1) & 0x03030303u) << 4);
  }
  float qa0, qa1, qb0, qb1;
  idot16x2(ca, d0, &qa0, &qa1);
  idot16x2(cb, d1, &qb0, &qb1);
  // scales: quarter q group t/16 -> sc[c*8 + 2q + t/16]
  // the four scales sit in bytes c*8 + 4h .. +3, i.e. in word 2c + h of the 16 scale bytes
  const uint32_t sw = (c ? (hh ? sc.w : sc.z) : (hh ? sc.y : sc.x));
  const float sa0 = (float)(int8_t)byte_of(sw, 0), sa1 = (float)(int8_t)byte_of(sw, 1);
  const float sb0 = (float)(int8_t)byte_of(sw, 2), sb1 = (float)(int8_t)byte_of(sw, 3);
  // sum (q - 32) x = sum q x - 32 sum x over each 16-element group
  const float r = sa0 * (qa0 - 32.f * (float)s4.x) + sa1 * (qa1 - 32.f * (float)s4.y) +
                  sb0 * (qb0 - 32.f * (float)s4.z) + sb1 * (qb1 - 32.f * (float)s4.w);
  return h2f(drow[b]) * r * xv.sb[b];
}

// Q8_0 unit u = blocks 2u and 2u+1.
QC_DEV float unit_q80(const uint8_t* row, const __half* drow, uint32_t u, const XView& xv) {
  const uint8_t* blk = row + u * 64;
  const uint4 a = ldg16(blk), b = ldg16(blk + 16), c = ldg16(blk + 32), e = ldg16(blk + 48);
  const uint8_t* du = xv.dig + u * kUnitDigitBytes;
  const Digits32 d0 = load_digits32(du, 0), d1 = load_digits32(du, 32);
  const uint32_t w0[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t w1[8] = {c.x, c.y, c.z, c.w, e.x, e.y, e.z, e.w};
  const float q0 = idot32(w0, d0), q1 = idot32(w1, d1);
  const __half2 dd = *reinterpret_cast<const __half2*>(drow + 2 * u);
  return (__low2float(dd) * q0 + __high2float(dd) * q1) * xv.sb[u >> 2];
}

// Q4_0 unit u = blocks 2u, 2u+1; byte t of a block holds elements t (low) and 16+t (high).
QC_DEV float unit_q40(const uint8_t* row, const __half* drow, uint32_t u, const XView& xv) {
  const uint4 a = ldg16(row + u * 32), b = ldg16(row + u * 32 + 16);
  const uint8_t* du = xv.dig + u * kUnitDigitBytes;
  const Digits32 d0 = load_digits32(du, 0), d1 = load_digits32(du, 32);
  const int4 s4 = *reinterpret_cast<const int4*>(xv.sx + u * 4);
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
  uint32_t c0[8], c1[8];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    c0[j] = wa[j] & 0x0f0f0f0fu;
    c0[j + 4] = (wa[j] >> 4) & 0x0f0f0f0fu;
    c1[j] = wb[j] & 0x0f0f0f0fu;
    c1[j + 4] = (wb[j] >> 4) & 0x0f0f0f0fu;
  }
  const float q0 = idot32(c0, d0), q1 = idot32(c1, d1);
  const __half2 dd = *reinterpret_cast<const __half2*>(drow + 2 * u);
  const float r0 = q0 - 8.f * (float)(s4.x + s4.y), r1 = q1 - 8.f * (float)(s4.z + s4.w);
  return (__low2float(dd) * r0 + __high2float(dd) * r1) * xv.sb[u >> 2];
}

QC_DEV float unit_f16(const uint8_t* row, uint32_t u, const XView& xv) {
  const uint8_t* p = row + u * 128;
  const float* x = xv.xf + u * kUnitFloats;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint4 v = ldg16(p + 16 * k);
    const float4 xa = *reinterpret_cast<const float4*>(x + 8 * k), xb = *reinterpret_cast<const float4*>(x + 8 * k + 4);
    float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    acc = fmaf(f.x, xa.x, acc);
    acc = fmaf(f.y, xa.y, acc);
    f = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    acc = fmaf(f.x, xa.z, acc);
    acc = fmaf(f.y, xa.w, acc);
    f = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
    acc = fmaf(f.x, xb.x, acc);
    acc = fmaf(f.y, xb.y, acc);
    f = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
    acc = fmaf(f.x, xb.z, acc);
    acc = fmaf(f.y, xb.w, acc);
  }
  return acc;
}

QC_DEV float unit_f32(const uint8_t* row, uint32_t u, const XView& xv) {
  const uint8_t* p = row + u * 256;
  const float* x = xv.xf + u * kUnitFloats;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const uint4 v = ldg16(p + 16 * k);
    const float4 xv4 = *reinterpret_cast<const float4*>(x + 4 * k);
    acc = fmaf(__uint_as_float(v.x), xv4.x, acc);
    acc = fmaf(__uint_as_float(v.y), xv4.y, acc);
    acc = fmaf(__uint_as_float(v.z), xv4.z, acc);
    acc = fmaf(__uint_as_float(v.w), xv4.w, acc);
  }
  return acc;
}

template <uint32_t KIND>
QC_DEV float unit_dot(const uint8_t* row, const __half* drow, uint32_t u, const XView& xv) {
  if constexpr (KIND == Q4_K) return unit_q4k(row, u, xv);
  else if constexpr (KIND == Q5_K) return unit_q5k(row, u, xv);
  else if constexpr (KIND == Q6_K) return unit_q6k(row, drow, u, xv);
  else if constexpr (KIND == Q8_0) return unit_q80(row, drow, u, xv);
  else if constexpr (KIND == Q4_0) return unit_q40(row, drow, u, xv);
  else if constexpr (KIND == F16) return unit_f16(row, u, xv);
  else return unit_f32(row, u, xv);
}

// This lane's partial of row `r` of expert `e`: units lane_in_row, +lpr, ... (the
// caller sums the partials of the lpr lanes of the row).
template <uint32_t KIND>
QC_DEV float row_partial_k(const MatDesc& m, uint32_t e, uint32_t r, uint32_t lane_in_row, const XView& xv) {
  const uint8_t* row = m.w + e * m.expert_stride + (uint64_t)r * m.row_stride;
  const __half* drow = m.d ? m.d + e * m.d_expert_stride + (uint64_t)r * m.d_stride : nullptr;
  float acc = 0.f;
#pragma unroll 2
  for (uint32_t k = 0; k < m.upl; k++) acc += unit_dot<KIND>(row, drow, lane_in_row + k * m.lpr, xv);
  return acc;
}

QC_DEV float row_partial(const MatDesc& m, uint32_t e, uint32_t r, uint32_t lane_in_row, const XView& xv) {
  switch (m.kind) {
    case Q4_K: return row_partial_k<Q4_K>(m, e, r, lane_in_row, xv);
    case Q5_K: return row_partial_k<Q5_K>(m, e, r, lane_in_row, xv);
    case Q6_K: return row_partial_k<Q6_K>(m, e, r, lane_in_row, xv);
    case Q8_0: return row_partial_k<Q8_0>(m, e, r, lane_in_row, xv);
    case Q4_0: return row_partial_k<Q4_0>(m, e, r, lane_in_row, xv);
    case F16: return row_partial_k<F16>(m, e, r, lane_in_row, xv);
    default: return row_partial_k<F32>(m, e, r, lane_in_row, xv);
  }
}

}  // namespace qc
