// Shared device helpers for the Qwen3-MoE decode engine (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QC_DEV __device__ __forceinline__

namespace qc {

// GGML type ids (reference quant.rs:5-11).
enum Kind : uint32_t { F32 = 0, F16 = 1, Q4_0 = 2, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

// Device layout of one matrix (or of expert 0 of an expert stack; expert e
// starts e*expert_stride bytes / e*d_expert_stride halves further).
//
// Q4_K, Q5_K      raw GGUF super-blocks (144 / 176 bytes, already 16-aligned)
// Q6_K            per block: ql[128] qh[64] scales[16] (208 bytes) + d in a plane
// Q8_0            per block: qs[32] + d in a plane
// Q4_0            per block: qs[16] + d in a plane
// F16, F32        raw rows padded with zeros to a multiple of 64 bytes
struct MatDesc {
  const uint8_t* w;
  const __half* d;
  uint32_t kind, rows, cols;
  uint32_t units;  // work units per row (unit_elems() elements each)
  uint32_t lpr;    // lanes cooperating on one row (power of two, divides units, <= 32)
  uint32_t upl;    // units per lane = units / lpr
  uint64_t row_stride;       // bytes between rows of the main plane
  uint64_t d_stride;         // halves between rows of the d plane
  uint64_t expert_stride;    // bytes between experts of the main plane
  uint64_t d_expert_stride;  // halves between experts of the d plane
};

__host__ __device__ inline uint32_t unit_elems(uint32_t kind) {
  switch (kind) {
    case Q4_K: case Q5_K: case Q6_K: return 64;
    case Q8_0: case Q4_0: return 32;
    case F16: return 32;
    default: return 16;  // F32
  }
}

QC_DEV uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
QC_DEV float h2f(__half h) { return __half2float(h); }
QC_DEV float h2f_bits(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffff))); }

// IEEE totalOrder key of f32::total_cmp (larger key == larger value), as an unsigned order.
QC_DEV uint32_t total_key_u(float f) {
  int32_t i = __float_as_int(f);
  i ^= (int32_t)(((uint32_t)(i >> 31)) >> 1);
  return (uint32_t)i ^ 0x80000000u;
}

template <int W = 32>
QC_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
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
// Fused dequant dot products: the contribution of one work unit of a row to
// sum_i w_i * x_i.  `xs` is the activation vector in shared memory, zero
// padded to units*unit_elems.  The per-sub-block scales are factored out of the
// inner sums (sum (d*sc*q - dmin*m) x = d*sc * sum q x - dmin*m * sum x); the
// result differs from the reference's element-by-element fold only by fp32
// rounding of the reordered sum.

// Four consecutive floats of shared memory.
QC_DEV float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// sum over the 4 nibbles (bits 4k..4k+3 of every byte of w, k = 0 or 1) times 4 floats.
QC_DEV void nib_dot(uint32_t w, int shift, float4 x, float& acc, float& xsum) {
  const uint32_t q = (w >> shift) & 0x0f0f0f0fu;
  acc = fmaf((float)(q & 0xff), x.x, acc);
  acc = fmaf((float)((q >> 8) & 0xff), x.y, acc);
  acc = fmaf((float)((q >> 16) & 0xff), x.z, acc);
  acc = fmaf((float)(q >> 24), x.w, acc);
  xsum += (x.x + x.y) + (x.z + x.w);
}

// Q4_K unit u = (block u/4, pair u%4): sub-blocks 2p (low nibbles) and 2p+1 (high nibbles).
QC_DEV float unit_q4k(const uint8_t* row, uint32_t u, const float* xs) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 144;
  const uint4 hd = ldg16(blk);
  const uint4 q0 = ldg16(blk + 16 + 32 * p), q1 = ldg16(blk + 32 + 32 * p);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(&hd) + 4;
  int sc0, m0, sc1, m1;
  kq_scale(s, 2 * p, &sc0, &m0);
  kq_scale(s, 2 * p + 1, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float* x0 = xs + b * 256 + 64 * p;  // low nibbles: elements 64p + t
  const float* x1 = x0 + 32;                // high nibbles: elements 64p + 32 + t
  float a0 = 0.f, a1 = 0.f, s0 = 0.f, s1 = 0.f;
  const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int k = 0; k < 8; k++) {
    nib_dot(wq[k], 0, lds4(x0 + 4 * k), a0, s0);
    nib_dot(wq[k], 4, lds4(x1 + 4 * k), a1, s1);
  }
  return (d * (float)sc0) * a0 - (dmin * (float)m0) * s0 + (d * (float)sc1) * a1 - (dmin * (float)m1) * s1;
}

// Q5_K: as Q4_K plus the fifth bit: qh[t] bit g belongs to element 32g + t.
QC_DEV float unit_q5k(const uint8_t* row, uint32_t u, const float* xs) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 176;
  const uint4 hd = ldg16(blk);
  const uint4 h0 = ldg16(blk + 16), h1 = ldg16(blk + 32);
  const uint4 q0 = ldg16(blk + 48 + 32 * p), q1 = ldg16(blk + 64 + 32 * p);
  const uint8_t* s = reinterpret_cast<const uint8_t*>(&hd) + 4;
  int sc0, m0, sc1, m1;
  kq_scale(s, 2 * p, &sc0, &m0);
  kq_scale(s, 2 * p + 1, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float* x0 = xs + b * 256 + 64 * p;
  const float* x1 = x0 + 32;
  float a0 = 0.f, a1 = 0.f, s0 = 0.f, s1 = 0.f;
  const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t wh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const int g0 = 2 * p, g1 = 2 * p + 1;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    // fifth bits of the 4 bytes of wh[k], moved to bit 4 of each byte
    const uint32_t hb0 = ((wh[k] >> g0) & 0x01010101u) << 4, hb1 = ((wh[k] >> g1) & 0x01010101u) << 4;
    const uint32_t lo = (wq[k] & 0x0f0f0f0fu) | hb0, hi = ((wq[k] >> 4) & 0x0f0f0f0fu) | hb1;
    const float4 xa = lds4(x0 + 4 * k), xb = lds4(x1 + 4 * k);
    a0 = fmaf((float)(lo & 0xff), xa.x, a0);
    a0 = fmaf((float)((lo >> 8) & 0xff), xa.y, a0);
    a0 = fmaf((float)((lo >> 16) & 0xff), xa.z, a0);
    a0 = fmaf((float)(lo >> 24), xa.w, a0);
    a1 = fmaf((float)(hi & 0xff), xb.x, a1);
    a1 = fmaf((float)((hi >> 8) & 0xff), xb.y, a1);
    a1 = fmaf((float)((hi >> 16) & 0xff), xb.z, a1);
    a1 = fmaf((float)(hi >> 24), xb.w, a1);
    s0 += (xa.x + xa.y) + (xa.z + xa.w);
    s1 += (xb.x + xb.y) + (xb.z + xb.w);
  }
  return (d * (float)sc0) * a0 - (dmin * (float)m0) * s0 + (d * (float)sc1) * a1 - (dmin * (float)m1) * s1;
}

// Q6_K unit u = (block u/4, chunk (u/2)%2, half u%2): elements c*128 + 32q + 16h + t, q<4, t<16.
QC_DEV float unit_q6k(const uint8_t* row, const __half* drow, uint32_t u, const float* xs) {
  const uint32_t b = u >> 2, c = (u >> 1) & 1, hh = u & 1;
  const uint8_t* blk = row + b * 208;
  const uint4 l0 = ldg16(blk + c * 64 + 16 * hh);       // quarters 0 (low nibble) and 2 (high nibble)
  const uint4 l1 = ldg16(blk + c * 64 + 32 + 16 * hh);  // quarters 1 and 3
  const uint4 qh = ldg16(blk + 128 + c * 32 + 16 * hh); // two bits per quarter
  const uint4 sc = ldg16(blk + 192);
  const int8_t* scb = reinterpret_cast<const int8_t*>(&sc) + c * 8 + hh;
  const float d = h2f(drow[b]);
  const float* xb = xs + b * 256 + c * 128 + 16 * hh;
  const uint32_t wl0[4] = {l0.x, l0.y, l0.z, l0.w}, wl1[4] = {l1.x, l1.y, l1.z, l1.w};
  const uint32_t wh[4] = {qh.x, qh.y, qh.z, qh.w};
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, xsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int k = 0; k < 4; k++) {  // 4 bytes (t = 4k..4k+3) at a time
    const uint32_t qv[4] = {
        (wl0[k] & 0x0f0f0f0fu) | ((wh[k] & 0x03030303u) << 4),
        (wl1[k] & 0x0f0f0f0fu) | (((wh[k] >> 2) & 0x03030303u) << 4),
        ((wl0[k] >> 4) & 0x0f0f0f0fu) | (((wh[k] >> 4) & 0x03030303u) << 4),
        ((wl1[k] >> 4) & 0x0f0f0f0fu) | (((wh[k] >> 6) & 0x03030303u) << 4)};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float4 x = lds4(xb + 32 * q + 4 * k);
      acc[q] = fmaf((float)(qv[q] & 0xff), x.x, acc[q]);
      acc[q] = fmaf((float)((qv[q] >> 8) & 0xff), x.y, acc[q]);
      acc[q] = fmaf((float)((qv[q] >> 16) & 0xff), x.z, acc[q]);
      acc[q] = fmaf((float)(qv[q] >> 24), x.w, acc[q]);
      xsum[q] += (x.x + x.y) + (x.z + x.w);
    }
  }
  float r = 0.f;
#pragma unroll
  for (int q = 0; q < 4; q++) r += (d * (float)scb[2 * q]) * (acc[q] - 32.f * xsum[q]);
  return r;
}

// Q8_0 unit = one block of 32.
QC_DEV float unit_q80(const uint8_t* row, const __half* drow, uint32_t u, const float* xs) {
  const uint8_t* blk = row + u * 32;
  const uint4 a = ldg16(blk), b = ldg16(blk + 16);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const float* x = xs + u * 32;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const float4 xv = lds4(x + 4 * k);
    acc = fmaf((float)(int8_t)(w[k] & 0xff), xv.x, acc);
    acc = fmaf((float)(int8_t)((w[k] >> 8) & 0xff), xv.y, acc);
    acc = fmaf((float)(int8_t)((w[k] >> 16) & 0xff), xv.z, acc);
    acc = fmaf((float)(int8_t)(w[k] >> 24), xv.w, acc);
  }
  return h2f(drow[u]) * acc;
}

// Q4_0 unit = one block of 32: byte t holds elements t (low nibble) and 16 + t (high nibble).
QC_DEV float unit_q40(const uint8_t* row, const __half* drow, uint32_t u, const float* xs) {
  const uint4 a = ldg16(row + u * 16);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
  const float* x = xs + u * 32;
  float acc = 0.f, sum = 0.f;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    nib_dot(w[k], 0, lds4(x + 4 * k), acc, sum);
    nib_dot(w[k], 4, lds4(x + 16 + 4 * k), acc, sum);
  }
  return h2f(drow[u]) * (acc - 8.f * sum);
}

QC_DEV float unit_f16(const uint8_t* row, uint32_t u, const float* xs) {
  const uint8_t* p = row + u * 64;
  const float* x = xs + u * 32;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint4 v = ldg16(p + 16 * k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      const float2 xv = *reinterpret_cast<const float2*>(x + 8 * k + 2 * j);
      acc = fmaf(f.x, xv.x, acc);
      acc = fmaf(f.y, xv.y, acc);
    }
  }
  return acc;
}

QC_DEV float unit_f32(const uint8_t* row, uint32_t u, const float* xs) {
  const uint8_t* p = row + u * 64;
  const float* x = xs + u * 16;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const uint4 v = ldg16(p + 16 * k);
    const float4 xv = lds4(x + 4 * k);
    acc = fmaf(__uint_as_float(v.x), xv.x, acc);
    acc = fmaf(__uint_as_float(v.y), xv.y, acc);
    acc = fmaf(__uint_as_float(v.z), xv.z, acc);
    acc = fmaf(__uint_as_float(v.w), xv.w, acc);
  }
  return acc;
}

template <uint32_t KIND>
QC_DEV float unit_dot(const uint8_t* row, const __half* drow, uint32_t u, const float* xs) {
  if constexpr (KIND == Q4_K) return unit_q4k(row, u, xs);
  else if constexpr (KIND == Q5_K) return unit_q5k(row, u, xs);
  else if constexpr (KIND == Q6_K) return unit_q6k(row, drow, u, xs);
  else if constexpr (KIND == Q8_0) return unit_q80(row, drow, u, xs);
  else if constexpr (KIND == Q4_0) return unit_q40(row, drow, u, xs);
  else if constexpr (KIND == F16) return unit_f16(row, u, xs);
  else return unit_f32(row, u, xs);
}

// This lane's partial of row `r` of expert `e`: units lane_in_row, +lpr, ... (the
// caller sums the partials of the lpr lanes of the row).
template <uint32_t KIND>
QC_DEV float row_partial_k(const MatDesc& m, uint32_t e, uint32_t r, uint32_t lane_in_row, const float* xs) {
  const uint8_t* row = m.w + e * m.expert_stride + (uint64_t)r * m.row_stride;
  const __half* drow = m.d ? m.d + e * m.d_expert_stride + (uint64_t)r * m.d_stride : nullptr;
  float acc = 0.f;
  for (uint32_t k = 0; k < m.upl; k++) acc += unit_dot<KIND>(row, drow, lane_in_row + k * m.lpr, xs);
  return acc;
}

QC_DEV float row_partial(const MatDesc& m, uint32_t e, uint32_t r, uint32_t lane_in_row, const float* xs) {
  switch (m.kind) {
    case Q4_K: return row_partial_k<Q4_K>(m, e, r, lane_in_row, xs);
    case Q5_K: return row_partial_k<Q5_K>(m, e, r, lane_in_row, xs);
    case Q6_K: return row_partial_k<Q6_K>(m, e, r, lane_in_row, xs);
    case Q8_0: return row_partial_k<Q8_0>(m, e, r, lane_in_row, xs);
    case Q4_0: return row_partial_k<Q4_0>(m, e, r, lane_in_row, xs);
    case F16: return row_partial_k<F16>(m, e, r, lane_in_row, xs);
    default: return row_partial_k<F32>(m, e, r, lane_in_row, xs);
  }
}

}  // namespace qc
