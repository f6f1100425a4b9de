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

// Device layout of one matrix (or of an expert stack).  A row is processed in
// "units" of 64 consecutive elements.  Rows are stored in groups of 8,
//   group g = [rows 8g..8g+7: main_bytes each][rows 8g..8g+7: d_bytes each],
// so any run of whole groups is one contiguous, 16-byte-aligned span.
//
// main plane per row:
// Q4_K, Q5_K   raw GGUF super-blocks (144 / 176 bytes); no d values
// Q6_K         per block: ql[128] qh[64] scales[16] (208 bytes); d values (f16) after the group
// Q8_0         per block: qs[32]; d values after the group; rows padded to an even block count
// Q4_0         per block: qs[16]; d values after the group; rows padded to an even block count
// F16, F32     raw rows padded with zeros to a multiple of 64 elements
struct MatDesc {
  const uint8_t* w;
  uint32_t kind, rows, cols;
  uint32_t units;  // ceil(cols / 64)
  uint32_t lpr;    // lanes cooperating on one row (power of two, divides units, <= 32)
  uint32_t upl;    // units per lane = units / lpr
  uint32_t main_bytes, d_bytes, group_bytes;
  uint64_t expert_stride;  // bytes between experts (ceil(rows/8) groups)
};

// Row r of expert e, relative to a base holding groups from `g_base` on.
__host__ __device__ inline const uint8_t* row_ptr(const MatDesc& m, const uint8_t* base, uint32_t r) {
  return base + (uint64_t)(r >> 3) * m.group_bytes + (r & 7) * m.main_bytes;
}
__host__ __device__ inline const __half* drow_ptr(const MatDesc& m, const uint8_t* base, uint32_t r) {
  return reinterpret_cast<const __half*>(base + (uint64_t)(r >> 3) * m.group_bytes + 8 * m.main_bytes +
                                         (r & 7) * m.d_bytes);
}
__host__ __device__ inline const uint8_t* expert_base(const MatDesc& m, uint32_t e) {
  return m.w + (uint64_t)e * m.expert_stride;
}

__host__ __device__ inline bool uses_float_x(uint32_t kind) { return kind == F16 || kind == F32; }

QC_DEV uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// 16-byte load from global (S = false) or shared memory (S = true).
template <bool S>
QC_DEV uint4 ld16(const void* p) {
  if constexpr (S) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return v;
  } else {
    return ldg16(p);
  }
}
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

// Per-head RMSNorm + NeoX RoPE of one head vector held in shared memory by one warp.
QC_DEV void head_norm_rope(float* v, const float* __restrict__ w, uint32_t D, float eps, const float2* __restrict__ cs) {
  const uint32_t lane = threadIdx.x & 31;
  float ss = 0.f;
  for (uint32_t i = lane; i < D; i += 32) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float s = 1.0f / sqrtf(ss / (float)D + eps);
  for (uint32_t i = lane; i < D; i += 32) v[i] = __fmul_rn(v[i], __fmul_rn(s, w[i]));
  __syncwarp();
  // ops.rs:17-28: (a, b) -> (a c - b s, a s + b c) for pairs (i, i + D/2)
  for (uint32_t i = lane; i < D / 2; i += 32) {
    const float a = v[i], b = v[i + D / 2];
    const float2 t = cs[i];
    v[i] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
    v[i + D / 2] = __fadd_rn(__fmul_rn(a, t.y), __fmul_rn(b, t.x));
  }
  __syncwarp();
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
// (d0, d1 in [-128, 127], |d2| <= 32).  Weight codes (nibbles, 5/6-bit values,
// int8) then meet the activations in exact dp4a integer dot products; the
// only rounding is that of xi (2^-22 of the block maximum) and of the final
// float combination.  Per unit u (64 elements) the three digit planes are
// stored as [d0 x64][d1 x64][d2 x64][pad 16] = 208 bytes: the pad puts the
// 16-byte reads of 8 consecutive units in 8 different bank groups.
// F16/F32 matrices read a float copy instead: 64 floats + 4 pad per unit.
constexpr uint32_t kUnitDigitBytes = 208;
constexpr uint32_t kUnitFloats = 68;
constexpr float kXRange = 2097152.f;  // 2^21

struct XView {
  const uint8_t* dig;  // [units][208]
  const int* sx;       // [units][4]: sum of xi over each 16 elements
  const float* sb;     // [units/4]: x scale of each 256-block (x = xi * sb)
  const float* xf;     // [units][68] padded float copy (F16/F32 only), may be null
};

// Units are staged in whole 256-element blocks.
__host__ __device__ inline uint32_t units4(uint32_t units) { return (units + 3) & ~3u; }
// Shared-memory bytes of one XView of `units` units.
__host__ __device__ inline uint32_t xview_bytes(uint32_t units, bool with_float) {
  const uint32_t u = units4(units);
  uint32_t b = u * kUnitDigitBytes + u * 16 + (u / 4) * 4;
  b = (b + 15) & ~15u;
  if (with_float) b += u * kUnitFloats * 4;
  return b;
}
__host__ __device__ inline XView xview_at(const uint8_t* mem, uint32_t units, bool with_float) {
  const uint32_t u = units4(units);
  XView v;
  v.dig = mem;
  v.sx = reinterpret_cast<const int*>(mem + u * kUnitDigitBytes);
  v.sb = reinterpret_cast<const float*>(mem + u * kUnitDigitBytes + u * 16);
  v.xf = with_float
             ? reinterpret_cast<const float*>(mem + ((u * kUnitDigitBytes + u * 16 + (u / 4) * 4 + 15) & ~15u))
             : nullptr;
  return v;
}

// Quantize the 8 values a lane holds (elements e..e+7 of unit u, one 256-block
// per warp) and store digits, 16-element sums, the block scale and the float copy.
QC_DEV void store_lane8(uint8_t* mem, uint32_t units, bool with_float, uint32_t u, uint32_t e, const float (&x)[8]) {
  const uint32_t lane = threadIdx.x & 31;
  float mx = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) mx = fmaxf(mx, fabsf(x[k]));
  mx = warp_max(mx);
  const float inv = mx > 0.f ? kXRange / mx : 0.f;
  const XView xv = xview_at(mem, units, with_float);
  if (lane == 0) const_cast<float*>(xv.sb)[u >> 2] = mx > 0.f ? mx / kXRange : 0.f;
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
  s += __shfl_xor_sync(0xffffffffu, s, 1);  // lanes (2j, 2j+1) of a unit hold one 16-group
  uint8_t* du = mem + u * kUnitDigitBytes + e;
  *reinterpret_cast<uint2*>(du) = make_uint2(w0[0], w0[1]);
  *reinterpret_cast<uint2*>(du + 64) = make_uint2(w1[0], w1[1]);
  *reinterpret_cast<uint2*>(du + 128) = make_uint2(w2[0], w2[1]);
  if ((lane & 1) == 0) const_cast<int*>(xv.sx)[u * 4 + (e >> 4)] = s;
  if (with_float) {
    float* f = const_cast<float*>(xv.xf) + u * kUnitFloats + e;
    *reinterpret_cast<float4*>(f) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(f + 4) = make_float4(x[4], x[5], x[6], x[7]);
  }
}

// Stage `nv` vectors of n elements each (v(j, i) for vector j, element i < n;
// zero beyond) as consecutive XViews of xview_bytes(units) bytes.  If RMS, the
// vector (nv must be 1) is x[i] and becomes x[i] * (s * w[i]) with
// s = 1/sqrt(mean(x^2) + eps) (reference ops.rs:3-15, the product s*w first).
// Each thread owns 8 consecutive elements per pass, a warp one 256-block; all
// loads of up to 4 passes are issued before any arithmetic.  All threads of
// the block must call; ends with __syncthreads().
template <bool RMS, class F>
QC_DEV void stage_vectors(uint8_t* mem, uint32_t nv, uint32_t n, uint32_t units, bool with_float, F v,
                          const float* __restrict__ w, float eps, float* red) {
  const uint32_t per = units4(units) * 64;  // padded elements per vector
  const uint32_t total = nv * per, xb = xview_bytes(units, with_float);
  constexpr int P = 4;
  for (uint32_t base = 0; base < total; base += P * blockDim.x * 8) {
    float x[P][8], ww[P][8];
#pragma unroll
    for (int p = 0; p < P; p++) {
      const uint32_t i0 = base + (p * blockDim.x + threadIdx.x) * 8;
      const uint32_t j = i0 / per, e = i0 % per;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const bool ok = i0 < total && e + k < n;
        x[p][k] = ok ? v(j, e + k) : 0.f;
        if constexpr (RMS) ww[p][k] = ok ? w[e + k] : 0.f;
      }
    }
    if constexpr (RMS) {
      float ss = 0.f;
#pragma unroll
      for (int p = 0; p < P; p++)
#pragma unroll
        for (int k = 0; k < 8; k++) ss = fmaf(x[p][k], x[p][k], ss);
      ss = block_sum(ss, red);
      const float sc = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll
      for (int p = 0; p < P; p++)
#pragma unroll
        for (int k = 0; k < 8; k++) x[p][k] = __fmul_rn(x[p][k], __fmul_rn(sc, ww[p][k]));
    }
#pragma unroll
    for (int p = 0; p < P; p++) {
      const uint32_t i0 = base + (p * blockDim.x + threadIdx.x) * 8;
      if (base + (p * blockDim.x + (threadIdx.x & ~31u)) * 8 < total) {  // warp-uniform: whole 256-blocks
        const uint32_t j = i0 / per, e = i0 % per;
        store_lane8(mem + j * xb, units, with_float, e >> 6, e & 63, x[p]);
      }
    }
  }
  __syncthreads();
}

QC_DEV int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }
QC_DEV float combine(int a0, int a1, int a2) { return (float)a0 + 256.f * (float)a1 + 65536.f * (float)a2; }
// The plane sums as one integer, sum q * xi = a0 + 256 a1 + 65536 a2, computed mod 2^32: exact when
// the true sum fits an int32, i.e. |sum q xi| <= n * max|q| * 2^21 < 2^31 (32 codes of up to 5 bits,
// or 16 codes of up to 6 bits; not 8-bit codes).  One int-to-float conversion instead of three.
QC_DEV int icombine(int a0, int a1, int a2) {
  return (int)((uint32_t)a0 + ((uint32_t)a1 << 8) + ((uint32_t)a2 << 16));
}
// The float of a small integer (|x| < 2^22) without the conversion unit: the bits of 1.5 * 2^23
// plus x hold 1.5 * 2^23 + x exactly, and the subtraction is exact.
QC_DEV float small_i2f(int x) { return __int_as_float(0x4B400000 + x) - 12582912.f; }

// The activation data of one unit held in registers: d[4p + q] = digit plane p,
// elements 16q..16q+15; s = sums of xi over the four 16-element groups; sb = scale.
struct UnitX {
  uint4 d[12];
  int4 s;
  float sb;
};
QC_DEV UnitX load_unit_x(const XView& xv, uint32_t u) {
  UnitX ux;
  const uint4* a = reinterpret_cast<const uint4*>(xv.dig + u * kUnitDigitBytes);
#pragma unroll
  for (int i = 0; i < 12; i++) ux.d[i] = a[i];
  ux.s = *reinterpret_cast<const int4*>(xv.sx + u * 4);
  ux.sb = xv.sb[u >> 2];
  return ux;
}
QC_DEV uint32_t wsel(const uint4& t, int j) {
  switch (j & 3) {
    case 0: return t.x;
    case 1: return t.y;
    case 2: return t.z;
    default: return t.w;
  }
}
// Digit word j (elements 4j..4j+3, j < 16) of plane p.
QC_DEV uint32_t dword(const UnitX& ux, int p, int j) { return wsel(ux.d[4 * p + (j >> 2)], j); }

// sum of 32 codes (codes[j]: elements h*32 + 4j .. +3) times xi, exact in three dp4a chains: as an
// integer (codes of up to 5 bits), or as a float (any int8 codes).
QC_DEV int idot32i(const uint32_t (&codes)[8], const UnitX& ux, int h) {
  int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    a0 = dp4a(codes[j], dword(ux, 0, 8 * h + j), a0);
    a1 = dp4a(codes[j], dword(ux, 1, 8 * h + j), a1);
    a2 = dp4a(codes[j], dword(ux, 2, 8 * h + j), a2);
  }
  return icombine(a0, a1, a2);
}
QC_DEV float idot32(const uint32_t (&codes)[8], const UnitX& ux, int h) {
  int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    a0 = dp4a(codes[j], dword(ux, 0, 8 * h + j), a0);
    a1 = dp4a(codes[j], dword(ux, 1, 8 * h + j), a1);
    a2 = dp4a(codes[j], dword(ux, 2, 8 * h + j), a2);
  }
  return combine(a0, a1, a2);
}
// As idot32i but split into the two 16-element halves (Q6_K scale groups; codes of up to 6 bits).
QC_DEV void idot16x2i(const uint32_t (&codes)[8], const UnitX& ux, int h, int* lo, int* hi) {
  int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    a0 = dp4a(codes[j], dword(ux, 0, 8 * h + j), a0);
    a1 = dp4a(codes[j], dword(ux, 1, 8 * h + j), a1);
    a2 = dp4a(codes[j], dword(ux, 2, 8 * h + j), a2);
    b0 = dp4a(codes[j + 4], dword(ux, 0, 8 * h + j + 4), b0);
    b1 = dp4a(codes[j + 4], dword(ux, 1, 8 * h + j + 4), b1);
    b2 = dp4a(codes[j + 4], dword(ux, 2, 8 * h + j + 4), b2);
  }
  *lo = icombine(a0, a1, a2);
  *hi = icombine(b0, b1, b2);
}

// 6-bit scale and min of sub-blocks j and j+1 (j even) from the 12 packed bytes
// s0|s1|s2 (quant.rs:25-34), without branches: both belong to the same half.
QC_DEV void kq_scale_pair(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t j, float* sc0, float* m0, float* sc1,
                          float* m1) {
  const uint32_t jj = j & 3, hi = j >> 2;
  // bytes jj and jj+1 of each word
  const uint32_t a = __byte_perm(s0, 0, 0x4440 | jj) | (__byte_perm(s0, 0, 0x4440 | (jj + 1)) << 8);
  const uint32_t b = __byte_perm(s1, 0, 0x4440 | jj) | (__byte_perm(s1, 0, 0x4440 | (jj + 1)) << 8);
  const uint32_t c = __byte_perm(s2, 0, 0x4440 | jj) | (__byte_perm(s2, 0, 0x4440 | (jj + 1)) << 8);
  // low half (j < 4): a & 63, b & 63; high half: (c & 15) | (a >> 6) << 4, (c >> 4) | (b >> 6) << 4
  const uint32_t sl = a & 0x3f3fu, ml = b & 0x3f3fu;
  const uint32_t sh = (c & 0x0f0fu) | (((a >> 6) & 0x0303u) << 4), mh = ((c >> 4) & 0x0f0fu) | (((b >> 6) & 0x0303u) << 4);
  const uint32_t sv = hi ? sh : sl, mv = hi ? mh : ml;
  *sc0 = small_i2f((int)(sv & 0xff));
  *sc1 = small_i2f((int)(sv >> 8));
  *m0 = small_i2f((int)(mv & 0xff));
  *m1 = small_i2f((int)(mv >> 8));
}

// ---- unit dot products: the contribution of unit u (64 elements) of one row ----

// Q4_K unit u = (block u/4, pair p = u%4): sub-blocks 2p (low nibbles) and 2p+1 (high nibbles).
template <bool S>
QC_DEV float unit_q4k(const uint8_t* row, uint32_t u, const UnitX& ux) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 144;
  const uint4 hd = ld16<S>(blk);
  const uint4 q0 = ld16<S>(blk + 16 + 32 * p), q1 = ld16<S>(blk + 32 + 32 * p);
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    lo[j] = w[j] & 0x0f0f0f0fu;
    hi[j] = (w[j] >> 4) & 0x0f0f0f0fu;
  }
  const float qlo = (float)idot32i(lo, ux, 0), qhi = (float)idot32i(hi, ux, 1);
  float sc0, m0, sc1, m1;
  kq_scale_pair(hd.y, hd.z, hd.w, 2 * p, &sc0, &m0, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float r = sc0 * qlo + sc1 * qhi;
  const float mm = m0 * (float)(ux.s.x + ux.s.y) + m1 * (float)(ux.s.z + ux.s.w);
  return (d * r - dmin * mm) * ux.sb;
}

// Q5_K: as Q4_K plus the fifth bit: qh[t] bit g belongs to element 32g + t.
template <bool S>
QC_DEV float unit_q5k(const uint8_t* row, uint32_t u, const UnitX& ux) {
  const uint32_t b = u >> 2, p = u & 3;
  const uint8_t* blk = row + b * 176;
  const uint4 hd = ld16<S>(blk);
  const uint4 h0 = ld16<S>(blk + 16), h1 = ld16<S>(blk + 32);
  const uint4 q0 = ld16<S>(blk + 48 + 32 * p), q1 = ld16<S>(blk + 64 + 32 * p);
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t h[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
  const uint32_t g0 = 2 * p, g1 = 2 * p + 1;
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    lo[j] = (w[j] & 0x0f0f0f0fu) | (((h[j] >> g0) & 0x01010101u) << 4);
    hi[j] = ((w[j] >> 4) & 0x0f0f0f0fu) | (((h[j] >> g1) & 0x01010101u) << 4);
  }
  const float qlo = (float)idot32i(lo, ux, 0), qhi = (float)idot32i(hi, ux, 1);
  float sc0, m0, sc1, m1;
  kq_scale_pair(hd.y, hd.z, hd.w, g0, &sc0, &m0, &sc1, &m1);
  const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
  const float r = sc0 * qlo + sc1 * qhi;
  const float mm = m0 * (float)(ux.s.x + ux.s.y) + m1 * (float)(ux.s.z + ux.s.w);
  return (d * r - dmin * mm) * ux.sb;
}

// Q6_K unit u = (block u/4, chunk c = (u/2)%2, half h = u%2): quarters 2h (elements
// c*128+64h+t) and 2h+1 (c*128+64h+32+t), t < 32; four 16-element scale groups.
template <bool S>
QC_DEV float unit_q6k(const uint8_t* row, const __half* drow, uint32_t u, const UnitX& ux) {
  const uint32_t b = u >> 2, c = (u >> 1) & 1, hh = u & 1;
  const uint8_t* blk = row + b * 208;
  const uint4 l0 = ld16<S>(blk + c * 64), l1 = ld16<S>(blk + c * 64 + 16);       // quarter 2h: ql[c*64 + t]
  const uint4 l2 = ld16<S>(blk + c * 64 + 32), l3 = ld16<S>(blk + c * 64 + 48);  // quarter 2h+1: ql[c*64+32+t]
  const uint4 qa = ld16<S>(blk + 128 + c * 32), qb = ld16<S>(blk + 128 + c * 32 + 16);
  const uint4 sc = ld16<S>(blk + 192);
  const uint32_t la[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
  const uint32_t lb[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
  const uint32_t qh[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  const uint32_t ns = 4 * hh, s0 = 4 * hh, s1 = 4 * hh + 2;
  uint32_t ca[8], cb[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    ca[j] = ((la[j] >> ns) & 0x0f0f0f0fu) | (((qh[j] >> s0) & 0x03030303u) << 4);
    cb[j] = ((lb[j] >> ns) & 0x0f0f0f0fu) | (((qh[j] >> s1) & 0x03030303u) << 4);
  }
  int ia0, ia1, ib0, ib1;
  idot16x2i(ca, ux, 0, &ia0, &ia1);
  idot16x2i(cb, ux, 1, &ib0, &ib1);
  const float qa0 = (float)ia0, qa1 = (float)ia1, qb0 = (float)ib0, qb1 = (float)ib1;
  // the four scales sit in bytes c*8 + 4h .. +3, i.e. in word 2c + h of the 16 scale bytes
  const uint32_t sw = (c ? (hh ? sc.w : sc.z) : (hh ? sc.y : sc.x));
  const float sa0 = small_i2f((int8_t)byte_of(sw, 0)), sa1 = small_i2f((int8_t)byte_of(sw, 1));
  const float sb0 = small_i2f((int8_t)byte_of(sw, 2)), sb1 = small_i2f((int8_t)byte_of(sw, 3));
  // sum (q - 32) x = sum q x - 32 sum x over each 16-element group
  const float r = sa0 * (qa0 - 32.f * (float)ux.s.x) + sa1 * (qa1 - 32.f * (float)ux.s.y) +
                  sb0 * (qb0 - 32.f * (float)ux.s.z) + sb1 * (qb1 - 32.f * (float)ux.s.w);
  return h2f(drow[b]) * r * ux.sb;
}

// Q8_0 unit u = blocks 2u and 2u+1.
template <bool S>
QC_DEV float unit_q80(const uint8_t* row, const __half* drow, uint32_t u, const UnitX& ux) {
  const uint8_t* blk = row + u * 64;
  const uint4 a = ld16<S>(blk), b = ld16<S>(blk + 16), c = ld16<S>(blk + 32), e = ld16<S>(blk + 48);
  const uint32_t w0[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const uint32_t w1[8] = {c.x, c.y, c.z, c.w, e.x, e.y, e.z, e.w};
  const float q0 = idot32(w0, ux, 0), q1 = idot32(w1, ux, 1);
  const __half2 dd = *reinterpret_cast<const __half2*>(drow + 2 * u);
  return (__low2float(dd) * q0 + __high2float(dd) * q1) * ux.sb;
}

// Q4_0 unit u = blocks 2u, 2u+1; byte t of a block holds elements t (low) and 16+t (high).
template <bool S>
QC_DEV float unit_q40(const uint8_t* row, const __half* drow, uint32_t u, const UnitX& ux) {
  const uint4 a = ld16<S>(row + u * 32), b = ld16<S>(row + u * 32 + 16);
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
  uint32_t c0[8], c1[8];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    c0[j] = wa[j] & 0x0f0f0f0fu;
    c0[j + 4] = (wa[j] >> 4) & 0x0f0f0f0fu;
    c1[j] = wb[j] & 0x0f0f0f0fu;
    c1[j + 4] = (wb[j] >> 4) & 0x0f0f0f0fu;
  }
  const float q0 = (float)idot32i(c0, ux, 0), q1 = (float)idot32i(c1, ux, 1);
  const __half2 dd = *reinterpret_cast<const __half2*>(drow + 2 * u);
  const float r0 = q0 - 8.f * (float)(ux.s.x + ux.s.y), r1 = q1 - 8.f * (float)(ux.s.z + ux.s.w);
  return (__low2float(dd) * r0 + __high2float(dd) * r1) * ux.sb;
}

// Float activations of one unit held in registers (F16/F32 matrices).
struct UnitXF {
  float4 f[16];
};
QC_DEV UnitXF load_unit_xf(const XView& xv, uint32_t u) {
  UnitXF ux;
  const float4* a = reinterpret_cast<const float4*>(xv.xf + u * kUnitFloats);
#pragma unroll
  for (int i = 0; i < 16; i++) ux.f[i] = a[i];
  return ux;
}

template <bool S>
QC_DEV float unit_f16(const uint8_t* row, uint32_t u, const UnitXF& ux) {
  const uint8_t* p = row + u * 128;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint4 v = ld16<S>(p + 16 * k);
    const float4 xa = ux.f[2 * k], xb = ux.f[2 * k + 1];
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

template <bool S>
QC_DEV float unit_f32(const uint8_t* row, uint32_t u, const UnitXF& ux) {
  const uint8_t* p = row + u * 256;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 16; k++) {
    const uint4 v = ld16<S>(p + 16 * k);
    acc = fmaf(__uint_as_float(v.x), ux.f[k].x, acc);
    acc = fmaf(__uint_as_float(v.y), ux.f[k].y, acc);
    acc = fmaf(__uint_as_float(v.z), ux.f[k].z, acc);
    acc = fmaf(__uint_as_float(v.w), ux.f[k].w, acc);
  }
  return acc;
}

template <uint32_t KIND>
struct UnitXOf {
  using type = UnitX;
};
template <>
struct UnitXOf<F16> {
  using type = UnitXF;
};
template <>
struct UnitXOf<F32> {
  using type = UnitXF;
};

template <uint32_t KIND>
QC_DEV typename UnitXOf<KIND>::type load_x(const XView& xv, uint32_t u) {
  if constexpr (KIND == F16 || KIND == F32) return load_unit_xf(xv, u);
  else return load_unit_x(xv, u);
}

template <uint32_t KIND, bool S>
QC_DEV float unit_dot(const uint8_t* row, const __half* drow, uint32_t u, const typename UnitXOf<KIND>::type& ux) {
  if constexpr (KIND == Q4_K) return unit_q4k<S>(row, u, ux);
  else if constexpr (KIND == Q5_K) return unit_q5k<S>(row, u, ux);
  else if constexpr (KIND == Q6_K) return unit_q6k<S>(row, drow, u, ux);
  else if constexpr (KIND == Q8_0) return unit_q80<S>(row, drow, u, ux);
  else if constexpr (KIND == Q4_0) return unit_q40<S>(row, drow, u, ux);
  else if constexpr (KIND == F16) return unit_f16<S>(row, u, ux);
  else return unit_f32<S>(row, u, ux);
}

// ---------------------------------------------------------------------------
// Warp-level matvec over rows [r0, r1) of a block.  Warp w takes row groups
// (G = 32/lpr rows each) w, w+nw, ...; lane (row slot, lr) always handles units
// lr, lr+lpr, ...  When a lane has one unit (upl == 1, the common case) its
// activation data is loaded into registers once for all rows.  addr(r, &row,
// &drow) gives the row pointers; emit(r, sum) runs on lane 0 of the row's group.
template <uint32_t KIND, bool S, class Addr, class Emit>
QC_DEV void warp_rows_k(const MatDesc& m, uint32_t r0, uint32_t r1, const XView& xv, Addr addr, Emit emit,
                        uint32_t warp, uint32_t nw) {
  const uint32_t lpr = m.lpr, G = 32 / lpr, lane = threadIdx.x & 31;
  const uint32_t lr = lane % lpr, slot = lane / lpr, stride = nw * G;
  // (formats of 6- and 8-bit codes hold more registers per row: two row groups per pass there)
  constexpr bool kFour = !(KIND == Q6_K || KIND == Q8_0);
  if (m.upl == 1 && lpr >= 2 && !kFour) {
    // two row groups per pass (b and b + stride): one shuffle trades half of each lane's pair of sums
    // with its partner lr ^ h, then one reduction over h lanes finishes both (row b on lane lr 0, row
    // b + stride on lane h)
    const auto ux = load_x<KIND>(xv, lr);
    const uint32_t h = lpr >> 1;
    const bool up = lr >= h;
#pragma unroll 1
    for (uint32_t b = r0 + warp * G; b < r1; b += 2 * stride) {
      const uint32_t ra = b + slot, rb = b + stride + slot;
      float va = 0.f, vb = 0.f;
      const uint8_t* row;
      const __half* drow;
      if (ra < r1) {
        addr(ra, &row, &drow);
        va = unit_dot<KIND, S>(row, drow, lr, ux);
      }
      if (rb < r1) {
        addr(rb, &row, &drow);
        vb = unit_dot<KIND, S>(row, drow, lr, ux);
      }
      float v = (up ? vb : va) + __shfl_xor_sync(0xffffffffu, up ? va : vb, h);
      for (uint32_t o = h >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lr == 0 && ra < r1) emit(ra, v);
      if (lr == h && rb < r1) emit(rb, v);
    }
  } else if (m.upl == 1 && lpr >= 4) {
    // four row groups per pass (b + i * stride, i < 4): four independent dot chains per lane, and
    // one reduction for all four: a shuffle over lr ^ h (h = lpr / 2) trades the pairs (0, 1) / (2, 3),
    // one over lr ^ h/2 trades within each pair, then the remaining lpr / 4 lanes are summed (row i
    // ends on lane lr = i * lpr / 4)
    const auto ux = load_x<KIND>(xv, lr);
    const uint32_t h = lpr >> 1, q = lpr >> 2;
    const bool up = lr & h, mid = lr & q;
#pragma unroll 1
    for (uint32_t b = r0 + warp * G; b < r1; b += 4 * stride) {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t r = b + i * stride + slot;
        v[i] = 0.f;
        if (r < r1) {
          const uint8_t* row;
          const __half* drow;
          addr(r, &row, &drow);
          v[i] = unit_dot<KIND, S>(row, drow, lr, ux);
        }
      }
      const float k0 = up ? v[2] : v[0], k1 = up ? v[3] : v[1];
      const float w0 = k0 + __shfl_xor_sync(0xffffffffu, up ? v[0] : v[2], h);
      const float w1 = k1 + __shfl_xor_sync(0xffffffffu, up ? v[1] : v[3], h);
      float w = (mid ? w1 : w0) + __shfl_xor_sync(0xffffffffu, mid ? w0 : w1, q);
      for (uint32_t o = q >> 1; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
      if ((lr & (q - 1)) == 0) {
        const uint32_t i = (up ? 2 : 0) + (mid ? 1 : 0), r = b + i * stride + slot;
        if (r < r1) emit(r, w);
      }
    }
  } else if (m.upl == 1) {
    const auto ux = load_x<KIND>(xv, lr);
#pragma unroll 2
    for (uint32_t b = r0 + warp * G; b < r1; b += stride) {
      const uint32_t r = b + slot;
      float acc = 0.f;
      if (r < r1) {
        const uint8_t* row;
        const __half* drow;
        addr(r, &row, &drow);
        acc = unit_dot<KIND, S>(row, drow, lr, ux);
      }
      acc = group_sum(acc, lpr);
      if (lr == 0 && r < r1) emit(r, acc);
    }
  } else {
#pragma unroll 1
    for (uint32_t b = r0 + warp * G; b < r1; b += stride) {
      const uint32_t r = b + slot;
      float acc = 0.f;
      if (r < r1) {
        const uint8_t* row;
        const __half* drow;
        addr(r, &row, &drow);
#pragma unroll 1
        for (uint32_t k = 0; k < m.upl; k++) {
          const uint32_t u = lr + k * lpr;
          acc += unit_dot<KIND, S>(row, drow, u, load_x<KIND>(xv, u));
        }
      }
      acc = group_sum(acc, lpr);
      if (lr == 0 && r < r1) emit(r, acc);
    }
  }
}

// All warps of the block (warp = threadIdx.x/32) or, with explicit arguments, one subset.
template <bool S, class Addr, class Emit>
QC_DEV void warp_rows(const MatDesc& m, uint32_t r0, uint32_t r1, const XView& xv, Addr addr, Emit emit,
                      uint32_t warp = threadIdx.x >> 5, uint32_t nw = blockDim.x >> 5) {
  switch (m.kind) {
    case Q4_K: warp_rows_k<Q4_K, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    case Q5_K: warp_rows_k<Q5_K, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    case Q6_K: warp_rows_k<Q6_K, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    case Q8_0: warp_rows_k<Q8_0, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    case Q4_0: warp_rows_k<Q4_0, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    case F16: warp_rows_k<F16, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
    default: warp_rows_k<F32, S>(m, r0, r1, xv, addr, emit, warp, nw); break;
  }
}
// Rows of a matrix held in shared memory from row `rbase` on.
struct SmemRows {
  const MatDesc* m;
  const uint8_t* base;
  uint32_t rbase;
  QC_DEV void operator()(uint32_t r, const uint8_t** row, const __half** drow) const {
    *row = row_ptr(*m, base, r - rbase);
    *drow = drow_ptr(*m, base, r - rbase);
  }
};

// One row's partial for lane lr of its lpr-lane group (units lr, lr+lpr, ...).
template <bool S>
QC_DEV float row_partial(const MatDesc& m, const uint8_t* row, const __half* drow, uint32_t lr, const XView& xv) {
  float acc = 0.f;
  for (uint32_t k = 0; k < m.upl; k++) {
    const uint32_t u = lr + k * m.lpr;
    switch (m.kind) {
      case Q4_K: acc += unit_q4k<S>(row, u, load_unit_x(xv, u)); break;
      case Q5_K: acc += unit_q5k<S>(row, u, load_unit_x(xv, u)); break;
      case Q6_K: acc += unit_q6k<S>(row, drow, u, load_unit_x(xv, u)); break;
      case Q8_0: acc += unit_q80<S>(row, drow, u, load_unit_x(xv, u)); break;
      case Q4_0: acc += unit_q40<S>(row, drow, u, load_unit_x(xv, u)); break;
      case F16: acc += unit_f16<S>(row, u, load_unit_xf(xv, u)); break;
      default: acc += unit_f32<S>(row, u, load_unit_xf(xv, u)); break;
    }
  }
  return acc;
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (cp.async, 16 bytes per request).
QC_DEV void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
QC_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
QC_DEV void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
QC_DEV void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Copy `bytes` (a multiple of 16; both addresses 16-byte aligned) with all threads of the block.
QC_DEV void copy_async(uint8_t* dst, const uint8_t* src, uint64_t bytes) {
  for (uint64_t o = threadIdx.x * 16ull; o < bytes; o += blockDim.x * 16ull) cp16(dst + o, src + o);
}
// Copy row groups [g0, g1) of expert e of m to dst.
QC_DEV void copy_groups(uint8_t* dst, const MatDesc& m, uint32_t e, uint32_t g0, uint32_t g1) {
  if (g1 > g0) copy_async(dst, expert_base(m, e) + (uint64_t)g0 * m.group_bytes, (uint64_t)(g1 - g0) * m.group_bytes);
}

}  // namespace qc
