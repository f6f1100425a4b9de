// Standalone matrix kernels: raw-GGUF -> device-layout repack, bit-exact
// dequant, and the dequant-fused matvec y = W x.
//
// These back the per-matvec entry points of the C ABI (qc_matrix_*), which
// replace the reference's `Backend::matvec` / `Vulkan::packed_matvec`
// (src/backend.rs:14-23, 174-353).  The whole-token decode path uses the fused
// kernels in decode.cu, built from the same device functions.
#include "common.cuh"
#include "kernels.h"

namespace qc {

// ---------------------------------------------------------------------------
// Repack: raw GGUF rows (src, `n_rows` rows of `raw_row` bytes) into the device
// layout.  One thread per block (quantized kinds) or per 16-byte chunk of the
// padded output row (F16/F32).
__global__ void k_repack(const uint8_t* __restrict__ src, uint64_t n_rows, uint64_t raw_row, uint32_t kind,
                         uint64_t cols, uint8_t* __restrict__ dst, uint64_t row_stride, __half* __restrict__ dplane,
                         uint64_t d_stride) {
  uint64_t per_row, valid;  // output blocks (or 16-byte chunks) per row, and how many come from the source
  switch (kind) {
    case Q4_K: case Q5_K: case Q6_K: per_row = valid = cols / 256; break;
    case Q8_0: case Q4_0: per_row = d_stride; valid = cols / 32; break;
    default: per_row = row_stride / 16; valid = per_row; break;
  }
  const uint64_t total = n_rows * per_row;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / per_row, k = i % per_row;
    const uint8_t* s = src + r * raw_row;
    uint8_t* o = dst + r * row_stride;
    const bool pad = k >= valid;
    switch (kind) {
      case Q4_K:
        for (int j = 0; j < 144; j++) o[k * 144 + j] = s[k * 144 + j];
        break;
      case Q5_K:
        for (int j = 0; j < 176; j++) o[k * 176 + j] = s[k * 176 + j];
        break;
      case Q6_K:
        for (int j = 0; j < 208; j++) o[k * 208 + j] = s[k * 210 + j];
        dplane[r * d_stride + k] = __ushort_as_half((unsigned short)(s[k * 210 + 208] | (s[k * 210 + 209] << 8)));
        break;
      case Q8_0:
        for (int j = 0; j < 32; j++) o[k * 32 + j] = pad ? 0 : s[k * 34 + 2 + j];
        dplane[r * d_stride + k] =
            __ushort_as_half(pad ? (unsigned short)0 : (unsigned short)(s[k * 34] | (s[k * 34 + 1] << 8)));
        break;
      case Q4_0:
        for (int j = 0; j < 16; j++) o[k * 16 + j] = pad ? 0 : s[k * 18 + 2 + j];
        dplane[r * d_stride + k] =
            __ushort_as_half(pad ? (unsigned short)0 : (unsigned short)(s[k * 18] | (s[k * 18 + 1] << 8)));
        break;
      default: {  // F16 / F32: 16-byte chunk k of the padded row
        const uint64_t esz = kind == F16 ? 2 : 4, nbytes = cols * esz;
        for (int j = 0; j < 16; j++) {
          const uint64_t b = k * 16 + j;
          o[b] = b < nbytes ? s[b] : 0;
        }
      }
    }
  }
}

// Bit-exact dequant of expert `e` (all rows) to out[r*cols + c] (reference quant.rs:36-80).
__global__ void k_dequant(MatDesc m, uint32_t e, float* __restrict__ out) {
  const uint64_t total = (uint64_t)m.rows * m.cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(i / m.cols), c = (uint32_t)(i % m.cols);
    const uint8_t* row = m.w + e * m.expert_stride + (uint64_t)r * m.row_stride;
    const __half* drow = m.d ? m.d + e * m.d_expert_stride + (uint64_t)r * m.d_stride : nullptr;
    out[i] = dequant_one(m, row, drow, c);
  }
}

// y = W_e x.  Each warp takes 32/lpr rows at a time; lpr lanes share a row.
template <uint32_t KIND>
__global__ void __launch_bounds__(256) k_matvec(MatDesc m, uint32_t e, const float* __restrict__ x,
                                                float* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t smem[];
  const XView xv = stage_x(smem, m.cols, m.units, uses_float_x(KIND), [&](uint32_t i) { return x[i]; });
  const uint32_t lane = threadIdx.x & 31, lpr = m.lpr, G = 32 / lpr;
  const uint32_t wpb = blockDim.x >> 5;
  const uint32_t gw = blockIdx.x * wpb + (threadIdx.x >> 5), nw = gridDim.x * wpb;
  for (uint32_t base = gw * G; base < m.rows; base += nw * G) {
    const uint32_t r = base + lane / lpr, lr = lane % lpr;
    float p = r < m.rows ? row_partial_k<KIND>(m, e, r, lr, xv) : 0.f;
    p = group_sum(p, lpr);
    if (lr == 0 && r < m.rows) y[r] = p;
  }
}

// ---------------------------------------------------------------------------
void launch_repack(const uint8_t* src, uint64_t n_rows, uint64_t raw_row, uint32_t kind, uint64_t cols, uint8_t* dst,
                   uint64_t row_stride, __half* dplane, uint64_t d_stride, cudaStream_t s) {
  k_repack<<<148 * 8, 256, 0, s>>>(src, n_rows, raw_row, kind, cols, dst, row_stride, dplane, d_stride);
}

void launch_dequant(const MatDesc& m, uint32_t e, float* out, cudaStream_t s) {
  k_dequant<<<148 * 8, 256, 0, s>>>(m, e, out);
}

uint32_t matvec_grid(const MatDesc& m, int sms) {
  const uint32_t rows_per_block = 8 * (32 / m.lpr);
  uint32_t need = (m.rows + rows_per_block - 1) / rows_per_block;
  uint32_t cap = (uint32_t)sms * 8;
  return need < cap ? need : cap;
}

void launch_matvec(const MatDesc& m, uint32_t e, const float* x, float* y, int sms, cudaStream_t s) {
  const uint32_t grid = matvec_grid(m, sms);
  const size_t smem = matvec_smem(m);
  switch (m.kind) {
    case Q4_K: k_matvec<Q4_K><<<grid, 256, smem, s>>>(m, e, x, y); break;
    case Q5_K: k_matvec<Q5_K><<<grid, 256, smem, s>>>(m, e, x, y); break;
    case Q6_K: k_matvec<Q6_K><<<grid, 256, smem, s>>>(m, e, x, y); break;
    case Q8_0: k_matvec<Q8_0><<<grid, 256, smem, s>>>(m, e, x, y); break;
    case Q4_0: k_matvec<Q4_0><<<grid, 256, smem, s>>>(m, e, x, y); break;
    case F16: k_matvec<F16><<<grid, 256, smem, s>>>(m, e, x, y); break;
    default: k_matvec<F32><<<grid, 256, smem, s>>>(m, e, x, y); break;
  }
}

size_t matvec_smem(const MatDesc& m) { return xview_bytes(m.units, uses_float_x(m.kind)); }

cudaError_t matvec_prepare(int max_smem) {
  cudaError_t err = cudaSuccess;
#define QC_ATTR(K)                                                                                      \
  if (err == cudaSuccess)                                                                               \
    err = cudaFuncSetAttribute(k_matvec<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  QC_ATTR(Q4_K) QC_ATTR(Q5_K) QC_ATTR(Q6_K) QC_ATTR(Q8_0) QC_ATTR(Q4_0) QC_ATTR(F16) QC_ATTR(F32)
#undef QC_ATTR
  return err;
}

}  // namespace qc
