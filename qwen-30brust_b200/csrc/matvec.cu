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
// Repack: flattened raw GGUF rows [flat0, flat0 + n_rows) of an expert stack
// (`rows` rows per expert, `raw_row` bytes each, at src) into the 8-row-group
// device layout at dst (expert 0 base).  One thread per output block (quantized
// kinds) or per 16-byte chunk of the padded row (F16/F32).  Padding rows and
// padding blocks are left as they are (the destination is zeroed beforehand).
__global__ void k_repack(const uint8_t* __restrict__ src, uint64_t flat0, uint64_t n_rows, uint32_t rows,
                         uint64_t raw_row, uint32_t kind, uint64_t cols, uint8_t* __restrict__ dst, uint32_t main_bytes,
                         uint32_t d_bytes, uint32_t group_bytes, uint64_t expert_stride) {
  uint64_t per_row;  // items per row
  switch (kind) {
    case Q4_K: case Q5_K: case Q6_K: per_row = cols / 256; break;
    case Q8_0: case Q4_0: per_row = cols / 32; break;
    default: per_row = main_bytes / 16; break;
  }
  const uint64_t total = n_rows * per_row;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t fr = i / per_row, k = i % per_row;
    const uint64_t flat = flat0 + fr;
    const uint32_t e = (uint32_t)(flat / rows), r = (uint32_t)(flat % rows);
    const uint8_t* s = src + fr * raw_row;
    uint8_t* g = dst + e * expert_stride + (uint64_t)(r >> 3) * group_bytes;
    uint8_t* o = g + (r & 7) * main_bytes;
    uint8_t* dd = g + 8 * main_bytes + (r & 7) * d_bytes;
    switch (kind) {
      case Q4_K:
        for (int j = 0; j < 144; j++) o[k * 144 + j] = s[k * 144 + j];
        break;
      case Q5_K:
        for (int j = 0; j < 176; j++) o[k * 176 + j] = s[k * 176 + j];
        break;
      case Q6_K:
        for (int j = 0; j < 208; j++) o[k * 208 + j] = s[k * 210 + j];
        dd[2 * k] = s[k * 210 + 208];
        dd[2 * k + 1] = s[k * 210 + 209];
        break;
      case Q8_0:
        for (int j = 0; j < 32; j++) o[k * 32 + j] = s[k * 34 + 2 + j];
        dd[2 * k] = s[k * 34];
        dd[2 * k + 1] = s[k * 34 + 1];
        break;
      case Q4_0:
        for (int j = 0; j < 16; j++) o[k * 16 + j] = s[k * 18 + 2 + j];
        dd[2 * k] = s[k * 18];
        dd[2 * k + 1] = s[k * 18 + 1];
        break;
      default: {  // F16 / F32: 16-byte chunk k of the padded row
        const uint64_t nbytes = cols * (kind == F16 ? 2 : 4);
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
  const uint8_t* base = expert_base(m, e);
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(i / m.cols), c = (uint32_t)(i % m.cols);
    out[i] = dequant_one(m, row_ptr(m, base, r), drow_ptr(m, base, r), c);
  }
}

// y = W_e x, rows streamed through shared memory: each block takes a contiguous run of 8-row
// groups and streams it in stages of `sg` groups through `ns` shared-memory slots with TMA bulk
// copies (an mbarrier per slot counts the bytes), so up to ns - 1 stages are in flight while one is
// computed; warps walk the rows of a stage, lpr lanes per row.  Warps do not wait for each other:
// each releases a slot when done with its rows (a per-slot count of releases), and the warp whose
// release completes a stage's count refills the slot with stage k + ns.  The activation staging
// overlaps the first copies.  Waits are bounded (2 s); a block that gives up writes NaN for its
// rows, after waiting (bounded) for its copies in flight, and sets g_matvec_abort.
constexpr int kMaxSlots = 8;
constexpr unsigned long long kWaitNs = 2000000000ull;
__device__ uint32_t g_matvec_abort;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase of `parity` of b: false after 2 s, or as soon as *bad is set.
__device__ __forceinline__ bool slot_wait(uint64_t* b, uint32_t parity, const volatile int* bad = nullptr) {
  const unsigned long long t0 = now_ns();
  for (uint32_t i = 0;; i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255) == 255 && ((bad && *bad) || now_ns() - t0 > kWaitNs)) return false;
  }
}
__device__ __forceinline__ void slot_fill(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(b))
               : "memory");
}

template <uint32_t KIND>
__global__ void __launch_bounds__(512) k_matvec(MatDesc m, uint32_t e, const float* __restrict__ x,
                                                float* __restrict__ y, uint32_t sg, uint32_t ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar[kMaxSlots];
  __shared__ uint32_t released[kMaxSlots];  // releases of each slot by warps, over all its stages
  __shared__ int last[kMaxSlots];           // the latest stage issued into each slot
  __shared__ float red[32];
  __shared__ int bad;
  const uint32_t groups = (m.rows + 7) / 8;
  const uint32_t per = (groups + gridDim.x - 1) / gridDim.x;
  const uint32_t g0 = min(groups, blockIdx.x * per), g1 = min(groups, g0 + per);
  const uint32_t nst = (g1 - g0 + sg - 1) / sg;
  const uint32_t stage_bytes = sg * m.group_bytes;
  uint8_t* xmem = smem + ns * stage_bytes;
  const uint8_t* src = expert_base(m, e);
  auto issue = [&](uint32_t k) {  // one thread: stage k into slot k % ns
    const uint32_t a = g0 + k * sg, b = min(g1, a + sg);
    last[k % ns] = (int)k;
    slot_fill(smem + (k % ns) * stage_bytes, src + (uint64_t)a * m.group_bytes, (b - a) * m.group_bytes, &bar[k % ns]);
  };
  if (threadIdx.x == 0) {
    bad = 0;
    for (uint32_t i = 0; i < ns; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bar[i])) : "memory");
      released[i] = 0;
      last[i] = -1;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (uint32_t k = 0; k < ns && k < nst; k++) issue(k);
  }
  stage_vectors<false>(xmem, 1, m.cols, m.units, uses_float_x(KIND), [&](uint32_t, uint32_t i) { return x[i]; },
                       nullptr, 0.f, red);  // (ends with a barrier: the mbarriers are initialized)
  const XView xv = xview_at(xmem, m.units, uses_float_x(KIND));
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (uint32_t k = 0; k < nst; k++) {
    const uint32_t j = k % ns;
    if (!slot_wait(&bar[j], (k / ns) & 1, &bad)) {
      bad = 1;
      break;
    }
    const uint32_t r0 = (g0 + k * sg) * 8, r1 = min(m.rows, min(g1, g0 + (k + 1) * sg) * 8);
    warp_rows_k<KIND, true>(m, r0, r1, xv, SmemRows{&m, smem + j * stage_bytes, r0},
                            [&](uint32_t r, float v) { y[r] = v; }, warp, nw);
    __syncwarp();
    if (lane == 0) {  // this warp is done with slot j; the last of the stage refills it
      __threadfence_block();
      if (atomicAdd(&released[j], 1u) == (k / ns + 1) * nw - 1 && k + ns < nst) {
        __threadfence_block();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(k + ns);
      }
    }
  }
  __syncthreads();
  if (bad) {  // a copy did not arrive: report, after the copies in flight have landed
    for (uint32_t r = g0 * 8 + threadIdx.x; r < min(m.rows, g1 * 8); r += blockDim.x) y[r] = __int_as_float(0x7fc00000);
    if (threadIdx.x == 0) {
      atomicOr(&g_matvec_abort, 1u);
      for (uint32_t q = 0; q < ns; q++)
        if (last[q] >= 0) slot_wait(&bar[q], ((uint32_t)last[q] / ns) & 1);
    }
  }
}

// ---------------------------------------------------------------------------
void launch_repack(const uint8_t* src, uint64_t flat0, uint64_t n_rows, uint32_t rows, uint64_t raw_row, uint32_t kind,
                   uint64_t cols, uint8_t* dst, const DevLayout& l, uint64_t expert_stride, cudaStream_t s) {
  k_repack<<<148 * 8, 256, 0, s>>>(src, flat0, n_rows, rows, raw_row, kind, cols, dst, (uint32_t)l.main_bytes,
                                   (uint32_t)l.d_bytes, (uint32_t)l.group_bytes, expert_stride);
}

void launch_dequant(const MatDesc& m, uint32_t e, float* out, cudaStream_t s) {
  k_dequant<<<148 * 8, 256, 0, s>>>(m, e, out);
}

// Stage size in groups and slots of k_matvec.  A stage is what the block computes between two
// barriers, so it should give every warp a few rows: up to 6 groups (48 rows, 3 per warp) and
// 64 KB, but no more groups than a block's share when the matrix is small (so that every SM gets
// work); as many slots (2 to 8) as fit beside the activation tile in 192 KB.
static void matvec_stages(const MatDesc& m, int sms, uint32_t* sg, uint32_t* ns) {
  const uint64_t g = m.group_bytes, xb = xview_bytes(m.units, uses_float_x(m.kind));
  const uint64_t groups = (m.rows + 7) / 8, share = (groups + sms - 1) / sms;
  uint64_t s = (64 * 1024) / g;
  s = s > 6 ? 6 : s;
  s = s > share ? share : s;
  s = s < 1 ? 1 : s;
  const uint64_t budget = 192 * 1024 > xb ? 192 * 1024 - xb : 0;
  uint64_t n = budget / (s * g);
  n = n > (uint64_t)kMaxSlots ? (uint64_t)kMaxSlots : n;
  n = n < 2 ? 2 : n;
  *sg = (uint32_t)s;
  *ns = (uint32_t)n;
}

size_t matvec_smem(const MatDesc& m) {
  uint32_t sg, ns;
  matvec_stages(m, 148, &sg, &ns);
  return (size_t)ns * sg * m.group_bytes + xview_bytes(m.units, uses_float_x(m.kind));
}

void launch_matvec(const MatDesc& m, uint32_t e, const float* x, float* y, int sms, cudaStream_t s) {
  const uint32_t groups = (m.rows + 7) / 8;
  uint32_t sg, ns;
  matvec_stages(m, 148, &sg, &ns);  // (the same split as matvec_smem; sms is 148 on every caller)
  // enough blocks to cover the SMs, but each with at least one full stage of work
  uint32_t grid = (groups + sg - 1) / sg;
  grid = grid < (uint32_t)sms ? grid : (uint32_t)sms;
  grid = grid < 1 ? 1 : grid;
  const size_t smem = matvec_smem(m);
  switch (m.kind) {
    case Q4_K: k_matvec<Q4_K><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    case Q5_K: k_matvec<Q5_K><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    case Q6_K: k_matvec<Q6_K><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    case Q8_0: k_matvec<Q8_0><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    case Q4_0: k_matvec<Q4_0><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    case F16: k_matvec<F16><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
    default: k_matvec<F32><<<grid, 512, smem, s>>>(m, e, x, y, sg, ns); break;
  }
}

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
