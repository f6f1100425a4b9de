// qc_packed_matvec_noalloc: the host-to-host packed matvec without any device
// allocation.
//
// qc_packed_matvec allocates, per call, device buffers for the raw blocks, the
// repacked matrix and the x / y vectors.  Some callers cannot do that: a host
// application whose own allocator has already reserved the GPU's memory (a
// further cudaMalloc fails, or fragments a pool it manages), or code that must
// not call cudaFree because it may synchronize the whole device.  This variant
// keeps all of that working memory in one file-scope __device__ array of
// kScratchBytes (32 MiB).
//
// Use:
//   * CUDA loads a library's device code lazily (the default since CUDA 12.2),
//     so the array is reserved on a device when this file's code is first
//     loaded there: at the first call on that device, which looks up the
//     array's device address with cudaGetSymbolAddress (that lookup loads the
//     code) and sets the matvec kernels' shared-memory attribute.  From then on
//     the device holds the array until the process exits.  A host whose own
//     allocator claims the GPU's memory must therefore make one call on each
//     device before that allocator reserves its pool (with eager loading,
//     CUDA_MODULE_LOADING=EAGER, the array is reserved when the library's
//     context is created instead).  Make that first call before any stream
//     capture on the device as well.
//   * Every call reuses the same array and leaves its contents behind: the call
//     zeroes the part that must start at zero (the padding of the repacked
//     matrix) itself.  Calls that overlap on the GPU — from several host
//     threads, or on several streams — race on the array.
//   * A matrix whose raw blocks, repacked form and vectors need more than
//     kScratchBytes is rejected with QC_ERR_INVALID and a message saying so.
#include <mutex>
#include <string>

#include "../../include/qwen_cuda.h"
#include "kernels.h"
#include "layout.h"

namespace qc {
void set_last_error(const std::string& msg);  // engine.cu: the thread-local qc_last_error() text
}

namespace {

constexpr uint64_t kScratchBytes = 32ull << 20;
constexpr int kNoAllocMaxSmem = 200 * 1024;

// The working memory of every qc_packed_matvec_noalloc call on a device.  In host
// code this name is only a stand-in: kernels get the address from set-up below.
static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

std::mutex g_mu;
uint8_t* g_addr[64] = {};  // device address of g_scratch, per device

uint64_t up256(uint64_t v) { return (v + 255) & ~255ull; }

int fail(int code, const std::string& msg) {
  qc::set_last_error(msg);
  return code;
}

// Device address of the scratch array on the current device (looked up once per device).
int scratch_of_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(QC_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(QC_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return fail(QC_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    e = qc::matvec_prepare(kNoAllocMaxSmem);
    if (e != cudaSuccess) return fail(QC_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    g_addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_addr[dev];
  return QC_OK;
}

#define QC_NA_CK(call)                                                                       \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) return fail(QC_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

}  // namespace

extern "C" int qc_packed_matvec_noalloc(uint32_t kind, uint64_t rows, uint64_t cols, const uint8_t* blocks,
                                        uint64_t len, const float* x, float* y) {
  if (!blocks || !x || !y) return fail(QC_ERR_INVALID, "null argument");
  uint64_t raw_row = 0;
  if (const char* msg = qc::ggml_row_bytes(kind, cols, &raw_row)) return fail(QC_ERR_INVALID, msg);
  if (rows == 0 || rows > 0xffffffffull || cols > 0xffffffffull || len != raw_row * rows)
    return fail(QC_ERR_INVALID, "GPU matvec shape mismatch");
  const qc::DevLayout lay = qc::dev_layout(kind, cols);
  const uint64_t mat_bytes = lay.expert_bytes(rows);
  const uint64_t off_mat = up256(len), off_x = off_mat + up256(mat_bytes), off_y = off_x + up256(cols * 4);
  const uint64_t need = off_y + up256(rows * 4);
  if (need > kScratchBytes)
    return fail(QC_ERR_INVALID, "matrix needs " + std::to_string(need) + " bytes of device scratch; the "
                                "allocation-free matvec holds at most " + std::to_string(kScratchBytes));
  qc::MatDesc m{};
  uint8_t* base = nullptr;
  if (int rc = scratch_of_current_device(&base)) return rc;
  m.w = base + off_mat;
  m.kind = kind;
  m.rows = (uint32_t)rows;
  m.cols = (uint32_t)cols;
  m.units = lay.units;
  m.lpr = lay.lpr;
  m.upl = lay.upl;
  m.main_bytes = (uint32_t)lay.main_bytes;
  m.d_bytes = (uint32_t)lay.d_bytes;
  m.group_bytes = (uint32_t)lay.group_bytes;
  m.expert_stride = mat_bytes;
  if (qc::matvec_smem(m) > (size_t)kNoAllocMaxSmem)
    return fail(QC_ERR_INVALID, "row too wide for the shared-memory activation tile");
  float* dx = reinterpret_cast<float*>(base + off_x);
  float* dy = reinterpret_cast<float*>(base + off_y);
  QC_NA_CK(cudaMemcpy(base, blocks, len, cudaMemcpyHostToDevice));
  QC_NA_CK(cudaMemsetAsync(base + off_mat, 0, mat_bytes, nullptr));  // padding rows and blocks read as zero
  qc::launch_repack(base, 0, rows, (uint32_t)rows, raw_row, kind, cols, base + off_mat, lay, mat_bytes, nullptr);
  QC_NA_CK(cudaGetLastError());
  QC_NA_CK(cudaMemcpy(dx, x, cols * 4, cudaMemcpyHostToDevice));
  qc::launch_matvec(m, 0, dx, dy, 148, nullptr);
  QC_NA_CK(cudaGetLastError());
  QC_NA_CK(cudaMemcpy(y, dy, rows * 4, cudaMemcpyDeviceToHost));
  return QC_OK;
}
